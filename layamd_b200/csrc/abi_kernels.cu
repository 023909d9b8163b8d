// Kernel-level C entry points: the encoder GEMM on caller-owned device buffers, used by the GEMM
// sweep (isolated encoder-GEMM benchmark) and by the kernel parity tests. They are additions to
// the reference ABI; the engine itself never calls them.
#include "kernels.h"
#include "laya_api.h"
#include <cstdio>
#include <mutex>
#include <vector>

namespace {
std::mutex g_mu;
std::vector<int*> g_err;  // one device error word per device
int* err_word(int dev) {
  std::lock_guard<std::mutex> lk(g_mu);
  if ((int)g_err.size() <= dev) g_err.resize(dev + 1, nullptr);
  if (!g_err[dev]) {
    if (laya::gemm_prepare_device() != cudaSuccess) return nullptr;
    if (cudaMalloc(&g_err[dev], sizeof(int)) != cudaSuccess) return nullptr;
    cudaMemset(g_err[dev], 0, sizeof(int));
  }
  return g_err[dev];
}
int num_sms(int dev) {
  int n = 0;
  cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev);
  return n > 0 ? n : 1;
}
}  // namespace

extern "C" int laya_b200_gemm(const void* A, const void* W, void* out, float* resid, const float* bias, int M,
                              int N, int K, int planes, int epi, int out_mode, int act, int bn,
                              const float* cos_t, const float* sin_t, const int* pos, int rope_cols,
                              int geglu_I, void* stream, int sync) {
  using namespace laya;
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess) return -1;
  if ((planes != 1 && planes != 2) || M <= 0 || N <= 0 || K <= 0) return -2;
  CUtensorMap ta, tb;
  if (!make_operand_map(&ta, A, (uint64_t)K, (uint64_t)M, (uint64_t)planes, 128)) return -3;
  if (bn != 128 && bn != 256 && bn != kGemmPair) return -2;
  const uint32_t box_b = bn == kGemmPair ? 128u : static_cast<uint32_t>(bn);  // a pair tile loads 128 B rows per CTA
  if (!make_operand_map(&tb, W, (uint64_t)K, (uint64_t)N, (uint64_t)planes, box_b)) return -3;
  GemmShape sh{M, N, K, planes == 2 ? 3 : 1};
  const int ncols = epi == EPI_GEGLU ? geglu_I : N;
  CUtensorMap tc;
  const bool f32 = epi == EPI_RESID || out_mode == OUT_F32;
  void* dst = epi == EPI_RESID ? static_cast<void*>(resid) : out;
  if (!dst || !make_output_map(&tc, dst, f32, (uint64_t)ncols, (uint64_t)M, f32 ? 1 : (out_mode == OUT_BF16X2 ? 2 : 1)))
    return -3;
  GemmEpi ep;
  ep.kind = epi;
  ep.out_mode = out_mode;
  ep.bias = bias;
  ep.act = act;
  ep.cos_t = cos_t;
  ep.sin_t = sin_t;
  ep.pos = pos;
  ep.rope_cols = rope_cols;
  ep.geglu_I = geglu_I;
  int* err = err_word(dev);
  if (!err) return -4;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  cudaError_t e = gemm_launch(ta, tb, tc, bn, sh, ep, err, num_sms(dev), st);
  if (e != cudaSuccess) {
    fprintf(stderr, "[laya] gemm launch: %s\n", cudaGetErrorString(e));
    return -5;
  }
  if (sync) {
    if (cudaStreamSynchronize(st) != cudaSuccess) return -6;
    int h = 0;
    cudaMemcpy(&h, err, sizeof(int), cudaMemcpyDeviceToHost);
    if (h) {
      cudaMemset(err, 0, sizeof(int));
      return -100 - h;
    }
  }
  return 0;
}
