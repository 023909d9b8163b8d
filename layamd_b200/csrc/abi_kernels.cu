// Kernel-level C entry points: the encoder GEMM on caller-owned device buffers, used by the GEMM
// sweep (isolated encoder-GEMM benchmark) and by the kernel parity tests. They are additions to
// the reference ABI; the engine itself never calls them.
#include <cstdio>
#include <mutex>
#include <vector>

#include "kernels.h"
#include "laya_api.h"

namespace {
std::mutex g_err_mu;
std::vector<int*> g_err_word;  // per device: the error word of the kernel-level entry points

std::mutex g_mu;
struct DevState {
  bool ready = false;
  float* ws = nullptr;       // split-K partials (grown on demand)
  size_t ws_floats = 0;
};
std::vector<DevState> g_dev;

DevState* dev_state(int dev) {
  if ((int)g_dev.size() <= dev) g_dev.resize(dev + 1);
  DevState& d = g_dev[dev];
  if (!d.ready) {
    if (laya::gemm_prepare_device() != cudaSuccess) return nullptr;
    d.ready = true;
  }
  return &d;
}
}  // namespace

namespace laya {
int* entry_error_word(int dev) {
  std::lock_guard<std::mutex> lk(g_err_mu);
  if (dev < 0) return nullptr;
  if ((int)g_err_word.size() <= dev) g_err_word.resize(dev + 1, nullptr);
  if (!g_err_word[dev]) {
    int* p = nullptr;
    if (cudaMalloc(&p, sizeof(int)) != cudaSuccess) return nullptr;
    if (cudaMemset(p, 0, sizeof(int)) != cudaSuccess) {
      cudaFree(p);
      return nullptr;
    }
    g_err_word[dev] = p;
  }
  return g_err_word[dev];
}
}  // namespace laya

namespace {
int* existing_error_word(int dev) {
  std::lock_guard<std::mutex> lk(g_err_mu);
  return dev >= 0 && dev < (int)g_err_word.size() ? g_err_word[dev] : nullptr;
}
int num_sms(int dev) {
  int n = 0;
  cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev);
  return n > 0 ? n : 1;
}

// Shared body of the GEMM entry points. ws (splits x M x N fp32 partials) is used when splits > 1.
int run_gemm(const void* A, const void* W, void* out, float* resid, const float* bias, int M, int N, int K, int planes,
             int epi, int out_mode, int act, int bn, const float* cos_t, const float* sin_t, const int* pos,
             int rope_cols, int geglu_I, void* stream, int sync, int splits, float* ws, int* err, int dev) {
  using namespace laya;
  if ((planes != 1 && planes != 2) || M <= 0 || N <= 0 || K <= 0) return -2;
  if (bn != 128 && bn != 256 && bn != kGemmPair) return -2;
  // at most one K slice per 64-wide K block (of every product segment in parity mode)
  if (splits > ((K + 63) / 64) * (planes == 2 ? 3 : 1)) return -2;
  CUtensorMap ta, tb, tc;
  if (!make_operand_map(&ta, A, (uint64_t)K, (uint64_t)M, (uint64_t)planes, 128)) return -3;
  const uint32_t box_b = bn == kGemmPair ? 128u : static_cast<uint32_t>(bn);  // a pair tile loads 128 B rows per CTA
  if (!make_operand_map(&tb, W, (uint64_t)K, (uint64_t)N, (uint64_t)planes, box_b)) return -3;
  const int ncols = epi == EPI_GEGLU ? geglu_I : N;
  const bool f32 = epi == EPI_RESID || out_mode == OUT_F32;
  void* dst = epi == EPI_RESID ? static_cast<void*>(resid) : out;
  if (!dst || !make_output_map(&tc, dst, f32, (uint64_t)ncols, (uint64_t)M, f32 ? 1 : (out_mode == OUT_BF16X2 ? 2 : 1)))
    return -3;
  GemmShape sh{M, N, K, planes == 2 ? 3 : 1};
  sh.splits = splits;
  sh.ws = ws;
  sh.dst = dst;
  sh.dst_plane = (long long)M * ncols;
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
}  // namespace

extern "C" int laya_b200_gemm(const void* A, const void* W, void* out, float* resid, const float* bias, int M,
                              int N, int K, int planes, int epi, int out_mode, int act, int bn,
                              const float* cos_t, const float* sin_t, const int* pos, int rope_cols,
                              int geglu_I, void* stream, int sync) {
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess) return -1;
  int* err = laya::entry_error_word(dev);
  if (!err) return -4;
  {
    std::lock_guard<std::mutex> lk(g_mu);
    if (!dev_state(dev)) return -4;
  }
  return run_gemm(A, W, out, resid, bias, M, N, K, planes, epi, out_mode, act, bn, cos_t, sin_t, pos, rope_cols,
                  geglu_I, stream, sync, 1, nullptr, err, dev);
}

extern "C" int laya_b200_gemm_splitk(const void* A, const void* W, void* out, float* resid, const float* bias, int M,
                                     int N, int K, int planes, int epi, int out_mode, int act, int bn,
                                     const float* cos_t, const float* sin_t, const int* pos, int rope_cols,
                                     int geglu_I, int splits, void* stream, int sync) {
  using namespace laya;
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess) return -1;
  if (splits < 1 || splits > kMaxSplits || (splits > 1 && bn == kGemmPair) || M <= 0 || N <= 0) return -2;
  float* ws = nullptr;
  int* err = entry_error_word(dev);
  if (!err) return -4;
  {
    std::lock_guard<std::mutex> lk(g_mu);
    DevState* d = dev_state(dev);
    if (!d) return -4;
    const size_t need_ws = splitk_ws_floats(M, N, splits);
    if (splits > 1 && d->ws_floats < need_ws) {
      if (d->ws) cudaFree(d->ws);
      d->ws = nullptr;
      d->ws_floats = 0;
      if (cudaMalloc(&d->ws, need_ws * sizeof(float)) != cudaSuccess) return -4;
      d->ws_floats = need_ws;
    }
    ws = d->ws;
  }
  return run_gemm(A, W, out, resid, bias, M, N, K, planes, epi, out_mode, act, bn, cos_t, sin_t, pos, rope_cols,
                  geglu_I, stream, sync, splits, ws, err, dev);
}

// ---------------------------------------------------------------- split-K with no allocation
// laya_b200_gemm_splitk_noalloc serves callers that may not allocate device memory themselves or
// let a library do it: a host whose memory manager reserves the GPU's memory up front (a serving
// stack with a caching allocator, where a cudaMalloc from outside can fail or fragment its pool),
// or a plugin host that forbids allocation inside its callbacks, where cudaMalloc's implicit device
// synchronisation would also stall every other stream. Its scratch (split-K partials, error word)
// is this fixed array in the library's device image instead: every GPU that loads the library holds
// its 16 MiB until the process exits, and every call on a device shares it.
namespace {
constexpr size_t kNoAllocWsFloats = size_t(4) << 20;  // fp32 partials: splits x M x N <= 4 Mi (16 MiB)
constexpr size_t kNoAllocWsBytes = kNoAllocWsFloats * sizeof(float);
constexpr size_t kNoAllocBytes = kNoAllocWsBytes + 256;  // + the error word
constexpr int kNoAllocMaxDevices = 64;
}  // namespace

// In host code this name is only a stand-in: its device address comes from cudaGetSymbolAddress.
static __device__ __align__(256) unsigned char g_noalloc_scratch[kNoAllocBytes];

namespace {
std::mutex g_noalloc_mu;
unsigned char* g_noalloc_base[kNoAllocMaxDevices];  // device address of g_noalloc_scratch, per device

// Set-up on the first call on a device (with that device current): the kernels' shared-memory
// limits, the array's device address and a zero error word. None of it allocates.
unsigned char* noalloc_scratch(int dev) {
  std::lock_guard<std::mutex> lk(g_noalloc_mu);
  if (!g_noalloc_base[dev]) {
    cudaError_t e = laya::gemm_prepare_device();
    if (e != cudaSuccess) {
      fprintf(stderr, "[laya] gemm_noalloc: device %d set-up failed: %s\n", dev, cudaGetErrorString(e));
      return nullptr;
    }
    void* p = nullptr;
    e = cudaGetSymbolAddress(&p, g_noalloc_scratch);
    if (e != cudaSuccess || !p) {
      fprintf(stderr, "[laya] gemm_noalloc: no device address for the static scratch on device %d: %s\n", dev,
              cudaGetErrorString(e));
      return nullptr;
    }
    // the error word starts at zero once; after that it keeps a kernel's code until a call with
    // sync != 0 or laya_b200_kernel_error reads it
    e = cudaMemset(static_cast<unsigned char*>(p) + kNoAllocWsBytes, 0, sizeof(int));
    if (e != cudaSuccess) {
      fprintf(stderr, "[laya] gemm_noalloc: clearing the error word on device %d failed: %s\n", dev,
              cudaGetErrorString(e));
      return nullptr;
    }
    g_noalloc_base[dev] = static_cast<unsigned char*>(p);
  }
  return g_noalloc_base[dev];
}
unsigned char* noalloc_scratch_if_set_up(int dev) {
  std::lock_guard<std::mutex> lk(g_noalloc_mu);
  return dev >= 0 && dev < kNoAllocMaxDevices ? g_noalloc_base[dev] : nullptr;
}
}  // namespace

extern "C" int laya_b200_gemm_splitk_noalloc(const void* A, const void* W, void* out, float* resid, const float* bias,
                                             int M, int N, int K, int planes, int epi, int out_mode, int act, int bn,
                                             const float* cos_t, const float* sin_t, const int* pos, int rope_cols,
                                             int geglu_I, int splits, void* stream, int sync) {
  using namespace laya;
  if (splits < 1 || splits > kMaxSplits || (splits > 1 && bn == kGemmPair) || M <= 0 || N <= 0) return -2;
  const size_t need_ws = splits > 1 ? splitk_ws_floats(M, N, splits) : 0;
  if (need_ws > kNoAllocWsFloats) {
    fprintf(stderr,
            "[laya] laya_b200_gemm_splitk_noalloc: M %d x N %d in %d slices needs %zu partial floats; the "
            "static scratch holds %zu (use laya_b200_gemm_splitk)\n",
            M, N, splits, need_ws, kNoAllocWsFloats);
    return -7;
  }
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess) return -1;
  if (dev < 0 || dev >= kNoAllocMaxDevices) return -4;
  unsigned char* base = noalloc_scratch(dev);
  if (!base) return -4;
  float* ws = reinterpret_cast<float*>(base);
  int* err = reinterpret_cast<int*>(base + kNoAllocWsBytes);
  // The array keeps whatever the last call left. The partials need no clearing: run_gemm gives every
  // slice at least one K block, so every slice overwrites its whole plane. The error word is not
  // cleared here, so that a code an earlier call with sync = 0 left is reported, not lost.
  return run_gemm(A, W, out, resid, bias, M, N, K, planes, epi, out_mode, act, bn, cos_t, sin_t, pos, rope_cols,
                  geglu_I, stream, sync, splits, ws, err, dev);
}

// ---------------------------------------------------------------- asynchronous error reports
extern "C" int laya_b200_kernel_error(int device) {
  int ndev = 0;
  if (cudaGetDeviceCount(&ndev) != cudaSuccess || device < 0 || device >= ndev) return -1;
  int prev = 0;
  cudaGetDevice(&prev);
  if (cudaSetDevice(device) != cudaSuccess) return -1;
  int code = 0;
  int rc = 0;
  if (cudaDeviceSynchronize() != cudaSuccess) rc = -2;
  int* words[2] = {existing_error_word(device), nullptr};
  if (unsigned char* base = noalloc_scratch_if_set_up(device)) words[1] = reinterpret_cast<int*>(base + kNoAllocWsBytes);
  for (int* w : words) {
    if (!w || rc) continue;
    int h = 0;
    if (cudaMemcpy(&h, w, sizeof(int), cudaMemcpyDeviceToHost) != cudaSuccess) {
      rc = -2;
      break;
    }
    if (h) {
      if (!code) code = h;
      if (cudaMemset(w, 0, sizeof(int)) != cudaSuccess) rc = -2;
    }
  }
  cudaSetDevice(prev);
  return rc ? rc : code;
}
