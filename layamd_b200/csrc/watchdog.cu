// Self-test of the bounded mbarrier wait (mbar_wait in common.cuh) that guards every pipeline stage of
// the GEMM and attention kernels. The reference engine has no device-side failure detection (it exits
// on any HIP error); here a stalled pipeline ends its kernel with an error code instead of hanging the
// GPU, and this entry point shows that path on real hardware without faulting anything: one thread
// waits on a barrier phase that no thread or copy ever completes, the budget runs out, the code is
// recorded, and the kernel returns normally.
#include "common.cuh"
#include "kernels.h"
#include "laya_api.h"

namespace laya {
namespace {

__global__ void watchdog_selftest_kernel(int* err, long long* cycles) {
  __shared__ alignas(8) uint64_t bar;
  __shared__ int abort_flag;
  if (threadIdx.x == 0) {
    mbar_init(smem_u32(&bar), 1);  // one arrival would complete phase 0; none is ever made
    abort_flag = 0;
    fence_mbar_init();
  }
  __syncthreads();
  if (threadIdx.x == 0) {
    const long long t0 = clock64();
    const bool completed = mbar_wait(smem_u32(&bar), 0, &abort_flag, err, kErrSelfTest);
    cycles[0] = clock64() - t0;
    cycles[1] = completed ? 1 : 0;
  }
}

}  // namespace
}  // namespace laya

extern "C" int laya_b200_watchdog_selftest(int device, int* code, long long* cycles, float* ms) {
  if (!code || !cycles || !ms) return -2;
  if (cudaSetDevice(device) != cudaSuccess) return -2;
  // the kernel records its code in the error word of the kernel-level entry points, where it stays
  // (first writer wins) until laya_b200_kernel_error or a synchronous entry call reads it
  int* d_err = laya::entry_error_word(device);
  long long* d_cyc = nullptr;
  cudaEvent_t a = nullptr, b = nullptr;
  int rc = -2;
  if (!d_err) return -2;
  {
    // a code still pending from an earlier call would hide this kernel's: report it instead
    int pending = 0;
    if (cudaMemcpy(&pending, d_err, sizeof(int), cudaMemcpyDeviceToHost) != cudaSuccess) return -2;
    if (pending) return -3;
  }
  if (cudaMalloc(&d_cyc, 2 * sizeof(long long)) == cudaSuccess &&
      cudaMemset(d_cyc, 0, 2 * sizeof(long long)) == cudaSuccess &&
      cudaEventCreate(&a) == cudaSuccess && cudaEventCreate(&b) == cudaSuccess) {
    cudaEventRecord(a, 0);
    laya::watchdog_selftest_kernel<<<1, 32>>>(d_err, d_cyc);
    const cudaError_t le = cudaGetLastError();
    cudaEventRecord(b, 0);
    long long h_cyc[2] = {0, 0};
    if (le == cudaSuccess && cudaEventSynchronize(b) == cudaSuccess &&
        cudaMemcpy(code, d_err, sizeof(int), cudaMemcpyDeviceToHost) == cudaSuccess &&
        cudaMemcpy(h_cyc, d_cyc, sizeof(h_cyc), cudaMemcpyDeviceToHost) == cudaSuccess &&
        cudaEventElapsedTime(ms, a, b) == cudaSuccess) {
      *cycles = h_cyc[1] ? -h_cyc[0] : h_cyc[0];  // negative: the phase completed, which it must not
      rc = 0;
    }
  }
  if (a) cudaEventDestroy(a);
  if (b) cudaEventDestroy(b);
  if (d_cyc) cudaFree(d_cyc);
  return rc;
}
