// Device-side building blocks shared by the sm_100a kernels of the Laya B200 engine:
// bf16 packing, bounded mbarrier waits, TMA bulk-tensor loads and the tcgen05 (UMMA/TMEM)
// instructions, all as inline PTX. Every spin-wait here gives up after a cycle budget, records an
// error code in a device flag the host reads back after the pass, and lets the kernel return.
#pragma once
#include <cuda_runtime.h>
#include <cuda_bf16.h>
#include <stdint.h>
#include <cstdlib>
#include <utility>

namespace laya {

// Error codes written into the per-replica device error word (first writer wins).
enum DevErr : int {
  kErrNone = 0,
  kErrGemmFull = 1,      // MMA issuer timed out waiting for a TMA stage
  kErrGemmEmpty = 2,     // producer timed out waiting for a free stage
  kErrGemmAccFull = 3,   // epilogue timed out waiting for the accumulator
  kErrGemmAccEmpty = 4,  // MMA issuer timed out waiting for the epilogue to drain TMEM
  kErrGemmDrain = 5,     // abort path: in-flight work did not drain in time
  kErrAttnLoad = 16,     // attention producer timed out waiting for a K / V buffer to be released
  kErrAttnMma = 17,      // attention MMA issuer timed out waiting for Q / K / V / P
  kErrAttnSoftmax = 18,  // attention softmax warps timed out waiting for S or O
  kErrSelfTest = 30,     // watchdog self-test: a wait on a barrier phase that nothing completes
  // debug bounds mode (LAYA_DEBUG_BOUNDS builds): an index read from the packing maps is out of range
  kErrBoundsLnSrc = 40,    // LayerNorm source row (token id / gathered row) beyond its table
  kErrBoundsLnSeq = 41,    // LayerNorm row -> question or question type out of range
  kErrBoundsRope = 42,     // GEMM RoPE position beyond the cos / sin tables
  kErrBoundsAttn = 43,     // attention work item: sequence, rows or query block out of range
  kErrBoundsGather = 44,   // gathered attention: source or destination row out of range
  kErrBoundsHead = 45,     // decision-head outputs: marker rows or logit slots out of range
};

// ---------------------------------------------------------------- programmatic dependent launch
// With LAYA_PDL=1 every kernel of the pass is launched with programmatic stream serialization: the
// next kernel on the stream may be scheduled as soon as all blocks of the current one have started
// (pdl_trigger at their top), so its launch and prologue (barrier set-up, TMEM allocation) overlap
// the current kernel's tail. Each kernel calls pdl_wait() before its first global-memory access,
// which returns once the previous kernel has completed and its writes are visible (completion is
// transitive along the stream); without the attribute both are no-ops. Off by default: measured on
// the C2 pass and at batch 1 it made no difference outside run-to-run noise.
__device__ __forceinline__ void pdl_trigger() { asm volatile("griddepcontrol.launch_dependents;" ::: "memory"); }
__device__ __forceinline__ void pdl_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }

inline bool pdl_enabled() {
  static const bool on = [] {
    const char* v = getenv("LAYA_PDL");
    return v && *v && atoi(v) != 0;
  }();
  return on;
}
template <typename... KArgs, typename... Args>
inline cudaError_t launch_pdl(void (*kernel)(KArgs...), dim3 grid, dim3 block, size_t smem, cudaStream_t st,
                              Args&&... args) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = block;
  cfg.dynamicSmemBytes = smem;
  cfg.stream = st;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = pdl_enabled() ? 1 : 0;
  return cudaLaunchKernelEx(&cfg, kernel, std::forward<Args>(args)...);
}

// ~2^31 SM cycles (~1 s at 1.9 GHz): far beyond any legitimate wait inside one tile.
constexpr long long kWaitBudgetCycles = 1ll << 31;

__device__ __forceinline__ uint32_t smem_u32(const void* p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

__device__ __forceinline__ uint32_t pack_bf16x2(float lo, float hi) {
  __nv_bfloat162 v = __floats2bfloat162_rn(lo, hi);
  return *reinterpret_cast<uint32_t*>(&v);
}

__device__ __forceinline__ float gelu_erf(float x) {
  return 0.5f * x * (1.f + erff(x * 0.70710678118654752f));
}

// GELU with the exact-erf definition, x * Phi(x), for the GEMM epilogues: Phi from the complementary
// error function in the rational-times-Gaussian form of Abramowitz & Stegun, Handbook of
// Mathematical Functions, eq. 7.1.26 (|erf error| <= 1.5e-7): with z = |x| / sqrt(2) and
// t = 1 / (1 + 0.3275911 z), erfc(z) = t (a1 + t (a2 + t (a3 + t (a4 + t a5)))) exp(-z^2). One
// reciprocal and one 2^x on the special-function unit and seven FMAs; measured against the fp64 GELU
// over [-12, 12] in fp32 arithmetic its absolute error stays below 6e-7.
__device__ __forceinline__ float gelu_as(float x) {
  const float z = fabsf(x) * 0.70710678118654752f;
  float t;
  asm("rcp.approx.ftz.f32 %0, %1;" : "=f"(t) : "f"(fmaf(0.3275911f, z, 1.f)));
  const float poly =
      t * fmaf(t, fmaf(t, fmaf(t, fmaf(t, 1.061405429f, -1.453152027f), 1.421413741f), -0.284496736f), 0.254829592f);
  float g;  // exp(-z^2) = 2^(-z^2 log2 e)
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(g) : "f"(-z * z * 1.4426950408889634f));
  const float q = 0.5f * poly * g;  // Phi(-|x|) = erfc(|x| / sqrt 2) / 2
  return x * (x >= 0.f ? 1.f - q : q);
}

// ---------------------------------------------------------------- mbarrier
__device__ __forceinline__ void mbar_init(uint32_t bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(bar), "r"(count) : "memory");
}
__device__ __forceinline__ void fence_mbar_init() {
  asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}
__device__ __forceinline__ void mbar_expect_tx(uint32_t bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(bar), "r"(bytes) : "memory");
}
__device__ __forceinline__ void mbar_arrive(uint32_t bar) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(bar) : "memory");
}
__device__ __forceinline__ bool mbar_try(uint32_t bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(ok)
      : "r"(bar), "r"(parity)
      : "memory");
  return ok != 0;
}
// Debug bounds mode. Built with -DLAYA_DEBUG_BOUNDS, LAYA_IN_BOUNDS(cond, err, code) records `code`
// in the error word (first writer wins) and yields false when `cond` fails, so the caller skips the
// access instead of reading or writing out of range; in normal builds it is `true` and costs nothing.
__device__ __forceinline__ bool bounds_fail(int* err, int code) {
  if (err) atomicCAS(err, 0, code);
  return false;
}
#ifdef LAYA_DEBUG_BOUNDS
#define LAYA_IN_BOUNDS(cond, err, code) ((cond) ? true : ::laya::bounds_fail((err), (code)))
#else
#define LAYA_IN_BOUNDS(cond, err, code) true
#endif

// Bounded wait on phase `parity`. Returns false (after recording `code`) when the budget runs out
// or when another role of the CTA has already aborted (`*abort` set).
__device__ __forceinline__ bool mbar_wait(uint32_t bar, uint32_t parity, volatile int* abort,
                                          int* err, int code) {
  if (mbar_try(bar, parity)) return true;
  const long long t0 = clock64();
  while (true) {
    if (mbar_try(bar, parity)) return true;
    if (*abort) return false;
    if (clock64() - t0 > kWaitBudgetCycles) {
      *abort = 1;
      if (err) atomicCAS(err, 0, code);
      return false;
    }
  }
}

// ---------------------------------------------------------------- TMA
// 3-D tiled bulk-tensor load (coordinates innermost first) completing on an mbarrier.
// Every CTA fetches its own tiles; no load is shared between CTAs.
__device__ __forceinline__ void tma_load_3d(uint32_t dst, const void* tmap, int c0, int c1, int c2,
                                            uint32_t bar) {
  asm volatile(
      "cp.async.bulk.tensor.3d.shared::cluster.global.mbarrier::complete_tx::bytes"
      " [%0], [%1, {%2, %3, %4}], [%5];" ::"r"(dst),
      "l"(reinterpret_cast<uint64_t>(tmap)), "r"(c0), "r"(c1), "r"(c2), "r"(bar)
      : "memory");
}
// Asynchronous prefetch of `bytes` (a multiple of 16, 16-byte aligned) of global memory into L2.
__device__ __forceinline__ void prefetch_l2_bulk(const void* p, uint32_t bytes) {
  asm volatile("cp.async.bulk.prefetch.L2.global [%0], %1;" ::"l"(reinterpret_cast<uint64_t>(p)), "r"(bytes)
               : "memory");
}
__device__ __forceinline__ void tma_prefetch_desc(const void* tmap) {
  asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(tmap)) : "memory");
}

// ---------------------------------------------------------------- tcgen05 / TMEM
__device__ __forceinline__ void tmem_alloc(uint32_t dst_smem, uint32_t ncols) {
  asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(dst_smem),
               "r"(ncols)
               : "memory");
}
__device__ __forceinline__ void tmem_relinquish() {
  asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
}
__device__ __forceinline__ void tmem_dealloc(uint32_t taddr, uint32_t ncols) {
  asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(taddr), "r"(ncols)
               : "memory");
}
__device__ __forceinline__ void tc_fence_before() {
  asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
}
__device__ __forceinline__ void tc_fence_after() {
  asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
}
// D[tmem] (+)= A[smem] * B[smem]^T, bf16 inputs, fp32 accumulate; issued by one thread.
__device__ __forceinline__ void umma_bf16(uint32_t d_tmem, uint64_t adesc, uint64_t bdesc,
                                          uint32_t idesc, uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n\t}" ::"r"(d_tmem),
      "l"(adesc), "l"(bdesc), "r"(idesc), "r"(accumulate)
      : "memory");
}
// D[tmem] (+)= A[tmem] * B[smem]^T: the A operand (M rows = TMEM lanes, K bf16 values packed two per
// 32-bit column, the low half first) is read from tensor memory.
__device__ __forceinline__ void umma_bf16_ts(uint32_t d_tmem, uint32_t a_tmem, uint64_t bdesc, uint32_t idesc,
                                             uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], [%1], %2, %3, p;\n\t}" ::"r"(d_tmem),
      "r"(a_tmem), "l"(bdesc), "r"(idesc), "r"(accumulate)
      : "memory");
}
// 32 lanes x 32 consecutive 32-bit columns from registers into tensor memory, then wait.
__device__ __forceinline__ void tmem_st32u(uint32_t taddr, const uint32_t (&v)[32]) {
  asm volatile(
      "tcgen05.st.sync.aligned.32x32b.x32.b32 [%0], "
      "{%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,%16,"
      "%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31,%32};\n\t"
      "tcgen05.wait::st.sync.aligned;" ::"r"(taddr),
      "r"(v[0]), "r"(v[1]), "r"(v[2]), "r"(v[3]), "r"(v[4]), "r"(v[5]), "r"(v[6]), "r"(v[7]),
      "r"(v[8]), "r"(v[9]), "r"(v[10]), "r"(v[11]), "r"(v[12]), "r"(v[13]), "r"(v[14]), "r"(v[15]),
      "r"(v[16]), "r"(v[17]), "r"(v[18]), "r"(v[19]), "r"(v[20]), "r"(v[21]), "r"(v[22]), "r"(v[23]),
      "r"(v[24]), "r"(v[25]), "r"(v[26]), "r"(v[27]), "r"(v[28]), "r"(v[29]), "r"(v[30]), "r"(v[31])
      : "memory");
}
// Arrive once on `bar` when every tcgen05 op issued so far by this thread has completed.
__device__ __forceinline__ void umma_commit(uint32_t bar) {
  asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(bar)
               : "memory");
}
// 32 lanes x 32 consecutive fp32 columns: thread i of the warp gets lane (base+i), columns c..c+31.
// The wait is part of the same asm statement so no use of the destination registers can be
// scheduled before the asynchronous load has completed.
__device__ __forceinline__ void tmem_ld32(uint32_t taddr, float (&v)[32]) {
  uint32_t r[32];
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x32.b32 "
      "{%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,"
      "%16,%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31}, [%32];\n\t"
      "tcgen05.wait::ld.sync.aligned;"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]),
        "=r"(r[7]), "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]),
        "=r"(r[14]), "=r"(r[15]), "=r"(r[16]), "=r"(r[17]), "=r"(r[18]), "=r"(r[19]),
        "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]), "=r"(r[24]), "=r"(r[25]),
        "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]), "=r"(r[30]), "=r"(r[31])
      : "r"(taddr)
      : "memory");
#pragma unroll
  for (int i = 0; i < 32; ++i) v[i] = __uint_as_float(r[i]);
}

// 32 lanes x 64 consecutive fp32 columns in one load (one wait), as tmem_ld32.
__device__ __forceinline__ void tmem_ld64(uint32_t taddr, float (&v)[64]) {
  uint32_t r[64];
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x64.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,%16,%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31,%32,%33,%34,%35,%36,%37,%38,%39,%40,%41,%42,%43,%44,%45,%46,%47,%48,%49,%50,%51,%52,%53,%54,%55,%56,%57,%58,%59,%60,%61,%62,%63}, [%64];\n\t"
      "tcgen05.wait::ld.sync.aligned;"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]), "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15]), "=r"(r[16]), "=r"(r[17]), "=r"(r[18]), "=r"(r[19]), "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]), "=r"(r[24]), "=r"(r[25]), "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]), "=r"(r[30]), "=r"(r[31]), "=r"(r[32]), "=r"(r[33]), "=r"(r[34]), "=r"(r[35]), "=r"(r[36]), "=r"(r[37]), "=r"(r[38]), "=r"(r[39]), "=r"(r[40]), "=r"(r[41]), "=r"(r[42]), "=r"(r[43]), "=r"(r[44]), "=r"(r[45]), "=r"(r[46]), "=r"(r[47]), "=r"(r[48]), "=r"(r[49]), "=r"(r[50]), "=r"(r[51]), "=r"(r[52]), "=r"(r[53]), "=r"(r[54]), "=r"(r[55]), "=r"(r[56]), "=r"(r[57]), "=r"(r[58]), "=r"(r[59]), "=r"(r[60]), "=r"(r[61]), "=r"(r[62]), "=r"(r[63])
      : "r"(taddr)
      : "memory");
#pragma unroll
  for (int i = 0; i < 64; ++i) v[i] = __uint_as_float(r[i]);
}

// 32 lanes x 32 consecutive fp32 columns from registers into tensor memory (the inverse of
// tmem_ld32), waiting for the store to complete.
__device__ __forceinline__ void tmem_st32(uint32_t taddr, const float (&v)[32]) {
  asm volatile(
      "tcgen05.st.sync.aligned.32x32b.x32.b32 [%0], "
      "{%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,%16,"
      "%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31,%32};\n\t"
      "tcgen05.wait::st.sync.aligned;" ::"r"(taddr),
      "r"(__float_as_uint(v[0])), "r"(__float_as_uint(v[1])), "r"(__float_as_uint(v[2])), "r"(__float_as_uint(v[3])),
      "r"(__float_as_uint(v[4])), "r"(__float_as_uint(v[5])), "r"(__float_as_uint(v[6])), "r"(__float_as_uint(v[7])),
      "r"(__float_as_uint(v[8])), "r"(__float_as_uint(v[9])), "r"(__float_as_uint(v[10])), "r"(__float_as_uint(v[11])),
      "r"(__float_as_uint(v[12])), "r"(__float_as_uint(v[13])), "r"(__float_as_uint(v[14])), "r"(__float_as_uint(v[15])),
      "r"(__float_as_uint(v[16])), "r"(__float_as_uint(v[17])), "r"(__float_as_uint(v[18])), "r"(__float_as_uint(v[19])),
      "r"(__float_as_uint(v[20])), "r"(__float_as_uint(v[21])), "r"(__float_as_uint(v[22])), "r"(__float_as_uint(v[23])),
      "r"(__float_as_uint(v[24])), "r"(__float_as_uint(v[25])), "r"(__float_as_uint(v[26])), "r"(__float_as_uint(v[27])),
      "r"(__float_as_uint(v[28])), "r"(__float_as_uint(v[29])), "r"(__float_as_uint(v[30])), "r"(__float_as_uint(v[31]))
      : "memory");
}

// Shared-memory matrix descriptor for a K-major bf16 tile stored as rows of 64 elements
// (128 bytes) with the 128-byte TMA swizzle: 8-row core groups 1024 bytes apart.
__device__ __forceinline__ uint64_t sdesc_k128(uint32_t saddr) {
  uint64_t d = 0;
  d |= static_cast<uint64_t>((saddr >> 4) & 0x3FFFu);  // start address
  d |= static_cast<uint64_t>(1) << 16;                   // leading byte offset (unused, swizzled K-major)
  d |= static_cast<uint64_t>(1024 >> 4) << 32;           // stride byte offset: next 8-row group
  d |= static_cast<uint64_t>(1) << 46;                   // descriptor version (sm_100)
  d |= static_cast<uint64_t>(2) << 61;                   // 128-byte swizzle
  return d;
}

// ---------------------------------------------------------------- CTA-pair (cluster of 2) forms
__device__ __forceinline__ uint32_t cluster_ctarank() {
  uint32_t r;
  asm volatile("mov.u32 %0, %%cluster_ctarank;" : "=r"(r));
  return r;
}
__device__ __forceinline__ uint32_t cluster_id_x() {
  uint32_t r;
  asm volatile("mov.u32 %0, %%clusterid.x;" : "=r"(r));
  return r;
}
__device__ __forceinline__ uint32_t num_clusters_x() {
  uint32_t r;
  asm volatile("mov.u32 %0, %%nclusterid.x;" : "=r"(r));
  return r;
}
// Every thread of both CTAs of the cluster (not warp-aligned, so divergent warps may call it).
__device__ __forceinline__ void cluster_sync_all() {
  asm volatile("barrier.cluster.arrive.release;\n\tbarrier.cluster.wait.acquire;" ::: "memory");
}
// Address of the same shared-memory location in CTA `rank` of the cluster.
__device__ __forceinline__ uint32_t mapa_shared(uint32_t addr, uint32_t rank) {
  uint32_t r;
  asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(r) : "r"(addr), "r"(rank));
  return r;
}
__device__ __forceinline__ void mbar_arrive_cluster(uint32_t cluster_addr) {
  asm volatile("mbarrier.arrive.release.cluster.shared::cluster.b64 _, [%0];" ::"r"(cluster_addr) : "memory");
}
// TMA load into this CTA's shared memory whose completion is counted on the barrier at the same
// offset in the even CTA of the pair (the peer bit of the barrier address cleared). The data lands
// only in the issuing CTA's shared memory.
__device__ __forceinline__ void tma_load_3d_pair(uint32_t dst, const void* tmap, int c0, int c1, int c2,
                                                 uint32_t bar) {
  asm volatile(
      "cp.async.bulk.tensor.3d.cta_group::2.shared::cluster.global.mbarrier::complete_tx::bytes"
      " [%0], [%1, {%2, %3, %4}], [%5];" ::"r"(dst),
      "l"(reinterpret_cast<uint64_t>(tmap)), "r"(c0), "r"(c1), "r"(c2), "r"(bar & 0xFEFFFFFFu)
      : "memory");
}
__device__ __forceinline__ void tmem_alloc_pair(uint32_t dst_smem, uint32_t ncols) {
  asm volatile("tcgen05.alloc.cta_group::2.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(dst_smem), "r"(ncols)
               : "memory");
}
__device__ __forceinline__ void tmem_relinquish_pair() {
  asm volatile("tcgen05.relinquish_alloc_permit.cta_group::2.sync.aligned;" ::: "memory");
}
__device__ __forceinline__ void tmem_dealloc_pair(uint32_t taddr, uint32_t ncols) {
  asm volatile("tcgen05.dealloc.cta_group::2.sync.aligned.b32 %0, %1;" ::"r"(taddr), "r"(ncols) : "memory");
}
// 2-SM MMA issued by the even CTA: D[256 x N] over both CTAs' tensor memory, A rows and B rows split
// between the two CTAs' shared memory at the same offsets.
__device__ __forceinline__ void umma_bf16_pair(uint32_t d_tmem, uint64_t adesc, uint64_t bdesc, uint32_t idesc,
                                               uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::2.kind::f16 [%0], %1, %2, %3, p;\n\t}" ::"r"(d_tmem),
      "l"(adesc), "l"(bdesc), "r"(idesc), "r"(accumulate)
      : "memory");
}
// Arrive once on the barrier at offset `bar` in both CTAs of the pair when the MMAs issued so far
// complete: one commit to this CTA's barrier, one to the peer's through its cluster address.
__device__ __forceinline__ void umma_commit_pair(uint32_t bar, uint32_t bar_peer) {
  asm volatile("tcgen05.commit.cta_group::2.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(bar) : "memory");
  asm volatile("tcgen05.commit.cta_group::2.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(bar_peer)
               : "memory");
}

// Shared-memory matrix descriptor for an MN-major bf16 tile (N contiguous): rows are K, each 64
// elements (128 bytes) wide with the 128-byte TMA swizzle, 8-row K groups 1024 bytes apart. A tile
// 64 wide in N is one swizzle atom, so the stride between atoms along N is never used; it is set to
// the same 1024 bytes.
__device__ __forceinline__ uint64_t sdesc_mn128(uint32_t saddr) {
  uint64_t d = 0;
  d |= static_cast<uint64_t>((saddr >> 4) & 0x3FFFu);  // start address
  d |= static_cast<uint64_t>(1024 >> 4) << 16;           // leading byte offset: next N atom (unused)
  d |= static_cast<uint64_t>(1024 >> 4) << 32;           // stride byte offset: next 8-row K group
  d |= static_cast<uint64_t>(1) << 46;                   // descriptor version (sm_100)
  d |= static_cast<uint64_t>(2) << 61;                   // 128-byte swizzle
  return d;
}

// ---- one row of D = 128*NV fp32 values per warp, lane holding columns 4*(lane + 32*i) .. +3 ----
__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
  for (int o = 16; o; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}

// In place: v = (v - mean) / sqrt(var + eps) * w (+ b), mean and variance two-pass in fp32 over the
// warp's row (torch.nn.LayerNorm's definition). Every LayerNorm of the engine goes through this one
// routine, so a fused and a separate LayerNorm of the same row give the same bits.
template <int NV>
__device__ __forceinline__ void layer_norm_regs(float4 (&v)[NV], const float* w, const float* b, float eps, int D,
                                                int lane) {
  float s = 0.f;
#pragma unroll
  for (int i = 0; i < NV; ++i) s += (v[i].x + v[i].y) + (v[i].z + v[i].w);
  const float mean = warp_sum(s) / D;
  float q = 0.f;
#pragma unroll
  for (int i = 0; i < NV; ++i) {
    v[i].x -= mean; v[i].y -= mean; v[i].z -= mean; v[i].w -= mean;
    q += (v[i].x * v[i].x + v[i].y * v[i].y) + (v[i].z * v[i].z + v[i].w * v[i].w);
  }
  const float rstd = 1.f / sqrtf(warp_sum(q) / D + eps);
#pragma unroll
  for (int i = 0; i < NV; ++i) {
    const float4 g = reinterpret_cast<const float4*>(w)[lane + 32 * i];
    float4 r = make_float4(v[i].x * rstd * g.x, v[i].y * rstd * g.y, v[i].z * rstd * g.z, v[i].w * rstd * g.w);
    if (b) {
      const float4 bb = reinterpret_cast<const float4*>(b)[lane + 32 * i];
      r.x += bb.x; r.y += bb.y; r.z += bb.z; r.w += bb.w;
    }
    v[i] = r;
  }
}

// The row as bf16 (hi) and, with two planes, the bf16 rounding of what the hi plane missed (lo).
template <int NV>
__device__ __forceinline__ void store_bf16_planes(const float4 (&v)[NV], __nv_bfloat16* hi_row, __nv_bfloat16* lo_row,
                                                  int planes, int lane) {
  uint2* hi = reinterpret_cast<uint2*>(hi_row);
  uint2* lo = reinterpret_cast<uint2*>(lo_row);
#pragma unroll
  for (int i = 0; i < NV; ++i) {
    const uint32_t h0 = pack_bf16x2(v[i].x, v[i].y), h1 = pack_bf16x2(v[i].z, v[i].w);
    __stcs(hi + lane + 32 * i, make_uint2(h0, h1));  // streaming stores (measured: LayerNorm 4 % faster)
    if (planes == 2) {
      const float2 f0 = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(&h0));
      const float2 f1 = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(&h1));
      __stcs(lo + lane + 32 * i,
             make_uint2(pack_bf16x2(v[i].x - f0.x, v[i].y - f0.y), pack_bf16x2(v[i].z - f1.x, v[i].w - f1.y)));
    }
  }
}

// Instruction descriptor: bf16 x bf16 -> fp32, both operands K-major, M x N tile.
__host__ __device__ constexpr uint32_t idesc_bf16(int M, int N) {
  return (1u << 4)      // D format fp32
         | (1u << 7)    // A format bf16
         | (1u << 10)   // B format bf16
         | (static_cast<uint32_t>(N >> 3) << 17) | (static_cast<uint32_t>(M >> 4) << 24);
}

}  // namespace laya
