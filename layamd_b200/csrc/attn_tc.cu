// Encoder attention on the 5th-generation tensor cores (tcgen05 + TMEM + TMA), head dim 64, bf16
// Q/K/V read in place from the packed qkv rows [T, 3D] (q | k | v, heads of 64), bf16 output rows
// [T, D]. Replaces the reference's k_flash_wmma (src/kernels.hip:154-242, 351-356) for the encoder
// layers and the first head layer; the gathered last head layer keeps the mma.sync kernel (attn.cu).
//
// Persistent: two CTAs per SM (each 192 threads, 97 KB of shared memory, 256 TMEM columns). Work
// units (128 query rows of one sequence x one head, the item list sorted longest first) are claimed
// dynamically from a global counter, so the longest remaining unit always goes to the next free CTA,
// and each CTA runs its units through a software pipeline that continues across unit boundaries:
//   warp 0      TMA producer: claims units and publishes them to the other roles through a 4-deep
//               ring in shared memory; the unit's Q tile into one of two Q slots, then 64-key K and V tiles
//               into a 4-stage ring (a stage is released when its PV is done), running ahead into
//               the next units
//   warp 1      TMEM owner + MMA issuer: S = Q K^T (128 x 64 fp32 in one TMEM buffer; S(c+1) is
//               issued as soon as the softmax warps have copied S(c) into registers, so it forms
//               while the softmax of chunk c runs) and O += P V (128 x 64 fp32 in TMEM; P is the A
//               operand read from tensor memory, V the B operand read MN-major from its TMA tile)
//   warps 2..5  softmax, one query row per thread (the row's TMEM lane), one pass over the 64 scores
//               of a chunk: mask, row max, p = 2^(s*c - m), row sum, P as bf16 pairs into one of two
//               TMEM buffers. The reference max m is only raised (and O rescaled in TMEM, which waits
//               for the PV in flight) when it grows by more than 2^8, so chunks normally never wait
//               for the tensor core; at the end of a unit each thread writes its row of O / l.
// Keys come only from the unit's own sequence; sliding-window layers visit [q0 - window,
// q0 + 128 + window). 32-key groups that no row of a warp can see are skipped, groups every row sees
// completely skip the masking. Masked keys get p = 0 exactly; K / V rows beyond the sequence
// (another sequence's rows, or zero fill past the buffer) only ever meet p = 0, so they must hold
// finite values (the engine's qkv buffer starts zeroed).
#include "common.cuh"
#include "kernels.h"

namespace laya {
namespace {

constexpr int kRows = 128;                      // query rows per unit
constexpr int kKeys = 64;                       // keys per chunk
constexpr int kStages = 4;                      // K / V ring depth
constexpr int kThreads = 192;
constexpr int kRing = 4;                        // claimed units published ahead to the MMA / softmax roles
constexpr uint32_t kQBytes = 128 * 64 * 2;      // 16 KB
constexpr uint32_t kKVBytes = 64 * 64 * 2;      // 8 KB
constexpr uint32_t kTmemCols = 256;             // S at 0, O at 64 / 128, P at 192 / 224 (two CTAs per SM)
constexpr uint32_t kTmemS = 0;
constexpr uint32_t kTmemO = 64;                 // O of unit parity p at 64 + 64 p
constexpr uint32_t kTmemP = 192;                // P bf16 [128 lanes][64 keys] = 32 columns per buffer
constexpr uint32_t kIdescS = idesc_bf16(128, 64);
constexpr uint32_t kIdescPV = idesc_bf16(128, 64) | (1u << 16);  // B operand (V) MN-major

// One work unit: 128 query rows [q0, q0+128) of the sequence at packed rows [base, base+len) x head
// h; keys [lo, lo + 64*nch). nch == 0 marks the end of the work.
struct Unit {
  int base, len, q0, h, lo, nch;
};

struct AttnSmem {
  alignas(1024) uint8_t q[2][kQBytes];
  alignas(1024) uint8_t k[kStages][kKVBytes];
  alignas(1024) uint8_t v[kStages][kKVBytes];
  Unit units[kRing];
  alignas(8) uint64_t ufull[kRing], uempty[kRing];
  uint64_t qfull[2], qempty[2], kfull[kStages], vfull[kStages], kvempty[kStages];
  uint64_t sfull, sfree, pfull[2], pfree[2], drain;
  uint32_t tmem;
  int abort;
};
constexpr size_t attn_smem_bytes() { return sizeof(AttnSmem) + 1024; }

// 2^x on the special-function unit (PTX ex2.approx.ftz.f32; 2^-inf = 0)
__device__ __forceinline__ float ex2(float x) {
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}

// Packed pairs of fp32 lanes (sm_100 f32x2 FMA pipe, CUDA's float2 builtins): d = a * b + c and
// d = a + b, each lane rounded to nearest.
__device__ __forceinline__ float2 ffma2(float2 a, float2 b, float2 c) { return __ffma2_rn(a, b, c); }
__device__ __forceinline__ float2 fadd2(float2 a, float2 b) { return __fadd2_rn(a, b); }
__device__ __forceinline__ float fmax3(float a, float b, float c) {
  float d;
  asm("max.f32 %0, %1, %2, %3;" : "=f"(d) : "f"(a), "f"(b), "f"(c));
  return d;
}

// Asynchronous tensor-memory load / store halves: the matching wait names the registers as
// operands, so no use of the loaded values (or reuse of the stored ones) is scheduled across it.
__device__ __forceinline__ void tmem_ld64_issue(uint32_t taddr, uint32_t (&r)[64]) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x64.b32 "
      "{%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,%16,%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,"
      "%28,%29,%30,%31,%32,%33,%34,%35,%36,%37,%38,%39,%40,%41,%42,%43,%44,%45,%46,%47,%48,%49,%50,%51,%52,%53,"
      "%54,%55,%56,%57,%58,%59,%60,%61,%62,%63}, [%64];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
        "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15]),
        "=r"(r[16]), "=r"(r[17]), "=r"(r[18]), "=r"(r[19]), "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]),
        "=r"(r[24]), "=r"(r[25]), "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]), "=r"(r[30]), "=r"(r[31]),
        "=r"(r[32]), "=r"(r[33]), "=r"(r[34]), "=r"(r[35]), "=r"(r[36]), "=r"(r[37]), "=r"(r[38]), "=r"(r[39]),
        "=r"(r[40]), "=r"(r[41]), "=r"(r[42]), "=r"(r[43]), "=r"(r[44]), "=r"(r[45]), "=r"(r[46]), "=r"(r[47]),
        "=r"(r[48]), "=r"(r[49]), "=r"(r[50]), "=r"(r[51]), "=r"(r[52]), "=r"(r[53]), "=r"(r[54]), "=r"(r[55]),
        "=r"(r[56]), "=r"(r[57]), "=r"(r[58]), "=r"(r[59]), "=r"(r[60]), "=r"(r[61]), "=r"(r[62]), "=r"(r[63])
      : "r"(taddr)
      : "memory");
}
__device__ __forceinline__ void tmem_ld64_wait(uint32_t (&r)[64]) {
  asm volatile("tcgen05.wait::ld.sync.aligned;"
               : "+r"(r[0]), "+r"(r[1]), "+r"(r[2]), "+r"(r[3]), "+r"(r[4]), "+r"(r[5]), "+r"(r[6]), "+r"(r[7]),
                 "+r"(r[8]), "+r"(r[9]), "+r"(r[10]), "+r"(r[11]), "+r"(r[12]), "+r"(r[13]), "+r"(r[14]),
                 "+r"(r[15]), "+r"(r[16]), "+r"(r[17]), "+r"(r[18]), "+r"(r[19]), "+r"(r[20]), "+r"(r[21]),
                 "+r"(r[22]), "+r"(r[23]), "+r"(r[24]), "+r"(r[25]), "+r"(r[26]), "+r"(r[27]), "+r"(r[28]),
                 "+r"(r[29]), "+r"(r[30]), "+r"(r[31]), "+r"(r[32]), "+r"(r[33]), "+r"(r[34]), "+r"(r[35]),
                 "+r"(r[36]), "+r"(r[37]), "+r"(r[38]), "+r"(r[39]), "+r"(r[40]), "+r"(r[41]), "+r"(r[42]),
                 "+r"(r[43]), "+r"(r[44]), "+r"(r[45]), "+r"(r[46]), "+r"(r[47]), "+r"(r[48]), "+r"(r[49]),
                 "+r"(r[50]), "+r"(r[51]), "+r"(r[52]), "+r"(r[53]), "+r"(r[54]), "+r"(r[55]), "+r"(r[56]),
                 "+r"(r[57]), "+r"(r[58]), "+r"(r[59]), "+r"(r[60]), "+r"(r[61]), "+r"(r[62]), "+r"(r[63])
               :
               : "memory");
}
__device__ __forceinline__ void tmem_st32_issue(uint32_t taddr, const uint32_t (&v)[32]) {
  asm volatile(
      "tcgen05.st.sync.aligned.32x32b.x32.b32 [%0], "
      "{%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,%16,"
      "%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31,%32};" ::"r"(taddr),
      "r"(v[0]), "r"(v[1]), "r"(v[2]), "r"(v[3]), "r"(v[4]), "r"(v[5]), "r"(v[6]), "r"(v[7]),
      "r"(v[8]), "r"(v[9]), "r"(v[10]), "r"(v[11]), "r"(v[12]), "r"(v[13]), "r"(v[14]), "r"(v[15]),
      "r"(v[16]), "r"(v[17]), "r"(v[18]), "r"(v[19]), "r"(v[20]), "r"(v[21]), "r"(v[22]), "r"(v[23]),
      "r"(v[24]), "r"(v[25]), "r"(v[26]), "r"(v[27]), "r"(v[28]), "r"(v[29]), "r"(v[30]), "r"(v[31])
      : "memory");
}
__device__ __forceinline__ void tmem_st32_wait(const uint32_t (&v)[32]) {
  asm volatile("tcgen05.wait::st.sync.aligned;" ::"r"(v[0]), "r"(v[1]), "r"(v[2]), "r"(v[3]), "r"(v[4]),
               "r"(v[5]), "r"(v[6]), "r"(v[7]), "r"(v[8]), "r"(v[9]), "r"(v[10]), "r"(v[11]), "r"(v[12]),
               "r"(v[13]), "r"(v[14]), "r"(v[15]), "r"(v[16]), "r"(v[17]), "r"(v[18]), "r"(v[19]), "r"(v[20]),
               "r"(v[21]), "r"(v[22]), "r"(v[23]), "r"(v[24]), "r"(v[25]), "r"(v[26]), "r"(v[27]), "r"(v[28]),
               "r"(v[29]), "r"(v[30]), "r"(v[31])
               : "memory");
}

// Bounded wait for the completion of the last phase issued on a TMA barrier (abort path).
__device__ __forceinline__ void drain_phase(uint32_t bar, int issued, int* err) {
  if (issued <= 0) return;
  const long long t0 = clock64();
  while (!mbar_try(bar, (issued - 1) & 1)) {
    if (clock64() - t0 > kWaitBudgetCycles) { atomicCAS(err, 0, kErrGemmDrain); return; }
  }
}

// Unit w of the launch (item w / H, head w % H); false past the last one. Items hold
// {seq, q0, base, len}, longest sequences first; unused slots (seq < 0) sit at the end.
__device__ __forceinline__ bool unit_of(const AttnArgs& a, int w, int nwork, Unit& u) {
  if (w >= nwork) return false;
  const int4 it = __ldg(reinterpret_cast<const int4*>(a.items) + w / a.H);
  if (it.x < 0) return false;
  // debug bounds mode: a unit whose rows fall outside qkv is dropped (as if it were past the end)
  if (!LAYA_IN_BOUNDS(a.rows <= 0 || (it.z >= 0 && it.w > 0 && it.z + it.w <= a.rows && it.y >= 0 && it.y < it.w &&
                                      (a.n_seq <= 0 || it.x < a.n_seq)),
                      a.err, kErrBoundsAttn))
    return false;
  u.h = w % a.H;
  u.q0 = it.y;
  u.base = it.z;
  u.len = it.w;
  u.lo = a.window > 0 ? max(0, u.q0 - a.window) : 0;
  const int hi = a.window > 0 ? min(u.len, u.q0 + kRows + a.window) : u.len;
  u.nch = (hi - u.lo + kKeys - 1) / kKeys;  // >= 1: q0 < len
  return true;
}

// Consumer side of the unit ring: the `ui`-th unit this CTA claimed (all lanes of a warp call it).
__device__ __forceinline__ bool take_unit(AttnSmem& S, int ui, Unit& u, volatile int* abort, int* err, int code,
                                          int lane) {
  const int rs = ui % kRing;
  if (!mbar_wait(smem_u32(&S.ufull[rs]), (ui / kRing) & 1, abort, err, code)) return false;
  u = S.units[rs];
  __syncwarp(__activemask());
  if (lane == 0) mbar_arrive(smem_u32(&S.uempty[rs]));
  return u.nch > 0;
}

__global__ void __launch_bounds__(kThreads, 2)
    attn_tc_kernel(const __grid_constant__ CUtensorMap tq, const __grid_constant__ CUtensorMap tkv, const AttnArgs a,
                   int* ticket, int* err) {
  pdl_trigger();
  extern __shared__ uint8_t smem_raw[];
  AttnSmem& S = *reinterpret_cast<AttnSmem*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int D = a.H * 64;
  const int nwork = a.n_items * a.H;

  if (threadIdx.x == 0) {
    for (int i = 0; i < 2; ++i) {
      mbar_init(smem_u32(&S.qfull[i]), 1);
      mbar_init(smem_u32(&S.qempty[i]), 1);
      mbar_init(smem_u32(&S.pfull[i]), 4);
      mbar_init(smem_u32(&S.pfree[i]), 1);
    }
    for (int i = 0; i < kStages; ++i) {
      mbar_init(smem_u32(&S.kfull[i]), 1);
      mbar_init(smem_u32(&S.vfull[i]), 1);
      mbar_init(smem_u32(&S.kvempty[i]), 1);
    }
    for (int i = 0; i < kRing; ++i) {
      mbar_init(smem_u32(&S.ufull[i]), 1);
      mbar_init(smem_u32(&S.uempty[i]), 5);  // the MMA issuer and the four softmax warps
    }
    mbar_init(smem_u32(&S.sfull), 1);
    mbar_init(smem_u32(&S.sfree), 4);
    mbar_init(smem_u32(&S.drain), 1);
    S.abort = 0;
    fence_mbar_init();
  }
  if (warp == 0 && lane == 0) { tma_prefetch_desc(&tq); tma_prefetch_desc(&tkv); }
  if (warp == 1) { tmem_alloc(smem_u32(&S.tmem), kTmemCols); tmem_relinquish(); }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = S.tmem;
  pdl_wait();  // qkv (and the work counter's reset by the previous launch) are complete
  volatile int* abort = &S.abort;

  if (warp == 0) {
    if (lane == 0) {
      // ---------------- TMA producer. Chunk c uses K / V stage c % kStages (phase c / kStages).
      int nq[2] = {0, 0}, nk[kStages] = {}, nv[kStages] = {};
      int c = 0, ui = 0, nu = 0;
      bool ok = true;
      while (ok) {
        // claim the next unit (dynamic: the longest remaining first) and publish it
        const int rs = nu % kRing;
        if (nu >= kRing && !mbar_wait(smem_u32(&S.uempty[rs]), ((nu / kRing) - 1) & 1, abort, err, kErrAttnLoad)) break;
        Unit u;
        const bool valid = unit_of(a, atomicAdd(ticket, 1), nwork, u);
        if (!valid) u.nch = 0;
        S.units[rs] = u;
        mbar_arrive(smem_u32(&S.ufull[rs]));
        ++nu;
        if (!valid) break;
        const int qs = ui & 1;
        if (ui >= 2 && !mbar_wait(smem_u32(&S.qempty[qs]), ((ui >> 1) - 1) & 1, abort, err, kErrAttnLoad)) break;
        mbar_expect_tx(smem_u32(&S.qfull[qs]), kQBytes);
        tma_load_3d(smem_u32(S.q[qs]), &tq, u.h * 64, u.base + u.q0, 0, smem_u32(&S.qfull[qs]));
        ++nq[qs];
        ++ui;
        for (int j = 0; j < u.nch; ++j, ++c) {
          const int st = c % kStages, ph = ((c / kStages) - 1) & 1;
          const int krow = u.base + u.lo + j * kKeys;
          if (c >= kStages && !mbar_wait(smem_u32(&S.kvempty[st]), ph, abort, err, kErrAttnLoad)) { ok = false; break; }
          mbar_expect_tx(smem_u32(&S.kfull[st]), kKVBytes);
          tma_load_3d(smem_u32(S.k[st]), &tkv, D + u.h * 64, krow, 0, smem_u32(&S.kfull[st]));
          ++nk[st];
          mbar_expect_tx(smem_u32(&S.vfull[st]), kKVBytes);
          tma_load_3d(smem_u32(S.v[st]), &tkv, 2 * D + u.h * 64, krow, 0, smem_u32(&S.vfull[st]));
          ++nv[st];
        }
      }
      if (*abort) {  // let the loads in flight land before the CTA can exit
        for (int i = 0; i < 2; ++i) drain_phase(smem_u32(&S.qfull[i]), nq[i], err);
        for (int i = 0; i < kStages; ++i) {
          drain_phase(smem_u32(&S.kfull[i]), nk[i], err);
          drain_phase(smem_u32(&S.vfull[i]), nv[i], err);
        }
      }
    }
  } else if (warp == 1) {
    if (lane == 0) {
      // ---------------- MMA issuer; the PV of chunk c is issued after the S of chunk c+1
      bool issued = false, ok = true;
      int c = 0, ui = 0;
      int pend_c = -1, pend_j = 0;  // chunk whose PV is still to be issued
      uint32_t pend_o = kTmemO;     // its O accumulator (per unit parity)
      auto issue_pv = [&]() -> bool {
        const int st = pend_c % kStages, pb = pend_c & 1;
        if (!mbar_wait(smem_u32(&S.pfull[pb]), (pend_c >> 1) & 1, abort, err, kErrAttnMma)) return false;
        if (!mbar_wait(smem_u32(&S.vfull[st]), (pend_c / kStages) & 1, abort, err, kErrAttnMma)) return false;
        tc_fence_after();
        const uint32_t v_b = smem_u32(S.v[st]);
#pragma unroll
        for (int kk = 0; kk < kKeys / 16; ++kk)  // 16 keys = 8 packed TMEM columns of P per step
          umma_bf16_ts(tmem + pend_o, tmem + kTmemP + pb * 32 + kk * 8, sdesc_mn128(v_b + kk * 2048), kIdescPV,
                       (pend_j > 0 || kk > 0) ? 1u : 0u);
        umma_commit(smem_u32(&S.pfree[pb]));
        umma_commit(smem_u32(&S.kvempty[st]));
        pend_c = -1;
        return true;
      };
      Unit u;
      for (int nu = 0; ok && take_unit(S, nu, u, abort, err, kErrAttnMma, 0); ++nu) {
        const int qs = ui & 1;
        if (!mbar_wait(smem_u32(&S.qfull[qs]), (ui >> 1) & 1, abort, err, kErrAttnMma)) break;
        ++ui;
        const uint32_t q_a = smem_u32(S.q[qs]);
        for (int j = 0; j < u.nch; ++j, ++c) {
          const int st = c % kStages;
          if (!mbar_wait(smem_u32(&S.kfull[st]), (c / kStages) & 1, abort, err, kErrAttnMma)) { ok = false; break; }
          // the softmax has read S(c-1) out of TMEM
          if (c >= 1 && !mbar_wait(smem_u32(&S.sfree), (c - 1) & 1, abort, err, kErrAttnMma)) {
            ok = false;
            break;
          }
          tc_fence_after();
          const uint32_t k_b = smem_u32(S.k[st]);
#pragma unroll
          for (int k = 0; k < 4; ++k)
            umma_bf16(tmem + kTmemS, sdesc_k128(q_a + k * 32), sdesc_k128(k_b + k * 32), kIdescS, k > 0 ? 1u : 0u);
          issued = true;
          umma_commit(smem_u32(&S.sfull));
          if (j == u.nch - 1) umma_commit(smem_u32(&S.qempty[qs]));
          if (pend_c >= 0 && !issue_pv()) { ok = false; break; }
          pend_c = c;
          pend_j = j;
          pend_o = kTmemO + static_cast<uint32_t>(((ui - 1) & 1) * 64);
        }
      }
      if (ok && pend_c >= 0) issue_pv();
      if (*abort && issued) {  // the MMAs already issued finish before TMEM is released
        umma_commit(smem_u32(&S.drain));
        const long long t0 = clock64();
        while (!mbar_try(smem_u32(&S.drain), 0)) {
          if (clock64() - t0 > kWaitBudgetCycles) { atomicCAS(err, 0, kErrGemmDrain); break; }
        }
      }
    }
  } else {
    // ---------------- softmax warps 2..5; warp w owns TMEM lanes (query rows) 32*(w%4) .. +31
    const int qw = warp & 3;
    const int row = qw * 32 + lane;
    const uint32_t tl = tmem + (static_cast<uint32_t>(qw * 32) << 16);
    const float cs = a.scale * 1.4426950408889634f;  // softmax in base 2
    const int win = a.window;
    bf16* out = static_cast<bf16*>(a.out);
    int c = 0, uiu = 0;
    bool ok = true;
    // The epilogue of a unit (O / l out of TMEM into the output rows) runs after the first chunk of
    // the next unit, when the unit's last PV has long finished; O is double-buffered per unit parity.
    struct Pending {
      bool on;
      int cl;          // last chunk of the unit
      uint32_t oc;     // its O columns
      long long row0;  // output row of this thread (packed)
      int h;
      bool valid;      // this thread's query row lies inside the sequence
      float inv;       // 1 / l
    } pe{false, 0, 0, 0, 0, false, 0.f};
    auto flush = [&]() -> bool {
      if (!pe.on) return true;
      pe.on = false;
      if (!mbar_wait(smem_u32(&S.pfree[pe.cl & 1]), (pe.cl >> 1) & 1, abort, err, kErrAttnSoftmax)) return false;
      tc_fence_after();
      uint4* dst = reinterpret_cast<uint4*>(out + pe.row0 * D + pe.h * 64);
#pragma unroll
      for (int half = 0; half < 2; ++half) {
        float o[32];
        tmem_ld32(tl + pe.oc + 32 * half, o);
        if (pe.valid) {
#pragma unroll
          for (int j8 = 0; j8 < 4; ++j8) {
            const float* v = o + 8 * j8;
            const float inv = pe.inv;
            dst[4 * half + j8] = make_uint4(pack_bf16x2(v[0] * inv, v[1] * inv), pack_bf16x2(v[2] * inv, v[3] * inv),
                                            pack_bf16x2(v[4] * inv, v[5] * inv), pack_bf16x2(v[6] * inv, v[7] * inv));
          }
        }
      }
      tc_fence_before();  // O is rewritten by the unit after next only after this warp's later arrivals
      return true;
    };
    Unit u;
    int nu = 0;
    bool have = take_unit(S, nu++, u, abort, err, kErrAttnSoftmax, lane);
    while (ok && have) {
      const uint32_t oc = kTmemO + static_cast<uint32_t>((uiu & 1) * 64);
      ++uiu;
      const int qpos = u.q0 + row;
      const int wr0 = u.q0 + qw * 32;  // first query position of this warp
      // keys this row can see: [vlo, vlo + span)
      const int vlo = win > 0 ? max(0, qpos - win) : 0;
      const int vhi = win > 0 ? min(u.len, qpos + win + 1) : u.len;
      const unsigned span = vhi > vlo ? static_cast<unsigned>(vhi - vlo) : 0u;
      float m_used = -INFINITY;
      float2 la = make_float2(0.f, 0.f), lb = make_float2(0.f, 0.f);
      for (int j = 0; j < u.nch; ++j, ++c) {
        const int k0 = u.lo + j * kKeys, pb = c & 1;
        // per 32-key group, warp-uniform: 0 nobody sees a key, 1 some keys masked, 2 all visible
        int gk[2];
#pragma unroll
        for (int g = 0; g < 2; ++g) {
          const int kg0 = k0 + 32 * g, kg1 = kg0 + 31;
          if (win == 0) {
            gk[g] = kg0 >= u.len ? 0 : (kg1 < u.len ? 2 : 1);
          } else {
            const bool none = kg0 >= u.len || kg1 < wr0 - win || kg0 > wr0 + 31 + win;
            const bool all = kg1 < u.len && kg0 >= wr0 + 31 - win && kg1 <= wr0 + win;
            gk[g] = none ? 0 : (all ? 2 : 1);
          }
        }
        // mask (invisible scores -> -inf) and row max (three-input max, four chains)
        if (!mbar_wait(smem_u32(&S.sfull), c & 1, abort, err, kErrAttnSoftmax)) { ok = false; break; }
        tc_fence_after();
        uint32_t tr[64];
        tmem_ld64_issue(tl + kTmemS, tr);
        tmem_ld64_wait(tr);
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(smem_u32(&S.sfree));  // S may take chunk c+1
        float mq[4] = {-INFINITY, -INFINITY, -INFINITY, -INFINITY};
#pragma unroll
        for (int g = 0; g < 2; ++g) {
          if (gk[g] == 1) {
            const int d0 = k0 + 32 * g - vlo;
#pragma unroll
            for (int i = 0; i < 32; ++i)
              if (static_cast<unsigned>(d0 + i) >= span) tr[32 * g + i] = 0xff800000u;  // -inf
          }
          if (gk[g] != 0) {
#pragma unroll
            for (int i = 0; i < 32; i += 2)
              mq[(i >> 1) & 3] = fmax3(mq[(i >> 1) & 3], __uint_as_float(tr[32 * g + i]), __uint_as_float(tr[32 * g + i + 1]));
          }
        }
        const float mx = fmax3(mq[0], mq[1], fmaxf(mq[2], mq[3])) * cs;
        // raise the reference max only when it grows by more than 2^8 (p stays <= 256 otherwise)
        const float m_new = fmaxf(m_used, mx);
        const bool resc = m_new > m_used + 8.f;
        // O (and l) hold something to rescale only once a key of this row has been visible: until
        // then every P of the row was 0, so its O row is exactly 0 (and the V rows are finite)
        const bool resc_o = resc && m_used != -INFINITY;
        float alpha = 1.f;
        if (resc) {
          alpha = ex2(m_used - m_new);  // 0 on the first visible chunk (m_used = -inf)
          la.x *= alpha; la.y *= alpha; lb.x *= alpha; lb.y *= alpha;
          m_used = m_new;
        }
        const float msub = m_used == -INFINITY ? 0.f : m_used;
        const float2 cs2 = make_float2(cs, cs), nm2 = make_float2(-msub, -msub);
        uint32_t pk[32];
#pragma unroll
        for (int g = 0; g < 2; ++g) {
          if (gk[g] == 0) {
#pragma unroll
            for (int i = 0; i < 16; ++i) pk[16 * g + i] = 0u;
          } else {
#pragma unroll
            for (int i = 0; i < 16; ++i) {
              const float2 x =
                  ffma2(make_float2(__uint_as_float(tr[32 * g + 2 * i]), __uint_as_float(tr[32 * g + 2 * i + 1])), cs2, nm2);
              const float2 pp = make_float2(ex2(x.x), ex2(x.y));
              if (i & 1) lb = fadd2(lb, pp); else la = fadd2(la, pp);
              pk[16 * g + i] = pack_bf16x2(pp.x, pp.y);
            }
          }
        }
        // O may only be rescaled once the PV in flight (chunk c-1) has landed; a row's first visible
        // chunk needs no rescale
        if (j > 0 && __any_sync(0xffffffffu, resc_o)) {
          if (!mbar_wait(smem_u32(&S.pfree[(c - 1) & 1]), ((c - 1) >> 1) & 1, abort, err, kErrAttnSoftmax)) {
            ok = false;
            break;
          }
          tc_fence_after();
#pragma unroll
          for (int half = 0; half < 2; ++half) {
            float o[32];
            tmem_ld32(tl + oc + 32 * half, o);
#pragma unroll
            for (int i = 0; i < 32; ++i) o[i] *= alpha;
            tmem_st32(tl + oc + 32 * half, o);
          }
        }
        // P buffer pb was last read by the PV of chunk c-2
        if (c >= 2 && !mbar_wait(smem_u32(&S.pfree[pb]), ((c >> 1) - 1) & 1, abort, err, kErrAttnSoftmax)) {
          ok = false;
          break;
        }
        tc_fence_after();
        tmem_st32_issue(tl + kTmemP + pb * 32, pk);
        tmem_st32_wait(pk);
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(smem_u32(&S.pfull[pb]));
        if (j == 0 && !flush()) { ok = false; break; }
      }
      if (!ok) break;
      // ---- this unit's epilogue, deferred until after the next unit's first chunk
      const float l = (la.x + la.y) + (lb.x + lb.y);
      pe.on = true;
      pe.cl = c - 1;
      pe.oc = oc;
      pe.row0 = (long long)u.base + qpos;
      pe.h = u.h;
      pe.valid = row < u.len - u.q0;
      pe.inv = l > 0.f ? 1.f / l : 0.f;
      have = take_unit(S, nu++, u, abort, err, kErrAttnSoftmax, lane);
    }
    if (ok && !flush()) ok = false;
  }

  tc_fence_before();
  __syncwarp();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem, kTmemCols);
  }
  // The last CTA out resets the work counter for the next launch: every CTA has made its final
  // claim before it counts itself out.
  if (threadIdx.x == 0) {
    __threadfence();
    if (atomicAdd(ticket + 1, 1) == static_cast<int>(gridDim.x) - 1) {
      ticket[0] = 0;
      ticket[1] = 0;
      __threadfence();
    }
  }
}

int g_num_sms = 0;

}  // namespace

cudaError_t attn_tc_prepare_device() {
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return e;
  e = cudaDeviceGetAttribute(&g_num_sms, cudaDevAttrMultiProcessorCount, dev);
  if (e != cudaSuccess) return e;
  return cudaFuncSetAttribute(attn_tc_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                              static_cast<int>(attn_smem_bytes()));
}

cudaError_t attn_tc_launch(const CUtensorMap& tq, const CUtensorMap& tkv, const AttnArgs& a, int* ticket, int* err,
                           cudaStream_t st) {
  if (a.gathered || a.out_planes != 1 || a.n_items <= 0 || a.H <= 0 || !ticket) return cudaErrorInvalidValue;
  const int work = a.n_items * a.H;
  const int sms = g_num_sms > 0 ? g_num_sms : 148;
  const int grid = work < 2 * sms ? work : 2 * sms;
  return launch_pdl(attn_tc_kernel, dim3(grid), dim3(kThreads), attn_smem_bytes(), st, tq, tkv, a, ticket, err);
}

}  // namespace laya
