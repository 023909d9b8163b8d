// Persistent tcgen05 GEMM for sm_100a: C[M,N] = A[M,K] * B[N,K]^T, bf16 operands, fp32 accumulation
// in tensor memory, fused epilogues. Replaces the reference's hipBLAS / hipBLASLt / wgemm GEMM layer
// (src/engine.hip:238-391, src/wgemm.hip:24-151): the projections Wqkv, Wo, Wi, Wmo and the head /
// scorer Linears all run through this one kernel family.
//
// CTA layout (192 threads, one CTA per SM):
//   warp 0      TMA producer: 64-wide K slabs of A (128 rows) and B (BN rows) into a STAGES-deep ring
//   warp 1      TMEM owner + MMA issuer: 4 x tcgen05.mma (128 x BN x 16) per slab into one of two
//               TMEM accumulators, so the epilogue of tile i overlaps the main loop of tile i+1
//   warps 2..5  epilogue: tcgen05.ld of their 32-lane TMEM quarter (one output row per thread), the
//               fused math (bias / ReLU / GELU / RoPE / GeGLU / fp32 residual add) and the stores.
// gemm_prepare_device() must run once per device (it raises the dynamic shared-memory limit).
// Tiles are walked in row-block-major order with N fastest, so the CTAs in flight share one weight
// matrix through L2 and read each activation row block from HBM once.
#include "common.cuh"
#include "kernels.h"
#include <algorithm>
#include <cstdio>

namespace laya {

namespace {

constexpr int kBM = 128;
constexpr int kBK = 64;
constexpr int kThreads = 192;

template <int BN>
struct StagesFor { static constexpr int value = BN == 256 ? 4 : 6; };

template <int BN, int STAGES>
struct GemmSmem {
  alignas(1024) bf16 a[STAGES][kBM * kBK];
  alignas(1024) bf16 b[STAGES][BN * kBK];
  alignas(1024) uint8_t stg[4][8192];  // epilogue staging: two 32-row x 128-byte tiles per epilogue warp
  alignas(8) uint64_t full[STAGES];
  uint64_t empty[STAGES];
  uint64_t accf[2];
  uint64_t acce[2];
  uint64_t drain;
  uint32_t tmem;
  int abort;
};

template <int BN>
constexpr size_t gemm_smem_bytes() {
  return sizeof(GemmSmem<BN, StagesFor<BN>::value>) + 1024;
}

__device__ __forceinline__ float apply_act(float v, int act) {
  if (act == ACT_RELU) return fmaxf(v, 0.f);
  if (act == ACT_GELU) return gelu_as(v);
  return v;
}

// ---- epilogue output path: per-warp double-buffered 32-row staging tiles (4 KB each, 128-byte rows
// in the 128-byte swizzle) written one row per thread, then stored (or reduce-added) to global
// memory by one TMA bulk-tensor operation issued by lane 0. A buffer is reused only after the store
// issued from it two rounds earlier has finished reading shared memory.
struct Stager {
  uint8_t* base;  // 8 KB, 1024-byte aligned
  int buf;
};

__device__ __forceinline__ uint8_t* stg_acquire(Stager& s, int lane) {
  if (lane == 0) asm volatile("cp.async.bulk.wait_group.read 1;" ::: "memory");
  __syncwarp();
  return s.base + s.buf * 4096;
}

__device__ __forceinline__ void stg_issue(Stager& s, int lane, const CUtensorMap* map, int col, int row, int plane,
                                          bool reduce_add) {
  asm volatile("fence.proxy.async.shared::cta;" ::: "memory");  // generic-proxy writes -> TMA reads
  __syncwarp();
  if (lane == 0) {
    const uint32_t src = smem_u32(s.base + s.buf * 4096);
    if (reduce_add)
      asm volatile("cp.reduce.async.bulk.tensor.3d.global.shared::cta.add.tile.bulk_group [%0, {%2, %3, %4}], [%1];"
                   ::"l"(reinterpret_cast<uint64_t>(map)), "r"(src), "r"(col), "r"(row), "r"(plane)
                   : "memory");
    else
      asm volatile("cp.async.bulk.tensor.3d.global.shared::cta.tile.bulk_group [%0, {%2, %3, %4}], [%1];"
                   ::"l"(reinterpret_cast<uint64_t>(map)), "r"(src), "r"(col), "r"(row), "r"(plane)
                   : "memory");
    asm volatile("cp.async.bulk.commit_group;" ::: "memory");
  }
  s.buf ^= 1;
}

__device__ __forceinline__ void stg_drain(int lane) {
  if (lane == 0) asm volatile("cp.async.bulk.wait_group 0;" ::: "memory");
  __syncwarp();
}

// Row `lane` of a 32 x 64 bf16 tile / 32 x 32 fp32 tile, 16-byte chunk j at (j ^ (lane % 8)).
__device__ __forceinline__ void put_bf16_row(uint8_t* tile, int lane, const float* v) {
#pragma unroll
  for (int j = 0; j < 8; ++j) {
    const uint4 q = make_uint4(pack_bf16x2(v[8 * j], v[8 * j + 1]), pack_bf16x2(v[8 * j + 2], v[8 * j + 3]),
                               pack_bf16x2(v[8 * j + 4], v[8 * j + 5]), pack_bf16x2(v[8 * j + 6], v[8 * j + 7]));
    *reinterpret_cast<uint4*>(tile + lane * 128 + ((j ^ (lane & 7)) << 4)) = q;
  }
}
__device__ __forceinline__ void put_f32_row(uint8_t* tile, int lane, const float* v) {
#pragma unroll
  for (int j = 0; j < 8; ++j)
    *reinterpret_cast<float4*>(tile + lane * 128 + ((j ^ (lane & 7)) << 4)) =
        make_float4(v[4 * j], v[4 * j + 1], v[4 * j + 2], v[4 * j + 3]);
}

// 64 consecutive output columns of the warp's 32 rows: one bf16 box (plus the lo plane in
// OUT_BF16X2 mode), or two fp32 boxes.
__device__ __forceinline__ void emit64(Stager& s, int lane, const CUtensorMap* map, int mode, float (&v)[64], int col,
                                       int row0) {
  if (mode == OUT_F32) {
    uint8_t* t = stg_acquire(s, lane);
    put_f32_row(t, lane, v);
    stg_issue(s, lane, map, col, row0, 0, false);
    t = stg_acquire(s, lane);
    put_f32_row(t, lane, v + 32);
    stg_issue(s, lane, map, col + 32, row0, 0, false);
    return;
  }
  uint8_t* t = stg_acquire(s, lane);
  put_bf16_row(t, lane, v);
  stg_issue(s, lane, map, col, row0, 0, false);
  if (mode == OUT_BF16X2) {
#pragma unroll
    for (int i = 0; i < 64; ++i) v[i] -= __bfloat162float(__float2bfloat16_rn(v[i]));
    t = stg_acquire(s, lane);
    put_bf16_row(t, lane, v);
    stg_issue(s, lane, map, col, row0, 1, false);
  }
}

// Epilogue of one tile for one warp (32 rows starting at row0; thread `lane` holds row row0+lane
// after each tcgen05.ld). Every tcgen05.ld is executed by the whole warp. Output boxes are clipped by
// the TMA unit at the row extent of the output map.
// `ld(off, v)` fills v with tile columns off..off+31 of this thread's row: from tensor memory, or
// (split-K) summed from the workspace partials.
template <int BN, int EPI, class Loader>
__device__ __forceinline__ void epilogue_tile(const Loader& ld, int row0, int lane, int nb, const GemmShape& sh,
                                              const GemmEpi& ep, const CUtensorMap* out_map, Stager& stg) {
  const int row = row0 + lane;
  const bool valid = row < sh.M;
  if constexpr (EPI == EPI_GEGLU) {
    // B rows are interleaved in groups of 64: [64 input rows, their 64 gate rows] per 128 columns.
    for (int s = 0; s < BN; s += 128) {
      const int ocol = nb * (BN / 2) + s / 2;  // first output column of this 128-column group
      if (ocol >= ep.geglu_I) break;
      float v[64];
#pragma unroll
      for (int c = 0; c < 64; c += 32) {
        float xin[32], gate[32];
        __syncwarp();
        ld(s + c, xin);
        ld(s + 64 + c, gate);
#pragma unroll
        for (int i = 0; i < 32; ++i) v[c + i] = gelu_as(xin[i]) * gate[i];
      }
      emit64(stg, lane, out_map, ep.out_mode, v, ocol, row0);
    }
  } else if constexpr (EPI == EPI_ROPE) {
    // cos/sin of this row's position are the same for every head: load them once per tile, as
    // 16 independent 16-byte loads, and reuse them for the BN/64 heads of the tile.
    float cs[32], sn[32];
    const bool any_rot = nb * BN < ep.rope_cols;
    if (any_rot && valid) {
      int p = ep.pos[row];
      if (!LAYA_IN_BOUNDS(ep.rope_rows <= 0 || (p >= 0 && p < ep.rope_rows), ep.err, kErrBoundsRope)) p = 0;
      const float4* ct = reinterpret_cast<const float4*>(ep.cos_t + (size_t)p * 32);
      const float4* st = reinterpret_cast<const float4*>(ep.sin_t + (size_t)p * 32);
#pragma unroll
      for (int i = 0; i < 8; ++i) {
        const float4 c4 = ct[i], s4 = st[i];
        cs[4 * i] = c4.x; cs[4 * i + 1] = c4.y; cs[4 * i + 2] = c4.z; cs[4 * i + 3] = c4.w;
        sn[4 * i] = s4.x; sn[4 * i + 1] = s4.y; sn[4 * i + 2] = s4.z; sn[4 * i + 3] = s4.w;
      }
    }
    for (int h = 0; h < BN; h += 64) {
      const int col = nb * BN + h;
      if (col >= sh.N) break;
      float v[64];
      __syncwarp();
      ld(h, *reinterpret_cast<float(*)[32]>(v));
      ld(h + 32, *reinterpret_cast<float(*)[32]>(v + 32));
      if (ep.bias) {
#pragma unroll
        for (int i = 0; i < 64; ++i) v[i] += ep.bias[col + i];
      }
      if (valid && col < ep.rope_cols) {
#pragma unroll
        for (int i = 0; i < 32; ++i) {
          const float a = v[i], b = v[32 + i];
          v[i] = a * cs[i] - b * sn[i];
          v[32 + i] = b * cs[i] + a * sn[i];
        }
      }
      emit64(stg, lane, out_map, ep.out_mode, v, col, row0);
    }
  } else if constexpr (EPI == EPI_RESID) {
    // x += acc (+ bias) as a TMA reduce-add of 32 x 32 fp32 boxes: the read-modify-write of the
    // residual happens in L2, never in registers.
    for (int c = 0; c < BN; c += 32) {
      const int col = nb * BN + c;
      if (col >= sh.N) break;
      float v[32];
      __syncwarp();
      ld(c, v);
      if (ep.bias) {
#pragma unroll
        for (int i = 0; i < 32; ++i) v[i] += ep.bias[col + i];
      }
      uint8_t* t = stg_acquire(stg, lane);
      put_f32_row(t, lane, v);
      stg_issue(stg, lane, out_map, col, row0, 0, true);
    }
  } else {
    for (int c = 0; c < BN; c += 64) {
      const int col = nb * BN + c;
      if (col >= sh.N) break;
      float v[64];
      __syncwarp();
      ld(c, *reinterpret_cast<float(*)[32]>(v));
      ld(c + 32, *reinterpret_cast<float(*)[32]>(v + 32));  // N is a multiple of 64
      if (ep.bias) {
#pragma unroll
        for (int i = 0; i < 64; ++i) v[i] += ep.bias[col + i];
      }
      if (ep.act != ACT_NONE) {
#pragma unroll
        for (int i = 0; i < 64; ++i) v[i] = apply_act(v[i], ep.act);
      }
      emit64(stg, lane, out_map, ep.out_mode, v, col, row0);
    }
  }
}

template <int BN, int EPI, bool SPLIT>
__global__ void __launch_bounds__(kThreads, 1)
    gemm_tc_kernel(const __grid_constant__ CUtensorMap ta, const __grid_constant__ CUtensorMap tb,
                   const __grid_constant__ CUtensorMap tc, const GemmShape sh, const GemmEpi ep, int* err) {
  constexpr int STAGES = StagesFor<BN>::value;
  constexpr uint32_t kIdesc = idesc_bf16(kBM, BN);
  constexpr uint32_t kStageBytes = (kBM + BN) * kBK * 2;
  using Smem = GemmSmem<BN, STAGES>;
  pdl_trigger();
  extern __shared__ uint8_t smem_raw[];
  Smem& S = *reinterpret_cast<Smem*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int num_n = (sh.N + BN - 1) / BN;
  const int splits = SPLIT ? sh.splits : 1;
  // work unit w = (output tile t, K slice sp), slices of one tile adjacent so they run concurrently
  const int work = ((sh.M + kBM - 1) / kBM) * num_n * splits;
  const int kb_seg = (sh.K + kBK - 1) / kBK;
  const int nkb = kb_seg * sh.nseg;

  if (threadIdx.x == 0) {
    for (int s = 0; s < STAGES; ++s) { mbar_init(smem_u32(&S.full[s]), 1); mbar_init(smem_u32(&S.empty[s]), 1); }
    for (int a = 0; a < 2; ++a) { mbar_init(smem_u32(&S.accf[a]), 1); mbar_init(smem_u32(&S.acce[a]), 4); }
    mbar_init(smem_u32(&S.drain), 1);
    S.abort = 0;
    fence_mbar_init();
  }
  if (warp == 0 && lane == 0) { tma_prefetch_desc(&ta); tma_prefetch_desc(&tb); tma_prefetch_desc(&tc); }
  if (warp == 1) { tmem_alloc(smem_u32(&S.tmem), 2 * BN); tmem_relinquish(); }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = S.tmem;
  pdl_wait();  // the previous kernel's outputs (this GEMM's A operand, the residual) are complete
  volatile int* abort = &S.abort;

  if (warp == 0) {
    if (lane == 0) {
      // ---------------- TMA producer
      uint32_t stage = 0, phase = 0;
      uint32_t issued_mask = 0, last_phase = 0;  // for the abort drain
      for (int w = blockIdx.x; w < work; w += gridDim.x) {
        const int t = w / splits, sp = w - t * splits;
        const int mb = t / num_n, nb = t - (t / num_n) * num_n;
        const int kb0 = sp * nkb / splits, kb1 = (sp + 1) * nkb / splits;
        bool ok = true;
        for (int kb = kb0; kb < kb1; ++kb) {
          if (!mbar_wait(smem_u32(&S.empty[stage]), phase ^ 1, abort, err, kErrGemmEmpty)) { ok = false; break; }
          const int seg = kb / kb_seg;
          const int kk = (kb - seg * kb_seg) * kBK;
          const int ap = seg == 2 ? 1 : 0, bp = seg == 1 ? 1 : 0;
          const uint32_t fb = smem_u32(&S.full[stage]);
          mbar_expect_tx(fb, kStageBytes);
          tma_load_3d(smem_u32(S.a[stage]), &ta, kk, mb * kBM, ap, fb);
          tma_load_3d(smem_u32(S.b[stage]), &tb, kk, nb * BN, bp, fb);
          issued_mask |= 1u << stage;
          last_phase = (last_phase & ~(1u << stage)) | (phase << stage);
          if (++stage == STAGES) { stage = 0; phase ^= 1; }
        }
        if (!ok) break;
      }
      if (*abort) {
        // Let every TMA write that may still be in flight land before the CTA can exit.
        const long long t0 = clock64();
        for (int s = 0; s < STAGES; ++s) {
          if (!(issued_mask & (1u << s))) continue;
          while (!mbar_try(smem_u32(&S.full[s]), (last_phase >> s) & 1)) {
            if (clock64() - t0 > kWaitBudgetCycles) { atomicCAS(err, 0, kErrGemmDrain); break; }
          }
        }
      }
    }
  } else if (warp == 1) {
    if (lane == 0) {
      // ---------------- MMA issuer
      uint32_t stage = 0, phase = 0;
      int local = 0;
      bool issued_any = false;
      for (int w = blockIdx.x; w < work; w += gridDim.x, ++local) {
        const int sp = w - (w / splits) * splits;
        const int kb0 = sp * nkb / splits, kb1 = (sp + 1) * nkb / splits;
        const int acc = local & 1;
        const uint32_t accph = (local >> 1) & 1;
        if (!mbar_wait(smem_u32(&S.acce[acc]), accph ^ 1, abort, err, kErrGemmAccEmpty)) break;
        tc_fence_after();
        const uint32_t d = tmem + acc * BN;
        bool ok = true;
        for (int kb = kb0; kb < kb1; ++kb) {
          if (!mbar_wait(smem_u32(&S.full[stage]), phase, abort, err, kErrGemmFull)) { ok = false; break; }
          tc_fence_after();
          const uint32_t a0 = smem_u32(S.a[stage]), b0 = smem_u32(S.b[stage]);
#pragma unroll
          for (int k = 0; k < kBK / 16; ++k)
            umma_bf16(d, sdesc_k128(a0 + k * 32), sdesc_k128(b0 + k * 32), kIdesc,
                      (kb != kb0 || k != 0) ? 1u : 0u);
          issued_any = true;
          umma_commit(smem_u32(&S.empty[stage]));
          if (++stage == STAGES) { stage = 0; phase ^= 1; }
        }
        if (!ok) break;
        umma_commit(smem_u32(&S.accf[acc]));
      }
      if (*abort && issued_any) {
        // Wait for the MMAs already issued before TMEM is released.
        umma_commit(smem_u32(&S.drain));
        const long long t0 = clock64();
        while (!mbar_try(smem_u32(&S.drain), 0)) {
          if (clock64() - t0 > kWaitBudgetCycles) { atomicCAS(err, 0, kErrGemmDrain); break; }
        }
      }
    }
  } else {
    // ---------------- epilogue warps 2..5; warp w may only touch TMEM lanes 32*(w%4) .. +31
    const int q = warp & 3;
    Stager stager{S.stg[q], 0};
    int local = 0;
    for (int w = blockIdx.x; w < work; w += gridDim.x, ++local) {
      const int t = w / splits, sp = w - t * splits;
      const int acc = local & 1;
      const uint32_t accph = (local >> 1) & 1;
      const int mb = t / num_n, nb = t - (t / num_n) * num_n;
      const int row0 = mb * kBM + q * 32;
      if (!mbar_wait(smem_u32(&S.accf[acc]), accph, abort, err, kErrGemmAccFull)) break;
      tc_fence_after();
      const uint32_t tbase = tmem + acc * BN + (static_cast<uint32_t>(q * 32) << 16);
      if constexpr (!SPLIT) {
        epilogue_tile<BN, EPI>([&](int off, float (&v)[32]) { tmem_ld32(tbase + off, v); }, row0, lane, nb, sh, ep,
                               &tc, stager);
      } else {
        // Split-K: this slice's fp32 partial tile into plane `sp` of the workspace (TMA stores of
        // the staged 32 x 32 chunks; `tc` maps the workspace here). splitk_reduce_kernel then sums
        // the planes in slice order and runs the epilogue, so no CTA waits for another and the
        // result does not depend on which slice finished first.
        const int cols = min(BN, sh.N - nb * BN);
        for (int c = 0; c < cols; c += 32) {
          float v[32];
          __syncwarp();
          tmem_ld32(tbase + c, v);
          uint8_t* tile = stg_acquire(stager, lane);
          put_f32_row(tile, lane, v);
          stg_issue(stager, lane, &tc, nb * BN + c, row0, sp, false);
        }
      }
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(smem_u32(&S.acce[acc]));
    }
    stg_drain(lane);  // output stores finished before the CTA can exit
  }

  tc_fence_before();
  // Lanes 1..31 of the producer and MMA warps got here while lane 0 ran its loop: reconverge each
  // warp first, because the block barrier must be reached by whole warps.
  __syncwarp();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem, 2 * BN);
  }
}

// ------------------------------------------------------------------ split-K epilogue
// out = epilogue(sum over slices s of ws[s]) for rows < M, the slices summed in order. One thread per
// (row, 64-column output block, t = 0..7): output columns 4t..4t+3 and 32+4t..35+4t of the block (a
// RoPE rotation pairs column i with i + 32), or for GeGLU the block's outputs 8t..8t+7, whose input
// and gate sums sit at accumulator columns 128*blk + 8t.. and 128*blk + 64 + 8t.. (interleaved B).
__device__ __forceinline__ float4 add4(float4 a, float4 b) {
  return make_float4(a.x + b.x, a.y + b.y, a.z + b.z, a.w + b.w);
}

// Four consecutive output columns of one row in the epilogue's output format.
__device__ __forceinline__ void put4(const GemmShape& sh, const GemmEpi& ep, long long row, int ncols, int col,
                                     float4 v) {
  const long long at = row * ncols + col;
  if (ep.out_mode == OUT_F32) {
    *reinterpret_cast<float4*>(static_cast<float*>(sh.dst) + at) = v;
    return;
  }
  bf16* o = static_cast<bf16*>(sh.dst);
  const uint32_t h0 = pack_bf16x2(v.x, v.y), h1 = pack_bf16x2(v.z, v.w);
  *reinterpret_cast<uint2*>(o + at) = make_uint2(h0, h1);
  if (ep.out_mode == OUT_BF16X2) {
    const float2 f0 = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(&h0));
    const float2 f1 = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(&h1));
    *reinterpret_cast<uint2*>(o + sh.dst_plane + at) =
        make_uint2(pack_bf16x2(v.x - f0.x, v.y - f0.y), pack_bf16x2(v.z - f1.x, v.w - f1.y));
  }
}

template <int EPI>
__global__ void __launch_bounds__(256) splitk_reduce_kernel(const GemmShape sh, const GemmEpi ep) {
  pdl_trigger();
  pdl_wait();
  const int ncols = EPI == EPI_GEGLU ? ep.geglu_I : sh.N;
  const int per_row = (ncols / 64) * 8;
  const long long gid = static_cast<long long>(blockIdx.x) * 256 + threadIdx.x;
  const long long row = gid / per_row;
  if (row >= sh.M) return;
  const int rem = static_cast<int>(gid - row * per_row), blk = rem >> 3, t = rem & 7;
  const size_t plane = static_cast<size_t>(sh.M) * sh.N;
  const float* ws = sh.ws + static_cast<size_t>(row) * sh.N;
  auto sum4 = [&](int col) {
    float4 a = __ldcg(reinterpret_cast<const float4*>(ws + col));
    for (int s = 1; s < sh.splits; ++s) a = add4(a, __ldcg(reinterpret_cast<const float4*>(ws + s * plane + col)));
    return a;
  };
  if constexpr (EPI == EPI_GEGLU) {
    const int in = 128 * blk + 8 * t, out = 64 * blk + 8 * t;
    const float4 x0 = sum4(in), x1 = sum4(in + 4), g0 = sum4(in + 64), g1 = sum4(in + 68);
    put4(sh, ep, row, ncols, out,
         make_float4(gelu_as(x0.x) * g0.x, gelu_as(x0.y) * g0.y, gelu_as(x0.z) * g0.z, gelu_as(x0.w) * g0.w));
    put4(sh, ep, row, ncols, out + 4,
         make_float4(gelu_as(x1.x) * g1.x, gelu_as(x1.y) * g1.y, gelu_as(x1.z) * g1.z, gelu_as(x1.w) * g1.w));
  } else {
    const int c0 = 64 * blk + 4 * t, c1 = c0 + 32;
    float4 a = sum4(c0), b = sum4(c1);
    if (ep.bias) {
      a = add4(a, *reinterpret_cast<const float4*>(ep.bias + c0));
      b = add4(b, *reinterpret_cast<const float4*>(ep.bias + c1));
    }
    if constexpr (EPI == EPI_RESID) {
      float4* x0 = reinterpret_cast<float4*>(static_cast<float*>(sh.dst) + row * sh.N + c0);
      float4* x1 = reinterpret_cast<float4*>(static_cast<float*>(sh.dst) + row * sh.N + c1);
      *x0 = add4(*x0, a);
      *x1 = add4(*x1, b);
      return;
    }
    if constexpr (EPI == EPI_ROPE) {
      if (c0 < ep.rope_cols) {
        long long p = ep.pos[row];
        if (!LAYA_IN_BOUNDS(ep.rope_rows <= 0 || (p >= 0 && p < ep.rope_rows), ep.err, kErrBoundsRope)) p = 0;
        const float4 cs = *reinterpret_cast<const float4*>(ep.cos_t + p * 32 + 4 * t);
        const float4 sn = *reinterpret_cast<const float4*>(ep.sin_t + p * 32 + 4 * t);
        const float4 ra = make_float4(a.x * cs.x - b.x * sn.x, a.y * cs.y - b.y * sn.y, a.z * cs.z - b.z * sn.z,
                                      a.w * cs.w - b.w * sn.w);
        const float4 rb = make_float4(b.x * cs.x + a.x * sn.x, b.y * cs.y + a.y * sn.y, b.z * cs.z + a.z * sn.z,
                                      b.w * cs.w + a.w * sn.w);
        a = ra;
        b = rb;
      }
    } else if (ep.act != ACT_NONE) {
      a = make_float4(apply_act(a.x, ep.act), apply_act(a.y, ep.act), apply_act(a.z, ep.act), apply_act(a.w, ep.act));
      b = make_float4(apply_act(b.x, ep.act), apply_act(b.y, ep.act), apply_act(b.z, ep.act), apply_act(b.w, ep.act));
    }
    put4(sh, ep, row, ncols, c0, a);
    put4(sh, ep, row, ncols, c1, b);
  }
}

// Split-K residual epilogue with the following LayerNorm: one warp per row, x[row] += the slices'
// sum (+ bias) in the same order as splitk_reduce_kernel, then ln_out[row] = LayerNorm(x[row]) * ln_w
// through layer_norm_regs (as the LayerNorm kernel computes it).
template <int NV>
__global__ void __launch_bounds__(256) splitk_reduce_ln_kernel(const GemmShape sh, const GemmEpi ep) {
  pdl_trigger();
  pdl_wait();
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const long long row = static_cast<long long>(blockIdx.x) * 8 + warp;
  if (row >= sh.M) return;
  const size_t plane = static_cast<size_t>(sh.M) * sh.N;
  const float4* ws = reinterpret_cast<const float4*>(sh.ws + static_cast<size_t>(row) * sh.N);
  float4* x = reinterpret_cast<float4*>(static_cast<float*>(sh.dst) + row * sh.N);
  // slice by slice, the lane's NV pieces of a slice (and of x with the first) in flight together
  float4 a[NV], v[NV];
#pragma unroll
  for (int i = 0; i < NV; ++i) {
    a[i] = __ldcg(ws + lane + 32 * i);
    v[i] = x[lane + 32 * i];
  }
  for (int s = 1; s < sh.splits; ++s) {
    float4 p[NV];
#pragma unroll
    for (int i = 0; i < NV; ++i) p[i] = __ldcg(ws + s * (plane / 4) + lane + 32 * i);
#pragma unroll
    for (int i = 0; i < NV; ++i) a[i] = add4(a[i], p[i]);
  }
#pragma unroll
  for (int i = 0; i < NV; ++i) {
    const int c = lane + 32 * i;
    if (ep.bias) a[i] = add4(a[i], reinterpret_cast<const float4*>(ep.bias)[c]);
    v[i] = add4(v[i], a[i]);
    x[c] = v[i];
  }
  layer_norm_regs<NV>(v, ep.ln_w, nullptr, ep.ln_eps, sh.N, lane);
  store_bf16_planes<NV>(v, ep.ln_out + row * sh.N, ep.ln_out + ep.ln_plane + row * sh.N, ep.ln_planes, lane);
}

// ------------------------------------------------------------------ CTA-pair variant
// The same pipeline on a cluster of two CTAs (one per SM) computing a 256 x 256 tile with the 2-SM
// MMA (tcgen05.mma.cta_group::2): each CTA stages its own 128 rows of A and its own 128 rows of B, so
// per output element each SM reads a third less operand data than the 128 x 256 single-CTA tile.
// The even CTA issues the MMAs; both CTAs' TMA loads complete on the even CTA's `full` barrier, MMA
// completion is committed to both CTAs' `empty` / `accf` barriers, and both CTAs' epilogue warps
// arrive on the even CTA's `acce` barrier. Each CTA's epilogue owns its 128 accumulator rows.
constexpr int kPairStages = 6;

struct GemmSmemPair {
  alignas(1024) bf16 a[kPairStages][128 * kBK];
  alignas(1024) bf16 b[kPairStages][128 * kBK];
  alignas(1024) uint8_t stg[4][8192];
  alignas(8) uint64_t full[kPairStages];
  uint64_t empty[kPairStages];
  uint64_t accf[2];
  uint64_t acce[2];
  uint64_t drain;
  uint32_t tmem;
  int abort;
};
constexpr size_t gemm_pair_smem_bytes() { return sizeof(GemmSmemPair) + 1024; }

template <int EPI>
__global__ void __cluster_dims__(2, 1, 1) __launch_bounds__(kThreads, 1)
    gemm_tc_pair_kernel(const __grid_constant__ CUtensorMap ta, const __grid_constant__ CUtensorMap tb,
                        const __grid_constant__ CUtensorMap tc, const GemmShape sh, const GemmEpi ep, int* err) {
  constexpr int BN = 256;
  constexpr uint32_t kIdesc = idesc_bf16(256, BN);
  constexpr uint32_t kPairStageBytes = 2u * (128 + 128) * kBK * 2;  // both CTAs' A and B halves
  pdl_trigger();
  extern __shared__ uint8_t smem_raw[];
  GemmSmemPair& S =
      *reinterpret_cast<GemmSmemPair*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const uint32_t rank = cluster_ctarank();
  const bool leader = rank == 0;
  const int cid = static_cast<int>(cluster_id_x()), ncl = static_cast<int>(num_clusters_x());
  const int num_n = (sh.N + BN - 1) / BN;
  const int tiles = ((sh.M + 255) / 256) * num_n;
  const int kb_seg = (sh.K + kBK - 1) / kBK;
  const int nkb = kb_seg * sh.nseg;

  if (threadIdx.x == 0) {
    for (int s = 0; s < kPairStages; ++s) { mbar_init(smem_u32(&S.full[s]), 1); mbar_init(smem_u32(&S.empty[s]), 1); }
    for (int a = 0; a < 2; ++a) { mbar_init(smem_u32(&S.accf[a]), 1); mbar_init(smem_u32(&S.acce[a]), 8); }
    mbar_init(smem_u32(&S.drain), 1);
    S.abort = 0;
    fence_mbar_init();
  }
  if (warp == 0 && lane == 0) { tma_prefetch_desc(&ta); tma_prefetch_desc(&tb); tma_prefetch_desc(&tc); }
  if (warp == 1) { tmem_alloc_pair(smem_u32(&S.tmem), 2 * BN); tmem_relinquish_pair(); }
  tc_fence_before();
  cluster_sync_all();  // both CTAs' barriers are initialised before any cross-CTA signal
  tc_fence_after();
  const uint32_t tmem = S.tmem;
  pdl_wait();  // the previous kernel's outputs (this GEMM's A operand, the residual) are complete
  volatile int* abort = &S.abort;

  if (warp == 0) {
    if (lane == 0) {
      uint32_t stage = 0, phase = 0;
      uint32_t issued_mask = 0, last_phase = 0;
      for (int t = cid; t < tiles; t += ncl) {
        const int mb = t / num_n, nb = t - (t / num_n) * num_n;
        bool ok = true;
        for (int kb = 0; kb < nkb; ++kb) {
          if (!mbar_wait(smem_u32(&S.empty[stage]), phase ^ 1, abort, err, kErrGemmEmpty)) { ok = false; break; }
          const int seg = kb / kb_seg;
          const int kk = (kb - seg * kb_seg) * kBK;
          const int ap = seg == 2 ? 1 : 0, bp = seg == 1 ? 1 : 0;
          const uint32_t fb = smem_u32(&S.full[stage]);
          if (leader) mbar_expect_tx(fb, kPairStageBytes);
          tma_load_3d_pair(smem_u32(S.a[stage]), &ta, kk, mb * 256 + (int)rank * 128, ap, fb);
          tma_load_3d_pair(smem_u32(S.b[stage]), &tb, kk, nb * BN + (int)rank * 128, bp, fb);
          issued_mask |= 1u << stage;
          last_phase = (last_phase & ~(1u << stage)) | (phase << stage);
          if (++stage == kPairStages) { stage = 0; phase ^= 1; }
        }
        if (!ok) break;
      }
      if (*abort && leader) {
        const long long t0 = clock64();
        for (int s = 0; s < kPairStages; ++s) {
          if (!(issued_mask & (1u << s))) continue;
          while (!mbar_try(smem_u32(&S.full[s]), (last_phase >> s) & 1)) {
            if (clock64() - t0 > kWaitBudgetCycles) { atomicCAS(err, 0, kErrGemmDrain); break; }
          }
        }
      }
    }
  } else if (warp == 1) {
    if (lane == 0 && leader) {
      uint32_t stage = 0, phase = 0;
      int local = 0;
      for (int t = cid; t < tiles; t += ncl, ++local) {
        const int acc = local & 1;
        const uint32_t accph = (local >> 1) & 1;
        if (!mbar_wait(smem_u32(&S.acce[acc]), accph ^ 1, abort, err, kErrGemmAccEmpty)) break;
        tc_fence_after();
        const uint32_t d = tmem + acc * BN;
        bool ok = true;
        for (int kb = 0; kb < nkb; ++kb) {
          if (!mbar_wait(smem_u32(&S.full[stage]), phase, abort, err, kErrGemmFull)) { ok = false; break; }
          tc_fence_after();
          const uint32_t a0 = smem_u32(S.a[stage]), b0 = smem_u32(S.b[stage]);
#pragma unroll
          for (int k = 0; k < kBK / 16; ++k)
            umma_bf16_pair(d, sdesc_k128(a0 + k * 32), sdesc_k128(b0 + k * 32), kIdesc, (kb | k) != 0 ? 1u : 0u);
          umma_commit_pair(smem_u32(&S.empty[stage]), mapa_shared(smem_u32(&S.empty[stage]), 1));
          if (++stage == kPairStages) { stage = 0; phase ^= 1; }
        }
        if (!ok) break;
        umma_commit_pair(smem_u32(&S.accf[acc]), mapa_shared(smem_u32(&S.accf[acc]), 1));
      }
      // every earlier commit has landed in both CTAs once this one has
      umma_commit_pair(smem_u32(&S.drain), mapa_shared(smem_u32(&S.drain), 1));
    }
    if (lane == 0) {
      const long long t0 = clock64();
      while (!mbar_try(smem_u32(&S.drain), 0)) {
        if (clock64() - t0 > kWaitBudgetCycles) { atomicCAS(err, 0, kErrGemmDrain); break; }
      }
    }
  } else {
    const int q = warp & 3;
    Stager stager{S.stg[q], 0};
    const uint32_t acce_leader0 = mapa_shared(smem_u32(&S.acce[0]), 0);
    const uint32_t acce_leader1 = mapa_shared(smem_u32(&S.acce[1]), 0);
    int local = 0;
    for (int t = cid; t < tiles; t += ncl, ++local) {
      const int acc = local & 1;
      const uint32_t accph = (local >> 1) & 1;
      const int mb = t / num_n, nb = t - (t / num_n) * num_n;
      const int row0 = mb * 256 + (int)rank * 128 + q * 32;
      if (!mbar_wait(smem_u32(&S.accf[acc]), accph, abort, err, kErrGemmAccFull)) break;
      tc_fence_after();
      const uint32_t tbase = tmem + acc * BN + (static_cast<uint32_t>(q * 32) << 16);
      epilogue_tile<BN, EPI>([&](int off, float (&v)[32]) { tmem_ld32(tbase + off, v); }, row0, lane, nb, sh, ep,
                             &tc, stager);
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive_cluster(acc ? acce_leader1 : acce_leader0);
    }
    stg_drain(lane);
  }

  tc_fence_before();
  __syncwarp();
  cluster_sync_all();  // no CTA leaves while its peer may still signal or read its shared memory
  if (warp == 1) {
    __syncwarp();
    tc_fence_after();
    tmem_dealloc_pair(tmem, 2 * BN);
  }
}

typedef CUresult (*EncodeTiledFn)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*, const cuuint64_t*,
                                  const cuuint64_t*, const cuuint32_t*, const cuuint32_t*, CUtensorMapInterleave,
                                  CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

EncodeTiledFn encode_fn() {
  static EncodeTiledFn fn = nullptr;
  if (!fn) {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<EncodeTiledFn>(p);
  }
  return fn;
}

template <int BN, int EPI>
cudaError_t prepare_one() {
  cudaError_t e = cudaFuncSetAttribute(gemm_tc_kernel<BN, EPI, false>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                       (int)gemm_smem_bytes<BN>());
  if (e != cudaSuccess) return e;
  return cudaFuncSetAttribute(gemm_tc_kernel<BN, EPI, true>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                              (int)gemm_smem_bytes<BN>());
}

template <int BN, int EPI>
cudaError_t launch_one(const CUtensorMap& ta, const CUtensorMap& tb, const CUtensorMap& tc, const GemmShape& sh,
                       const GemmEpi& ep, int* err, int grid_ctas, cudaStream_t st) {
  constexpr size_t smem = gemm_smem_bytes<BN>();
  const int work = ((sh.M + kBM - 1) / kBM) * ((sh.N + BN - 1) / BN) * (sh.splits > 1 ? sh.splits : 1);
  const int grid = work < grid_ctas ? work : grid_ctas;
  if (grid <= 0) return cudaSuccess;
  if (sh.splits > 1) {
    CUtensorMap tp;  // the workspace [splits][M][N] fp32, the target of the slices' partial tiles
    if (!make_output_map(&tp, sh.ws, true, (uint64_t)sh.N, (uint64_t)sh.M, (uint64_t)sh.splits))
      return cudaErrorInvalidValue;
    cudaError_t e =
        launch_pdl(gemm_tc_kernel<BN, EPI, true>, dim3(grid), dim3(kThreads), smem, st, ta, tb, tp, sh, ep, err);
    if (e != cudaSuccess) return e;
    if constexpr (EPI == EPI_RESID) {
      if (ep.ln_w) {  // the following LayerNorm in the same pass over the rows
        const dim3 g((unsigned)((sh.M + 7) / 8));
        switch (sh.N / 128) {
          case 2: return launch_pdl(splitk_reduce_ln_kernel<2>, g, dim3(256), 0, st, sh, ep);
          case 4: return launch_pdl(splitk_reduce_ln_kernel<4>, g, dim3(256), 0, st, sh, ep);
          case 6: return launch_pdl(splitk_reduce_ln_kernel<6>, g, dim3(256), 0, st, sh, ep);
          case 8: return launch_pdl(splitk_reduce_ln_kernel<8>, g, dim3(256), 0, st, sh, ep);
          default: return cudaErrorInvalidValue;
        }
      }
    }
    const int ncols = EPI == EPI_GEGLU ? ep.geglu_I : sh.N;
    const long long threads = (long long)sh.M * (ncols / 64) * 8;
    return launch_pdl(splitk_reduce_kernel<EPI>, dim3((unsigned)((threads + 255) / 256)), dim3(256), 0, st, sh, ep);
  }
  return launch_pdl(gemm_tc_kernel<BN, EPI, false>, dim3(grid), dim3(kThreads), smem, st, ta, tb, tc, sh, ep, err);
}

template <int BN>
cudaError_t launch_bn(const CUtensorMap& ta, const CUtensorMap& tb, const CUtensorMap& tc, const GemmShape& sh,
                      const GemmEpi& ep, int* err, int grid_ctas, cudaStream_t st) {
  switch (ep.kind) {
    case EPI_STORE: return launch_one<BN, EPI_STORE>(ta, tb, tc, sh, ep, err, grid_ctas, st);
    case EPI_ROPE: return launch_one<BN, EPI_ROPE>(ta, tb, tc, sh, ep, err, grid_ctas, st);
    case EPI_GEGLU: return launch_one<BN, EPI_GEGLU>(ta, tb, tc, sh, ep, err, grid_ctas, st);
    case EPI_RESID: return launch_one<BN, EPI_RESID>(ta, tb, tc, sh, ep, err, grid_ctas, st);
  }
  return cudaErrorInvalidValue;
}

constexpr int kMaxDevices = 64;
int g_pair_clusters[kMaxDevices];  // co-resident CTA pairs per device (0: not measured yet)

template <int EPI>
cudaError_t prepare_pair(int* clusters) {
  cudaError_t e = cudaFuncSetAttribute(gemm_tc_pair_kernel<EPI>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                       (int)gemm_pair_smem_bytes());
  if (e != cudaSuccess) return e;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(2, 1, 1);
  cfg.blockDim = dim3(kThreads, 1, 1);
  cfg.dynamicSmemBytes = gemm_pair_smem_bytes();
  int n = 0;
  e = cudaOccupancyMaxActiveClusters(&n, gemm_tc_pair_kernel<EPI>, &cfg);
  if (e != cudaSuccess) return e;
  if (*clusters == 0 || n < *clusters) *clusters = n;
  return cudaSuccess;
}

template <int EPI>
cudaError_t launch_pair(const CUtensorMap& ta, const CUtensorMap& tb, const CUtensorMap& tc, const GemmShape& sh,
                        const GemmEpi& ep, int* err, int clusters, cudaStream_t st) {
  const int tiles = ((sh.M + 255) / 256) * ((sh.N + 255) / 256);
  const int ncl = tiles < clusters ? tiles : clusters;
  if (ncl <= 0) return cudaSuccess;
  return launch_pdl(gemm_tc_pair_kernel<EPI>, dim3(2 * ncl), dim3(kThreads), gemm_pair_smem_bytes(), st, ta, tb, tc, sh,
                    ep, err);
}

}  // namespace

int gemm_pair_clusters() {
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= kMaxDevices) return 0;
  return g_pair_clusters[dev];
}

bool make_operand_map(CUtensorMap* map, const void* base, uint64_t K, uint64_t rows, uint64_t planes,
                      uint32_t box_rows) {
  EncodeTiledFn fn = encode_fn();
  if (!fn) return false;
  if ((K * 2) % 16 != 0 || (reinterpret_cast<uintptr_t>(base) & 15) != 0 || box_rows > 256) return false;
  cuuint64_t dims[3] = {K, rows, planes};
  cuuint64_t strides[2] = {K * 2, K * 2 * rows};
  cuuint32_t box[3] = {static_cast<cuuint32_t>(kBK), box_rows, 1};
  cuuint32_t es[3] = {1, 1, 1};
  CUresult r = fn(map, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 3, const_cast<void*>(base), dims, strides, box, es,
                  CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                  CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  return r == CUDA_SUCCESS;
}

bool make_output_map(CUtensorMap* map, const void* base, bool f32, uint64_t ld, uint64_t rows, uint64_t planes) {
  EncodeTiledFn fn = encode_fn();
  if (!fn) return false;
  const uint64_t es = f32 ? 4 : 2;
  if ((ld * es) % 16 != 0 || (reinterpret_cast<uintptr_t>(base) & 15) != 0) return false;
  cuuint64_t dims[3] = {ld, rows, planes};
  cuuint64_t strides[2] = {ld * es, ld * es * rows};
  cuuint32_t box[3] = {static_cast<cuuint32_t>(128 / es), 32, 1};  // 128-byte rows, 32 rows
  cuuint32_t estr[3] = {1, 1, 1};
  CUresult r = fn(map, f32 ? CU_TENSOR_MAP_DATA_TYPE_FLOAT32 : CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 3,
                  const_cast<void*>(base), dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
                  CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  return r == CUDA_SUCCESS;
}

cudaError_t gemm_prepare_device() {
  cudaError_t e = cudaSuccess;
  for (cudaError_t r : {prepare_one<128, EPI_STORE>(), prepare_one<128, EPI_ROPE>(), prepare_one<128, EPI_GEGLU>(),
                        prepare_one<128, EPI_RESID>(), prepare_one<256, EPI_STORE>(), prepare_one<256, EPI_ROPE>(),
                        prepare_one<256, EPI_GEGLU>(), prepare_one<256, EPI_RESID>()})
    if (r != cudaSuccess) e = r;
  int dev = 0;
  if (cudaGetDevice(&dev) == cudaSuccess && dev >= 0 && dev < kMaxDevices) {
    int clusters = 0;
    for (cudaError_t r : {prepare_pair<EPI_STORE>(&clusters), prepare_pair<EPI_ROPE>(&clusters),
                          prepare_pair<EPI_GEGLU>(&clusters), prepare_pair<EPI_RESID>(&clusters)})
      if (r != cudaSuccess) e = r;
    g_pair_clusters[dev] = clusters;
  }
  return e;
}

cudaError_t gemm_launch(const CUtensorMap& ta, const CUtensorMap& tb, const CUtensorMap& tc, int bn,
                        const GemmShape& sh, const GemmEpi& ep_in, int* err, int grid_ctas, cudaStream_t st) {
  if (sh.M <= 0) return cudaSuccess;
  GemmEpi ep = ep_in;
  ep.err = err;
  if (sh.splits > 1 && (bn == kGemmPair || !sh.ws || !sh.dst || sh.splits > kMaxSplits ||
                        (reinterpret_cast<uintptr_t>(sh.ws) & 15) != 0 || (reinterpret_cast<uintptr_t>(sh.dst) & 15) != 0 ||
                        (ep.out_mode == OUT_BF16X2 && ep.kind != EPI_RESID && sh.dst_plane % 4 != 0)))
    return cudaErrorInvalidValue;
  if (sh.N % 64 != 0 || sh.K % 8 != 0 || (sh.nseg != 1 && sh.nseg != 3)) return cudaErrorInvalidValue;
  // every K slice must own at least one K block: a slice without one would store an accumulator it
  // never wrote as its partial
  if (sh.splits > 1 && sh.splits > ((sh.K + 63) / 64) * sh.nseg) return cudaErrorInvalidValue;
  if (ep.ln_w && (ep.kind != EPI_RESID || sh.splits < 2 || sh.N % 256 != 0 || sh.N > 1024 || !ep.ln_out ||
                  (ep.ln_planes != 1 && ep.ln_planes != 2) ||
                  ((reinterpret_cast<uintptr_t>(ep.ln_w) | reinterpret_cast<uintptr_t>(ep.ln_out)) & 15) != 0 ||
                  (ep.ln_planes == 2 && ep.ln_plane % 8 != 0)))
    return cudaErrorInvalidValue;
  if (ep.kind == EPI_GEGLU && (ep.geglu_I % 64 != 0 || sh.N != 2 * ep.geglu_I)) return cudaErrorInvalidValue;
  if (ep.kind == EPI_ROPE && (ep.rope_cols % 64 != 0 || !ep.pos || !ep.cos_t || !ep.sin_t))
    return cudaErrorInvalidValue;
  if (bn == 256) return launch_bn<256>(ta, tb, tc, sh, ep, err, grid_ctas, st);
  if (bn == 128) return launch_bn<128>(ta, tb, tc, sh, ep, err, grid_ctas, st);
  if (bn == kGemmPair) {
    const int clusters = std::min(gemm_pair_clusters(), grid_ctas / 2);
    if (clusters <= 0) return cudaErrorInvalidConfiguration;
    switch (ep.kind) {
      case EPI_STORE: return launch_pair<EPI_STORE>(ta, tb, tc, sh, ep, err, clusters, st);
      case EPI_ROPE: return launch_pair<EPI_ROPE>(ta, tb, tc, sh, ep, err, clusters, st);
      case EPI_GEGLU: return launch_pair<EPI_GEGLU>(ta, tb, tc, sh, ep, err, clusters, st);
      case EPI_RESID: return launch_pair<EPI_RESID>(ta, tb, tc, sh, ep, err, clusters, st);
    }
  }
  return cudaErrorInvalidValue;
}

}  // namespace laya
