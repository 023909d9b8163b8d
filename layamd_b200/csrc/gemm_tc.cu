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
  if (act == ACT_GELU) return gelu_erf(v);
  return v;
}

// Stores 32 consecutive values of one row. off is the element offset of the first value.
__device__ __forceinline__ void store_row32(const float (&v)[32], const GemmEpi& ep, long long off) {
  if (ep.out_mode == OUT_F32) {
    float4* p = reinterpret_cast<float4*>(static_cast<float*>(ep.out) + off);
#pragma unroll
    for (int i = 0; i < 8; ++i) p[i] = make_float4(v[4 * i], v[4 * i + 1], v[4 * i + 2], v[4 * i + 3]);
    return;
  }
  bf16* base = static_cast<bf16*>(ep.out);
  uint4* hi = reinterpret_cast<uint4*>(base + off);
  uint32_t h[16];
#pragma unroll
  for (int i = 0; i < 16; ++i) h[i] = pack_bf16x2(v[2 * i], v[2 * i + 1]);
#pragma unroll
  for (int i = 0; i < 4; ++i) hi[i] = make_uint4(h[4 * i], h[4 * i + 1], h[4 * i + 2], h[4 * i + 3]);
  if (ep.out_mode == OUT_BF16X2) {
    uint4* lo = reinterpret_cast<uint4*>(base + ep.plane + off);
    uint32_t l[16];
#pragma unroll
    for (int i = 0; i < 16; ++i) {
      __nv_bfloat162 hv = *reinterpret_cast<__nv_bfloat162*>(&h[i]);
      float2 hf = __bfloat1622float2(hv);
      l[i] = pack_bf16x2(v[2 * i] - hf.x, v[2 * i + 1] - hf.y);
    }
#pragma unroll
    for (int i = 0; i < 4; ++i) lo[i] = make_uint4(l[4 * i], l[4 * i + 1], l[4 * i + 2], l[4 * i + 3]);
  }
}

// Epilogue of one tile for one thread (one output row). Every tcgen05.ld is executed by the whole
// warp; only the stores depend on the row being valid.
template <int BN, int EPI>
__device__ __forceinline__ void epilogue_tile(uint32_t tbase, int row, int nb, const GemmShape& sh,
                                              const GemmEpi& ep) {
  const bool valid = row < sh.M;
  if constexpr (EPI == EPI_GEGLU) {
    // B rows are interleaved in groups of 64: [64 input rows, their 64 gate rows] per 128 columns.
    for (int s = 0; s < BN; s += 128) {
      const int ocol = nb * (BN / 2) + s / 2;  // first output column of this 128-column group
      if (ocol >= ep.geglu_I) break;
      for (int c = 0; c < 64; c += 32) {
        float xin[32], gate[32];
        __syncwarp();
        tmem_ld32(tbase + s + c, xin);
        tmem_ld32(tbase + s + 64 + c, gate);
        if (valid) {
#pragma unroll
          for (int i = 0; i < 32; ++i) xin[i] = gelu_erf(xin[i]) * gate[i];
          store_row32(xin, ep, (long long)row * ep.ld + ocol + c);
        }
      }
    }
  } else if constexpr (EPI == EPI_ROPE) {
    for (int h = 0; h < BN; h += 64) {
      const int col = nb * BN + h;
      if (col >= sh.N) break;
      float x1[32], x2[32];
      __syncwarp();
      tmem_ld32(tbase + h, x1);
      tmem_ld32(tbase + h + 32, x2);
      if (valid) {
        if (ep.bias) {
#pragma unroll
          for (int i = 0; i < 32; ++i) { x1[i] += ep.bias[col + i]; x2[i] += ep.bias[col + 32 + i]; }
        }
        if (col < ep.rope_cols) {
          const int p = ep.pos[row];
          const float* ct = ep.cos_t + (size_t)p * 32;
          const float* st = ep.sin_t + (size_t)p * 32;
#pragma unroll
          for (int i = 0; i < 32; ++i) {
            const float c = ct[i], s = st[i];
            const float a = x1[i], b = x2[i];
            x1[i] = a * c - b * s;
            x2[i] = b * c + a * s;
          }
        }
        const long long off = (long long)row * ep.ld + col;
        store_row32(x1, ep, off);
        store_row32(x2, ep, off + 32);
      }
    }
  } else {
    for (int c = 0; c < BN; c += 32) {
      const int col = nb * BN + c;
      if (col >= sh.N) break;
      float v[32];
      __syncwarp();
      tmem_ld32(tbase + c, v);
      if (!valid) continue;
      if (ep.bias) {
#pragma unroll
        for (int i = 0; i < 32; ++i) v[i] += ep.bias[col + i];
      }
      if constexpr (EPI == EPI_RESID) {
        float4* x = reinterpret_cast<float4*>(ep.resid + (long long)row * ep.ld + col);
#pragma unroll
        for (int i = 0; i < 8; ++i) {
          float4 r = x[i];
          r.x += v[4 * i]; r.y += v[4 * i + 1]; r.z += v[4 * i + 2]; r.w += v[4 * i + 3];
          x[i] = r;
        }
      } else {
        if (ep.act != ACT_NONE) {
#pragma unroll
          for (int i = 0; i < 32; ++i) v[i] = apply_act(v[i], ep.act);
        }
        store_row32(v, ep, (long long)row * ep.ld + col);
      }
    }
  }
}

template <int BN, int EPI>
__global__ void __launch_bounds__(kThreads, 1)
    gemm_tc_kernel(const __grid_constant__ CUtensorMap ta, const __grid_constant__ CUtensorMap tb,
                   const GemmShape sh, const GemmEpi ep, int* err) {
  constexpr int STAGES = StagesFor<BN>::value;
  constexpr uint32_t kIdesc = idesc_bf16(kBM, BN);
  constexpr uint32_t kStageBytes = (kBM + BN) * kBK * 2;
  using Smem = GemmSmem<BN, STAGES>;
  extern __shared__ uint8_t smem_raw[];
  Smem& S = *reinterpret_cast<Smem*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int num_n = (sh.N + BN - 1) / BN;
  const int tiles = ((sh.M + kBM - 1) / kBM) * num_n;
  const int kb_seg = (sh.K + kBK - 1) / kBK;
  const int nkb = kb_seg * sh.nseg;

  if (threadIdx.x == 0) {
    for (int s = 0; s < STAGES; ++s) { mbar_init(smem_u32(&S.full[s]), 1); mbar_init(smem_u32(&S.empty[s]), 1); }
    for (int a = 0; a < 2; ++a) { mbar_init(smem_u32(&S.accf[a]), 1); mbar_init(smem_u32(&S.acce[a]), 4); }
    mbar_init(smem_u32(&S.drain), 1);
    S.abort = 0;
    fence_mbar_init();
  }
  if (warp == 0 && lane == 0) { tma_prefetch_desc(&ta); tma_prefetch_desc(&tb); }
  if (warp == 1) { tmem_alloc(smem_u32(&S.tmem), 2 * BN); tmem_relinquish(); }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = S.tmem;
  volatile int* abort = &S.abort;

  if (warp == 0) {
    if (lane == 0) {
      // ---------------- TMA producer
      uint32_t stage = 0, phase = 0;
      uint32_t issued_mask = 0, last_phase = 0;  // for the abort drain
      for (int t = blockIdx.x; t < tiles; t += gridDim.x) {
        const int mb = t / num_n, nb = t - (t / num_n) * num_n;
        bool ok = true;
        for (int kb = 0; kb < nkb; ++kb) {
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
      for (int t = blockIdx.x; t < tiles; t += gridDim.x, ++local) {
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
            umma_bf16(d, sdesc_k128(a0 + k * 32), sdesc_k128(b0 + k * 32), kIdesc, (kb | k) != 0 ? 1u : 0u);
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
    int local = 0;
    for (int t = blockIdx.x; t < tiles; t += gridDim.x, ++local) {
      const int acc = local & 1;
      const uint32_t accph = (local >> 1) & 1;
      if (!mbar_wait(smem_u32(&S.accf[acc]), accph, abort, err, kErrGemmAccFull)) break;
      tc_fence_after();
      const int mb = t / num_n, nb = t - (t / num_n) * num_n;
      const int row = mb * kBM + q * 32 + lane;
      const uint32_t tbase = tmem + acc * BN + (static_cast<uint32_t>(q * 32) << 16);
      epilogue_tile<BN, EPI>(tbase, row, nb, sh, ep);
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(smem_u32(&S.acce[acc]));
    }
  }

  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    __syncwarp();
    tc_fence_after();
    tmem_dealloc(tmem, 2 * BN);
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
  return cudaFuncSetAttribute(gemm_tc_kernel<BN, EPI>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                              (int)gemm_smem_bytes<BN>());
}

template <int BN, int EPI>
cudaError_t launch_one(const CUtensorMap& ta, const CUtensorMap& tb, const GemmShape& sh, const GemmEpi& ep,
                       int* err, int grid_ctas, cudaStream_t st) {
  constexpr size_t smem = gemm_smem_bytes<BN>();
  const int tiles = ((sh.M + kBM - 1) / kBM) * ((sh.N + BN - 1) / BN);
  const int grid = tiles < grid_ctas ? tiles : grid_ctas;
  if (grid <= 0) return cudaSuccess;
  gemm_tc_kernel<BN, EPI><<<grid, kThreads, smem, st>>>(ta, tb, sh, ep, err);
  return cudaGetLastError();
}

template <int BN>
cudaError_t launch_bn(const CUtensorMap& ta, const CUtensorMap& tb, const GemmShape& sh, const GemmEpi& ep,
                      int* err, int grid_ctas, cudaStream_t st) {
  switch (ep.kind) {
    case EPI_STORE: return launch_one<BN, EPI_STORE>(ta, tb, sh, ep, err, grid_ctas, st);
    case EPI_ROPE: return launch_one<BN, EPI_ROPE>(ta, tb, sh, ep, err, grid_ctas, st);
    case EPI_GEGLU: return launch_one<BN, EPI_GEGLU>(ta, tb, sh, ep, err, grid_ctas, st);
    case EPI_RESID: return launch_one<BN, EPI_RESID>(ta, tb, sh, ep, err, grid_ctas, st);
  }
  return cudaErrorInvalidValue;
}

}  // namespace

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

cudaError_t gemm_prepare_device() {
  cudaError_t e = cudaSuccess;
  for (cudaError_t r : {prepare_one<128, EPI_STORE>(), prepare_one<128, EPI_ROPE>(), prepare_one<128, EPI_GEGLU>(),
                        prepare_one<128, EPI_RESID>(), prepare_one<256, EPI_STORE>(), prepare_one<256, EPI_ROPE>(),
                        prepare_one<256, EPI_GEGLU>(), prepare_one<256, EPI_RESID>()})
    if (r != cudaSuccess) e = r;
  return e;
}

cudaError_t gemm_launch(const CUtensorMap& ta, const CUtensorMap& tb, int bn, const GemmShape& sh,
                        const GemmEpi& ep, int* err, int grid_ctas, cudaStream_t st) {
  if (sh.M <= 0) return cudaSuccess;
  if (sh.N % 32 != 0 || sh.K % 8 != 0 || (sh.nseg != 1 && sh.nseg != 3)) return cudaErrorInvalidValue;
  if (ep.kind == EPI_GEGLU && (ep.geglu_I % 64 != 0 || sh.N != 2 * ep.geglu_I)) return cudaErrorInvalidValue;
  if (ep.kind == EPI_ROPE && (ep.rope_cols % 64 != 0 || !ep.pos || !ep.cos_t || !ep.sin_t))
    return cudaErrorInvalidValue;
  if (ep.kind == EPI_RESID ? ep.resid == nullptr : ep.out == nullptr) return cudaErrorInvalidValue;
  if (bn == 256) return launch_bn<256>(ta, tb, sh, ep, err, grid_ctas, st);
  if (bn == 128) return launch_bn<128>(ta, tb, sh, ep, err, grid_ctas, st);
  return cudaErrorInvalidValue;
}

}  // namespace laya
