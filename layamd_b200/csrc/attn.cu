// Fused attention over packed variable-length sequences, head dim 64. Replaces the reference's
// RDNA3 WMMA flash kernels k_flash_wmma / k_flash_wmma_gather (src/kernels.hip:154-242, 351-381).
//
// Layout: Q/K/V are read in place from the packed qkv rows [T, 3D] (q | k | v, heads of 64); output
// rows [rows, D] (heads merged). A work item is 64 query rows of one sequence; the grid is
// (items, heads). Keys come only from the item's own sequence (its first packed row and length), so
// no row attends across a sequence boundary and no padding rows are needed. Sliding-window layers
// visit only the key blocks inside |q - k| <= window (window = local_attention / 2, inclusive, the
// bidirectional band of transformers' sliding_window_bidirectional_overlay).
//
//   attn_bf16_kernel  bf16 Q/K/V, fp32 online softmax, bf16 tensor-core MMA (mma.sync m16n8k16):
//                     S = Q K^T and O += P V per 64-key block, cp.async double-buffered K/V tiles in
//                     XOR-swizzled shared memory, ldmatrix fragment loads.
//   attn_f32_kernel   fp32 Q/K/V and fp32 arithmetic throughout (one thread per query); the
//                     attention of the fp32-parity mode. Writes hi/lo bf16 planes for the next GEMM.
// Gathered mode (the last head layer): the queries of an item are an explicit list of packed rows
// (a question's option markers and its CLS row) written to explicit output rows, over full
// attention of that question's sequence.
#include "common.cuh"
#include "kernels.h"

namespace laya {
namespace {

__device__ __forceinline__ uint32_t swz(int row, int chunk) {  // byte offset in a [64][64] bf16 tile
  return static_cast<uint32_t>(row * 128 + ((chunk ^ (row & 7)) << 4));
}
__device__ __forceinline__ void cp_async16(uint32_t dst, const void* src, bool valid) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;" ::"r"(dst), "l"(src), "r"(valid ? 16 : 0)
               : "memory");
}
__device__ __forceinline__ void cp_async_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
template <int N>
__device__ __forceinline__ void cp_async_wait() {
  asm volatile("cp.async.wait_group %0;" ::"n"(N) : "memory");
}
__device__ __forceinline__ void ldsm_x4(uint32_t addr, uint32_t& r0, uint32_t& r1, uint32_t& r2, uint32_t& r3) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0,%1,%2,%3}, [%4];"
               : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3)
               : "r"(addr));
}
__device__ __forceinline__ void ldsm_x4_t(uint32_t addr, uint32_t& r0, uint32_t& r1, uint32_t& r2, uint32_t& r3) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.trans.shared.b16 {%0,%1,%2,%3}, [%4];"
               : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3)
               : "r"(addr));
}
__device__ __forceinline__ void mma_bf16_16816(float (&d)[4], const uint32_t (&a)[4], uint32_t b0, uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
      "{%0,%1,%2,%3};"
      : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
      : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
}

template <bool GATHER>
__global__ void __launch_bounds__(128) attn_bf16_kernel(const AttnArgs a) {
  __shared__ __align__(128) uint8_t sQ[64 * 128];
  __shared__ __align__(128) uint8_t sK[2][64 * 128];
  __shared__ __align__(128) uint8_t sV[2][64 * 128];
  __shared__ int s_src[64], s_dst[64];

  pdl_trigger();
  pdl_wait();
  const AttnItem it = a.items[blockIdx.x];
  if (it.seq < 0) return;
  if (!LAYA_IN_BOUNDS(a.n_seq <= 0 || it.seq < a.n_seq, a.err, kErrBoundsAttn)) return;
  const int h = blockIdx.y;
  const int D = a.H * 64;
  const long long ld = 3LL * D;
  const int base = a.soff[it.seq], len = a.slen[it.seq];
  if (!LAYA_IN_BOUNDS(a.rows <= 0 || (base >= 0 && len > 0 && base + len <= a.rows &&
                                      (GATHER ? (it.nq >= 1 && it.nq <= 64) : (it.q0 >= 0 && it.q0 < len))),
                      a.err, kErrBoundsAttn))
    return;
  const bf16* qkv = static_cast<const bf16*>(a.qkv);
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;

  int nq;
  if (GATHER) {
    nq = it.nq;
    if (tid < 64) {
      s_src[tid] = tid < nq ? a.gsrc[it.goff + tid] : base;
      s_dst[tid] = tid < nq ? a.gdst[it.goff + tid] : -1;
      if (!LAYA_IN_BOUNDS(a.rows <= 0 || (s_src[tid] >= base && s_src[tid] < base + len &&
                                          s_dst[tid] < (a.rows_out > 0 ? a.rows_out : a.rows)),
                          a.err, kErrBoundsGather)) {
        s_src[tid] = base;  // the query reads its sequence's first row and its output is dropped
        s_dst[tid] = -1;
      }
    }
    __syncthreads();
  } else {
    nq = min(64, len - it.q0);
  }
  int lo = 0, hi = len;
  if (!GATHER && a.window > 0) {
    lo = max(0, it.q0 - a.window);
    hi = min(len, it.q0 + 64 + a.window);
  }
  lo &= ~63;
  const int nblk = (hi - lo + 63) >> 6;

  const uint32_t sq = smem_u32(sQ);
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const int id = tid + 128 * i, r = id >> 3, c = id & 7;
    const bool v = r < nq;
    const long long prow = GATHER ? (long long)s_src[r] : (long long)base + it.q0 + (v ? r : 0);
    cp_async16(sq + swz(r, c), qkv + prow * ld + h * 64 + c * 8, v);
  }
  auto load_kv = [&](int blk, int buf) {
    const int k0 = lo + blk * 64;
    const uint32_t sk = smem_u32(sK[buf]), sv = smem_u32(sV[buf]);
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const int id = tid + 128 * i, r = id >> 3, c = id & 7;
      const bool v = k0 + r < hi;
      const bf16* src = qkv + ((long long)base + (v ? k0 + r : 0)) * ld + h * 64 + c * 8;
      cp_async16(sk + swz(r, c), src + D, v);
      cp_async16(sv + swz(r, c), src + 2 * D, v);
    }
  };
  load_kv(0, 0);
  cp_async_commit();

  uint32_t qf[4][4];
  float o[8][4];
#pragma unroll
  for (int j = 0; j < 8; ++j) o[j][0] = o[j][1] = o[j][2] = o[j][3] = 0.f;
  float mrow[2] = {-INFINITY, -INFINITY}, lrow[2] = {0.f, 0.f};
  const float sl2 = a.scale * 1.4426950408889634f;  // softmax in base 2
  const int qbase = (GATHER ? 0 : it.q0) + warp * 16 + (lane >> 2);

  for (int blk = 0; blk < nblk; ++blk) {
    const int buf = blk & 1;
    if (blk + 1 < nblk) {
      load_kv(blk + 1, buf ^ 1);
      cp_async_commit();
      cp_async_wait<1>();
    } else {
      cp_async_wait<0>();
    }
    __syncthreads();
    if (blk == 0) {
#pragma unroll
      for (int kk = 0; kk < 4; ++kk) {
        const int m = lane >> 3, r = warp * 16 + (m & 1) * 8 + (lane & 7), c = kk * 2 + (m >> 1);
        ldsm_x4(sq + swz(r, c), qf[kk][0], qf[kk][1], qf[kk][2], qf[kk][3]);
      }
    }
    const uint32_t sk = smem_u32(sK[buf]), sv = smem_u32(sV[buf]);
    float s[8][4];
#pragma unroll
    for (int j = 0; j < 8; ++j) s[j][0] = s[j][1] = s[j][2] = s[j][3] = 0.f;
#pragma unroll
    for (int kk = 0; kk < 4; ++kk) {
#pragma unroll
      for (int j = 0; j < 8; j += 2) {
        const int m = lane >> 3, r = j * 8 + (m >> 1) * 8 + (lane & 7), c = kk * 2 + (m & 1);
        uint32_t b0, b1, b2, b3;
        ldsm_x4(sk + swz(r, c), b0, b1, b2, b3);
        mma_bf16_16816(s[j], qf[kk], b0, b1);
        mma_bf16_16816(s[j + 1], qf[kk], b2, b3);
      }
    }
    const int k0 = lo + blk * 64;
    float mx[2] = {mrow[0], mrow[1]};
#pragma unroll
    for (int j = 0; j < 8; ++j) {
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        const int rh = e >> 1;
        const int kpos = k0 + j * 8 + (lane & 3) * 2 + (e & 1);
        const int qpos = qbase + rh * 8;
        const bool ok = kpos < len && (GATHER || a.window == 0 || abs(qpos - kpos) <= a.window);
        s[j][e] = ok ? s[j][e] * sl2 : -INFINITY;
        mx[rh] = fmaxf(mx[rh], s[j][e]);
      }
    }
    float msub[2], alpha[2];
#pragma unroll
    for (int rh = 0; rh < 2; ++rh) {
      mx[rh] = fmaxf(mx[rh], __shfl_xor_sync(0xffffffffu, mx[rh], 1));
      mx[rh] = fmaxf(mx[rh], __shfl_xor_sync(0xffffffffu, mx[rh], 2));
      msub[rh] = mx[rh] == -INFINITY ? 0.f : mx[rh];
      alpha[rh] = exp2f(mrow[rh] - msub[rh]);
      mrow[rh] = mx[rh];
      lrow[rh] *= alpha[rh];
    }
#pragma unroll
    for (int j = 0; j < 8; ++j) {
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        const int rh = e >> 1;
        const float p = exp2f(s[j][e] - msub[rh]);
        s[j][e] = p;
        lrow[rh] += p;
      }
      o[j][0] *= alpha[0];
      o[j][1] *= alpha[0];
      o[j][2] *= alpha[1];
      o[j][3] *= alpha[1];
    }
#pragma unroll
    for (int kk = 0; kk < 4; ++kk) {
      const uint32_t pa[4] = {pack_bf16x2(s[2 * kk][0], s[2 * kk][1]), pack_bf16x2(s[2 * kk][2], s[2 * kk][3]),
                              pack_bf16x2(s[2 * kk + 1][0], s[2 * kk + 1][1]),
                              pack_bf16x2(s[2 * kk + 1][2], s[2 * kk + 1][3])};
#pragma unroll
      for (int jd = 0; jd < 8; jd += 2) {
        const int m = lane >> 3, r = kk * 16 + (m & 1) * 8 + (lane & 7), c = jd + (m >> 1);
        uint32_t b0, b1, b2, b3;
        ldsm_x4_t(sv + swz(r, c), b0, b1, b2, b3);
        mma_bf16_16816(o[jd], pa, b0, b1);
        mma_bf16_16816(o[jd + 1], pa, b2, b3);
      }
    }
    __syncthreads();
  }

  float inv[2];
#pragma unroll
  for (int rh = 0; rh < 2; ++rh) {
    float l = lrow[rh];
    l += __shfl_xor_sync(0xffffffffu, l, 1);
    l += __shfl_xor_sync(0xffffffffu, l, 2);
    inv[rh] = l > 0.f ? 1.f / l : 0.f;
  }
  // Stage this warp's 16 output rows in its own rows of the Q tile, then store 16-byte chunks.
  __syncwarp();
  const int r0 = warp * 16 + (lane >> 2);
#pragma unroll
  for (int jd = 0; jd < 8; ++jd) {
    *reinterpret_cast<uint32_t*>(sQ + swz(r0, jd) + (lane & 3) * 4) = pack_bf16x2(o[jd][0] * inv[0], o[jd][1] * inv[0]);
    *reinterpret_cast<uint32_t*>(sQ + swz(r0 + 8, jd) + (lane & 3) * 4) =
        pack_bf16x2(o[jd][2] * inv[1], o[jd][3] * inv[1]);
  }
  __syncwarp();
  bf16* out = static_cast<bf16*>(a.out);
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const int id = lane + 32 * i, r = warp * 16 + (id >> 3), c = id & 7;
    if (r < nq && (!GATHER || s_dst[r] >= 0)) {  // s_dst < 0: dropped by a debug bounds check
      const long long dst = GATHER ? (long long)s_dst[r] : (long long)base + it.q0 + r;
      *reinterpret_cast<uint4*>(out + dst * D + h * 64 + c * 8) = *reinterpret_cast<const uint4*>(sQ + swz(r, c));
    }
  }
}

template <bool GATHER>
__global__ void __launch_bounds__(64) attn_f32_kernel(const AttnArgs a) {
  __shared__ __align__(16) float sK[32][64];
  __shared__ __align__(16) float sV[32][64];
  pdl_trigger();
  pdl_wait();
  const AttnItem it = a.items[blockIdx.x];
  if (it.seq < 0) return;
  if (!LAYA_IN_BOUNDS(a.n_seq <= 0 || it.seq < a.n_seq, a.err, kErrBoundsAttn)) return;
  const int h = blockIdx.y, D = a.H * 64, tid = threadIdx.x;
  const long long ld = 3LL * D;
  const int base = a.soff[it.seq], len = a.slen[it.seq];
  if (!LAYA_IN_BOUNDS(a.rows <= 0 || (base >= 0 && len > 0 && base + len <= a.rows &&
                                      (GATHER ? (it.nq >= 1 && it.nq <= 64) : (it.q0 >= 0 && it.q0 < len))),
                      a.err, kErrBoundsAttn))
    return;
  const float* qkv = static_cast<const float*>(a.qkv);
  const int nq = GATHER ? it.nq : min(64, len - it.q0);
  bool qv = tid < nq;
  if (GATHER && qv) {
    const int gs = a.gsrc[it.goff + tid], gd = a.gdst[it.goff + tid];
    if (!LAYA_IN_BOUNDS(a.rows <= 0 || (gs >= base && gs < base + len && gd >= 0 &&
                                        gd < (a.rows_out > 0 ? a.rows_out : a.rows)),
                        a.err, kErrBoundsGather))
      qv = false;
  }
  const long long qrow = GATHER ? (qv ? (long long)a.gsrc[it.goff + tid] : base)
                                : (long long)base + it.q0 + (qv ? tid : 0);
  const int qpos = GATHER ? 0 : it.q0 + tid;
  float q[64], o[64];
  {
    const float4* qp = reinterpret_cast<const float4*>(qkv + qrow * ld + h * 64);
#pragma unroll
    for (int i = 0; i < 16; ++i) {
      const float4 v = qp[i];
      q[4 * i] = v.x; q[4 * i + 1] = v.y; q[4 * i + 2] = v.z; q[4 * i + 3] = v.w;
    }
  }
#pragma unroll
  for (int d = 0; d < 64; ++d) o[d] = 0.f;
  int lo = 0, hi = len;
  if (!GATHER && a.window > 0) {
    lo = max(0, it.q0 - a.window);
    hi = min(len, it.q0 + 64 + a.window);
  }
  float m = -INFINITY, l = 0.f;
  for (int k0 = lo; k0 < hi; k0 += 32) {
    __syncthreads();
#pragma unroll
    for (int i = 0; i < 8; ++i) {
      const int id = tid + 64 * i, r = id >> 4, c = id & 15;
      const bool v = k0 + r < hi;
      const float* src = qkv + ((long long)base + (v ? k0 + r : 0)) * ld + h * 64 + c * 4;
      const float4 kz = v ? *reinterpret_cast<const float4*>(src + D) : make_float4(0.f, 0.f, 0.f, 0.f);
      const float4 vz = v ? *reinterpret_cast<const float4*>(src + 2 * D) : make_float4(0.f, 0.f, 0.f, 0.f);
      *reinterpret_cast<float4*>(&sK[r][c * 4]) = kz;
      *reinterpret_cast<float4*>(&sV[r][c * 4]) = vz;
    }
    __syncthreads();
    float s[32];
    float mx = m;
#pragma unroll
    for (int j = 0; j < 32; ++j) {
      const int kpos = k0 + j;
      float dot = 0.f;
#pragma unroll
      for (int d = 0; d < 64; ++d) dot = fmaf(q[d], sK[j][d], dot);
      const bool ok = kpos < hi && (GATHER || a.window == 0 || abs(qpos - kpos) <= a.window);
      s[j] = ok ? dot * a.scale : -INFINITY;
      mx = fmaxf(mx, s[j]);
    }
    const float msub = mx == -INFINITY ? 0.f : mx;
    const float alpha = expf(m - msub);
    m = mx;
    l *= alpha;
#pragma unroll
    for (int d = 0; d < 64; ++d) o[d] *= alpha;
#pragma unroll
    for (int j = 0; j < 32; ++j) {
      const float p = expf(s[j] - msub);
      l += p;
#pragma unroll
      for (int d = 0; d < 64; ++d) o[d] = fmaf(p, sV[j][d], o[d]);
    }
  }
  if (!qv) return;
  const float inv = l > 0.f ? 1.f / l : 0.f;
  const long long dst = GATHER ? (long long)a.gdst[it.goff + tid] : (long long)base + it.q0 + tid;
  bf16* out = static_cast<bf16*>(a.out) + dst * D + h * 64;
#pragma unroll
  for (int i = 0; i < 8; ++i) {
    uint32_t hw[4], lw[4];
#pragma unroll
    for (int e = 0; e < 4; ++e) {
      const float x0 = o[8 * i + 2 * e] * inv, x1 = o[8 * i + 2 * e + 1] * inv;
      hw[e] = pack_bf16x2(x0, x1);
      const float2 hf = __bfloat1622float2(*reinterpret_cast<__nv_bfloat162*>(&hw[e]));
      lw[e] = pack_bf16x2(x0 - hf.x, x1 - hf.y);
    }
    reinterpret_cast<uint4*>(out)[i] = make_uint4(hw[0], hw[1], hw[2], hw[3]);
    if (a.out_planes == 2) reinterpret_cast<uint4*>(out + a.out_plane)[i] = make_uint4(lw[0], lw[1], lw[2], lw[3]);
  }
}

}  // namespace

cudaError_t attn_bf16_launch(const AttnArgs& a, cudaStream_t st) {
  if (a.n_items <= 0) return cudaSuccess;
  dim3 grid(a.n_items, a.H);
  if (a.gathered) return launch_pdl(attn_bf16_kernel<true>, grid, dim3(128), 0, st, a);
  return launch_pdl(attn_bf16_kernel<false>, grid, dim3(128), 0, st, a);
}

cudaError_t attn_f32_launch(const AttnArgs& a, cudaStream_t st) {
  if (a.n_items <= 0) return cudaSuccess;
  dim3 grid(a.n_items, a.H);
  if (a.gathered) return launch_pdl(attn_f32_kernel<true>, grid, dim3(64), 0, st, a);
  return launch_pdl(attn_f32_kernel<false>, grid, dim3(64), 0, st, a);
}

}  // namespace laya
