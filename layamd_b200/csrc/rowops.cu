// Row kernels of the Laya B200 engine: the LayerNorm family and the decision-head outputs.
//
// ln_kernel replaces the reference's k_ln (embedding gather + LN, src/kernels.hip:35-64), the LN half
// of k_res_ln (src/kernels.hip:105-137; the residual add itself is fused into the GEMM epilogue here)
// and k_gather (src/kernels.hip:267-271). One warp owns one row of D = 128*NV fp32 values held in
// registers as float4 (16-byte coalesced loads and stores); mean and variance are two-pass in fp32 and
// the normaliser is 1/sqrt(var + eps), as torch.nn.LayerNorm computes it. Optional outputs: the fp32
// source row (gather), the normalised fp32 row (may overwrite the source in place: the final norm +
// type embedding is written back into the residual stream), and bf16 planes of either the normalised
// row or a second LayerNorm of it (the next layer's input, hi/lo planes in fp32-parity mode).
//
// head_out_kernel replaces k_bias_to_float + k_act_head (src/kernels.hip:273-307): per question, the
// scorer's final Linear(d, 1) at each option marker, softmax features of those logits and the act
// head MLP on the question's CLS row.
#include "common.cuh"
#include "kernels.h"

namespace laya {
namespace {

template <int NV>
__global__ void __launch_bounds__(256) ln_kernel(const LnArgs a) {
  pdl_trigger();
  pdl_wait();
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  // Rows in reverse block order: the first blocks read the rows that the residual GEMM before this
  // kernel wrote last, while they are still in L2 (LayerNorm stage of the C2 pass 3.25 -> 3.16 ms).
  const int row = (gridDim.x - 1 - blockIdx.x) * 8 + warp;
  if (row >= a.rows) return;
  const int D = a.D;
  const long long src_row = a.ids ? (long long)a.ids[row] : a.gidx ? (long long)a.gidx[row] : (long long)row;
  if (!LAYA_IN_BOUNDS(a.src_rows <= 0 || (src_row >= 0 && src_row < a.src_rows), a.err, kErrBoundsLnSrc)) return;
  const float4* src = reinterpret_cast<const float4*>(a.src + src_row * D);
  float4 v[NV];
#pragma unroll
  for (int i = 0; i < NV; ++i) v[i] = __ldcs(src + lane + 32 * i);  // read once: evict-first
  if (a.copy_f32) {
    float4* c = reinterpret_cast<float4*>(a.copy_f32 + (long long)row * D);
#pragma unroll
    for (int i = 0; i < NV; ++i) c[lane + 32 * i] = v[i];
  }
  if (a.w) {
    layer_norm_regs<NV>(v, a.w, a.b, a.eps, D, lane);
    if (a.type_emb) {
      const int s = a.rowseq[row];
      if (s >= 0 && LAYA_IN_BOUNDS((a.n_seq <= 0 || s < a.n_seq) && a.qtype[s] >= 0 && a.qtype[s] < 3, a.err,
                                   kErrBoundsLnSeq)) {
        const float4* t = reinterpret_cast<const float4*>(a.type_emb + (long long)a.qtype[s] * D);
#pragma unroll
        for (int i = 0; i < NV; ++i) {
          const float4 tt = t[lane + 32 * i];
          v[i].x += tt.x; v[i].y += tt.y; v[i].z += tt.z; v[i].w += tt.w;
        }
      }
    }
  }
  if (a.out_f32) {
    float4* y = reinterpret_cast<float4*>(a.out_f32 + (long long)row * D);
#pragma unroll
    for (int i = 0; i < NV; ++i) y[lane + 32 * i] = v[i];
  }
  if (a.out_bf) {
    if (a.w2) layer_norm_regs<NV>(v, a.w2, a.b2, a.eps2, D, lane);
    store_bf16_planes<NV>(v, a.out_bf + (long long)row * D, a.out_bf + a.out_plane + (long long)row * D, a.out_planes,
                          lane);
  }
}

// One warp: the dot product of a D-element row (fp32 or bf16, 16-byte aligned, D a multiple of 128
// and at most 1024) with the fp32 vector w. Every load of the lane is issued before the first use.
__device__ __forceinline__ float row_dot(const void* row, bool f32, const float* w, int D, int lane) {
  const float4* w4 = reinterpret_cast<const float4*>(w);
  float s = 0.f;
  if (f32) {
    const float4* r4 = static_cast<const float4*>(row);
    float4 x[8], y[8];
#pragma unroll
    for (int i = 0; i < 8; ++i)
      if (lane + 32 * i < D / 4) { x[i] = r4[lane + 32 * i]; y[i] = w4[lane + 32 * i]; }
#pragma unroll
    for (int i = 0; i < 8; ++i)
      if (lane + 32 * i < D / 4) s += (x[i].x * y[i].x + x[i].y * y[i].y) + (x[i].z * y[i].z + x[i].w * y[i].w);
  } else {
    const uint4* r8 = static_cast<const uint4*>(row);
    uint4 x[4];
    float4 y[8];
#pragma unroll
    for (int i = 0; i < 4; ++i)
      if (lane + 32 * i < D / 8) {
        x[i] = r8[lane + 32 * i];
        y[2 * i] = w4[2 * (lane + 32 * i)];
        y[2 * i + 1] = w4[2 * (lane + 32 * i) + 1];
      }
#pragma unroll
    for (int i = 0; i < 4; ++i)
      if (lane + 32 * i < D / 8) {
        const __nv_bfloat162* h = reinterpret_cast<const __nv_bfloat162*>(&x[i]);
        const float2 f0 = __bfloat1622float2(h[0]), f1 = __bfloat1622float2(h[1]);
        const float2 f2 = __bfloat1622float2(h[2]), f3 = __bfloat1622float2(h[3]);
        s += (f0.x * y[2 * i].x + f0.y * y[2 * i].y) + (f1.x * y[2 * i].z + f1.y * y[2 * i].w) +
             ((f2.x * y[2 * i + 1].x + f2.y * y[2 * i + 1].y) + (f3.x * y[2 * i + 1].z + f3.y * y[2 * i + 1].w));
      }
  }
  return warp_sum(s);
}

// Grid (B, S): CTA (b, s) computes question b's marker logits and softmax features, then hidden units
// [s*256/S, (s+1)*256/S) of the act head. With S = 1 the CTA finishes the question alone; with S > 1
// each slice stores its hidden units to a.hid, and the slice that arrives last on a.hid_count[b]
// reads all 256 back, computes the outputs (in the same order as S = 1, so the results do not
// depend on S) and resets the counter.
__global__ void __launch_bounds__(256) head_out_kernel(const HeadOutArgs a) {
  __shared__ float s_logit[256];
  __shared__ __align__(16) float s_in[1024 + 8];
  __shared__ float s_hid[256];
  __shared__ int s_last;
  pdl_trigger();
  pdl_wait();
  const int b = blockIdx.x, tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int S = gridDim.y, slice = blockIdx.y, rows = 256 / S;
  const int D = a.D, nm = a.nmark[b], mo = a.moff[b];
  if (!LAYA_IN_BOUNDS(nm >= 1 && nm <= 256 && mo >= 0 && (a.n_logits <= 0 || mo + nm <= a.n_logits), a.err,
                      kErrBoundsHead))
    return;
  // scorer output Linear(d, 1) at every option marker of this question, one warp per marker
  for (int k = warp; k < nm; k += 8) {
    const long long row = mo + k;
    const void* hr = a.hs_f32 ? static_cast<const void*>(static_cast<const float*>(a.hs) + row * D)
                              : static_cast<const void*>(static_cast<const bf16*>(a.hs) + row * D);
    const float s = row_dot(hr, a.hs_f32 != 0, a.w3, D, lane) + a.b3;
    if (lane == 0) {
      s_logit[k] = s;
      if (slice == 0) a.logits[mo + k] = s;
    }
  }
  for (int i = tid; i < D; i += 256) s_in[i] = a.cls[(long long)b * D + i];
  __syncthreads();
  if (tid == 0) {
    // softmax over the question's option logits -> [top1, top1-top2, entropy/log(max(k,2)), max(k,2)/255]
    float mx = -INFINITY;
    for (int i = 0; i < nm; ++i) mx = fmaxf(mx, s_logit[i]);
    float sum = 0.f;
    for (int i = 0; i < nm; ++i) sum += expf(s_logit[i] - mx);
    float t1 = 0.f, t2 = 0.f, ent = 0.f;
    for (int i = 0; i < nm; ++i) {
      const float p = expf(s_logit[i] - mx) / sum;
      ent -= p * logf(fmaxf(p, 1e-9f));
      if (p > t1) { t2 = t1; t1 = p; } else if (p > t2) { t2 = p; }
    }
    const float k = (float)(nm < 2 ? 2 : nm);
    s_in[D] = t1;
    s_in[D + 1] = t1 - t2;
    s_in[D + 2] = ent / logf(k);
    s_in[D + 3] = k / 255.f;
  }
  __syncthreads();
  // act head hidden layer: 256 rows of D + 4 weights, two rows per step of each warp with all of the
  // lane's (at most nine) 16-byte pieces of both rows in flight together
  const int K4 = (D + 4) / 4;  // D + 4 is a multiple of 4: every row starts 16-byte aligned
  const float4* s4 = reinterpret_cast<const float4*>(s_in);
  const int per_warp = rows / 8;  // 32, 16, 8 or 4: even
  for (int j = slice * rows + warp * per_warp; j < slice * rows + (warp + 1) * per_warp; j += 2) {
    const float4* r0 = reinterpret_cast<const float4*>(a.w0) + (long long)j * K4;
    const float4* r1 = r0 + K4;
    float4 w0[9], w1[9];
#pragma unroll
    for (int i = 0; i < 9; ++i)
      if (lane + 32 * i < K4) { w0[i] = r0[lane + 32 * i]; w1[i] = r1[lane + 32 * i]; }
    float s0 = 0.f, s1 = 0.f;
#pragma unroll
    for (int i = 0; i < 9; ++i)
      if (lane + 32 * i < K4) {
        const float4 x = s4[lane + 32 * i];
        s0 += (w0[i].x * x.x + w0[i].y * x.y) + (w0[i].z * x.z + w0[i].w * x.w);
        s1 += (w1[i].x * x.x + w1[i].y * x.y) + (w1[i].z * x.z + w1[i].w * x.w);
      }
    s0 = warp_sum(s0);
    s1 = warp_sum(s1);
    if (lane == 0) {
      const float h0 = gelu_erf(s0 + a.b0[j]), h1 = gelu_erf(s1 + a.b0[j + 1]);
      if (S == 1) {
        s_hid[j] = h0;
        s_hid[j + 1] = h1;
      } else {
        a.hid[(long long)b * 256 + j] = h0;
        a.hid[(long long)b * 256 + j + 1] = h1;
      }
    }
  }
  if (S > 1) {
    __threadfence();  // this slice's hidden units are visible before its arrival is counted
    __syncthreads();
    if (tid == 0) s_last = atomicAdd(&a.hid_count[b], 1) == S - 1;
    __syncthreads();
    if (!s_last) return;
    __threadfence();
    s_hid[tid] = __ldcg(a.hid + (long long)b * 256 + tid);  // 256 threads, 256 hidden units
    if (tid == 0) a.hid_count[b] = 0;  // every slice has arrived: ready for the next launch
  }
  __syncthreads();
  for (int j = warp; j < a.n_act; j += 8) {
    const float* wr = a.w2 + (long long)j * 256;
    float x[8];
#pragma unroll
    for (int i = 0; i < 8; ++i) x[i] = wr[lane + 32 * i];
    float s = 0.f;
#pragma unroll
    for (int i = 0; i < 8; ++i) s = fmaf(x[i], s_hid[lane + 32 * i], s);
    s = warp_sum(s);
    if (lane == 0) a.act[(long long)b * a.n_act + j] = s + a.b2[j];
  }
}

}  // namespace

cudaError_t ln_launch(const LnArgs& a, cudaStream_t st) {
  if (a.rows <= 0) return cudaSuccess;
  if (a.D % 128 != 0 || a.D > 1024) return cudaErrorInvalidValue;
  const int grid = (a.rows + 7) / 8;
  switch (a.D / 128) {
    case 1: return launch_pdl(ln_kernel<1>, dim3(grid), dim3(256), 0, st, a);
    case 2: return launch_pdl(ln_kernel<2>, dim3(grid), dim3(256), 0, st, a);
    case 3: return launch_pdl(ln_kernel<3>, dim3(grid), dim3(256), 0, st, a);
    case 4: return launch_pdl(ln_kernel<4>, dim3(grid), dim3(256), 0, st, a);
    case 5: return launch_pdl(ln_kernel<5>, dim3(grid), dim3(256), 0, st, a);
    case 6: return launch_pdl(ln_kernel<6>, dim3(grid), dim3(256), 0, st, a);
    case 7: return launch_pdl(ln_kernel<7>, dim3(grid), dim3(256), 0, st, a);
    default: return launch_pdl(ln_kernel<8>, dim3(grid), dim3(256), 0, st, a);
  }
}

cudaError_t head_out_launch(const HeadOutArgs& a, cudaStream_t st) {
  if (a.B <= 0) return cudaSuccess;
  if (a.D > 1024 || a.D % 128 != 0 || a.n_act > 256) return cudaErrorInvalidValue;  // 16-byte row pieces
  // slices per question: as many of 8, 4, 2 as leave every slice an SM of its own
  static const int sms = [] {  // the devices of one host are alike
    int dev = 0, n = 0;
    if (cudaGetDevice(&dev) != cudaSuccess || cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess)
      return 1;
    return n;
  }();
  int S = 1;
  if (a.hid && a.hid_count)
    for (int s = 8; s > 1; s /= 2)
      if (a.B * s <= sms) { S = s; break; }
  return launch_pdl(head_out_kernel, dim3(a.B, S), dim3(256), 0, st, a);
}

}  // namespace laya
