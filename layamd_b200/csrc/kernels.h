// Host-side launchers for the sm_100a kernels of the Laya B200 engine. Device pointers only; every
// launcher enqueues on the given stream and never synchronises, so a whole pass can be captured in
// one CUDA graph.
#pragma once
#include <cuda.h>
#include <cuda_runtime.h>
#include <cuda_bf16.h>
#include <stdint.h>

namespace laya {

typedef __nv_bfloat16 bf16;

// ------------------------------------------------------------------ GEMM (tcgen05 + TMA + TMEM)
// C[M, N] = A[M, K] * B[N, K]^T with both operands K-major bf16 ("nn.Linear" layout: B is the
// weight as stored, [out, in]). Operands are stored as planes: plane 0 = bf16(x); in fp32-parity
// mode plane 1 = bf16(x - plane0), and the K loop runs three segments (A0*B0, A0*B1, A1*B0).
enum EpiKind : int { EPI_STORE = 0, EPI_ROPE = 1, EPI_GEGLU = 2, EPI_RESID = 3 };
enum OutMode : int { OUT_BF16 = 0, OUT_BF16X2 = 1, OUT_F32 = 2 };
enum Act : int { ACT_NONE = 0, ACT_RELU = 1, ACT_GELU = 2 };

struct GemmShape {
  int M;     // rows of A that are valid (rows beyond are computed from whatever the buffer holds and never stored)
  int N;     // rows of B, a multiple of 64 (for EPI_GEGLU: 2*I, interleaved as [64 input rows, their 64 gate rows]...)
  int K;     // reduction length of one segment
  int nseg;  // 1 (bf16) or 3 (split-bf16 fp32 emulation)
  // Split-K (single-CTA tiles only): the K loop is cut into `splits` slices run by different CTAs.
  // Slice s stores its fp32 partial tile into plane s of ws[splits][M][N] (16-byte aligned); a second
  // kernel sums the planes in slice order and runs the epilogue into `dst`, the buffer the output map
  // covers (x [M][N] fp32 for EPI_RESID, else [planes][M][cols] in the output format, planes
  // `dst_plane` elements apart).
  int splits = 1;
  float* ws = nullptr;
  void* dst = nullptr;
  long long dst_plane = 0;
};
constexpr int kMaxSplits = 8;
// Split-K workspace of an engine replica (fp32 partials): 32 Mi floats (128 MB) cover every split
// count the planner picks.
constexpr size_t kSplitWsFloats = size_t(32) << 20;
// Workspace floats a split-K launch needs.
inline size_t splitk_ws_floats(int M, int N, int splits) { return (size_t)splits * M * N; }
// Slice count for `tiles` 128 x 128 output tiles of `kblocks` 64-wide K blocks on `sms` SMs: the S
// minimising waves(tiles * S) * ceil(kblocks / S) + (S > 1 ? kSplitReduceBlocks : 0), i.e. the main
// loop in K-block times plus the partials' round trip through memory and the reduce kernel, which
// measured about 28 K-block times (11 us) on B200 at 512 rows. At least 4 K blocks per slice; 1 when
// the tiles already fill the GPU. At 512 rows this splits the long-K GEMMs (MLP-out, K = 2624; the
// head's FFN-2, K = 4096) and keeps whole-K tiles for K = 1024. `credit`: K-block times that a split
// saves elsewhere — a LayerNorm launch that the reduce kernel absorbs (a residual GEMM followed by a
// LayerNorm), subtracted from every S > 1.
constexpr int kSplitReduceBlocks = 28;
inline int splitk_choose(int tiles, int kblocks, int sms, int credit = 0) {
  if (tiles >= sms) return 1;
  int best = 1;
  long long best_cost = kblocks;
  for (int s = 2; s <= kMaxSplits; ++s) {
    if (kblocks / s < 4) break;
    const long long waves = (tiles * s + sms - 1) / sms;
    const long long cost = waves * ((kblocks + s - 1) / s) + kSplitReduceBlocks - credit;
    if (cost < best_cost) { best_cost = cost; best = s; }
  }
  return best;
}

// The epilogue writes through the output tensor map `tc` of gemm_launch (make_output_map): bf16
// planes for OUT_BF16 / OUT_BF16X2 (plane 1 = lo part), fp32 for OUT_F32 and for EPI_RESID, whose
// result is added into the existing contents (x += acc) by TMA reduce-add.
struct GemmEpi {
  int kind = EPI_STORE;
  int out_mode = OUT_BF16;
  const float* bias = nullptr; // [N] fp32, optional
  int act = ACT_NONE;
  const float* cos_t = nullptr;  // EPI_ROPE: [max_pos, 32] tables for this layer's theta
  const float* sin_t = nullptr;
  const int* pos = nullptr;      // EPI_ROPE: position of each row within its sequence
  int rope_cols = 0;             // EPI_ROPE: rotate columns [0, rope_cols) (q and k), head dim 64
  int geglu_I = 0;               // EPI_GEGLU: output width I (a multiple of 64)
  // EPI_RESID with split-K only (GemmShape::splits > 1): the reduce kernel also writes
  // ln_out = LayerNorm(x) * ln_w (no bias) as bf16 planes (ln_planes of them, ln_plane elements
  // apart) from the new x of each row, the LayerNorm kernel's arithmetic; N a multiple of 128, <= 1024.
  const float* ln_w = nullptr;
  float ln_eps = 1e-5f;
  bf16* ln_out = nullptr;
  long long ln_plane = 0;
  int ln_planes = 1;
  // debug bounds mode: rows of the RoPE tables (positions must lie below it) and the error word
  // (gemm_launch fills it from its `err`)
  int rope_rows = 0;
  int* err = nullptr;
};

// Output map of the GEMM epilogue over [planes][rows][ld] (bf16) or [rows][ld] (fp32, planes 1):
// {32 rows x 128 bytes} boxes with the 128-byte swizzle. Rows beyond `rows` are never written.
bool make_output_map(CUtensorMap* map, const void* base, bool f32, uint64_t ld, uint64_t rows, uint64_t planes);

// Builds a 3-D tensor map {K, rows, planes} over a bf16 operand with a {64, box_rows, 1} box and the
// 128-byte swizzle. Returns false if the driver rejects it (alignment).
bool make_operand_map(CUtensorMap* map, const void* base, uint64_t K, uint64_t rows, uint64_t planes,
                      uint32_t box_rows);

// Raises the dynamic shared-memory limit of every GEMM instantiation on the current device; call
// once per device before the first gemm_launch there.
cudaError_t gemm_prepare_device();

// Tile selector for gemm_launch: one CTA per 128 x 128 or 128 x 256 tile (bn = 128 / 256, `tb` box
// height = bn), or a CTA pair per 256 x 256 tile with the 2-SM MMA (bn = kGemmPair, `tb` box 128).
constexpr int kGemmPair = 512;
// Co-resident CTA pairs of the pair kernel on the current device (set by gemm_prepare_device).
int gemm_pair_clusters();

// K-block times credited to a split whose reduce kernel absorbs the LayerNorm that follows the GEMM:
// the split costs the partials' round trip and the reduce (kSplitReduceBlocks) but saves the
// LayerNorm launch, leaving about 8. Measured at 512 rows (ModernBERT-large, one B200): the attention
// out-projection then splits 4 ways with the MLP LayerNorm in its reduce, 1.774 -> 1.687 ms per pass.
constexpr int kSplitLnCredit = 20;

// Tile and K split of one GEMM launch (host-only). Tile: the CTA-pair 256 x 256 tile when its tile
// count fills every co-resident pair twice, else the one-CTA width (128 or 256) with fewer whole
// waves, a 128 x 256 tile counting 1.6 of a 128 x 128 one (it reads each A block once per 256
// columns: at 512 rows the GeGLU GEMM runs one wave of 84 wide tiles in 13 us against two waves of
// 164 narrow ones in 17 us). K split (128-wide tiles only, when allowed): splitk_choose, with
// `ln_credit` when the reduce kernel can absorb the following LayerNorm, and no more slices than a
// workspace of `ws_floats` partials holds. nseg: K segments per K block (1 bf16, 3 fp32 parity).
struct GemmPlan {
  int bn = 128;
  int splits = 1;
};
inline GemmPlan gemm_plan(int M, int N, int K, int nseg, int num_sms, int pair_clusters, bool allow_split,
                          size_t ws_floats, int ln_credit) {
  GemmPlan p;
  if (N >= 256) {
    const long long tp = (long long)((M + 255) / 256) * ((N + 255) / 256);
    if (pair_clusters > 0 && tp >= 2LL * pair_clusters) {
      p.bn = kGemmPair;
    } else {
      const long long rows = (M + 127) / 128;
      const long long w128 = (rows * ((N + 127) / 128) + num_sms - 1) / num_sms;
      const long long w256 = (rows * ((N + 255) / 256) + num_sms - 1) / num_sms;
      p.bn = 10 * w128 > 16 * w256 ? 256 : 128;
    }
  }
  if (p.bn == 128 && allow_split) {
    const int tiles = ((M + 127) / 128) * ((N + 127) / 128);
    int s = splitk_choose(tiles, ((K + 63) / 64) * nseg, num_sms, ln_credit);
    while (s > 1 && splitk_ws_floats(M, N, s) > ws_floats) --s;
    p.splits = s;
  }
  return p;
}

// `grid_ctas` caps the persistent grid (CTAs; a pair counts as two).
cudaError_t gemm_launch(const CUtensorMap& ta, const CUtensorMap& tb, const CUtensorMap& tc, int bn,
                        const GemmShape& sh, const GemmEpi& ep, int* err, int grid_ctas, cudaStream_t st);

// ------------------------------------------------------------------ attention
// Work item of the attention kernels: 64 (mma.sync) or 128 (tcgen05) query rows of one sequence.
struct AttnItem {
  int seq;   // sequence index within the pass (< 0: unused slot)
  int q0;    // first query position within the sequence (contiguous mode)
  int goff;  // gathered mode: offset into the gathered-row lists; tcgen05 items: first packed row
  int nq;    // gathered mode: number of query rows (<= 64); tcgen05 items: sequence length
};
struct AttnArgs {
  const void* qkv;       // [rows, 3*D]: bf16 (fast path) or fp32 (parity path)
  void* out;             // bf16 planes [P][rows_out, D]
  long long out_plane;   // plane stride (elements) when P == 2
  int out_planes;        // 1 or 2
  const AttnItem* items;
  int n_items;
  const int* soff;       // [B] first packed row of each sequence
  const int* slen;       // [B] sequence length
  const int* gsrc;       // gathered mode: packed row of each listed query
  const int* gdst;       // gathered mode: output row of each listed query
  int gathered;          // 0: contiguous query blocks, 1: gathered queries (full attention)
  int H;                 // heads (head dim is 64)
  int window;            // half window (|q-k| <= window), 0 = global
  float scale;           // softmax scale (1/sqrt(64))
  // extents the debug bounds mode checks the maps against (0: unchecked), and its error word
  int rows = 0;          // rows of qkv
  int rows_out = 0;      // rows of out
  int n_seq = 0;         // entries of soff / slen
  int* err = nullptr;
};
cudaError_t attn_bf16_launch(const AttnArgs& a, cudaStream_t st);
cudaError_t attn_f32_launch(const AttnArgs& a, cudaStream_t st);

// tcgen05 attention (bf16, contiguous mode only): items are 128-query tiles (q0 a multiple of 128)
// holding {seq, q0, first packed row, length}, longest sequences first (the persistent CTAs claim
// (item, head) units in that order from `ticket`: two device ints, zero before the first launch and
// reset to zero by the last CTA of every launch); `tq` / `tkv` are make_operand_map over the qkv rows (K = 3*D, rows, 1 plane)
// with 128-row and 64-row boxes; out is one bf16 plane [rows, D]. The K / V rows read past a
// sequence's end must hold finite values. Bounded waits record an error code in *err.
// attn_tc_prepare_device() runs once per device first.
cudaError_t attn_tc_prepare_device();
cudaError_t attn_tc_launch(const CUtensorMap& tq, const CUtensorMap& tkv, const AttnArgs& a, int* ticket, int* err,
                           cudaStream_t st);

// ------------------------------------------------------------------ row kernels (LayerNorm family)
// One warp per row. Source row: emb[ids[r]] (embedding), x[gidx[r]] (gather) or x[r].
// v = source (+ add_row); y = LN(v) * w (+ b) (+ type_emb[qtype[rowseq[r]]]);
// optional second LayerNorm z = LN(y) * w2 (+ b2) feeding the bf16 planes.
struct LnArgs {
  int rows = 0, D = 0;
  float eps = 1e-5f;
  const float* src = nullptr;     // fp32 [*, D]
  const int* ids = nullptr;       // embedding lookup indices (src = table)
  const int* gidx = nullptr;      // gather indices
  const float* w = nullptr;       // LN gain (null: identity LayerNorm skipped, y = v)
  const float* b = nullptr;
  const float* type_emb = nullptr;  // [3, D]
  const int* qtype = nullptr;       // [B]
  const int* rowseq = nullptr;      // [rows], < 0: padding row (no type embedding)
  float* copy_f32 = nullptr;      // write v (pre-norm source row) as fp32 [rows, D]
  float* out_f32 = nullptr;       // write y as fp32 (may alias src when no gather)
  const float* w2 = nullptr;      // second LayerNorm (optional)
  const float* b2 = nullptr;
  float eps2 = 1e-5f;
  bf16* out_bf = nullptr;         // write (second LN ? z : y) as bf16 planes
  int out_planes = 1;
  long long out_plane = 0;
  // extents the debug bounds mode checks the maps against (0: unchecked), and its error word
  int src_rows = 0;               // rows of src that ids / gidx may name
  int n_seq = 0;                  // entries of qtype that rowseq may name
  int* err = nullptr;
};
cudaError_t ln_launch(const LnArgs& a, cudaStream_t st);

// ------------------------------------------------------------------ decision-head outputs
// One CTA per question: marker logits (scorer's final Linear(d,1)), softmax features, act head.
struct HeadOutArgs {
  int B = 0, D = 0, n_act = 0;
  const void* hs = nullptr;       // scorer hidden [KT, D] (GELU output), bf16 or fp32
  int hs_f32 = 0;
  const float* w3 = nullptr;      // [D]
  float b3 = 0.f;
  const float* cls = nullptr;     // fp32 CLS rows after the head [B, D]
  const int* moff = nullptr;      // [B] first gathered marker row / logit index of each question
  const int* nmark = nullptr;     // [B]
  const float* w0 = nullptr;      // act head Linear(D+4, 256): [256, D+4]
  const float* b0 = nullptr;
  const float* w2 = nullptr;      // Linear(256, n_act): [n_act, 256]
  const float* b2 = nullptr;
  float* logits = nullptr;        // [sum nmark]
  float* act = nullptr;           // [B, n_act]
  // Scratch of the sliced form (small batches: the act head's 256 hidden units of a question split
  // over several CTAs): hidden values [B, 256] and per-question arrival counters [B], zero at
  // allocation and left at zero by every launch. Null: one CTA per question.
  float* hid = nullptr;
  int* hid_count = nullptr;
  // extents the debug bounds mode checks the maps against (0: unchecked), and its error word
  int n_logits = 0;               // marker rows of hs / logit slots
  int* err = nullptr;
};
cudaError_t head_out_launch(const HeadOutArgs& a, cudaStream_t st);

// ------------------------------------------------------------------ kernel-level C entry points
// Error word shared by the kernel-level entry points on device `dev` (laya_b200_gemm,
// laya_b200_gemm_splitk, laya_b200_attention, laya_b200_watchdog_selftest): allocated and zeroed on
// first use, then sticky (first writer wins) until a synchronous call or laya_b200_kernel_error
// reads and clears it. Null if the allocation failed.
int* entry_error_word(int dev);

}  // namespace laya
