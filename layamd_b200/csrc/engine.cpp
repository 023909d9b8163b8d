// Laya B200 engine host code; see engine.hpp for the design. Host C++ over the CUDA runtime: no
// kernel is launched from here directly, only through the launchers of kernels.h.
#include "engine.hpp"

#include <algorithm>
#include <chrono>
#include <cmath>
#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <mutex>
#include <numeric>
#include <thread>

namespace laya {

namespace {

#define LAYA_TRY(expr)                                                                                   \
  do {                                                                                                   \
    cudaError_t e_ = (expr);                                                                             \
    if (e_ != cudaSuccess) {                                                                             \
      if (err) *err = std::string(#expr) + ": " + cudaGetErrorString(e_);                                \
      return false;                                                                                      \
    }                                                                                                    \
  } while (0)

uint16_t f32_to_bf16(float f) {
  uint32_t u;
  memcpy(&u, &f, 4);
  if ((u & 0x7fffffffu) > 0x7f800000u) return 0x7fc0;  // NaN
  u += 0x7fffu + ((u >> 16) & 1u);                     // round to nearest even
  return static_cast<uint16_t>(u >> 16);
}
float bf16_to_f32(uint16_t h) {
  const uint32_t u = static_cast<uint32_t>(h) << 16;
  float f;
  memcpy(&f, &u, 4);
  return f;
}

int env_int(const char* k, int d) {
  const char* v = getenv(k);
  return v && *v ? atoi(v) : d;
}

size_t align4(size_t n) { return (n + 3) & ~size_t(3); }

// Offsets (in ints) of the per-pass metadata arrays inside the staging block.
struct MetaLayout {
  size_t ids, pos, rowseq, soff, slen, qt, nm, moff, items, items128, gitems, gsrc, gdst, grow, total;
  int items_cap, items128_cap, gitems_cap;
};
MetaLayout meta_layout(int Tpad, int n, int R) {
  MetaLayout L;
  size_t o = 0;
  auto take = [&](size_t cnt) { size_t r = o; o += align4(cnt); return r; };
  L.items_cap = Tpad / 64 + n;
  L.items128_cap = Tpad / 128 + n;
  L.gitems_cap = R / 64 + n + 1;
  L.ids = take(Tpad);
  L.pos = take(Tpad);
  L.rowseq = take(Tpad);
  L.soff = take(n);
  L.slen = take(n);
  L.qt = take(n);
  L.nm = take(n);
  L.moff = take(n);
  L.items = take((size_t)L.items_cap * 4);
  L.items128 = take((size_t)L.items128_cap * 4);
  L.gitems = take((size_t)L.gitems_cap * 4);
  L.gsrc = take(R);
  L.gdst = take(R);
  L.grow = take(R);
  L.total = o;
  return L;
}

}  // namespace

bool validate_batch(int B, const int* lens, const int* nmark, const int* markers, int max_len) {
  if (B < 0) return false;
  size_t mo = 0;
  for (int b = 0; b < B; ++b) {
    if (lens[b] < 1 || lens[b] > max_len || nmark[b] < 1 || nmark[b] > kMaxMarkers) return false;
    for (int k = 0; k < nmark[b]; ++k)
      if (markers[mo + k] < 0 || markers[mo + k] >= lens[b]) return false;
    mo += nmark[b];
  }
  return true;
}

bool plan_passes(int B, const int* lens, const int* nmark, int pass_tokens, int max_seqs, int max_gathered,
                 std::vector<PassPlan>* out) {
  out->clear();
  int b0 = 0;
  while (b0 < B) {
    PassPlan p;
    p.b0 = b0;
    while (b0 + p.n < B && p.n < max_seqs) {
      const int b = b0 + p.n;
      if (p.n > 0 && (p.T + lens[b] > pass_tokens || p.KT + nmark[b] + p.n + 1 > max_gathered)) break;
      if (p.n == 0 && (lens[b] > pass_tokens || nmark[b] + 1 > max_gathered)) return false;
      p.T += lens[b];
      p.KT += nmark[b];
      ++p.n;
    }
    p.Tpad = (p.T + 63) / 64 * 64;
    p.R = p.KT + p.n;
    out->push_back(p);
    b0 += p.n;
  }
  return true;
}

void fill_pass_meta(const PassPlan& p, const Question* qs, int pad_id, int* m) {
  const MetaLayout L = meta_layout(p.Tpad, p.n, p.R);
  AttnItem* items = reinterpret_cast<AttnItem*>(m + L.items);
  AttnItem* items128 = reinterpret_cast<AttnItem*>(m + L.items128);
  AttnItem* gitems = reinterpret_cast<AttnItem*>(m + L.gitems);
  int r = 0, mo = 0, it = 0, it128 = 0, git = 0, gl = 0;
  for (int i = 0; i < p.n; ++i) {
    const Question& q = qs[p.b0 + i];
    m[L.soff + i] = r;
    m[L.slen + i] = q.len;
    m[L.qt + i] = q.qtype;
    m[L.nm + i] = q.nmark;
    m[L.moff + i] = mo;
    memcpy(m + L.ids + r, q.ids, (size_t)q.len * 4);
    for (int j = 0; j < q.len; ++j) {
      m[L.pos + r + j] = j;
      m[L.rowseq + r + j] = i;
    }
    for (int q0 = 0; q0 < q.len; q0 += 64) items[it++] = AttnItem{i, q0, 0, 0};
    for (int q0 = 0; q0 < q.len; q0 += 128) items128[it128++] = AttnItem{i, q0, r, q.len};  // base row, length
    const int cnt = q.nmark + 1;
    for (int k = 0; k < q.nmark; ++k) {
      m[L.gsrc + gl + k] = r + q.markers[k];
      m[L.gdst + gl + k] = mo + k;
      m[L.grow + mo + k] = r + q.markers[k];
    }
    m[L.gsrc + gl + q.nmark] = r;
    m[L.gdst + gl + q.nmark] = p.KT + i;
    m[L.grow + p.KT + i] = r;
    for (int c0 = 0; c0 < cnt; c0 += 64) gitems[git++] = AttnItem{i, 0, gl + c0, std::min(64, cnt - c0)};
    gl += cnt;
    r += q.len;
    mo += q.nmark;
  }
  for (int j = r; j < p.Tpad; ++j) {
    m[L.ids + j] = pad_id;
    m[L.pos + j] = 0;
    m[L.rowseq + j] = -1;
  }
  // the persistent tcgen05 attention deals its units out round robin: longest sequences first
  std::stable_sort(items128, items128 + it128, [](const AttnItem& a, const AttnItem& b) { return a.nq > b.nq; });
  for (; it < L.items_cap; ++it) items[it] = AttnItem{-1, 0, 0, 0};
  for (; it128 < L.items128_cap; ++it128) items128[it128] = AttnItem{-1, 0, 0, 0};
  for (; git < L.gitems_cap; ++git) gitems[git] = AttnItem{-1, 0, 0, 0};
}

size_t pass_meta_ints(const PassPlan& p) { return meta_layout(p.Tpad, p.n, p.R).total; }

void corrupt_pass_meta(const PassPlan& p, int* m, int which, int vocab) {
  const MetaLayout L = meta_layout(p.Tpad, p.n, p.R);
  const int last = p.n - 1;
  switch (which) {
    case 1: m[L.soff + last] += 1; break;                         // question offset
    case 2: m[L.qt + last] = 3; break;                            // question type
    case 3: m[L.nm + last] = kMaxMarkers + 1; break;              // marker count
    case 4: m[L.ids + p.T - 1] = vocab; break;                    // token id past the vocabulary
    case 5: m[L.rowseq + p.T - 1] = p.n; break;                   // row -> question
    case 6: reinterpret_cast<AttnItem*>(m + L.items)[0].q0 = 64 * ((m[L.slen] + 63) / 64); break;  // 64-row item
    case 7: m[L.gsrc + 0] = m[L.soff] + m[L.slen]; break;         // gathered query outside its question
    case 8: m[L.grow + p.R - 1] = p.T; break;                     // gathered row past the packed rows
    default: break;
  }
}

int check_pass_meta(const PassPlan& p, const int* m, const PackLimits& lim) {
  const MetaLayout L = meta_layout(p.Tpad, p.n, p.R);
  if (p.n < 1 || p.n > lim.max_seqs || p.Tpad > lim.max_rows || p.Tpad % 64 != 0 || p.T > p.Tpad ||
      p.R != p.KT + p.n || p.R > lim.max_gathered)
    return 1;  // pass shape beyond the arena
  const int *ids = m + L.ids, *pos = m + L.pos, *rowseq = m + L.rowseq, *soff = m + L.soff, *slen = m + L.slen,
            *qt = m + L.qt, *nm = m + L.nm, *moff = m + L.moff, *gsrc = m + L.gsrc, *gdst = m + L.gdst,
            *grow = m + L.grow;
  int r = 0, mo = 0;
  for (int i = 0; i < p.n; ++i) {  // questions back to back, in order
    if (soff[i] != r || slen[i] < 1 || slen[i] > lim.max_len) return 2;
    if (qt[i] < 0 || qt[i] > 2) return 3;
    if (nm[i] < 1 || nm[i] > kMaxMarkers || moff[i] != mo) return 4;
    r += slen[i];
    mo += nm[i];
  }
  if (r != p.T || mo != p.KT) return 5;
  for (int j = 0; j < p.Tpad; ++j) {  // per-row maps
    if (ids[j] < 0 || ids[j] >= lim.vocab) return 6;
    const int s = rowseq[j];
    if (j < p.T ? (s < 0 || s >= p.n || j < soff[s] || j >= soff[s] + slen[s] || pos[j] != j - soff[s])
                : (s != -1 || pos[j] != 0))
      return 7;
  }
  // every row of every question in exactly one query block: a question's blocks are adjacent in the
  // list, in order, starting at 0 and ending at its last row; unused slots only after the last block
  auto items_ok = [&](const AttnItem* it, int cap, int rows_per, bool tc) {
    std::vector<char> done(p.n, 0);
    int cur = -1, next_q0 = 0, used = 0;
    for (int k = 0; k < cap; ++k) {
      const int s = it[k].seq;
      if (s < 0) break;
      ++used;
      if (s >= p.n || (tc && (it[k].goff != soff[s] || it[k].nq != slen[s]))) return false;
      if (s != cur) {
        if (cur >= 0 && next_q0 < slen[cur]) return false;  // the previous question is incomplete
        if (done[s]) return false;
        done[s] = 1;
        cur = s;
        next_q0 = 0;
      }
      if (it[k].q0 != next_q0 || next_q0 >= slen[s]) return false;
      next_q0 += rows_per;
    }
    for (int k = used; k < cap; ++k)
      if (it[k].seq >= 0) return false;
    if (cur < 0 || next_q0 < slen[cur]) return false;
    for (int i = 0; i < p.n; ++i)
      if (!done[i]) return false;
    return true;
  };
  if (!items_ok(reinterpret_cast<const AttnItem*>(m + L.items), L.items_cap, 64, false)) return 8;
  if (!items_ok(reinterpret_cast<const AttnItem*>(m + L.items128), L.items128_cap, 128, true)) return 9;
  const AttnItem* g = reinterpret_cast<const AttnItem*>(m + L.gitems);
  long long gl = 0;
  for (int k = 0; k < L.gitems_cap; ++k) {  // gathered queries: markers then the CLS row
    if (g[k].seq < 0) continue;
    const int s = g[k].seq;
    if (s >= p.n || g[k].nq < 1 || g[k].nq > 64 || g[k].goff != gl || g[k].goff + g[k].nq > p.R) return 10;
    for (int t = g[k].goff; t < g[k].goff + g[k].nq; ++t)
      if (gsrc[t] < soff[s] || gsrc[t] >= soff[s] + slen[s] || gdst[t] < 0 || gdst[t] >= p.R) return 11;
    gl += g[k].nq;
  }
  if (gl != p.R) return 12;
  for (int t = 0; t < p.R; ++t)
    if (grow[t] < 0 || grow[t] >= p.T) return 13;
  return 0;
}

// ===================================================================== Replica (one GPU)
class Replica {
 public:
  Engine& E;
  const Config& cfg;
  int dev = 0, P = 1, nseg = 1, num_sms = 148, pair_clusters = 0;
  // split-K workspace (fp32 partials of every slice), sized at load
  float* ws = nullptr;
  size_t ws_floats = 0;
  bool use_splitk = true;
  // LAYA_SPLIT_LN=0: a split-K residual GEMM leaves its LayerNorm to the LN kernel (same K split)
  bool split_ln = true;
  // K-block times credited to a split whose reduce kernel can absorb the following LayerNorm launch
  // (kSplitLnCredit; LAYA_SPLIT_LN_CREDIT overrides)
  int split_ln_credit = kSplitLnCredit;
  cudaStream_t st = nullptr;
  std::vector<void*> allocs;
  std::vector<void*> host_allocs;

  // weights
  float *tok_emb = nullptr, *emb_norm = nullptr, *final_norm = nullptr, *type_emb = nullptr;
  struct Layer {
    float* attn_norm = nullptr;
    float* mlp_norm = nullptr;
    Mat Wqkv, Wo, Wi, Wmo;
  };
  struct Head {
    float *n1w, *n1b, *n2w, *n2b, *inB, *outB, *l1B, *l2B;
    Mat inW, outW, l1W, l2W;
  };
  std::vector<Layer> enc;
  std::vector<Head> head;
  Mat sc1;
  float *sc_nw = nullptr, *sc_nb = nullptr, *sc1B = nullptr, *sc3W = nullptr;
  float sc3B = 0.f;
  float *a0W = nullptr, *a0B = nullptr, *a2W = nullptr, *a2B = nullptr;
  float *cos_g = nullptr, *sin_g = nullptr, *cos_l = nullptr, *sin_l = nullptr;

  // activations
  int Tcap = 0, Rcap = 0, Bcap = 0;
  float* x = nullptr;
  void* qkv = nullptr;
  Operand xn, ao, mg, ff, xng, aog, ffg, xs;
  // epilogue output maps (TMA store / reduce-add targets)
  CUtensorMap out_qkv, out_mg, out_ff, out_ffg, out_x, out_xg, out_hs;
  CUtensorMap qkv_map, qkv_map64;  // bf16 qkv rows as TMA sources of the tcgen05 attention (Q / K,V boxes)
  bool attn_tc = false;
  bool attn_small = true;  // LAYA_ATTN_SMALL=0: the tcgen05 attention for small passes too
  int* d_attn_ticket = nullptr;  // work counter of the persistent attention kernel
  float* xg = nullptr;
  void* hs = nullptr;
  float *d_logits = nullptr, *d_act = nullptr;
  float* d_head_hid = nullptr;  // sliced act head of small batches: hidden units [Bcap, 256]
  int* d_head_cnt = nullptr;    // and per-question arrival counters [Bcap]
  int* d_err = nullptr;

  // per-pass staging
  int* h_meta = nullptr;
  int* d_meta = nullptr;
  size_t meta_cap = 0;
  float* h_out = nullptr;  // logits [Rcap] | act [Bcap * n_act] | err

  // graphs
  std::map<std::tuple<int, int, int, int>, cudaGraphExec_t> graphs;
  bool capturing = false;

  // profiling: per stage (device ms, launches)
  std::vector<std::pair<std::string, std::pair<double, long long>>> prof_acc;
  std::vector<std::tuple<const char*, cudaEvent_t, cudaEvent_t>> prof_pending;
  std::vector<cudaEvent_t> ev_pool;
  size_t ev_used = 0;

  // staged pass (benchmark replay)
  std::vector<Question> staged;
  PassPlan staged_plan;
  cudaGraphExec_t staged_graph = nullptr;
  // the same pass captured with an event pair around every stage (laya_replay_profiled)
  cudaGraphExec_t staged_prof_graph = nullptr;
  std::vector<std::tuple<const char*, cudaEvent_t, cudaEvent_t>> staged_prof_events;
  bool capturing_prof = false;

  // Failure injection for host-side tests (LAYA_FAIL_REPLICA=i[:n] at load): this replica's next
  // n non-empty shards return -2 before anything is uploaded or launched.
  int fail_runs = 0;
  int plant_id = 0;  // debug-bounds builds: LAYA_DEBUG_PLANT_ID test hook (see fill)

  Replica(Engine& e, int d) : E(e), cfg(e.cfg), dev(d) {}
  ~Replica() { release(); }

  void release() {
    cudaSetDevice(dev);
    if (st) cudaStreamSynchronize(st);
    for (auto& kv : graphs) cudaGraphExecDestroy(kv.second);
    graphs.clear();
    if (staged_graph) cudaGraphExecDestroy(staged_graph);
    staged_graph = nullptr;
    drop_staged_profile();
    for (auto ev : ev_pool) cudaEventDestroy(ev);
    ev_pool.clear();
    for (void* p : allocs) cudaFree(p);
    allocs.clear();
    for (void* p : host_allocs) cudaFreeHost(p);
    host_allocs.clear();
    if (st) cudaStreamDestroy(st);
    st = nullptr;
  }

  template <typename T>
  bool dalloc(T** p, size_t bytes, std::string* err) {
    void* q = nullptr;
    LAYA_TRY(cudaMalloc(&q, bytes < 16 ? 16 : bytes));
    LAYA_TRY(cudaMemset(q, 0, bytes < 16 ? 16 : bytes));
    allocs.push_back(q);
    *p = static_cast<T*>(q);
    return true;
  }

  bool upload_vec(const SafeTensors& st_, const std::string& name, float** out, std::string* err, size_t expect = 0) {
    std::vector<float> v;
    if (!st_.to_f32(name, &v, err)) return false;
    if (expect && v.size() != expect) { *err = name + ": unexpected size"; return false; }
    if (!dalloc(out, v.size() * 4, err)) return false;
    LAYA_TRY(cudaMemcpy(*out, v.data(), v.size() * 4, cudaMemcpyHostToDevice));
    return true;
  }

  // [N, K] weight -> P bf16 planes (hi, and lo = bf16(w - hi) in parity mode), optionally with the
  // GeGLU row interleave: groups of 64 input rows followed by their 64 gate rows.
  bool upload_mat(const SafeTensors& st_, const std::string& name, int N, int K, Mat* m, std::string* err,
                  bool geglu = false) {
    std::vector<float> v;
    if (!st_.to_f32(name, &v, err)) return false;
    if (v.size() != (size_t)N * K) { *err = name + ": unexpected shape"; return false; }
    if (geglu) {
      const int I = N / 2;
      std::vector<float> w(v.size());
      int r = 0;
      for (int j = 0; j < I; j += 64) {
        for (int i = 0; i < 64; ++i, ++r) memcpy(&w[(size_t)r * K], &v[(size_t)(j + i) * K], (size_t)K * 4);
        for (int i = 0; i < 64; ++i, ++r) memcpy(&w[(size_t)r * K], &v[(size_t)(I + j + i) * K], (size_t)K * 4);
      }
      v.swap(w);
    }
    std::vector<uint16_t> h((size_t)P * N * K);
    for (size_t i = 0; i < v.size(); ++i) {
      const uint16_t hi = f32_to_bf16(v[i]);
      h[i] = hi;
      if (P == 2) h[v.size() + i] = f32_to_bf16(v[i] - bf16_to_f32(hi));
    }
    if (!dalloc(&m->p, h.size() * 2, err)) return false;
    LAYA_TRY(cudaMemcpy(m->p, h.data(), h.size() * 2, cudaMemcpyHostToDevice));
    m->N = N;
    m->K = K;
    if (!make_operand_map(&m->m128, m->p, K, N, P, 128)) { *err = name + ": tensor map rejected"; return false; }
    if (N >= 256 && !make_operand_map(&m->m256, m->p, K, N, P, 256)) {
      *err = name + ": tensor map rejected";
      return false;
    }
    return true;
  }

  bool make_operand(Operand* op, int rows, int K, std::string* err) {
    op->rows = rows;
    op->K = K;
    op->plane = (long long)rows * K;
    if (!dalloc(&op->p, (size_t)P * rows * K * 2, err)) return false;
    if (!make_operand_map(&op->map, op->p, K, rows, P, 128)) { *err = "activation tensor map rejected"; return false; }
    return true;
  }

  bool load(const SafeTensors& W, std::string* err) {
    LAYA_TRY(cudaSetDevice(dev));
    LAYA_TRY(cudaDeviceGetAttribute(&num_sms, cudaDevAttrMultiProcessorCount, dev));
    LAYA_TRY(gemm_prepare_device());
    LAYA_TRY(attn_tc_prepare_device());
    pair_clusters = getenv("LAYA_NO_PAIR_GEMM") ? 0 : gemm_pair_clusters();
    LAYA_TRY(cudaStreamCreateWithFlags(&st, cudaStreamNonBlocking));
    P = E.precision == 1 ? 2 : 1;
    nseg = P == 2 ? 3 : 1;
    const int D = cfg.d, I = cfg.intermediate, FF = cfg.head_ffn, V = cfg.vocab;
    if (!upload_vec(W, "encoder.embeddings.tok_embeddings.weight", &tok_emb, err, (size_t)V * D)) return false;
    if (!upload_vec(W, "encoder.embeddings.norm.weight", &emb_norm, err, D)) return false;
    if (!upload_vec(W, "encoder.final_norm.weight", &final_norm, err, D)) return false;
    if (!upload_vec(W, "type_emb.weight", &type_emb, err, (size_t)3 * D)) return false;
    enc.resize(cfg.n_layers);
    char b[160];
    for (int i = 0; i < cfg.n_layers; ++i) {
      auto T = [&](const char* f) { snprintf(b, sizeof b, f, i); return std::string(b); };
      if (W.get(T("encoder.layers.%d.attn_norm.weight"))) {
        if (!upload_vec(W, T("encoder.layers.%d.attn_norm.weight"), &enc[i].attn_norm, err, D)) return false;
      }
      if (!upload_mat(W, T("encoder.layers.%d.attn.Wqkv.weight"), 3 * D, D, &enc[i].Wqkv, err)) return false;
      if (!upload_mat(W, T("encoder.layers.%d.attn.Wo.weight"), D, D, &enc[i].Wo, err)) return false;
      if (!upload_vec(W, T("encoder.layers.%d.mlp_norm.weight"), &enc[i].mlp_norm, err, D)) return false;
      if (!upload_mat(W, T("encoder.layers.%d.mlp.Wi.weight"), 2 * I, D, &enc[i].Wi, err, true)) return false;
      if (!upload_mat(W, T("encoder.layers.%d.mlp.Wo.weight"), D, I, &enc[i].Wmo, err)) return false;
    }
    head.resize(cfg.head_layers);
    for (int j = 0; j < cfg.head_layers; ++j) {
      auto T = [&](const char* f) { snprintf(b, sizeof b, f, j); return std::string(b); };
      Head& h = head[j];
      if (!upload_vec(W, T("head.layers.%d.norm1.weight"), &h.n1w, err, D) ||
          !upload_vec(W, T("head.layers.%d.norm1.bias"), &h.n1b, err, D) ||
          !upload_vec(W, T("head.layers.%d.norm2.weight"), &h.n2w, err, D) ||
          !upload_vec(W, T("head.layers.%d.norm2.bias"), &h.n2b, err, D) ||
          !upload_mat(W, T("head.layers.%d.self_attn.in_proj_weight"), 3 * D, D, &h.inW, err) ||
          !upload_vec(W, T("head.layers.%d.self_attn.in_proj_bias"), &h.inB, err, 3 * D) ||
          !upload_mat(W, T("head.layers.%d.self_attn.out_proj.weight"), D, D, &h.outW, err) ||
          !upload_vec(W, T("head.layers.%d.self_attn.out_proj.bias"), &h.outB, err, D) ||
          !upload_mat(W, T("head.layers.%d.linear1.weight"), FF, D, &h.l1W, err) ||
          !upload_vec(W, T("head.layers.%d.linear1.bias"), &h.l1B, err, FF) ||
          !upload_mat(W, T("head.layers.%d.linear2.weight"), D, FF, &h.l2W, err) ||
          !upload_vec(W, T("head.layers.%d.linear2.bias"), &h.l2B, err, D))
        return false;
    }
    if (!upload_vec(W, "scorer.0.weight", &sc_nw, err, D) || !upload_vec(W, "scorer.0.bias", &sc_nb, err, D) ||
        !upload_mat(W, "scorer.1.weight", D, D, &sc1, err) || !upload_vec(W, "scorer.1.bias", &sc1B, err, D) ||
        !upload_vec(W, "scorer.3.weight", &sc3W, err, D))
      return false;
    {
      std::vector<float> v;
      if (!W.to_f32("scorer.3.bias", &v, err)) return false;
      sc3B = v.at(0);
    }
    if (!upload_vec(W, "act_head.0.weight", &a0W, err, (size_t)256 * (D + 4)) ||
        !upload_vec(W, "act_head.0.bias", &a0B, err, 256) ||
        !upload_vec(W, "act_head.2.weight", &a2W, err, (size_t)cfg.n_act * 256) ||
        !upload_vec(W, "act_head.2.bias", &a2B, err, cfg.n_act))
      return false;
    if (!rope_tables(err)) return false;
    return alloc_arena(err);
  }

  // cos/sin [max_len, 32] per theta as transformers computes them: inv_freq = 1/theta^(2i/64) and
  // the angle pos*inv_freq in fp32, then cos/sin of that fp32 angle.
  bool rope_tables(std::string* err) {
    const int L = cfg.max_len, H2 = cfg.head_dim / 2;
    std::vector<float> cg((size_t)L * H2), sg(cg.size()), cl(cg.size()), sl(cg.size());
    for (int i = 0; i < H2; ++i) {
      const float e = static_cast<float>(2 * i) / static_cast<float>(cfg.head_dim);
      const float ig = 1.0f / static_cast<float>(std::pow((double)cfg.rope_theta_global, (double)e));
      const float il = 1.0f / static_cast<float>(std::pow((double)cfg.rope_theta_local, (double)e));
      for (int p = 0; p < L; ++p) {
        const float fg = static_cast<float>(p) * ig, fl = static_cast<float>(p) * il;
        cg[(size_t)p * H2 + i] = static_cast<float>(std::cos((double)fg));
        sg[(size_t)p * H2 + i] = static_cast<float>(std::sin((double)fg));
        cl[(size_t)p * H2 + i] = static_cast<float>(std::cos((double)fl));
        sl[(size_t)p * H2 + i] = static_cast<float>(std::sin((double)fl));
      }
    }
    for (auto pr : {std::make_pair(&cos_g, &cg), std::make_pair(&sin_g, &sg), std::make_pair(&cos_l, &cl),
                    std::make_pair(&sin_l, &sl)}) {
      if (!dalloc(pr.first, pr.second->size() * 4, err)) return false;
      LAYA_TRY(cudaMemcpy(*pr.first, pr.second->data(), pr.second->size() * 4, cudaMemcpyHostToDevice));
    }
    return true;
  }

  bool alloc_arena(std::string* err) {
    const int D = cfg.d, I = cfg.intermediate, FF = cfg.head_ffn;
    Tcap = (E.max_tokens + 63) / 64 * 64;
    Rcap = E.max_gathered;
    Bcap = E.max_seqs;
    if (!dalloc(&x, (size_t)Tcap * D * 4, err)) return false;
    const size_t qkv_bytes = (size_t)Tcap * 3 * D * (P == 2 ? 4 : 2);
    if (!dalloc(reinterpret_cast<char**>(&qkv), qkv_bytes, err)) return false;
    // Rows beyond a pass's valid rows are read as masked keys by the tcgen05 attention (p = 0):
    // they must hold finite values; dalloc zeroes every buffer, and later passes only ever leave
    // finite GEMM results there.
    attn_tc = P == 1 && !(getenv("LAYA_ATTN_MMA_SYNC") && atoi(getenv("LAYA_ATTN_MMA_SYNC")) != 0);
    attn_small = env_int("LAYA_ATTN_SMALL", 1) != 0;
    if (attn_tc && (!make_operand_map(&qkv_map, qkv, 3 * (uint64_t)D, Tcap, 1, 128) ||
                    !make_operand_map(&qkv_map64, qkv, 3 * (uint64_t)D, Tcap, 1, 64))) {
      *err = "qkv tensor map rejected";
      return false;
    }
    if (!make_operand(&xn, Tcap, D, err) || !make_operand(&ao, Tcap, D, err) || !make_operand(&mg, Tcap, I, err) ||
        !make_operand(&ff, Tcap, FF, err) || !make_operand(&xng, Rcap, D, err) || !make_operand(&aog, Rcap, D, err) ||
        !make_operand(&ffg, Rcap, FF, err) || !make_operand(&xs, Rcap, D, err))
      return false;
    if (!dalloc(&xg, (size_t)Rcap * D * 4, err)) return false;
    if (!dalloc(reinterpret_cast<char**>(&hs), (size_t)Rcap * D * (P == 2 ? 4 : 2), err)) return false;
    const bool f32acts = P == 2;  // fp32 qkv / scorer hidden in parity mode
    if (!make_output_map(&out_qkv, qkv, f32acts, 3 * D, Tcap, 1) || !make_output_map(&out_mg, mg.p, false, I, Tcap, P) ||
        !make_output_map(&out_ff, ff.p, false, FF, Tcap, P) || !make_output_map(&out_ffg, ffg.p, false, FF, Rcap, P) ||
        !make_output_map(&out_x, x, true, D, Tcap, 1) || !make_output_map(&out_xg, xg, true, D, Rcap, 1) ||
        !make_output_map(&out_hs, hs, f32acts, D, Rcap, 1)) {
      *err = "output tensor map rejected";
      return false;
    }
    if (!dalloc(&d_logits, (size_t)Rcap * 4, err)) return false;
    if (!dalloc(&d_act, (size_t)Bcap * cfg.n_act * 4, err)) return false;
    if (!dalloc(&d_head_hid, (size_t)Bcap * 256 * 4, err)) return false;
    if (!dalloc(&d_head_cnt, (size_t)Bcap * 4, err)) return false;
    if (!dalloc(&d_err, 16, err)) return false;
    if (!dalloc(&d_attn_ticket, 16, err)) return false;
    // Split-K (LAYA_SPLITK=0 turns it off): when the 128 x 128 tiles of a GEMM cannot fill the
    // GPU (a few thousand rows at most: batch-1 and small calls), its K loop is cut into slices
    // whose partials a second kernel sums in order. 32 M floats (128 MB) cover every split count.
    use_splitk = !(getenv("LAYA_SPLITK") && atoi(getenv("LAYA_SPLITK")) == 0);
    split_ln = !(getenv("LAYA_SPLIT_LN") && atoi(getenv("LAYA_SPLIT_LN")) == 0);
    if (getenv("LAYA_SPLIT_LN_CREDIT")) split_ln_credit = atoi(getenv("LAYA_SPLIT_LN_CREDIT"));
    if (use_splitk) {
      ws_floats = kSplitWsFloats;
      if (!dalloc(&ws, ws_floats * 4, err)) return false;
    }
    const MetaLayout L = meta_layout(Tcap, Bcap, Rcap);
    meta_cap = L.total;
    if (!dalloc(&d_meta, meta_cap * 4, err)) return false;
    void* hp = nullptr;
    LAYA_TRY(cudaMallocHost(&hp, meta_cap * 4));
    host_allocs.push_back(hp);
    h_meta = static_cast<int*>(hp);
    LAYA_TRY(cudaMallocHost(&hp, ((size_t)Rcap + (size_t)Bcap * cfg.n_act + 4) * 4));
    host_allocs.push_back(hp);
    h_out = static_cast<float*>(hp);
    return true;
  }

  // ------------------------------------------------------------------ one pass
  // Fills the pinned staging block for pass `p` of `qs` (and checks it in debug bounds mode).
  bool pack_ok = true;
  void fill(const PassPlan& p, const Question* qs) {
    fill_pass_meta(p, qs, cfg.pad_id, h_meta);
    pack_ok = true;
    if (E.debug_bounds) {
      PackLimits lim{cfg.vocab, cfg.max_len, Tcap, Rcap, Bcap};
      const int bad = check_pass_meta(p, h_meta, lim);
      if (bad) {
        fprintf(stderr, "[laya] device %d: packing check %d failed for a pass of %d questions (debug bounds mode)\n",
                dev, bad, p.n);
        pack_ok = false;
      }
    }
#ifdef LAYA_DEBUG_BOUNDS
    // Test hook of debug-bounds builds only (LAYA_DEBUG_PLANT_ID=n at load): the next n passes get a
    // token id one past the vocabulary after the host check, so the embedding kernel's own bounds
    // check must catch it on the device (code 40). The row it would read lies inside the table's
    // allocation granule, so even a missing check could not fault.
    if (plant_id > 0) {
      --plant_id;
      h_meta[meta_layout(p.Tpad, p.n, p.R).ids + p.T - 1] = cfg.vocab;
    }
#endif
  }

  cudaError_t first_err = cudaSuccess;
  void chk(cudaError_t e) {
    if (e != cudaSuccess && first_err == cudaSuccess) first_err = e;
  }
  // kernel launches of the pass being enqueued, and cumulative I/O counters (laya_io_stats)
  int pass_launches = 0;
  long long n_launches = 0, n_h2d = 0, n_d2h = 0;
  std::map<std::tuple<int, int, int, int>, int> graph_launches;
  int staged_launches = 0;
  void launched(cudaError_t e) {
    chk(e);
    ++pass_launches;
  }
  void count_pass(const PassPlan& p, int launches) {
    n_launches += launches;
    n_h2d += (long long)meta_layout(p.Tpad, p.n, p.R).total * 4;
    n_d2h += (long long)p.KT * 4 + (long long)p.n * cfg.n_act * 4 + 4;
  }
  cudaEvent_t take_event() {
    if (ev_used == ev_pool.size()) {
      cudaEvent_t ev;
      cudaEventCreate(&ev);
      ev_pool.push_back(ev);
    }
    return ev_pool[ev_used++];
  }
  template <typename F>
  void stage(const char* name, F&& fn) {
    const bool timed = E.prof_on && !capturing;
    const bool graph_timed = capturing && capturing_prof;  // event-record nodes in the captured graph
    cudaEvent_t a = nullptr, b = nullptr;
    if (timed) {
      a = take_event();
      b = take_event();
      cudaEventRecord(a, st);
    } else if (graph_timed) {
      cudaEventCreate(&a);
      cudaEventCreate(&b);
      // external records become event-record nodes of the graph (a plain record inside a capture
      // only orders work within the capture)
      chk(cudaEventRecordWithFlags(a, st, cudaEventRecordExternal));
    }
    fn();
    if (timed) {
      cudaEventRecord(b, st);
      prof_pending.emplace_back(name, a, b);
    } else if (graph_timed) {
      chk(cudaEventRecordWithFlags(b, st, cudaEventRecordExternal));
      staged_prof_events.emplace_back(name, a, b);
    }
  }
  void drop_staged_profile() {
    if (staged_prof_graph) cudaGraphExecDestroy(staged_prof_graph);
    staged_prof_graph = nullptr;
    for (auto& t : staged_prof_events) {
      cudaEventDestroy(std::get<1>(t));
      cudaEventDestroy(std::get<2>(t));
    }
    staged_prof_events.clear();
  }
  // adds one timed launch of stage `name` to the profile table
  void prof_add(const char* name, float ms) {
    for (auto& kv : prof_acc)
      if (kv.first == name) {
        kv.second.first += ms;
        kv.second.second += 1;
        return;
      }
    prof_acc.push_back({name, {(double)ms, 1}});
  }
  void prof_collect() {
    for (auto& t : prof_pending) {
      float ms = 0.f;
      cudaEventElapsedTime(&ms, std::get<1>(t), std::get<2>(t));
      prof_add(std::get<0>(t), ms);
    }
    prof_pending.clear();
    ev_used = 0;
  }

  // out: the epilogue's output map; dst / dst_plane: the buffer it covers (for a split-K launch,
  // whose epilogue runs in a second kernel on plain pointers). ln_w: for a residual GEMM, the gain of
  // the LayerNorm that follows it into xn; when the GEMM runs split-K, its reduce kernel writes that
  // LayerNorm too and gemm() returns true (the caller then skips its LayerNorm launch).
  bool gemm(const Operand& A, int M, const Mat& W, const CUtensorMap& out, void* dst, long long dst_plane,
            GemmEpi ep, const float* ln_w = nullptr) {
    // a residual GEMM followed by a bias-free LayerNorm over at most 1024 columns: a split-K reduce
    // kernel can write that LayerNorm too
    const bool ln_fusable = ln_w && ep.kind == EPI_RESID && W.N % 256 == 0 && W.N <= 1024;
    const GemmPlan plan = gemm_plan(M, W.N, W.K, nseg, num_sms, pair_clusters, use_splitk, ws_floats,
                                    ln_fusable ? split_ln_credit : 0);
    const int bn = plan.bn;
    GemmShape sh{M, W.N, W.K, nseg};
    bool ln_fused = false;
    if (plan.splits > 1) {
      // too few 128 x 128 tiles to fill the GPU: the K loop in slices (deterministic partial sums)
      sh.splits = plan.splits;
      sh.ws = ws;
      sh.dst = dst;
      sh.dst_plane = dst_plane;
      if (ln_fusable && split_ln) {
        ep.ln_w = ln_w;
        ep.ln_eps = cfg.norm_eps;
        ep.ln_out = xn.p;
        ep.ln_plane = xn.plane;
        ep.ln_planes = P;
        ln_fused = true;
      }
    }
    launched(gemm_launch(A.map, bn == 256 ? W.m256 : W.m128, out, bn, sh, ep, d_err, num_sms, st));
    return ln_fused;
  }
  GemmEpi epi_store(int out_mode, const float* bias, int act) const {
    GemmEpi e;
    e.kind = EPI_STORE;
    e.out_mode = out_mode;
    e.bias = bias;
    e.act = act;
    return e;
  }
  GemmEpi epi_resid(const float* bias) const {
    GemmEpi e;
    e.kind = EPI_RESID;
    e.bias = bias;
    return e;
  }
  int act_mode() const { return P == 2 ? OUT_BF16X2 : OUT_BF16; }
  LnArgs ln_base(int rows) const {
    LnArgs a;
    a.rows = rows;
    a.D = cfg.d;
    a.eps = cfg.norm_eps;
    a.out_planes = P;
    a.err = d_err;
    return a;
  }
  // extents of the current pass for the debug bounds checks of the attention kernels
  int pass_rows = 0, pass_rows_out = 0, pass_seqs = 0;
  void attend(const AttnItem* items, int n_items, const int* soff, const int* slen, int window, void* out,
              long long out_plane, const int* gsrc, const int* gdst) {
    AttnArgs a;
    a.rows = pass_rows;
    a.rows_out = gsrc ? pass_rows_out : pass_rows;
    a.n_seq = pass_seqs;
    a.err = d_err;
    a.qkv = qkv;
    a.out = out;
    a.out_plane = out_plane;
    a.out_planes = P;
    a.items = items;
    a.n_items = n_items;
    a.soff = soff;
    a.slen = slen;
    a.gsrc = gsrc;
    a.gdst = gdst;
    a.gathered = gsrc != nullptr;
    a.H = cfg.d / 64;
    a.window = window;
    a.scale = 0.125f;  // 1/sqrt(64)
    launched(P == 2 ? attn_f32_launch(a, st) : attn_bf16_launch(a, st));
  }

  // Attention of every packed row into `ao`: the tcgen05 kernel over 128-row items in bf16 mode,
  // the mma.sync / fp32 kernels over 64-row items otherwise (parity mode, LAYA_ATTN_MMA_SYNC=1, or a
  // small pass). Small passes: the tcgen05 kernel's 128-row units x heads leave most SMs idle and each
  // unit is a serial chain over its keys, so the mma.sync kernel's 64-row items (one CTA each) finish
  // sooner. Measured on a B200 with 512-token sequences (sliding / global layers, µs per launch): 512
  // rows 9.3 / 12.8 tcgen05 against 5.8 / 10.6 mma.sync, 1024 rows 9.4 / 13.2 against 7.5 / 14.8,
  // 2048 rows 11.0 / 15.2 against 12.2 / 30.0; hence the mma.sync kernel for sliding layers up to
  // kAttnSmallSliding rows and for global layers up to kAttnSmallGlobal rows.
  static constexpr int kAttnSmallSliding = 1024, kAttnSmallGlobal = 512;
  void attend_rows(const AttnItem* items, int n_items, const AttnItem* items128, int n_items128, const int* soff,
                   const int* slen, int window) {
    const bool small = pass_rows <= (window > 0 ? kAttnSmallSliding : kAttnSmallGlobal) && attn_small;
    if (!attn_tc || small) {
      attend(items, n_items, soff, slen, window, ao.p, ao.plane, nullptr, nullptr);
      return;
    }
    AttnArgs a;
    a.rows = pass_rows;
    a.rows_out = pass_rows;
    a.n_seq = pass_seqs;
    a.err = d_err;
    a.qkv = qkv;
    a.out = ao.p;
    a.out_plane = ao.plane;
    a.out_planes = 1;
    a.items = items128;
    a.n_items = n_items128;
    a.soff = soff;
    a.slen = slen;
    a.gathered = 0;
    a.H = cfg.d / 64;
    a.window = window;
    a.scale = 0.125f;  // 1/sqrt(64)
    launched(attn_tc_launch(qkv_map, qkv_map64, a, d_attn_ticket, d_err, st));
  }

  bool dumping() const { return !E.dump_dir.empty() && !capturing && this == E.reps[0].get(); }
  void dump(const char* name, const float* src, int rows) {
    if (!dumping()) return;
    std::vector<float> h((size_t)rows * cfg.d);
    chk(cudaStreamSynchronize(st));
    chk(cudaMemcpy(h.data(), src, h.size() * 4, cudaMemcpyDeviceToHost));
    const std::string fn = E.dump_dir + "/" + name + ".bin";
    if (FILE* f = fopen(fn.c_str(), "wb")) {
      fwrite(h.data(), 4, h.size(), f);
      fclose(f);
    }
  }

  // Enqueues one pass on the stream: metadata upload (h2d), every kernel, result download (d2h).
  void enqueue(const PassPlan& p, bool h2d, bool d2h) {
    const int D = cfg.d, I = cfg.intermediate, FF = cfg.head_ffn, NL = cfg.n_layers, HL = cfg.head_layers;
    const int M = p.Tpad, R = p.R, KT = p.KT;
    const MetaLayout L = meta_layout(p.Tpad, p.n, p.R);
    const int* dm = d_meta;
    const int *ids = dm + L.ids, *pos = dm + L.pos, *rowseq = dm + L.rowseq, *soff = dm + L.soff,
              *slen = dm + L.slen, *qt = dm + L.qt, *nm = dm + L.nm, *moff = dm + L.moff, *gsrc = dm + L.gsrc,
              *gdst = dm + L.gdst, *grow = dm + L.grow;
    const AttnItem* items = reinterpret_cast<const AttnItem*>(dm + L.items);
    const AttnItem* items128 = reinterpret_cast<const AttnItem*>(dm + L.items128);
    const AttnItem* gitems = reinterpret_cast<const AttnItem*>(dm + L.gitems);
    const int qkv_mode = P == 2 ? OUT_F32 : OUT_BF16;
    pass_rows = M;
    pass_rows_out = R;
    pass_seqs = p.n;
    char nb[32];
    if (h2d) stage("h2d", [&] { chk(cudaMemcpyAsync(d_meta, h_meta, L.total * 4, cudaMemcpyHostToDevice, st)); });

    stage("embed_ln", [&] {
      LnArgs a = ln_base(M);
      a.src = tok_emb;
      a.ids = ids;
      a.src_rows = cfg.vocab;
      a.w = emb_norm;
      a.out_f32 = x;
      a.out_bf = xn.p;
      a.out_plane = xn.plane;
      a.w2 = enc[0].attn_norm;  // layer 0 of ModernBERT has no attn_norm (Identity)
      a.eps2 = cfg.norm_eps;
      launched(ln_launch(a, st));
    });
    dump("emb", x, p.T);
    for (int l = 0; l < NL; ++l) {
      const bool glob = cfg.layer_types[l] == AttnKind::Global;
      stage("gemm_qkv", [&] {
        GemmEpi e = epi_store(qkv_mode, nullptr, ACT_NONE);
        e.kind = EPI_ROPE;
        e.cos_t = glob ? cos_g : cos_l;
        e.sin_t = glob ? sin_g : sin_l;
        e.pos = pos;
        e.rope_cols = 2 * D;
        e.rope_rows = cfg.max_len;
        gemm(xn, M, enc[l].Wqkv, out_qkv, qkv, 0, e);
      });
      stage(glob ? "attn_global" : "attn_sliding", [&] {
        attend_rows(items, L.items_cap, items128, L.items128_cap, soff, slen, glob ? 0 : cfg.local_attention / 2);
      });
      bool mlp_ln_done = false;  // the MLP LayerNorm, fused into a split-K reduce
      stage("gemm_attn_out", [&] { mlp_ln_done = gemm(ao, M, enc[l].Wo, out_x, x, 0, epi_resid(nullptr), enc[l].mlp_norm); });
      if (!mlp_ln_done) stage("ln", [&] {
        LnArgs a = ln_base(M);
        a.src = x;
        a.w = enc[l].mlp_norm;
        a.out_bf = xn.p;
        a.out_plane = xn.plane;
        launched(ln_launch(a, st));
      });
      stage("gemm_mlp_in", [&] {
        GemmEpi e = epi_store(act_mode(), nullptr, ACT_NONE);
        e.kind = EPI_GEGLU;
        e.geglu_I = I;
        gemm(xn, M, enc[l].Wi, out_mg, mg.p, mg.plane, e);
      });
      bool ln_done = false;  // the next layer's attention LayerNorm, fused into a split-K reduce
      stage("gemm_mlp_out", [&] {
        ln_done = gemm(mg, M, enc[l].Wmo, out_x, x, 0, epi_resid(nullptr), l + 1 < NL ? enc[l + 1].attn_norm : nullptr);
      });
      snprintf(nb, sizeof nb, "enc%d", l);
      dump(nb, x, p.T);
      if (!ln_done) stage("ln", [&] {
        LnArgs a = ln_base(M);
        a.src = x;
        a.out_bf = xn.p;
        a.out_plane = xn.plane;
        if (l + 1 < NL) {
          a.w = enc[l + 1].attn_norm;
        } else {  // final norm + type embedding back into x, then the first head layer's norm1
          a.w = final_norm;
          a.type_emb = type_emb;
          a.qtype = qt;
          a.rowseq = rowseq;
          a.n_seq = p.n;
          a.out_f32 = x;
          a.w2 = head[0].n1w;
          a.b2 = head[0].n1b;
          a.eps2 = 1e-5f;  // nn.TransformerEncoderLayer default layer_norm_eps
        }
        launched(ln_launch(a, st));
      });
    }
    dump("final", x, p.T);
    for (int j = 0; j < HL; ++j) {
      const Head& h = head[j];
      const bool last = j == HL - 1;
      stage("head_gemm", [&] { gemm(xn, M, h.inW, out_qkv, qkv, 0, epi_store(qkv_mode, h.inB, ACT_NONE)); });
      if (!last) {
        stage("head_attn", [&] { attend_rows(items, L.items_cap, items128, L.items128_cap, soff, slen, 0); });
        stage("head_gemm", [&] { gemm(ao, M, h.outW, out_x, x, 0, epi_resid(h.outB)); });
        stage("head_ln", [&] {
          LnArgs a = ln_base(M);
          a.eps = 1e-5f;
          a.src = x;
          a.w = h.n2w;
          a.b = h.n2b;
          a.out_bf = xn.p;
          a.out_plane = xn.plane;
          launched(ln_launch(a, st));
        });
        stage("head_gemm", [&] { gemm(xn, M, h.l1W, out_ff, ff.p, ff.plane, epi_store(act_mode(), h.l1B, ACT_RELU)); });
        stage("head_gemm", [&] { gemm(ff, M, h.l2W, out_x, x, 0, epi_resid(h.l2B)); });
        stage("head_ln", [&] {
          LnArgs a = ln_base(M);
          a.eps = 1e-5f;
          a.src = x;
          a.w = head[j + 1].n1w;
          a.b = head[j + 1].n1b;
          a.out_bf = xn.p;
          a.out_plane = xn.plane;
          launched(ln_launch(a, st));
        });
        snprintf(nb, sizeof nb, "head%d", j);
        dump(nb, x, p.T);
      } else {
        // only the option-marker rows and the CLS rows are read after the last head layer
        stage("head_attn", [&] { attend(gitems, L.gitems_cap, soff, slen, 0, aog.p, aog.plane, gsrc, gdst); });
        stage("head_ln", [&] {
          LnArgs a = ln_base(R);
          a.src = x;
          a.gidx = grow;
          a.src_rows = M;
          a.out_f32 = xg;
          launched(ln_launch(a, st));
        });
        stage("head_gemm", [&] { gemm(aog, R, h.outW, out_xg, xg, 0, epi_resid(h.outB)); });
        stage("head_ln", [&] {
          LnArgs a = ln_base(R);
          a.eps = 1e-5f;
          a.src = xg;
          a.w = h.n2w;
          a.b = h.n2b;
          a.out_bf = xng.p;
          a.out_plane = xng.plane;
          launched(ln_launch(a, st));
        });
        stage("head_gemm", [&] { gemm(xng, R, h.l1W, out_ffg, ffg.p, ffg.plane, epi_store(act_mode(), h.l1B, ACT_RELU)); });
        stage("head_gemm", [&] { gemm(ffg, R, h.l2W, out_xg, xg, 0, epi_resid(h.l2B)); });
        snprintf(nb, sizeof nb, "head%d", j);
        dump(nb, xg, R);
      }
    }
    stage("scorer", [&] {
      LnArgs a = ln_base(KT);
      a.src = xg;
      a.w = sc_nw;
      a.b = sc_nb;
      a.eps = 1e-5f;
      a.out_bf = xs.p;
      a.out_plane = xs.plane;
      launched(ln_launch(a, st));
      gemm(xs, KT, sc1, out_hs, hs, 0, epi_store(P == 2 ? OUT_F32 : OUT_BF16, sc1B, ACT_GELU));
    });
    stage("head_out", [&] {
      HeadOutArgs a;
      a.B = p.n;
      a.D = D;
      a.n_act = cfg.n_act;
      a.hs = hs;
      a.hs_f32 = P == 2;
      a.w3 = sc3W;
      a.b3 = sc3B;
      a.cls = xg + (size_t)KT * D;
      a.moff = moff;
      a.nmark = nm;
      a.w0 = a0W;
      a.b0 = a0B;
      a.w2 = a2W;
      a.b2 = a2B;
      a.logits = d_logits;
      a.act = d_act;
      a.hid = d_head_hid;
      a.hid_count = d_head_cnt;
      a.n_logits = KT;
      a.err = d_err;
      launched(head_out_launch(a, st));
    });
    if (d2h) {
      stage("d2h", [&] {
        chk(cudaMemcpyAsync(h_out, d_logits, (size_t)KT * 4, cudaMemcpyDeviceToHost, st));
        chk(cudaMemcpyAsync(h_out + Rcap, d_act, (size_t)p.n * cfg.n_act * 4, cudaMemcpyDeviceToHost, st));
        chk(cudaMemcpyAsync(h_out + Rcap + (size_t)Bcap * cfg.n_act, d_err, 4, cudaMemcpyDeviceToHost, st));
      });
    }
  }

  // Runs one pass (graph replay when possible) and leaves its results in h_out. Returns 0 or -2.
  int execute(const PassPlan& p) {
    first_err = cudaSuccess;
    const bool graphs_ok = E.use_graphs && !E.prof_on && E.dump_dir.empty();
    const auto key = std::make_tuple(p.Tpad, p.n, p.R, p.KT);
    bool done = false;
    if (graphs_ok) {
      auto it = graphs.find(key);
      if (it == graphs.end() && graphs.size() < 512) {
        cudaGraph_t g = nullptr;
        cudaGraphExec_t ex = nullptr;
        if (cudaStreamBeginCapture(st, cudaStreamCaptureModeThreadLocal) == cudaSuccess) {
          capturing = true;
          pass_launches = 0;
          enqueue(p, true, true);
          capturing = false;
          const cudaError_t ce = cudaStreamEndCapture(st, &g);
          if (ce == cudaSuccess && first_err == cudaSuccess && cudaGraphInstantiate(&ex, g, 0) == cudaSuccess) {
            it = graphs.emplace(key, ex).first;
            graph_launches[key] = pass_launches;
          } else {
            fprintf(stderr, "[laya] graph capture failed (%s); continuing without graphs\n",
                    cudaGetErrorString(first_err != cudaSuccess ? first_err : ce));
            (void)cudaGetLastError();
            E.use_graphs = false;
            first_err = cudaSuccess;
          }
          if (g) cudaGraphDestroy(g);
        }
      }
      if (it != graphs.end()) {
        chk(cudaGraphLaunch(it->second, st));
        count_pass(p, graph_launches[key]);
        done = true;
      }
    }
    if (!done) {
      pass_launches = 0;
      enqueue(p, true, true);
      count_pass(p, pass_launches);
    }
    chk(cudaStreamSynchronize(st));
    if (E.prof_on) prof_collect();
    int* herr = reinterpret_cast<int*>(h_out + Rcap + (size_t)Bcap * cfg.n_act);
    if (first_err != cudaSuccess || *herr != 0) {
      fprintf(stderr, "[laya] device %d: pass failed (%s, kernel code %d)\n", dev, cudaGetErrorString(first_err),
              *herr);
      if (*herr) {
        int zero = 0;
        cudaMemcpy(d_err, &zero, 4, cudaMemcpyHostToDevice);
        *herr = 0;
        // an aborted attention launch can leave its work / exit counters part-way: clear them
        if (d_attn_ticket) cudaMemset(d_attn_ticket, 0, 16);
      }
      (void)cudaGetLastError();
      return -2;
    }
    return 0;
  }

  void scatter(const PassPlan& p, const Question* qs) {
    const MetaLayout L = meta_layout(p.Tpad, p.n, p.R);
    for (int i = 0; i < p.n; ++i) {
      const Question& q = qs[p.b0 + i];
      memcpy(q.logits, h_out + h_meta[L.moff + i], (size_t)q.nmark * 4);
      memcpy(q.act, h_out + Rcap + (size_t)i * cfg.n_act, (size_t)cfg.n_act * 4);
    }
  }

  // Runs every question of `qs` (this replica's shard) through as many passes as needed.
  int run(const std::vector<Question>& qs) {
    if (qs.empty()) return 0;
    if (fail_runs > 0) {
      --fail_runs;
      fprintf(stderr, "[laya] device %d: injected failure (LAYA_FAIL_REPLICA), nothing launched\n", dev);
      return -2;
    }
    if (cudaSetDevice(dev) != cudaSuccess) return -2;
    std::vector<int> lens(qs.size()), nms(qs.size());
    for (size_t i = 0; i < qs.size(); ++i) { lens[i] = qs[i].len; nms[i] = qs[i].nmark; }
    std::vector<PassPlan> plans;
    if (!plan_passes((int)qs.size(), lens.data(), nms.data(), E.pass_tokens, Bcap, Rcap, &plans)) return -1;
    for (const PassPlan& p : plans) {
      fill(p, qs.data());
      if (!pack_ok) return -3;
      const int rc = execute(p);
      if (rc) return rc;
      scatter(p, qs.data());
    }
    return 0;
  }

  // ------------------------------------------------------------------ benchmark staging
  int stage_batch(const std::vector<Question>& qs) {
    if (cudaSetDevice(dev) != cudaSuccess) return -2;
    staged = qs;
    if (staged_graph) { cudaGraphExecDestroy(staged_graph); staged_graph = nullptr; }
    drop_staged_profile();
    if (qs.empty()) return 0;
    std::vector<int> lens(qs.size()), nms(qs.size());
    for (size_t i = 0; i < qs.size(); ++i) { lens[i] = qs[i].len; nms[i] = qs[i].nmark; }
    std::vector<PassPlan> plans;
    if (!plan_passes((int)qs.size(), lens.data(), nms.data(), E.pass_tokens, Bcap, Rcap, &plans)) return -1;
    if (plans.size() != 1) return -3;  // the staged batch must be one pass
    staged_plan = plans[0];
    fill(staged_plan, staged.data());
    if (!pack_ok) return -3;
    first_err = cudaSuccess;
    chk(cudaMemcpyAsync(d_meta, h_meta, meta_layout(staged_plan.Tpad, staged_plan.n, staged_plan.R).total * 4,
                        cudaMemcpyHostToDevice, st));
    chk(cudaStreamSynchronize(st));
    cudaGraph_t g = nullptr;
    if (cudaStreamBeginCapture(st, cudaStreamCaptureModeThreadLocal) != cudaSuccess) return -2;
    capturing = true;
    pass_launches = 0;
    enqueue(staged_plan, false, false);  // inputs stay resident in HBM; outputs stay on the device
    staged_launches = pass_launches;
    capturing = false;
    if (cudaStreamEndCapture(st, &g) != cudaSuccess || first_err != cudaSuccess) return -2;
    const cudaError_t ie = cudaGraphInstantiate(&staged_graph, g, 0);
    cudaGraphDestroy(g);
    return ie == cudaSuccess ? 0 : -2;
  }
  int replay(int iters, double* ms) {
    *ms = 0.0;
    if (staged.empty()) return 0;
    if (!staged_graph) return -4;
    if (cudaSetDevice(dev) != cudaSuccess) return -2;
    // a forward call since staging may have reused the metadata buffers: upload the staged pass again
    fill(staged_plan, staged.data());
    if (cudaMemcpy(d_meta, h_meta, meta_layout(staged_plan.Tpad, staged_plan.n, staged_plan.R).total * 4,
                   cudaMemcpyHostToDevice) != cudaSuccess)
      return -2;
    cudaEvent_t a, b;
    cudaEventCreate(&a);
    cudaEventCreate(&b);
    first_err = cudaSuccess;
    chk(cudaEventRecord(a, st));
    for (int i = 0; i < iters; ++i) chk(cudaGraphLaunch(staged_graph, st));
    n_launches += (long long)iters * staged_launches;
    chk(cudaEventRecord(b, st));
    chk(cudaEventSynchronize(b));
    float f = 0.f;
    cudaEventElapsedTime(&f, a, b);
    cudaEventDestroy(a);
    cudaEventDestroy(b);
    *ms = f;
    int herr = 0;
    cudaMemcpy(&herr, d_err, 4, cudaMemcpyDeviceToHost);
    return first_err == cudaSuccess && herr == 0 ? 0 : -2;
  }
  // Replays the staged pass `iters` times back to back as a graph that also records an event pair
  // around every stage, then adds the last replay's stage times to the profile table (prof_acc).
  int replay_profiled(int iters) {
    if (staged.empty() || iters < 1) return 0;
    if (!staged_graph) return -4;
    if (cudaSetDevice(dev) != cudaSuccess) return -2;
    first_err = cudaSuccess;
    if (!staged_prof_graph) {
      cudaGraph_t g = nullptr;
      if (cudaStreamBeginCapture(st, cudaStreamCaptureModeThreadLocal) != cudaSuccess) return -2;
      capturing = true;
      capturing_prof = true;
      enqueue(staged_plan, false, false);
      capturing = false;
      capturing_prof = false;
      if (cudaStreamEndCapture(st, &g) != cudaSuccess || first_err != cudaSuccess) {
        if (g) cudaGraphDestroy(g);
        drop_staged_profile();
        return -2;
      }
      const cudaError_t ie = cudaGraphInstantiate(&staged_prof_graph, g, 0);
      cudaGraphDestroy(g);
      if (ie != cudaSuccess) {
        staged_prof_graph = nullptr;
        drop_staged_profile();
        return -2;
      }
    }
    fill(staged_plan, staged.data());
    if (cudaMemcpy(d_meta, h_meta, meta_layout(staged_plan.Tpad, staged_plan.n, staged_plan.R).total * 4,
                   cudaMemcpyHostToDevice) != cudaSuccess)
      return -2;
    for (int i = 0; i < iters; ++i) chk(cudaGraphLaunch(staged_prof_graph, st));
    n_launches += (long long)iters * staged_launches;
    chk(cudaStreamSynchronize(st));
    if (first_err != cudaSuccess) return -2;
    for (auto& t : staged_prof_events) {
      float ms = 0.f;
      if (cudaEventElapsedTime(&ms, std::get<1>(t), std::get<2>(t)) != cudaSuccess) return -2;
      prof_add(std::get<0>(t), ms);
    }
    int herr = 0;
    cudaMemcpy(&herr, d_err, 4, cudaMemcpyDeviceToHost);
    return herr == 0 ? 0 : -2;
  }
  int staged_results() {
    if (staged.empty()) return 0;
    if (cudaSetDevice(dev) != cudaSuccess) return -2;
    const PassPlan& p = staged_plan;
    fill(p, staged.data());
    if (cudaMemcpy(h_out, d_logits, (size_t)p.KT * 4, cudaMemcpyDeviceToHost) != cudaSuccess ||
        cudaMemcpy(h_out + Rcap, d_act, (size_t)p.n * cfg.n_act * 4, cudaMemcpyDeviceToHost) != cudaSuccess)
      return -2;
    scatter(p, staged.data());
    return 0;
  }
};

// ===================================================================== Engine
Engine::Engine() = default;
Engine::~Engine() {
  reps.clear();
  workers.clear();
}

bool Engine::load(const std::string& dir, int prec, const std::string& devices, std::string* err) {
  try {
    cfg = Config::load(dir + "/encoder/config.json", dir + "/rl_agent_config.json");
  } catch (const std::exception& e) {
    *err = e.what();
    return false;
  }
  precision = prec;
  if (const char* p = getenv("LAYA_PRECISION")) {
    if (prec == 0 && (!strcmp(p, "fp32parity") || !strcmp(p, "fp32") || !strcmp(p, "1"))) precision = 1;
  }
  if (cfg.head_dim != 64 || cfg.d % 128 != 0 || cfg.d > 1024 || cfg.intermediate % 64 != 0 || cfg.head_layers < 1 ||
      cfg.n_act < 1 || cfg.n_act > 256 || cfg.max_len < 1) {
    *err = "unsupported model shape (needs head_dim 64, d a multiple of 128 up to 1024, intermediate a multiple of "
           "64, 1+ head layers, 1..256 act outputs)";
    return false;
  }
  if (getenv("LAYA_VERBOSE")) cfg.dump();
  max_tokens = std::max(env_int("LAYA_MAX_TOKENS", 131072), cfg.max_len);
  pass_tokens = std::min(std::max(env_int("LAYA_PASS_TOKENS", max_tokens), cfg.max_len), max_tokens);
  max_seqs = std::max(env_int("LAYA_MAX_SEQS", 4096), 1);
  max_gathered = std::max(max_tokens / 4, 2 * (kMaxMarkers + 1));
  use_graphs = env_int("LAYA_GRAPHS", 1) != 0;
  prof_on = getenv("LAYA_PROFILE") != nullptr;
  if (const char* d = getenv("LAYA_DUMP_DIR")) dump_dir = d;

  std::vector<int> devs;
  std::string list = devices;
  if (list.empty() && getenv("LAYA_DEVICES")) list = getenv("LAYA_DEVICES");
  for (size_t i = 0; i < list.size();) {
    size_t j = list.find(',', i);
    if (j == std::string::npos) j = list.size();
    if (j > i) devs.push_back(atoi(list.substr(i, j - i).c_str()));
    i = j + 1;
  }
  if (devs.empty()) {
    int d = 0;
    if (cudaGetDevice(&d) != cudaSuccess) { *err = "no CUDA device"; return false; }
    devs.push_back(d);
  }
  int ndev = 0;
  if (cudaGetDeviceCount(&ndev) != cudaSuccess || ndev == 0) { *err = "no CUDA device"; return false; }
  for (int d : devs)
    if (d < 0 || d >= ndev) { *err = "bad device ordinal in device list"; return false; }

  SafeTensors W;
  if (!W.open(dir + "/model.safetensors", err)) return false;
  int prev = 0;
  cudaGetDevice(&prev);
  std::vector<std::string> errs(devs.size());
  std::vector<int> ok(devs.size(), 0);
  for (int d : devs) reps.emplace_back(new Replica(*this, d));
  workers.resize(devs.size());
  for (size_t i = 1; i < devs.size(); ++i) workers[i].reset(new Worker());
  each_replica([&](size_t i) {
    ok[i] = reps[i]->load(W, &errs[i]) ? 1 : 0;
    return 0;
  });
  cudaSetDevice(prev);
  for (size_t i = 0; i < devs.size(); ++i)
    if (!ok[i]) { *err = "device " + std::to_string(devs[i]) + ": " + errs[i]; return false; }
  debug_bounds = kDebugBoundsBuild || env_int("LAYA_DEBUG_BOUNDS", 0) != 0;
  if (kDebugBoundsBuild)
    for (auto& r : reps) r->plant_id = env_int("LAYA_DEBUG_PLANT_ID", 0);
  if (const char* f = getenv("LAYA_FAIL_REPLICA")) {
    const int i = atoi(f);
    const char* c = strchr(f, ':');
    if (i >= 0 && i < (int)reps.size()) reps[i]->fail_runs = c ? atoi(c + 1) : 1;
  }
  if (getenv("LAYA_VERBOSE"))
    printf("[laya] ready: %zu device(s) max_tokens/pass=%d graphs=%d precision=%s\n", reps.size(), pass_tokens,
           (int)use_graphs, precision ? "fp32parity" : "bf16");
  return true;
}

// ===================================================================== workers
Worker::Worker() : th_([this] { loop(); }) {}

Worker::~Worker() {
  {
    std::lock_guard<std::mutex> lk(mu_);
    stop_ = true;
  }
  cv_.notify_all();
  th_.join();
}

void Worker::post(std::function<int()> job) {
  {
    std::lock_guard<std::mutex> lk(mu_);
    job_ = std::move(job);
    has_job_ = true;
    done_ = false;
  }
  cv_.notify_all();
}

int Worker::wait() {
  std::unique_lock<std::mutex> lk(mu_);
  cv_.wait(lk, [&] { return done_; });
  done_ = false;
  return rc_;
}

void Worker::loop() {
  std::unique_lock<std::mutex> lk(mu_);
  for (;;) {
    cv_.wait(lk, [&] { return has_job_ || stop_; });
    if (!has_job_) return;  // stop, nothing pending
    std::function<int()> job = std::move(job_);
    has_job_ = false;
    lk.unlock();
    int rc;
    try {
      rc = job();
    } catch (...) {
      rc = -2;
    }
    lk.lock();
    rc_ = rc;
    done_ = true;
    cv_.notify_all();
  }
}

int Engine::each_replica(const std::function<int(size_t)>& fn) {
  const size_t G = reps.size();
  for (size_t i = 1; i < G; ++i) workers[i]->post([&fn, i] { return fn(i); });
  std::vector<int> rc(G, 0);
  try {
    rc[0] = fn(0);
  } catch (...) {
    rc[0] = -2;
  }
  for (size_t i = 1; i < G; ++i) rc[i] = workers[i]->wait();  // every worker finishes before the call returns
  for (int r : rc)
    if (r) return r;
  return 0;
}

// ===================================================================== request sharding
ShardModel shard_model(const Config& c) {
  ShardModel m;
  m.d = c.d;
  m.intermediate = c.intermediate;
  m.head_ffn = c.head_ffn > 0 ? c.head_ffn : 4LL * c.d;
  m.n_layers = c.n_layers;
  m.n_global = 0;
  for (int l = 0; l < c.n_layers && l < (int)c.layer_types.size(); ++l)
    if (c.layer_types[l] == AttnKind::Global) ++m.n_global;
  m.window = c.local_attention;
  return m;
}

long long question_cost(const ShardModel& m, int L, int k) {
  const long long D = m.d, I = m.intermediate, FF = m.head_ffn, NL = m.n_layers, ng = m.n_global;
  const long long ns = NL - ng, h = m.window / 2, l = L, kk = k;
  // keys inside |q - key| <= h summed over the queries of one sequence:
  // sum_q min(L-1, q+h) - max(0, q-h) + 1, in closed form
  const long long t = l > h ? l - h : 0, u = l - 1 - h > 0 ? l - 1 - h : 0;
  const long long band = t * (t - 1) / 2 + t * h + (l - t) * (l - 1) - u * (u + 1) / 2 + l;
  const long long gemm = 2 * l * (4 * D * D + 3 * I * D) * NL     // encoder: QKV, out, MLP-in (2I), MLP-out
                         + 2 * l * (4 * D * D + 2 * D * FF)       // head layer 0 on every row
                         + 2 * l * 3 * D * D                      // head layer 1: K, V (and Q) of every row
                         + 2 * (kk + 1) * (D * D + 2 * D * FF)    // head layer 1 on the gathered rows
                         + 2 * kk * D * D;                        // scorer
  const long long glob = 4 * D * l * l * (ng + 1)                 // global layers and head layer 0
                         + 4 * D * l * (kk + 1);                  // head layer 1, gathered queries
  const long long slide = 4 * D * ns * band;
  return 4 * gemm + 14 * glob + 26 * slide;
}

void shard_owners(int B, const int* lens, const int* nmark, int G, const ShardModel& m, int* owner) {
  std::vector<long long> cost(B);
  for (int b = 0; b < B; ++b) cost[b] = question_cost(m, lens[b], nmark[b]);
  std::vector<int> order(B);
  std::iota(order.begin(), order.end(), 0);
  std::stable_sort(order.begin(), order.end(), [&](int a, int b) { return cost[a] > cost[b]; });
  std::vector<long long> load(G, 0);
  for (int b : order) {
    const int g = (int)(std::min_element(load.begin(), load.end()) - load.begin());
    owner[b] = g;
    load[g] += cost[b];
  }
}

// Questions of each replica for one call (shard_owners), in input order inside each shard.
std::vector<std::vector<Question>> Engine::shard(int B, const int* lens, const int* ids, const int* nmark,
                                                 const int* markers, const int* qtypes, float* logits, float* act) {
  const int G = (int)reps.size();
  std::vector<Question> all(B);
  size_t io = 0, mo = 0;
  for (int b = 0; b < B; ++b) {
    all[b] = Question{lens[b], nmark[b], qtypes[b], ids + io, markers + mo, logits + mo, act + (size_t)b * cfg.n_act};
    io += lens[b];
    mo += nmark[b];
  }
  std::vector<std::vector<Question>> out(G);
  if (G == 1) {
    out[0] = std::move(all);
    return out;
  }
  std::vector<int> owner(B);
  shard_owners(B, lens, nmark, G, shard_model(cfg), owner.data());
  for (int b = 0; b < B; ++b) out[owner[b]].push_back(all[b]);
  return out;
}

bool validate_tokens(int B, const int* lens, const int* ids, const int* qtypes, int vocab) {
  size_t nt = 0;
  for (int b = 0; b < B; ++b) {
    if (qtypes[b] < 0 || qtypes[b] > 2) return false;
    nt += lens[b];
  }
  for (size_t t = 0; t < nt; ++t)
    if (ids[t] < 0 || ids[t] >= vocab) return false;
  return true;
}

int Engine::forward_batch(int B, const int* lens, const int* ids, const int* nmark, const int* markers,
                          const int* qtypes, float* logits, float* act) {
  if (!validate_batch(B, lens, nmark, markers, cfg.max_len)) return -1;
  if (!validate_tokens(B, lens, ids, qtypes, cfg.vocab)) return -1;
  if (B == 0) return 0;
  auto shards = shard(B, lens, ids, nmark, markers, qtypes, logits, act);
  if (reps.size() == 1) return reps[0]->run(shards[0]);
  return each_replica([&](size_t i) { return reps[i]->run(shards[i]); });
}

int Engine::stage(int B, const int* lens, const int* ids, const int* nmark, const int* markers, const int* qtypes) {
  if (!validate_batch(B, lens, nmark, markers, cfg.max_len)) return -1;
  if (!validate_tokens(B, lens, ids, qtypes, cfg.vocab)) return -1;
  // keep private copies: the staged pass replays them
  size_t nt = 0, nk = 0;
  for (int b = 0; b < B; ++b) { nt += lens[b]; nk += nmark[b]; }
  st_lens_.assign(lens, lens + B);
  st_ids_.assign(ids, ids + nt);
  st_nmark_.assign(nmark, nmark + B);
  st_markers_.assign(markers, markers + nk);
  st_qt_.assign(qtypes, qtypes + B);
  st_B_ = B;
  static thread_local std::vector<float> sink;
  sink.assign(nk + (size_t)B * cfg.n_act + 1, 0.f);
  auto shards = shard(B, st_lens_.data(), st_ids_.data(), st_nmark_.data(), st_markers_.data(), st_qt_.data(),
                      sink.data(), sink.data() + nk);
  return each_replica([&](size_t i) { return reps[i]->stage_batch(shards[i]); });
}

int Engine::replay(int iters, double* ms) {
  std::vector<double> t(reps.size(), 0.0);
  const int rc = each_replica([&](size_t i) { return reps[i]->replay(iters, &t[i]); });
  *ms = *std::max_element(t.begin(), t.end());
  return rc;
}

int Engine::replay_profiled(int iters) {
  return each_replica([&](size_t i) { return reps[i]->replay_profiled(iters); });
}

int Engine::staged_results(float* logits, float* act) {
  if (st_B_ == 0) return 0;
  auto shards = shard(st_B_, st_lens_.data(), st_ids_.data(), st_nmark_.data(), st_markers_.data(), st_qt_.data(),
                      logits, act);
  for (size_t i = 0; i < reps.size(); ++i) {
    reps[i]->staged = shards[i];
    const int r = reps[i]->staged_results();
    if (r) return r;
  }
  return 0;
}

void Engine::prof_report(int iters) {
  std::vector<std::pair<std::string, std::pair<double, long long>>> acc;
  for (auto& r : reps)
    for (auto& kv : r->prof_acc) {
      bool f = false;
      for (auto& a : acc)
        if (a.first == kv.first) { a.second.first += kv.second.first; a.second.second += kv.second.second; f = true; }
      if (!f) acc.push_back(kv);
    }
  if (acc.empty()) return;
  double tot = 0;
  for (auto& kv : acc) tot += kv.second.first;
  std::sort(acc.begin(), acc.end(), [](auto& a, auto& b) { return a.second.first > b.second.first; });
  iters = iters > 0 ? iters : 1;
  printf("\n%-18s %9s %7s %9s\n", "stage", "ms/fwd", "%", "launches");
  for (auto& kv : acc)
    printf("%-18s %9.3f %6.1f%% %9lld\n", kv.first.c_str(), kv.second.first / iters, 100 * kv.second.first / tot,
           kv.second.second);
  printf("%-18s %9.3f (device time, stages back to back)\n", "TOTAL", tot / iters);
}

void Engine::prof_reset() {
  for (auto& r : reps) r->prof_acc.clear();
}

int Engine::prof_get(const std::string& name, double* ms, long long* launches) {
  double m = 0;
  long long n = 0;
  bool found = false;
  for (auto& r : reps)
    for (auto& kv : r->prof_acc)
      if (kv.first == name) { m += kv.second.first; n += kv.second.second; found = true; }
  if (ms) *ms = m;
  if (launches) *launches = n;
  return found ? 0 : -1;
}

void Engine::io_stats(long long* launches, long long* h2d, long long* d2h, bool reset) {
  long long a = 0, b = 0, c = 0;
  for (auto& r : reps) {
    a += r->n_launches;
    b += r->n_h2d;
    c += r->n_d2h;
    if (reset) r->n_launches = r->n_h2d = r->n_d2h = 0;
  }
  if (launches) *launches = a;
  if (h2d) *h2d = b;
  if (d2h) *d2h = c;
}

void Engine::tune_all() {
  // The GEMM tile width is chosen per launch from the tile count (pick_bn); nothing to pre-tune.
}

}  // namespace laya
