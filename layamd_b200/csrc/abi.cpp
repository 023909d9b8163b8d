// C ABI of the engine (declared in include/laya_api.h). The first ten functions keep the reference's
// names, signatures and return contract (src/engine.hip:543-559).
#include <algorithm>
#include <cstdio>
#include <cstring>
#include <string>
#include <vector>

#include "engine.hpp"
#include "kernels.h"
#include "laya_api.h"

using laya::Engine;

namespace {
Engine* E(void* h) { return static_cast<Engine*>(h); }

void* create(const char* dir, int precision, const char* devices) {
  if (!dir) return nullptr;
  Engine* e = new Engine();
  std::string err;
  if (!e->load(dir, precision, devices ? devices : "", &err)) {
    fprintf(stderr, "[laya] load failed: %s\n", err.c_str());
    delete e;
    return nullptr;
  }
  return e;
}
}  // namespace

extern "C" {

void* laya_create(const char* dir) { return create(dir, 0, nullptr); }

void* laya_create_ex(const char* dir, int precision, const char* devices) {
  return create(dir, precision == 1 ? 1 : 0, devices);
}

void laya_destroy(void* h) { delete E(h); }

int laya_forward_batch(void* h, int B, const int* lens, const int* ids, const int* nmark, const int* markers,
                       const int* qtypes, float* logits, float* act) {
  if (!h || B < 0 || (B > 0 && (!lens || !ids || !nmark || !markers || !qtypes || !logits || !act))) return -1;
  return E(h)->forward_batch(B, lens, ids, nmark, markers, qtypes, logits, act);
}

void laya_forward(void* h, const int* ids, int S, int valid_len, const int* markers, int K, int qtype, float* logits,
                  float* act) {
  (void)S;
  if (!h) return;
  (void)E(h)->forward_batch(1, &valid_len, ids, &K, markers, &qtype, logits, act);
}

int laya_n_act(void* h) { return h ? E(h)->cfg.n_act : 0; }
int laya_max_len(void* h) { return h ? E(h)->cfg.max_len : 0; }
int laya_max_markers(void* h) {
  (void)h;
  return laya::kMaxMarkers;
}
float laya_temperature(void* h, int qtype) {
  if (!h || qtype < 0 || qtype >= (int)E(h)->cfg.temperature.size()) return 1.0f;
  return E(h)->cfg.temperature[qtype];
}
void laya_prof_report(void* h, int iters) {
  if (h) E(h)->prof_report(iters);
}
void laya_prof_reset(void* h) {
  if (h) E(h)->prof_reset();
}
void laya_tune_all(void* h) {
  if (h) E(h)->tune_all();
}
int laya_num_devices(void* h) { return h ? (int)E(h)->reps.size() : 0; }
void laya_prof_enable(void* h, int on) {
  if (h) E(h)->prof_on = on != 0;
}
int laya_prof_get(void* h, const char* name, double* ms, long long* launches) {
  if (!h || !name) return -1;
  return E(h)->prof_get(name, ms, launches);
}

int laya_plan_passes_cfg(int max_len, int pass_tokens, int max_seqs, int B, const int* lens, const int* nmark,
                         const int* markers, int cap, int* pass_first, int* pass_count, int* pass_rows) {
  if (!laya::validate_batch(B, lens, nmark, markers, max_len)) return -1;
  std::vector<laya::PassPlan> plans;
  const int max_gathered = std::max(pass_tokens / 4, 2 * (laya::kMaxMarkers + 1));
  if (!laya::plan_passes(B, lens, nmark, std::max(pass_tokens, max_len), std::max(max_seqs, 1), max_gathered, &plans))
    return -1;
  for (int i = 0; i < (int)plans.size() && i < cap; ++i) {
    if (pass_first) pass_first[i] = plans[i].b0;
    if (pass_count) pass_count[i] = plans[i].n;
    if (pass_rows) pass_rows[i] = plans[i].T;
  }
  return (int)plans.size();
}

int laya_plan_passes(void* h, int B, const int* lens, const int* nmark, const int* markers, int cap, int* pass_first,
                     int* pass_count, int* pass_rows) {
  if (!h) return -1;
  Engine* e = E(h);
  if (!laya::validate_batch(B, lens, nmark, markers, e->cfg.max_len)) return -1;
  std::vector<laya::PassPlan> plans;
  if (!laya::plan_passes(B, lens, nmark, e->pass_tokens, e->max_seqs, e->max_gathered, &plans)) return -1;
  for (int i = 0; i < (int)plans.size() && i < cap; ++i) {
    if (pass_first) pass_first[i] = plans[i].b0;
    if (pass_count) pass_count[i] = plans[i].n;
    if (pass_rows) pass_rows[i] = plans[i].T;
  }
  return (int)plans.size();
}

int laya_pack_check(int max_len, int vocab, int pad_id, int pass_tokens, int max_seqs, int B, const int* lens,
                    const int* ids, const int* nmark, const int* markers, const int* qtypes, int corrupt) {
  if (B < 0 || (B > 0 && (!lens || !ids || !nmark || !markers || !qtypes)) || vocab <= 0 || max_len <= 0 ||
      pad_id < 0 || pad_id >= vocab)
    return -1;
  if (!laya::validate_batch(B, lens, nmark, markers, max_len)) return -1;
  for (int b = 0; b < B; ++b)
    if (qtypes[b] < 0 || qtypes[b] > 2) return -1;
  size_t nt = 0;
  for (int b = 0; b < B; ++b) nt += lens[b];
  for (size_t t = 0; t < nt; ++t)
    if (ids[t] < 0 || ids[t] >= vocab) return -1;
  const int rows = std::max(pass_tokens, max_len);
  const int seqs = std::max(max_seqs, 1);
  const int gathered = std::max(rows / 4, 2 * (laya::kMaxMarkers + 1));
  std::vector<laya::PassPlan> plans;
  if (!laya::plan_passes(B, lens, nmark, rows, seqs, gathered, &plans)) return -1;
  std::vector<laya::Question> qs(B);
  size_t io = 0, mo = 0;
  for (int b = 0; b < B; ++b) {
    qs[b] = laya::Question{lens[b], nmark[b], qtypes[b], ids + io, markers + mo, nullptr, nullptr};
    io += lens[b];
    mo += nmark[b];
  }
  const laya::PackLimits lim{vocab, max_len, (rows + 63) / 64 * 64, gathered, seqs};
  std::vector<int> meta;
  for (size_t i = 0; i < plans.size(); ++i) {
    const laya::PassPlan& p = plans[i];
    meta.assign(laya::pass_meta_ints(p), 0);
    laya::fill_pass_meta(p, qs.data(), pad_id, meta.data());
    if (i == 0 && corrupt > 0) laya::corrupt_pass_meta(p, meta.data(), corrupt, vocab);
    const int bad = laya::check_pass_meta(p, meta.data(), lim);
    if (bad) return -100 - bad;
  }
  return static_cast<int>(plans.size());
}

int laya_debug_bounds_build(void) { return laya::kDebugBoundsBuild ? 1 : 0; }

int laya_shard_plan(int ndev, int B, const int* lens, const int* nmark, int d, int intermediate, int n_layers,
                    int n_global, int window, int* owner) {
  if (ndev < 1 || B < 0 || (B > 0 && (!lens || !nmark || !owner)) || d <= 0 || intermediate <= 0 || n_layers <= 0 ||
      n_global < 0 || n_global > n_layers || window < 0)
    return -1;
  laya::ShardModel m;
  m.d = d;
  m.intermediate = intermediate;
  m.head_ffn = 4LL * d;
  m.n_layers = n_layers;
  m.n_global = n_global;
  m.window = window;
  laya::shard_owners(B, lens, nmark, ndev, m, owner);
  return 0;
}

int laya_plan_gemm(int M, int N, int K, int parity, int num_sms, int pair_clusters, int ln_fusable, int* bn,
                   int* splits) {
  if (M <= 0 || N <= 0 || K <= 0 || num_sms <= 0 || pair_clusters < 0 || !bn || !splits) return -1;
  const laya::GemmPlan p = laya::gemm_plan(M, N, K, parity ? 3 : 1, num_sms, pair_clusters, true, laya::kSplitWsFloats,
                                           ln_fusable ? laya::kSplitLnCredit : 0);
  *bn = p.bn;
  *splits = p.splits;
  return 0;
}

int laya_stage(void* h, int B, const int* lens, const int* ids, const int* nmark, const int* markers,
               const int* qtypes) {
  if (!h || B < 0 || (B > 0 && (!lens || !ids || !nmark || !markers || !qtypes))) return -1;
  return E(h)->stage(B, lens, ids, nmark, markers, qtypes);
}

int laya_replay(void* h, int iters, double* ms) {
  if (!h || !ms || iters < 0) return -1;
  return E(h)->replay(iters, ms);
}

int laya_replay_profiled(void* h, int iters) {
  if (!h || iters < 0) return -1;
  return E(h)->replay_profiled(iters);
}

int laya_staged_results(void* h, float* logits, float* act) {
  if (!h || !logits || !act) return -1;
  return E(h)->staged_results(logits, act);
}

int laya_io_stats(void* h, long long* launches, long long* h2d_bytes, long long* d2h_bytes, int reset) {
  if (!h) return -1;
  E(h)->io_stats(launches, h2d_bytes, d2h_bytes, reset != 0);
  return 0;
}

int laya_set_dump_dir(void* h, const char* dir) {
  if (!h) return -1;
  E(h)->dump_dir = dir ? dir : "";
  return 0;
}

}  // extern "C"
