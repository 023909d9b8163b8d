// Laya B200 engine: host orchestration of one forward pass per packed batch of questions, on one
// replica per GPU. Restates the reference Engine (src/engine.hip:50-541) for sm_100a:
//   * weights uploaded once per device: bf16 GEMM operands in [out, in] (K-major) layout with TMA
//     descriptors (plus a second bf16 "lo" plane per matrix in fp32-parity mode), every vector
//     (LayerNorm gains, biases, embeddings, head weights) in fp32;
//   * a static arena sized for LAYA_MAX_TOKENS rows, so the request path never allocates;
//   * questions packed back to back with no per-sequence padding (row maps drive RoPE, attention
//     and the type embedding), a pass padded only to a multiple of 64 rows;
//   * per-pass metadata staged in one pinned host block and uploaded with one copy; each pass shape
//     (padded rows, questions, gathered rows) is captured once as a CUDA graph and replayed;
//   * with several devices, each forward call shards its questions across the replicas (longest
//     processing time first on the question length), each replica running the single-GPU path in
//     its own host thread; no collective.
#pragma once
#include <cuda.h>
#include <cuda_runtime.h>

#include <map>
#include <memory>
#include <string>
#include <tuple>
#include <vector>

#include "kernels.h"
#include "model_files.hpp"

namespace laya {

constexpr int kMaxMarkers = 255;  // options per question (the act head encodes the count as k/255)

// One pass of the packer: questions [b0, b0 + n) of the (per-replica) question list.
struct PassPlan {
  int b0 = 0, n = 0;
  int T = 0, Tpad = 0;  // packed rows, padded to 64
  int KT = 0, R = 0;    // marker rows, gathered rows (markers then one CLS row per question)
};

// Greedy in-order packing (src/engine.hip:497-505): add questions while the packed rows stay within
// pass_tokens, the pass holds at most max_seqs questions and at most max_gathered gathered rows.
// Returns false if a single question cannot fit.
bool plan_passes(int B, const int* lens, const int* nmark, int pass_tokens, int max_seqs, int max_gathered,
                 std::vector<PassPlan>* out);

// Validation of one forward call (src/engine.hip:492-496): every length in [1, max_len], every
// marker count in [1, 255], every marker inside its sequence.
bool validate_batch(int B, const int* lens, const int* nmark, const int* markers, int max_len);

// Replica of each question when a call is sharded over G replicas: longest question first onto the
// least-loaded replica (load = length + 64 per question); ties keep input order.
void shard_owners(int B, const int* lens, int G, int* owner);

struct Mat {  // a GEMM weight: planes x [N, K] bf16 with its TMA descriptors
  bf16* p = nullptr;
  int N = 0, K = 0;
  CUtensorMap m128, m256;
};

struct Operand {  // an activation used as GEMM A operand: planes x [rows, K] bf16
  bf16* p = nullptr;
  int rows = 0, K = 0;
  long long plane = 0;
  CUtensorMap map;
};

struct Question {  // one question of the caller's batch, by reference into the caller's arrays
  int len, nmark, qtype;
  const int* ids;
  const int* markers;
  float* logits;  // destination of its nmark logits
  float* act;     // destination of its n_act act logits
};

class Replica;

class Engine {
 public:
  Config cfg;
  int precision = 0;  // 0 bf16, 1 fp32 parity
  int max_tokens = 131072, pass_tokens = 131072, max_seqs = 4096, max_gathered = 0;
  bool use_graphs = true;
  bool prof_on = false;
  std::string dump_dir;
  std::vector<std::unique_ptr<Replica>> reps;

  Engine();
  ~Engine();
  bool load(const std::string& dir, int precision, const std::string& devices, std::string* err);
  int forward_batch(int B, const int* lens, const int* ids, const int* nmark, const int* markers, const int* qtypes,
                    float* logits, float* act);
  int stage(int B, const int* lens, const int* ids, const int* nmark, const int* markers, const int* qtypes);
  int replay(int iters, double* ms);
  int replay_profiled(int iters);
  int staged_results(float* logits, float* act);
  void prof_report(int iters);
  void prof_reset();
  int prof_get(const std::string& name, double* ms, long long* launches);
  void tune_all();
  // Cumulative kernel launches and host<->device bytes of the forward / replay calls on every
  // replica; reset clears them.
  void io_stats(long long* launches, long long* h2d, long long* d2h, bool reset);

 private:
  // staged batch for laya_stage / laya_replay
  std::vector<int> st_lens_, st_ids_, st_nmark_, st_markers_, st_qt_;
  int st_B_ = 0;
  std::vector<std::vector<Question>> shard(int B, const int* lens, const int* ids, const int* nmark,
                                           const int* markers, const int* qtypes, float* logits, float* act);
};

}  // namespace laya
