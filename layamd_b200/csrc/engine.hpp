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
//     processing time first on the question's modelled device time), each replica running the
//     single-GPU path on its own long-lived host thread; no collective.
#pragma once
#include <cuda.h>
#include <cuda_runtime.h>

#include <condition_variable>
#include <functional>
#include <map>
#include <memory>
#include <mutex>
#include <string>
#include <thread>
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

// Limits a pass's metadata must respect (the arena it is uploaded into and the model's tables).
struct PackLimits {
  int vocab, max_len;
  int max_rows, max_gathered, max_seqs;
};

// Ints of pass `p`'s metadata block.
size_t pass_meta_ints(const PassPlan& p);

// Test hook of laya_pack_check: breaks map number `which` (1-8: question offset, question type,
// marker count, token id, row -> question, 64-row item, gathered source row, gathered row) of a filled
// block, so that a test can show that check_pass_meta catches it. Host memory only.
void corrupt_pass_meta(const PassPlan& p, int* m, int which, int vocab);

// True in builds compiled with -DLAYA_DEBUG_BOUNDS (device-side index checks in every kernel).
#ifdef LAYA_DEBUG_BOUNDS
constexpr bool kDebugBoundsBuild = true;
#else
constexpr bool kDebugBoundsBuild = false;
#endif

// Model dimensions the shard cost model needs (a subset of Config, so host-only callers can pass
// them by value).
struct ShardModel {
  long long d = 1024, intermediate = 2624, head_ffn = 4096;
  int n_layers = 28, n_global = 10, window = 128;  // window: full width, |q - k| <= window / 2
};
ShardModel shard_model(const Config& c);

// Device cost of one question of length L with k options, in quarter-FLOPs at the encoder GEMMs' rate:
// the algorithmic FLOPs of the forward pass (every GEMM of the encoder and both head layers, the
// global and sliding attention, head-layer attention, the gathered rows of the last head layer and
// the scorer), each term weighted by how long a FLOP of that kind takes on a B200 relative to a GEMM
// FLOP. Measured on the C2 pass in bf16: GEMMs 1116 TFLOP/s, global attention 316, sliding attention
// 175, so the weights are 4 (GEMM), 14 (global / head attention) and 26 (sliding attention) per FLOP.
// Integer arithmetic, so that a restatement reproduces the assignment exactly.
long long question_cost(const ShardModel& m, int L, int k);

// Token ids inside [0, vocab) and question types 0..2 (an addition to the reference's validation,
// whose embedding gather would read outside its table for such an id).
bool validate_tokens(int B, const int* lens, const int* ids, const int* qtypes, int vocab);

// Replica of each question when a call is sharded over G replicas: longest processing time first
// (question_cost, descending; ties in input order) onto the least-loaded replica (lowest index on a
// tie). Each replica then runs its questions in input order.
void shard_owners(int B, const int* lens, const int* nmark, int G, const ShardModel& m, int* owner);

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

// Fills the per-pass metadata block (token ids, positions, row -> question map, per-question offsets,
// lengths, types and marker offsets, the three attention work-item lists and the gathered-row maps)
// for pass `p` of `qs` into `m` (meta_layout order).
void fill_pass_meta(const PassPlan& p, const Question* qs, int pad_id, int* m);

// Debug bounds mode, host side: checks every map of a filled metadata block against the pass and
// `lim` (ids inside the vocabulary, rows inside their question, work items covering every row once,
// gathered rows inside their question and the gathered buffer, ...). Returns 0, or the number of the
// first check that failed (1-13).
int check_pass_meta(const PassPlan& p, const int* m, const PackLimits& lim);

class Replica;

// A host thread that runs one job at a time for one replica, started at load and kept for the
// handle's life, so a sharded call costs a hand-off instead of a thread start per replica.
class Worker {
 public:
  Worker();
  ~Worker();
  Worker(const Worker&) = delete;
  Worker& operator=(const Worker&) = delete;
  void post(std::function<int()> job);  // the previous job must have been waited for
  int wait();                           // blocks until the posted job returns; its result
 private:
  void loop();
  std::mutex mu_;
  std::condition_variable cv_;
  std::function<int()> job_;
  bool has_job_ = false, done_ = false, stop_ = false;
  int rc_ = 0;
  std::thread th_;
};

class Engine {
 public:
  Config cfg;
  int precision = 0;  // 0 bf16, 1 fp32 parity
  int max_tokens = 131072, pass_tokens = 131072, max_seqs = 4096, max_gathered = 0;
  bool use_graphs = true;
  bool prof_on = false;
  // debug bounds mode (LAYA_DEBUG_BOUNDS=1, or a debug-bounds build): every pass's metadata is checked
  // on the host before it is uploaded (check_pass_meta); a failed check returns -3 without launching
  bool debug_bounds = false;
  std::string dump_dir;
  std::vector<std::unique_ptr<Replica>> reps;
  // workers[i] runs replica i's part of a call for i >= 1; replica 0 runs on the caller's thread
  std::vector<std::unique_ptr<Worker>> workers;

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
  // Runs fn(i) for every replica i at once (replica 0 on the calling thread, the others on their
  // workers), waits for all of them and returns the first non-zero result in replica order.
  int each_replica(const std::function<int(size_t)>& fn);
  std::vector<std::vector<Question>> shard(int B, const int* lens, const int* ids, const int* nmark,
                                           const int* markers, const int* qtypes, float* logits, float* act);
};

}  // namespace laya
