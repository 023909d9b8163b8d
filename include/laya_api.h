/* C ABI of the Laya B200 engine (liblaya_b200.so).
 *
 * The first ten declarations are the reference engine's ABI, unchanged in name, signature and
 * meaning (mauimauer/layamd src/laya_api.h:5-19, implemented at src/engine.hip:543-559), so the
 * reference's ctypes server (server/laya_server.py:18-31), its parity tool (src/test_parity.cpp)
 * and its bench tool (src/bench_engine.cpp) bind to this library without change. Everything after
 * them is an addition with no counterpart in the reference.
 *
 * Threading: a handle is driven by one caller thread at a time, as in the reference
 * (docs/architecture.md:84-85). Calls are synchronous: forward returns after the results are in
 * the caller's arrays.
 */
#pragma once
#ifdef __cplusplus
extern "C" {
#endif

/* Loads `dir` (model.safetensors, encoder/config.json, rl_agent_config.json) onto the GPUs named by
 * LAYA_DEVICES (default: the current device) and sizes every buffer for LAYA_MAX_TOKENS rows.
 * Replaces src/laya_api.h:5. The reference exits the process on a load error; this library prints
 * the reason and returns NULL instead. */
void* laya_create(const char* dir);

/* B questions in one call. ids/markers are concatenated per question; markers are positions within
 * that question's sequence. logits receive sum(nmark) raw scorer logits in input order, act B*n_act
 * raw act-head logits. Returns 0, or -1 without touching the outputs when any 1<=lens[b]<=max_len,
 * 1<=nmark[b]<=255 or 0<=marker<lens[b] fails, or (an addition: the reference reads outside its
 * embedding table instead) a token id lies outside [0, vocab) or a qtype outside 0..2. Replaces
 * src/laya_api.h:8-9
 * (src/engine.hip:489-539). Also returns -2 when the GPU reported an error for this call, and -3 in
 * debug bounds mode when a pass's packing maps failed their host check (nothing was launched). */
int laya_forward_batch(void* h, int B, const int* lens, const int* ids, const int* nmark, const int* markers,
                       const int* qtypes, float* logits, float* act);

/* Single-question form; S is ignored and valid_len is the length. Input errors are ignored
 * silently, as in the reference. Replaces src/laya_api.h:10-11 (src/engine.hip:549-551). */
void laya_forward(void* h, const int* ids, int S, int valid_len, const int* markers, int K, int qtype,
                  float* logits, float* act);

int laya_n_act(void* h);       /* len(act_costs)+1 from rl_agent_config.json (src/laya_api.h:12) */
int laya_max_len(void* h);     /* max_len from rl_agent_config.json (src/laya_api.h:13) */
int laya_max_markers(void* h); /* 255 (src/laya_api.h:14) */
/* Calibration temperature of a question type (src/laya_api.h:15); 1.0 for a qtype outside the
 * configured list (the reference does not check the index). */
float laya_temperature(void* h, int qtype);
/* Per-stage device-time table printed to stdout, divided by `iters` (src/laya_api.h:16). Stages are
 * timed only while profiling is on (LAYA_PROFILE set at load, or laya_prof_enable). */
void laya_prof_report(void* h, int iters);
void laya_prof_reset(void* h); /* src/laya_api.h:17 */
/* Chooses the GEMM tile width for every (M bucket, N, K) the model can hit up front, so serving
 * never tunes on the request path (src/laya_api.h:19). */
void laya_tune_all(void* h);

/* ----------------------------------------------------------------- additions (no reference
 * counterpart) */

/* Releases every device and host resource of the handle. */
void laya_destroy(void* h);

/* laya_create with an explicit precision and device list.
 * precision 0: bf16 operands, fp32 accumulation and fp32 residual stream (production path).
 * precision 1: fp32-parity mode: every GEMM runs as three bf16 products on hi/lo splits of both
 *              operands (A_hi*W_hi + A_hi*W_lo + A_lo*W_hi) and attention runs in fp32.
 * devices: comma-separated CUDA device ordinals ("0", "0,1,2,3"); NULL or "" uses LAYA_DEVICES or
 * the current device. With several devices, each forward call shards its questions across them. */
void* laya_create_ex(const char* dir, int precision, const char* devices);

/* Number of devices (replicas) the handle runs on. */
int laya_num_devices(void* h);

/* Turns per-stage profiling on or off (CUDA events around every launch; graphs are bypassed while
 * it is on). */
void laya_prof_enable(void* h, int on);

/* Copies the accumulated time (ms) and launch count of stage `name` (e.g. "gemm_qkv"); returns 0 or
 * -1 if the stage was never timed. */
int laya_prof_get(void* h, const char* name, double* ms, long long* launches);

/* Packs a batch exactly like laya_forward_batch would (validation included) and reports the pass
 * layout without touching a GPU: n_passes, and for each pass its first question, question count and
 * packed row count (arrays of capacity `cap`). Returns the number of passes or -1 on invalid input. */
int laya_plan_passes(void* h, int B, const int* lens, const int* nmark, const int* markers, int cap,
                     int* pass_first, int* pass_count, int* pass_rows);

/* Same packing rules as laya_plan_passes for a configuration given by value, with no handle
 * (max_len, pass_tokens, max_seqs); for host-side tests. */
int laya_plan_passes_cfg(int max_len, int pass_tokens, int max_seqs, int B, const int* lens, const int* nmark,
                         const int* markers, int cap, int* pass_first, int* pass_count, int* pass_rows);

/* The engine's plan for one GEMM launch, host-only (no counterpart in the reference, which autotunes
 * per shape at start-up, src/engine.hip:293-379): *bn = 128 or 256 (one CTA per 128 x bn tile) or
 * 512 (a CTA pair per 256 x 256 tile), *splits = K slices (1 = whole K). M packed rows, the weight's
 * N x K, parity != 0 for the fp32-parity mode (three bf16 products per K block), the device's SM count
 * and co-resident CTA pairs, ln_fusable != 0 for a residual GEMM whose following bias-free LayerNorm
 * a split's reduce kernel can take over (with the default credit; LAYA_SPLIT_LN_CREDIT changes only
 * the engine's own choice). Returns 0 or -1. */
int laya_plan_gemm(int M, int N, int K, int parity, int num_sms, int pair_clusters, int ln_fusable, int* bn,
                   int* splits);

/* No counterpart in the reference. Debug bounds mode, host side and host-only: validates a batch like
 * laya_forward_batch (plus qtypes in 0..2 and ids inside the vocabulary), packs it into passes of at
 * most pass_tokens rows and max_seqs questions, fills every pass's metadata block exactly as the
 * engine uploads it (token ids, positions, row -> question map, offsets, the attention work items
 * and gathered-row maps) and checks every map against the pass and the arena. corrupt > 0 breaks map
 * number `corrupt` (1-8) of the first pass before the check, so a test can show that the check
 * catches it. Returns the number of passes checked, -1 for an invalid batch, or -100-n when check n
 * failed. The engine runs the same check on every pass when loaded with LAYA_DEBUG_BOUNDS=1 or from a
 * debug-bounds build, and then returns -3 from laya_forward_batch without launching anything. */
int laya_pack_check(int max_len, int vocab, int pad_id, int pass_tokens, int max_seqs, int B, const int* lens,
                    const int* ids, const int* nmark, const int* markers, const int* qtypes, int corrupt);

/* No counterpart in the reference. 1 when this library was built with -DLAYA_DEBUG_BOUNDS: every
 * kernel then checks the indices it reads from the packing maps (token ids, rows, work items,
 * gathered rows, marker offsets, RoPE positions) against their extents, records code 40-45 in the
 * error word and skips the access instead of reading or writing out of range (laya_forward_batch
 * then returns -2). 0 in the normal build, whose kernels carry no such checks. */
int laya_debug_bounds_build(void);

/* The replica (0..ndev-1) each of B questions goes to when a call is sharded over ndev GPUs, as
 * laya_forward_batch does it, for a model of hidden size d, GeGLU width `intermediate`, n_layers
 * encoder layers of which n_global use global attention, sliding window `window` (full width) and a
 * head FFN of 4d; host-only. Longest processing time first on each question's modelled device time
 * (its algorithmic FLOPs for length lens[b] and nmark[b] options, attention FLOPs weighted by their
 * measured cost relative to GEMM FLOPs) onto the least-loaded replica. Returns 0 or -1. */
int laya_shard_plan(int ndev, int B, const int* lens, const int* nmark, int d, int intermediate, int n_layers,
                    int n_global, int window, int* owner);

/* Benchmark support: validates, packs and uploads one batch (it must fit one pass per device) and
 * keeps it resident; laya_replay then runs the staged pass `iters` times back to back on every
 * device with the inputs already in HBM and writes the device time of the slowest device, measured
 * with CUDA events on the engine's stream, to *ms. laya_staged_results copies the last replay's
 * outputs out like laya_forward_batch. Return 0 or a negative error. */
int laya_stage(void* h, int B, const int* lens, const int* ids, const int* nmark, const int* markers,
               const int* qtypes);
int laya_replay(void* h, int iters, double* ms);
int laya_staged_results(void* h, float* logits, float* act);
/* Benchmark support (no counterpart in the reference): replays the staged pass `iters` times back
 * to back as a second graph that also records a CUDA event pair around every stage, and adds the
 * stage times of the last replay to the profile table read by laya_prof_get, so that per-stage device
 * times are taken in the same steady state as laya_replay. Return 0 or a negative error. */
int laya_replay_profiled(void* h, int iters);

/* Cumulative counters of the forward and replay calls since the last reset, summed over devices:
 * kernel launches of this library, bytes copied host->device and device->host. reset != 0 clears
 * them after reading. */
int laya_io_stats(void* h, long long* launches, long long* h2d_bytes, long long* d2h_bytes, int reset);

/* Writes the residual stream after the embedding, after every encoder layer (before the final
 * norm), after the final norm + type embedding, and after each head layer for the last forward call
 * when dumping is on: files emb.bin, enc<i>.bin, final.bin, head<i>.bin (fp32, one row per packed
 * token of pass 0, sequences back to back in input order; head<last>.bin holds the gathered rows:
 * markers of every question in order, then one CLS row per question). NULL turns dumping off. */
int laya_set_dump_dir(void* h, const char* dir);

/* Isolated encoder GEMM on caller-owned device memory (the GEMM sweep and kernel tests):
 * out = epilogue(A[planes][M][K] * W[planes][N][K]^T). epi: 0 store, 1 store with RoPE on columns
 * < rope_cols, 2 GeGLU (W interleaved in groups of bn/2, out has geglu_I columns), 3 fp32 residual
 * add into resid[M][N]. out_mode: 0 bf16, 1 bf16 hi/lo planes, 2 fp32. act: 0 none, 1 ReLU, 2 GELU.
 * bn: 128 or 256 (one CTA per 128 x bn tile) or 512 (a CTA pair per 256 x 256 tile, 2-SM MMA).
 * planes 2 selects the three-product fp32 emulation. stream may be NULL. With
 * sync != 0 the call waits for the GPU and returns -100-code if a kernel reported an error (this
 * call's, or one left unread by an earlier call with sync = 0: see laya_b200_kernel_error). */
int laya_b200_gemm(const void* A, const void* W, void* out, float* resid, const float* bias, int M, int N, int K,
                   int planes, int epi, int out_mode, int act, int bn, const float* cos_t, const float* sin_t,
                   const int* pos, int rope_cols, int geglu_I, void* stream, int sync);

/* laya_b200_gemm with the K loop split into `splits` slices (1..8, and at most one per 64-wide K
 * block: ceil(K / 64), x3 in parity mode; else -2) run by different CTAs, for small M where the
 * output tiles alone cannot fill the GPU (one-CTA tiles, bn 128 or 256). The fp32 partials
 * go to a workspace the library allocates on the device and keeps for later calls; a second kernel
 * sums them in slice order and applies the epilogue, so results do not depend on scheduling. Calls
 * that overlap on the GPU (other streams) share that workspace and must not be issued. */
int laya_b200_gemm_splitk(const void* A, const void* W, void* out, float* resid, const float* bias, int M, int N,
                          int K, int planes, int epi, int out_mode, int act, int bn, const float* cos_t,
                          const float* sin_t, const int* pos, int rope_cols, int geglu_I, int splits, void* stream,
                          int sync);

/* Isolated encoder attention on caller-owned device memory (attention tests and benchmark); replaces
 * the reference's k_flash_wmma launch (src/kernels.hip:351-356) at kernel level. qkv: bf16
 * [rows][3 * 64 * H] (q | k | v, heads of 64), sequences packed back to back with lengths lens[B]
 * (host array, sum <= rows); out: bf16 [rows][64 * H]. window 0: full attention within each
 * sequence, else |q - k| <= window. impl 0: tcgen05 kernel, 1: mma.sync kernel. Rows of qkv past the
 * sequences must hold finite values. Uses a library-owned metadata buffer per device: calls must not
 * overlap on the GPU. Returns 0, -2 bad arguments, -100-code if the kernel reported an error (sync). */
int laya_b200_attention(const void* qkv, void* out, int rows, int B, const int* lens, int H, int window, int impl,
                        void* stream, int sync);

/* No counterpart in the reference (whose engine exits on any GPU error). Exercises, on GPU `device`,
 * the bounded wait that every pipeline kernel of this library uses on its mbarriers: one thread waits
 * on a barrier phase that nothing completes, gives up after the wait budget (about 2^31 SM cycles,
 * roughly one second), records its error code in a device word and returns, so the kernel ends
 * normally and the context stays usable. The word is the one the kernel-level entry points share
 * (see laya_b200_kernel_error), and the code stays there until it is read. Writes the recorded code
 * (30) to *code, the wait's length in SM cycles to *cycles and the kernel's device time to *ms.
 * Returns 0, -2 if a CUDA call failed, or -3 without launching when that word already holds an
 * earlier, unread code. */
int laya_b200_watchdog_selftest(int device, int* code, long long* cycles, float* ms);

/* No counterpart in the reference. Kernel errors of the kernel-level entry points on GPU `device`
 * (laya_b200_gemm, laya_b200_gemm_splitk, laya_b200_gemm_splitk_noalloc, laya_b200_attention, the
 * watchdog self-test). A kernel whose bounded wait ran out records a code in a device word (the first
 * code wins) and ends; a call with sync != 0 reports it as -100-code, but a call with sync = 0 cannot,
 * so the word keeps the code until it is read: by the next call with sync != 0 on the same word, or by
 * this function. It waits for all work on the device, reads and clears both words (the one the
 * allocating entries share and the one in the allocation-free entry's static array) and returns the
 * first code found (GEMM 1-5, attention 16-18, self-test 30), 0 if none, -1 for a bad device
 * ordinal, -2 if a CUDA call failed. It allocates nothing. */
int laya_b200_kernel_error(int device);

/* No counterpart in the reference. laya_b200_gemm_splitk for callers that cannot allocate device
 * memory: a host whose memory manager reserves the GPU's memory up front (a serving stack with a
 * caching allocator) or a plugin host that forbids allocation in its callbacks, where a cudaMalloc
 * could fail, fragment the host's pool or stall every stream with its implicit synchronisation. Same
 * arguments and results; it calls no cudaMalloc or cudaFree. Its scratch is a fixed 16 MiB array in
 * the library's device image, held by every GPU that loads the library until the process exits:
 * splits x M x N must stay <= 4194304 fp32 partials, else the call prints why and returns -7
 * without launching. The first call on a device sets up
 * (kernel attributes and the array's device address, no allocation); make it before any stream
 * capture. Every call on a device shares the array: calls that overlap on the GPU (other streams,
 * other threads) race and must not be issued. Every slice overwrites its whole plane of partials
 * (splits may not exceed the K blocks, ceil(K / 64) x 3 in parity mode, else -2), so no call sees
 * another's partials. The error word in the array is zeroed at set-up and then kept: a code left by
 * a call with sync = 0 is reported by the next call with sync != 0 or by laya_b200_kernel_error. */
int laya_b200_gemm_splitk_noalloc(const void* A, const void* W, void* out, float* resid, const float* bias, int M,
                                  int N, int K, int planes, int epi, int out_mode, int act, int bn,
                                  const float* cos_t, const float* sin_t, const int* pos, int rope_cols,
                                  int geglu_I, int splits, void* stream, int sync);

#ifdef __cplusplus
}
#endif
