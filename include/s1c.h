/* s1c.h -- C ABI of libs1c, the B200 (sm_100a) model forward of sys1rust.
 *
 * The library replaces the MLX backend behind the reference's `laya_core::Backend` trait
 * (runtime/crates/laya-core/src/backend.rs:109-133): one handle per GPU owns the encoder, the
 * decision-head layers, the type embedding and the scorer, takes a collated batch and returns
 * the masked scorer logits and the pooled position-0 head state.
 *
 * Conventions
 *  - Every function returning s1c_status returns S1C_OK (0) or a negative code; the handle's
 *    s1c_last_error() (or s1c_create_error() when s1c_create failed) gives the text. No C++
 *    exception crosses this boundary.
 *  - Host pointers are borrowed for the duration of the call; outputs are caller-owned
 *    buffers of the stated size.
 *  - Calls on one handle must be serialised (the reference runs every forward on its single
 *    inference thread, runtime/crates/sys1rust/src/worker.rs:1-4); different handles are
 *    independent and may be driven from different threads.
 */
#ifndef S1C_H
#define S1C_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#if defined(__GNUC__)
#define S1C_API __attribute__((visibility("default")))
#else
#define S1C_API
#endif

typedef int32_t s1c_status;
#define S1C_OK 0
#define S1C_ERR_ARG (-1)            /* malformed batch or argument (Error::Backend / 422-class input) */
#define S1C_ERR_CUDA (-2)           /* a CUDA runtime call failed */
#define S1C_ERR_WEIGHTS (-3)        /* missing or mis-shaped tensor (Error::Weights) */
#define S1C_ERR_CONFIG (-4)         /* config the kernels do not support (Error::Config) */
#define S1C_ERR_DEVICE_TIMEOUT (-5) /* a bounded device-side wait ran out; the context stays usable */
#define S1C_ERR_UNSUPPORTED (-6)    /* no sm_100 device */
#define S1C_ERR_BUSY (-7)           /* serving: admission cap reached, "server busy, try again later" (503, Retry-After: 1) */
#define S1C_ERR_DEAD (-8)           /* serving: no inference worker, "inference worker is not running" (503) */
#define S1C_ERR_TIMEOUT (-9)        /* serving: result not ready within the wait's timeout; the ticket stays valid */
#define S1C_ERR_SELFCHECK (-10)     /* load check: a kernel differs from the plain computation and no checked kernel can take its place */

/* Tensor element types accepted at load (the conversions of laya-core/src/weights.rs:82-115). */
#define S1C_DT_F32 0
#define S1C_DT_F16 1
#define S1C_DT_BF16 2
#define S1C_DT_F64 3

/* Encoder + head configuration: the normalised `EncoderConfig` (laya-core/src/config.rs:64-202)
 * plus the head layer count of `AgentConfig` (config.rs:9-30). */
typedef struct s1c_model_desc {
  int32_t vocab_size;
  int32_t hidden_size;         /* d; multiple of 256 (768 and 1024 for the published encoders) */
  int32_t num_layers;
  int32_t num_heads;           /* head_dim = d / num_heads must be 64 */
  int32_t intermediate_size;   /* I; Wi is [2I, d], Wo is [d, I]; multiple of 32 */
  float norm_eps;
  int32_t local_attention;     /* window width; a query sees keys with |i - j| <= local_attention / 2 */
  float global_rope_theta;
  float local_rope_theta;
  const uint8_t* layer_is_local; /* [num_layers], 1 = sliding-window layer */
  int32_t head_layers;         /* decision-head transformer layers (>= 1) */
  int32_t max_position;        /* longest row the backend accepts (RoPE table length) */
  int32_t max_tokens;          /* initial activation capacity in packed tokens (grows on demand) */
} s1c_model_desc;

/* One named tensor of the checkpoint, in host memory, row-major (the safetensors view). */
typedef struct s1c_tensor {
  const char* name;
  int32_t dtype;      /* S1C_DT_* */
  int32_t ndim;
  int64_t shape[4];
  const void* data;
} s1c_tensor;

/* `laya_core::Batch` as plain data (backend.rs:74-98): row-major padded ids, 1/0 mask with
 * right padding, per-row lengths, marker positions (n*kmax, zero past marker_count), qtype. */
typedef struct s1c_batch {
  size_t n;
  size_t len;
  size_t kmax;
  const uint32_t* input_ids;      /* [n*len] */
  const uint32_t* attention_mask; /* [n*len] */
  const size_t* seq_lens;         /* [n] */
  const uint32_t* marker_pos;     /* [n*kmax] */
  const size_t* marker_count;     /* [n] */
  const uint32_t* qtype;          /* [n] 0 choice, 1 score, 2 noul */
} s1c_batch;

/* The unpadded form of the same batch: the real tokens of every row back to back. Row r is
 * ids[cu_seqlens[r] .. cu_seqlens[r+1]); marker positions are positions inside the row. */
typedef struct s1c_varlen {
  int32_t n;
  int32_t kmax;
  const uint32_t* ids;          /* [cu_seqlens[n]] */
  const int32_t* cu_seqlens;    /* [n+1], cu_seqlens[0] = 0 */
  const uint32_t* marker_pos;   /* [n*kmax] */
  const int32_t* marker_count;  /* [n] */
  const uint32_t* qtype;        /* [n] */
} s1c_varlen;

typedef struct s1c_backend s1c_backend;

/* Build a backend on `device` from named tensors: replaces `MlxBackend::new`
 * (laya-mlx/src/lib.rs:960-1150) / the factory `make_backend` (lib.rs:593-604). Converts every
 * matrix to bf16 and every vector to fp32, interleaves Wi for the GeGLU epilogue, uploads.
 * The environment variable S1C_SETTINGS, read here, is a comma list of kernel choices (an unknown
 * key or value fails the call with S1C_ERR_CONFIG): attn=auto|tc|mma (attention kernel; auto:
 * tcgen05 on full rows when its grid fills the SMs, else mma.sync), gemm=auto|1cta|2cta|splitk|csk,
 * graphs=0|1 (CUDA graph per batch shape), pdl=0|1 (programmatic dependent launch),
 * buckets=<tokens>:<tokens>:... (packed-token buckets, default 128:256:...:1024:1280:...:2048;
 * buckets=0 turns them off), warm=<rows>:... (row counts s1c_warmup runs at every bucket, default 1),
 * trace=0|1, layers=0|1, ops=0|1 (the reference's tracing knobs: per forward a stderr line with the
 * shape, the graph use, the host enqueue and the device time; per encoder layer device times; per
 * kernel summed device times; layers and ops launch kernel by kernel; with the asynchronous entry
 * point the lines describe the last forward before s1c_synchronize), check=0|1 (default 1) and
 * check_fail=<kernel>[+<kernel>...].
 * Buckets (the reference's `buckets` / `warm` settings, laya-mlx/src/lib.rs:89-94): a batch of n
 * rows whose packed tokens fit a bucket runs as the bucket's shape, with dummy rows (at least one,
 * row count a power of two up to 64; none when the tokens fill the bucket) holding the remaining
 * tokens, and marker slots padded to 4 (past 4 markers, to a multiple of 16). The dummy rows are
 * computed apart from the batch's rows and dropped, so a bucket's CUDA graph (captured at the
 * shape's first forward or by s1c_warmup) replays every batch of that shape; larger batches run
 * their exact shape (graph captured at its second forward).
 * Load check (the reference's load-time kernel checks and fallback rule, lib.rs:319-362): every
 * kernel the forward can pick runs once on small seeded problems (GEMMs with each epilogue,
 * attention global and sliding window over ragged rows) and is compared with a double-precision
 * host computation, each output element within 1e-2 * (1 + |expected|). A failing two-CTA or
 * cluster split-K GEMM or tcgen05 attention is turned off for this handle (one stderr line; the
 * one-CTA GEMM / mma.sync attention take its work; s1c_active_kernels names it); a failing
 * one-CTA GEMM or mma.sync attention, or a failing kernel forced by the settings, fails the call
 * with S1C_ERR_SELFCHECK. check_fail (1cta, 2cta, csk, splitk, tc, mma) plants a wrong expected
 * value in those kernels' checks, for tests of the fallback rule. */
S1C_API s1c_status s1c_create(const s1c_model_desc* desc, const s1c_tensor* tensors, int32_t n_tensors, int32_t device,
                      s1c_backend** out);
/* s1c_create with the settings given as a string (the comma list above; NULL reads S1C_SETTINGS),
 * for hosts that pass `BackendOptions::tuning` (laya-core/src/backend.rs:22-42) instead of setting
 * the environment. The key `parallel_load` (the runtime's own setting) is accepted and ignored. */
S1C_API s1c_status s1c_create_with_settings(const s1c_model_desc* desc, const s1c_tensor* tensors, int32_t n_tensors,
                                            int32_t device, const char* settings, s1c_backend** out);
S1C_API void s1c_destroy(s1c_backend* b);
S1C_API const char* s1c_last_error(const s1c_backend* b);
/* Error text of the last call without a backend handle that failed on the calling thread
 * (s1c_create, s1c_weights_*, s1c_server_*, s1c_gemm, s1c_attention). */
S1C_API const char* s1c_create_error(void);

/* `Backend::name` (backend.rs:111), e.g. "cuda(sm_100a,bf16)". */
S1C_API const char* s1c_name(const s1c_backend* b);
/* `Backend::active_kernels` (backend.rs:116-118): comma-separated kernels of this build. */
S1C_API const char* s1c_active_kernels(const s1c_backend* b);
/* `Backend::padded_len` (backend.rs:121-123): the varlen path needs no padding. */
S1C_API size_t s1c_padded_len(const s1c_backend* b, size_t len, size_t rows);
/* `Backend::warmup` (backend.rs:125-127): one forward per (bucket, `warm=` row count) as the
 * reference's warm_buckets (lib.rs:1152-1173), which captures each such bucket shape's CUDA graph. */
S1C_API s1c_status s1c_warmup(s1c_backend* b);

/* `Backend::forward` (backend.rs:112; MlxBackend::forward lib.rs:1833-1863): logits [n*kmax]
 * with -1e4 at slots past marker_count, pooled [n*hidden] (position 0 of the head output). */
S1C_API s1c_status s1c_forward_padded(s1c_backend* b, const s1c_batch* batch, float* logits, float* pooled);

/* The same forward from the unpadded layout; `hidden` (nullable) receives the encoder's final
 * hidden state of every packed token, [cu_seqlens[n] * hidden] f32. */
S1C_API s1c_status s1c_forward_varlen(s1c_backend* b, const s1c_varlen* in, float* logits, float* pooled, float* hidden);

/* Device-resident variant: `in` holds HOST metadata (cu_seqlens, markers, qtype) and `d_ids`
 * the token ids already in device memory; outputs are device pointers (hidden nullable). The
 * work is enqueued on the handle's stream and the call returns after it completes. */
S1C_API s1c_status s1c_forward_device(s1c_backend* b, const s1c_varlen* in, const uint32_t* d_ids, float* d_logits,
                              float* d_pooled, float* d_hidden);

/* As s1c_forward_device, but returns once the work is enqueued on the handle's stream: several
 * forwards can be in flight, and the host prepares the next batch while the GPU runs. Inputs and
 * outputs must stay valid until s1c_synchronize returns; the outputs of consecutive calls must not
 * alias unless the caller orders them. Device-side errors surface at s1c_synchronize. */
S1C_API s1c_status s1c_forward_device_async(s1c_backend* b, const s1c_varlen* in, const uint32_t* d_ids,
                                            float* d_logits, float* d_pooled, float* d_hidden);
/* Wait for every forward enqueued on this handle and report any device-side error. */
S1C_API s1c_status s1c_synchronize(s1c_backend* b);

/* `Backend::encoder_hidden` (backend.rs:128-132; lib.rs:1869-1878): [n*len*hidden] f32 in the
 * padded layout, as the reference's hook computes it: real positions hold the encoder's final
 * hidden state, and so do padding positions within local_attention / 2 of the row's last real
 * token (the batch's padding id at its padded index, attending the row's real tokens; no real
 * position attends it). Padding positions farther away are written as 0: in the reference's
 * sliding-window layers every key they may see is masked (a softmax over -1e4 entries only), which
 * this path does not reproduce. The logits and pooled rows of `forward` do not depend on padding
 * positions. */
S1C_API s1c_status s1c_encoder_hidden(s1c_backend* b, const s1c_batch* batch, float* out);

/* Isolated GEMM on device pointers (the encoder GEMM sweep and kernel tests): out = epi(A B^T)
 * with A [M,K] and B [N,K] bf16 row-major. epi: 0 store (act 0 none / 1 ReLU / 2 GELU, bias
 * nullable, out_f32), 1 RoPE (q,k heads in columns [0, rope_cols), positions d_pos below 8192, theta),
 * 2 GeGLU (B interleaved per 128 rows, out [M, out_cols] bf16), 3 fp32 residual add in place,
 * 4 f16 residual add in place (the encoder's residual stream; bias nullable).
 * variant: 0 by shape, 1 one-CTA 128x256 tiles, 2 two-CTA 256x256 tiles (cta_group::2), 3 one-CTA with
 * the K dimension split across CTAs (fp32 partial sums reduced in a workspace, then the epilogue),
 * 4 cluster split-K (the CTAs of a thread-block cluster split K and reduce their partial tiles
 * through distributed shared memory in one launch; what variant 0 picks for few output tiles).
 * `stream` is a cudaStream_t (NULL = legacy default stream); the call does not synchronise. */
S1C_API s1c_status s1c_gemm(int32_t epi, const void* d_A, const void* d_B, void* d_out, int32_t M, int32_t N, int32_t K,
                            const float* d_bias, int32_t act, int32_t out_f32, const int32_t* d_pos, float rope_theta,
                            int32_t rope_cols, int32_t out_cols, int32_t variant, void* stream);

/* Isolated varlen attention on device pointers (head_dim 64): q/k/v/o with row pitches, host
 * cu_seqlens [n+1]; window < 0 = global. impl 0 = tcgen05 kernel (v must lie in k's rows: same
 * pitch, 64-aligned column offset), 1 = mma.sync kernel. Blocks until done. */
S1C_API s1c_status s1c_attention(const void* d_q, const void* d_k, const void* d_v, void* d_o, int32_t q_stride,
                                 int32_t k_stride, int32_t v_stride, int32_t o_stride, int32_t heads,
                                 const int32_t* cu_seqlens, int32_t n, int32_t window, float scale, int32_t impl,
                                 void* stream);

/* Run this handle's forwards on `stream` (a cudaStream_t of the handle's device); NULL returns
 * to the handle's own stream. Lets a caller order forwards with its own work and time them with
 * events on that stream. */
S1C_API s1c_status s1c_set_stream(s1c_backend* b, void* stream);

/* Per-kernel timing: with `on` = 1 every launch of later forwards is bracketed by CUDA events on
 * the forward's stream (statistics cleared); 0 turns it off. */
S1C_API s1c_status s1c_profile(s1c_backend* b, int32_t on);
/* Text report of the profile, one line per kernel: "name launches total_ms flops bytes" (FLOPs and
 * bytes are algorithmic). Returns the size needed including the terminating 0. */
S1C_API size_t s1c_profile_report(const s1c_backend* b, char* buf, size_t cap);

/* Split-K GEMM that allocates nothing (no counterpart in the reference). Same arguments and result
 * as s1c_gemm with variant 3 for epilogues 0 to 3 (epi 4, the f16 residual add, is refused with
 * S1C_ERR_ARG), for callers that cannot allocate device memory: a serving loop that
 * must not stall in cudaMalloc / cudaFree (both can synchronise the whole device), or a host whose
 * framework owns all device memory through its own pool. The fp32 partial sums go to a fixed
 * 4 MiB array compiled into this library (held by every GPU that loads it until the process
 * exits), so at least two split slices must fit: 2 * ceil(M / 128) * 128 * N * 4 bytes <= 4 MiB,
 * else the call returns S1C_ERR_ARG with the limit in s1c_create_error(). The first call on a
 * device looks up that device's array addresses (make it before any stream capture). All calls
 * share the array and the last call's partial sums stay in it; calls whose work overlaps on the
 * GPU race on it. The call does not synchronise. A bounded device-side wait that runs out inside
 * these kernels is not reported by this entry point (its status word is never read back): the
 * call returns S1C_OK and the output is incomplete. */
S1C_API s1c_status s1c_gemm_splitk_noalloc(int32_t epi, const void* d_A, const void* d_B, void* d_out, int32_t M,
                                           int32_t N, int32_t K, const float* d_bias, int32_t act, int32_t out_f32,
                                           const int32_t* d_pos, float rope_theta, int32_t rope_cols,
                                           int32_t out_cols, void* stream);

/* Self-test of the device-side failure detection: a kernel waits, with a budget of `budget_ns`
 * (1e6 .. 2e9), on an mbarrier that nothing completes, once in the single-thread form the TMA and
 * MMA roles use and once in the warp form the epilogue / softmax roles use. Both waits must give up
 * and return. codes[0] / codes[1] receive the status codes they recorded (1 and 4, the codes a
 * forward reports inside S1C_ERR_DEVICE_TIMEOUT), codes[2] / codes[3] whether each wait claimed
 * success (0). Returns S1C_OK when the kernel ended; the device stays usable. */
S1C_API s1c_status s1c_selftest_wait_timeout(int32_t device, int64_t budget_ns, int32_t* codes);

/* Number of this library's kernel launches the last forward on this handle enqueued. */
S1C_API int64_t s1c_last_launch_count(const s1c_backend* b);

/* ---- Checkpoint files (laya_core::Weights, runtime/crates/laya-core/src/weights.rs:10-77) ----
 * A memory-mapped `model.safetensors`, validated when opened: an interrupted download fails at
 * open with the file's path and length, never inside a later call. Tensor views point into the
 * mapping and stay valid until s1c_weights_close. Errors are S1C_ERR_WEIGHTS with the text in
 * s1c_create_error(), worded as the reference's Error::Weights messages. */
typedef struct s1c_weights s1c_weights;

/* Weights::open (weights.rs:23-43): maps <model_dir>/model.safetensors. Errors:
 *   "'model.safetensors' not found in <model_dir>"
 *   "<model_dir>/model.safetensors (<bytes> bytes) is truncated or not a safetensors file: <why>" */
S1C_API s1c_status s1c_weights_open(const char* model_dir, s1c_weights** out);
S1C_API void s1c_weights_close(s1c_weights* w);
/* Weights::names (weights.rs:50-57): the tensor count; names in header order via s1c_weights_tensor. */
S1C_API int32_t s1c_weights_count(const s1c_weights* w);
/* Index of the tensor called `name`, or -1. */
S1C_API int32_t s1c_weights_find(const s1c_weights* w, const char* name);
/* View of tensor i (name, dtype, shape, data in the mapping). Float dtypes only, as to_f32
 * converts (weights.rs:82-105): F32, F16, BF16, F64; others are "unsupported dtype <X>". */
S1C_API s1c_status s1c_weights_tensor(const s1c_weights* w, int32_t i, s1c_tensor* out);
/* Weights::verify (weights.rs:66-77): the encoder., type_emb., scorer. and act_head. families are
 * present; else "checkpoint is missing '<prefix>' parameters; expected an RL Agent decision model". */
S1C_API s1c_status s1c_weights_verify(const s1c_weights* w);
/* s1c_create over every float tensor of an open checkpoint (F16 / F32 / F64 converted at load). */
S1C_API s1c_status s1c_create_from_weights(const s1c_model_desc* desc, const s1c_weights* w, int32_t device,
                                           s1c_backend** out);

/* ---- Serving: cross-request batching over GPU workers --------------------------------------
 * Replaces the reference server's single inference thread (runtime/crates/sys1rust/src/worker.rs)
 * with one worker per backend that packs queued requests from many clients into varlen batches,
 * keeping its admission contract (http.rs:168-230): submit never blocks; over the concurrency cap it
 * returns S1C_ERR_BUSY at once. A request is the tokenised row of one `Agent::predict` call. The
 * permit is held from submit until the result is collected (s1c_server_wait) or the ticket is
 * cancelled; a cancelled request still queued is dropped unrun (worker.rs:202-205). A failed forward
 * fails the requests of its batch only. Error texts: s1c_create_error(). */
typedef struct s1c_server s1c_server;

/* The forward a worker runs on one packed batch: outputs as s1c_forward_varlen (logits [n*kmax],
 * pooled [n*hidden]); on failure return a negative status and optionally point *error at a
 * message valid until the next call with the same ctx. */
typedef s1c_status (*s1c_server_forward_fn)(void* ctx, const s1c_varlen* batch, float* logits, float* pooled,
                                            const char** error);

typedef struct s1c_server_opts {
  int32_t max_concurrent;   /* admission cap; <= 0: 16, the reference's DEFAULT_MAX_CONCURRENT (config.rs:14) */
  int32_t max_batch_tokens; /* packed tokens per batch; <= 0: 16384 (a longer request runs alone) */
  int32_t max_batch_rows;   /* rows per batch; <= 0: 1024 */
  int32_t linger_us;        /* wait up to this long for more requests when under half a batch is queued */
} s1c_server_opts;

/* One request: token ids of the row (`collate_to`'s row layout, sequence.rs:44-104), marker
 * positions inside the row, question type (0 choice, 1 score, 2 noul). Copied at submit. */
typedef struct s1c_request {
  const uint32_t* ids;
  int32_t len;
  const uint32_t* marker_pos;
  int32_t n_markers;
  uint32_t qtype;
} s1c_request;

typedef struct s1c_server_stats {
  uint64_t batches, rows, tokens, failed_batches, busy_rejections, cancelled_skipped;
  int32_t in_flight, queued, workers_alive;
} s1c_server_stats;

/* One worker per backend (each handle then belongs to the server until s1c_server_destroy). */
S1C_API s1c_status s1c_server_create(s1c_backend* const* backends, int32_t n_backends, const s1c_server_opts* opts,
                                     s1c_server** out);
/* Workers running `fn` with ctx[i] (tests, other engines); `hidden` sizes the pooled rows. */
S1C_API s1c_status s1c_server_create_with(s1c_server_forward_fn fn, void* const* ctx, int32_t n_workers,
                                          int32_t hidden, const s1c_server_opts* opts, s1c_server** out);
/* Queue a request. S1C_ERR_BUSY over the cap, S1C_ERR_DEAD once stopped, S1C_ERR_ARG for a
 * malformed row (empty, or a marker outside the row). */
S1C_API s1c_status s1c_server_submit(s1c_server* s, const s1c_request* req, uint64_t* ticket);
/* Wait for a result (timeout_ms < 0: no limit) and collect it, releasing the permit: logits
 * [n_markers], pooled [hidden], infer_ms (nullable) = the batch's forward time. S1C_ERR_TIMEOUT
 * leaves the ticket pending. Any other status ends the ticket. */
S1C_API s1c_status s1c_server_wait(s1c_server* s, uint64_t ticket, int32_t timeout_ms, float* logits, float* pooled,
                                   float* infer_ms);
/* The client went away: drop the ticket (unrun if still queued) and release its permit. */
S1C_API s1c_status s1c_server_cancel(s1c_server* s, uint64_t ticket);
S1C_API s1c_status s1c_server_get_stats(s1c_server* s, s1c_server_stats* out);
/* Stop accepting, fail the queued requests with S1C_ERR_DEAD, let running batches finish and
 * join the workers. Collect or cancel outstanding tickets afterwards. */
S1C_API void s1c_server_stop(s1c_server* s);
/* Stop (if needed) and free. No other call on `s` may be running or follow. */
S1C_API void s1c_server_destroy(s1c_server* s);

/* ---- Decode: answers from the forward's outputs (laya-core/src/decode.rs) -------------------
 * The arithmetic of `decode_answers` (decode.rs:318-413) on the host: temperature-scaled softmax
 * over each row's options, entropy confidence, the per-type answer values and the action head's
 * probability (`ActHead::probs`, decode.rs:232-253, on the features of `act_features`,
 * decode.rs:257-267). The result object's JSON (labels, legends, 4-decimal rounding) is the
 * caller's. */
typedef struct s1c_act_head {
  int32_t d_in;   /* hidden + 4 */
  int32_t hidden; /* width of the first layer */
  int32_t n_act;  /* action classes (len(act_costs) + 1) */
  const float* w0; /* [hidden, d_in] */
  const float* b0; /* [hidden] */
  const float* w2; /* [n_act, hidden] */
  const float* b2; /* [n_act] */
} s1c_act_head;

typedef struct s1c_answer {
  int32_t qtype;            /* 0 choice, 1 score, 2 noul */
  int32_t k;                /* options of the row (marker_count) */
  int32_t argmax;           /* most probable option (first maximum) */
  double score;             /* score: expected level sum_i i p_i */
  double noul;              /* noul: p of option 1 */
  double confidence;        /* choice / score: 1 - H(p) / ln k; noul: max(p1, 1 - p1) */
  double answer_confidence; /* choice: p[argmax]; score: max p; noul: max(p1, 1 - p1) */
  float act_probability;    /* action head, class 0 */
} s1c_answer;

/* Decode n rows: logits [n*kmax] (masked slots -1e4) and pooled [n*hidden] as the forward returns
 * them, marker_count [n], qtype [n], temperature [n] (the row's calibration scale, already
 * clamped: Temperatures::scale, decode.rs:80-86). probs (nullable) receives [n*kmax] option
 * probabilities (0 past marker_count). Errors: S1C_ERR_WEIGHTS for an action head whose input is
 * not hidden + 4 wide (decode.rs:155-207 wording), S1C_ERR_ARG otherwise. */
S1C_API s1c_status s1c_decode(const float* logits, const float* pooled, int32_t n, int32_t kmax, int32_t hidden,
                              const int32_t* marker_count, const uint32_t* qtype, const double* temperature,
                              const s1c_act_head* head, double* probs, s1c_answer* out);

#ifdef __cplusplus
}
#endif
#endif /* S1C_H */
