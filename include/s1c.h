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

/* Tensor element types accepted at load (the conversions of laya-core/src/weights.rs:82-115). */
#define S1C_DT_F32 0
#define S1C_DT_F16 1
#define S1C_DT_BF16 2

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
 * matrix to bf16 and every vector to fp32, interleaves Wi for the GeGLU epilogue, uploads. */
S1C_API s1c_status s1c_create(const s1c_model_desc* desc, const s1c_tensor* tensors, int32_t n_tensors, int32_t device,
                      s1c_backend** out);
S1C_API void s1c_destroy(s1c_backend* b);
S1C_API const char* s1c_last_error(const s1c_backend* b);
/* Error text of the last s1c_create that failed on the calling thread. */
S1C_API const char* s1c_create_error(void);

/* `Backend::name` (backend.rs:111), e.g. "cuda(sm_100a,bf16)". */
S1C_API const char* s1c_name(const s1c_backend* b);
/* `Backend::active_kernels` (backend.rs:116-118): comma-separated kernels of this build. */
S1C_API const char* s1c_active_kernels(const s1c_backend* b);
/* `Backend::padded_len` (backend.rs:121-123): the varlen path needs no padding. */
S1C_API size_t s1c_padded_len(const s1c_backend* b, size_t len, size_t rows);
/* `Backend::warmup` (backend.rs:125-127). */
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
 * padded layout. Real positions hold the encoder's final hidden state; padding positions are
 * never computed by the varlen path and are written as 0. */
S1C_API s1c_status s1c_encoder_hidden(s1c_backend* b, const s1c_batch* batch, float* out);

/* Isolated GEMM on device pointers (the encoder GEMM sweep and kernel tests): out = epi(A B^T)
 * with A [M,K] and B [N,K] bf16 row-major. epi: 0 store (act 0 none / 1 ReLU / 2 GELU, bias
 * nullable, out_f32), 1 RoPE (q,k heads in columns [0, rope_cols), positions d_pos, theta),
 * 2 GeGLU (B interleaved per 128 rows, out [M, out_cols] bf16), 3 fp32 residual add in place.
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
 * as s1c_gemm with variant 3, for callers that cannot allocate device memory: a serving loop that
 * must not stall in cudaMalloc / cudaFree (both can synchronise the whole device), or a host whose
 * framework owns all device memory through its own pool. The fp32 partial sums go to a fixed
 * 4 MiB array compiled into this library (held by every GPU that loads it until the process
 * exits), so at least two split slices must fit: 2 * ceil(M / 128) * 128 * N * 4 bytes <= 4 MiB,
 * else the call returns S1C_ERR_ARG with the limit in s1c_create_error(). The first call on a
 * device looks up that device's array addresses (make it before any stream capture). All calls
 * share the array and the last call's partial sums stay in it; calls whose work overlaps on the
 * GPU race on it. The call does not synchronise. */
S1C_API s1c_status s1c_gemm_splitk_noalloc(int32_t epi, const void* d_A, const void* d_B, void* d_out, int32_t M,
                                           int32_t N, int32_t K, const float* d_bias, int32_t act, int32_t out_f32,
                                           const int32_t* d_pos, float rope_theta, int32_t rope_cols,
                                           int32_t out_cols, void* stream);

/* Number of this library's kernel launches the last forward on this handle enqueued. */
S1C_API int64_t s1c_last_launch_count(const s1c_backend* b);

#ifdef __cplusplus
}
#endif
#endif /* S1C_H */
