//! Raw bindings of `libs1c` (`include/s1c.h`), the B200 (sm_100a) model forward of sys1rust.
//!
//! Every item mirrors the header one for one: `#[repr(C)]` structs with the header's field order
//! and widths (`size_t` is `usize`, `int32_t` is `i32`), the status and dtype constants, and one
//! `extern "C"` declaration per entry point. Safe wrappers live in the `laya-cuda` crate.
#![allow(non_camel_case_types)]

use std::ffi::{c_char, c_void};

pub type s1c_status = i32;
pub const S1C_OK: i32 = 0;
pub const S1C_ERR_ARG: i32 = -1;
pub const S1C_ERR_CUDA: i32 = -2;
pub const S1C_ERR_WEIGHTS: i32 = -3;
pub const S1C_ERR_CONFIG: i32 = -4;
pub const S1C_ERR_DEVICE_TIMEOUT: i32 = -5;
pub const S1C_ERR_UNSUPPORTED: i32 = -6;
pub const S1C_ERR_BUSY: i32 = -7;
pub const S1C_ERR_DEAD: i32 = -8;
pub const S1C_ERR_TIMEOUT: i32 = -9;
pub const S1C_ERR_SELFCHECK: i32 = -10;

pub const S1C_DT_F32: i32 = 0;
pub const S1C_DT_F16: i32 = 1;
pub const S1C_DT_BF16: i32 = 2;
pub const S1C_DT_F64: i32 = 3;

/// Opaque handle of one model on one GPU.
#[repr(C)]
pub struct s1c_backend {
    _p: [u8; 0],
}
/// Opaque memory-mapped checkpoint.
#[repr(C)]
pub struct s1c_weights {
    _p: [u8; 0],
}
/// Opaque serving queue.
#[repr(C)]
pub struct s1c_server {
    _p: [u8; 0],
}

#[repr(C)]
pub struct s1c_model_desc {
    pub vocab_size: i32,
    pub hidden_size: i32,
    pub num_layers: i32,
    pub num_heads: i32,
    pub intermediate_size: i32,
    pub norm_eps: f32,
    pub local_attention: i32,
    pub global_rope_theta: f32,
    pub local_rope_theta: f32,
    pub layer_is_local: *const u8,
    pub head_layers: i32,
    pub max_position: i32,
    pub max_tokens: i32,
}

#[repr(C)]
pub struct s1c_tensor {
    pub name: *const c_char,
    pub dtype: i32,
    pub ndim: i32,
    pub shape: [i64; 4],
    pub data: *const c_void,
}

/// `laya_core::Batch` field for field (the vectors as pointers).
#[repr(C)]
pub struct s1c_batch {
    pub n: usize,
    pub len: usize,
    pub kmax: usize,
    pub input_ids: *const u32,
    pub attention_mask: *const u32,
    pub seq_lens: *const usize,
    pub marker_pos: *const u32,
    pub marker_count: *const usize,
    pub qtype: *const u32,
}

#[repr(C)]
pub struct s1c_varlen {
    pub n: i32,
    pub kmax: i32,
    pub ids: *const u32,
    pub cu_seqlens: *const i32,
    pub marker_pos: *const u32,
    pub marker_count: *const i32,
    pub qtype: *const u32,
}

#[repr(C)]
#[derive(Default, Clone, Copy)]
pub struct s1c_server_opts {
    pub max_concurrent: i32,
    pub max_batch_tokens: i32,
    pub max_batch_rows: i32,
    pub linger_us: i32,
}

#[repr(C)]
pub struct s1c_request {
    pub ids: *const u32,
    pub len: i32,
    pub marker_pos: *const u32,
    pub n_markers: i32,
    pub qtype: u32,
}

#[repr(C)]
#[derive(Default, Clone, Copy, Debug)]
pub struct s1c_server_stats {
    pub batches: u64,
    pub rows: u64,
    pub tokens: u64,
    pub failed_batches: u64,
    pub busy_rejections: u64,
    pub cancelled_skipped: u64,
    pub in_flight: i32,
    pub queued: i32,
    pub workers_alive: i32,
}

#[repr(C)]
pub struct s1c_act_head {
    pub d_in: i32,
    pub hidden: i32,
    pub n_act: i32,
    pub w0: *const f32,
    pub b0: *const f32,
    pub w2: *const f32,
    pub b2: *const f32,
}

#[repr(C)]
#[derive(Default, Clone, Copy, Debug)]
pub struct s1c_answer {
    pub qtype: i32,
    pub k: i32,
    pub argmax: i32,
    pub score: f64,
    pub noul: f64,
    pub confidence: f64,
    pub answer_confidence: f64,
    pub act_probability: f32,
}

/// The forward a serving worker runs on one packed batch (`s1c_server_create_with`).
pub type s1c_server_forward_fn = Option<
    unsafe extern "C" fn(
        ctx: *mut c_void,
        batch: *const s1c_varlen,
        logits: *mut f32,
        pooled: *mut f32,
        error: *mut *const c_char,
    ) -> s1c_status,
>;

#[link(name = "s1c")]
extern "C" {
    // ---- backend handle (laya_core::Backend) ----
    pub fn s1c_create(desc: *const s1c_model_desc, tensors: *const s1c_tensor, n_tensors: i32, device: i32,
                      out: *mut *mut s1c_backend) -> s1c_status;
    pub fn s1c_create_with_settings(desc: *const s1c_model_desc, tensors: *const s1c_tensor, n_tensors: i32,
                                    device: i32, settings: *const c_char, out: *mut *mut s1c_backend) -> s1c_status;
    pub fn s1c_destroy(b: *mut s1c_backend);
    pub fn s1c_last_error(b: *const s1c_backend) -> *const c_char;
    pub fn s1c_create_error() -> *const c_char;
    pub fn s1c_name(b: *const s1c_backend) -> *const c_char;
    pub fn s1c_active_kernels(b: *const s1c_backend) -> *const c_char;
    pub fn s1c_padded_len(b: *const s1c_backend, len: usize, rows: usize) -> usize;
    pub fn s1c_warmup(b: *mut s1c_backend) -> s1c_status;
    pub fn s1c_forward_padded(b: *mut s1c_backend, batch: *const s1c_batch, logits: *mut f32,
                              pooled: *mut f32) -> s1c_status;
    pub fn s1c_forward_varlen(b: *mut s1c_backend, v: *const s1c_varlen, logits: *mut f32, pooled: *mut f32,
                              hidden: *mut f32) -> s1c_status;
    pub fn s1c_forward_device(b: *mut s1c_backend, v: *const s1c_varlen, d_ids: *const u32, d_logits: *mut f32,
                              d_pooled: *mut f32, d_hidden: *mut f32) -> s1c_status;
    pub fn s1c_forward_device_async(b: *mut s1c_backend, v: *const s1c_varlen, d_ids: *const u32,
                                    d_logits: *mut f32, d_pooled: *mut f32, d_hidden: *mut f32) -> s1c_status;
    pub fn s1c_synchronize(b: *mut s1c_backend) -> s1c_status;
    pub fn s1c_encoder_hidden(b: *mut s1c_backend, batch: *const s1c_batch, out: *mut f32) -> s1c_status;
    pub fn s1c_set_stream(b: *mut s1c_backend, stream: *mut c_void) -> s1c_status;
    pub fn s1c_profile(b: *mut s1c_backend, on: i32) -> s1c_status;
    pub fn s1c_profile_report(b: *const s1c_backend, buf: *mut c_char, cap: usize) -> usize;
    pub fn s1c_last_launch_count(b: *const s1c_backend) -> i64;

    // ---- isolated kernels (tests, sweeps) ----
    pub fn s1c_gemm(epi: i32, d_a: *const c_void, d_b: *const c_void, d_out: *mut c_void, m: i32, n: i32, k: i32,
                    d_bias: *const f32, act: i32, out_f32: i32, d_pos: *const i32, rope_theta: f32,
                    rope_cols: i32, out_cols: i32, variant: i32, stream: *mut c_void) -> s1c_status;
    pub fn s1c_attention(d_q: *const c_void, d_k: *const c_void, d_v: *const c_void, d_o: *mut c_void,
                         q_stride: i32, k_stride: i32, v_stride: i32, o_stride: i32, heads: i32,
                         cu_seqlens: *const i32, n: i32, window: i32, scale: f32, imp: i32,
                         stream: *mut c_void) -> s1c_status;
    pub fn s1c_gemm_splitk_noalloc(epi: i32, d_a: *const c_void, d_b: *const c_void, d_out: *mut c_void, m: i32,
                                   n: i32, k: i32, d_bias: *const f32, act: i32, out_f32: i32, d_pos: *const i32,
                                   rope_theta: f32, rope_cols: i32, out_cols: i32,
                                   stream: *mut c_void) -> s1c_status;
    pub fn s1c_selftest_wait_timeout(device: i32, budget_ns: i64, codes: *mut i32) -> s1c_status;

    // ---- checkpoint files (laya_core::Weights) ----
    pub fn s1c_weights_open(model_dir: *const c_char, out: *mut *mut s1c_weights) -> s1c_status;
    pub fn s1c_weights_close(w: *mut s1c_weights);
    pub fn s1c_weights_count(w: *const s1c_weights) -> i32;
    pub fn s1c_weights_find(w: *const s1c_weights, name: *const c_char) -> i32;
    pub fn s1c_weights_tensor(w: *const s1c_weights, i: i32, out: *mut s1c_tensor) -> s1c_status;
    pub fn s1c_weights_verify(w: *const s1c_weights) -> s1c_status;
    pub fn s1c_create_from_weights(desc: *const s1c_model_desc, w: *const s1c_weights, device: i32,
                                   out: *mut *mut s1c_backend) -> s1c_status;

    // ---- serving queue (sys1rust's inference worker) ----
    pub fn s1c_server_create(backends: *const *mut s1c_backend, n_backends: i32, opts: *const s1c_server_opts,
                             out: *mut *mut s1c_server) -> s1c_status;
    pub fn s1c_server_create_with(f: s1c_server_forward_fn, ctx: *const *mut c_void, n_workers: i32, hidden: i32,
                                  opts: *const s1c_server_opts, out: *mut *mut s1c_server) -> s1c_status;
    pub fn s1c_server_submit(s: *mut s1c_server, req: *const s1c_request, ticket: *mut u64) -> s1c_status;
    pub fn s1c_server_wait(s: *mut s1c_server, ticket: u64, timeout_ms: i32, logits: *mut f32, pooled: *mut f32,
                           infer_ms: *mut f32) -> s1c_status;
    pub fn s1c_server_cancel(s: *mut s1c_server, ticket: u64) -> s1c_status;
    pub fn s1c_server_get_stats(s: *mut s1c_server, out: *mut s1c_server_stats) -> s1c_status;
    pub fn s1c_server_stop(s: *mut s1c_server);
    pub fn s1c_server_destroy(s: *mut s1c_server);

    // ---- decode (laya_core::decode arithmetic) ----
    pub fn s1c_decode(logits: *const f32, pooled: *const f32, n: i32, kmax: i32, hidden: i32,
                      marker_count: *const i32, qtype: *const u32, temperature: *const f64,
                      head: *const s1c_act_head, probs: *mut f64, out: *mut s1c_answer) -> s1c_status;
}
