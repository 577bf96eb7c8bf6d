//! `laya_core::Backend` on B200 GPUs through libs1c (the `cuda-ffi` crate).
//!
//! A drop-in for the MLX backend (`laya-mlx/src/lib.rs:593-604`, `make_backend`): `Agent::load`
//! (`laya-core/src/agent.rs:79-80`) and `testing::run_parity` (`laya-core/src/testing.rs:390`) take
//! [`make_backend`] / [`factory`] unchanged. [`Server`] is the cross-request batching queue over one
//! or more GPUs that replaces sys1rust's single inference thread (`sys1rust/src/worker.rs:103-223`).
//!
//! Settings come from `BackendOptions::tuning` (or `SYS1_MLX` when that is `None`, as for the MLX
//! backend) and go to the library as a string: `attn=`, `gemm=`, `graphs=`, `pdl=`, `buckets=`,
//! `warm=`, `check=` (see `include/s1c.h`). This crate reads one key itself, `device=<ordinal>`
//! (default 0), and removes it before the library sees the list.

use cuda_ffi as ffi;
use laya_core::{Backend, BackendOptions, BackendOutput, Batch, Error, ModelConfig, Result, Weights};
use safetensors::Dtype;
use std::ffi::{c_char, CStr, CString};
use std::sync::Mutex;

fn text(p: *const c_char) -> String {
    if p.is_null() {
        return String::new();
    }
    // SAFETY: libs1c returns NUL-terminated strings that live at least until the next call.
    unsafe { CStr::from_ptr(p) }.to_string_lossy().into_owned()
}

/// The library's status codes as the reference's error kinds (`laya-core/src/error.rs`).
fn status(rc: i32, msg: String) -> Result<()> {
    match rc {
        ffi::S1C_OK => Ok(()),
        ffi::S1C_ERR_WEIGHTS => Err(Error::Weights(msg)),
        ffi::S1C_ERR_CONFIG => Err(Error::Config(msg)),
        _ => Err(Error::Backend(msg)),
    }
}

/// The model forward of one GPU. Calls are serialised on the handle (the reference runs every
/// forward on its single inference thread).
pub struct CudaBackend {
    h: Mutex<*mut ffi::s1c_backend>,
    hidden: usize,
    name: String,
    kernels: &'static [&'static str],
}

// SAFETY: the handle is only used under the mutex; libs1c allows a handle to move between threads.
unsafe impl Send for CudaBackend {}
unsafe impl Sync for CudaBackend {}

impl Drop for CudaBackend {
    fn drop(&mut self) {
        let h = *self.h.get_mut().unwrap();
        if !h.is_null() {
            // SAFETY: the handle came from s1c_create and is destroyed once.
            unsafe { ffi::s1c_destroy(h) };
        }
    }
}

impl CudaBackend {
    /// Build the backend on GPU `device` from the checkpoint's tensors (F32 / F16 / BF16 / F64
    /// converted at load) with the library settings `settings`.
    pub fn new(w: &Weights, cfg: &ModelConfig, device: i32, settings: &str) -> Result<Self> {
        let e = &cfg.encoder;
        let local: Vec<u8> = e.layer_is_local.iter().map(|&l| l as u8).collect();
        let desc = ffi::s1c_model_desc {
            vocab_size: e.vocab_size as i32,
            hidden_size: e.hidden_size as i32,
            num_layers: e.num_hidden_layers as i32,
            num_heads: e.num_attention_heads as i32,
            intermediate_size: e.intermediate_size as i32,
            norm_eps: e.norm_eps as f32,
            local_attention: e.local_attention as i32,
            global_rope_theta: e.global_rope_theta as f32,
            local_rope_theta: e.local_rope_theta as f32,
            layer_is_local: local.as_ptr(),
            head_layers: cfg.agent.head_layers as i32,
            max_position: e.max_position_embeddings as i32,
            max_tokens: 16384,
        };
        // Views into the mapping: names, dtypes, shapes and data pointers of every float tensor.
        let st = w.view()?;
        let mut names = Vec::new();
        let mut tensors = Vec::new();
        for (name, t) in st.tensors() {
            let dtype = match t.dtype() {
                Dtype::F32 => ffi::S1C_DT_F32,
                Dtype::F16 => ffi::S1C_DT_F16,
                Dtype::BF16 => ffi::S1C_DT_BF16,
                Dtype::F64 => ffi::S1C_DT_F64,
                _ => continue, // integer buffers are not weights
            };
            if t.shape().len() > 4 {
                return Err(Error::Weights(format!("{name}: more than 4 dimensions")));
            }
            let mut shape = [0i64; 4];
            for (i, &s) in t.shape().iter().enumerate() {
                shape[i] = s as i64;
            }
            let cname = CString::new(name.as_str()).map_err(|e| Error::Weights(e.to_string()))?;
            tensors.push(ffi::s1c_tensor {
                name: cname.as_ptr(),
                dtype,
                ndim: t.shape().len() as i32,
                shape,
                data: t.data().as_ptr().cast(),
            });
            names.push(cname);
        }
        let settings = CString::new(settings).map_err(|e| Error::Config(e.to_string()))?;
        let mut h = std::ptr::null_mut();
        // SAFETY: every pointer in `desc` and `tensors` stays valid for the call (the library copies).
        let rc = unsafe {
            ffi::s1c_create_with_settings(&desc, tensors.as_ptr(), tensors.len() as i32, device, settings.as_ptr(),
                                          &mut h)
        };
        status(rc, text(unsafe { ffi::s1c_create_error() }))?;
        let name = text(unsafe { ffi::s1c_name(h) });
        // Backend::active_kernels returns 'static names: one small leak per backend built.
        let list: Vec<&'static str> = text(unsafe { ffi::s1c_active_kernels(h) })
            .split(',')
            .map(|s| &*Box::leak(s.trim().to_string().into_boxed_str()))
            .filter(|s| !s.is_empty())
            .collect();
        Ok(Self { h: Mutex::new(h), hidden: e.hidden_size, name, kernels: Box::leak(list.into_boxed_slice()) })
    }

    fn cbatch(b: &Batch) -> ffi::s1c_batch {
        ffi::s1c_batch {
            n: b.n,
            len: b.len,
            kmax: b.kmax,
            input_ids: b.input_ids.as_ptr(),
            attention_mask: b.attention_mask.as_ptr(),
            seq_lens: b.seq_lens.as_ptr(),
            marker_pos: b.marker_pos.as_ptr(),
            marker_count: b.marker_count.as_ptr(),
            qtype: b.qtype.as_ptr(),
        }
    }

    fn check(h: *mut ffi::s1c_backend, rc: i32) -> Result<()> {
        if rc == ffi::S1C_OK {
            return Ok(());
        }
        status(rc, text(unsafe { ffi::s1c_last_error(h) }))
    }

    /// The raw handle, for [`Server::new`] (which then owns the handle's forwards).
    fn raw(&self) -> *mut ffi::s1c_backend {
        *self.h.lock().unwrap()
    }
}

impl Backend for CudaBackend {
    fn name(&self) -> String {
        self.name.clone()
    }

    fn forward(&self, b: &Batch) -> Result<BackendOutput> {
        let h = self.h.lock().unwrap();
        let cb = Self::cbatch(b);
        let mut logits = vec![0f32; b.n * b.kmax];
        let mut pooled = vec![0f32; b.n * self.hidden];
        // SAFETY: the batch's vectors and the outputs outlive the call.
        let rc = unsafe { ffi::s1c_forward_padded(*h, &cb, logits.as_mut_ptr(), pooled.as_mut_ptr()) };
        Self::check(*h, rc)?;
        Ok(BackendOutput { logits, pooled })
    }

    fn active_kernels(&self) -> &'static [&'static str] {
        self.kernels
    }

    fn padded_len(&self, len: usize, rows: usize) -> usize {
        let h = self.h.lock().unwrap();
        // SAFETY: plain query on a live handle.
        unsafe { ffi::s1c_padded_len(*h, len, rows) }
    }

    fn warmup(&self) -> Result<()> {
        let h = self.h.lock().unwrap();
        let rc = unsafe { ffi::s1c_warmup(*h) };
        Self::check(*h, rc)
    }

    /// Real positions hold the encoder's final hidden state, and so do padding positions within
    /// `local_attention / 2` of the row's last real token, as the reference computes them;
    /// padding positions farther away are 0 (`forward` does not depend on any of them).
    fn encoder_hidden(&self, b: &Batch) -> Result<Option<Vec<f32>>> {
        let h = self.h.lock().unwrap();
        let cb = Self::cbatch(b);
        let mut out = vec![0f32; b.n * b.len * self.hidden];
        let rc = unsafe { ffi::s1c_encoder_hidden(*h, &cb, out.as_mut_ptr()) };
        Self::check(*h, rc)?;
        Ok(Some(out))
    }
}

/// Split `device=<n>` off the settings list; the rest goes to the library.
fn device_and_settings(opts: &BackendOptions) -> Result<(i32, String)> {
    let mut device = 0i32;
    let mut rest = Vec::new();
    for kv in opts.settings().split(',').filter(|s| !s.is_empty()) {
        match kv.split_once('=') {
            Some(("device", v)) => {
                device = v
                    .parse()
                    .map_err(|_| Error::Config(format!("settings: `{kv}`: `{v}` is not a whole number")))?
            }
            _ => rest.push(kv),
        }
    }
    Ok((device, rest.join(",")))
}

/// Build the CUDA backend from a checkpoint: the signature of `laya_mlx::make_backend`
/// (`laya-mlx/src/lib.rs:593-600`), so `Agent::load(dir, &opts, Box::new(laya_cuda::make_backend))`
/// loads the model onto the GPU.
pub fn make_backend(w: &Weights, cfg: &ModelConfig, opts: &BackendOptions) -> Result<Box<dyn Backend>> {
    let (device, settings) = device_and_settings(opts)?;
    Ok(Box::new(CudaBackend::new(w, cfg, device, &settings)?))
}

/// Factory for [`laya_core::testing::run_parity`].
pub fn factory() -> laya_core::testing::Factory {
    Box::new(make_backend)
}

/// Cross-request batching over GPU workers (`s1c_server_*`): one worker per backend packs queued
/// requests into varlen batches. Backends may sit on different GPUs: each worker drives its own.
/// Submitting never blocks; over the admission cap it returns [`Submit::Busy`] (the 503 with
/// `Retry-After: 1`, `sys1rust/src/http.rs:168-230`).
pub struct Server {
    s: *mut ffi::s1c_server,
    hidden: usize,
    _backends: Vec<CudaBackend>,
}

// SAFETY: libs1c's serving calls are thread-safe on one server.
unsafe impl Send for Server {}
unsafe impl Sync for Server {}

pub enum Submit {
    Ticket(u64),
    Busy,
    NotRunning,
}

impl Server {
    /// Take ownership of `backends` (one worker each; they may be on different GPUs).
    pub fn new(backends: Vec<CudaBackend>, opts: ffi::s1c_server_opts) -> Result<Self> {
        let hidden = backends.first().map(|b| b.hidden).ok_or_else(|| Error::Config("no backends".into()))?;
        let raw: Vec<*mut ffi::s1c_backend> = backends.iter().map(|b| b.raw()).collect();
        let mut s = std::ptr::null_mut();
        let rc = unsafe { ffi::s1c_server_create(raw.as_ptr(), raw.len() as i32, &opts, &mut s) };
        status(rc, text(unsafe { ffi::s1c_create_error() }))?;
        Ok(Self { s, hidden, _backends: backends })
    }

    /// Queue one tokenised row (`collate_to`'s row layout) with its marker positions.
    pub fn submit(&self, ids: &[u32], markers: &[u32], qtype: u32) -> Result<Submit> {
        let req = ffi::s1c_request {
            ids: ids.as_ptr(),
            len: ids.len() as i32,
            marker_pos: markers.as_ptr(),
            n_markers: markers.len() as i32,
            qtype,
        };
        let mut ticket = 0u64;
        match unsafe { ffi::s1c_server_submit(self.s, &req, &mut ticket) } {
            ffi::S1C_OK => Ok(Submit::Ticket(ticket)),
            ffi::S1C_ERR_BUSY => Ok(Submit::Busy),
            ffi::S1C_ERR_DEAD => Ok(Submit::NotRunning),
            rc => status(rc, text(unsafe { ffi::s1c_create_error() })).map(|_| Submit::Busy),
        }
    }

    /// Wait for and collect a result: the row's marker logits and its pooled state.
    pub fn wait(&self, ticket: u64, n_markers: usize) -> Result<(Vec<f32>, Vec<f32>)> {
        let (mut logits, mut pooled) = (vec![0f32; n_markers], vec![0f32; self.hidden]);
        let rc = unsafe {
            ffi::s1c_server_wait(self.s, ticket, -1, logits.as_mut_ptr(), pooled.as_mut_ptr(), std::ptr::null_mut())
        };
        status(rc, text(unsafe { ffi::s1c_create_error() }))?;
        Ok((logits, pooled))
    }

    /// The client went away: drop the request (unrun if still queued).
    pub fn cancel(&self, ticket: u64) {
        unsafe { ffi::s1c_server_cancel(self.s, ticket) };
    }

    pub fn stats(&self) -> ffi::s1c_server_stats {
        let mut st = ffi::s1c_server_stats::default();
        unsafe { ffi::s1c_server_get_stats(self.s, &mut st) };
        st
    }
}

impl Drop for Server {
    fn drop(&mut self) {
        // stops the workers before the backends they drive are destroyed
        unsafe { ffi::s1c_server_destroy(self.s) };
    }
}
