//! Safe Rust binding of libglypr_cuda.so, shaped after the seams of glypr-core
//! (crates/glypr-core/src) that the B200 backend sits behind:
//!
//! * [`CudaEmbedder`] -- the whole-model path: `GlyprEmbedder::load_gguf_q8` (lib.rs:176-229)
//!   and `embed_batch` on token ids (lib.rs:731-952, `EmbeddingGemma2Model::forward` +
//!   `pool_and_normalize`, model.rs:498-705).  Returns `Vec<Vec<f32>>` like the reference.
//! * [`CudaQ8Linear`] -- a `LinearOp::CudaQ8_0 { weight_q8_bytes, out_dim, in_dim }` variant
//!   beside `MetalQ8_0` (linear.rs:6-15, forward at linear.rs:150-172) over device pointers.
//! * [`flash_attention`] -- the `AttentionMode::CudaFlash` slot (attention/mod.rs:255-262,
//!   `AttentionBackend::compute_attention`, attention/traits.rs:37-46).
//! * [`Engine`] -- the server's batching worker (glypr-server/src/engine.rs:157-325).
//! * [`Tokenizer`] -- `GlyprTokenizer::from_gguf_metadata` / `encode` (tokenizer.rs:77-229).
//!
//! Errors carry the library's message, which reuses the reference's texts (for example
//! "Input sequence length (n) exceeds model max_position_embeddings (m)", model.rs:500-506).

pub mod ffi;

use std::ffi::{c_int, c_void, CStr, CString};
use std::fmt;
use std::ptr;

/// A failed call: the library's status code and its `glp_last_error()` message.
#[derive(Debug, Clone, PartialEq, Eq)]
pub struct GlpError {
    pub code: i32,
    pub message: String,
}

impl fmt::Display for GlpError {
    fn fmt(&self, f: &mut fmt::Formatter<'_>) -> fmt::Result {
        write!(f, "[glp error {}] {}", self.code, self.message)
    }
}

impl std::error::Error for GlpError {}

pub type Result<T> = std::result::Result<T, GlpError>;

fn check(rc: c_int) -> Result<()> {
    if rc == ffi::GLP_OK {
        return Ok(());
    }
    // the message is thread-local in the library: read it on the failing thread, right away
    let message = unsafe { CStr::from_ptr(ffi::glp_last_error()) }.to_string_lossy().into_owned();
    Err(GlpError { code: rc, message })
}

fn cstring(s: &str) -> Result<CString> {
    CString::new(s).map_err(|_| GlpError { code: ffi::GLP_ERR_INVALID_ARG, message: "string contains NUL".into() })
}

/// Options of `glp_open` (launch-chunk size and the per-device memory limit).
#[derive(Clone, Copy, Debug, Default)]
pub struct OpenOptions {
    pub max_batch_tokens: i64,
    pub max_batch_seqs: i32,
    pub device_memory_limit_mib: i32,
}

/// A GGUF model replicated on one or more GPUs (the reference's `GlyprEmbedder` for its text
/// path).  Calls may come from one thread at a time; the library runs one worker per device.
pub struct CudaEmbedder {
    ctx: *mut ffi::glp_ctx,
    info: ffi::glp_model_info_t,
}

// The context is used from one thread at a time (it is not Sync); moving it is fine.
unsafe impl Send for CudaEmbedder {}

impl CudaEmbedder {
    /// `GlyprEmbedder::load_gguf_q8(path, device)`: parse the GGUF (config.rs:76-250 keys) and
    /// upload one replica per device in `devices` (empty: the current CUDA device).
    pub fn load_gguf(path: &str, devices: &[i32], options: OpenOptions) -> Result<Self> {
        let p = cstring(path)?;
        let opt = ffi::glp_options {
            max_batch_tokens: options.max_batch_tokens,
            max_batch_seqs: options.max_batch_seqs,
            device_memory_limit_mib: options.device_memory_limit_mib,
            reserved: [0; 5],
        };
        let mut ctx = ptr::null_mut();
        let ids = if devices.is_empty() { ptr::null() } else { devices.as_ptr() };
        check(unsafe { ffi::glp_open(p.as_ptr(), ids, devices.len() as c_int, &opt, &mut ctx) })?;
        let mut info = ffi::glp_model_info_t::default();
        if let Err(e) = check(unsafe { ffi::glp_model_info(ctx, &mut info) }) {
            unsafe { ffi::glp_close(ctx) };
            return Err(e);
        }
        Ok(Self { ctx, info })
    }

    pub fn info(&self) -> &ffi::glp_model_info_t {
        &self.info
    }

    pub fn embedding_dim(&self) -> usize {
        self.info.embedding_dim as usize
    }

    /// Right-padded ids `[n_seq * max_len]` and `lengths` -> L2-normalised embeddings of
    /// `out_dim` values (Matryoshka-truncated and renormalised below the model's width).
    pub fn embed_ids(&self, ids: &[i32], lengths: &[i32], max_len: usize, out_dim: usize) -> Result<Vec<Vec<f32>>> {
        let n = lengths.len();
        if ids.len() < n * max_len {
            return Err(GlpError { code: ffi::GLP_ERR_INVALID_ARG, message: "ids shorter than n_seq * max_len".into() });
        }
        let mut out = vec![0f32; n * out_dim];
        check(unsafe {
            ffi::glp_embed_tokens(
                self.ctx,
                ids.as_ptr(),
                lengths.as_ptr(),
                n as c_int,
                max_len as c_int,
                out_dim as c_int,
                out.as_mut_ptr(),
                ptr::null_mut(),
            )
        })?;
        Ok(out.chunks(out_dim.max(1)).map(|c| c.to_vec()).collect())
    }

    /// `embed_batch` on token-id sequences (lib.rs:731-952 after tokenisation): pads them,
    /// embeds them and returns one vector per sequence; `truncate_dim` as the reference's.
    pub fn embed_batch(&self, sequences: &[Vec<u32>], truncate_dim: Option<usize>) -> Result<Vec<Vec<f32>>> {
        if sequences.is_empty() {
            return Ok(Vec::new());
        }
        let max_len = sequences.iter().map(|s| s.len()).max().unwrap_or(0).max(1);
        let mut ids = vec![0i32; sequences.len() * max_len];
        let mut lengths = Vec::with_capacity(sequences.len());
        for (i, s) in sequences.iter().enumerate() {
            for (j, &t) in s.iter().enumerate() {
                ids[i * max_len + j] = t as i32;
            }
            lengths.push(s.len() as i32);
        }
        let dim = truncate_dim.unwrap_or(self.embedding_dim()).min(self.embedding_dim());
        self.embed_ids(&ids, &lengths, max_len, dim)
    }

    /// Status word of the device kernels' bounded waits on device `dev_index` (0 = none).
    pub fn device_status(&self, dev_index: usize) -> Result<i32> {
        let mut st: c_int = 0;
        check(unsafe { ffi::glp_device_status(self.ctx, dev_index as c_int, &mut st) })?;
        Ok(st)
    }

    pub(crate) fn raw(&self) -> *mut ffi::glp_ctx {
        self.ctx
    }
}

impl Drop for CudaEmbedder {
    fn drop(&mut self) {
        unsafe { ffi::glp_close(self.ctx) }
    }
}

/// `LinearOp::CudaQ8_0`: a Q8_0 linear whose raw GGUF rows (`[out_dim, in_dim / 32 * 34]`
/// bytes, the layout `LinearOp::MetalQ8_0` keeps) live in device memory owned by the caller.
pub struct CudaQ8Linear {
    pub weight_q8_bytes: *const c_void,
    pub out_dim: usize,
    pub in_dim: usize,
}

impl CudaQ8Linear {
    /// `forward(x)`: y[m, out_dim] = x[m, in_dim] (bf16, device) * dequant(W)^T, y f32 or bf16,
    /// stream-ordered on `stream` (a cudaStream_t; null = the legacy default stream).
    ///
    /// # Safety
    /// `x` and `y` must be device pointers of at least `m * in_dim` bf16 and `m * out_dim`
    /// outputs on the current CUDA device.
    pub unsafe fn forward(&self, x: *const c_void, m: usize, y: *mut c_void, y_is_f32: bool, stream: *mut c_void) -> Result<()> {
        check(ffi::glp_q8_0_gemm(
            self.weight_q8_bytes,
            self.out_dim as c_int,
            self.in_dim as c_int,
            x,
            m as c_int,
            y,
            y_is_f32 as c_int,
            stream,
        ))
    }
}

/// `AttentionMode::CudaFlash` over a packed, normed and RoPE'd qkv tensor
/// `[T, (n_q_heads + 2 n_kv_heads) * 256]` f16 with sequence offsets `cu_seqlens[n_seq + 1]`
/// (device); `window > 0` applies |i - j| <= window.  Writes `[T, n_q_heads * 256]` f16.
///
/// # Safety
/// All pointers are device pointers on the current CUDA device, sized as described.
#[allow(clippy::too_many_arguments)]
pub unsafe fn flash_attention(
    qkv: *const c_void,
    cu_seqlens: *const i32,
    n_seq: usize,
    max_len: usize,
    n_q_heads: usize,
    n_kv_heads: usize,
    window: usize,
    out: *mut c_void,
    stream: *mut c_void,
) -> Result<()> {
    check(ffi::glp_flash_attention(
        qkv,
        cu_seqlens,
        n_seq as c_int,
        max_len as c_int,
        n_q_heads as c_int,
        n_kv_heads as c_int,
        256,
        window as c_int,
        out,
        stream,
    ))
}

/// Status of the kernel-level entry points on `device`: Ok(0) when no bounded wait expired.
pub fn kernel_status(device: i32) -> Result<i32> {
    let mut st: c_int = 0;
    check(unsafe { ffi::glp_kernel_status(device, &mut st) })?;
    Ok(st)
}

/// The server's batching worker over a model context (`EngineHandle`, engine.rs:120-150):
/// `embed` may be called from any number of threads and blocks until its batch is done.
pub struct Engine<'a> {
    e: *mut ffi::glp_engine,
    dim: usize,
    _ctx: std::marker::PhantomData<&'a CudaEmbedder>,
}

unsafe impl Send for Engine<'_> {}
unsafe impl Sync for Engine<'_> {}

impl<'a> Engine<'a> {
    /// While the engine runs it is the context's only caller (the borrow enforces it).
    pub fn new(model: &'a mut CudaEmbedder, max_batch: usize, queue_capacity: usize) -> Result<Self> {
        let mut e = ptr::null_mut();
        check(unsafe { ffi::glp_engine_create(model.raw(), max_batch as c_int, queue_capacity as c_int, &mut e) })?;
        Ok(Self { e, dim: model.embedding_dim(), _ctx: std::marker::PhantomData })
    }

    pub fn embed(&self, ids: &[i32], truncate_dim: Option<usize>) -> Result<Vec<f32>> {
        let d = match truncate_dim {
            Some(t) if t > 0 && t < self.dim => t,
            _ => self.dim,
        };
        let mut out = vec![0f32; d];
        let td = if d == self.dim { 0 } else { d as c_int };
        check(unsafe { ffi::glp_engine_embed(self.e, ids.as_ptr(), ids.len() as c_int, td, out.as_mut_ptr()) })?;
        Ok(out)
    }
}

impl Drop for Engine<'_> {
    fn drop(&mut self) {
        unsafe { ffi::glp_engine_destroy(self.e) }
    }
}

/// The GGUF BPE tokenizer (`GlyprTokenizer::from_gguf_metadata`, tokenizer.rs:77-138).
pub struct Tokenizer {
    t: *mut ffi::glp_tokenizer,
}

unsafe impl Send for Tokenizer {}
unsafe impl Sync for Tokenizer {}

impl Tokenizer {
    pub fn from_gguf(path: &str) -> Result<Self> {
        let p = cstring(path)?;
        let mut t = ptr::null_mut();
        check(unsafe { ffi::glp_tokenizer_from_gguf(p.as_ptr(), &mut t) })?;
        Ok(Self { t })
    }

    /// Ids of `text` in one of the GLP_TOKENS_* forms (`GlyprTokenizer::encode` is
    /// `ffi::GLP_TOKENS_SINGLE`, the batch and server path `ffi::GLP_TOKENS_SEQUENCE`).
    pub fn encode(&self, text: &str, form: i32) -> Result<Vec<u32>> {
        let cap = 3 * text.len() + 2;
        let mut ids = vec![0i32; cap.max(1)];
        let mut n: c_int = 0;
        check(unsafe {
            ffi::glp_tokenize(self.t, text.as_ptr().cast(), text.len(), form, ids.as_mut_ptr(), ids.len() as c_int, &mut n)
        })?;
        ids.truncate(n as usize);
        Ok(ids.into_iter().map(|v| v as u32).collect())
    }
}

impl Drop for Tokenizer {
    fn drop(&mut self) {
        unsafe { ffi::glp_tokenizer_free(self.t) }
    }
}
