//! Raw declarations of include/glypr_cuda.h, one for one (a CPU test of this repository parses
//! both files and checks every function's name, parameter count and parameter types).
#![allow(non_camel_case_types)]

use std::ffi::{c_char, c_double, c_float, c_int, c_void};

pub const GLP_OK: c_int = 0;
pub const GLP_ERR_INVALID_ARG: c_int = 1;
pub const GLP_ERR_IO: c_int = 2;
pub const GLP_ERR_FORMAT: c_int = 3;
pub const GLP_ERR_UNSUPPORTED: c_int = 4;
pub const GLP_ERR_CUDA: c_int = 5;
pub const GLP_ERR_OOM: c_int = 6;
pub const GLP_ERR_DEVICE: c_int = 7;
pub const GLP_ERR_CONTEXT_LIMIT: c_int = 8;
pub const GLP_MAX_DEVICES: usize = 16;
pub const GLP_PROFILE_KINDS: usize = 14;
pub const GLP_TOKENS_BARE: c_int = 0;
pub const GLP_TOKENS_SINGLE: c_int = 1;
pub const GLP_TOKENS_SEQUENCE: c_int = 2;
pub const GLP_DEFAULT_MAX_SEQ_LEN: c_int = 8320;

#[repr(C)]
pub struct glp_ctx {
    _private: [u8; 0],
}
#[repr(C)]
pub struct glp_engine {
    _private: [u8; 0],
}
#[repr(C)]
pub struct glp_tokenizer {
    _private: [u8; 0],
}

#[repr(C)]
#[derive(Clone, Copy, Debug, Default)]
pub struct glp_options {
    pub max_batch_tokens: i64,
    pub max_batch_seqs: c_int,
    pub device_memory_limit_mib: c_int,
    pub reserved: [c_int; 5],
}

#[repr(C)]
#[derive(Clone, Copy, Debug, Default)]
pub struct glp_model_info_t {
    pub n_layers: c_int,
    pub hidden: c_int,
    pub ffn: c_int,
    pub n_heads: c_int,
    pub n_kv_heads: c_int,
    pub head_dim: c_int,
    pub vocab: c_int,
    pub embedding_dim: c_int,
    pub max_position: c_int,
    pub sliding_window: c_int,
    pub weight_type: c_int,
    pub n_devices: c_int,
    pub device_bytes: i64,
}

#[repr(C)]
#[derive(Clone, Copy, Debug, Default)]
pub struct glp_timing {
    pub n_devices: c_int,
    pub device_ms: [c_float; GLP_MAX_DEVICES],
}

#[repr(C)]
#[derive(Clone, Copy, Debug)]
pub struct glp_profile {
    pub n_kinds: c_int,
    pub names: [*const c_char; GLP_PROFILE_KINDS],
    pub launches: [i64; GLP_PROFILE_KINDS],
    pub total_ms: [c_double; GLP_PROFILE_KINDS],
    pub flops: [c_double; GLP_PROFILE_KINDS],
    pub bytes: [c_double; GLP_PROFILE_KINDS],
    pub total_launches: i64,
}

pub type glp_batch_fn = Option<
    unsafe extern "C" fn(
        user: *mut c_void,
        ids: *const i32,
        lengths: *const i32,
        n_seq: c_int,
        max_len: c_int,
        out_dim: c_int,
        out: *mut c_float,
    ) -> c_int,
>;

extern "C" {
    pub fn glp_open(
        gguf_path: *const c_char,
        device_ids: *const c_int,
        n_devices: c_int,
        opt: *const glp_options,
        out: *mut *mut glp_ctx,
    ) -> c_int;
    pub fn glp_close(ctx: *mut glp_ctx);
    pub fn glp_last_error() -> *const c_char;
    pub fn glp_model_info(ctx: *const glp_ctx, info: *mut glp_model_info_t) -> c_int;
    pub fn glp_embed_tokens(
        ctx: *mut glp_ctx,
        ids: *const i32,
        lengths: *const i32,
        n_seq: c_int,
        max_len: c_int,
        out_dim: c_int,
        out: *mut c_float,
        timing: *mut glp_timing,
    ) -> c_int;
    pub fn glp_embed_tokens_sharded(
        fns: *const glp_batch_fn,
        users: *const *mut c_void,
        n_executors: c_int,
        embedding_dim: c_int,
        ids: *const i32,
        lengths: *const i32,
        n_seq: c_int,
        max_len: c_int,
        out_dim: c_int,
        out: *mut c_float,
    ) -> c_int;
    pub fn glp_embed_packed_device(
        ctx: *mut glp_ctx,
        dev_index: c_int,
        d_ids: *const i32,
        d_cu_seqlens: *const i32,
        h_cu_seqlens: *const i32,
        n_seq: c_int,
        out_dim: c_int,
        d_out: *mut c_float,
        stream: *mut c_void,
    ) -> c_int;
    pub fn glp_device_status(ctx: *mut glp_ctx, dev_index: c_int, status: *mut c_int) -> c_int;
    pub fn glp_status_text(status: c_int) -> *const c_char;
    pub fn glp_profile_enable(ctx: *mut glp_ctx, dev_index: c_int, enable: c_int) -> c_int;
    pub fn glp_profile_read(ctx: *mut glp_ctx, dev_index: c_int, out: *mut glp_profile) -> c_int;
    pub fn glp_engine_create(
        ctx: *mut glp_ctx,
        max_batch: c_int,
        queue_capacity: c_int,
        out: *mut *mut glp_engine,
    ) -> c_int;
    pub fn glp_engine_create_with_executor(
        fn_: glp_batch_fn,
        user: *mut c_void,
        embedding_dim: c_int,
        max_batch: c_int,
        queue_capacity: c_int,
        out: *mut *mut glp_engine,
    ) -> c_int;
    pub fn glp_engine_embed(
        e: *mut glp_engine,
        ids: *const i32,
        len: c_int,
        truncate_dim: c_int,
        out: *mut c_float,
    ) -> c_int;
    pub fn glp_engine_stats(
        e: *mut glp_engine,
        requests: *mut i64,
        batches: *mut i64,
        largest_batch: *mut c_int,
    ) -> c_int;
    pub fn glp_engine_destroy(e: *mut glp_engine);
    pub fn glp_tokenizer_from_gguf(gguf_path: *const c_char, out: *mut *mut glp_tokenizer) -> c_int;
    pub fn glp_tokenizer_from_vocab(
        tokens: *const *const c_char,
        n_tokens: c_int,
        merges: *const *const c_char,
        n_merges: c_int,
        out: *mut *mut glp_tokenizer,
    ) -> c_int;
    pub fn glp_tokenizer_free(tok: *mut glp_tokenizer);
    pub fn glp_tokenizer_info(tok: *const glp_tokenizer, n_tokens: *mut c_int, n_merges: *mut c_int) -> c_int;
    pub fn glp_tokenize(
        tok: *const glp_tokenizer,
        text: *const c_char,
        text_len: usize,
        form: c_int,
        ids: *mut i32,
        cap: c_int,
        n_ids: *mut c_int,
    ) -> c_int;
    pub fn glp_tokenize_batch(
        tok: *const glp_tokenizer,
        texts: *const *const c_char,
        text_lens: *const usize,
        n_texts: c_int,
        form: c_int,
        limit: c_int,
        n_threads: c_int,
        ids: *mut i32,
        ids_cap: usize,
        offsets: *mut i64,
    ) -> c_int;
    pub fn glp_format_query(
        query: *const c_char,
        query_len: usize,
        task: *const c_char,
        out: *mut c_char,
        cap: usize,
        n_out: *mut usize,
    ) -> c_int;
    pub fn glp_format_document(
        content: *const c_char,
        content_len: usize,
        title: *const c_char,
        out: *mut c_char,
        cap: usize,
        n_out: *mut usize,
    ) -> c_int;
    pub fn glp_task_format(
        task: *const c_char,
        title: *const c_char,
        text: *const c_char,
        text_len: usize,
        out: *mut c_char,
        cap: usize,
        n_out: *mut usize,
    ) -> c_int;
    pub fn glp_embed_texts(
        ctx: *mut glp_ctx,
        tok: *const glp_tokenizer,
        texts: *const *const c_char,
        text_lens: *const usize,
        n_texts: c_int,
        form: c_int,
        max_seq_len: c_int,
        out_dim: c_int,
        out: *mut c_float,
    ) -> c_int;
    pub fn glp_engine_embed_text(
        e: *mut glp_engine,
        tok: *const glp_tokenizer,
        text: *const c_char,
        text_len: usize,
        task: *const c_char,
        title: *const c_char,
        truncate_dim: c_int,
        out: *mut c_float,
    ) -> c_int;
    pub fn glp_q8_0_dequant(d_blocks: *const c_void, n_blocks: i64, d_out: *mut c_float, stream: *mut c_void) -> c_int;
    pub fn glp_q8_0_gemm(
        d_q8_w: *const c_void,
        n: c_int,
        k: c_int,
        d_x_bf16: *const c_void,
        m: c_int,
        d_y: *mut c_void,
        y_is_f32: c_int,
        stream: *mut c_void,
    ) -> c_int;
    pub fn glp_q8_0_gemm_noalloc(
        d_q8_w: *const c_void,
        n: c_int,
        k: c_int,
        d_x_bf16: *const c_void,
        m: c_int,
        d_y: *mut c_void,
        y_is_f32: c_int,
        stream: *mut c_void,
    ) -> c_int;
    pub fn glp_kernel_status(device: c_int, status: *mut c_int) -> c_int;
    pub fn glp_selftest_wait_timeout(device: c_int, limit_us: c_int) -> c_int;
    pub fn glp_bf16_gemm(
        d_w_bf16: *const c_void,
        n: c_int,
        k: c_int,
        d_x_bf16: *const c_void,
        m: c_int,
        d_y: *mut c_void,
        y_is_f32: c_int,
        stream: *mut c_void,
    ) -> c_int;
    pub fn glp_gate_up_geglu(
        d_w_gate: *const c_void,
        d_w_up: *const c_void,
        f: c_int,
        k: c_int,
        d_x: *const c_void,
        m: c_int,
        d_out: *mut c_void,
        stream: *mut c_void,
    ) -> c_int;
    pub fn glp_qkv_norm_rope(
        d_w_qkv: *const c_void,
        n_q_heads: c_int,
        n_kv_heads: c_int,
        k: c_int,
        d_x: *const c_void,
        m: c_int,
        d_q_gain: *const c_float,
        d_k_gain: *const c_float,
        d_pos: *const i32,
        theta: c_double,
        max_pos: c_int,
        eps: c_float,
        d_out: *mut c_void,
        stream: *mut c_void,
    ) -> c_int;
    pub fn glp_flash_attention(
        d_qkv: *const c_void,
        d_cu_seqlens: *const i32,
        n_seq: c_int,
        max_len: c_int,
        n_q_heads: c_int,
        n_kv_heads: c_int,
        head_dim: c_int,
        window: c_int,
        d_out: *mut c_void,
        stream: *mut c_void,
    ) -> c_int;
}
