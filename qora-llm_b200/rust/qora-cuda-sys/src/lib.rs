//! Raw bindings of `include/qora_cuda.h`, the C ABI of libqora_cuda.so (the B200 engine
//! that replaces the reference crate's `forward_decode_raw` / `raw_prefill` math,
//! src/gemv.rs:872-1190). Every item below has the same name, field order and types as
//! its C declaration; `tests/test_rust_binding.py` checks that against the header.
//! The safe layer with the reference's names is in [`safe`].
#![allow(non_camel_case_types)]

use std::os::raw::{c_char, c_int, c_void};

pub mod safe;

pub type qora_status = c_int;

pub const QORA_OK: qora_status = 0;
pub const QORA_ERR_INVALID: qora_status = 1;
pub const QORA_ERR_IO: qora_status = 2;
pub const QORA_ERR_CUDA: qora_status = 3;
pub const QORA_ERR_OOM: qora_status = 4;
pub const QORA_ERR_RANGE: qora_status = 5;
pub const QORA_ERR_TIMEOUT: qora_status = 6;
pub const QORA_ERR_UNSUPPORTED: qora_status = 7;
pub const QORA_ERR_NCCL: qora_status = 8;

pub const QORA_FORMAT_F16: u32 = 0;
pub const QORA_FORMAT_Q4: u32 = 1;
pub const QORA_FLAG_PER_OP_KERNELS: u32 = 1;
pub const QORA_FLAG_TOKEN_PREFILL: u32 = 2;
pub const QORA_PROMPT_TOKEN_STEPS: u32 = 0;
pub const QORA_PROMPT_TENSOR_CORES: u32 = 1;
pub const QORA_KV_F32: u32 = 0;
pub const QORA_KV_F16: u32 = 1;
pub const QORA_GEMV_STATIC_FLOATS: u32 = 512 * 1024;
pub const QORA_GEMV_STATIC_TILES: u32 = 1024;

pub const QORA_KERNEL_QKV: c_int = 0;
pub const QORA_KERNEL_ATTENTION: c_int = 1;
pub const QORA_KERNEL_O: c_int = 2;
pub const QORA_KERNEL_GATE_UP: c_int = 3;
pub const QORA_KERNEL_DOWN: c_int = 4;
pub const QORA_KERNEL_LM_HEAD: c_int = 5;

/// One weight matrix, borrowed (`WeightRef`, src/gemv.rs:66-96): Q4 `packed` + `scales`,
/// or F16 `data`.
#[repr(C)]
#[derive(Clone, Copy, Debug)]
pub struct qora_matrix_view {
    pub packed: *const u8,
    pub scales: *const u16,
    pub data: *const u16,
    pub k: u64,
    pub n: u64,
}

#[repr(C)]
#[derive(Clone, Copy, Debug)]
pub struct qora_layer_view {
    pub q_proj: qora_matrix_view,
    pub k_proj: qora_matrix_view,
    pub v_proj: qora_matrix_view,
    pub o_proj: qora_matrix_view,
    pub gate_proj: qora_matrix_view,
    pub up_proj: qora_matrix_view,
    pub down_proj: qora_matrix_view,
    pub input_norm_gamma: *const u16,
    pub post_attn_norm_gamma: *const u16,
    pub num_heads: u32,
    pub num_kv_heads: u32,
    pub head_dim: u32,
    pub num_kv_groups: u32,
}

/// The borrowed slices of `DecodeWeights` (src/gemv.rs:177-206, `layer_ref` /
/// `embed_ref` :248-271); the engine copies them to the device and keeps no pointer.
#[repr(C)]
#[derive(Clone, Copy, Debug)]
pub struct qora_weights_view {
    pub format: u32,
    pub num_layers: u32,
    pub vocab: u32,
    pub hidden: u32,
    pub rope_half_dim: u32,
    pub no_rope_layers: *const u8,
    pub layers: *const qora_layer_view,
    pub embed: qora_matrix_view,
    pub final_norm_gamma: *const u16,
    pub rope_cos: *const f32,
    pub rope_sin: *const f32,
    pub rope_rows: u64,
}

#[repr(C)]
pub struct qora_engine {
    _private: [u8; 0],
}

#[repr(C)]
pub struct qora_kv {
    _private: [u8; 0],
}

#[repr(C)]
#[derive(Clone, Copy, Debug, Default)]
pub struct qora_engine_options {
    pub n_gpus: i32,
    pub first_device: i32,
    pub flags: u32,
    pub tp_size: i32,
    pub tp_rank: i32,
}

#[repr(C)]
#[derive(Clone, Copy, Debug, Default, PartialEq, Eq)]
pub struct qora_tp_shard {
    pub q_head0: u32,
    pub q_heads: u32,
    pub kv_head0: u32,
    pub kv_heads: u32,
    pub mlp0: u32,
    pub mlp_n: u32,
    pub mlp_padded: u32,
    pub vocab0: u32,
    pub vocab_n: u32,
}

/// The sampling fields of `GenerateParams` (src/generate.rs:8-35).
#[repr(C)]
#[derive(Clone, Copy, Debug)]
pub struct qora_sampling {
    pub temperature: f32,
    pub top_p: f32,
    pub top_k: u32,
    pub repetition_penalty: f32,
    pub presence_penalty: f32,
    pub ban_token: i32,
}

extern "C" {
    pub fn qora_last_error() -> *const c_char;
    pub fn qora_version() -> *const c_char;
    pub fn qora_engine_create_from_file(
        qora_path: *const c_char,
        opts: *const qora_engine_options,
        out: *mut *mut qora_engine,
    ) -> qora_status;
    pub fn qora_engine_create(
        weights: *const qora_weights_view,
        opts: *const qora_engine_options,
        out: *mut *mut qora_engine,
    ) -> qora_status;
    pub fn qora_engine_destroy(engine: *mut qora_engine);
    pub fn qora_tp_export(engine: *mut qora_engine, buf: *mut c_void, cap: usize, len: *mut usize) -> qora_status;
    pub fn qora_tp_plan(
        format: u32,
        num_heads: u32,
        num_kv_heads: u32,
        intermediate: u32,
        vocab: u32,
        tp_size: i32,
        tp_rank: i32,
        out: *mut qora_tp_shard,
    ) -> qora_status;
    pub fn qora_tp_connect(engine: *mut qora_engine, handles: *const c_void, len_per_rank: usize) -> qora_status;
    pub fn qora_engine_info(
        engine: *const qora_engine,
        num_layers: *mut u32,
        vocab: *mut u32,
        hidden: *mut u32,
        format: *mut u32,
        device_bytes: *mut u64,
    ) -> qora_status;
    pub fn qora_kv_create(engine: *mut qora_engine, max_seq: u32, batch: u32, out: *mut *mut qora_kv) -> qora_status;
    pub fn qora_kv_create_ex(
        engine: *mut qora_engine,
        max_seq: u32,
        batch: u32,
        kv_dtype: u32,
        out: *mut *mut qora_kv,
    ) -> qora_status;
    pub fn qora_kv_destroy(kv: *mut qora_kv);
    pub fn qora_kv_length(kv: *const qora_kv, seq_idx: u32, len: *mut u32) -> qora_status;
    pub fn qora_kv_reset(kv: *mut qora_kv, seq_idx: u32) -> qora_status;
    pub fn qora_kv_import(
        kv: *mut qora_kv,
        layer: u32,
        k: *const f32,
        v: *const f32,
        seq_len: u32,
        seq_idx: u32,
    ) -> qora_status;
    pub fn qora_kv_export(
        kv: *const qora_kv,
        layer: u32,
        k: *mut f32,
        v: *mut f32,
        seq_len: u32,
        seq_idx: u32,
    ) -> qora_status;
    pub fn qora_prefill(
        engine: *mut qora_engine,
        kv: *mut qora_kv,
        ids: *const u32,
        n: u32,
        seq_idx: u32,
        logits_or_null: *mut f32,
        argmax_out: *mut u32,
    ) -> qora_status;
    pub fn qora_decode_step(
        engine: *mut qora_engine,
        kv: *mut qora_kv,
        tokens: *const u32,
        logits_or_null: *mut f32,
        argmax_out: *mut u32,
    ) -> qora_status;
    pub fn qora_generate_greedy(
        engine: *mut qora_engine,
        kv: *mut qora_kv,
        first_token: u32,
        n_tokens: u32,
        out_tokens: *mut u32,
    ) -> qora_status;
    pub fn qora_generate_greedy_batch(
        engine: *mut qora_engine,
        kv: *mut qora_kv,
        first_tokens: *const u32,
        n_tokens: u32,
        out_tokens: *mut u32,
        device_ms: *mut f32,
    ) -> qora_status;
    pub fn qora_layer_step(engine: *mut qora_engine, kv: *mut qora_kv, layer: u32, x_inout: *mut f32) -> qora_status;
    pub fn qora_q4_gemv(
        d_x: *const f32,
        d_packed: *const u8,
        d_scales: *const u16,
        k: u64,
        n: u64,
        d_y: *mut f32,
        stream: *mut c_void,
    ) -> qora_status;
    pub fn qora_q4_gemv_static(
        d_x: *const f32,
        d_packed: *const u8,
        d_scales: *const u16,
        k: u64,
        n: u64,
        d_y: *mut f32,
        stream: *mut c_void,
    ) -> qora_status;
    pub fn qora_q4_dequant(
        d_packed: *const u8,
        d_scales: *const u16,
        n: u64,
        row0: u64,
        rows: u64,
        d_out: *mut f32,
        stream: *mut c_void,
    ) -> qora_status;
    pub fn qora_q4_gate_up(
        d_x: *const f32,
        d_gate_packed: *const u8,
        d_gate_scales: *const u16,
        d_up_packed: *const u8,
        d_up_scales: *const u16,
        k: u64,
        n: u64,
        d_out: *mut f32,
        stream: *mut c_void,
    ) -> qora_status;
    pub fn qora_sample(
        engine: *mut qora_engine,
        row: u32,
        history: *const u32,
        n_history: u32,
        params: *const qora_sampling,
        rng_state: *mut u64,
        token_out: *mut u32,
    ) -> qora_status;
    pub fn qora_sample_logits(
        d_logits: *const f32,
        vocab: u32,
        d_history: *const u32,
        n_history: u32,
        params: *const qora_sampling,
        rng_state: *mut u64,
        token_out: *mut u32,
        stream: *mut c_void,
    ) -> qora_status;
    pub fn qora_f16_gemm(
        d_x: *const f32,
        d_w: *const u16,
        m: u64,
        k: u64,
        n: u64,
        d_y: *mut f32,
        stream: *mut c_void,
    ) -> qora_status;
    pub fn qora_q4_lm_head(
        d_x: *const f32,
        d_packed: *const u8,
        d_scales: *const u16,
        vocab: u64,
        hidden: u64,
        d_logits: *mut f32,
        d_argmax: *mut u32,
        stream: *mut c_void,
    ) -> qora_status;
    pub fn qora_generate_greedy_timed(
        engine: *mut qora_engine,
        kv: *mut qora_kv,
        first_token: u32,
        n_tokens: u32,
        out_tokens: *mut u32,
        device_ms: *mut f32,
    ) -> qora_status;
    pub fn qora_engine_time_kernel(
        engine: *mut qora_engine,
        kv: *mut qora_kv,
        kernel: c_int,
        reps: u32,
        ms_per_launch: *mut f32,
        bytes_per_launch: *mut u64,
        launches: *mut u32,
    ) -> qora_status;
    pub fn qora_engine_set_trace(engine: *mut qora_engine, enable: c_int) -> qora_status;
    pub fn qora_engine_get_trace(engine: *mut qora_engine, out: *mut u64, cap: usize, n: *mut usize) -> qora_status;
    pub fn qora_engine_launches_per_step(engine: *const qora_engine, launches: *mut u32) -> qora_status;
    pub fn qora_engine_prompt_path(engine: *const qora_engine, path: *mut u32) -> qora_status;
}
