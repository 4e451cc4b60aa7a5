//! Safe layer over the raw bindings, with the reference crate's names and argument
//! meaning: `load_model` (src/save.rs:154), `DecodeWeights` (src/gemv.rs:177-206),
//! `empty_kv_cache` / `RawKvCache` (src/gemv.rs:154-166), `forward_decode_raw`
//! (src/gemv.rs:872), `raw_prefill` (src/gemv.rs:1027), the greedy branch of
//! `sample_token_top_k` (src/generate.rs:346-352) and the sampling step with penalties
//! (src/generate.rs:345-394, on the device).
//!
//! Error behaviour follows the reference: `load_model` returns `io::Result`, and the
//! forward functions panic on bad input (the panic message carries the library's
//! `qora_last_error()`). Each `try_*` variant returns `Result<_, Error>` instead, for a
//! host that maps failures itself (the reference's GPU path turned panics into
//! `Err(String)`, src/gpu_inference.rs:523-533). Nothing falls back to the CPU.
//!
//! Differences of type, not of meaning: the cache lives on the device, so `RawKvCache`
//! is a handle bound to its engine's lifetime rather than a `Vec` of host rows (import
//! and export move host rows in the reference's token-major layout), and it has a fixed
//! capacity (`max_seq`).

use std::ffi::{CStr, CString};
use std::fmt;
use std::io;
use std::marker::PhantomData;
use std::path::Path;
use std::ptr::{self, NonNull};

use crate::*;

/// Capacity of the caches that `empty_kv_cache` and `raw_prefill` create.
pub const DEFAULT_MAX_SEQ: u32 = 4096;

#[derive(Debug, Clone, PartialEq, Eq)]
pub struct Error {
    pub status: qora_status,
    pub message: String,
}

impl fmt::Display for Error {
    fn fmt(&self, f: &mut fmt::Formatter<'_>) -> fmt::Result {
        write!(f, "qora_cuda status {}: {}", self.status, self.message)
    }
}

impl std::error::Error for Error {}

impl From<Error> for io::Error {
    fn from(e: Error) -> io::Error {
        let kind = match e.status {
            QORA_ERR_INVALID => io::ErrorKind::InvalidData,
            _ => io::ErrorKind::Other,
        };
        io::Error::new(kind, e)
    }
}

fn invalid(message: String) -> Error {
    Error { status: QORA_ERR_INVALID, message }
}

fn last_error() -> String {
    // SAFETY: the library returns a NUL-terminated thread-local string ("" if none).
    unsafe {
        let p = qora_last_error();
        if p.is_null() {
            String::new()
        } else {
            CStr::from_ptr(p).to_string_lossy().into_owned()
        }
    }
}

fn check(status: qora_status) -> Result<(), Error> {
    if status == QORA_OK {
        Ok(())
    } else {
        Err(Error { status, message: last_error() })
    }
}

fn to_u32(n: usize, what: &str) -> Result<u32, Error> {
    u32::try_from(n).map_err(|_| Error { status: QORA_ERR_RANGE, message: format!("{what} {n} exceeds u32") })
}

/// The model resident on one GPU (or one tensor-parallel shard of it).
pub struct DecodeWeights {
    e: NonNull<qora_engine>,
    num_layers: u32,
    vocab: u32,
    hidden: u32,
    format: u32,
}

// An engine is driven by one host thread at a time; it may move between threads.
unsafe impl Send for DecodeWeights {}

impl DecodeWeights {
    /// Load a .qora file with explicit options (device, tensor-parallel rank, flags).
    pub fn try_load(path: &Path, opts: &qora_engine_options) -> Result<Self, Error> {
        let c = CString::new(path.to_string_lossy().into_owned()).map_err(|_| invalid("path contains NUL".into()))?;
        let mut e = ptr::null_mut();
        check(unsafe { qora_engine_create_from_file(c.as_ptr(), opts, &mut e) })?;
        Self::wrap(e)
    }

    /// Upload borrowed host weights (the slices `DecodeWeights` holds).
    ///
    /// # Safety
    /// Every pointer in `view` (and in the layer views it points to) must be valid for
    /// the sizes the view states for the duration of the call.
    pub unsafe fn from_view(view: &qora_weights_view, opts: &qora_engine_options) -> Result<Self, Error> {
        let mut e = ptr::null_mut();
        check(qora_engine_create(view, opts, &mut e))?;
        Self::wrap(e)
    }

    fn wrap(e: *mut qora_engine) -> Result<Self, Error> {
        let e = NonNull::new(e).ok_or_else(|| invalid("the library returned no engine".into()))?;
        let mut w = DecodeWeights { e, num_layers: 0, vocab: 0, hidden: 0, format: 0 };
        let mut bytes = 0u64;
        check(unsafe {
            qora_engine_info(w.e.as_ptr(), &mut w.num_layers, &mut w.vocab, &mut w.hidden, &mut w.format, &mut bytes)
        })?;
        Ok(w)
    }

    pub fn num_layers(&self) -> usize {
        self.num_layers as usize
    }
    pub fn vocab(&self) -> usize {
        self.vocab as usize
    }
    pub fn hidden(&self) -> usize {
        self.hidden as usize
    }
    /// QORA_FORMAT_Q4 or QORA_FORMAT_F16
    pub fn format(&self) -> u32 {
        self.format
    }
    pub fn as_ptr(&self) -> *mut qora_engine {
        self.e.as_ptr()
    }
}

impl Drop for DecodeWeights {
    fn drop(&mut self) {
        unsafe { qora_engine_destroy(self.e.as_ptr()) }
    }
}

/// `save::load_model` (src/save.rs:154): load a .qora file onto GPU 0.
pub fn load_model(path: &Path) -> io::Result<DecodeWeights> {
    DecodeWeights::try_load(path, &qora_engine_options::default()).map_err(io::Error::from)
}

/// A device KV cache: `batch` independent sequences of up to `max_seq` positions.
pub struct RawKvCache<'w> {
    kv: NonNull<qora_kv>,
    batch: u32,
    max_seq: u32,
    _engine: PhantomData<&'w DecodeWeights>,
}

impl<'w> RawKvCache<'w> {
    /// kv_dtype: QORA_KV_F32 (the reference's cache) or QORA_KV_F16 (opt-in binary16).
    pub fn try_new(w: &'w DecodeWeights, max_seq: u32, batch: u32, kv_dtype: u32) -> Result<Self, Error> {
        let mut kv = ptr::null_mut();
        check(unsafe { qora_kv_create_ex(w.as_ptr(), max_seq, batch, kv_dtype, &mut kv) })?;
        let kv = NonNull::new(kv).ok_or_else(|| invalid("the library returned no cache".into()))?;
        Ok(RawKvCache { kv, batch, max_seq, _engine: PhantomData })
    }

    /// Positions filled in sequence `seq` (the `usize` of the reference's tuple).
    pub fn seq_len(&self, seq: u32) -> Result<usize, Error> {
        let mut n = 0u32;
        check(unsafe { qora_kv_length(self.kv.as_ptr(), seq, &mut n) })?;
        Ok(n as usize)
    }
    pub fn len(&self) -> usize {
        self.seq_len(0).unwrap_or_else(|e| panic!("RawKvCache::len: {e}"))
    }
    pub fn is_empty(&self) -> bool {
        self.len() == 0
    }
    pub fn batch(&self) -> u32 {
        self.batch
    }
    pub fn max_seq(&self) -> u32 {
        self.max_seq
    }
    pub fn reset(&mut self, seq: u32) -> Result<(), Error> {
        check(unsafe { qora_kv_reset(self.kv.as_ptr(), seq) })
    }

    /// Import seq_len token-major rows `[seq_len][kv_row]` of one layer (kv_row =
    /// kv_heads * head_dim), as in the reference's `(k, v, len)` tuple.
    pub fn import_layer(&mut self, layer: u32, k: &[f32], v: &[f32], kv_row: usize, seq: u32) -> Result<(), Error> {
        if kv_row == 0 || k.len() != v.len() || k.len() % kv_row != 0 {
            return Err(invalid(format!("k/v lengths {}/{} for rows of {kv_row}", k.len(), v.len())));
        }
        let n = to_u32(k.len() / kv_row, "seq_len")?;
        check(unsafe { qora_kv_import(self.kv.as_ptr(), layer, k.as_ptr(), v.as_ptr(), n, seq) })
    }

    /// Export the first `seq_len` rows of one layer.
    pub fn export_layer(&self, layer: u32, seq_len: usize, kv_row: usize, seq: u32) -> Result<(Vec<f32>, Vec<f32>), Error> {
        let n = to_u32(seq_len, "seq_len")?;
        let mut k = vec![0f32; seq_len * kv_row];
        let mut v = vec![0f32; seq_len * kv_row];
        check(unsafe { qora_kv_export(self.kv.as_ptr(), layer, k.as_mut_ptr(), v.as_mut_ptr(), n, seq) })?;
        Ok((k, v))
    }

    pub fn as_ptr(&self) -> *mut qora_kv {
        self.kv.as_ptr()
    }
}

impl Drop for RawKvCache<'_> {
    fn drop(&mut self) {
        unsafe { qora_kv_destroy(self.kv.as_ptr()) }
    }
}

/// `empty_kv_cache` (src/gemv.rs:159) for this engine: one f32 sequence of
/// DEFAULT_MAX_SEQ positions.
pub fn empty_kv_cache(w: &DecodeWeights) -> RawKvCache<'_> {
    RawKvCache::try_new(w, DEFAULT_MAX_SEQ, 1, QORA_KV_F32).unwrap_or_else(|e| panic!("empty_kv_cache: {e}"))
}

/// `forward_decode_raw` (src/gemv.rs:872): one decode step of sequence 0, appending one
/// KV row; the logits `[vocab]`.
pub fn try_forward_decode_raw(w: &DecodeWeights, token_id: usize, kv: &mut RawKvCache<'_>) -> Result<Vec<f32>, Error> {
    let tok = to_u32(token_id, "token id")?;
    let mut logits = vec![0f32; w.vocab()];
    let mut am = 0u32;
    check(unsafe { qora_decode_step(w.as_ptr(), kv.as_ptr(), &tok, logits.as_mut_ptr(), &mut am) })?;
    Ok(logits)
}

pub fn forward_decode_raw(w: &DecodeWeights, token_id: usize, kv: &mut RawKvCache<'_>) -> Vec<f32> {
    try_forward_decode_raw(w, token_id, kv).unwrap_or_else(|e| panic!("forward_decode_raw: {e}"))
}

/// The greedy fast path of a decode step: only the argmax (first maximum) leaves the
/// device.
pub fn decode_greedy(w: &DecodeWeights, token_id: u32, kv: &mut RawKvCache<'_>) -> Result<u32, Error> {
    let mut am = 0u32;
    check(unsafe { qora_decode_step(w.as_ptr(), kv.as_ptr(), &token_id, ptr::null_mut(), &mut am) })?;
    Ok(am)
}

/// `raw_prefill` (src/gemv.rs:1027) into a fresh cache of `max_seq` positions: the
/// logits of the last id and the cache.
pub fn try_raw_prefill<'w>(w: &'w DecodeWeights, ids: &[u32], max_seq: u32) -> Result<(Vec<f32>, RawKvCache<'w>), Error> {
    let mut kv = RawKvCache::try_new(w, max_seq, 1, QORA_KV_F32)?;
    let n = to_u32(ids.len(), "prompt length")?;
    let mut logits = vec![0f32; w.vocab()];
    let mut am = 0u32;
    check(unsafe { qora_prefill(w.as_ptr(), kv.as_ptr(), ids.as_ptr(), n, 0, logits.as_mut_ptr(), &mut am) })?;
    Ok((logits, kv))
}

pub fn raw_prefill<'w>(w: &'w DecodeWeights, ids: &[u32]) -> (Vec<f32>, RawKvCache<'w>) {
    try_raw_prefill(w, ids, DEFAULT_MAX_SEQ).unwrap_or_else(|e| panic!("raw_prefill: {e}"))
}

/// n greedy tokens after `first_token`, fed back on the device (no host round trip per
/// token); the decode-only loop of src/main.rs:105-117.
pub fn generate_greedy(w: &DecodeWeights, kv: &mut RawKvCache<'_>, first_token: u32, n: usize) -> Result<Vec<u32>, Error> {
    let nn = to_u32(n, "token count")?;
    let mut out = vec![0u32; n];
    check(unsafe { qora_generate_greedy(w.as_ptr(), kv.as_ptr(), first_token, nn, out.as_mut_ptr()) })?;
    Ok(out)
}

/// Greedy branch of `sample_token_top_k` (src/generate.rs:346-352): the first maximum
/// (index 0 if there is none).
pub fn greedy(logits: &[f32]) -> u32 {
    let mut best = 0usize;
    let mut max = f32::NEG_INFINITY;
    for (i, &x) in logits.iter().enumerate() {
        if x > max {
            max = x;
            best = i;
        }
    }
    best as u32
}

/// The sampling fields of `GenerateParams` (defaults as src/generate.rs:22-35).
#[derive(Clone, Copy, Debug, PartialEq)]
pub struct SamplingParams {
    pub temperature: f32,
    pub top_p: f32,
    pub top_k: u32,
    pub repetition_penalty: f32,
    pub presence_penalty: f32,
    /// set to -inf after the penalties (the thinking branch bans EOS)
    pub ban_token: Option<u32>,
}

impl Default for SamplingParams {
    fn default() -> Self {
        SamplingParams {
            temperature: 0.6,
            top_p: 0.95,
            top_k: 20,
            repetition_penalty: 1.1,
            presence_penalty: 1.5,
            ban_token: None,
        }
    }
}

/// The next token from the logits of row `row` of the last step (left on the device):
/// the reference's penalties over `history`, then `sample_token_top_k`; `rng_state` is
/// the reference `Rng`'s xorshift64 state, advanced exactly as `next_f32` would.
pub fn sample_next(w: &DecodeWeights, row: u32, history: &[u32], p: &SamplingParams, rng_state: &mut u64) -> Result<u32, Error> {
    let ban = match p.ban_token {
        None => -1,
        Some(t) => i32::try_from(t).map_err(|_| invalid(format!("ban_token {t}")))?,
    };
    let s = qora_sampling {
        temperature: p.temperature,
        top_p: p.top_p,
        top_k: p.top_k,
        repetition_penalty: p.repetition_penalty,
        presence_penalty: p.presence_penalty,
        ban_token: ban,
    };
    let n = to_u32(history.len(), "history length")?;
    let mut tok = 0u32;
    check(unsafe { qora_sample(w.as_ptr(), row, history.as_ptr(), n, &s, rng_state, &mut tok) })?;
    Ok(tok)
}

/// Shard arithmetic of a tensor-parallel group (host-only).
pub fn tp_plan(format: u32, num_heads: u32, num_kv_heads: u32, intermediate: u32, vocab: u32, tp_size: i32,
               tp_rank: i32) -> Result<qora_tp_shard, Error> {
    let mut s = qora_tp_shard::default();
    check(unsafe { qora_tp_plan(format, num_heads, num_kv_heads, intermediate, vocab, tp_size, tp_rank, &mut s) })?;
    Ok(s)
}
