"""Host-side mirror of the reference decode API over libqora_cuda.so (ctypes).

Reference interface (Rust crate `qora`) -> here:
  save::load_model(path)                     (src/save.rs:154)   -> load_model(path)
  gemv::empty_kv_cache(layers, kv_heads, hd) (src/gemv.rs:159)   -> empty_kv_cache(w, max_seq)
  gemv::forward_decode_raw(&w, token, &mut kv) (src/gemv.rs:872) -> forward_decode_raw(w, token, kv)
  gemv::raw_prefill(&w, &ids)                (src/gemv.rs:1027)  -> raw_prefill(w, ids)
  greedy sample_token_top_k (src/generate.rs:346-352)            -> DecodeWeights.decode_step(...)

Errors: the reference returns io::Error from load_model and panics on bad input; here
every failure raises QoraError carrying the library's status code and message. There is
no CPU fallback: if the CUDA library cannot be loaded, the import of this module's
functions raises.
"""
from __future__ import annotations

import ctypes as C
import os
from typing import Optional, Tuple

import numpy as np

from . import abi
from .qora_format import Model

HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(HERE, "libqora_cuda.so")

FLAG_PER_OP_KERNELS = 1  # QORA_FLAG_PER_OP_KERNELS
FLAG_TOKEN_PREFILL = 2  # QORA_FLAG_TOKEN_PREFILL

STATUS = {0: "OK", 1: "INVALID", 2: "IO", 3: "CUDA", 4: "OOM", 5: "RANGE", 6: "TIMEOUT",
          7: "UNSUPPORTED", 8: "NCCL"}

# every function include/qora_cuda.h declares, with its ctypes signature
_vp, _u32, _u64, _i32 = C.c_void_p, C.c_uint32, C.c_uint64, C.c_int32
_P = C.POINTER
SIGNATURES = {
    "qora_last_error": (C.c_char_p, []),
    "qora_version": (C.c_char_p, []),
    "qora_engine_create_from_file": (C.c_int, [C.c_char_p, _vp, _P(_vp)]),
    "qora_engine_create": (C.c_int, [_vp, _vp, _P(_vp)]),
    "qora_engine_destroy": (None, [_vp]),
    "qora_engine_info": (C.c_int, [_vp, _P(_u32), _P(_u32), _P(_u32), _P(_u32), _P(_u64)]),
    "qora_kv_create": (C.c_int, [_vp, _u32, _u32, _P(_vp)]),
    "qora_kv_create_ex": (C.c_int, [_vp, _u32, _u32, _u32, _P(_vp)]),
    "qora_kv_destroy": (None, [_vp]),
    "qora_kv_length": (C.c_int, [_vp, _u32, _P(_u32)]),
    "qora_kv_reset": (C.c_int, [_vp, _u32]),
    "qora_kv_import": (C.c_int, [_vp, _u32, _vp, _vp, _u32, _u32]),
    "qora_kv_export": (C.c_int, [_vp, _u32, _vp, _vp, _u32, _u32]),
    "qora_prefill": (C.c_int, [_vp, _vp, _vp, _u32, _u32, _vp, _vp]),
    "qora_decode_step": (C.c_int, [_vp, _vp, _vp, _vp, _vp]),
    "qora_generate_greedy": (C.c_int, [_vp, _vp, _u32, _u32, _vp]),
    "qora_generate_greedy_batch": (C.c_int, [_vp, _vp, _vp, _u32, _vp, _P(C.c_float)]),
    "qora_layer_step": (C.c_int, [_vp, _vp, _u32, _vp]),
    "qora_generate_greedy_timed": (C.c_int, [_vp, _vp, _u32, _u32, _vp, _P(C.c_float)]),
    "qora_engine_time_kernel": (C.c_int, [_vp, _vp, C.c_int, _u32, _P(C.c_float), _P(_u64),
                                          _P(_u32)]),
    "qora_engine_launches_per_step": (C.c_int, [_vp, _P(_u32)]),
    "qora_engine_prompt_path": (C.c_int, [_vp, _P(_u32)]),
    "qora_engine_set_trace": (C.c_int, [_vp, C.c_int]),
    "qora_engine_get_trace": (C.c_int, [_vp, _vp, C.c_size_t, _P(C.c_size_t)]),
    "qora_tp_export": (C.c_int, [_vp, _vp, C.c_size_t, _P(C.c_size_t)]),
    "qora_tp_connect": (C.c_int, [_vp, C.c_char_p, C.c_size_t]),
    "qora_tp_plan": (C.c_int, [_u32, _u32, _u32, _u32, _u32, _i32, _i32, _vp]),
    "qora_q4_gemv": (C.c_int, [_vp, _vp, _vp, _u64, _u64, _vp, _vp]),
    "qora_q4_gemv_static": (C.c_int, [_vp, _vp, _vp, _u64, _u64, _vp, _vp]),
    "qora_q4_dequant": (C.c_int, [_vp, _vp, _u64, _u64, _u64, _vp, _vp]),
    "qora_q4_gate_up": (C.c_int, [_vp, _vp, _vp, _vp, _vp, _u64, _u64, _vp, _vp]),
    "qora_q4_lm_head": (C.c_int, [_vp, _vp, _vp, _u64, _u64, _vp, _vp, _vp]),
    "qora_f16_gemm": (C.c_int, [_vp, _vp, _u64, _u64, _u64, _vp, _vp]),
    "qora_sample": (C.c_int, [_vp, _u32, _vp, _u32, _vp, _P(_u64), _P(_u32)]),
    "qora_sample_logits": (C.c_int, [_vp, _u32, _vp, _u32, _vp, _P(_u64), _P(_u32), _vp]),
}


class QoraError(RuntimeError):
    def __init__(self, status: int, msg: str):
        super().__init__(f"{STATUS.get(status, status)}: {msg}")
        self.status = status


_lib = None


def lib():
    """Load libqora_cuda.so (raises if it is missing: there is no fallback)."""
    global _lib
    if _lib is None:
        if not os.path.exists(LIB_PATH):
            raise ImportError(f"{LIB_PATH} is not built (run qora-llm_b200/build.py)")
        L = C.CDLL(LIB_PATH)
        for name, (res, args) in SIGNATURES.items():
            fn = getattr(L, name)
            fn.restype = res
            fn.argtypes = args
        _lib = L
    return _lib


def check(status: int):
    if status != 0:
        raise QoraError(status, lib().qora_last_error().decode(errors="replace"))


def _ptr(a: np.ndarray):
    return a.ctypes.data


class DecodeWeights:
    """An engine: the model resident on the GPU (the `DecodeWeights` of src/gemv.rs:195)."""

    def __init__(self, model: Optional[Model] = None, path: Optional[str] = None,
                 device: int = 0, n_gpus: int = 1, per_op_kernels: bool = False,
                 tp_size: int = 1, tp_rank: int = 0, token_prefill: bool = False):
        """tp_size > 1: this engine is rank tp_rank of a tensor-parallel group (one engine
        per GPU); call tp_export() on every rank and tp_connect(all_handles) on each.
        token_prefill: Q4 prompts run as one decode step per token (no tensor-core prompt
        pass, no second copy of the projections)."""
        self.per_op_kernels = per_op_kernels
        self.tp_size, self.tp_rank = tp_size, tp_rank
        flags = (FLAG_PER_OP_KERNELS if per_op_kernels else 0) | (FLAG_TOKEN_PREFILL if token_prefill else 0)
        opts = abi.EngineOptions(n_gpus, device, flags, tp_size, tp_rank)
        h = C.c_void_p()
        if path is not None:
            check(lib().qora_engine_create_from_file(os.fsencode(path), C.byref(opts), C.byref(h)))
        else:
            view = abi.BorrowedView(model)
            check(lib().qora_engine_create(view.ref(), C.byref(opts), C.byref(h)))
        self.h = h
        nl, v, hd, fmt, nb = _u32(), _u32(), _u32(), _u32(), _u64()
        check(lib().qora_engine_info(h, C.byref(nl), C.byref(v), C.byref(hd), C.byref(fmt),
                                     C.byref(nb)))
        self.num_layers, self.vocab, self.hidden = nl.value, v.value, hd.value
        self.format, self.device_bytes = fmt.value, nb.value

    def close(self):
        if getattr(self, "h", None):
            lib().qora_engine_destroy(self.h)
            self.h = None

    def tp_export(self) -> bytes:
        """This rank's opaque peer handle (qora_tp_export)."""
        n = C.c_size_t()
        check(lib().qora_tp_export(self.h, None, 0, C.byref(n)))
        buf = C.create_string_buffer(n.value)
        check(lib().qora_tp_export(self.h, buf, n.value, C.byref(n)))
        return buf.raw[: n.value]

    def tp_connect(self, handles) -> None:
        """Map every rank's buffers; `handles` lists all ranks' tp_export() bytes in rank
        order (qora_tp_connect)."""
        handles = list(handles)
        size = len(handles[0])
        if len(handles) != self.tp_size or any(len(h) != size for h in handles):
            raise ValueError("need one handle of equal size per rank")
        blob = b"".join(handles)
        check(lib().qora_tp_connect(self.h, blob, size))

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

    def __enter__(self):
        return self

    def __exit__(self, *a):
        self.close()

    # ---- KV
    def new_kv(self, max_seq: int, batch: int = 1, dtype: str = "f32") -> "KVCache":
        """A cache for `batch` independent sequences (batch > 1: F16 engines). dtype "f16"
        is the opt-in binary16 cache (QORA_KV_F16: Q4 engines, persistent step)."""
        return KVCache(self, max_seq, batch, dtype)

    # ---- steps
    def decode_step(self, kv: "KVCache", token: int, want_logits: bool = False):
        tok = np.array([token], np.uint32)
        am = np.zeros(1, np.uint32)
        logits = np.empty(self.vocab, np.float32) if want_logits else None
        check(lib().qora_decode_step(self.h, kv.h, _ptr(tok),
                                     _ptr(logits) if logits is not None else None, _ptr(am)))
        return (int(am[0]), logits) if want_logits else int(am[0])

    def decode_batch(self, kv: "KVCache", tokens, want_logits: bool = False):
        """One decode step of every sequence of `kv`: (argmax [batch], logits [batch][vocab]
        or None)."""
        tok = np.ascontiguousarray(tokens, dtype=np.uint32)
        if tok.size != kv.batch:
            raise ValueError(f"{tok.size} tokens for {kv.batch} sequences")
        am = np.zeros(kv.batch, np.uint32)
        logits = np.empty((kv.batch, self.vocab), np.float32) if want_logits else None
        check(lib().qora_decode_step(self.h, kv.h, _ptr(tok),
                                     _ptr(logits) if logits is not None else None, _ptr(am)))
        return am, logits

    def prefill(self, kv: "KVCache", ids, want_logits: bool = True, seq: int = 0):
        ids = np.ascontiguousarray(ids, dtype=np.uint32)
        am = np.zeros(1, np.uint32)
        logits = np.empty(self.vocab, np.float32) if want_logits else None
        check(lib().qora_prefill(self.h, kv.h, _ptr(ids), ids.size, int(seq),
                                 _ptr(logits) if logits is not None else None, _ptr(am)))
        return int(am[0]), logits

    def generate_greedy_batch(self, kv: "KVCache", first_tokens, n: int, timed: bool = False):
        """n greedy tokens for every sequence: out [n][batch] (and device ms if timed)."""
        first = np.ascontiguousarray(first_tokens, dtype=np.uint32)
        if first.size != kv.batch:
            raise ValueError(f"{first.size} tokens for {kv.batch} sequences")
        out = np.zeros((n, kv.batch), np.uint32)
        ms = C.c_float()
        check(lib().qora_generate_greedy_batch(self.h, kv.h, _ptr(first), int(n), _ptr(out),
                                               C.byref(ms) if timed else None))
        return (out, ms.value) if timed else out

    def generate_greedy(self, kv: "KVCache", first_token: int, n: int) -> np.ndarray:
        out = np.zeros(n, np.uint32)
        check(lib().qora_generate_greedy(self.h, kv.h, int(first_token), int(n), _ptr(out)))
        return out

    def generate_greedy_timed(self, kv: "KVCache", first_token: int, n: int):
        """Greedy tokens plus the CUDA-event device time (ms) of the n decode steps."""
        out = np.zeros(n, np.uint32)
        ms = C.c_float()
        check(lib().qora_generate_greedy_timed(self.h, kv.h, int(first_token), int(n), _ptr(out),
                                               C.byref(ms)))
        return out, ms.value

    KERNELS = {"qkv": 0, "attention": 1, "o": 2, "gate_up": 3, "down": 4, "lm_head": 5}

    def time_kernel(self, kv: "KVCache", kernel: str, reps: int = 5):
        """(mean ms per launch, algorithmic bytes per launch, launches timed)."""
        ms, nb, nl = C.c_float(), _u64(), _u32()
        check(lib().qora_engine_time_kernel(self.h, kv.h, self.KERNELS[kernel], int(reps),
                                            C.byref(ms), C.byref(nb), C.byref(nl)))
        return ms.value, nb.value, nl.value

    def set_trace(self, on: bool = True):
        """Record per-CTA phase timestamps of the persistent decode kernel."""
        check(lib().qora_engine_set_trace(self.h, 1 if on else 0))

    def get_trace(self) -> np.ndarray:
        n = C.c_size_t()
        check(lib().qora_engine_get_trace(self.h, None, 0, C.byref(n)))
        out = np.zeros(n.value, np.uint64)
        check(lib().qora_engine_get_trace(self.h, _ptr(out), out.size, C.byref(n)))
        return out

    def sample(self, history, temperature: float, top_p: float, top_k: int,
               repetition_penalty: float = 1.0, presence_penalty: float = 0.0, ban_token: int = -1,
               state: int = 1, row: int = 0):
        """Sample from the last step's logits on the device (qora_sample): the reference's
        penalties + sample_token_top_k. Returns (token, new xorshift64 state)."""
        hist = np.ascontiguousarray(history, dtype=np.uint32)
        p = abi.Sampling(temperature, top_p, top_k, repetition_penalty, presence_penalty, ban_token)
        st, tok = _u64(int(state)), _u32()
        check(lib().qora_sample(self.h, int(row), _ptr(hist) if hist.size else None, hist.size, C.byref(p),
                                C.byref(st), C.byref(tok)))
        return tok.value, st.value

    def launches_per_step(self) -> int:
        n = _u32()
        check(lib().qora_engine_launches_per_step(self.h, C.byref(n)))
        return n.value

    def prefill_path(self) -> str:
        """How prefill() runs a prompt of two or more tokens: "tensor cores" (all rows at
        once, layer by layer) or "token steps" (one decode step per token)."""
        n = _u32()
        check(lib().qora_engine_prompt_path(self.h, C.byref(n)))
        return "tensor cores" if n.value == 1 else "token steps"

    def layer_step(self, kv: "KVCache", layer: int, x) -> np.ndarray:
        x = np.ascontiguousarray(x, dtype=np.float32).copy()
        check(lib().qora_layer_step(self.h, kv.h, int(layer), _ptr(x)))
        return x


KV_DTYPES = {"f32": 0, "f16": 1}  # QORA_KV_F32, QORA_KV_F16


class KVCache:
    """Device KV cache (RawKvCache); import/export use f32 token-major
    [seq][kv_heads][128] host rows whatever the device element type."""

    def __init__(self, w: DecodeWeights, max_seq: int, batch: int = 1, dtype: str = "f32"):
        if dtype not in KV_DTYPES:
            raise ValueError(f"KV dtype {dtype!r}: one of {sorted(KV_DTYPES)}")
        h = C.c_void_p()
        check(lib().qora_kv_create_ex(w.h, int(max_seq), int(batch), KV_DTYPES[dtype], C.byref(h)))
        self.h, self.w, self.max_seq, self.batch, self.dtype = h, w, max_seq, batch, dtype

    def close(self):
        if getattr(self, "h", None):
            lib().qora_kv_destroy(self.h)
            self.h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

    def __len__(self):
        return self.length(0)

    def length(self, seq: int = 0) -> int:
        n = _u32()
        check(lib().qora_kv_length(self.h, int(seq), C.byref(n)))
        return n.value

    def reset(self, seq: int = 0):
        check(lib().qora_kv_reset(self.h, int(seq)))

    def import_layer(self, layer: int, k, v, seq: int = 0):
        k = np.ascontiguousarray(k, dtype=np.float32)
        v = np.ascontiguousarray(v, dtype=np.float32)
        check(lib().qora_kv_import(self.h, int(layer), _ptr(k), _ptr(v), k.shape[0], int(seq)))

    def export_layer(self, layer: int, n: int, stride: int, seq: int = 0) -> Tuple[np.ndarray, np.ndarray]:
        k = np.empty((n, stride), np.float32)
        v = np.empty((n, stride), np.float32)
        check(lib().qora_kv_export(self.h, int(layer), _ptr(k), _ptr(v), int(n), int(seq)))
        return k, v


# ---------------------------------------------------------------- reference-named API
def load_model(path: str, device: int = 0) -> DecodeWeights:
    return DecodeWeights(path=path, device=device)


def empty_kv_cache(weights: DecodeWeights, max_seq: int = 4096) -> KVCache:
    return weights.new_kv(max_seq)


def forward_decode_raw(weights: DecodeWeights, token_id: int, kv: KVCache) -> np.ndarray:
    return weights.decode_step(kv, token_id, want_logits=True)[1]


def raw_prefill(weights: DecodeWeights, token_ids, max_seq: int = 4096):
    kv = weights.new_kv(max_seq)
    _, logits = weights.prefill(kv, token_ids, want_logits=True)
    return logits, kv


# ---------------------------------------------------------------- kernel entries
def _stream_ptr(stream):
    if stream is None:
        return None
    return int(getattr(stream, "cuda_stream", stream))


def q4_gemv(x_ptr, packed_ptr, scales_ptr, k, n, y_ptr, stream=None):
    check(lib().qora_q4_gemv(x_ptr, packed_ptr, scales_ptr, k, n, y_ptr, _stream_ptr(stream)))


def q4_gemv_static(x_ptr, packed_ptr, scales_ptr, k, n, y_ptr, stream=None):
    """qora_q4_gemv on the library's fixed static scratch (allocates nothing)."""
    check(lib().qora_q4_gemv_static(x_ptr, packed_ptr, scales_ptr, k, n, y_ptr, _stream_ptr(stream)))


def q4_dequant(packed_ptr, scales_ptr, n, row0, rows, out_ptr, stream=None):
    check(lib().qora_q4_dequant(packed_ptr, scales_ptr, n, row0, rows, out_ptr, _stream_ptr(stream)))


def q4_gate_up(x_ptr, gp, gs, up, us, k, n, out_ptr, stream=None):
    check(lib().qora_q4_gate_up(x_ptr, gp, gs, up, us, k, n, out_ptr, _stream_ptr(stream)))


def q4_lm_head(x_ptr, packed_ptr, scales_ptr, vocab, hidden, logits_ptr, argmax_ptr, stream=None):
    check(lib().qora_q4_lm_head(x_ptr, packed_ptr, scales_ptr, vocab, hidden, logits_ptr,
                                argmax_ptr, _stream_ptr(stream)))


def f16_gemm(x_ptr, w_ptr, m, k, n, y_ptr, stream=None):
    """y[m][n] = x[m][k] . W[k][n], W f16 row-major (qora_f16_gemm, tcgen05)."""
    check(lib().qora_f16_gemm(x_ptr, w_ptr, m, k, n, y_ptr, _stream_ptr(stream)))


def sample_logits(logits_ptr, vocab, history_ptr, n_history, temperature, top_p, top_k,
                  repetition_penalty=1.0, presence_penalty=0.0, ban_token=-1, state=1, stream=None):
    """qora_sample_logits on device pointers. Returns (token, new state)."""
    p = abi.Sampling(temperature, top_p, top_k, repetition_penalty, presence_penalty, ban_token)
    st, tok = _u64(int(state)), _u32()
    check(lib().qora_sample_logits(logits_ptr, vocab, history_ptr, n_history, C.byref(p), C.byref(st),
                                   C.byref(tok), _stream_ptr(stream)))
    return tok.value, st.value


def tp_plan(fmt: int, num_heads: int, num_kv_heads: int, intermediate: int, vocab: int, tp: int, rank: int) -> dict:
    """The shard a tensor-parallel rank holds (qora_tp_plan; host arithmetic only)."""
    out = abi.TpShard()
    check(lib().qora_tp_plan(fmt, num_heads, num_kv_heads, intermediate, vocab, tp, rank, C.byref(out)))
    return {n: getattr(out, n) for n, _ in abi.TpShard._fields_}
