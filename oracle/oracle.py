"""TEST INFRASTRUCTURE ONLY: ctypes wrapper of oracle/libqora_oracle.so, the CPU
restatement of the reference QORA decode path (src/gemv.rs, src/simd.rs, src/save.rs,
src/generate.rs:346-352). Used by tests/ as the parity checker and by bench.py's
cpu_baseline leg and `--impl reference` arm as the timed CPU baseline; never by the
engine. Build with `make -C oracle` (or __graft_entry__.build())."""
from __future__ import annotations

import ctypes as C
import importlib
import os
import subprocess
import sys

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(HERE)
LIB_PATH = os.path.join(HERE, "libqora_oracle.so")

if ROOT not in sys.path:
    sys.path.insert(0, ROOT)
_pkg = importlib.import_module("qora-llm_b200")
abi = _pkg.abi
qf = _pkg.qora_format

_f32p = np.ctypeslib.ndpointer(np.float32, flags="C_CONTIGUOUS")
_u8p = np.ctypeslib.ndpointer(np.uint8, flags="C_CONTIGUOUS")
_u16p = np.ctypeslib.ndpointer(np.uint16, flags="C_CONTIGUOUS")
_u32p = np.ctypeslib.ndpointer(np.uint32, flags="C_CONTIGUOUS")
_sz = C.c_size_t


def build(force: bool = False) -> str:
    if force or not os.path.exists(LIB_PATH):
        subprocess.run(["make", "-C", HERE, "-s"], check=True)
    return LIB_PATH


_lib = None


def lib():
    global _lib
    if _lib is not None:
        return _lib
    build()
    L = C.CDLL(LIB_PATH)
    sig = {
        "orc_set_threads": (None, [C.c_int]), "orc_get_threads": (C.c_int, []),
        "orc_set_avx512": (None, [C.c_int]), "orc_get_avx512": (C.c_int, []),
        "orc_host_has_avx512": (C.c_int, []),
        "orc_model_load": (C.c_void_p, [C.c_char_p, C.c_char_p, _sz]),
        "orc_model_from_view": (C.c_void_p, [C.c_void_p, C.c_char_p, _sz]),
        "orc_model_free": (None, [C.c_void_p]),
        "orc_model_vocab": (C.c_uint32, [C.c_void_p]),
        "orc_model_hidden": (C.c_uint32, [C.c_void_p]),
        "orc_model_layers": (C.c_uint32, [C.c_void_p]),
        "orc_model_format": (C.c_uint32, [C.c_void_p]),
        "orc_kv_new": (C.c_void_p, [C.c_void_p]), "orc_kv_free": (None, [C.c_void_p]),
        "orc_kv_len": (C.c_uint32, [C.c_void_p, C.c_uint32]),
        "orc_kv_import": (C.c_int, [C.c_void_p, C.c_uint32, _f32p, _f32p, C.c_uint32]),
        "orc_kv_export": (C.c_int, [C.c_void_p, C.c_uint32, _f32p, _f32p, C.c_uint32]),
        "orc_kv_set_f16": (C.c_int, [C.c_void_p, C.c_int]),
        "orc_round_f16": (None, [_f32p, _f32p, C.c_size_t]),
        "orc_f16_to_f32": (C.c_float, [C.c_uint16]),
        "orc_gemv_q4": (None, [_f32p, _u8p, _u16p, _sz, _sz, _f32p]),
        "orc_gemv_q4_rows": (None, [_f32p, _u8p, _u16p, _sz, _sz, _sz, _f32p]),
        "orc_fused_gate_up_q4": (None, [_f32p, _u8p, _u16p, _u8p, _u16p, _sz, _sz, _f32p]),
        "orc_gemv_f16": (None, [_f32p, _u16p, _sz, _sz, _f32p]),
        "orc_gemm_q4": (None, [_f32p, _sz, _u8p, _u16p, _sz, _sz, _f32p]),
        "orc_gemm_f16": (None, [_f32p, _sz, _u16p, _sz, _sz, _f32p]),
        "orc_embed_q4": (None, [_u8p, _u16p, _sz, _sz, _f32p]),
        "orc_dequant_q4_rows": (None, [_u8p, _u16p, _sz, _sz, _sz, _f32p]),
        "orc_rms_norm": (None, [_f32p, _u16p, _sz, _f32p]),
        "orc_rope": (None, [_f32p, _sz, _sz, _f32p, _f32p, _sz, _sz]),
        "orc_softmax": (None, [_f32p, _sz]),
        "orc_lm_head_q4": (None, [_f32p, _u8p, _u16p, _sz, _sz, _f32p]),
        "orc_lm_head_f16": (None, [_f32p, _u16p, _sz, _sz, _f32p]),
        "orc_argmax": (C.c_uint32, [_f32p, _sz]),
        "orc_rng_next_f32": (C.c_float, [C.POINTER(C.c_uint64)]),
        "orc_sample_top_k": (C.c_uint32, [_f32p, _sz, C.c_float, C.c_float, _sz, C.POINTER(C.c_uint64)]),
        "orc_sample": (C.c_uint32, [_f32p, _sz, _u32p, _sz, C.c_float, C.c_float, _sz, C.c_float, C.c_float,
                                    C.c_int64, C.POINTER(C.c_uint64)]),
        "orc_forward_decode": (C.c_int, [C.c_void_p, C.c_uint32, C.c_void_p, _f32p]),
        "orc_layer_forward": (C.c_int, [C.c_void_p, C.c_uint32, _f32p, C.c_void_p]),
        "orc_prefill": (C.c_int, [C.c_void_p, _u32p, _sz, C.c_void_p, _f32p]),
        "orc_generate_greedy": (C.c_int, [C.c_void_p, _u32p, _sz, _sz, C.c_void_p, _u32p,
                                          C.c_void_p]),
    }
    for name, (res, args) in sig.items():
        fn = getattr(L, name)
        fn.restype = res
        fn.argtypes = args
    _lib = L
    return L


def set_threads(t: int) -> None:
    lib().orc_set_threads(int(t))


def get_threads() -> int:
    return lib().orc_get_threads()


def set_avx512(on: bool) -> None:
    lib().orc_set_avx512(1 if on else 0)


def f32(a):
    return np.ascontiguousarray(a, dtype=np.float32)


# ------------------------------------------------------------------ primitives
def gemv_q4(x, m):
    y = np.empty(m.n, np.float32)
    lib().orc_gemv_q4(f32(x), m.packed, m.scales, m.k, m.n, y)
    return y


def gemv_q4_rows(x, m, k0, k1):
    y = np.empty(m.n, np.float32)
    lib().orc_gemv_q4_rows(f32(x), m.packed, m.scales, m.n, k0, k1, y)
    return y


def fused_gate_up_q4(x, g, u):
    y = np.empty(g.n, np.float32)
    lib().orc_fused_gate_up_q4(f32(x), g.packed, g.scales, u.packed, u.scales, g.k, g.n, y)
    return y


def gemv_f16(x, m):
    y = np.empty(m.n, np.float32)
    lib().orc_gemv_f16(f32(x), m.data, m.k, m.n, y)
    return y


def gemm_f16(x, m):
    """gemm_f16 (src/gemv.rs:571-588): scalar, single-threaded, no FMA."""
    x = f32(x)
    y = np.empty((x.shape[0], m.n), np.float32)
    lib().orc_gemm_f16(x, x.shape[0], m.data, m.k, m.n, y)
    return y


def gemm_q4(x, m):
    x = f32(x)
    y = np.empty((x.shape[0], m.n), np.float32)
    lib().orc_gemm_q4(x, x.shape[0], m.packed, m.scales, m.k, m.n, y)
    return y


def embed_q4(m, row):
    y = np.empty(m.n, np.float32)
    lib().orc_embed_q4(m.packed, m.scales, m.n, row, y)
    return y


def dequant_q4_rows(m, row0, rows):
    y = np.empty((rows, m.n), np.float32)
    lib().orc_dequant_q4_rows(m.packed, m.scales, m.n, row0, rows, y)
    return y


def rms_norm(x, gamma):
    y = np.empty(len(x), np.float32)
    lib().orc_rms_norm(f32(x), gamma, len(x), y)
    return y


def rope(data, heads, head_dim, cos, sin, half, pos):
    d = f32(data).copy()
    lib().orc_rope(d, heads, head_dim, cos, sin, half, pos)
    return d


def softmax(s):
    s = f32(s).copy()
    lib().orc_softmax(s, len(s))
    return s


def lm_head_q4(x, m):
    y = np.empty(m.k, np.float32)
    lib().orc_lm_head_q4(f32(x), m.packed, m.scales, m.k, m.n, y)
    return y


def argmax(logits):
    return int(lib().orc_argmax(f32(logits), len(logits)))


# ------------------------------------------------------------------ model level
def sample(logits, history, temperature, top_p, top_k, repetition_penalty=1.0, presence_penalty=0.0,
           ban=-1, state=1):
    """One sampling step of the reference generation loop (penalties, then
    sample_token_top_k, src/generate.rs:64-92, :345-394). Returns (token, new_state)."""
    hist = np.ascontiguousarray(history, dtype=np.uint32)
    st = C.c_uint64(int(state))
    tok = lib().orc_sample(f32(logits), len(logits), hist, hist.size, float(temperature), float(top_p),
                           int(top_k), float(repetition_penalty), float(presence_penalty), int(ban),
                           C.byref(st))
    return int(tok), int(st.value)


class OracleModel:
    """A model resident in the oracle (copied from a qora_format.Model or a file)."""

    def __init__(self, model=None, path=None):
        err = C.create_string_buffer(512)
        if path is not None:
            h = lib().orc_model_load(os.fsencode(path), err, 512)
        else:
            view = abi.BorrowedView(model)
            h = lib().orc_model_from_view(C.addressof(view.view), err, 512)
        if not h:
            raise qf.QoraFormatError(err.value.decode())
        self.h = h
        self.vocab = lib().orc_model_vocab(h)
        self.hidden = lib().orc_model_hidden(h)
        self.num_layers = lib().orc_model_layers(h)

    def close(self):
        if self.h:
            lib().orc_model_free(self.h)
            self.h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

    def new_kv(self, dtype="f32"):
        """dtype "f16": the opt-in binary16 cache (values rounded as they enter)."""
        return OracleKV(self, dtype)

    def forward_decode(self, token, kv):
        out = np.empty(self.vocab, np.float32)
        rc = lib().orc_forward_decode(self.h, int(token), kv.h, out)
        if rc:
            raise ValueError(f"orc_forward_decode rc={rc}")
        return out

    def layer_forward(self, layer, x, kv):
        x = f32(x).copy()
        rc = lib().orc_layer_forward(self.h, int(layer), x, kv.h)
        if rc:
            raise ValueError(f"orc_layer_forward rc={rc}")
        return x

    def prefill(self, ids, kv):
        ids = np.ascontiguousarray(ids, dtype=np.uint32)
        out = np.empty(self.vocab, np.float32)
        rc = lib().orc_prefill(self.h, ids, ids.size, kv.h, out)
        if rc:
            raise ValueError(f"orc_prefill rc={rc}")
        return out

    def generate_greedy(self, prompt, n_new, kv=None):
        kv = kv or self.new_kv()
        prompt = np.ascontiguousarray(prompt, dtype=np.uint32)
        toks = np.zeros(n_new, np.uint32)
        margins = np.zeros(n_new, np.float32)
        rc = lib().orc_generate_greedy(self.h, prompt, prompt.size, n_new, kv.h, toks,
                                       margins.ctypes.data)
        if rc:
            raise ValueError(f"orc_generate_greedy rc={rc}")
        return toks, margins


def round_f16(x):
    """x rounded to the nearest binary16 value (ties to even), as f32 (orc_round_f16)."""
    x = f32(x)
    out = np.empty_like(x)
    lib().orc_round_f16(x.reshape(-1), out.reshape(-1), x.size)
    return out


class OracleKV:
    def __init__(self, m: OracleModel, dtype="f32"):
        if dtype not in ("f32", "f16"):
            raise ValueError(f"KV dtype {dtype!r}")
        self.m = m
        self.h = lib().orc_kv_new(m.h)
        if dtype == "f16" and lib().orc_kv_set_f16(self.h, 1):
            raise ValueError("orc_kv_set_f16 failed")

    def __del__(self):
        try:
            if self.h:
                lib().orc_kv_free(self.h)
                self.h = None
        except Exception:
            pass

    def length(self, layer=0):
        return lib().orc_kv_len(self.h, layer)

    def import_layer(self, layer, k, v):
        k, v = f32(k), f32(v)
        n = k.shape[0]
        if lib().orc_kv_import(self.h, layer, k.reshape(-1), v.reshape(-1), n):
            raise ValueError("orc_kv_import failed")

    def export_layer(self, layer, n, stride):
        k = np.empty(n * stride, np.float32)
        v = np.empty(n * stride, np.float32)
        if lib().orc_kv_export(self.h, layer, k, v, n):
            raise ValueError("orc_kv_export failed")
        return k.reshape(n, stride), v.reshape(n, stride)
