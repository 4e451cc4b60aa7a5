"""ctypes mirror of the structs in include/qora_cuda.h and helpers that build a
`qora_weights_view` over the arrays of a `qora_format.Model` (borrowed, like the
`WeightRef` slices of src/gemv.rs:66-96)."""
from __future__ import annotations

import ctypes as C

import numpy as np

from .qora_format import Model, Matrix, FORMAT_Q4


class MatrixView(C.Structure):
    _fields_ = [("packed", C.c_void_p), ("scales", C.c_void_p), ("data", C.c_void_p),
                ("k", C.c_uint64), ("n", C.c_uint64)]


class LayerView(C.Structure):
    _fields_ = [(name, MatrixView) for name in
                ("q_proj", "k_proj", "v_proj", "o_proj", "gate_proj", "up_proj", "down_proj")] + [
        ("input_norm_gamma", C.c_void_p), ("post_attn_norm_gamma", C.c_void_p),
        ("num_heads", C.c_uint32), ("num_kv_heads", C.c_uint32), ("head_dim", C.c_uint32),
        ("num_kv_groups", C.c_uint32)]


class WeightsView(C.Structure):
    _fields_ = [("format", C.c_uint32), ("num_layers", C.c_uint32), ("vocab", C.c_uint32),
                ("hidden", C.c_uint32), ("rope_half_dim", C.c_uint32),
                ("no_rope_layers", C.c_void_p), ("layers", C.POINTER(LayerView)),
                ("embed", MatrixView), ("final_norm_gamma", C.c_void_p),
                ("rope_cos", C.c_void_p), ("rope_sin", C.c_void_p), ("rope_rows", C.c_uint64)]


class EngineOptions(C.Structure):
    _fields_ = [("n_gpus", C.c_int32), ("first_device", C.c_int32), ("flags", C.c_uint32),
                ("tp_size", C.c_int32), ("tp_rank", C.c_int32)]


class TpShard(C.Structure):
    """qora_tp_shard (include/qora_cuda.h)."""
    _fields_ = [(n, C.c_uint32) for n in ("q_head0", "q_heads", "kv_head0", "kv_heads", "mlp0", "mlp_n",
                                          "mlp_padded", "vocab0", "vocab_n")]


class Sampling(C.Structure):
    """qora_sampling (include/qora_cuda.h)."""
    _fields_ = [("temperature", C.c_float), ("top_p", C.c_float), ("top_k", C.c_uint32),
                ("repetition_penalty", C.c_float), ("presence_penalty", C.c_float),
                ("ban_token", C.c_int32)]


def _ptr(a: np.ndarray | None):
    if a is None:
        return None
    assert a.flags["C_CONTIGUOUS"]
    return a.ctypes.data


def _mview(m: Matrix, keep: list) -> MatrixView:
    for a in (m.packed, m.scales, m.data):
        if a is not None:
            keep.append(a)
    return MatrixView(_ptr(m.packed), _ptr(m.scales), _ptr(m.data), m.k, m.n)


class BorrowedView:
    """A WeightsView plus references that keep every borrowed array alive."""

    def __init__(self, model: Model):
        keep: list = []
        layers = (LayerView * model.num_layers)()
        for i, L in enumerate(model.layers):
            lv = layers[i]
            for name in ("q_proj", "k_proj", "v_proj", "o_proj", "gate_proj", "up_proj",
                         "down_proj"):
                setattr(lv, name, _mview(getattr(L, name), keep))
            keep += [L.input_norm_gamma, L.post_attn_norm_gamma]
            lv.input_norm_gamma = _ptr(L.input_norm_gamma)
            lv.post_attn_norm_gamma = _ptr(L.post_attn_norm_gamma)
            lv.num_heads, lv.num_kv_heads = L.num_heads, L.num_kv_heads
            lv.head_dim, lv.num_kv_groups = L.head_dim, L.num_kv_groups
        no_rope = np.ascontiguousarray(model.no_rope_layers, dtype=np.uint8)
        keep += [no_rope, model.final_norm_gamma, model.rope_cos, model.rope_sin, layers]
        self.view = WeightsView(
            model.format, model.num_layers, model.vocab, model.hidden, model.rope_half_dim,
            _ptr(no_rope), C.cast(layers, C.POINTER(LayerView)), _mview(model.embed, keep),
            _ptr(model.final_norm_gamma), _ptr(model.rope_cos), _ptr(model.rope_sin),
            model.rope_rows)
        self._keep = keep
        self.model = model

    def ref(self):
        return C.byref(self.view)


def is_q4(model: Model) -> bool:
    return model.format == FORMAT_Q4
