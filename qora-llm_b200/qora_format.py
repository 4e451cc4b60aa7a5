"""The `.qora` weight file (magic ``QOR3``, version 1) and seeded synthetic models.

Byte layout follows the reference writer/reader (src/save.rs:119-151 and :154-262):
little-endian; header ``QOR3`` + u32 version + u8 format (0 = F16, 1 = Q4); u32
num_layers, vocab, hidden, rope_half_dim; ``no_rope_layers`` as u64 length + one byte per
layer (nonzero = apply RoPE, src/gemv.rs:885/:903); per layer the seven projections
q, k, v, o, gate, up, down (each u64 k, u64 n, then Q4: u64-prefixed packed bytes and
u64-prefixed f16 scales, or F16: u64-prefixed f16 data — src/gemv.rs:341-356), the two
f16 norm vectors and four u32 (num_heads, num_kv_heads, head_dim, num_kv_groups); then
the embedding weight (k = vocab, n = hidden), the final norm and the f32 RoPE cos / sin
tables ([rows][rope_half_dim]).

The reference has no quantiser or converter (src/gemv.rs:168-171 is empty and
`save_model` has no caller), so `synth_model` defines the synthetic distributions:
Q4 codes uniform in [-7, 7] stored as q + 8, scales f16(|N(0, 0.02)| / 7), norm gains
f16(1 + N(0, 0.02)), the tied embedding f32 N(0, 0.02) quantised per group of 32 along
hidden with scale = absmax / 7 (f16) and q = clamp(round(v / scale) + 8, 0, 15), RoPE
tables cos / sin(pos * theta^(-2i / head_dim)) computed in f64 and stored as f32.
"""
from __future__ import annotations

import dataclasses
import io
import struct
from typing import List, Optional

import numpy as np

MAGIC = b"QOR3"
VERSION = 1
FORMAT_F16 = 0
FORMAT_Q4 = 1
GROUP = 32

PROJ_NAMES = ("q_proj", "k_proj", "v_proj", "o_proj", "gate_proj", "up_proj", "down_proj")


class QoraFormatError(ValueError):
    """Malformed .qora contents (the reader's io::ErrorKind::InvalidData)."""


@dataclasses.dataclass
class Matrix:
    k: int
    n: int
    packed: Optional[np.ndarray] = None  # uint8 [k*n/2]  (Q4)
    scales: Optional[np.ndarray] = None  # uint16 [k*n/32] f16 bits (Q4)
    data: Optional[np.ndarray] = None    # uint16 [k*n] f16 bits (F16)

    @property
    def is_q4(self) -> bool:
        return self.packed is not None

    def nbytes(self) -> int:
        if self.is_q4:
            return int(self.packed.nbytes + self.scales.nbytes)
        return int(self.data.nbytes)


@dataclasses.dataclass
class Layer:
    q_proj: Matrix
    k_proj: Matrix
    v_proj: Matrix
    o_proj: Matrix
    gate_proj: Matrix
    up_proj: Matrix
    down_proj: Matrix
    input_norm_gamma: np.ndarray        # uint16 [hidden]
    post_attn_norm_gamma: np.ndarray    # uint16 [hidden]
    num_heads: int
    num_kv_heads: int
    head_dim: int
    num_kv_groups: int

    def mats(self) -> List[Matrix]:
        return [getattr(self, n) for n in PROJ_NAMES]


@dataclasses.dataclass
class Model:
    format: int
    num_layers: int
    vocab: int
    hidden: int
    rope_half_dim: int
    no_rope_layers: np.ndarray   # uint8 [num_layers]; nonzero = apply RoPE
    layers: List[Layer]
    embed: Matrix
    final_norm_gamma: np.ndarray  # uint16 [hidden]
    rope_cos: np.ndarray          # float32 [rows * half]
    rope_sin: np.ndarray

    @property
    def rope_rows(self) -> int:
        return int(self.rope_cos.size // max(1, self.rope_half_dim))

    def weight_bytes(self) -> int:
        tot = sum(m.nbytes() for L in self.layers for m in L.mats())
        tot += sum(L.input_norm_gamma.nbytes + L.post_attn_norm_gamma.nbytes for L in self.layers)
        return tot + self.embed.nbytes() + self.final_norm_gamma.nbytes


# ------------------------------------------------------------------------------ writer
def _w_u32(f, v):
    f.write(struct.pack("<I", v))


def _w_u64(f, v):
    f.write(struct.pack("<Q", v))


def _w_vec(f, arr: np.ndarray):
    arr = np.ascontiguousarray(arr)
    _w_u64(f, arr.size)
    f.write(memoryview(arr).cast("B"))


def _w_matrix(f, m: Matrix, fmt: int):
    _w_u64(f, m.k)
    _w_u64(f, m.n)
    if fmt == FORMAT_Q4:
        _w_vec(f, m.packed.astype(np.uint8, copy=False))
        _w_vec(f, m.scales.astype(np.uint16, copy=False))
    else:
        _w_vec(f, m.data.astype(np.uint16, copy=False))


def write_qora(model: Model, path) -> None:
    """Write `model` in the save_model layout (src/save.rs:119-151)."""
    with open(path, "wb") as f:
        f.write(MAGIC)
        _w_u32(f, VERSION)
        f.write(struct.pack("<B", model.format))
        for v in (model.num_layers, model.vocab, model.hidden, model.rope_half_dim):
            _w_u32(f, v)
        _w_vec(f, (model.no_rope_layers != 0).astype(np.uint8))
        for L in model.layers:
            for m in L.mats():
                _w_matrix(f, m, model.format)
            _w_vec(f, L.input_norm_gamma)
            _w_vec(f, L.post_attn_norm_gamma)
            for v in (L.num_heads, L.num_kv_heads, L.head_dim, L.num_kv_groups):
                _w_u32(f, v)
        _w_matrix(f, model.embed, model.format)
        _w_vec(f, model.final_norm_gamma)
        _w_vec(f, model.rope_cos.astype(np.float32, copy=False))
        _w_vec(f, model.rope_sin.astype(np.float32, copy=False))


# ------------------------------------------------------------------------------ reader
class _Reader:
    def __init__(self, f):
        self.f = f

    def need(self, n: int) -> bytes:
        b = self.f.read(n)
        if len(b) != n:
            raise QoraFormatError("short read")
        return b

    def u8(self):
        return self.need(1)[0]

    def u32(self):
        return struct.unpack("<I", self.need(4))[0]

    def u64(self):
        return struct.unpack("<Q", self.need(8))[0]

    def vec(self, dtype) -> np.ndarray:
        n = self.u64()
        if n > (1 << 36):
            raise QoraFormatError("implausible vector length")
        itemsize = np.dtype(dtype).itemsize
        raw = self.need(n * itemsize)
        return np.frombuffer(raw, dtype=dtype).copy()


def _r_matrix(r: _Reader, fmt: int) -> Matrix:  # read_weight_data (src/save.rs:217-238)
    k, n = r.u64(), r.u64()
    if fmt == FORMAT_F16:
        m = Matrix(k, n, data=r.vec(np.uint16))
        if m.data.size != k * n:
            raise QoraFormatError("f16 weight size mismatch")
        return m
    if fmt == FORMAT_Q4:
        m = Matrix(k, n, packed=r.vec(np.uint8), scales=r.vec(np.uint16))
        if n % GROUP or m.packed.size != k * n // 2 or m.scales.size != k * n // GROUP:
            raise QoraFormatError("q4 weight size mismatch")
        return m
    raise QoraFormatError(f"Unknown format id {fmt}")


def read_qora(path) -> Model:
    """Read a .qora file (load_model, src/save.rs:154-210)."""
    with open(path, "rb") as fh:
        r = _Reader(io.BufferedReader(fh, buffer_size=8 << 20))
        if r.need(4) != MAGIC:
            raise QoraFormatError("Invalid magic bytes")
        version = r.u32()
        if version != VERSION:
            raise QoraFormatError(f"Unsupported version {version}, expected {VERSION}")
        fmt = r.u8()
        num_layers, vocab, hidden, half = r.u32(), r.u32(), r.u32(), r.u32()
        no_rope = r.vec(np.uint8)
        if no_rope.size != num_layers:
            raise QoraFormatError("no_rope_layers length != num_layers")
        layers = []
        for _ in range(num_layers):
            mats = [_r_matrix(r, fmt) for _ in range(7)]
            g1, g2 = r.vec(np.uint16), r.vec(np.uint16)
            nh, nkv, hd, ng = r.u32(), r.u32(), r.u32(), r.u32()
            layers.append(Layer(*mats, g1, g2, nh, nkv, hd, ng))
        embed = _r_matrix(r, fmt)
        final = r.vec(np.uint16)
        cos, sin = r.vec(np.float32), r.vec(np.float32)
    return Model(fmt, num_layers, vocab, hidden, half, no_rope, layers, embed, final, cos, sin)


# ------------------------------------------------------------------------------ synthetic
SMOLLM3_3B = dict(num_layers=36, vocab=128256, hidden=2048, intermediate=11008,
                  num_heads=16, num_kv_heads=4, head_dim=128, rope_theta=5e6,
                  rope_rows=65536)

# byte value for each pair (lo, hi) of codes drawn as one integer in [0, 225)
_PAIR_LUT = np.array([((v % 15) + 1) | (((v // 15) + 1) << 4) for v in range(225)],
                     dtype=np.uint8)


def _rng_q4_packed(rng: np.random.Generator, nbytes: int) -> np.ndarray:
    """Packed nibbles q + 8 with codes q uniform in [-7, 7] (nibbles 1..15)."""
    return _PAIR_LUT[rng.integers(0, 225, size=nbytes, dtype=np.uint8)]


def _rng_scales(rng: np.random.Generator, count: int) -> np.ndarray:
    s = np.abs(rng.standard_normal(count, dtype=np.float32) * np.float32(0.02)) / np.float32(7.0)
    return s.astype(np.float16).view(np.uint16)


def _rng_gamma(rng, n):
    return (np.float32(1.0) + rng.standard_normal(n, dtype=np.float32) * np.float32(0.02)).astype(
        np.float16).view(np.uint16)


def round_half_away(v: np.ndarray) -> np.ndarray:
    """f32::round semantics (half away from zero)."""
    return np.sign(v) * np.floor(np.abs(v) + np.float32(0.5))


def quantize_q4_rows(w: np.ndarray):
    """Quantise a float32 [rows][cols] matrix per group of 32 along cols (the Q4 scheme of
    src/gemv.rs:7-9: scale = absmax/7 stored as f16, q = round(v/scale) + 8 in [0, 15]).
    Returns (packed uint8 [rows*cols/2], scales uint16 [rows*cols/32])."""
    rows, cols = w.shape
    g = w.reshape(rows, cols // GROUP, GROUP)
    absmax = np.abs(g).max(axis=2)
    scale16 = (absmax / np.float32(7.0)).astype(np.float16)
    s32 = scale16.astype(np.float32)
    with np.errstate(divide="ignore", invalid="ignore"):
        q = np.where(s32[..., None] > 0, round_half_away(g / s32[..., None]), 0.0)
    q = np.clip(q + 8, 0, 15).astype(np.uint8).reshape(rows, cols)
    packed = (q[:, 0::2] | (q[:, 1::2] << 4)).astype(np.uint8).reshape(-1)
    return packed, scale16.view(np.uint16).reshape(-1)


def rope_tables(rows: int, head_dim: int, theta: float):
    half = head_dim // 2
    inv = theta ** (-(2.0 * np.arange(half, dtype=np.float64)) / head_dim)
    ang = np.arange(rows, dtype=np.float64)[:, None] * inv[None, :]
    return np.cos(ang).astype(np.float32).reshape(-1), np.sin(ang).astype(np.float32).reshape(-1)


def synth_q4_matrix(rng, k, n) -> Matrix:
    return Matrix(k, n, packed=_rng_q4_packed(rng, k * n // 2), scales=_rng_scales(rng, k * n // GROUP))


def synth_f16_matrix(rng, k, n) -> Matrix:
    d = (rng.standard_normal(k * n, dtype=np.float32) * np.float32(0.02)).astype(np.float16)
    return Matrix(k, n, data=d.view(np.uint16))


def synth_layer(rng, fmt, hidden, intermediate, nh, nkv, hd) -> Layer:
    mk = synth_q4_matrix if fmt == FORMAT_Q4 else synth_f16_matrix
    shapes = [(hidden, nh * hd), (hidden, nkv * hd), (hidden, nkv * hd), (nh * hd, hidden),
              (hidden, intermediate), (hidden, intermediate), (intermediate, hidden)]
    mats = [mk(rng, k, n) for k, n in shapes]
    return Layer(*mats, _rng_gamma(rng, hidden), _rng_gamma(rng, hidden), nh, nkv, hd, nh // nkv)


def synth_embed(rng, fmt, vocab, hidden, chunk_rows=8192) -> Matrix:
    if fmt == FORMAT_F16:
        return synth_f16_matrix(rng, vocab, hidden)
    packed = np.empty(vocab * hidden // 2, np.uint8)
    scales = np.empty(vocab * hidden // GROUP, np.uint16)
    for r0 in range(0, vocab, chunk_rows):
        r1 = min(vocab, r0 + chunk_rows)
        w = rng.standard_normal((r1 - r0, hidden), dtype=np.float32) * np.float32(0.02)
        p, s = quantize_q4_rows(w)
        packed[r0 * hidden // 2:r1 * hidden // 2] = p
        scales[r0 * hidden // GROUP:r1 * hidden // GROUP] = s
    return Matrix(vocab, hidden, packed=packed, scales=scales)


def synth_model(seed: int = 0, fmt: int = FORMAT_Q4, num_layers: int = 36, vocab: int = 128256,
                hidden: int = 2048, intermediate: int = 11008, num_heads: int = 16,
                num_kv_heads: int = 4, head_dim: int = 128, rope_theta: float = 5e6,
                rope_rows: int = 65536, rope_every: int = 4) -> Model:
    """Seeded random-init model with the SmolLM3-3B architecture by default. RoPE is
    applied on layers i with i % rope_every == rope_every - 1 (3, 7, ..., 35)."""
    rng = np.random.default_rng(seed)
    layers = [synth_layer(rng, fmt, hidden, intermediate, num_heads, num_kv_heads, head_dim)
              for _ in range(num_layers)]
    embed = synth_embed(rng, fmt, vocab, hidden)
    final = _rng_gamma(rng, hidden)
    cos, sin = rope_tables(rope_rows, head_dim, rope_theta)
    no_rope = np.array([1 if (i % rope_every) == rope_every - 1 else 0 for i in range(num_layers)],
                       dtype=np.uint8)
    return Model(fmt, num_layers, vocab, hidden, head_dim // 2, no_rope, layers, embed, final,
                 cos, sin)


# ------------------------------------------------------------------------------ numerics
def f16_bits_to_f32(bits: np.ndarray) -> np.ndarray:
    return bits.view(np.float16).astype(np.float32)


def dequant_q4(m: Matrix, dtype=np.float32) -> np.ndarray:
    """Dense [k][n] values (q - 8) * f32(scale) (exact in f32)."""
    p = m.packed.reshape(m.k, m.n // 2)
    q = np.empty((m.k, m.n), np.int8)
    q[:, 0::2] = (p & 0x0F).astype(np.int8) - 8
    q[:, 1::2] = (p >> 4).astype(np.int8) - 8
    s = f16_bits_to_f32(m.scales).reshape(m.k, m.n // GROUP)
    out = q.reshape(m.k, m.n // GROUP, GROUP).astype(np.float32) * s[..., None]
    return out.reshape(m.k, m.n).astype(dtype)
