"""The .qora container (src/save.rs layout): round trip, byte-level header, and the
reader's error behaviour on corrupted / truncated files (src/save.rs:158-169, :233-236),
for both the Python reader and the oracle's C++ reader."""
import struct

import numpy as np
import pytest


def tiny(qf, seed=0, **kw):
    args = dict(num_layers=2, vocab=64, hidden=1024, intermediate=512, num_heads=8,
                num_kv_heads=2, head_dim=128, rope_rows=32)
    args.update(kw)
    return qf.synth_model(seed=seed, **args)


def test_round_trip(tmp_path, qf):
    m = tiny(qf)
    p = tmp_path / "m.qora"
    qf.write_qora(m, p)
    r = qf.read_qora(p)
    assert (r.format, r.num_layers, r.vocab, r.hidden, r.rope_half_dim) == (
        m.format, m.num_layers, m.vocab, m.hidden, m.rope_half_dim)
    assert np.array_equal(r.no_rope_layers, m.no_rope_layers)
    for La, Lb in zip(m.layers, r.layers):
        for a, b in zip(La.mats(), Lb.mats()):
            assert (a.k, a.n) == (b.k, b.n)
            assert np.array_equal(a.packed, b.packed) and np.array_equal(a.scales, b.scales)
        assert np.array_equal(La.input_norm_gamma, Lb.input_norm_gamma)
        assert (La.num_heads, La.num_kv_heads, La.head_dim, La.num_kv_groups) == (
            Lb.num_heads, Lb.num_kv_heads, Lb.head_dim, Lb.num_kv_groups)
    assert np.array_equal(r.embed.packed, m.embed.packed)
    assert np.array_equal(r.rope_cos, m.rope_cos) and np.array_equal(r.rope_sin, m.rope_sin)


def test_header_bytes(tmp_path, qf):
    m = tiny(qf, num_layers=4)
    p = tmp_path / "m.qora"
    qf.write_qora(m, p)
    b = p.read_bytes()
    assert b[:4] == b"QOR3"
    assert struct.unpack("<I", b[4:8])[0] == 1
    assert b[8] == 1  # Q4
    assert struct.unpack("<4I", b[9:25]) == (4, 64, 1024, 64)
    assert struct.unpack("<Q", b[25:33])[0] == 4
    assert list(b[33:37]) == [0, 0, 0, 1]  # RoPE on layer 3 only
    # first weight record: k, n, packed length prefix
    assert struct.unpack("<3Q", b[37:61]) == (1024, 1024, 1024 * 1024 // 2)


def test_synthetic_distributions(qf):
    m = tiny(qf, num_layers=1, vocab=256)
    p = m.layers[0].gate_proj.packed
    nib = np.concatenate([p & 15, p >> 4])
    assert nib.min() == 1 and nib.max() == 15  # codes uniform in [-7, 7]
    s = qf.f16_bits_to_f32(m.layers[0].gate_proj.scales)
    assert (s >= 0).all() and 0.001 < s.mean() < 0.003  # |N(0,0.02)|/7 has mean ~0.00228
    g = qf.f16_bits_to_f32(m.layers[0].input_norm_gamma)
    assert abs(g.mean() - 1) < 0.01
    # embedding quantiser: absmax/7 scale, codes within [0, 15] and absmax element at +-7
    e = qf.dequant_q4(m.embed)
    assert e.shape == (256, 1024)


def _corrupt(tmp_path, qf, mutate):
    m = tiny(qf)
    p = tmp_path / "bad.qora"
    qf.write_qora(m, p)
    b = bytearray(p.read_bytes())
    b = mutate(b)
    p.write_bytes(bytes(b))
    return p


CORRUPTIONS = {
    "magic": (lambda b: b"QOR4" + b[4:], "magic"),
    "version": (lambda b: b[:4] + struct.pack("<I", 2) + b[8:], "version"),
    "format": (lambda b: b[:8] + bytes([7]) + b[9:], "format"),
    "truncated": (lambda b: b[: len(b) // 2], "short read"),
    "empty": (lambda b: b"", "short read"),
}


@pytest.mark.parametrize("kind", sorted(CORRUPTIONS))
def test_corrupted_python_reader(tmp_path, qf, kind):
    mut, msg = CORRUPTIONS[kind]
    p = _corrupt(tmp_path, qf, mut)
    with pytest.raises(qf.QoraFormatError, match="(?i)" + msg.split()[0]):
        qf.read_qora(p)


@pytest.mark.parametrize("kind", sorted(CORRUPTIONS))
def test_corrupted_oracle_reader(tmp_path, qf, orc, kind):
    mut, msg = CORRUPTIONS[kind]
    p = _corrupt(tmp_path, qf, mut)
    with pytest.raises(qf.QoraFormatError, match="(?i)" + msg.split()[0]):
        orc.OracleModel(path=p)


def test_quantizer_round_trip(qf):
    rng = np.random.default_rng(3)
    w = rng.standard_normal((8, 64), dtype=np.float32) * np.float32(0.02)
    packed, scales = qf.quantize_q4_rows(w)
    mat = qf.Matrix(8, 64, packed=packed, scales=scales)
    d = qf.dequant_q4(mat)
    s = qf.f16_bits_to_f32(scales).reshape(8, 2)
    assert np.all(np.abs(d - w) <= s.repeat(32, axis=1) * 0.5 + 1e-7)
    # the element of largest magnitude in each group maps to code +-7
    q = np.empty((8, 64), np.int16)
    q[:, 0::2] = (packed.reshape(8, 32) & 15).astype(np.int16) - 8
    q[:, 1::2] = (packed.reshape(8, 32) >> 4).astype(np.int16) - 8
    assert np.abs(q).max() == 7


@pytest.mark.parametrize("kind", sorted(CORRUPTIONS))
def test_corrupted_engine_reader(tmp_path, qf, pkg, kind):
    """The engine's own (memory-mapped) reader rejects the same files before any device
    work: a truncated file is an I/O error, the rest are invalid contents."""
    mut, msg = CORRUPTIONS[kind]
    p = _corrupt(tmp_path, qf, mut)
    with pytest.raises(pkg.QoraError) as ei:
        pkg.DecodeWeights(path=str(p))
    want = 2 if msg == "short read" else 1  # QORA_ERR_IO / QORA_ERR_INVALID
    assert ei.value.status == want, str(ei.value)


def test_engine_reader_accepts_valid_file(tmp_path, qf, pkg):
    """A well-formed file passes the engine's reader and view validation; without a GPU the
    first failure is the device (QORA_ERR_CUDA), with one the engine loads."""
    try:
        import torch
        if torch.cuda.is_available():
            pytest.skip("a GPU is present (the GPU tests load files)")
    except Exception:
        pass
    p = tmp_path / "ok.qora"
    qf.write_qora(tiny(qf), p)
    with pytest.raises(pkg.QoraError) as ei:
        pkg.DecodeWeights(path=str(p))
    assert ei.value.status == 3, str(ei.value)


@pytest.mark.parametrize("k,n", [(1 << 32, 1 << 32), (1 << 40, 16), (1 << 21, 1 << 20)])
def test_engine_reader_rejects_wrapping_shapes(tmp_path, qf, pkg, k, n):
    """A matrix header whose k*n would wrap (or exceed 2^40 elements) is rejected before any
    size arithmetic: the first layer's q_proj shape is overwritten in a valid file."""
    m = tiny(qf)
    p = tmp_path / "shape.qora"
    qf.write_qora(m, p)
    b = bytearray(p.read_bytes())
    off = 4 + 4 + 1 + 4 * 4 + 8 + m.num_layers  # header, no_rope_layers vector
    assert struct.unpack_from("<QQ", b, off) == (m.layers[0].q_proj.k, m.layers[0].q_proj.n)
    struct.pack_into("<QQ", b, off, k, n)
    p.write_bytes(bytes(b))
    with pytest.raises(pkg.QoraError, match="implausible matrix shape") as ei:
        pkg.DecodeWeights(path=str(p))
    assert ei.value.status == 1
