"""Pins for the CPU oracle (the reference restatement). The reference ships no tests or
golden vectors, so the oracle is pinned by hand-built known answers (nibble order and
offset, src/gemv.rs:727-731), by bit-level properties the reference's algorithm implies
(threshold and ordered k-split, src/gemv.rs:650-674), by the committed golden fixtures
(tests/golden/), and by an independent float64 NumPy restatement of the model."""
import os

import numpy as np
import pytest

from ref_numpy import RefModel

GOLDEN = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden")


def rel_l2(a, b):
    a, b = np.asarray(a, np.float64), np.asarray(b, np.float64)
    return float(np.linalg.norm(a - b) / max(np.linalg.norm(b), 1e-300))


def f16bits(x):
    return np.array([x], np.float16).view(np.uint16)[0]


def test_nibble_known_answer(qf, orc):
    # byte 0x8F: low nibble 15 -> element 0 = (15-8)*s = +7s; high nibble 8 -> 0
    s = np.float16(0.5)
    packed = np.array([0x8F] + [0x88] * 15, np.uint8)
    scales = np.array([f16bits(s)], np.uint16)
    m = qf.Matrix(1, 32, packed=packed, scales=scales)
    row = orc.embed_q4(m, 0)
    assert row[0] == 3.5 and row[1] == 0.0 and np.all(row[2:] == 0)
    y = orc.gemv_q4(np.array([2.0], np.float32), m)
    assert y[0] == 7.0 and np.all(y[1:] == 0)
    # byte 0x10: low nibble 0 -> -8s, high nibble 1 -> -7s
    m.packed = np.array([0x10] * 16, np.uint8)
    row = orc.embed_q4(m, 0)
    assert np.all(row[0::2] == -4.0) and np.all(row[1::2] == -3.5)


def test_dequant_matches_numpy_exactly(qf, orc):
    rng = np.random.default_rng(5)
    m = qf.synth_q4_matrix(rng, 16, 256)
    d = orc.dequant_q4_rows(m, 0, 16)
    assert np.array_equal(d, qf.dequant_q4(m))


@pytest.mark.parametrize("k,n", [(1, 32), (3, 64), (64, 1024), (2048, 512), (2048, 2048), (2048, 11008), (11008, 2048)])
@pytest.mark.parametrize("T", [1, 3, 8])
def test_gemv_q4_vs_float64(qf, orc, k, n, T):
    rng = np.random.default_rng(k * 7 + n)
    m = qf.synth_q4_matrix(rng, k, n)
    x = rng.standard_normal(k).astype(np.float32)
    orc.set_threads(T)
    y = orc.gemv_q4(x, m)
    ref = x.astype(np.float64) @ qf.dequant_q4(m, np.float64)
    assert rel_l2(y, ref) < 3e-6


def test_gemv_threshold_and_ordered_split(qf, orc):
    rng = np.random.default_rng(11)
    # below 4,000,000: one sequential pass whatever T
    small = qf.synth_q4_matrix(rng, 2048, 512)
    x = rng.standard_normal(2048).astype(np.float32)
    orc.set_threads(5)
    assert np.array_equal(orc.gemv_q4(x, small), orc.gemv_q4_rows(x, small, 0, 2048))
    # at/above: T chunks of ceil(k/T) rows, partials added in chunk order from 0
    big = qf.synth_q4_matrix(rng, 2048, 2048)
    for T in (1, 3, 8):
        orc.set_threads(T)
        ck = -(-2048 // T)
        acc = np.zeros(2048, np.float32)
        for t in range(T):
            if t * ck < 2048:
                acc = acc + orc.gemv_q4_rows(x, big, t * ck, min(2048, (t + 1) * ck))
        assert np.array_equal(orc.gemv_q4(x, big), acc)
    orc.set_threads(1)


def test_avx512_and_scalar_paths_agree(qf, orc):
    lib = orc.lib()
    if not lib.orc_host_has_avx512():
        pytest.skip("host has no AVX-512")
    rng = np.random.default_rng(2)
    m = qf.synth_q4_matrix(rng, 512, 1024)
    g = qf.synth_q4_matrix(rng, 512, 1024)
    x = rng.standard_normal(512).astype(np.float32)
    outs = []
    for on in (False, True):
        orc.set_avx512(on)
        outs.append((orc.gemv_q4(x, m), orc.fused_gate_up_q4(x, m, g)))
    orc.set_avx512(True)
    assert np.array_equal(outs[0][0], outs[1][0])
    assert np.array_equal(outs[0][1], outs[1][1])


def test_fused_gate_up_vs_float64(qf, orc):
    rng = np.random.default_rng(9)
    g = qf.synth_q4_matrix(rng, 2048, 1024)
    u = qf.synth_q4_matrix(rng, 2048, 1024)
    x = rng.standard_normal(2048).astype(np.float32)
    orc.set_threads(4)
    y = orc.fused_gate_up_q4(x, g, u)
    gv = x.astype(np.float64) @ qf.dequant_q4(g, np.float64)
    uv = x.astype(np.float64) @ qf.dequant_q4(u, np.float64)
    ref = gv / (1 + np.exp(-gv)) * uv
    assert rel_l2(y, ref) < 5e-6


def test_lm_head_vs_float64_and_argmax_ties(qf, orc):
    rng = np.random.default_rng(4)
    e = qf.synth_embed(rng, qf.FORMAT_Q4, 1000, 1024)
    x = rng.standard_normal(1024).astype(np.float32)
    lg = orc.lm_head_q4(x, e)
    ref = qf.dequant_q4(e, np.float64) @ x.astype(np.float64)
    assert rel_l2(lg, ref) < 3e-6
    assert orc.argmax(lg) == int(np.argmax(lg))
    tie = np.array([1.0, 3.0, 2.0, 3.0, -np.inf], np.float32)
    assert orc.argmax(tie) == 1  # first strict maximum (src/generate.rs:349-351)
    assert orc.argmax(np.array([np.nan, np.nan], np.float32)) == 0


def test_rms_norm_bit_exact_sequential(qf, orc):
    rng = np.random.default_rng(6)
    x = rng.standard_normal(2048).astype(np.float32)
    g = (1 + 0.02 * rng.standard_normal(2048)).astype(np.float16)
    out = orc.rms_norm(x, g.view(np.uint16))
    s = np.float32(0)
    for v in x:
        s = np.float32(s + np.float32(v * v))
    inv = np.float32(1) / np.sqrt(np.float32(s / np.float32(2048) + np.float32(1e-6)))
    ref = (x * inv) * g.astype(np.float32)
    assert np.array_equal(out, ref)


def test_rope_bit_exact(qf, orc):
    rng = np.random.default_rng(8)
    cos, sin = qf.rope_tables(16, 128, 5e6)
    d = rng.standard_normal(4 * 128).astype(np.float32)
    out = orc.rope(d, 4, 128, cos, sin, 64, 7)
    v = d.reshape(4, 128)
    c, s = cos.reshape(16, 64)[7], sin.reshape(16, 64)[7]
    ref = np.concatenate([v[:, :64] * c - v[:, 64:] * s, v[:, 64:] * c + v[:, :64] * s], axis=1)
    assert np.array_equal(out, ref.reshape(-1))


def test_softmax(orc):
    s = np.array([1.0, 2.0, 3.0, -1e30], np.float32)
    p = orc.softmax(s)
    ref = np.exp(s.astype(np.float64) - 3) / np.exp(s.astype(np.float64) - 3).sum()
    assert np.allclose(p, ref, rtol=1e-6, atol=1e-30) and p[3] == 0.0


def test_f16_gemv(qf, orc):
    rng = np.random.default_rng(12)
    m = qf.synth_f16_matrix(rng, 2048, 2048)
    x = rng.standard_normal(2048).astype(np.float32)
    orc.set_threads(4)
    y = orc.gemv_f16(x, m)
    ref = x.astype(np.float64) @ qf.f16_bits_to_f32(m.data).astype(np.float64).reshape(2048, 2048)
    assert rel_l2(y, ref) < 3e-6


@pytest.fixture(scope="module")
def small_model(qf):
    return qf.synth_model(seed=21, num_layers=4, vocab=512, hidden=1024, intermediate=1024,
                          num_heads=8, num_kv_heads=2, head_dim=128, rope_rows=64)


def test_model_decode_vs_float64(qf, orc, small_model):
    orc.set_threads(4)
    om = orc.OracleModel(small_model)
    kv = om.new_kv()
    ref = RefModel(small_model, qf)
    rkv = ref.new_kv()
    for tok in (5, 77, 300, 1, 511, 42):
        lo = om.forward_decode(tok, kv)
        lr = ref.decode(tok, rkv)
        assert rel_l2(lo, lr) < 1e-5
        assert int(np.argmax(lo)) == int(np.argmax(lr))
    assert kv.length(0) == 6 and kv.length(3) == 6


def test_prefill_equals_decode_sequence(qf, orc, small_model):
    orc.set_threads(2)
    om = orc.OracleModel(small_model)
    ids = np.array([3, 9, 100, 7, 200, 5, 6], np.uint32)
    kv_a = om.new_kv()
    la = om.prefill(ids, kv_a)
    kv_b = om.new_kv()
    for t in ids:
        lb = om.forward_decode(int(t), kv_b)
    assert rel_l2(la, lb) < 1e-5 and np.argmax(la) == np.argmax(lb)
    ka, va = kv_a.export_layer(3, len(ids), 256)
    kb, vb = kv_b.export_layer(3, len(ids), 256)
    assert rel_l2(ka, kb) < 1e-5 and rel_l2(va, vb) < 1e-5


def test_file_and_view_agree(tmp_path, qf, orc, small_model):
    p = tmp_path / "s.qora"
    qf.write_qora(small_model, p)
    a = orc.OracleModel(small_model)
    b = orc.OracleModel(path=p)
    ka, kb = a.new_kv(), b.new_kv()
    assert np.array_equal(a.forward_decode(17, ka), b.forward_decode(17, kb))


def test_golden_fixtures(qf, orc):
    """Committed vectors (tests/golden/make_golden.py) still reproduce: guards the oracle
    and the synthetic generator against silent drift."""
    path = os.path.join(GOLDEN, "golden_small.npz")
    g = np.load(path)
    cfg = {k[4:]: int(g[k]) for k in g.files if k.startswith("cfg_")}
    model = qf.synth_model(**cfg)
    orc.set_threads(int(g["threads"]))
    om = orc.OracleModel(model)
    toks, margins = om.generate_greedy(g["prompt"], len(g["tokens"]))
    assert np.array_equal(toks, g["tokens"])
    kv = om.new_kv()
    lg = om.prefill(g["prompt"], kv)
    assert np.array_equal(lg, g["prefill_logits"])
    x = orc.gemv_q4(g["gemv_x"], model.layers[0].gate_proj)
    assert np.array_equal(x, g["gemv_y"])
    orc.set_threads(1)


# ---------------------------------------------------------------- sampling (src/generate.rs)
def _py_sample(logits, hist, temperature, top_p, top_k, rep, pres, ban, state):
    """Independent restatement of the reference sampling step (f32 arithmetic via numpy
    scalars): penalties (src/generate.rs:64-92), sample_token_top_k (:345-394), Rng (:38-61)."""
    f = np.float32
    l = np.array(logits, np.float32)
    if rep > 1.0:
        for tok in hist[len(hist) - min(len(hist), 64):]:
            l[tok] = l[tok] / f(rep) if l[tok] > 0 else l[tok] * f(rep)
    if pres > 0.0 and len(hist):
        for tok in sorted(set(int(t) for t in hist)):
            l[tok] = l[tok] - f(pres)
    if ban >= 0:
        l[ban] = -np.inf
    if temperature <= 0.0:
        return int(np.argmax(l)), state
    inv_temp = f(1.0) / f(temperature)
    mx = f(np.max(l))
    order = sorted(range(len(l)), key=lambda i: -float(l[i]))  # stable: ties keep index order
    k = min(top_k, len(l)) if top_k > 0 else len(l)
    probs = [(i, f(np.exp(f((l[i] - mx) * inv_temp)))) for i in order[:k]]
    s = f(0.0)
    for _, p in probs:
        s = f(s + p)
    if s <= 0:
        return probs[0][0], state
    inv = f(f(1.0) / s)
    probs = [(i, f(p * inv)) for i, p in probs]
    cum, cut = f(0.0), len(probs)
    for j, (_, p) in enumerate(probs):
        cum = f(cum + p)
        if cum >= f(top_p):
            cut = j + 1
            break
    tot = f(0.0)
    for _, p in probs[:cut]:
        tot = f(tot + p)
    if tot <= 0:
        return probs[0][0], state
    m = (1 << 64) - 1
    state ^= (state << 13) & m
    state ^= state >> 7
    state ^= (state << 17) & m
    r = f(f(state >> 40) / f(16777216.0)) * tot
    acc = f(0.0)
    for i, p in probs[:cut]:
        acc = f(acc + p)
        if acc >= r:
            return i, state
    return probs[0][0], state


def test_sampling_restatement_pins_oracle(orc):
    """The oracle's sampling step against the Python restatement on seeded cases:
    identical tokens and generator states (greedy, top-k/top-p, penalties with repeated
    history tokens, a banned token)."""
    rng = np.random.default_rng(5)
    cases = [(0.0, 0.95, 20, 1.0, 0.0, -1), (0.6, 0.95, 20, 1.1, 1.5, -1), (1.0, 1.0, 1, 1.0, 0.0, -1),
             (0.3, 0.5, 50, 1.3, 0.0, 7), (1.5, 0.99, 200, 1.0, 0.7, 3)]
    for it in range(40):
        V = int(rng.integers(50, 400))
        logits = (rng.standard_normal(V) * rng.uniform(0.5, 4)).astype(np.float32)
        hist = rng.integers(0, V, size=int(rng.integers(0, 90))).astype(np.uint32)
        if hist.size > 3:
            hist[-2] = hist[-1]  # a duplicate inside the 64-token window
        t, tp, k, rp, pp, ban = cases[it % len(cases)]
        ban = ban if ban < V else -1
        state = int(rng.integers(1, 2**63))
        a = orc.sample(logits, hist, t, tp, k, rp, pp, ban, state)
        b = _py_sample(logits, hist, t, tp, k, rp, pp, ban, state)
        assert a == b, (it, a, b)


# ---------------------------------------------------------------- opt-in binary16 KV
def test_round_f16_matches_numpy(orc):
    """orc_round_f16 against numpy's float32 -> float16 conversion (round to nearest
    even), bit for bit: random bit patterns, every midpoint between adjacent positive
    binary16 values (the ties) and its f32 neighbours, overflow and subnormal edges."""
    rng = np.random.default_rng(0)
    parts = [rng.integers(0, 2**32, size=200_000, dtype=np.uint64).astype(np.uint32).view(np.float32)]
    for s in (1e-6, 1e-3, 1.0, 1e3, 6e4):
        parts.append((rng.standard_normal(50_000) * s).astype(np.float32))
    f = np.arange(0, 0x7C00, dtype=np.uint16).view(np.float16).astype(np.float64)
    mids = ((f[:-1] + f[1:]) / 2).astype(np.float32)  # exact: <= 12 significant bits
    parts += [mids, -mids, np.nextafter(mids, np.float32(np.inf)), np.nextafter(mids, np.float32(0))]
    parts.append(np.array([0.0, -0.0, 65504.0, 65519.996, 65520.0, -65520.0, 2.0**-24, 2.0**-25,
                           3 * 2.0**-26, 1e-45, np.inf, -np.inf, np.nan], np.float32))
    x = np.concatenate(parts).astype(np.float32)
    with np.errstate(over="ignore", invalid="ignore"):
        want = x.astype(np.float16).astype(np.float32)
    got = orc.round_f16(x)
    nan = np.isnan(x)
    assert np.array_equal(got[~nan].view(np.uint32), want[~nan].view(np.uint32))
    assert np.all(np.isnan(got[nan]))


def test_kv_f16_mode_vs_float64(qf, orc):
    """The oracle's binary16 cache against the float64 restatement with float16-rounded
    K/V, on one decoder layer: rounding amplifies differences of the last f32 bits into
    whole binary16 steps (an element on the other side of a rounding boundary), which
    compound over layers, so the pin uses one layer, where the two agree ~17x closer than
    the f16 and f32 caches do."""
    orc.set_threads(4)
    m = qf.synth_model(seed=21, num_layers=1, vocab=512, hidden=1024, intermediate=1024,
                       num_heads=8, num_kv_heads=2, head_dim=128, rope_rows=64)
    om = orc.OracleModel(m)
    kv, kv32 = om.new_kv("f16"), om.new_kv()
    ref = RefModel(m, qf, kv_f16=True)
    rkv = ref.new_kv()
    for tok in (5, 77, 300, 1, 511, 42):
        lo = om.forward_decode(tok, kv)
        lr = ref.decode(tok, rkv)
        l32 = om.forward_decode(tok, kv32)
        assert rel_l2(lo, lr) < 3e-5
        assert int(np.argmax(lo)) == int(np.argmax(lr))
        assert 1e-4 < rel_l2(lo, l32) < 1e-2  # a different cache, close to the f32 one


def test_kv_f16_cache_contents(orc, small_model):
    """Every cached value is a binary16 value; layer 0 of the first step holds exactly the
    rounded values of the f32 cache (same inputs up to there)."""
    om = orc.OracleModel(small_model)
    kv, kv32 = om.new_kv("f16"), om.new_kv()
    toks = (5, 77, 300, 1)
    for i, tok in enumerate(toks):
        om.forward_decode(tok, kv)
        om.forward_decode(tok, kv32)
        if i == 0:
            k16, v16 = kv.export_layer(0, 1, 256)
            k32, v32 = kv32.export_layer(0, 1, 256)
            assert np.array_equal(k16, orc.round_f16(k32)) and np.array_equal(v16, orc.round_f16(v32))
    for layer in range(4):
        k, v = kv.export_layer(layer, len(toks), 256)
        assert np.array_equal(k, orc.round_f16(k)) and np.array_equal(v, orc.round_f16(v))


def test_kv_f16_import_prefill_and_mode_switch(qf, orc):
    """Import rounds; prefill attends to the rounded keys/values like a decode sequence
    (one layer: see test_kv_f16_mode_vs_float64 on amplification); mode switch only on an
    empty cache."""
    orc.set_threads(3)
    om = orc.OracleModel(qf.synth_model(seed=21, num_layers=1, vocab=512, hidden=1024, intermediate=1024,
                                        num_heads=8, num_kv_heads=2, head_dim=128, rope_rows=64))
    rng = np.random.default_rng(8)
    K = rng.standard_normal((9, 256)).astype(np.float32)
    V = rng.standard_normal((9, 256)).astype(np.float32)
    kv = om.new_kv("f16")
    kv.import_layer(0, K, V)
    k, v = kv.export_layer(0, 9, 256)
    assert np.array_equal(k, orc.round_f16(K)) and np.array_equal(v, orc.round_f16(V))
    ids = np.array([3, 9, 100, 7, 200, 5, 6], np.uint32)
    kv_a, kv_b = om.new_kv("f16"), om.new_kv("f16")
    la = om.prefill(ids, kv_a)
    for t in ids:
        lb = om.forward_decode(int(t), kv_b)
    assert rel_l2(la, lb) < 1e-5 and np.argmax(la) == np.argmax(lb)
    assert orc.lib().orc_kv_set_f16(kv_b.h, 0) != 0  # not on a non-empty cache
    with pytest.raises(ValueError):
        om.new_kv("bf16")
