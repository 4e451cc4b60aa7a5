"""Opt-in binary16 KV cache (QORA_KV_F16) on the persistent Q4 decode step, through the C
ABI, against the oracle's binary16 mode: K and V are rounded to nearest even as they
enter the cache (decode append, import) and attention reads the rounded values.

Bars: imported rows bit-exact after the round trip (export == round_f16(import));
logits within rel-L2 1e-3 of the oracle (rounding turns differences
in the last bits of two f32 computations of a key into whole binary16 steps, which then
compound over layers, so the measured values sit near 1e-4 instead of 1e-6); greedy
tokens identical."""
import ctypes as C

import numpy as np
import pytest

pytestmark = pytest.mark.gpu

LOGIT_TOL = 1e-3


def rel_l2(a, b):
    a, b = np.asarray(a, np.float64), np.asarray(b, np.float64)
    return float(np.linalg.norm(a - b) / max(np.linalg.norm(b), 1e-300))


@pytest.fixture(scope="module")
def model(qf):
    return qf.synth_model(seed=7, num_layers=4, vocab=2048, hidden=1024, intermediate=1536,
                          num_heads=8, num_kv_heads=2, head_dim=128, rope_rows=4096)


@pytest.fixture(scope="module")
def engine(pkg, model):
    w = pkg.DecodeWeights(model=model)
    yield w
    w.close()


@pytest.fixture(scope="module")
def oracle_model(orc, model):
    orc.set_threads(8)
    return orc.OracleModel(model)


def test_kv16_import_export_rounds(engine, orc):
    rng = np.random.default_rng(1)
    kv = engine.new_kv(512, dtype="f16")
    K = (rng.standard_normal((300, 256)) * 3).astype(np.float32)
    V = (rng.standard_normal((300, 256)) * 3).astype(np.float32)
    for layer in range(engine.num_layers):
        kv.import_layer(layer, K, V)
    k, v = kv.export_layer(2, 300, 256)
    assert np.array_equal(k.view(np.uint32), orc.round_f16(K).view(np.uint32))
    assert np.array_equal(v.view(np.uint32), orc.round_f16(V).view(np.uint32))
    assert len(kv) == 300


def test_kv16_teacher_forced(engine, oracle_model):
    w, om = engine, oracle_model
    kv = w.new_kv(256, dtype="f16")
    okv = om.new_kv("f16")
    rng = np.random.default_rng(3)
    worst = 0.0
    for tok in rng.integers(0, w.vocab, size=30):
        am, lg = w.decode_step(kv, int(tok), want_logits=True)
        lo = om.forward_decode(int(tok), okv)
        worst = max(worst, rel_l2(lg, lo))
        top = np.sort(lo)[-2:]
        assert am == int(np.argmax(lo)), f"argmax differs, oracle margin {top[1] - top[0]}"
    print(f"binary16 KV teacher-forced worst logits rel-L2 {worst:.3e}")
    assert worst < LOGIT_TOL
    # every cached value is a binary16 value
    k, v = kv.export_layer(1, 30, 256)
    assert np.array_equal(k, k.astype(np.float16).astype(np.float32))
    assert np.array_equal(v, v.astype(np.float16).astype(np.float32))


def test_kv16_prefill_then_greedy(engine, oracle_model):
    w, om = engine, oracle_model
    prompt = np.random.default_rng(4).integers(0, w.vocab, size=12).astype(np.uint32)
    kv = w.new_kv(256, dtype="f16")
    first, lg = w.prefill(kv, prompt)
    okv = om.new_kv("f16")
    lo = om.prefill(prompt, okv)
    assert rel_l2(lg, lo) < LOGIT_TOL
    assert first == int(np.argmax(lo))
    toks = w.generate_greedy(kv, first, 40)
    ref, margins = om.generate_greedy(prompt, 41, om.new_kv("f16"))
    assert ref[0] == first
    assert np.array_equal(toks, ref[1:]), f"min oracle margin {margins.min()}"


def test_kv16_long_context(engine, oracle_model, orc):
    """2,500 imported positions per layer (40 position chunks per KV head, 135 binary16
    rows per ring stage), then teacher-forced steps; the f32 cache given the same import
    lands close but not equal."""
    w, om = engine, oracle_model
    rng = np.random.default_rng(9)
    n = 2500
    kv, kv32 = w.new_kv(n + 16, dtype="f16"), w.new_kv(n + 16)
    okv = om.new_kv("f16")
    for layer in range(w.num_layers):
        K = rng.standard_normal((n, 256)).astype(np.float32)
        V = rng.standard_normal((n, 256)).astype(np.float32)
        kv.import_layer(layer, K, V)
        kv32.import_layer(layer, K, V)
        okv.import_layer(layer, K, V)
    worst, apart = 0.0, 1.0
    for tok in rng.integers(0, w.vocab, size=8):
        am, lg = w.decode_step(kv, int(tok), want_logits=True)
        _, l32 = w.decode_step(kv32, int(tok), want_logits=True)
        lo = om.forward_decode(int(tok), okv)
        worst = max(worst, rel_l2(lg, lo))
        apart = min(apart, rel_l2(l32, lo))
        top = np.sort(lo)[-2:]
        assert am == int(np.argmax(lo)), f"argmax differs, oracle margin {top[1] - top[0]}"
    print(f"binary16 KV at {n} positions: worst logits rel-L2 {worst:.3e} (f32 cache {apart:.3e} away)")
    assert worst < LOGIT_TOL
    assert apart > 0.0


def test_kv16_rejections(pkg, qf, engine, model):
    w = engine
    with pytest.raises(pkg.QoraError, match="UNSUPPORTED"):
        w.new_kv(10 ** 5, dtype="f16")  # beyond the persistent step's attention plan
    with pytest.raises(ValueError):
        w.new_kv(64, dtype="bf16")
    h = C.c_void_p()
    assert pkg.engine.lib().qora_kv_create_ex(w.h, 64, 1, 7, C.byref(h)) == 1  # QORA_ERR_INVALID
    kv = w.new_kv(64, dtype="f16")
    with pytest.raises(pkg.QoraError, match="UNSUPPORTED"):
        w.layer_step(kv, 0, np.zeros(w.hidden, np.float32))  # per-op kernels read f32 caches
    wp = pkg.DecodeWeights(model=model, per_op_kernels=True)
    with pytest.raises(pkg.QoraError, match="UNSUPPORTED"):
        wp.new_kv(64, dtype="f16")
    wp.close()
    m16 = qf.synth_model(seed=3, fmt=qf.FORMAT_F16, num_layers=1, vocab=256, hidden=1024, intermediate=1536,
                         num_heads=8, num_kv_heads=2, head_dim=128, rope_rows=64)
    w16 = pkg.DecodeWeights(model=m16)
    with pytest.raises(pkg.QoraError, match="UNSUPPORTED"):
        w16.new_kv(32, dtype="f16")
    w16.close()
