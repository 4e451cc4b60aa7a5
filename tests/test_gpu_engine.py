"""Engine-level parity on the GPU: one decoder layer (benchmark config 2), whole decode
steps teacher-forced with random tokens, prefill + greedy generation, the .qora file
path, error behaviour and determinism — all through the C ABI, against the oracle.

Tolerances: logits within rel-L2 1e-3 of the oracle (the measured
value is printed and typically ~1e-6); one layer's output within 1e-5; greedy token
sequences identical."""
import numpy as np
import pytest

pytestmark = pytest.mark.gpu

LOGIT_TOL = 1e-3
LAYER_TOL = 1e-5


def rel_l2(a, b):
    a, b = np.asarray(a, np.float64), np.asarray(b, np.float64)
    return float(np.linalg.norm(a - b) / max(np.linalg.norm(b), 1e-300))


@pytest.fixture(scope="module")
def small(qf):
    return qf.synth_model(seed=7, num_layers=4, vocab=2048, hidden=1024, intermediate=1536,
                          num_heads=8, num_kv_heads=2, head_dim=128, rope_rows=256)


@pytest.fixture(scope="module", params=["megakernel", "per_op_kernels"])
def small_engine(request, pkg, small):
    """Both decode paths: the persistent single-kernel step and the graph of per-op kernels."""
    w = pkg.DecodeWeights(model=small, per_op_kernels=request.param == "per_op_kernels")
    yield w
    w.close()


@pytest.fixture(scope="module")
def small_oracle(orc, small):
    orc.set_threads(8)
    return orc.OracleModel(small)


def test_layer_config2(pkg, qf, orc):
    """benchmark config 2: one SmolLM3 layer at batch 1, KV pre-filled with 512 rows of
    N(0,1), hidden N(0,1), position 512; a RoPE layer (index 3) and a NoPE layer."""
    model = qf.synth_model(seed=2, num_layers=4, vocab=256, rope_rows=1024)
    rng = np.random.default_rng(22)
    w = pkg.DecodeWeights(model=model)
    kv = w.new_kv(1024)
    om = orc.OracleModel(model)
    okv = om.new_kv()
    orc.set_threads(8)
    for layer in (3, 0):
        assert bool(model.no_rope_layers[layer]) == (layer == 3)
        K = rng.standard_normal((512, 512)).astype(np.float32)
        V = rng.standard_normal((512, 512)).astype(np.float32)
        kv.import_layer(layer, K, V)
        okv.import_layer(layer, K, V)
        x = rng.standard_normal(2048).astype(np.float32)
        y = w.layer_step(kv, layer, x)
        yo = om.layer_forward(layer, x, okv)
        err = rel_l2(y, yo)
        print(f"layer {layer} rel-L2 {err:.3e}")
        assert err < LAYER_TOL
        kg, vg = kv.export_layer(layer, 513, 512)
        ko, vo = okv.export_layer(layer, 513, 512)
        assert np.array_equal(kg[:512], K) and rel_l2(kg[512], ko[512]) < LAYER_TOL
        assert rel_l2(vg[512], vo[512]) < LAYER_TOL
    kv.close()
    w.close()


def test_decode_teacher_forced(small_engine, small_oracle):
    w, om = small_engine, small_oracle
    kv = w.new_kv(256)
    okv = om.new_kv()
    rng = np.random.default_rng(3)
    worst = 0.0
    for tok in rng.integers(0, w.vocab, size=40):
        am, lg = w.decode_step(kv, int(tok), want_logits=True)
        lo = om.forward_decode(int(tok), okv)
        worst = max(worst, rel_l2(lg, lo))
        top = np.sort(lo)[-2:]
        assert am == int(np.argmax(lo)), f"argmax differs, oracle margin {top[1] - top[0]}"
    print(f"teacher-forced worst logits rel-L2 {worst:.3e}")
    assert worst < LOGIT_TOL
    assert len(kv) == 40


def test_prefill_then_greedy(small_engine, small_oracle):
    w, om = small_engine, small_oracle
    prompt = np.random.default_rng(4).integers(0, w.vocab, size=12).astype(np.uint32)
    kv = w.new_kv(256)
    first, lg = w.prefill(kv, prompt)
    okv = om.new_kv()
    lo = om.prefill(prompt, okv)
    assert rel_l2(lg, lo) < LOGIT_TOL
    assert first == int(np.argmax(lo))
    toks = w.generate_greedy(kv, first, 40)
    ref, margins = om.generate_greedy(prompt, 41)
    assert ref[0] == first
    assert np.array_equal(toks, ref[1:]), f"min oracle margin {margins.min()}"
    assert len(kv) == 12 + 40


def test_decode_step_matches_generate(small_engine):
    w = small_engine
    a, b = w.new_kv(64), w.new_kv(64)
    toks = w.generate_greedy(a, 5, 10)
    t = 5
    seq = []
    for _ in range(10):
        t = w.decode_step(b, t)
        seq.append(t)
    assert np.array_equal(toks, np.array(seq, np.uint32))


def test_file_engine_equals_view_engine(tmp_path, pkg, qf, small, small_engine):
    p = tmp_path / "small.qora"
    qf.write_qora(small, p)
    wf = pkg.DecodeWeights(path=str(p), per_op_kernels=small_engine.per_op_kernels)
    ka, kb = small_engine.new_kv(16), wf.new_kv(16)
    for tok in (1, 2, 3):
        _, la = small_engine.decode_step(ka, tok, want_logits=True)
        _, lb = wf.decode_step(kb, tok, want_logits=True)
        assert np.array_equal(la, lb)
    wf.close()


def test_reference_named_api(pkg, small_engine, small_oracle):
    logits, kv = pkg.raw_prefill(small_engine, [9, 8, 7], max_seq=32)
    okv = small_oracle.new_kv()
    assert rel_l2(logits, small_oracle.prefill(np.array([9, 8, 7], np.uint32), okv)) < LOGIT_TOL
    lg = pkg.forward_decode_raw(small_engine, 11, kv)
    assert rel_l2(lg, small_oracle.forward_decode(11, okv)) < LOGIT_TOL


def test_errors(pkg, small_engine):
    w = small_engine
    kv = w.new_kv(4)
    with pytest.raises(pkg.QoraError, match="RANGE"):
        w.decode_step(kv, w.vocab)  # token id out of range
    for t in range(4):
        w.decode_step(kv, t)
    with pytest.raises(pkg.QoraError, match="RANGE"):
        w.decode_step(kv, 0)  # cache full
    with pytest.raises(pkg.QoraError, match="RANGE"):
        kv.import_layer(0, np.zeros((5, 256), np.float32), np.zeros((5, 256), np.float32))
    with pytest.raises(pkg.QoraError, match="RANGE"):
        w.new_kv(10 ** 6)  # beyond the RoPE table
    kv.reset()
    assert len(kv) == 0
    w.decode_step(kv, 3)
    with pytest.raises(pkg.QoraError, match="INVALID"):
        w.prefill(kv, [])


def test_deterministic(small_engine):
    w = small_engine
    outs = []
    for _ in range(2):
        kv = w.new_kv(32)
        outs.append([w.decode_step(kv, t, want_logits=True)[1] for t in (3, 1, 4, 1, 5)])
    for a, b in zip(*outs):
        assert np.array_equal(a, b)


def test_paths_agree(pkg, small):
    a = pkg.DecodeWeights(model=small)
    b = pkg.DecodeWeights(model=small, per_op_kernels=True)
    assert a.launches_per_step() == 1 and b.launches_per_step() > 1
    ka, kb = a.new_kv(64), b.new_kv(64)
    for tok in (7, 700, 70):
        am, la = a.decode_step(ka, tok, want_logits=True)
        bm, lb = b.decode_step(kb, tok, want_logits=True)
        assert am == bm and rel_l2(la, lb) < 1e-5
    a.close()
    b.close()


def test_engine_destroyed_before_cache(pkg, small):
    w = pkg.DecodeWeights(model=small)
    kv = w.new_kv(8)
    w.decode_step(kv, 1)
    w.close()  # the cache outlives its engine: it becomes inert, not dangling
    with pytest.raises(pkg.QoraError, match="INVALID"):
        kv.import_layer(0, np.zeros((1, 256), np.float32), np.zeros((1, 256), np.float32))
    kv.close()


def test_sample_on_device_matches_oracle(small_engine, orc):
    """qora_sample on the Q4 engine's last-step logits (kept on the device) against the
    oracle's sampling step on the same logits; the generator state threads through."""
    w = small_engine
    kv = w.new_kv(64)
    prompt = np.random.default_rng(31).integers(0, w.vocab, size=7).astype(np.uint32)
    first, _ = w.prefill(kv, prompt, want_logits=False)
    hist = list(prompt) + [first]
    tok, state = first, 0x2545F4914F6CDD1D
    for _ in range(6):
        am, logits = w.decode_step(kv, tok, want_logits=True)
        got = w.sample(hist, 0.7, 0.9, 20, 1.1, 1.5, -1, state)
        want = orc.sample(logits, hist, 0.7, 0.9, 20, 1.1, 1.5, -1, state)
        assert got == want
        assert w.sample([], 0.0, 1.0, 1)[0] == am
        tok, state = got
        hist.append(tok)
