"""F16-weight engines (benchmark config 5 at test sizes): batched decode of independent
sequences and chunked prefill, through the C ABI, against the CPU oracle.

Bars: logits within rel-L2 1e-3 of the oracle (measured values are printed; the
tensor-core GEMM splits each f32 activation into two f16 terms, so they sit near 1e-6);
greedy token sequences identical to the oracle's for every sequence of the batch."""
import numpy as np
import pytest

pytestmark = pytest.mark.gpu

LOGIT_TOL = 1e-3


def rel_l2(a, b):
    a, b = np.asarray(a, np.float64), np.asarray(b, np.float64)
    return float(np.linalg.norm(a - b) / max(np.linalg.norm(b), 1e-300))


@pytest.fixture(scope="module")
def f16_model(qf):
    return qf.synth_model(seed=17, fmt=qf.FORMAT_F16, num_layers=4, vocab=2048, hidden=1024,
                          intermediate=1536, num_heads=8, num_kv_heads=2, head_dim=128,
                          rope_rows=512)


@pytest.fixture(scope="module")
def f16_engine(pkg, f16_model):
    w = pkg.DecodeWeights(model=f16_model)
    yield w
    w.close()


@pytest.fixture(scope="module")
def f16_oracle(orc, f16_model):
    orc.set_threads(8)
    return orc.OracleModel(f16_model)


def _prompts(vocab, lens, seed):
    rng = np.random.default_rng(seed)
    return [rng.integers(0, vocab, size=n).astype(np.uint32) for n in lens]


def test_f16_prefill_and_decode_logits(f16_engine, f16_oracle):
    """Prefill logits, then teacher-forced decode steps, row by row against the oracle."""
    w, om = f16_engine, f16_oracle
    prompt = _prompts(w.vocab, [13], 3)[0]
    kv = w.new_kv(256)
    okv = om.new_kv()
    first, logits = w.prefill(kv, prompt)
    lo = om.prefill(prompt, okv)
    assert first == int(np.argmax(lo))
    r = rel_l2(logits, lo)
    assert r < LOGIT_TOL, r
    worst = r
    rng = np.random.default_rng(4)
    for tok in rng.integers(0, w.vocab, size=6):
        am, lg = w.decode_batch(kv, [int(tok)], want_logits=True)
        ref = om.forward_decode(int(tok), okv)
        worst = max(worst, rel_l2(lg[0], ref))
        assert am[0] == int(np.argmax(ref))
    assert worst < LOGIT_TOL, worst
    assert len(kv) == 13 + 6
    print(f"F16 prefill+decode logits: worst rel-L2 {worst:.3e}")


def test_f16_batched_greedy_matches_oracle(f16_engine, f16_oracle):
    """Eight sequences with ragged prompt lengths decode together; each sequence's greedy
    tokens equal the oracle's generation for that prompt alone."""
    w, om = f16_engine, f16_oracle
    lens = [5, 17, 9, 1, 30, 12, 7, 22]
    prompts = _prompts(w.vocab, lens, 8)
    kv = w.new_kv(128, batch=len(lens))
    firsts = []
    for b, p in enumerate(prompts):
        f, _ = w.prefill(kv, p, want_logits=False, seq=b)
        firsts.append(f)
    n = 20
    out = w.generate_greedy_batch(kv, firsts, n)
    assert out.shape == (n, len(lens))
    for b, p in enumerate(prompts):
        ref, margins = om.generate_greedy(p, n + 1)
        assert firsts[b] == ref[0], b
        assert np.array_equal(out[:, b], ref[1:]), f"seq {b}: min oracle margin {margins.min()}"
        assert kv.length(b) == lens[b] + n


def test_f16_batched_step_logits(f16_engine, f16_oracle):
    """One batched decode step with logits read back: every row matches the oracle's
    single-sequence step at that sequence's own position."""
    w, om = f16_engine, f16_oracle
    lens = [3, 11, 6]
    prompts = _prompts(w.vocab, lens, 9)
    kv = w.new_kv(64, batch=3)
    okvs = []
    for b, p in enumerate(prompts):
        w.prefill(kv, p, want_logits=False, seq=b)
        okv = om.new_kv()
        om.prefill(p, okv)
        okvs.append(okv)
    toks = [5, 1000, 2047]
    am, lg = w.decode_batch(kv, toks, want_logits=True)
    for b in range(3):
        ref = om.forward_decode(toks[b], okvs[b])
        assert rel_l2(lg[b], ref) < LOGIT_TOL
        assert am[b] == int(np.argmax(ref))


def test_f16_long_prefill_chunks(f16_engine, f16_oracle):
    """A 300-token prompt runs as three row chunks (128 + 128 + 44)."""
    w, om = f16_engine, f16_oracle
    prompt = _prompts(w.vocab, [300], 12)[0]
    kv = w.new_kv(320)
    first, logits = w.prefill(kv, prompt)
    lo = om.prefill(prompt, om.new_kv())
    r = rel_l2(logits, lo)
    assert r < LOGIT_TOL, r
    assert first == int(np.argmax(lo))
    print(f"F16 300-token prefill logits rel-L2 {r:.3e}")


def test_f16_batch32_config5_shape(f16_engine, f16_oracle):
    """32 sequences (config 5's larger batch) at test model size."""
    w, om = f16_engine, f16_oracle
    B, n = 32, 8
    prompts = _prompts(w.vocab, [16] * B, 32)
    kv = w.new_kv(64, batch=B)
    firsts = [w.prefill(kv, p, want_logits=False, seq=b)[0] for b, p in enumerate(prompts)]
    out, ms = w.generate_greedy_batch(kv, firsts, n, timed=True)
    assert ms > 0
    for b in (0, 7, 31):
        ref, margins = om.generate_greedy(prompts[b], n + 1)
        assert np.array_equal(out[:, b], ref[1:]), f"seq {b}: min margin {margins.min()}"


def test_f16_kv_roundtrip_and_errors(pkg, f16_engine, f16_model):
    w = f16_engine
    kv = w.new_kv(32, batch=2)
    rng = np.random.default_rng(1)
    K = rng.standard_normal((10, 256)).astype(np.float32)
    V = rng.standard_normal((10, 256)).astype(np.float32)
    for layer in range(w.num_layers):
        kv.import_layer(layer, K, V, seq=1)
    assert kv.length(1) == 10 and kv.length(0) == 0
    k2, v2 = kv.export_layer(2, 10, 256, seq=1)
    assert np.array_equal(k2, K) and np.array_equal(v2, V)
    with pytest.raises(pkg.QoraError):
        w.decode_batch(kv, [w.vocab, 0])  # token out of range
    with pytest.raises(pkg.QoraError):
        w.new_kv(32, batch=129)
    with pytest.raises(pkg.QoraError):
        w.prefill(kv, [1, 2, 3], seq=2)  # no such sequence
    kv.reset(1)
    assert kv.length(1) == 0


def test_f16_sample_from_batched_logits(f16_engine, orc):
    """qora_sample on each row of a batched step's logits (left on the device) equals the
    oracle's sampling step on the same logits read back."""
    w = f16_engine
    kv = w.new_kv(64, batch=3)
    prompts = _prompts(w.vocab, [4, 9, 6], 21)
    for b, p in enumerate(prompts):
        w.prefill(kv, p, want_logits=False, seq=b)
    am, lg = w.decode_batch(kv, [3, 4, 5], want_logits=True)
    state = 0x9E3779B97F4A7C15
    for b in range(3):
        hist = np.concatenate([prompts[b], [am[b]]]).astype(np.uint32)
        got = w.sample(hist, 0.6, 0.95, 20, 1.1, 1.5, -1, state, row=b)
        want = orc.sample(lg[b], hist, 0.6, 0.95, 20, 1.1, 1.5, -1, state)
        assert got == want, (b, got, want)
        state = got[1]
    # greedy through the same entry returns the step's argmax
    assert w.sample([], 0.0, 1.0, 1, row=1)[0] == am[1]
