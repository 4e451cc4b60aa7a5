"""The Q4 prompt pass on the tensor cores (raw_prefill, src/gemv.rs:1027-1190, with
gemm_q4 :680-706): every prompt row through one dequantising tcgen05 GEMM per projection,
against the oracle and against the same engine run token by token (QORA_FLAG_TOKEN_PREFILL).

Prompts of 2 to 300 tokens cover one row chunk, several chunks (128 rows each) and a
ragged last chunk; a prompt after earlier tokens covers the position offset. Tolerances:
logits within rel-L2 1e-3 of the oracle (the engine-wide bar), KV rows within rel-L2 1e-5
of the token-by-token engine's, greedy continuations identical to the oracle's."""
import numpy as np
import pytest

pytestmark = pytest.mark.gpu

LOGIT_TOL = 1e-3
KV_TOL = 1e-5


def rel_l2(a, b):
    a, b = np.asarray(a, np.float64), np.asarray(b, np.float64)
    return float(np.linalg.norm(a - b) / max(np.linalg.norm(b), 1e-300))


@pytest.fixture(scope="module")
def model(qf):
    return qf.synth_model(seed=11, num_layers=3, vocab=2048, hidden=1024, intermediate=1536,
                          num_heads=8, num_kv_heads=2, head_dim=128, rope_rows=512)


@pytest.fixture(scope="module")
def engines(pkg, model):
    tc = pkg.DecodeWeights(model=model)
    tok = pkg.DecodeWeights(model=model, token_prefill=True)
    assert tc.prefill_path() == "tensor cores" and tok.prefill_path() == "token steps"
    yield tc, tok
    tc.close()
    tok.close()


@pytest.fixture(scope="module")
def oracle(orc, model):
    orc.set_threads(8)
    return orc.OracleModel(model)


@pytest.mark.parametrize("n", [2, 5, 64, 128, 129, 300])
def test_prompt_pass_matches_oracle_and_token_path(engines, oracle, n):
    tc, tok = engines
    prompt = np.random.default_rng(100 + n).integers(0, tc.vocab, size=n).astype(np.uint32)
    ka, kb = tc.new_kv(400), tok.new_kv(400)
    fa, la = tc.prefill(ka, prompt)
    fb, lb = tok.prefill(kb, prompt)
    okv = oracle.new_kv()
    lo = oracle.prefill(prompt, okv)
    err, err_tok = rel_l2(la, lo), rel_l2(lb, lo)
    print(f"n={n}: prompt-pass logits rel-L2 {err:.3e} (token path {err_tok:.3e})")
    assert err < LOGIT_TOL
    assert fa == int(np.argmax(lo)) == fb
    assert len(ka) == len(kb) == n
    for layer in (0, 2):
        k1, v1 = ka.export_layer(layer, n, 256)
        k2, v2 = kb.export_layer(layer, n, 256)
        assert rel_l2(k1, k2) < KV_TOL and rel_l2(v1, v2) < KV_TOL


def test_long_prompt_then_greedy(engines, oracle):
    tc, _ = engines
    prompt = np.random.default_rng(5).integers(0, tc.vocab, size=300).astype(np.uint32)
    kv = tc.new_kv(400)
    first, _ = tc.prefill(kv, prompt, want_logits=False)
    toks = tc.generate_greedy(kv, first, 24)
    ref, margins = oracle.generate_greedy(prompt, 25)
    assert ref[0] == first
    assert np.array_equal(toks, ref[1:]), f"min oracle margin {margins.min()}"


def test_prompt_after_earlier_tokens(engines, oracle):
    """A prompt appended to a cache that already holds 3 positions: rows at positions
    3..42 (RoPE rows and causal prefix offset). The oracle's prompt pass starts at position
    0, as the reference's does, so the oracle decodes the tokens one by one instead."""
    tc, tok = engines
    rng = np.random.default_rng(9)
    head = rng.integers(0, tc.vocab, size=3).astype(np.uint32)
    tail = rng.integers(0, tc.vocab, size=40).astype(np.uint32)
    kv, kb, okv = tc.new_kv(128), tok.new_kv(128), oracle.new_kv()
    for t in head:
        tc.decode_step(kv, int(t))
        tok.decode_step(kb, int(t))
        oracle.forward_decode(int(t), okv)
    am, lg = tc.prefill(kv, tail)
    bm, lb = tok.prefill(kb, tail)
    for t in tail:
        lo = oracle.forward_decode(int(t), okv)
    assert rel_l2(lg, lo) < LOGIT_TOL and am == int(np.argmax(lo)) == bm
    assert rel_l2(lg, lb) < LOGIT_TOL
    assert len(kv) == 43


def test_prompt_pass_repeatable(engines):
    tc, _ = engines
    prompt = np.arange(70, dtype=np.uint32) * 13 % tc.vocab
    outs = []
    for _ in range(2):
        kv = tc.new_kv(96)
        outs.append(tc.prefill(kv, prompt)[1])
        kv.close()
    assert np.array_equal(outs[0], outs[1])
