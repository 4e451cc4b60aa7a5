"""Kernel-level parity on the GPU through the C ABI (device pointers from torch tensors)
against the CPU oracle. Tolerances: dequantisation is bit-exact (integer x f16 scale is
exact in f32); GEMV / gate-up / lm_head outputs within rel-L2 1e-5 of the oracle (the
north-star bar for logits is 1e-3; the kernels are held 100x tighter); greedy argmax
identical."""
import numpy as np
import pytest

pytestmark = pytest.mark.gpu

GEMV_TOL = 1e-5


def rel_l2(a, b):
    a, b = np.asarray(a, np.float64), np.asarray(b, np.float64)
    return float(np.linalg.norm(a - b) / max(np.linalg.norm(b), 1e-300))


@pytest.fixture(scope="module")
def torch():
    import torch as t
    assert t.cuda.is_available()
    return t


def dev(torch, a):
    return torch.from_numpy(np.ascontiguousarray(a)).cuda()


def run_gemv(pkg, torch, m, x):
    dp, ds, dx = dev(torch, m.packed), dev(torch, m.scales.view(np.int16)), dev(torch, x)
    y = torch.empty(m.n, dtype=torch.float32, device="cuda")
    pkg.engine.q4_gemv(dx.data_ptr(), dp.data_ptr(), ds.data_ptr(), m.k, m.n, y.data_ptr())
    torch.cuda.synchronize()
    return y.cpu().numpy()


def test_dequant_bit_exact(pkg, qf, orc, torch):
    rng = np.random.default_rng(1)
    m = qf.synth_q4_matrix(rng, 64, 11008)
    m.packed[:16] = np.arange(16, dtype=np.uint8) * 17  # every nibble value incl. 0 and 8
    dp, ds = dev(torch, m.packed), dev(torch, m.scales.view(np.int16))
    out = torch.empty((40, m.n), dtype=torch.float32, device="cuda")
    pkg.engine.q4_dequant(dp.data_ptr(), ds.data_ptr(), m.n, 7, 40, out.data_ptr())
    torch.cuda.synchronize()
    assert np.array_equal(out.cpu().numpy(), orc.dequant_q4_rows(m, 7, 40))
    assert np.array_equal(out.cpu().numpy(), qf.dequant_q4(m)[7:47])


def config1(qf):
    """benchmark config 1: gate_proj in the reference layout (k=2048 in, n=11008 out),
    seed 0, x ~ N(0,1)."""
    rng = np.random.default_rng(0)
    m = qf.synth_q4_matrix(rng, 2048, 11008)
    x = rng.standard_normal(2048).astype(np.float32)
    return m, x


def test_gemv_config1(pkg, qf, orc, torch):
    m, x = config1(qf)
    y = run_gemv(pkg, torch, m, x)
    orc.set_threads(8)
    ref = orc.gemv_q4(x, m)
    r64 = x.astype(np.float64) @ qf.dequant_q4(m, np.float64)
    assert rel_l2(y, ref) < GEMV_TOL, rel_l2(y, ref)
    assert rel_l2(y, r64) < GEMV_TOL
    # deterministic: fixed reduction order, no float atomics
    assert np.array_equal(y, run_gemv(pkg, torch, m, x))


@pytest.mark.parametrize("k,n", [(1, 32), (3, 64), (7, 96), (100, 288), (2048, 512),
                                 (2048, 3072), (11008, 2048), (513, 11008), (4096, 256),
                                 (64, 65536)])  # last: more tiles than CTAs, one box each
def test_gemv_shapes(pkg, qf, orc, torch, k, n):
    rng = np.random.default_rng(k + 31 * n)
    m = qf.synth_q4_matrix(rng, k, n)
    x = rng.standard_normal(k).astype(np.float32)
    x[::5] = 0.0  # the reference skips zero inputs; the result must not care
    y = run_gemv(pkg, torch, m, x)
    ref = x.astype(np.float64) @ qf.dequant_q4(m, np.float64)
    assert rel_l2(y, ref) < GEMV_TOL, rel_l2(y, ref)


def test_gemv_alternating_shapes_reuse_scratch(pkg, qf, torch):
    """The TMA GEMV's split-K partials travel as tagged words in one scratch that every
    call reuses, and each tile's finisher zeroes them: calls alternating between shapes
    with different tile and slot counts (config 1's gate_proj, a down_proj shape, a
    narrower one) must each return their own result, bit-identical when repeated."""
    rng = np.random.default_rng(29)
    shapes = [(2048, 11008), (11008, 2048), (2048, 4096)]
    cases = []
    for k, n in shapes:
        m = qf.synth_q4_matrix(rng, k, n)
        x = rng.standard_normal(k).astype(np.float32)
        cases.append((m, x, x.astype(np.float64) @ qf.dequant_q4(m, np.float64)))
    first = {}
    for rnd in range(3):
        for i in (0, 1, 2, 1, 0, 2):
            m, x, ref = cases[i]
            y = run_gemv(pkg, torch, m, x)
            assert rel_l2(y, ref) < GEMV_TOL, (rnd, i, rel_l2(y, ref))
            if i in first:
                assert np.array_equal(y, first[i]), (rnd, i)
            else:
                first[i] = y


def test_gemv_extreme_scales(pkg, qf, torch):
    """Large and tiny f16 scales and inputs keep the subnormal-nibble arithmetic exact
    enough (no overflow of the 2^64 pre-scale, no flush of small products)."""
    rng = np.random.default_rng(17)
    m = qf.synth_q4_matrix(rng, 256, 512)
    s = np.array([65504.0, 6.1e-5, 1.0, 0.0, 3.0e-8, 100.0], np.float16)
    m.scales = np.resize(s, m.scales.size).view(np.uint16)
    x = rng.standard_normal(256).astype(np.float32) * np.float32(1e3)
    y = run_gemv(pkg, torch, m, x)
    ref = x.astype(np.float64) @ qf.dequant_q4(m, np.float64)
    assert rel_l2(y, ref) < GEMV_TOL


def test_gate_up(pkg, qf, orc, torch):
    rng = np.random.default_rng(2)
    g = qf.synth_q4_matrix(rng, 2048, 11008)
    u = qf.synth_q4_matrix(rng, 2048, 11008)
    x = rng.standard_normal(2048).astype(np.float32)
    out = torch.empty(11008, dtype=torch.float32, device="cuda")
    a = [dev(torch, v) for v in (x, g.packed, g.scales.view(np.int16), u.packed, u.scales.view(np.int16))]
    pkg.engine.q4_gate_up(*[t.data_ptr() for t in a], 2048, 11008, out.data_ptr())
    torch.cuda.synchronize()
    orc.set_threads(8)
    ref = orc.fused_gate_up_q4(x, g, u)
    assert rel_l2(out.cpu().numpy(), ref) < GEMV_TOL


@pytest.mark.parametrize("vocab,hidden", [(128256, 2048), (1000, 1024), (77, 2048)])
def test_lm_head(pkg, qf, orc, torch, vocab, hidden):
    rng = np.random.default_rng(vocab)
    e = qf.synth_embed(rng, qf.FORMAT_Q4, vocab, hidden)
    x = rng.standard_normal(hidden).astype(np.float32)
    dp, ds, dx = dev(torch, e.packed), dev(torch, e.scales.view(np.int16)), dev(torch, x)
    lg = torch.empty(vocab, dtype=torch.float32, device="cuda")
    am = torch.zeros(1, dtype=torch.int32, device="cuda")
    pkg.engine.q4_lm_head(dx.data_ptr(), dp.data_ptr(), ds.data_ptr(), vocab, hidden,
                          lg.data_ptr(), am.data_ptr())
    torch.cuda.synchronize()
    orc.set_threads(8)
    ref = orc.lm_head_q4(x, e)
    assert rel_l2(lg.cpu().numpy(), ref) < GEMV_TOL
    top2 = np.sort(ref)[-2:]
    assert int(am.item()) == orc.argmax(ref), f"margin {top2[1] - top2[0]}"


def test_lm_head_argmax_tie_takes_lowest_index(pkg, qf, torch):
    rng = np.random.default_rng(5)
    vocab, hidden = 5000, 1024
    e = qf.synth_embed(rng, qf.FORMAT_Q4, vocab, hidden)
    x = rng.standard_normal(hidden).astype(np.float32)
    ref = qf.dequant_q4(e, np.float64) @ x.astype(np.float64)
    best = int(np.argmax(ref))
    P = e.packed.reshape(vocab, -1)
    S = e.scales.reshape(vocab, -1)
    for dup in (4321, 17):  # copies of the winning row above and below it
        P[dup] = P[best]
        S[dup] = S[best]
    dp, ds, dx = dev(torch, e.packed), dev(torch, e.scales.view(np.int16)), dev(torch, x)
    am = torch.zeros(1, dtype=torch.int32, device="cuda")
    pkg.engine.q4_lm_head(dx.data_ptr(), dp.data_ptr(), ds.data_ptr(), vocab, hidden, 0,
                          am.data_ptr())
    torch.cuda.synchronize()
    assert int(am.item()) == min(17, best)


# ---------------------------------------------------------------- F16 GEMM (tcgen05)
def run_f16_gemm(pkg, torch, x, m):
    dx, dw = dev(torch, x), dev(torch, m.data.view(np.int16))
    y = torch.empty((x.shape[0], m.n), dtype=torch.float32, device="cuda")
    pkg.engine.f16_gemm(dx.data_ptr(), dw.data_ptr(), x.shape[0], m.k, m.n, y.data_ptr())
    torch.cuda.synchronize()
    return y.cpu().numpy()


def test_f16_gemm_matches_oracle(pkg, qf, orc, torch):
    """Small case against the oracle's gemm_f16 (the reference's scalar F16 GEMM)."""
    rng = np.random.default_rng(3)
    m = qf.synth_f16_matrix(rng, 256, 384)
    x = rng.standard_normal((5, 256)).astype(np.float32)
    y = run_f16_gemm(pkg, torch, x, m)
    ref = orc.gemm_f16(x, m)
    assert rel_l2(y, ref) < GEMV_TOL, rel_l2(y, ref)


@pytest.mark.parametrize("rows,k,n", [(1, 2048, 3072), (8, 2048, 2048), (32, 11008, 2048),
                                      (128, 2048, 1536), (200, 512, 256), (3, 64, 128),
                                      (16, 2048, 22016)])
def test_f16_gemm_shapes(pkg, qf, torch, rows, k, n):
    """SmolLM3 projection shapes at batch 1/8/32, a full prefill chunk, two row blocks,
    the smallest tile, and gate|up: against an f64 product of the same f16 weights."""
    rng = np.random.default_rng(rows * 7 + k)
    m = qf.synth_f16_matrix(rng, k, n)
    x = rng.standard_normal((rows, k)).astype(np.float32)
    x[0, :7] *= 1e-3  # small and large magnitudes within one row
    if rows > 1:
        x[1] *= 300.0  # a row far above f16's comfortable range before its row scale
    y = run_f16_gemm(pkg, torch, x, m)
    w = qf.f16_bits_to_f32(m.data).reshape(k, n).astype(np.float64)
    ref = x.astype(np.float64) @ w
    assert rel_l2(y, ref) < GEMV_TOL, rel_l2(y, ref)
    # per element: error within a small multiple of f32 rounding of |x|.|w|
    bound = np.abs(x.astype(np.float64)) @ np.abs(w)
    assert np.all(np.abs(y - ref) <= 1e-5 * bound + 1e-30)


# ---------------------------------------------------------------- on-device sampling
@pytest.mark.parametrize("params", [(0.0, 0.95, 20, 1.0, 0.0, -1), (0.6, 0.95, 20, 1.1, 1.5, -1),
                                    (1.0, 1.0, 1, 1.0, 0.0, -1), (0.3, 0.5, 50, 1.3, 0.0, 7),
                                    (1.5, 0.99, 1000, 1.0, 0.7, 3), (0.6, 0.95, 20, 1.1, 1.5, 128012)])
def test_sample_logits_matches_oracle(pkg, orc, torch, params):
    """qora_sample_logits against the oracle's restatement of the reference sampling step
    (penalties, top-k/top-p, xorshift64 draw): same token, same generator state."""
    t, tp, k, rp, pp, ban = params
    rng = np.random.default_rng(int(k * 10 + t * 100))
    for V in (128256, 997):
        for it in range(6):
            logits = (rng.standard_normal(V) * rng.uniform(0.5, 6)).astype(np.float32)
            logits[int(rng.integers(0, V))] = logits.max()  # a tie for the first place
            hist = rng.integers(0, V, size=int(rng.integers(0, 300))).astype(np.uint32)
            if hist.size > 3:
                hist[-2] = hist[-1]
            b = ban if ban < V else -1
            state = int(rng.integers(1, 2**63))
            dl, dh = dev(torch, logits), dev(torch, hist.view(np.int32) if hist.size else np.zeros(1, np.int32))
            got = pkg.engine.sample_logits(dl.data_ptr(), V, dh.data_ptr(), hist.size, t, tp, k, rp, pp, b, state)
            want = orc.sample(logits, hist, t, tp, k, rp, pp, b, state)
            assert got == want, (V, it, got, want)
