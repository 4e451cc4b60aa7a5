"""qora_q4_gemv_static — the Q4 GEMV whose split-K scratch is the library's fixed
file-scope device array (no allocation) — against the CPU oracle's gemv_q4 (the
restatement of the reference's src/gemv.rs:646-675) on benchmark config 1's gate_proj,
and against qora_q4_gemv, through the C ABI.

The file name sorts last so that the test also runs after every other test of the
session has used the library; it passes alone in a fresh process as well. Two calls in
a row (and a shape change in between) check that each call leaves the shared arrival
counters at zero for the next one. Tolerance: within rel-L2 1e-5 of qora_q4_gemv (both
use the same plan and reduction order, so the results are in fact expected equal)."""
import numpy as np
import pytest

pytestmark = pytest.mark.gpu

TOL = 1e-5


def rel_l2(a, b):
    a, b = np.asarray(a, np.float64), np.asarray(b, np.float64)
    return float(np.linalg.norm(a - b) / max(np.linalg.norm(b), 1e-300))


@pytest.fixture(scope="module")
def torch():
    import torch as t
    assert t.cuda.is_available()
    return t


def _dev(torch, a):
    return torch.from_numpy(np.ascontiguousarray(a)).cuda()


def _case(qf, torch, seed, k, n):
    rng = np.random.default_rng(seed)
    m = qf.synth_q4_matrix(rng, k, n)
    x = rng.standard_normal(k).astype(np.float32)
    return [_dev(torch, v) for v in (x, m.packed, m.scales.view(np.int16))]


def _call(pkg, torch, fn, bufs, k, n):
    dx, dp, ds = bufs
    y = torch.full((n,), float("nan"), dtype=torch.float32, device="cuda")
    st = fn(dx.data_ptr(), dp.data_ptr(), ds.data_ptr(), k, n, y.data_ptr(), None)
    torch.cuda.synchronize()
    if st != 0:
        raise pkg.QoraError(st, pkg.engine.lib().qora_last_error().decode())
    return y.cpu().numpy()


def test_static_scratch_gemv_matches_allocating_gemv(pkg, qf, torch):
    lib = pkg.engine.lib()
    shapes = [(2048, 2048), (2048, 2048), (11008, 2048), (2048, 11008), (2048, 2048)]
    cases = {}
    for i, (k, n) in enumerate(shapes):
        if (k, n) not in cases:
            cases[(k, n)] = _case(qf, torch, 100 + i, k, n)
        bufs = cases[(k, n)]
        ref = _call(pkg, torch, lib.qora_q4_gemv, bufs, k, n)
        y1 = _call(pkg, torch, lib.qora_q4_gemv_static, bufs, k, n)
        y2 = _call(pkg, torch, lib.qora_q4_gemv_static, bufs, k, n)
        for y in (y1, y2):
            assert np.isfinite(y).all()
            assert rel_l2(y, ref) < TOL, (k, n, rel_l2(y, ref))
        assert np.array_equal(y1, y2)


def test_static_scratch_gemv_matches_oracle_config1(pkg, qf, orc, torch):
    """Config 1 (gate_proj, k=2048 in, n=11008 out, F1 layout, seed 0, x ~ N(0,1)):
    two calls in a row, each within rel-L2 1e-5 of the oracle and identical to the other."""
    lib = pkg.engine.lib()
    k, n = 2048, 11008
    rng = np.random.default_rng(0)
    m = qf.synth_q4_matrix(rng, k, n)
    x = rng.standard_normal(k).astype(np.float32)
    ref = orc.gemv_q4(x, m)
    bufs = [_dev(torch, v) for v in (x, m.packed, m.scales.view(np.int16))]
    y1 = _call(pkg, torch, lib.qora_q4_gemv_static, bufs, k, n)
    y2 = _call(pkg, torch, lib.qora_q4_gemv_static, bufs, k, n)
    for y in (y1, y2):
        assert np.isfinite(y).all()
        assert rel_l2(y, ref) < TOL, rel_l2(y, ref)
    assert np.array_equal(y1, y2)


def test_static_scratch_rejects_oversized_plans(pkg, torch):
    lib = pkg.engine.lib()
    max_tiles = 1024  # QORA_GEMV_STATIC_TILES
    k, n = 1, 32 * 8 * (max_tiles + 1)
    dx = torch.zeros(k, dtype=torch.float32, device="cuda")
    dp = torch.zeros(k * n // 2, dtype=torch.uint8, device="cuda")
    ds = torch.zeros(k * n // 32, dtype=torch.int16, device="cuda")
    y = torch.zeros(n, dtype=torch.float32, device="cuda")
    st = lib.qora_q4_gemv_static(dx.data_ptr(), dp.data_ptr(), ds.data_ptr(), k, n, y.data_ptr(), None)
    assert pkg.engine.STATUS.get(st) == "UNSUPPORTED"
    assert "static scratch" in lib.qora_last_error().decode()
    # the rejected call launched nothing: a normal call right after still works
    bufs = _case(pkg.qora_format, torch, 7, 512, 256)
    ref = _call(pkg, torch, lib.qora_q4_gemv, bufs, 512, 256)
    assert rel_l2(_call(pkg, torch, lib.qora_q4_gemv_static, bufs, 512, 256), ref) < TOL
