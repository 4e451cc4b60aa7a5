"""The C-ABI boundary without a GPU: libqora_cuda.so loads, exports every function that
include/qora_cuda.h declares, the Python mirror binds them all, and the product path
fails loudly (no silent CPU fallback) when no GPU is present."""
import ctypes
import os
import re
import subprocess

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
HEADER = os.path.join(ROOT, "include", "qora_cuda.h")


def declared_functions():
    with open(HEADER) as f:
        src = f.read()
    src = re.sub(r"/\*.*?\*/", "", src, flags=re.S)
    return sorted(set(re.findall(r"\b(qora_[a-z0-9_]+)\s*\(", src)))


@pytest.fixture(scope="module")
def cudalib(pkg):
    import importlib
    build = importlib.import_module("qora-llm_b200.build")
    build.build()
    return ctypes.CDLL(build.LIB)


def test_header_declares_the_boundary():
    names = declared_functions()
    for required in ("qora_engine_create", "qora_engine_create_from_file", "qora_kv_create",
                     "qora_kv_import", "qora_prefill", "qora_decode_step", "qora_kv_destroy",
                     "qora_engine_destroy", "qora_last_error", "qora_q4_gemv"):
        assert required in names


def test_library_exports_every_declared_symbol(cudalib):
    missing = [n for n in declared_functions() if not hasattr(cudalib, n)]
    assert not missing, missing


def test_exports_are_c_linkage(pkg):
    import importlib
    lib = importlib.import_module("qora-llm_b200.build").LIB
    out = subprocess.run(["nm", "-D", "--defined-only", lib], capture_output=True, text=True).stdout
    exported = set(re.findall(r" T (qora_\w+)$", out, flags=re.M))
    assert set(declared_functions()) <= exported


def test_python_mirror_binds_every_symbol(pkg):
    assert set(pkg.engine.SIGNATURES) == set(declared_functions())
    lib = pkg.engine.lib()
    assert lib.qora_version().decode().startswith("qora-b200")
    assert lib.qora_last_error() is not None


def test_no_silent_cpu_fallback_without_gpu(pkg, qf):
    try:
        import torch
        if torch.cuda.is_available():
            pytest.skip("a GPU is present")
    except Exception:
        pass
    m = qf.synth_model(seed=0, num_layers=1, vocab=64, hidden=1024, intermediate=512,
                       num_heads=8, num_kv_heads=2, head_dim=128, rope_rows=8)
    with pytest.raises(pkg.QoraError) as ei:
        pkg.DecodeWeights(model=m)
    assert ei.value.status == 3  # QORA_ERR_CUDA: no device, and no CPU fallback


def test_invalid_view_rejected_before_device_use(pkg, qf):
    m = qf.synth_model(seed=0, num_layers=1, vocab=64, hidden=1024, intermediate=512,
                       num_heads=8, num_kv_heads=2, head_dim=128, rope_rows=8)
    m.layers[0].q_proj.n = 1000  # wrong shape
    with pytest.raises(pkg.QoraError, match="INVALID"):
        pkg.DecodeWeights(model=m)
    # F16: the batched GEMM tiles the vocab by 64
    m2 = qf.synth_model(seed=0, num_layers=1, vocab=100, hidden=1024, intermediate=512,
                        num_heads=8, num_kv_heads=2, head_dim=128, rope_rows=8,
                        fmt=qf.FORMAT_F16)
    with pytest.raises(pkg.QoraError, match="UNSUPPORTED"):
        pkg.DecodeWeights(model=m2)
    # tensor-parallel degrees other than 1, 2, 4 and 8 are rejected for either format
    m3 = qf.synth_model(seed=0, num_layers=1, vocab=128, hidden=1024, intermediate=512,
                        num_heads=8, num_kv_heads=2, head_dim=128, rope_rows=8,
                        fmt=qf.FORMAT_F16)
    with pytest.raises(pkg.QoraError, match="tp_size 3"):
        pkg.DecodeWeights(model=m3, tp_size=3, tp_rank=0)
