"""Host checks of split-K geometry compiled from the shipped headers: the persistent
step's tile-aligned down_proj split (below) and the config-1 GEMV's box split
(tests/cpp/gemv_split_check.cu). The first: the shipped header (tests/cpp/split_check.cu includes qora-llm_b200/csrc/megakernel.cuh and
runs al_first / al_tile / al_span on the host; no GPU call): every row owned once, no CTA
across a tile boundary, consecutive slots per tile, per-CTA rows within the shared input
buffer, for SmolLM3-3B's shapes, its tensor-parallel splits and edge shapes."""
import os
import shutil
import subprocess

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def test_tile_aligned_split(tmp_path):
    nvcc = shutil.which("nvcc") or "/usr/local/cuda/bin/nvcc"
    if not os.path.exists(nvcc):
        pytest.skip("no nvcc")
    exe = tmp_path / "split_check"
    subprocess.run([nvcc, "-gencode", "arch=compute_100a,code=sm_100a", "-std=c++17", "--expt-relaxed-constexpr",
                    "-o", str(exe), os.path.join(ROOT, "tests", "cpp", "split_check.cu")], check=True)
    out = subprocess.run([str(exe)], capture_output=True, text=True, timeout=120)
    assert out.returncode == 0 and out.stdout.strip() == "ok", out.stdout + out.stderr


def test_gemv_box_split(tmp_path):
    nvcc = shutil.which("nvcc") or "/usr/local/cuda/bin/nvcc"
    if not os.path.exists(nvcc):
        pytest.skip("no nvcc")
    exe = tmp_path / "gemv_split_check"
    subprocess.run([nvcc, "-gencode", "arch=compute_100a,code=sm_100a", "-std=c++17", "--expt-relaxed-constexpr",
                    "-o", str(exe), os.path.join(ROOT, "tests", "cpp", "gemv_split_check.cu")], check=True)
    out = subprocess.run([str(exe)], capture_output=True, text=True, timeout=120)
    assert out.returncode == 0 and out.stdout.strip() == "ok", out.stdout + out.stderr
