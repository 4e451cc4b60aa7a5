"""The C++ host mirror (qora-llm_b200/host/qora_host.hpp): it compiles against the C ABI
header on any host (CPU test), and on a GPU its parity program — the reference's call
sequence (load_model, raw_prefill, forward_decode_raw, greedy, sampling, a rejected bad
token) against the C++ oracle — passes on a Q4 and an F16 model written to .qora files."""
import os
import shutil
import subprocess

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
SRC = os.path.join(ROOT, "tests", "cpp", "host_parity.cpp")
INC = ["-I", os.path.join(ROOT, "include"), "-I", os.path.join(ROOT, "qora-llm_b200", "host"),
       "-I", os.path.join(ROOT, "oracle")]


def _gxx():
    g = shutil.which("g++")
    if not g:
        pytest.skip("no g++")
    return g


def test_host_header_compiles():
    subprocess.run([_gxx(), "-std=c++17", "-fsyntax-only", "-Wall", "-Werror", *INC, SRC], check=True)


@pytest.mark.gpu
@pytest.mark.parametrize("fmt_name", ["q4", "f16"])
def test_host_parity_program(tmp_path, qf, orc, fmt_name):
    lib_dir = os.path.join(ROOT, "qora-llm_b200")
    exe = str(tmp_path / "host_parity")
    subprocess.run([_gxx(), "-std=c++17", "-O2", *INC, SRC, "-o", exe,
                    "-L", lib_dir, "-lqora_cuda", "-L", os.path.dirname(orc.LIB_PATH), "-lqora_oracle",
                    f"-Wl,-rpath,{lib_dir}", f"-Wl,-rpath,{os.path.dirname(orc.LIB_PATH)}"], check=True)
    fmt = qf.FORMAT_Q4 if fmt_name == "q4" else qf.FORMAT_F16
    model = qf.synth_model(seed=19, fmt=fmt, num_layers=3, vocab=2048, hidden=1024, intermediate=1536,
                           num_heads=8, num_kv_heads=2, head_dim=128, rope_rows=256)
    path = str(tmp_path / "model.qora")
    qf.write_qora(model, path)
    r = subprocess.run([exe, path, "12", "3", "141", "59", "26", "535", "897"], capture_output=True, text=True,
                       timeout=300)
    assert r.returncode == 0, r.stderr + r.stdout
    print(r.stdout.strip())
