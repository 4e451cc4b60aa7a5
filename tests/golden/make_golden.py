"""Regenerate tests/golden/golden_small.npz.

The reference (Rust, no cargo here) cannot produce vectors in this environment, so these
fixtures are outputs of the C++ oracle on a seeded synthetic model. They pin the oracle
and the synthetic generator against silent drift; the oracle itself is pinned by the
known-answer and float64 tests in tests/test_oracle.py.

    python tests/golden/make_golden.py
"""
import os
import sys

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(os.path.dirname(HERE))
sys.path.insert(0, ROOT)
sys.path.insert(0, os.path.join(ROOT, "oracle"))
import oracle  # noqa: E402

CFG = dict(seed=1234, num_layers=4, vocab=1024, hidden=1024, intermediate=1536, num_heads=8,
           num_kv_heads=2, head_dim=128, rope_rows=64)
THREADS = 4


def main():
    qf = oracle.qf
    model = qf.synth_model(**CFG)
    oracle.set_threads(THREADS)
    om = oracle.OracleModel(model)
    prompt = np.random.default_rng(99).integers(0, CFG["vocab"], size=8).astype(np.uint32)
    toks, margins = om.generate_greedy(prompt, 12)
    kv = om.new_kv()
    logits = om.prefill(prompt, kv)
    gx = np.random.default_rng(7).standard_normal(CFG["hidden"]).astype(np.float32)
    gy = oracle.gemv_q4(gx, model.layers[0].gate_proj)
    np.savez_compressed(os.path.join(HERE, "golden_small.npz"),
                        **{f"cfg_{k}": np.int64(v) for k, v in CFG.items()},
                        threads=np.int64(THREADS), prompt=prompt, tokens=toks, margins=margins,
                        prefill_logits=logits, gemv_x=gx, gemv_y=gy)
    print("tokens", toks.tolist(), "min margin", float(margins.min()))


if __name__ == "__main__":
    main()
