"""Tensor-parallel decode on 2, 4 and 8 GPUs (one engine per GPU, each in its own
process) against the CPU oracle: the same greedy tokens on every rank, identical to the
oracle's, and logits within rel-L2 1e-3 of the oracle.

Workers are started with `spawn`; the parent only relays the ranks' peer handles and
collects results. Every device-side wait in the engine is bounded, so a rank that fails
ends the others' steps with an error instead of a hang; the parent also bounds its own
waits and terminates the workers it started."""
import multiprocessing as mp
import queue

import numpy as np
import pytest

pytestmark = pytest.mark.gpu

LOGIT_TOL = 1e-3
N_GEN = 24


def _small_model(qf):
    # heads 8/2 and MLP 1536 (48 groups) divide by 2, 4 and 8
    return qf.synth_model(seed=11, num_layers=4, vocab=2048, hidden=1024, intermediate=1536,
                          num_heads=8, num_kv_heads=2, head_dim=128, rope_rows=256)


def _worker(rank, tp, to_parent, from_parent):
    try:
        import importlib
        import os
        import sys
        root = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
        sys.path.insert(0, root)
        pkg = importlib.import_module("qora-llm_b200")
        model = _small_model(pkg.qora_format)
        w = pkg.DecodeWeights(model=model, device=rank, tp_size=tp, tp_rank=rank)
        to_parent.put(("handle", rank, w.tp_export()))
        handles = from_parent.get(timeout=120)
        w.tp_connect(handles)
        kv = w.new_kv(128)
        prompt = np.random.default_rng(5).integers(0, w.vocab, size=10).astype(np.uint32)
        first, logits = w.prefill(kv, prompt)
        toks = w.generate_greedy(kv, first, N_GEN)
        am, step_logits = w.decode_step(kv, int(toks[-1]), want_logits=True)
        to_parent.put(("done", rank, (first, logits, toks, am, step_logits)))
        w.close()
    except Exception as exc:  # reported to the parent, which fails the test
        to_parent.put(("error", rank, repr(exc)))


def _run_tp(tp):
    ctx = mp.get_context("spawn")
    to_parent = ctx.Queue()
    inboxes = [ctx.Queue() for _ in range(tp)]
    procs = [ctx.Process(target=_worker, args=(r, tp, to_parent, inboxes[r]), daemon=True) for r in range(tp)]
    for p in procs:
        p.start()
    try:
        handles, results = {}, {}
        while len(results) < tp:
            kind, rank, payload = to_parent.get(timeout=600)
            if kind == "error":
                raise AssertionError(f"rank {rank}: {payload}")
            if kind == "handle":
                handles[rank] = payload
                if len(handles) == tp:
                    for q in inboxes:
                        q.put([handles[r] for r in range(tp)])
            else:
                results[rank] = payload
        return results
    except queue.Empty:
        raise AssertionError("tensor-parallel workers did not finish in time")
    finally:
        for p in procs:
            p.join(timeout=30)
            if p.is_alive():
                p.terminate()


def rel_l2(a, b):
    a, b = np.asarray(a, np.float64), np.asarray(b, np.float64)
    return float(np.linalg.norm(a - b) / max(np.linalg.norm(b), 1e-300))


@pytest.mark.parametrize("tp", [2, 4, 8])
def test_tensor_parallel_matches_oracle(tp, qf, orc):
    import torch
    if torch.cuda.device_count() < tp:
        pytest.skip(f"needs {tp} GPUs")
    results = _run_tp(tp)
    model = _small_model(qf)
    orc.set_threads(8)
    om = orc.OracleModel(model)
    prompt = np.random.default_rng(5).integers(0, model.vocab, size=10).astype(np.uint32)
    okv = om.new_kv()
    lo = om.prefill(prompt, okv)
    ref, margins = om.generate_greedy(prompt, N_GEN + 1)
    for rank in range(tp):
        first, logits, toks, am, step_logits = results[rank]
        assert first == int(np.argmax(lo)) == ref[0]
        assert rel_l2(logits, lo) < LOGIT_TOL, (rank, rel_l2(logits, lo))
        assert np.array_equal(toks, ref[1:]), f"rank {rank}: min oracle margin {margins.min()}"
        assert np.array_equal(step_logits, results[0][4])  # every rank holds the same logits
    print(f"tp={tp}: prefill logits rel-L2 {rel_l2(results[0][1], lo):.3e}")


# ---------------------------------------------------------------- F16 (config 5) under TP
def _small_f16(qf):
    # heads 8/2, MLP 1536 (768/384/192 channels per rank), vocab 2048 (16 tiles of 128)
    return qf.synth_model(seed=23, fmt=qf.FORMAT_F16, num_layers=3, vocab=2048, hidden=1024,
                          intermediate=1536, num_heads=8, num_kv_heads=2, head_dim=128, rope_rows=256)


F16_LENS = [5, 12, 3, 9]
F16_GEN = 12


def _worker_f16(rank, tp, to_parent, from_parent):
    try:
        import importlib
        import os
        import sys
        root = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
        sys.path.insert(0, root)
        pkg = importlib.import_module("qora-llm_b200")
        model = _small_f16(pkg.qora_format)
        w = pkg.DecodeWeights(model=model, device=rank, tp_size=tp, tp_rank=rank)
        to_parent.put(("handle", rank, w.tp_export()))
        w.tp_connect(from_parent.get(timeout=120))
        rng = np.random.default_rng(6)
        prompts = [rng.integers(0, w.vocab, size=n).astype(np.uint32) for n in F16_LENS]
        kv = w.new_kv(64, batch=len(F16_LENS))
        firsts, logits0 = [], None
        for b, p in enumerate(prompts):
            f, lg = w.prefill(kv, p, want_logits=(b == 0), seq=b)
            firsts.append(f)
            if b == 0:
                logits0 = lg
        toks = w.generate_greedy_batch(kv, firsts, F16_GEN)
        am, step_logits = w.decode_batch(kv, toks[-1], want_logits=True)
        to_parent.put(("done", rank, (firsts, logits0, toks, am, step_logits)))
        w.close()
    except Exception as exc:  # reported to the parent, which fails the test
        to_parent.put(("error", rank, repr(exc)))


def _run_tp_f16(tp):
    ctx = mp.get_context("spawn")
    to_parent = ctx.Queue()
    inboxes = [ctx.Queue() for _ in range(tp)]
    procs = [ctx.Process(target=_worker_f16, args=(r, tp, to_parent, inboxes[r]), daemon=True) for r in range(tp)]
    for p in procs:
        p.start()
    try:
        handles, results = {}, {}
        while len(results) < tp:
            kind, rank, payload = to_parent.get(timeout=600)
            if kind == "error":
                raise AssertionError(f"rank {rank}: {payload}")
            if kind == "handle":
                handles[rank] = payload
                if len(handles) == tp:
                    for q in inboxes:
                        q.put([handles[r] for r in range(tp)])
            else:
                results[rank] = payload
        return results
    except queue.Empty:
        raise AssertionError("tensor-parallel workers did not finish in time")
    finally:
        for p in procs:
            p.join(timeout=30)
            if p.is_alive():
                p.terminate()


@pytest.mark.parametrize("tp", [2, 4, 8])
def test_tensor_parallel_f16_batched_matches_oracle(tp, qf, orc):
    """F16 engines split over tp GPUs (tcgen05 GEMMs with the o_proj / down partials and
    the lm_head candidates exchanged over NVLink): 4 sequences prefilled then decoded
    together; every rank returns the oracle's greedy tokens and the same logits."""
    import torch
    if torch.cuda.device_count() < tp:
        pytest.skip(f"needs {tp} GPUs")
    results = _run_tp_f16(tp)
    model = _small_f16(qf)
    orc.set_threads(8)
    om = orc.OracleModel(model)
    rng = np.random.default_rng(6)
    prompts = [rng.integers(0, model.vocab, size=n).astype(np.uint32) for n in F16_LENS]
    refs = [om.generate_greedy(p, F16_GEN + 1) for p in prompts]
    lo = om.prefill(prompts[0], om.new_kv())
    for rank in range(tp):
        firsts, logits0, toks, am, step_logits = results[rank]
        assert rel_l2(logits0, lo) < LOGIT_TOL, (rank, rel_l2(logits0, lo))
        for b in range(len(F16_LENS)):
            ref, margins = refs[b]
            assert firsts[b] == ref[0]
            assert np.array_equal(toks[:, b], ref[1:]), f"rank {rank} seq {b}: min margin {margins.min()}"
        assert np.array_equal(step_logits, results[0][4])
        assert np.array_equal(am, results[0][3])
    print(f"F16 tp={tp}: prefill logits rel-L2 {rel_l2(results[0][1], lo):.3e}")
