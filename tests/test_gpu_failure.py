"""Failure detection without a GPU fault: a tensor-parallel rank whose peer never takes
part. Rank 1 of a 2-way group is created in a child process (it exports its receive
region and then only waits to be told to exit; it launches no kernel), rank 0 runs in this
process on the same GPU and steps alone. Its persistent kernel waits for rank 1's partial
sums — words nothing will ever write — until the bounded wait (2 s) runs out, then
records QORA_ERR_TIMEOUT and returns; the host reads the status, and the context stays
usable (a plain engine on the same device decodes afterwards). A multi-launch prompt pass
against the same missing peer reports the timeout after about one wait, not one per
launch."""
import multiprocessing as mp
import queue
import time

import numpy as np
import pytest

pytestmark = pytest.mark.gpu

TIMEOUT = 6  # QORA_ERR_TIMEOUT
DEVICE_WAIT_S = 2.0  # the kernels' bound on one wait


def _model(qf):
    return qf.synth_model(seed=11, num_layers=2, vocab=2048, hidden=1024, intermediate=1536,
                          num_heads=8, num_kv_heads=2, head_dim=128, rope_rows=256)


def _idle_rank(to_parent, from_parent):
    try:
        import importlib
        import os
        import sys
        root = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
        sys.path.insert(0, root)
        pkg = importlib.import_module("qora-llm_b200")
        w = pkg.DecodeWeights(model=_model(pkg.qora_format), device=0, tp_size=2, tp_rank=1)
        to_parent.put(("handle", w.tp_export()))
        from_parent.get(timeout=300)  # exit when told; never steps
        w.close()
    except Exception as exc:
        to_parent.put(("error", repr(exc)))


def test_missing_tp_peer_times_out_and_context_survives(pkg, qf):
    ctx = mp.get_context("spawn")
    to_parent, to_child = ctx.Queue(), ctx.Queue()
    child = ctx.Process(target=_idle_rank, args=(to_parent, to_child), daemon=True)
    child.start()
    try:
        kind, payload = to_parent.get(timeout=300)
        assert kind == "handle", payload
        model = _model(qf)
        w0 = pkg.DecodeWeights(model=model, device=0, tp_size=2, tp_rank=0)
        w0.tp_connect([w0.tp_export(), payload])
        kv = w0.new_kv(64)
        with pytest.raises(pkg.QoraError) as ei:
            w0.decode_step(kv, 17)
        assert ei.value.status == TIMEOUT, str(ei.value)
        kv.close()
        # a prompt pass runs several launches: the first one times out, the ones after it
        # see the recorded error and stop at once, so the whole call fails within about
        # one timeout (not one per prompt token) and keeps the timeout code
        kvp = w0.new_kv(64)
        t0 = time.monotonic()
        with pytest.raises(pkg.QoraError) as ei:
            w0.prefill(kvp, np.arange(1, 13, dtype=np.uint32), want_logits=False)
        took = time.monotonic() - t0
        assert ei.value.status == TIMEOUT, str(ei.value)
        assert took < 3 * DEVICE_WAIT_S, f"prefill took {took:.1f} s to report the timeout"
        kvp.close()
        w0.close()
        # the device still works: a single-GPU engine decodes and matches itself
        w = pkg.DecodeWeights(model=model, device=0)
        kv1 = w.new_kv(32)
        a = w.decode_step(kv1, 17)
        kv2 = w.new_kv(32)
        assert w.decode_step(kv2, 17) == a
        w.close()
    except queue.Empty:
        raise AssertionError("the idle rank did not start in time")
    finally:
        to_child.put("exit")
        child.join(timeout=60)
        if child.is_alive():
            child.terminate()
