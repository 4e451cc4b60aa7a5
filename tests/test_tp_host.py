"""Host logic of the N > 1 path on CPU: the shard plan every tensor-parallel rank uses
(qora_tp_plan, shared with the engines) and the decomposition it implies, run as
world_size-2 `gloo` process groups: each rank computes its shard of one decoder layer
and of lm_head in float64 NumPy, the row-split partials are summed with all_reduce (the
device does the same sum in rank order over NVLink), and the vocab-split argmax is the
all_reduce MAX of ordered 64-bit keys (value bits, then the inverted index: the first
maximum wins) — equal to the unsplit computation."""
import os
import socket

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as tmp

FMT_F16, FMT_Q4 = 0, 1


@pytest.mark.parametrize("fmt", [FMT_F16, FMT_Q4])
@pytest.mark.parametrize("tp", [1, 2, 4, 8])
def test_plan_partitions_the_model(pkg, fmt, tp):
    """Every query head, MLP channel and vocab row belongs to exactly one rank; each rank's
    query heads use KV heads it holds; SmolLM3-3B shapes."""
    nh, nkvh, inter, vocab = 16, 4, 11008, 128256
    plans = [pkg.engine.tp_plan(fmt, nh, nkvh, inter, vocab, tp, r) for r in range(tp)]
    heads, mlp, voc = [], [], []
    for p in plans:
        heads += list(range(p["q_head0"], p["q_head0"] + p["q_heads"]))
        mlp += list(range(p["mlp0"], p["mlp0"] + p["mlp_n"]))
        voc.append((p["vocab0"], p["vocab_n"]))
        for h in range(p["q_head0"], p["q_head0"] + p["q_heads"]):
            assert p["kv_head0"] <= h // (nh // nkvh) < p["kv_head0"] + p["kv_heads"]
        assert p["mlp_padded"] >= p["mlp_n"]
        if fmt == FMT_F16:
            assert p["mlp_padded"] % 64 == 0 and p["vocab0"] % 128 == 0 and p["vocab_n"] % 128 == 0
    assert heads == list(range(nh)) and mlp == list(range(inter))
    assert voc[0][0] == 0 and sum(n for _, n in voc) == vocab
    assert all(voc[i][0] + voc[i][1] == voc[i + 1][0] for i in range(tp - 1))


def test_plan_rejects_bad_groups(pkg):
    with pytest.raises(pkg.QoraError, match="INVALID"):
        pkg.engine.tp_plan(FMT_Q4, 16, 4, 11008, 128256, 3, 0)
    with pytest.raises(pkg.QoraError, match="INVALID"):
        pkg.engine.tp_plan(FMT_Q4, 16, 4, 11008, 128256, 2, 2)
    with pytest.raises(pkg.QoraError, match="UNSUPPORTED"):
        pkg.engine.tp_plan(FMT_Q4, 12, 4, 11008, 128256, 8, 0)  # heads do not divide


# ---------------------------------------------------------------- gloo, world_size 2
H, NH, NKV, HD, I, V, S = 256, 8, 2, 32, 384, 512, 7


def _weights():
    rng = np.random.default_rng(3)
    w = {k: rng.standard_normal(s) * 0.1 for k, s in
         dict(q=(H, NH * HD), k=(H, NKV * HD), v=(H, NKV * HD), o=(NH * HD, H), g=(H, I), u=(H, I),
              d=(I, H), emb=(V, H)).items()}
    w["x"] = rng.standard_normal(H)
    w["kc"] = rng.standard_normal((S, NKV * HD))  # cached rows incl. the new position
    w["vc"] = rng.standard_normal((S, NKV * HD))
    return w


def _attend(q, kc, vc, heads, kv_of):
    out = []
    for i, h in enumerate(heads):
        j = kv_of(h)
        s = kc[:, j * HD:(j + 1) * HD] @ q[i * HD:(i + 1) * HD] / np.sqrt(HD)
        p = np.exp(s - s.max())
        out.append((p / p.sum()) @ vc[:, j * HD:(j + 1) * HD])
    return np.concatenate(out)


def _layer_and_logits(w, plan=None, reduce=lambda a: a):
    """One layer (without norms: the split does not touch them) + lm_head, for the shard
    in `plan` (None: the whole model); `reduce` sums row-split partials over ranks."""
    grp = NH // NKV
    if plan is None:
        plan = dict(q_head0=0, q_heads=NH, kv_head0=0, kv_heads=NKV, mlp0=0, mlp_n=I, vocab0=0, vocab_n=V)
    h0, nh = plan["q_head0"], plan["q_heads"]
    kv0, nkv = plan["kv_head0"], plan["kv_heads"]
    x = w["x"]
    q = x @ w["q"][:, h0 * HD:(h0 + nh) * HD]
    kc = w["kc"][:, kv0 * HD:(kv0 + nkv) * HD]
    vc = w["vc"][:, kv0 * HD:(kv0 + nkv) * HD]
    a = _attend(q, kc, vc, range(h0, h0 + nh), lambda h: h // grp - kv0)
    x = x + reduce(a @ w["o"][h0 * HD:(h0 + nh) * HD])  # row split: one all-reduce
    m0, mn = plan["mlp0"], plan["mlp_n"]
    g, u = x @ w["g"][:, m0:m0 + mn], x @ w["u"][:, m0:m0 + mn]
    hh = g / (1 + np.exp(-g)) * u
    x = x + reduce(hh @ w["d"][m0:m0 + mn])  # row split: one all-reduce
    v0, vn = plan["vocab0"], plan["vocab_n"]
    logits = w["emb"][v0:v0 + vn] @ x
    return x, logits, v0


def _key(v, idx):
    b = np.float32(v).view(np.uint32).item()
    o = (~b & 0xFFFFFFFF) if b & 0x80000000 else (b | 0x80000000)
    return (o << 32) | (0xFFFFFFFF - idx)


def _rank_main(rank, world, port, fmt, results):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        import importlib
        import sys
        sys.path.insert(0, os.path.dirname(os.path.dirname(os.path.abspath(__file__))))
        pkg = importlib.import_module("qora-llm_b200")
        plan = pkg.engine.tp_plan(fmt, NH, NKV, I, V, world, rank)

        def allreduce(a):
            t = torch.from_numpy(np.ascontiguousarray(a))
            dist.all_reduce(t)
            return t.numpy()

        x, logits, v0 = _layer_and_logits(_weights(), plan, allreduce)
        # vocab-split greedy: this rank's first maximum as an ordered key, max over ranks
        i = int(np.argmax(logits))
        key = torch.tensor([_key(logits[i], v0 + i) - (1 << 63)], dtype=torch.int64)  # signed for gloo
        dist.all_reduce(key, op=dist.ReduceOp.MAX)
        am = 0xFFFFFFFF - ((int(key.item()) + (1 << 63)) & 0xFFFFFFFF)
        gathered = [None] * world
        dist.all_gather_object(gathered, (v0, logits.tolist()))
        results[rank] = (x.tolist(), am, gathered)
    finally:
        dist.destroy_process_group()


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


@pytest.mark.parametrize("fmt", [FMT_F16, FMT_Q4])
def test_gloo_two_ranks_reproduce_the_unsplit_layer(fmt):
    world = 2
    mgr = tmp.Manager()
    results = mgr.dict()
    tmp.spawn(_rank_main, args=(world, _free_port(), fmt, results), nprocs=world, join=True)
    w = _weights()
    x_ref, logits_ref, _ = _layer_and_logits(w)
    for r in range(world):
        x, am, gathered = results[r]
        assert np.allclose(x, x_ref, rtol=1e-12, atol=1e-12)
        full = np.zeros(V)
        for v0, lg in gathered:
            full[v0:v0 + len(lg)] = lg
        assert np.allclose(full, logits_ref, rtol=1e-12, atol=1e-12)
        assert am == int(np.argmax(logits_ref))
