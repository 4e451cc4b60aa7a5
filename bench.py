#!/usr/bin/env python
"""Decode throughput of the B200 engine on benchmark config 3: SmolLM3-3B architecture,
seeded random-init Q4 weights (synthetic; no checkpoint), 32-token prompt, greedy decode
at batch 1. A "step" is one decode step (one token through all 36 layers + lm_head +
argmax).

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]
    python bench.py --workload f16-batch [--batch 32] [--steps 128]   # benchmark config 5
    python bench.py --workload q4-long [--steps 128] [--kv f16]         # benchmark config 4
    python bench.py --workload q4-gemv                                 # benchmark config 1 (GB/s)

Prints one JSON line (rank 0). `value` is device time (CUDA events on the engine's
stream) of K greedy steps, each one launch of the persistent decode kernel, with the
token fed back on the device;
`e2e` is the same metric through the public C ABI (qora_decode_step) with host token
in / host argmax out every step. `--impl reference` times the reference's CPU decode
path (the C++ restatement in oracle/, all host threads) on the same workload.
"""
from __future__ import annotations

import argparse
import json
import os
import statistics
import subprocess
import sys
import threading
import time

import numpy as np

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)

METRIC = "decode tok/s (batch 1, SmolLM3-3B Q4)"
PROMPT = 32
SEED = 0
HIDDEN, LAYERS, VOCAB = 2048, 36, 128256
# algorithmic bytes of one decode step excluding KV (weights + norms + lm_head embedding
# read in full + final norm + the embedding row), and KV bytes per cached position
def weight_bytes_per_token(layers=LAYERS):
    return layers * (43_941_888 + 8_192) + 147_750_912 + 4_096 + 1_152


def kv_bytes_per_pos(layers=LAYERS, esz=4):
    """K and V bytes of one cached position over all layers (esz 4: f32, 2: binary16)."""
    return layers * 2 * 4 * 128 * esz


def peaks():
    try:
        with open(os.path.join(ROOT, "MEASURED_PEAKS.json")) as f:
            p = json.load(f)
        return float(p["hbm_gbs"]), "measured"
    except Exception:
        return 6650.0, "fallback"


class ClockSampler:
    """nvidia-smi samples during the timed region (SM clock, throttle reasons)."""

    Q = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
         "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
         "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, index: int):
        self.index = index
        self.proc = None
        self.lines = []

    def __enter__(self):
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", "-i", str(self.index), f"--query-gpu={self.Q}",
                 "--format=csv,noheader,nounits", "-lms", "100"],
                stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
            self.thread = threading.Thread(target=self._read, daemon=True)
            self.thread.start()
        except Exception:
            self.proc = None
        return self

    def _read(self):
        for line in self.proc.stdout:
            self.lines.append(line.strip())

    def __exit__(self, *a):
        if self.proc:
            self.proc.terminate()
            try:
                self.proc.wait(timeout=5)
            except Exception:
                self.proc.kill()

    def summary(self):
        sm, mx, reasons = [], None, set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for ln in self.lines:
            f = [x.strip() for x in ln.split(",")]
            if len(f) < 9:
                continue
            try:
                sm.append(float(f[1]))
                mx = float(f[2])
            except ValueError:
                continue
            for n, v in zip(names, f[5:9]):
                if v.lower() == "active":
                    reasons.add(n)
        if not sm:
            return {"sm_mhz": None, "sm_max_mhz": mx, "reasons": sorted(reasons), "samples": 0}
        return {"sm_mhz": statistics.median(sm), "sm_max_mhz": mx, "reasons": sorted(reasons),
                "samples": len(sm)}


def synth(layers=36):
    import importlib
    qf = importlib.import_module("qora-llm_b200").qora_format
    model = qf.synth_model(seed=SEED, num_layers=layers)
    prompt = np.random.default_rng(1).integers(0, VOCAB, size=PROMPT).astype(np.uint32)
    return model, prompt


def cpu_baseline(model, prompt, budget_s=15.0):
    """Oracle (C++ restatement of the reference CPU path) on this host's cores: decode
    steps fed the prompt ids one by one from an empty cache, bounded to ~budget_s."""
    sys.path.insert(0, os.path.join(ROOT, "oracle"))
    import oracle
    threads = os.cpu_count() or 1
    oracle.set_threads(threads)
    om = oracle.OracleModel(model)
    kv = om.new_kv()
    om.forward_decode(int(prompt[0]), kv)  # warm-up (page-in, pool start)
    t0 = time.perf_counter()
    n = 0
    while n < len(prompt) - 1 and (n < 2 or time.perf_counter() - t0 < budget_s):
        om.forward_decode(int(prompt[1 + n]), kv)
        n += 1
    dt = time.perf_counter() - t0
    om.close()
    return {"value": n / dt, "unit": "tok/s", "cores": threads, "kind": "port",
            "sample": f"{n} forward_decode_raw steps of config 3 (kv_len 2..{n + 1}), "
                      f"{threads} threads, AVX-512={'yes' if oracle.lib().orc_get_avx512() else 'no'}",
            "cpu": cpu_model()}


def cpu_model():
    try:
        for ln in open("/proc/cpuinfo"):
            if ln.startswith("model name"):
                return ln.split(":", 1)[1].strip()
    except Exception:
        pass
    return None


def config3(args, kv_len_mean):
    """The workload dict both arms print for config 3."""
    return {"workload": "config 3: SmolLM3-3B Q4 (36 layers, vocab 128256), 32-token prompt, "
                        "greedy decode at batch 1",
            "prompt": PROMPT, "kv_len_mean": kv_len_mean, "layers": args.layers,
            "l2": "inputs larger than L2: 1.73 GB of weights streamed per step"}


def run_reference(args, rank):
    if rank != 0:
        return 0
    model, prompt = synth(args.layers)
    sys.path.insert(0, os.path.join(ROOT, "oracle"))
    import oracle
    threads = os.cpu_count() or 1
    oracle.set_threads(threads)
    om = oracle.OracleModel(model)
    kv = om.new_kv()
    logits = om.prefill(prompt, kv)
    tok = oracle.argmax(logits)
    for _ in range(args.warmup):
        tok = oracle.argmax(om.forward_decode(tok, kv))
    t0 = time.perf_counter()
    for _ in range(args.steps):
        tok = oracle.argmax(om.forward_decode(tok, kv))
    dt = time.perf_counter() - t0
    v = args.steps / dt
    line = {
        "impl": "reference", "metric": METRIC, "value": v, "unit": "tok/s", "n_gpus": args.gpus,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": 1000 * dt / args.steps,
        "higher_is_better": True, "scaling": "strong", "vs_baseline": None, "dtype": "f32",
        "data": "synthetic (seeded random-init SmolLM3-3B Q4)",
        "config": config3(args, PROMPT + args.warmup + (args.steps - 1) / 2.0 + 1),
        "cpu_baseline": {"value": v, "unit": "tok/s", "cores": threads, "kind": "port",
                         "sample": f"{args.steps} greedy decode steps after a {PROMPT}-token prefill "
                                   f"and {args.warmup} warm-up steps (oracle/ C++ restatement of "
                                   f"src/gemv.rs + src/simd.rs, {threads} threads)",
                         "cpu": cpu_model()},
        "e2e": {"value": v, "unit": "tok/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)
    return 0


def run_ours(args, rank, world, local_rank):
    import importlib
    import torch
    pkg = importlib.import_module("qora-llm_b200")
    torch.cuda.set_device(local_rank)
    dist = None
    if world > 1:
        import datetime
        import torch.distributed as dist
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=600))
    model, prompt = synth(args.layers)
    if world > 1:
        # tensor parallelism: one engine per GPU; exchange the ranks' peer handles
        eng = pkg.DecodeWeights(model=model, device=local_rank, tp_size=world, tp_rank=rank)
        handles = [None] * world
        dist.all_gather_object(handles, eng.tp_export())
        eng.tp_connect(handles)
    else:
        eng = pkg.DecodeWeights(model=model, device=local_rank)
    K, W = args.steps, args.warmup
    cap = PROMPT + W + K + 8

    # ---- device-timed greedy decode (value): the same K steps (32-token prompt, W warm-up
    # steps, then K timed greedy steps on a fresh cache) repeated until >= 1 s of timed
    # decode has passed, so that the clock sampler sees the timed region; each repetition
    # is the max over ranks, the line reports the median repetition. Every rank runs the
    # same number of repetitions (fixed from K before timing).
    reps_n = max(1, min(64, -(-1000 // max(1, int(K * 1.2)))))
    rep_ms = []
    with ClockSampler(local_rank) as clk:
        for _ in range(reps_n):
            kv = eng.new_kv(cap)
            first, _ = eng.prefill(kv, prompt, want_logits=False)
            toks = eng.generate_greedy(kv, first, W)
            nxt = int(toks[-1]) if W else first
            kv_start = len(kv)
            if dist:
                dist.barrier()
            torch.cuda.synchronize()
            _, ms = eng.generate_greedy_timed(kv, nxt, K)
            torch.cuda.synchronize()
            ms_t = torch.tensor([ms], dtype=torch.float64, device="cuda")
            if dist:
                dist.all_reduce(ms_t, op=dist.ReduceOp.MAX)
            rep_ms.append(float(ms_t.item()))
            kv.close()
    ms = statistics.median(rep_ms)
    value = K / (ms / 1000.0)  # tokens of the one sequence all ranks decode together

    # ---- end to end through the C ABI: host token in, host argmax out, every step
    kv2 = eng.new_kv(cap)
    first2, _ = eng.prefill(kv2, prompt, want_logits=False)
    t = first2
    for _ in range(W):
        t = eng.decode_step(kv2, t)
    if dist:
        dist.barrier()
    t0 = time.perf_counter()
    for _ in range(K):
        t = eng.decode_step(kv2, t)
    e2e_s = time.perf_counter() - t0
    e2e_t = torch.tensor([e2e_s], dtype=torch.float64, device="cuda")
    if dist:
        dist.all_reduce(e2e_t, op=dist.ReduceOp.MAX)
    e2e = K / float(e2e_t.item())

    # ---- the prompt pass of the workload's 32-token prompt (host ids in, first token out;
    # wall clock around the C-ABI call, fresh cache each time, median of 5)
    pre_ms = []
    for _ in range(5):
        kvp = eng.new_kv(cap)
        torch.cuda.synchronize()
        if dist:
            dist.barrier()
        t0 = time.perf_counter()
        eng.prefill(kvp, prompt, want_logits=False)
        pre_ms.append((time.perf_counter() - t0) * 1000.0)
        kvp.close()

    # ---- dominant kernel. With the persistent step the whole decode step is ONE kernel
    # launch; its algorithmic bytes are the weights + KV rows it must stream.
    peak, peak_kind = peaks()
    mega = eng.launches_per_step() == 1
    mean_kv = kv_start + (K - 1) / 2.0 + 1
    step_bytes = weight_bytes_per_token(args.layers) + kv_bytes_per_pos(args.layers) * (mean_kv + 1)
    rank_bytes = step_bytes / world  # weights, lm_head rows and (up to tp 4) KV heads split evenly
    traffic = None
    tpath = os.path.join(ROOT, "profiles", "decode_megakernel_dram.json")
    if os.path.exists(tpath):
        try:
            traffic = json.load(open(tpath))["dram_bytes_per_launch"]
        except Exception:
            traffic = None
    if world > 1:
        traffic = None  # the committed ncu capture is of the single-GPU kernel
    if mega:
        kern = {"kernel": "decode megakernel (whole step: 36 layers + lm_head + argmax)"
                          + (f", one launch per rank of a {world}-way tensor-parallel group" if world > 1 else ""),
                "bytes_per_launch": rank_bytes, "us_per_launch": 1000 * ms / K,
                "launches_timed": K}
        achieved = rank_bytes / (ms / K / 1000.0) / 1e9
    else:
        kv = eng.new_kv(cap)
        kern_ms, kern_bytes, kern_n = eng.time_kernel(kv, "gate_up", reps=5)
        kv.close()
        kern = {"kernel": "q4 gate/up GEMV (+RMSNorm, SwiGLU)", "bytes_per_launch": kern_bytes,
                "us_per_launch": kern_ms * 1000, "launches_timed": kern_n}
        achieved = kern_bytes / (kern_ms / 1000.0) / 1e9
    line = {
        "metric": METRIC, "value": value, "unit": "tok/s", "n_gpus": world, "steps": K,
        "warmup": W, "ms_per_step": ms / K, "higher_is_better": True,
        "scaling": "strong", "vs_baseline": None, "dtype": "f32",
        "data": "synthetic (seeded random-init SmolLM3-3B Q4 weights, random prompt ids)",
        # the workload only (the reference arm prints the same dict); run details below
        "config": config3(args, mean_kv),
        "parallelism": "single GPU" if world == 1 else f"tp{world} (tensor parallel, NVLink peer all-reduce)",
        "detail": {
            "repetitions": f"median of {reps_n} repetitions of the {K} timed steps (fresh cache each)",
            "repetition_ms": rep_ms,
            "bytes_per_step": step_bytes,
            "step_hbm_GBps": step_bytes * (K / (ms / 1000.0)) / 1e9,
            "step_hbm_frac": step_bytes * (K / (ms / 1000.0)) / 1e9 / peak,
            "prefill_ms": statistics.median(pre_ms),
            "prefill_in_step_times": statistics.median(pre_ms) / (ms / K),
            "prefill_path": eng.prefill_path(),
        },
        "e2e": {"value": e2e, "unit": "tok/s", "h2d_bytes_per_step": 32, "d2h_bytes_per_step": 32},
        "gpu_launches": eng.launches_per_step() * K,  # per rank
        "roofline": dict(bound="hbm", achieved=achieved, peak=peak,
                         peak_kind=f"{peak_kind} hbm_gbs (copy)", unit="GB/s",
                         frac=achieved / peak, traffic=traffic, **kern),
        "clocks": clk.summary(),
    }
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        line["cpu_baseline"] = cpu_baseline(model, prompt, args.cpu_seconds)
    kv2.close()
    eng.close()
    if dist:
        dist.barrier()
        dist.destroy_process_group()
    if rank == 0:
        print(json.dumps(line), flush=True)
    return 0


F16_METRIC = "decode tok/s (batched, SmolLM3-3B F16)"
F16_PROMPT = 128
def f16_bytes_per_step(layers=LAYERS):  # every f16 weight once (+ norms, negligible)
    return 2 * (layers * 78_118_912 + VOCAB * HIDDEN)


def synth_f16(layers=36):
    import importlib
    qf = importlib.import_module("qora-llm_b200").qora_format
    return qf.synth_model(seed=SEED + 5, fmt=qf.FORMAT_F16, num_layers=layers, rope_rows=1024)


def f16_prompts(batch):
    return np.random.default_rng(2).integers(0, VOCAB, size=(batch, F16_PROMPT)).astype(np.uint32)


def f16_cpu_sample(model, budget_s, threads):
    """The reference's F16 CPU decode (forward_decode_raw with gemv_f16, oracle/) on this
    host: steps of one sequence from an empty cache, bounded to ~budget_s. The CPU path has
    no batching; B sequences cost B times one."""
    sys.path.insert(0, os.path.join(ROOT, "oracle"))
    import oracle
    oracle.set_threads(threads)
    om = oracle.OracleModel(model)
    kv = om.new_kv()
    ids = f16_prompts(1)[0]
    om.forward_decode(int(ids[0]), kv)  # warm-up
    t0 = time.perf_counter()
    n = 0
    while n < len(ids) - 1 and (n < 2 or time.perf_counter() - t0 < budget_s):
        om.forward_decode(int(ids[1 + n]), kv)
        n += 1
    dt = time.perf_counter() - t0
    om.close()
    return n / dt, n


def run_f16(args, rank, world, local_rank):
    """benchmark config 5: B independent sequences, 128-token prompts, greedy batched
    decode on one GPU (tcgen05 GEMMs)."""
    B, K, W = args.batch, args.steps, args.warmup
    threads = os.cpu_count() or 1
    model = synth_f16(args.layers)
    if args.impl == "reference":
        if rank != 0:
            return 0
        v, n = f16_cpu_sample(model, args.cpu_seconds, threads)
        line = {"impl": "reference", "metric": F16_METRIC, "value": v, "unit": "tok/s", "n_gpus": 1, "steps": n,
                "warmup": 1, "ms_per_step": 1000.0 / v, "higher_is_better": True, "scaling": "strong",
                "vs_baseline": None, "dtype": "f32", "data": "synthetic (seeded random-init SmolLM3-3B F16)",
                "config": {"workload": f"config 5: SmolLM3-3B F16, batch {B}, 128-token prompts, greedy decode",
                           "batch": B},
                "cpu_baseline": {"value": v, "unit": "tok/s", "cores": threads, "kind": "port",
                                 "sample": f"{n} forward_decode_raw steps of one sequence (the CPU path decodes "
                                           f"sequences one at a time), {threads} threads", "cpu": cpu_model()},
                "e2e": {"value": v, "unit": "tok/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}
        print(json.dumps(line), flush=True)
        return 0
    import importlib
    import torch
    pkg = importlib.import_module("qora-llm_b200")
    torch.cuda.set_device(local_rank)
    dist = None
    if world > 1:
        import datetime
        import torch.distributed as dist
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=600))
        eng = pkg.DecodeWeights(model=model, device=local_rank, tp_size=world, tp_rank=rank)
        handles = [None] * world
        dist.all_gather_object(handles, eng.tp_export())
        eng.tp_connect(handles)
    else:
        eng = pkg.DecodeWeights(model=model, device=local_rank)
    prompts = f16_prompts(B)
    cap = F16_PROMPT + W + K + 8

    def prefilled():
        kv = eng.new_kv(cap, batch=B)
        firsts = [eng.prefill(kv, prompts[b], want_logits=False, seq=b)[0] for b in range(B)]
        return kv, firsts

    # ---- device-timed batched greedy decode (value)
    kv, firsts = prefilled()
    torch.cuda.synchronize()
    t0 = time.perf_counter()
    kv_p, _ = prefilled()
    torch.cuda.synchronize()
    prefill_s = time.perf_counter() - t0
    kv_p.close()
    warm = eng.generate_greedy_batch(kv, firsts, W)
    nxt = warm[-1]
    if dist:
        dist.barrier()
    torch.cuda.synchronize()
    with ClockSampler(local_rank) as clk:
        _, ms = eng.generate_greedy_batch(kv, nxt, K, timed=True)
    torch.cuda.synchronize()
    if dist:
        ms_t = torch.tensor([ms], dtype=torch.float64, device="cuda")
        dist.all_reduce(ms_t, op=dist.ReduceOp.MAX)
        ms = float(ms_t.item())
    value = B * K / (ms / 1000.0)
    # ---- end to end through the C ABI: host tokens in, host argmax out, every step
    kv2, firsts2 = prefilled()
    t = np.asarray(firsts2, np.uint32)
    for _ in range(W):
        t, _ = eng.decode_batch(kv2, t)
    if dist:
        dist.barrier()
    t0 = time.perf_counter()
    for _ in range(K):
        t, _ = eng.decode_batch(kv2, t)
    e2e_s = time.perf_counter() - t0
    if dist:
        e_t = torch.tensor([e2e_s], dtype=torch.float64, device="cuda")
        dist.all_reduce(e_t, op=dist.ReduceOp.MAX)
        e2e_s = float(e_t.item())
    e2e = B * K / e2e_s
    peak, peak_kind = peaks()
    mean_pos = F16_PROMPT + W + (K - 1) / 2.0 + 1
    step_bytes = f16_bytes_per_step(args.layers) + B * kv_bytes_per_pos(args.layers) * mean_pos
    rank_bytes = step_bytes / world  # weights, lm_head rows and (to tp 4) KV heads split evenly
    achieved = rank_bytes / (ms / K / 1000.0) / 1e9
    line = {
        "metric": F16_METRIC, "value": value, "unit": "tok/s", "n_gpus": world, "steps": K, "warmup": W,
        "ms_per_step": ms / K, "higher_is_better": True, "scaling": "strong", "vs_baseline": None,
        "dtype": "f16 weights x f32 activations (f16 hi+lo split), f32 accumulate",
        "data": "synthetic (seeded random-init SmolLM3-3B F16 weights, random prompt ids)",
        "config": {"workload": f"config 5: SmolLM3-3B F16 (36 layers, vocab 128256), batch {B}, "
                               f"{F16_PROMPT}-token prompts, greedy decode",
                   "batch": B, "prompt": F16_PROMPT, "layers": args.layers, "kv_len_mean": mean_pos,
                   "parallelism": "single GPU" if world == 1 else f"tp{world} (tensor parallel, NVLink peer exchange)",
                   "bytes_per_step": step_bytes,
                   "l2": f"inputs larger than L2: {f16_bytes_per_step(args.layers) / 1e9:.2f} GB of weights "
                         "streamed per step",
                   "prefill_tok_s": B * F16_PROMPT / prefill_s},
        "e2e": {"value": e2e, "unit": "tok/s", "h2d_bytes_per_step": 4 * B, "d2h_bytes_per_step": 4 * B},
        "gpu_launches": (eng.launches_per_step() + 1) * K,
        "roofline": dict(bound="hbm", achieved=achieved, peak=peak, peak_kind=f"{peak_kind} hbm_gbs (copy)",
                         unit="GB/s", frac=achieved / peak, traffic=None,
                         kernel="whole batched decode step (4 tcgen05 GEMMs + attention per layer, lm_head)"
                                + (f", per rank of a {world}-way tensor-parallel group" if world > 1 else ""),
                         bytes_per_launch=rank_bytes, us_per_launch=1000 * ms / K, launches_timed=K),
        "clocks": clk.summary(),
    }
    if not args.no_cpu_baseline and rank == 0 and world == 1:
        v, n = f16_cpu_sample(model, args.cpu_seconds, threads)
        line["cpu_baseline"] = {"value": v, "unit": "tok/s", "cores": threads, "kind": "port",
                                "sample": f"{n} forward_decode_raw steps of one F16 sequence, {threads} threads "
                                          f"(the CPU path has no batching)", "cpu": cpu_model()}
    kv.close()
    kv2.close()
    eng.close()
    if dist:
        dist.barrier()
        dist.destroy_process_group()
    if rank == 0:
        print(json.dumps(line), flush=True)
    return 0


LONG_CTX = 32768


def long_kv(layers, seed=4):
    """Seeded f32 N(0,1) K/V rows for every layer, token-major [S][4*128] (config 4)."""
    rng = np.random.default_rng(seed)
    return [(rng.standard_normal((LONG_CTX, 512), dtype=np.float32),
             rng.standard_normal((LONG_CTX, 512), dtype=np.float32)) for _ in range(layers)]


def run_q4_long(args, rank, world, local_rank):
    """benchmark config 4: the Q4 model with every layer's KV cache pre-filled to 32768
    positions (qora_kv_import), then greedy decode at batch 1; attention KV reads
    dominate the bytes per token."""
    if world > 1:
        if rank == 0:
            print(json.dumps({"metric": METRIC + ", 32K context", "unavailable": "the long-context line is single-GPU"}))
        return 0
    K, W = args.steps, args.warmup
    threads = os.cpu_count() or 1
    model, prompt = synth(args.layers)
    kvs = long_kv(args.layers)
    first_tok = int(prompt[0])
    f16kv = args.kv == "f16"
    metric = "decode tok/s (batch 1, SmolLM3-3B Q4, 32K-token KV cache)"
    if f16kv:  # opt-in, reported separately: results differ from the f32 cache
        metric = "decode tok/s (batch 1, SmolLM3-3B Q4, 32K-token binary16 KV cache)"
    kv_note = ", binary16 KV (opt-in)" if f16kv else ""
    if args.impl == "reference":
        sys.path.insert(0, os.path.join(ROOT, "oracle"))
        import oracle
        oracle.set_threads(threads)
        om = oracle.OracleModel(model)
        okv = om.new_kv(args.kv)
        for layer, (k, v) in enumerate(kvs):
            okv.import_layer(layer, k, v)
        tok = oracle.argmax(om.forward_decode(first_tok, okv))
        t0 = time.perf_counter()
        n = 0
        while n < K and (n < 2 or time.perf_counter() - t0 < args.cpu_seconds):
            tok = oracle.argmax(om.forward_decode(tok, okv))
            n += 1
        v = n / (time.perf_counter() - t0)
        line = {"impl": "reference", "metric": metric, "value": v, "unit": "tok/s", "n_gpus": 1, "steps": n,
                "warmup": 1, "ms_per_step": 1000.0 / v, "higher_is_better": True, "scaling": "strong",
                "vs_baseline": None, "dtype": "f32", "data": "synthetic (seeded random-init SmolLM3-3B Q4, N(0,1) KV)",
                "config": {"workload": "config 4: SmolLM3-3B Q4, KV pre-filled to 32768 positions, greedy decode"
                                       + kv_note, "kv": args.kv},
                "cpu_baseline": {"value": v, "unit": "tok/s", "cores": threads, "kind": "port",
                                 "sample": f"{n} forward_decode_raw steps after the 32768-row import, {threads} threads",
                                 "cpu": cpu_model()},
                "e2e": {"value": v, "unit": "tok/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}
        print(json.dumps(line), flush=True)
        return 0
    import importlib
    import torch
    pkg = importlib.import_module("qora-llm_b200")
    torch.cuda.set_device(local_rank)
    eng = pkg.DecodeWeights(model=model, device=local_rank)
    cap = LONG_CTX + W + K + 8

    def filled():
        kv = eng.new_kv(cap, dtype=args.kv)
        for layer, (k, v) in enumerate(kvs):
            kv.import_layer(layer, k, v)
        return kv

    kv = filled()
    toks = eng.generate_greedy(kv, first_tok, W)
    torch.cuda.synchronize()
    with ClockSampler(local_rank) as clk:
        _, ms = eng.generate_greedy_timed(kv, int(toks[-1]), K)
    torch.cuda.synchronize()
    value = K / (ms / 1000.0)
    kv.close()
    kv2 = filled()
    t = first_tok
    for _ in range(W):
        t = eng.decode_step(kv2, t)
    t0 = time.perf_counter()
    for _ in range(K):
        t = eng.decode_step(kv2, t)
    e2e = K / (time.perf_counter() - t0)
    kv2.close()
    peak, peak_kind = peaks()
    mean_kv = LONG_CTX + W + (K - 1) / 2.0 + 1
    step_bytes = weight_bytes_per_token(args.layers) + kv_bytes_per_pos(args.layers, 2 if f16kv else 4) * (mean_kv + 1)
    achieved = step_bytes / (ms / K / 1000.0) / 1e9
    line = {
        "metric": metric, "value": value, "unit": "tok/s", "n_gpus": 1, "steps": K, "warmup": W,
        "ms_per_step": ms / K, "higher_is_better": True, "scaling": "strong", "vs_baseline": None, "dtype": "f32",
        "data": "synthetic (seeded random-init SmolLM3-3B Q4 weights, N(0,1) f32 KV rows)",
        "config": {"workload": "config 4: SmolLM3-3B Q4, KV of all 36 layers pre-filled to 32768 positions, "
                               "greedy decode at batch 1" + kv_note,
                   "kv": args.kv, "kv_len_mean": mean_kv, "layers": args.layers, "parallelism": "single GPU",
                   "bytes_per_step": step_bytes,
                   "l2": "inputs larger than L2: 6.6 GB of weights + KV streamed per step"},
        "e2e": {"value": e2e, "unit": "tok/s", "h2d_bytes_per_step": 4, "d2h_bytes_per_step": 4},
        "gpu_launches": eng.launches_per_step() * K,
        "roofline": dict(bound="hbm", achieved=achieved, peak=peak, peak_kind=f"{peak_kind} hbm_gbs (copy)",
                         unit="GB/s", frac=achieved / peak, traffic=None,
                         kernel="decode megakernel (whole step; attention over 32K cached rows per layer)",
                         bytes_per_launch=step_bytes, us_per_launch=1000 * ms / K, launches_timed=K),
        "clocks": clk.summary(),
    }
    eng.close()
    print(json.dumps(line), flush=True)
    return 0


# ---------------------------------------------------------------- config 1: Q4 GEMV
GEMV_METRIC = "Q4 GEMV HBM GB/s (config 1: gate_proj, k=2048 in, n=11008 out, reference F1 layout)"
GEMV_K, GEMV_N = 2048, 11008
L2_BYTES = 126 * 1024 * 1024


def gemv_bytes(k=GEMV_K, n=GEMV_N):
    """Algorithmic bytes of one GEMV: packed nibbles + f16 scales + x + y (12,733,440 for
    config 1)."""
    return k * n // 2 + k * n // 32 * 2 + k * 4 + n * 4


def config1():
    import importlib
    qf = importlib.import_module("qora-llm_b200").qora_format
    rng = np.random.default_rng(0)
    m = qf.synth_q4_matrix(rng, GEMV_K, GEMV_N)
    x = rng.standard_normal(GEMV_K).astype(np.float32)
    return m, x


def gemv_traffic():
    """DRAM bytes per launch of the config-1 GEMV from the committed ncu capture (or None)."""
    try:
        return json.load(open(os.path.join(ROOT, "profiles", "q4_gemv_config1_dram.json")))["dram_bytes_per_launch"]
    except Exception:
        return None


def gemv_cpu(m, x, steps, budget_s, threads):
    """The reference's gemv_q4 (oracle/: k-split over the host threads, AVX-512) timed per
    call on this host: median of >= 5 calls, bounded by ~budget_s. Returns (GB/s, calls)."""
    sys.path.insert(0, os.path.join(ROOT, "oracle"))
    import oracle
    oracle.set_threads(threads)
    oracle.gemv_q4(x, m)  # warm-up
    times, t_end = [], time.perf_counter() + budget_s
    while len(times) < max(5, steps) and (len(times) < 5 or time.perf_counter() < t_end):
        t0 = time.perf_counter()
        oracle.gemv_q4(x, m)
        times.append(time.perf_counter() - t0)
    return gemv_bytes() / statistics.median(times) / 1e9, len(times)


def run_q4_gemv(args, rank, world, local_rank):
    """benchmark config 1: the Q4 GEMV kernel alone (qora_q4_gemv on device buffers in the
    reference's F1 layout). Every launch reads a different copy of the weights, rotating
    over more than four times the L2 capacity, so each launch streams its weights from
    HBM; the K launches are captured in one CUDA graph and timed with CUDA events."""
    if world > 1:
        if rank == 0:
            print(json.dumps({"metric": GEMV_METRIC, "unavailable": "the config-1 GEMV line is single-GPU"}))
        return 0
    K, W = args.steps, args.warmup
    threads = os.cpu_count() or 1
    m, x = config1()
    cfg = {"workload": "config 1: one Q4 GEMV, gate_proj 2048 x 11008 (F1 layout, seed 0), x ~ N(0,1)",
           "k": GEMV_K, "n": GEMV_N, "bytes_per_gemv": gemv_bytes()}
    if args.impl == "reference":
        v, n = gemv_cpu(m, x, K, args.cpu_seconds, threads)
        line = {"impl": "reference", "metric": GEMV_METRIC, "value": v, "unit": "GB/s", "n_gpus": 1, "steps": n,
                "warmup": 1, "ms_per_step": gemv_bytes() / v / 1e6, "higher_is_better": True, "scaling": "strong",
                "vs_baseline": None, "dtype": "f32", "data": "synthetic (seeded Q4 gate_proj)", "config": cfg,
                "cpu_baseline": {"value": v, "unit": "GB/s", "cores": threads, "kind": "port",
                                 "sample": f"median of {n} gemv_q4 calls, {threads} threads", "cpu": cpu_model()},
                "e2e": {"value": v, "unit": "GB/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}
        print(json.dumps(line), flush=True)
        return 0
    import importlib
    import torch
    pkg = importlib.import_module("qora-llm_b200")
    torch.cuda.set_device(local_rank)
    copies = max(2, -(-4 * L2_BYTES // gemv_bytes()))
    packed = [torch.from_numpy(m.packed).cuda() for _ in range(copies)]
    scales = [torch.from_numpy(m.scales.view(np.int16)).cuda() for _ in range(copies)]
    dx = torch.from_numpy(x).cuda()
    dy = torch.empty(GEMV_N, dtype=torch.float32, device="cuda")
    stream = torch.cuda.Stream()

    def gemv(i, s):
        pkg.engine.q4_gemv(dx.data_ptr(), packed[i % copies].data_ptr(), scales[i % copies].data_ptr(),
                           GEMV_K, GEMV_N, dy.data_ptr(), stream=s)

    with torch.cuda.stream(stream):  # warm-up (also sizes the library's cached scratch)
        for i in range(W):
            gemv(i, stream)
    stream.synchronize()
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph, stream=stream):
        cap = torch.cuda.current_stream()
        for i in range(K):
            gemv(i, cap)
    graph.replay()  # untimed replay
    stream.synchronize()
    # replay the K-launch graph until >= 1 s has passed (so the clock sampler sees the
    # timed region), each replay timed with CUDA events; report the median replay
    reps, t_end = [], time.perf_counter() + 1.0
    with ClockSampler(local_rank) as clk:
        while len(reps) < 3 or time.perf_counter() < t_end:
            t0, t1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            t0.record(stream)
            with torch.cuda.stream(stream):
                graph.replay()
            t1.record(stream)
            t1.synchronize()
            reps.append(t0.elapsed_time(t1))
    ms = statistics.median(reps)
    value = gemv_bytes() / (ms / K / 1000.0) / 1e9
    # e2e: per step, x from pinned host memory, the GEMV through the C ABI, y back
    hx = torch.from_numpy(x).pin_memory()
    hy = torch.empty(GEMV_N, dtype=torch.float32).pin_memory()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(stream)
    with torch.cuda.stream(stream):
        for i in range(K):
            dx.copy_(hx, non_blocking=True)
            gemv(i, stream)
            hy.copy_(dy, non_blocking=True)
    e1.record(stream)
    e1.synchronize()
    e2e = gemv_bytes() / (e0.elapsed_time(e1) / K / 1000.0) / 1e9
    del graph
    peak, peak_kind = peaks()
    line = {
        "metric": GEMV_METRIC, "value": value, "unit": "GB/s", "n_gpus": 1, "steps": K, "warmup": W,
        "ms_per_step": ms / K, "higher_is_better": True, "scaling": "strong", "vs_baseline": None, "dtype": "f32",
        "data": "synthetic (seeded Q4 gate_proj, N(0,1) input)",
        "config": dict(cfg, weight_copies=copies,
                       l2=f"weights rotated over {copies} copies ({copies * gemv_bytes() / 1e6:.0f} MB, > 4x L2)",
                       timing=f"K launches in one CUDA graph, CUDA events around each replay; median of "
                              f"{len(reps)} replays over >= 1 s"),
        "e2e": {"value": e2e, "unit": "GB/s", "h2d_bytes_per_step": GEMV_K * 4, "d2h_bytes_per_step": GEMV_N * 4},
        "gpu_launches": K,
        "roofline": dict(bound="hbm", achieved=value, peak=peak, peak_kind=f"{peak_kind} hbm_gbs (copy)",
                         unit="GB/s", frac=value / peak, traffic=gemv_traffic(), kernel="q4 split-K GEMV (qora_q4_gemv)",
                         bytes_per_launch=gemv_bytes(), us_per_launch=1000 * ms / K, launches_timed=K),
        "clocks": clk.summary(),
    }
    if not args.no_cpu_baseline:
        v, n = gemv_cpu(m, x, 5, args.cpu_seconds, threads)
        line["cpu_baseline"] = {"value": v, "unit": "GB/s", "cores": threads, "kind": "port",
                                "sample": f"median of {n} gemv_q4 calls, {threads} threads", "cpu": cpu_model()}
    print(json.dumps(line), flush=True)
    return 0


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=256)
    ap.add_argument("--warmup", type=int, default=8)
    ap.add_argument("--impl", choices=("ours", "reference"), default="ours")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--cpu-seconds", type=float, default=15.0)
    ap.add_argument("--workload", choices=("q4", "q4-long", "f16-batch", "q4-gemv"), default="q4",
                    help="q4: config 3 batch-1 decode (the headline); q4-long: config 4; f16-batch: config 5; "
                         "q4-gemv: config 1 (the Q4 GEMV kernel alone, GB/s)")
    ap.add_argument("--batch", type=int, default=32, help="sequences for --workload f16-batch")
    ap.add_argument("--kv", choices=("f32", "f16"), default="f32",
                    help="KV cache element type for --workload q4-long (f16: the opt-in binary16 cache, "
                         "reported as its own metric)")
    ap.add_argument("--layers", type=int, default=36,
                    help="decoder layers of the synthetic model (36 = SmolLM3-3B; fewer only for "
                         "small profiling captures, never for a reported number)")
    args = ap.parse_args()
    if args.warmup < 3:
        ap.error("--warmup must be >= 3")
    rank = int(os.environ.get("RANK", "0"))
    world = int(os.environ.get("WORLD_SIZE", "1"))
    local_rank = int(os.environ.get("LOCAL_RANK", "0"))
    if args.workload == "f16-batch":
        return run_f16(args, rank, world, local_rank)
    if args.workload == "q4-long":
        return run_q4_long(args, rank, world, local_rank)
    if args.workload == "q4-gemv":
        return run_q4_gemv(args, rank, world, local_rank)
    if args.impl == "reference":
        return run_reference(args, rank)
    return run_ours(args, rank, world, local_rank)


if __name__ == "__main__":
    sys.exit(main())
