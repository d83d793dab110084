#!/usr/bin/env python
"""Benchmark of the SDPA path on B200: one JSON line per run (rank 0).

    python bench.py [--gpus N] [--steps K] [--warmup W] [--workload NAME] [--impl ours|reference]

Workloads (synthetic seeded inputs of each config's shape):
  gpt2_causal_fwd_bwd     cfg 3: q,k,v,dO [8,12,1024,64] N(0,1), causal, forward+backward (default)
  gpt2_floatmask_fwd_bwd  cfg 3 variant: additive float mask [1024,1024] of N(0,1)*0.1, non-causal
  nanogpt_causal_fwd_bwd  cfg 1: [64,6,256,64], causal, forward+backward
  mha_core_fwd_bwd        cfg 2 core: [32,8,128,64] with key padding lengths U[16,128], forward+backward
  long_causal_fwd         cfg 4: [1,16,32768,128] N(0,1)*0.5, causal, forward only
  long_causal_fwd_8k      cfg 4's shape at 8192 keys (a profiling case)
  decode_splitkv          cfg 5: q [64,32,1,128], K/V [64,32,8192,128], split-KV decode (GB/s)

Scaling is weak: under torchrun every rank runs the full workload on its own GPU (its shard of
a global batch N times larger); there is no data-path collective. ``value`` = work of all
ranks / max-over-ranks device time. The exception is long_causal_fwd on N > 1 GPUs: the ranks
share one sequence through ring attention (zig-zag shards, NCCL send/recv of K/V blocks,
logsumexp merge), so scaling is strong and ``value`` = the sequence's work / max device time.
"""
from __future__ import annotations

import argparse
import json
import math
import os
import statistics
import subprocess
import sys
import time

import numpy as np
import torch

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)

METRIC = "causal SDPA fwd+bwd TFLOP/s & decode HBM GB/s at 1/2/4/8 B200 vs host CPU"

WORKLOADS = {
    "gpt2_causal_fwd_bwd": dict(q=(8, 12, 1024, 64), kv=(8, 12, 1024, 64), causal=True, mask=None, amp=1.0,
                                bwd=True, cfg=3),
    "gpt2_floatmask_fwd_bwd": dict(q=(8, 12, 1024, 64), kv=(8, 12, 1024, 64), causal=False, mask="float",
                                   amp=1.0, bwd=True, cfg=3),
    "nanogpt_causal_fwd_bwd": dict(q=(64, 6, 256, 64), kv=(64, 6, 256, 64), causal=True, mask=None, amp=1.0,
                                   bwd=True, cfg=1),
    "mha_core_fwd_bwd": dict(q=(32, 8, 128, 64), kv=(32, 8, 128, 64), causal=False, mask="keypad", amp=1.0,
                             bwd=True, cfg=2),
    "long_causal_fwd": dict(q=(1, 16, 32768, 128), kv=(1, 16, 32768, 128), causal=True, mask=None, amp=0.5,
                            bwd=False, cfg=4),
    "decode_splitkv": dict(q=(64, 32, 1, 128), kv=(64, 32, 8192, 128), causal=False, mask=None, amp=1.0,
                           bwd=False, cfg=5),
    # Config 3 with attention dropout (GPT-2's 0.1): the keep mask is drawn every step.
    "gpt2_dropout_fwd_bwd": dict(q=(8, 12, 1024, 64), kv=(8, 12, 1024, 64), causal=True, mask=None, amp=1.0,
                                 bwd=True, cfg=3, dropout=0.1),
    # Config 4's shape at a quarter of its length: a case small enough for a full ncu capture
    # of the D = 128 forward (its DRAM traffic scales with the key blocks each tile streams).
    "long_causal_fwd_8k": dict(q=(1, 16, 8192, 128), kv=(1, 16, 8192, 128), causal=True, mask=None, amp=0.5,
                               bwd=False, cfg=4),
}


def pairs_per_head(L, S, causal):
    """Visible (query, key) pairs of one head; causal is top-left (row i sees keys <= i)."""
    if not causal:
        return L * S
    m = min(L, S)
    return m * (m + 1) // 2 + (L - m) * S


def work(w):
    """Algorithmic work of one call: (amount, unit). Forward = 4*D per visible pair; backward
    = 2.5x forward; decode = bytes of K, V, q and out."""
    B, H, L, D = w["q"]
    S = w["kv"][2]
    if w["cfg"] == 5:
        return 4.0 * (2 * B * H * S * D + 2 * B * H * L * D), "GB/s"
    fwd = 4.0 * D * pairs_per_head(L, S, w["causal"]) * B * H
    return fwd * (3.5 if w["bwd"] else 1.0), "TFLOP/s"


def kernel_work(w, name):
    """Algorithmic work attributed to one launch of a kernel (flops or bytes).
    Backward accounting (5 GEMM-equivalents of 2*D per pair: S, dP, dV, dK, dQ): the dK/dV
    kernel owns S, dP, dV, dK; the dQ kernel owns dQ (its recomputation of S and dP is
    overhead, not algorithmic work)."""
    B, H, L, D = w["q"]
    S = w["kv"][2]
    pairs = pairs_per_head(L, S, w["causal"]) * B * H
    gemm = 2.0 * D * pairs
    if name.startswith("fwd"):
        return 2 * gemm
    if name == "bwd_tc":  # dK/dV and dQ, run concurrently: one record spans both
        return 5 * gemm
    if "dkdv" in name:
        return 4 * gemm
    if "bwd_dq" in name:
        return gemm
    if name == "decode_split":
        return 4.0 * 2 * B * H * S * D
    return 0.0


def make_inputs(w, device, seed):
    gen = torch.Generator(device=device).manual_seed(seed)
    q = torch.randn(w["q"], device=device, generator=gen) * w["amp"]
    k = torch.randn(w["kv"], device=device, generator=gen) * w["amp"]
    v = torch.randn(w["kv"], device=device, generator=gen) * w["amp"]
    g = torch.randn(w["q"], device=device, generator=gen) if w["bwd"] else None
    L, S = w["q"][2], w["kv"][2]
    mask = None
    if w["mask"] == "float":
        mask = (torch.randn(L, S, device=device, generator=gen) * 0.1).view(1, 1, L, S)
    elif w["mask"] == "keypad":
        B = w["q"][0]
        rng = np.random.default_rng(seed)
        lengths = torch.from_numpy(rng.integers(16, S + 1, size=B)).to(device)
        keep = torch.arange(S, device=device)[None, :] < lengths[:, None]
        mask = keep.view(B, 1, 1, S)  # bool: True may attend
    return q, k, v, g, mask


def peaks():
    path = os.path.join(ROOT, "MEASURED_PEAKS.json")
    if os.path.exists(path):
        with open(path) as f:
            p = json.load(f)
        return dict(hbm=p["hbm_gbs"], bf16=p["bf16_tflops"], src="measured")
    return dict(hbm=6650.0, bf16=1590.0, src="fallback")


class ClockSampler:
    """nvidia-smi clocks and throttle reasons, sampled every 200 ms. Sampling is live before the
    timed region starts (the first sample has arrived) and one more sample is taken after it
    ends, so even a timed region shorter than the sampling period is bracketed by samples."""
    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, gpu_index):
        self.gpu = gpu_index
        self.proc = None
        self.lines = []
        self.first = 0

    def _read(self):
        for line in self.proc.stdout:
            if line.strip():
                self.lines.append(line)

    def _wait_for(self, n, timeout):
        t0 = time.time()
        while len(self.lines) < n and time.time() - t0 < timeout and self.proc.poll() is None:
            time.sleep(0.01)

    def __enter__(self):
        import threading
        try:
            self.proc = subprocess.Popen(["nvidia-smi", f"--id={self.gpu}", f"--query-gpu={self.FIELDS}",
                                          "--format=csv,noheader,nounits", "-lms", "200"],
                                         stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
        except OSError:
            self.proc = None
            return self
        self.reader = threading.Thread(target=self._read, daemon=True)
        self.reader.start()
        self._wait_for(1, 10.0)
        self.first = max(0, len(self.lines) - 1)  # the last sample before the timed region
        return self

    def __exit__(self, *exc):
        if self.proc is None:
            return
        self._wait_for(len(self.lines) + 1, 2.0)  # one sample after the timed region
        self.proc.terminate()
        try:
            self.proc.wait(timeout=5)
        except subprocess.TimeoutExpired:
            self.proc.kill()
            self.proc.wait()
        self.reader.join(timeout=5)
        self.lines = self.lines[self.first:]

    def summary(self):
        if not getattr(self, "lines", None):
            return None
        sm, mx, reasons = [], 0.0, set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for line in self.lines:
            parts = [p.strip() for p in line.split(",")]
            if len(parts) < 9:
                continue
            try:
                sm.append(float(parts[1]))
                mx = max(mx, float(parts[2]))
            except ValueError:
                continue
            for n, val in zip(names, parts[5:9]):
                if val.lower() == "active":
                    reasons.add(n)
        if not sm:
            return None
        return {"sm_mhz": statistics.median(sm), "sm_max_mhz": mx, "reasons": sorted(reasons),
                "samples": len(sm)}


def physical_gpu(local):
    vis = os.environ.get("CUDA_VISIBLE_DEVICES")
    if vis:
        ids = [x.strip() for x in vis.split(",") if x.strip()]
        if local < len(ids):
            return ids[local]
    return str(local)


def cpu_baseline(w, name, budget_s=12.0, threads=None):
    """The oracle (a C restatement of DenseCore's CPU flash path) on a bounded sample of the
    workload, timed on this host's cores. Returns the cpu_baseline object."""
    import oracle
    threads = threads or oracle.default_threads()
    B, H, L, D = w["q"]
    S = w["kv"][2]
    rng = np.random.default_rng(1)
    if w["cfg"] == 4:
        # Causal prefix sample: the first R rows of `heads` heads (keys <= row), extrapolated by
        # visible pairs; per-pair cost does not depend on the row.
        R, heads = (4096 if budget_s >= 10 else 2048), threads
        q, k, v = (rng.normal(size=(1, heads, R, D)).astype(np.float32) * w["amp"] for _ in range(3))
        t0 = time.perf_counter()
        oracle.flash_forward(q, k, v, causal=True, threads=threads)
        dt = time.perf_counter() - t0
        flops = 4.0 * D * pairs_per_head(R, R, True) * heads
        return {"value": flops / dt / 1e12, "unit": "TFLOP/s", "cores": threads, "kind": "port",
                "sample": f"causal prefix of {R} rows x {heads} heads of [1,16,32768,128], fwd, "
                          f"{dt:.1f} s"}
    if w.get("dropout"):
        # DenseCore runs dropout on its math path (functional.py:318-340): bmm through the
        # portable sgemm, one thread (torch_blas.rs:404-445), softmax, the sequential bernoulli
        # draw. Whole heads, one after another, including each head's draw.
        p = w["dropout"]
        gen = oracle.MtGenerator(1)
        done, dt = 0, 0.0
        while dt < budget_s and done < B * H:
            q, k, v, g = (rng.normal(size=(1, 1, L, D)).astype(np.float32) * w["amp"] for _ in range(4))
            t0 = time.perf_counter()
            keep = oracle.unpack_bits(gen.keep_bits(L * S, 1 - p), L * S)
            out, saved = oracle.sdpa_math_forward(q, k, v, causal=w["causal"], noise=oracle.dropout_noise(keep, p))
            oracle.sdpa_math_backward(g, v, saved)
            dt += time.perf_counter() - t0
            done += 1
        amount, unit = work(w)
        return {"value": amount / (B * H) * done / dt / 1e12, "unit": unit, "cores": 1, "kind": "port",
                "sample": f"{done} of {B * H} heads of {name} through the dropout math path "
                          f"(fwd+bwd, mask draw included), {dt:.1f} s"}
    # Whole (batch, head) tasks; tasks are independent, so a sample's rate is the full run's.
    nb = min(B, max(1, math.ceil(threads / H)))
    q = rng.normal(size=(nb, H, L, D)).astype(np.float32) * w["amp"]
    k, v = (rng.normal(size=(nb, H, S, D)).astype(np.float32) * w["amp"] for _ in range(2))
    g = rng.normal(size=(nb, H, L, D)).astype(np.float32)
    mask = None
    if w["mask"] == "float":
        mask = oracle.flash_mask((rng.normal(size=(L, S)) * 0.1).astype(np.float32), q.shape, S)
    elif w["mask"] == "keypad":
        lengths = rng.integers(16, S + 1, size=nb)
        keep = np.arange(S)[None, :] < lengths[:, None]
        mask = oracle.flash_mask(keep[:, None, None, :], q.shape, S)
    tasks_all = np.arange(nb * H)
    done, dt, rounds = 0, 0.0, 0
    while dt < budget_s and rounds < 64:
        tasks = tasks_all[: min(len(tasks_all), threads)]
        t0 = time.perf_counter()
        out, lse = oracle.flash_forward_tasks(q, k, v, tasks, mask, w["causal"], threads=threads)
        if w["bwd"]:
            oracle.flash_backward_tasks(g, q, k, v, out, lse, tasks, mask, w["causal"], threads=threads)
        dt += time.perf_counter() - t0
        done += len(tasks)
        rounds += 1
    amount, unit = work(w)
    per_task = amount / (B * H)
    scale = 1e9 if unit == "GB/s" else 1e12
    return {"value": per_task * done / dt / scale, "unit": unit, "cores": threads, "kind": "port",
            "sample": f"{done} of {B * H} (batch, head) tasks of {name} "
                      f"({'fwd+bwd' if w['bwd'] else 'fwd'}), {dt:.1f} s"}


def config_of(name, w, world, ring=False):
    """The workload a line measures (both arms print the same dict for the same run)."""
    return {"workload": name, "baseline_cfg": w["cfg"], "shape_q": list(w["q"]), "shape_kv": list(w["kv"]),
            "causal": w["causal"], "mask": w["mask"], "dropout_p": w.get("dropout", 0.0),
            "per_rank": ("zig-zag sequence shard (ring attention, NCCL send/recv)" if ring
                         else "full workload (weak scaling)"),
            "parallelism": f"ring{world}" if ring else f"dp{world}",
            "l2": "GPU arm: flushed (256 MB write) before every timed step"}


def run_reference(args, w, name, rank, world):
    """--impl reference: DenseCore's CPU algorithm (the oracle port; the Rust reference cannot
    be built here) on the host cores, each step a bounded sample of the workload."""
    if rank != 0:
        return
    import oracle
    threads = oracle.default_threads()
    vals = []
    for i in range(args.warmup + args.steps):
        cb = cpu_baseline(w, name, budget_s=2.0, threads=threads)
        if i >= args.warmup:
            vals.append(cb["value"])
    value = statistics.mean(vals)
    _, unit = work(w)
    cb["value"] = value
    ring = w["cfg"] == 4 and world > 1
    line = {"impl": "reference", "metric": METRIC, "value": value, "unit": unit, "n_gpus": world,
            "steps": args.steps, "warmup": args.warmup, "higher_is_better": True,
            "scaling": "strong" if ring else "weak", "vs_baseline": None, "dtype": "f32",
            "data": "synthetic (seeded N(0,1) of the config's shape)",
            "config": config_of(name, w, world, ring),
            "cpu_baseline": cb,
            "e2e": {"value": value, "unit": unit, "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}
    print(json.dumps(line), flush=True)


def _max_over_ranks(x, dist, device):
    if dist is None:
        return x
    t = torch.tensor([x], device=device, dtype=torch.float64)
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t.item())


def _barrier(dist):
    if dist is not None:
        dist.barrier()
    torch.cuda.synchronize()


def measure(name, w, device, dist, steps, warmup, *, agg_amount=None, inputs=None, ring=None, e2e=False,
            e2e_args=None, cpu=False, cpu_budget=12.0, clocks=False, seed=1234):
    """One workload on this rank's GPU: W untimed steps, then K timed steps (CUDA events around
    each, L2 flushed before each), max over ranks; a second, untimed pass of the same steps with
    the library's per-launch tracing gives the kernel breakdown and the roofline's unit.
    ``agg_amount`` is the algorithmic work all ranks do in one step together (default: this
    rank's workload times the world size). Every rank must call this with the same arguments
    (it takes barriers and all-reduces)."""
    import densecore_b200 as dc
    from densecore_b200 import _lib, _native

    if inputs is None:
        q, k, v, g, mask = make_inputs(w, device, seed=seed)
    else:
        q, k, v, g, mask = inputs
    causal = w["causal"]
    if ring is not None:
        def step():
            ring(q, k, v)
    elif w["cfg"] == 5:
        splits = _lib.load().dc_sdpa_decode_default_splits(q.shape[0], q.shape[1], k.shape[2])
        ws = torch.empty(_lib.load().dc_sdpa_decode_workspace_size(q.shape[0], q.shape[1], v.shape[3], splits),
                         dtype=torch.uint8, device=device)

        def step():
            _native._decode(q, k, v, None, None, splits, ws)
    elif w.get("dropout"):
        from densecore_b200.functional import _keep_mask
        n_weights = q.shape[0] * q.shape[1] * q.shape[2] * k.shape[2]
        dc.manual_seed(seed)

        def step():
            keep, ks = _keep_mask(n_weights, w["dropout"], device)
            out, lse = _native._flash_attention_dropout(q, k, v, causal, None, mask, keep, ks)
            _native._flash_attention_dropout_backward(g, q, k, v, out, lse, causal, None, mask, keep, ks)
    elif w["bwd"]:
        def step():
            out, lse = _native._flash_attention(q, k, v, causal, None, mask)
            _native._flash_attention_backward(g, q, k, v, out, lse, causal, None, mask)
    else:
        def step():
            _native._flash_attention(q, k, v, causal, None, mask)

    flush = torch.empty(64 * 1024 * 1024, dtype=torch.float32, device=device)  # 256 MB > 126 MB L2
    for _ in range(warmup):
        step()
    torch.cuda.synchronize()
    # The timed forward + backward steps replay a CUDA graph of one step (every kernel of the
    # step is launched by each replay): small workloads would otherwise wait on the host's
    # launches. Dropout (its generator state and temporary copies), decode and the ring (NCCL)
    # run eagerly.
    timed_step = step
    launch = "eager"
    graph = None
    if w["bwd"] and not w.get("dropout") and ring is None:
        side = torch.cuda.Stream(device)
        side.wait_stream(torch.cuda.current_stream(device))
        with torch.cuda.stream(side):
            step()
        torch.cuda.current_stream(device).wait_stream(side)
        torch.cuda.synchronize()
        graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(graph):
            step()
        timed_step = graph.replay
        launch = "cuda graph of one step"
        for _ in range(2):
            timed_step()
        torch.cuda.synchronize()

    starts = [torch.cuda.Event(enable_timing=True) for _ in range(steps)]
    ends = [torch.cuda.Event(enable_timing=True) for _ in range(steps)]
    _barrier(dist)
    local = device.index if device.index is not None else 0
    sampler = ClockSampler(physical_gpu(local)) if clocks else None
    if sampler is not None:
        sampler.__enter__()
    try:
        for i in range(steps):
            flush.zero_()
            starts[i].record()
            timed_step()
            ends[i].record()
        torch.cuda.synchronize()
    finally:
        if sampler is not None:
            sampler.__exit__(None, None, None)
    _barrier(dist)
    ms = sum(s_.elapsed_time(e_) for s_, e_ in zip(starts, ends)) / steps
    # Per-kernel breakdown from a second pass of the same steps with the library's tracing on:
    # it records two CUDA events around every launch, host work that would otherwise sit inside
    # the timed steps of small workloads.
    _lib.kernel_timing_report(reset=True)
    _lib.kernel_timing(True)
    for i in range(steps):
        flush.zero_()
        step()
    torch.cuda.synchronize()
    _lib.kernel_timing(False)
    _barrier(dist)
    kernels = _lib.kernel_timing_report(reset=True)
    del graph
    ms_max = _max_over_ranks(ms, dist, device)
    world = dist.get_world_size() if dist is not None else 1
    amount, unit = work(w)
    if agg_amount is None:
        agg_amount = amount * world
    scale = 1e9 if unit == "GB/s" else 1e12
    value = agg_amount / (ms_max / 1e3) / scale
    roofline = roofline_of(name, w, kernels, steps, ring, world, agg_amount / world if ring is not None else amount)
    launches = sum(v_[0] for k_, v_ in kernels.items() if k_ != "bwd_tc")  # bwd_tc spans two launches
    res = {"ms_per_step": ms_max, "value": value, "unit": unit, "launch": launch, "roofline": roofline,
           "kernels": {k_: {"launches": v_[0], "total_ms": v_[1]} for k_, v_ in kernels.items()},
           "gpu_launches": launches}
    if e2e:
        res["e2e"] = run_e2e(w, q, k, v, g, mask, e2e_args, device, scale, agg_amount, dist, ring)
    if cpu:
        res["cpu_baseline"] = cpu_baseline(w, name, budget_s=cpu_budget)
    if sampler is not None:
        res["clocks"] = sampler.summary()
    return res


def roofline_of(name, w, kernels, steps, ring, world, rank_amount):
    """Roofline of the dominant kernel (largest total device time in the traced pass). The
    tensor-core backward's dK/dV and dQ kernels share the GPU (two streams): their joint record
    "bwd_tc" is the unit, not either kernel alone."""
    pk = peaks()
    # Kernels without a roofline of their own (the dropout mask draw: integer generator work,
    # neither HBM- nor tensor-bound) are named in "slowest_kernel" but are not the unit.
    concurrent = ("bwd_dkdv_tc", "bwd_dq_tc") if "bwd_tc" in kernels else ()
    candidates = {k_: v_ for k_, v_ in kernels.items() if k_ not in concurrent}
    slowest = max(candidates.items(), key=lambda kv: kv[1][1])[0] if candidates else None
    candidates = {k_: v_ for k_, v_ in candidates.items() if kernel_work(w, k_) > 0 or ring is not None}
    dom = max(candidates.items(), key=lambda kv: kv[1][1]) if candidates else None
    if dom is None:
        return None
    kname, (launches, total_ms) = dom
    per_launch = kernel_work(w, kname)
    avg_ms = total_ms / max(launches, 1)
    if ring is not None:
        # Ring launches differ in size; per step the rank's forward launches together do
        # 1/world of the sequence's algorithmic flops.
        per_launch = rank_amount / (launches / steps)
    if kname == "decode_split" or w["cfg"] == 5:
        achieved = per_launch / (avg_ms / 1e3) / 1e9
        peak, ru, bound = pk["hbm"], "GB/s", "hbm"
    else:
        achieved = per_launch / (avg_ms / 1e3) / 1e12
        # Dense TF32 on sm_100 issues at half the bf16 rate: half the measured bf16 burst.
        peak, ru, bound = pk["bf16"] / 2.0, "TFLOP/s", "tensor"
    traffic = None
    tpath = os.path.join(ROOT, "profiles", "ncu_traffic.json")
    if os.path.exists(tpath):
        with open(tpath) as f:
            per = json.load(f).get(name, {})
        traffic = per.get(kname)
        if kname == "bwd_tc" and traffic is None and "bwd_dkdv_tc" in per and "bwd_dq_tc" in per:
            traffic = per["bwd_dkdv_tc"] + per["bwd_dq_tc"]
    return {"kernel": kname, "slowest_kernel": slowest, "bound": bound, "achieved": achieved, "peak": peak,
            "unit": ru, "frac": achieved / peak, "traffic": traffic, "avg_launch_ms": avg_ms,
            "peak_source": (f"{pk['src']} hbm_gbs" if bound == "hbm"
                            else f"{pk['src']} bf16_tflops / 2 (dense TF32 rate)")}


# The other configs of the baseline, measured on one GPU beside the headline (short runs, the
# CPU baseline on a short budget): (key, workload, precision).
SINGLE_GPU_EXTRAS = (
    ("cfg1_nanogpt", "nanogpt_causal_fwd_bwd", "3xtf32"),
    ("cfg2_mha_core", "mha_core_fwd_bwd", "3xtf32"),
    ("cfg3b_floatmask", "gpt2_floatmask_fwd_bwd", "3xtf32"),
    ("cfg3_tf32", "gpt2_causal_fwd_bwd", "tf32"),
    ("cfg4_long", "long_causal_fwd", "3xtf32"),
    ("cfg5_decode", "decode_splitkv", "3xtf32"),
)


def single_gpu_extras(device, steps):
    import densecore_b200 as dc
    out = {}
    for key, name, prec in SINGLE_GPU_EXTRAS:
        dc.set_sdpa_precision(prec)
        try:
            w = WORKLOADS[name]
            r = measure(name, w, device, None, steps, 3, cpu=prec == "3xtf32", cpu_budget=3.0, clocks=True)
        finally:
            dc.set_sdpa_precision(None)
        r.update(workload=name, precision=prec)
        out[key] = r
        torch.cuda.empty_cache()
    return out


def _guarded(extras, key, fn):
    """Runs one extra; an exception is recorded in its place instead of ending the run. (All
    ranks run the same code on the same shapes, so a failure is normally on every rank.)"""
    try:
        fn()
    except Exception as e:  # noqa: BLE001 -- reported in the JSON line
        extras[key] = {"error": f"{type(e).__name__}: {e}"[:500]}
        torch.cuda.empty_cache()


def multi_gpu_extras(device, dist, rank, world, steps, e2e_args):
    """At N > 1: config 3 strong-scaled over its 96 (batch, head) units, config 4 through ring
    attention (strong, with an in-run parity check), config 5 batch shards (strong)."""
    extras = {}
    _guarded(extras, "cfg3_strong", lambda: _cfg3_strong(extras, device, dist, rank, world, steps, e2e_args))
    _guarded(extras, "ring_cfg4", lambda: _ring_cfg4(extras, device, dist, rank, world, steps))
    _guarded(extras, "decode_shard", lambda: _decode_shard(extras, device, dist, rank, world, steps))
    return extras


def _cfg3_strong(extras, device, dist, rank, world, steps, e2e_args):
    # Config 3: the 96 independent (batch, head) units of [8, 12, 1024, 64] split evenly over the
    # ranks (12 per GPU at 8), as DenseCore's par_chunks splits them over threads
    # (torch_attention.rs:108-128). Each rank's units are a (1, 96/N, 1024, 64) slice; e2e
    # copies exactly that slice up from and its results back into pinned host buffers.
    w3 = WORKLOADS["gpt2_causal_fwd_bwd"]
    units = w3["q"][0] * w3["q"][1]
    if units % world == 0:
        per = units // world
        wr = dict(w3, q=(1, per, 1024, 64), kv=(1, per, 1024, 64))
        r = measure("gpt2_causal_fwd_bwd", wr, device, dist, steps, 3, agg_amount=work(w3)[0], e2e=True,
                    e2e_args=e2e_args, seed=4321 + rank, clocks=True)
        r.update(units_per_rank=per, scaling="strong",
                 scatter_gather="each rank copies its units' q, k, v, dO from pinned host memory and its "
                                "out, dq, dk, dv back (inside e2e's timed region)")
        extras["cfg3_strong"] = r
        torch.cuda.empty_cache()


def _ring_cfg4(extras, device, dist, rank, world, steps):
    from densecore_b200 import _native
    from densecore_b200.ring import NativeRingAttention, NcclCommunicator, RingAttention, zigzag_shard
    # Config 4 through ring attention (strong scaling): the C-ABI entry dc_ring_sdpa_fwd over an
    # NCCL communicator made through libnccl's C API (what a C or Rust host hands it), beside the
    # same ring driven from Python over torch.distributed, and the same forward on one GPU per
    # rank (all ranks at once) for the fraction of N x one GPU; then a parity check of every
    # rank's ring rows against single-GPU forwards of two heads over the whole sequence.
    w4 = WORKLOADS["long_causal_fwd"]
    S = w4["q"][2]
    if S % (2 * world) == 0:
        full = make_inputs(w4, device, seed=1234)
        q, k, v = (zigzag_shard(t, rank, world) for t in full[:3])
        comm = NcclCommunicator(device=device)
        try:
            ringn = NativeRingAttention(q.shape, k.shape, device, comm, causal=True)
            r = measure("long_causal_fwd", w4, device, dist, steps, 3, agg_amount=work(w4)[0],
                        inputs=(q, k, v, None, None), ring=ringn, clocks=True)
            out, lse = ringn(q, k, v)
            torch.cuda.synchronize()
        finally:
            dist.barrier()
            comm.destroy()
        ringt = RingAttention(q.shape, k.shape, device, causal=True)
        rt = measure("long_causal_fwd", w4, device, dist, steps, 3, agg_amount=work(w4)[0],
                     inputs=(q, k, v, None, None), ring=ringt)
        one = measure("long_causal_fwd", w4, device, dist, max(3, steps // 4), 3, agg_amount=work(w4)[0],
                      inputs=full, clocks=True)
        heads = [0, 9]
        so, sl = _native._flash_attention(*(t[:, heads].contiguous() for t in full[:3]), True)
        ref_o, ref_l = zigzag_shard(so, rank, world), zigzag_shard(sl.unsqueeze(-1), rank, world).squeeze(-1)
        err_o = float((out[:, heads] - ref_o).abs().max() / ref_o.abs().max())
        err_l = float((lse[:, heads] - ref_l).abs().max() / ref_l.abs().max())
        err = _max_over_ranks(max(err_o, err_l), dist, device)
        r.update(impl="dc_ring_sdpa_fwd (C ABI; NCCL send/recv on a side stream, merges in the library)",
                 scaling="strong", one_gpu_ms=one["ms_per_step"], one_gpu_value=one["value"],
                 one_gpu_clocks=one.get("clocks"),
                 frac_of_n_x_one_gpu=r["value"] / (world * one["value"]),
                 torch_ring={"ms_per_step": rt["ms_per_step"], "value": rt["value"],
                             "impl": "densecore_b200.ring.RingAttention (batch_isend_irecv over the NCCL process group)"},
                 parity={"max_rel_err": err, "tol": 1e-5, "ok": err <= 1e-5,
                         "what": "every rank's ring out and lse, heads 0 and 9, against a single-GPU forward "
                                 "of those heads over the whole sequence (max |delta| / max |ref|)"})
        extras["ring_cfg4"] = r
        del full, q, k, v, ringn, ringt, out, lse, so, sl
        torch.cuda.empty_cache()


def _decode_shard(extras, device, dist, rank, world, steps):
    # Config 5: the batch of 64 decode rows split over the ranks (8 per GPU at 8); each rank
    # streams its K/V shard (17.18 GB / N).
    w5 = WORKLOADS["decode_splitkv"]
    if w5["q"][0] % world == 0:
        bpr = w5["q"][0] // world
        wr = dict(w5, q=(bpr,) + w5["q"][1:], kv=(bpr,) + w5["kv"][1:])
        r = measure("decode_splitkv", wr, device, dist, steps, 3, agg_amount=work(w5)[0], seed=999 + rank,
                    clocks=True)
        r.update(batch_per_rank=bpr, scaling="strong",
                 frac_of_n_x_hbm=r["value"] / (world * peaks()["hbm"]))
        extras["decode_shard"] = r
        torch.cuda.empty_cache()


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=20)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--workload", default="gpt2_causal_fwd_bwd", choices=sorted(WORKLOADS))
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--precision", default="3xtf32", choices=["3xtf32", "tf32", "fp32"])
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--no-e2e", action="store_true")
    ap.add_argument("--no-extras", action="store_true", help="only the headline workload")
    args = ap.parse_args()
    if args.warmup < 3:
        ap.error("--warmup must be >= 3")
    name = args.workload
    w = WORKLOADS[name]
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if world != args.gpus:
        print(f"bench.py: --gpus {args.gpus} but WORLD_SIZE={world}", file=sys.stderr)
    if args.impl == "reference":
        run_reference(args, w, name, rank, world)
        return

    import densecore_b200 as dc
    from densecore_b200 import _lib

    torch.cuda.set_device(local)
    device = torch.device("cuda", local)
    dist = None
    if world > 1:
        import datetime
        import torch.distributed as dist
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=300), device_id=device)
    dc.set_sdpa_precision(args.precision)
    _lib.load()

    # Config 4 on several GPUs is sequence-parallel (ring attention over zig-zag shards of one
    # sequence: strong scaling); every other headline gives each rank a whole workload (weak
    # scaling).
    ring = None
    inputs = None
    agg = None
    if w["cfg"] == 4 and world > 1:
        from densecore_b200.ring import RingAttention, zigzag_shard
        full = make_inputs(w, device, seed=1234)
        q, k, v = (zigzag_shard(t, rank, world) for t in full[:3])
        del full
        inputs = (q, k, v, None, None)
        ring = RingAttention(q.shape, k.shape, device, causal=True)
        agg = work(w)[0]
    head = measure(name, w, device, dist, args.steps, args.warmup, agg_amount=agg, inputs=inputs, ring=ring,
                   e2e=not args.no_e2e, e2e_args=args, clocks=True, seed=1234 + rank,
                   cpu=rank == 0 and world == 1 and not args.no_cpu_baseline)
    del inputs, ring
    torch.cuda.empty_cache()

    extras = {}
    if not args.no_extras and name == "gpt2_causal_fwd_bwd" and args.precision == "3xtf32":
        if world == 1:
            extras["configs"] = single_gpu_extras(device, min(args.steps, 10))
        else:
            extras.update(multi_gpu_extras(device, dist, rank, world, min(args.steps, 10), args))
    dc.set_sdpa_precision(args.precision)

    if rank == 0:
        line = {"metric": METRIC, "value": head["value"], "unit": head["unit"], "n_gpus": world,
                "steps": args.steps, "warmup": args.warmup, "ms_per_step": head["ms_per_step"],
                "higher_is_better": True, "scaling": "strong" if w["cfg"] == 4 and world > 1 else "weak",
                "vs_baseline": None, "dtype": "f32" if args.precision == "fp32" else args.precision,
                "data": "synthetic (seeded N(0,1) of the config's shape)",
                "config": config_of(name, w, world, w["cfg"] == 4 and world > 1),
                "timing": {"launch": head["launch"], "precision": args.precision,
                           "kernel_breakdown": "a second, untimed pass of the same steps with per-launch tracing"},
                "roofline": head["roofline"], "kernels": head["kernels"], "gpu_launches": head["gpu_launches"],
                "e2e": head.get("e2e"), "cpu_baseline": head.get("cpu_baseline"), "clocks": head.get("clocks")}
        line.update(extras)
        print(json.dumps(line), flush=True)
    if dist is not None:
        dist.barrier()
        dist.destroy_process_group()


def run_e2e(w, q, k, v, g, mask, args, device, scale, amount, dist, ring=None):
    """The metric through the public API with host buffers: every step copies its inputs from
    pinned host memory and its outputs (out and, with a backward, the three gradients) back.
    Steps are pipelined the way a training or serving loop would run them: step i+1's inputs go
    up on one stream while step i computes on a second and step i-1's results come down on a
    third (three buffer slots, events guarding their reuse, the host at most three steps ahead)."""
    import densecore_b200 as dc
    ins = [q, k, v] + ([g] if g is not None else [])
    if w["cfg"] == 5:
        ins = [q]  # the KV cache is device-resident state; a decode step brings its query
    if ring is not None:
        outs_shape = [tuple(q.shape)]
    elif w["cfg"] == 5:
        outs_shape = [(w["q"][0], w["q"][1], 1, w["kv"][3])]
    elif w["bwd"]:
        outs_shape = [tuple(w["q"]), tuple(w["q"]), tuple(w["kv"]), tuple(w["kv"])]
    else:
        outs_shape = [tuple(w["q"])]
    nslot = 3  # a slot's copy back can overlap the next two steps' copies up and compute
    host_in = [[t.detach().cpu().pin_memory() for t in ins] for _ in range(nslot)]
    dev_in = [[torch.empty_like(t) for t in ins] for _ in range(nslot)]
    host_out = [[torch.empty(s_, dtype=torch.float32).pin_memory() for s_ in outs_shape] for _ in range(nslot)]
    s_h2d, s_comp, s_d2h = (torch.cuda.Stream(device) for _ in range(3))
    ev_in = [torch.cuda.Event() for _ in range(nslot)]    # the slot's inputs landed
    ev_used = [torch.cuda.Event() for _ in range(nslot)]  # the slot's compute finished
    ev_out = [torch.cuda.Event() for _ in range(nslot)]   # the slot's results are on the host
    used = [False] * nslot
    last_res = [None] * nslot  # each slot's latest results (device tensors), reused by copy_ceiling

    def compute(d):
        if ring is not None:
            return [ring(*d)[0]]
        if w["cfg"] == 5:
            return [dc.scaled_dot_product_attention(d[0], k, v)]
        if w["bwd"]:
            tq, tk, tv = (t.requires_grad_(True) for t in d[:3])
            y = dc.scaled_dot_product_attention(tq, tk, tv, attn_mask=mask, is_causal=w["causal"],
                                                dropout_p=w.get("dropout", 0.0))
            y.backward(d[3])
            res = [y.detach(), tq.grad, tk.grad, tv.grad]
            for t in (tq, tk, tv):
                t.grad = None
                t.requires_grad_(False)
            return res
        return [dc.scaled_dot_product_attention(*d[:3], attn_mask=mask, is_causal=w["causal"])]

    def step(i):
        sl = i % nslot
        if used[sl]:
            # The host stays at most nslot steps ahead, as a loop that reads its results back
            # does: the slot's previous results are on the host before its buffers are reused
            # (an event wait, not a device synchronisation: the other slot's step keeps the
            # copy engines and the GPU busy meanwhile).
            ev_out[sl].synchronize()
        with torch.cuda.stream(s_h2d):
            if used[sl]:
                s_h2d.wait_event(ev_used[sl])  # the slot's previous compute read its inputs
            for h, d in zip(host_in[sl], dev_in[sl]):
                d.copy_(h, non_blocking=True)
            ev_in[sl].record(s_h2d)
        with torch.cuda.stream(s_comp):
            s_comp.wait_event(ev_in[sl])
            res = compute(dev_in[sl])
            ev_used[sl].record(s_comp)
        with torch.cuda.stream(s_d2h):
            if used[sl]:
                s_d2h.wait_event(ev_out[sl])
            s_d2h.wait_event(ev_used[sl])
            for h, r in zip(host_out[sl], res):
                r.record_stream(s_d2h)  # the allocator keeps r until the copy is done
                h.copy_(r, non_blocking=True)
            ev_out[sl].record(s_d2h)
        used[sl] = True
        last_res[sl] = res

    # Results freed on the compute stream stay reserved until their copy stream is done with
    # them, so the caching allocator grows over the first pipelined steps; a cudaMalloc inside
    # the timed steps would stall the pipeline. With the host at most nslot steps ahead the
    # warm-up reaches its steady state; the allocations left inside the timed steps are
    # reported.
    warm = max(args.warmup, 12)
    for i in range(warm):
        step(i)
    torch.cuda.synchronize()
    if dist is not None:
        dist.barrier()
    allocs0 = torch.cuda.memory_stats(device).get("num_device_alloc", 0)
    cur = torch.cuda.current_stream(device)
    s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    s.record(cur)
    s_h2d.wait_event(s)
    for i in range(args.steps):
        step(warm + i)
    for sl in range(nslot):
        cur.wait_event(ev_out[sl])
    e.record(cur)
    torch.cuda.synchronize()
    allocs = torch.cuda.memory_stats(device).get("num_device_alloc", 0) - allocs0
    ms = s.elapsed_time(e) / args.steps
    copy_ms = copy_ceiling(host_in, dev_in, host_out, [[r for r in row] for row in last_res], args.steps, device,
                           dist)
    ms = _max_over_ranks(ms, dist, device)
    unit = "GB/s" if scale == 1e9 else "TFLOP/s"
    value = amount / (ms / 1e3) / scale
    ceiling = amount / (copy_ms / 1e3) / scale
    return {"value": value, "unit": unit, "ms_per_step": ms, "h2d_bytes_per_step": sum(t.numel() * 4 for t in host_in[0]),
            "d2h_bytes_per_step": sum(t.numel() * 4 for t in host_out[0]), "pipelined": True,
            "warmup_steps": warm, "device_allocs_in_timed_steps": allocs,
            "copy_ceiling": {"ms_per_step": copy_ms, "value": ceiling, "frac": value / ceiling,
                             "what": "the same per-step H2D and D2H copies through the same pinned buffers, "
                                     "streams and slots with no compute (max over ranks): the host link's "
                                     "bound on e2e"}}


def copy_ceiling(host_in, dev_in, host_out, dev_out, steps, device, dist):
    """ms per step of the e2e loop's copies alone: each step's inputs up on one stream and the
    previous step's results down on another, three slots, no compute; max over ranks."""
    nslot = len(host_in)
    s_h2d, s_d2h = torch.cuda.Stream(device), torch.cuda.Stream(device)
    ev_in = [torch.cuda.Event() for _ in range(nslot)]
    ev_out = [torch.cuda.Event() for _ in range(nslot)]
    used = [False] * nslot

    def step(i):
        sl = i % nslot
        if used[sl]:
            ev_out[sl].synchronize()
        with torch.cuda.stream(s_h2d):
            for h, d in zip(host_in[sl], dev_in[sl]):
                d.copy_(h, non_blocking=True)
            ev_in[sl].record(s_h2d)
        with torch.cuda.stream(s_d2h):
            s_d2h.wait_event(ev_in[sl])
            for h, r in zip(host_out[sl], dev_out[sl]):
                h.copy_(r, non_blocking=True)
            ev_out[sl].record(s_d2h)
        used[sl] = True

    for i in range(2 * nslot):
        step(i)
    torch.cuda.synchronize()
    if dist is not None:
        dist.barrier()
    cur = torch.cuda.current_stream(device)
    s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    s.record(cur)
    s_h2d.wait_event(s)
    for i in range(steps):
        step(2 * nslot + i)
    for sl in range(nslot):
        cur.wait_event(ev_out[sl])
    e.record(cur)
    torch.cuda.synchronize()
    return _max_over_ranks(s.elapsed_time(e) / steps, dist, device)

if __name__ == "__main__":
    main()
