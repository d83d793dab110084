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
        R, heads = 4096, threads
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
    line = {"impl": "reference", "metric": METRIC, "value": value, "unit": unit, "n_gpus": world,
            "steps": args.steps, "warmup": args.warmup, "higher_is_better": True, "scaling": "weak",
            "vs_baseline": None, "dtype": "f32", "data": "synthetic",
            "config": {"workload": name, "shape_q": list(w["q"]), "shape_kv": list(w["kv"]),
                       "causal": w["causal"], "mask": w["mask"], "dropout_p": w.get("dropout", 0.0),
                       "baseline_cfg": w["cfg"]},
            "cpu_baseline": cb,
            "e2e": {"value": value, "unit": unit, "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}
    print(json.dumps(line), flush=True)


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
    from densecore_b200 import _lib, _native

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
    # sequence: strong scaling); every other run gives each rank a whole workload (weak scaling).
    ring = None
    if w["cfg"] == 4 and world > 1:
        from densecore_b200.ring import RingAttention, zigzag_shard
        full = make_inputs(w, device, seed=1234)
        q, k, v = (zigzag_shard(t, rank, world) for t in full[:3])
        g, mask = None, None
        del full
        ring = RingAttention(q.shape, k.shape, device, causal=True)
    else:
        q, k, v, g, mask = make_inputs(w, device, seed=1234 + rank)
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
        dc.manual_seed(1234 + rank)

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
    for _ in range(args.warmup):
        step()
    torch.cuda.synchronize()
    # The timed forward + backward steps replay a CUDA graph of one step (every kernel of the
    # step is launched by each replay): small workloads would otherwise wait on the host's
    # launches. Dropout (its generator state and temporary copies), decode and the ring (NCCL)
    # run eagerly.
    timed_step = step
    launch = "eager"
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

    def barrier():
        if dist is not None:
            dist.barrier()
        torch.cuda.synchronize()

    starts = [torch.cuda.Event(enable_timing=True) for _ in range(args.steps)]
    ends = [torch.cuda.Event(enable_timing=True) for _ in range(args.steps)]
    barrier()
    with ClockSampler(physical_gpu(local)) as clocks:
        for i in range(args.steps):
            flush.zero_()
            starts[i].record()
            timed_step()
            ends[i].record()
        torch.cuda.synchronize()
    barrier()
    ms = sum(s.elapsed_time(e) for s, e in zip(starts, ends)) / args.steps
    # The per-kernel breakdown (and the roofline's kernel durations) comes from a second pass
    # of the same steps with the library's tracing on: it records two CUDA events around every
    # launch, host work that would otherwise sit inside the timed steps of small workloads.
    _lib.kernel_timing_report(reset=True)
    _lib.kernel_timing(True)
    for i in range(args.steps):
        flush.zero_()
        step()
    torch.cuda.synchronize()
    _lib.kernel_timing(False)
    barrier()
    kernels = _lib.kernel_timing_report(reset=True)
    ms_max = ms
    if dist is not None:
        t = torch.tensor([ms], device=device, dtype=torch.float64)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        ms_max = float(t.item())
    amount, unit = work(w)
    scale = 1e9 if unit == "GB/s" else 1e12
    ranks_work = 1 if ring is not None else world  # strong scaling: the ranks share one workload
    value = ranks_work * amount / (ms_max / 1e3) / scale

    # Roofline of the dominant kernel (largest total device time in the timed region). The
    # tensor-core backward's dK/dV and dQ kernels share the GPU (two streams): their joint
    # record "bwd_tc" is the unit, not either kernel alone.
    pk = peaks()
    # Kernels without a roofline of their own (the dropout mask draw: integer generator work,
    # neither HBM- nor tensor-bound) are named in "slowest_kernel" but are not the unit.
    concurrent = ("bwd_dkdv_tc", "bwd_dq_tc") if "bwd_tc" in kernels else ()
    candidates = {k_: v_ for k_, v_ in kernels.items() if k_ not in concurrent}
    slowest = max(candidates.items(), key=lambda kv: kv[1][1])[0] if candidates else None
    candidates = {k_: v_ for k_, v_ in candidates.items() if kernel_work(w, k_) > 0 or ring is not None}
    dom = max(candidates.items(), key=lambda kv: kv[1][1]) if candidates else None
    roofline = None
    if dom is not None:
        kname, (launches, total_ms) = dom
        per_launch = kernel_work(w, kname)
        avg_ms = total_ms / max(launches, 1)
        if ring is not None:
            # Ring launches differ in size; per step the rank's forward launches together do
            # 1/world of the sequence's algorithmic flops.
            per_launch = amount / world / (launches / args.steps)
        if unit == "GB/s":
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
        roofline = {"kernel": kname, "slowest_kernel": slowest, "bound": bound, "achieved": achieved, "peak": peak,
                    "unit": ru,
                    "frac": achieved / peak, "traffic": traffic, "avg_launch_ms": avg_ms,
                    "peak_source": (f"{pk['src']} hbm_gbs" if bound == "hbm"
                                    else f"{pk['src']} bf16_tflops / 2 (dense TF32 rate)")}
    launches = sum(v[0] for k_, v in kernels.items() if k_ != "bwd_tc")  # bwd_tc spans two launches

    # End to end through the public API with pinned host buffers; copies in the timed region.
    e2e = None
    if not args.no_e2e:
        e2e = run_e2e(w, q, k, v, g, mask, args, device, scale, amount, dist, ring)

    cb = None
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        cb = cpu_baseline(w, name)

    if rank == 0:
        line = {"metric": METRIC, "value": value, "unit": unit, "n_gpus": world, "steps": args.steps,
                "warmup": args.warmup, "ms_per_step": ms_max, "higher_is_better": True,
                "scaling": "strong" if ring is not None else "weak",
                "vs_baseline": None, "dtype": "f32" if args.precision == "fp32" else args.precision,
                "data": "synthetic (seeded N(0,1) of the config's shape)",
                "config": {"workload": name, "baseline_cfg": w["cfg"], "shape_q": list(w["q"]),
                           "shape_kv": list(w["kv"]), "causal": causal, "mask": w["mask"],
                           "dropout_p": w.get("dropout", 0.0),
                           "per_rank": ("zig-zag sequence shard (ring attention, NCCL send/recv)"
                                        if ring is not None else "full workload (weak scaling)"),
                           "parallelism": f"ring{world}" if ring is not None else f"dp{world}",
                           "precision": args.precision, "l2": "flushed (256 MB write) before every timed step",
                           "launch": launch,
                           "kernel_breakdown": "a second, untimed pass of the same steps with per-launch tracing"},
                "roofline": roofline, "kernels": {k_: {"launches": v_[0], "total_ms": v_[1]}
                                                  for k_, v_ in kernels.items()},
                "gpu_launches": launches, "e2e": e2e, "cpu_baseline": cb, "clocks": clocks.summary()}
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
    world = 1
    if dist is not None:
        world = dist.get_world_size()
        t = torch.tensor([ms], device=device, dtype=torch.float64)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        ms = float(t.item())
    if ring is not None:
        world = 1  # the ranks share one sequence
    return {"value": world * amount / (ms / 1e3) / scale, "unit": "GB/s" if scale == 1e9 else "TFLOP/s",
            "ms_per_step": ms, "h2d_bytes_per_step": sum(t.numel() * 4 for t in host_in[0]),
            "d2h_bytes_per_step": sum(t.numel() * 4 for t in host_out[0]), "pipelined": True,
            "warmup_steps": warm, "device_allocs_in_timed_steps": allocs}


if __name__ == "__main__":
    main()
