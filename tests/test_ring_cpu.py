"""Ring attention's host logic on CPU: gloo ranks (world size 2 and 4) run the zig-zag ring with
the CPU oracle standing in for the attention kernel and a torch logsumexp merge standing in for
dc_attn_merge. The reassembled output must equal the oracle's forward over the whole sequence
(src/torch_attention.rs:146-284) within 1e-5 * max|ref| (the partials are merged in another
order than one pass accumulates them)."""
import os
import socket

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from conftest import rel_err


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _oracle_attn(q, k, v, causal):
    import oracle
    out, lse = oracle.flash_forward(*(t.contiguous().numpy() for t in (q, k, v)), causal=causal)
    return torch.from_numpy(out), torch.from_numpy(lse)


def _torch_merge(out_acc, lse_acc, out_part, lse_part):
    lse_new = torch.logaddexp(lse_acc, lse_part)
    wa = torch.exp(lse_acc - lse_new).unsqueeze(-1)
    wp = torch.exp(lse_part - lse_new).unsqueeze(-1)
    out_acc.copy_(out_acc * wa + out_part * wp)
    lse_acc.copy_(lse_new)


def _inputs(shape, seed):
    rng = np.random.default_rng(seed)
    return [torch.from_numpy(rng.normal(size=shape).astype(np.float32) * 0.5) for _ in range(3)]


def _worker(rank, world, port, shape, causal, result_dir):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        from densecore_b200.ring import RingAttention, zigzag_shard
        q, k, v = (zigzag_shard(t, rank, world) for t in _inputs(shape, 5))
        ring = RingAttention(q.shape, k.shape, "cpu", causal=causal, attn_fn=_oracle_attn,
                             merge_fn=_torch_merge)
        for call in range(2):  # the exchange buffers are reused by a second call
            out, lse = ring(q, k, v)
        torch.save({"out": out, "lse": lse}, os.path.join(result_dir, f"r{rank}.pt"))
        dist.barrier()
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("world,causal", [(2, True), (4, True), (2, False)])
def test_ring_matches_full_sequence_oracle(world, causal, tmp_path):
    import oracle
    from densecore_b200.ring import zigzag_unshard
    shape = (1, 2, 64 * world, 64)
    mp.start_processes(_worker, args=(world, _free_port(), shape, causal, str(tmp_path)), nprocs=world,
                       join=True, start_method="spawn")
    parts = [torch.load(tmp_path / f"r{r}.pt") for r in range(world)]
    out = zigzag_unshard([p["out"] for p in parts]).numpy()
    lse = zigzag_unshard([p["lse"] for p in parts]).numpy()
    q, k, v = (t.numpy() for t in _inputs(shape, 5))
    ref_out, ref_lse = oracle.flash_forward(q, k, v, causal=causal)
    assert rel_err(out, ref_out) <= 1e-5
    assert rel_err(lse, ref_lse) <= 1e-5


def test_zigzag_round_trip_and_balance():
    from densecore_b200.ring import zigzag_indices, zigzag_shard, zigzag_unshard
    x = torch.arange(2 * 3 * 48 * 4, dtype=torch.float32).view(2, 3, 48, 4)
    for world in (1, 2, 3, 4):
        shards = [zigzag_shard(x, r, world) for r in range(world)]
        assert torch.equal(zigzag_unshard(shards), x)
    # Causal work per rank is equal: chunk r and 2P-1-r together see 2P+1 chunk-rows of keys.
    P, C = 4, 12
    work = []
    for r in range(P):
        a, b = zigzag_indices(2 * P * C, r, P)
        work.append(sum(i + 1 for i in range(a.start, a.stop)) + sum(i + 1 for i in range(b.start, b.stop)))
    assert len(set(work)) == 1
    with pytest.raises(ValueError):
        zigzag_indices(50, 0, 4)


def _peer_worker(rank, world, port, mode, timeout_s, result_dir):
    """Rank 1 either joins the ring late (inside the process group's timeout) or never joins
    (it sleeps past the timeout and leaves). Rank 0 records how its ring call ended."""
    import datetime
    import json
    import time
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=timeout_s))
    try:
        from densecore_b200.ring import RingAttention, zigzag_shard
        shape = (1, 2, 64 * world, 64)
        q, k, v = (zigzag_shard(t, rank, world) for t in _inputs(shape, 6))
        ring = RingAttention(q.shape, k.shape, "cpu", causal=True, attn_fn=_oracle_attn, merge_fn=_torch_merge)
        if rank == 1:
            time.sleep(timeout_s * (0.3 if mode == "late" else 2.0))
            if mode == "absent":
                return  # leaves without taking part; rank 0's receive can never complete
        t0 = time.monotonic()
        try:
            out, lse = ring(q, k, v)
            res = {"ok": True, "s": time.monotonic() - t0}
            torch.save({"out": out, "lse": lse}, os.path.join(result_dir, f"r{rank}.pt"))
        except Exception as e:  # the outcome under test: the host-side timeout raises
            res = {"ok": False, "type": type(e).__name__, "msg": str(e)[:300], "s": time.monotonic() - t0}
        with open(os.path.join(result_dir, f"r{rank}.json"), "w") as f:
            json.dump(res, f)
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("mode", ["late", "absent"])
def test_ring_peer_late_or_absent(mode, tmp_path):
    """A ring peer that arrives late (within the process group's timeout) only delays the
    result; a peer that never takes part makes the waiting rank's ring call raise once the
    timeout runs out, instead of hanging."""
    import json
    import oracle
    from densecore_b200.ring import zigzag_unshard
    world, timeout_s = 2, 3
    mp.start_processes(_peer_worker, args=(world, _free_port(), mode, timeout_s, str(tmp_path)), nprocs=world,
                       join=True, start_method="spawn")
    r0 = json.loads((tmp_path / "r0.json").read_text())
    if mode == "absent":
        assert not r0["ok"], "rank 0's ring call should fail when its peer never takes part"
        assert r0["type"] in ("RuntimeError", "DistBackendError"), r0
        assert r0["s"] < 10 * timeout_s, r0
        return
    assert r0["ok"], r0
    parts = [torch.load(tmp_path / f"r{r}.pt") for r in range(world)]
    out = zigzag_unshard([p["out"] for p in parts]).numpy()
    q, k, v = (t.numpy() for t in _inputs((1, 2, 64 * world, 64), 6))
    ref_out, _ = oracle.flash_forward(q, k, v, causal=True)
    assert rel_err(out, ref_out) <= 1e-5
