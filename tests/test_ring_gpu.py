"""Ring attention on the GPU kernels.

- One GPU: every rank of a P-rank ring emulated in one process (the same steps and
  logsumexp merges, no exchange) against the single-call forward and the CPU oracle.
- Two GPUs (skipped with fewer): real ranks over NCCL send/recv, against the single-call
  forward on one device.

Tolerance: 1e-5 * max|ref| (3xTF32), as for the forward itself.
"""
import os
import socket

import numpy as np
import pytest
import torch
import torch.multiprocessing as mp

import densecore_b200 as dc
import oracle
from conftest import rel_err

pytestmark = pytest.mark.gpu
DEV = "cuda:0"


def _inputs(shape, seed, amp=0.5, device=DEV):
    g = torch.Generator().manual_seed(seed)
    return [(torch.randn(shape, generator=g) * amp).to(device) for _ in range(3)]


@pytest.mark.parametrize("world,causal,D", [(4, True, 128), (2, True, 64), (3, False, 128), (8, True, 128)])
def test_ring_emulated_matches_single_forward(world, causal, D):
    from densecore_b200.ring import ring_emulate
    q, k, v = _inputs((1, 4, 512 * world, D), seed=world)
    out, lse = ring_emulate(q, k, v, world, causal=causal)
    ref_out, ref_lse = dc._flash_attention(q, k, v, causal)
    torch.cuda.synchronize()
    assert dc._lib.load().dc_device_status(0) == 0
    assert rel_err(out.cpu().numpy(), ref_out.cpu().numpy()) <= 1e-5
    assert rel_err(lse.cpu().numpy(), ref_lse.cpu().numpy()) <= 1e-5


def test_ring_emulated_matches_oracle():
    from densecore_b200.ring import ring_emulate
    q, k, v = _inputs((1, 2, 1024, 64), seed=11)
    out, lse = ring_emulate(q, k, v, 4, causal=True)
    ref_out, ref_lse = oracle.flash_forward(*(t.cpu().numpy() for t in (q, k, v)), causal=True)
    assert rel_err(out.cpu().numpy(), ref_out) <= 1e-5
    assert rel_err(lse.cpu().numpy(), ref_lse) <= 1e-5


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _nccl_worker(rank, world, port, shape, result_dir):
    import datetime

    import torch.distributed as dist
    from densecore_b200.ring import RingAttention, zigzag_shard
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    torch.cuda.set_device(rank)
    dev = torch.device("cuda", rank)
    dist.init_process_group("nccl", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=60),
                            device_id=dev)
    try:
        q, k, v = (zigzag_shard(t, rank, world) for t in _inputs(shape, seed=3, device=dev))
        ring = RingAttention(q.shape, k.shape, dev, causal=True)
        for _ in range(2):
            out, lse = ring(q, k, v)
        torch.cuda.synchronize()
        torch.save({"out": out.cpu(), "lse": lse.cpu(), "status": dc._lib.load().dc_device_status(0)},
                   os.path.join(result_dir, f"r{rank}.pt"))
        dist.barrier()
    finally:
        dist.destroy_process_group()


@pytest.mark.skipif(not torch.cuda.is_available() or torch.cuda.device_count() < 2,
                    reason="needs two GPUs")
def test_ring_over_nccl_two_gpus(tmp_path):
    from densecore_b200.ring import zigzag_unshard
    world, shape = 2, (1, 4, 4096, 128)
    mp.start_processes(_nccl_worker, args=(world, _free_port(), shape, str(tmp_path)), nprocs=world,
                       join=True, start_method="spawn")
    parts = [torch.load(tmp_path / f"r{r}.pt") for r in range(world)]
    assert all(p["status"] == 0 for p in parts)
    out = zigzag_unshard([p["out"] for p in parts]).numpy()
    lse = zigzag_unshard([p["lse"] for p in parts]).numpy()
    q, k, v = _inputs(shape, seed=3)
    ref_out, ref_lse = dc._flash_attention(q, k, v, True)
    assert rel_err(out, ref_out.cpu().numpy()) <= 1e-5
    assert rel_err(lse, ref_lse.cpu().numpy()) <= 1e-5


def _native_worker(rank, world, port, shape, causal, result_dir):
    import datetime

    import torch.distributed as dist
    from densecore_b200.ring import NativeRingAttention, NcclCommunicator, zigzag_shard
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    torch.cuda.set_device(rank)
    dev = torch.device("cuda", rank)
    dist.init_process_group("nccl", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=60),
                            device_id=dev)
    comm = None
    try:
        comm = NcclCommunicator(device=dev)
        q, k, v = (zigzag_shard(t, rank, world) for t in _inputs(shape, seed=4, device=dev))
        ring = NativeRingAttention(q.shape, k.shape, dev, comm, causal=causal)
        for _ in range(2):  # the workspace and the side stream are reused by a second call
            out, lse = ring(q, k, v)
        torch.cuda.synchronize()
        torch.save({"out": out.cpu(), "lse": lse.cpu(), "status": dc._lib.load().dc_device_status(0)},
                   os.path.join(result_dir, f"r{rank}.pt"))
        dist.barrier()
    finally:
        if comm is not None:
            comm.destroy()
        dist.destroy_process_group()


@pytest.mark.skipif(not torch.cuda.is_available() or torch.cuda.device_count() < 2,
                    reason="needs two GPUs")
@pytest.mark.parametrize("causal", [True, False])
def test_c_abi_ring_over_nccl_two_gpus(causal, tmp_path):
    # dc_ring_sdpa_fwd with a communicator made through libnccl's C API (what a C or Rust host
    # passes): every rank's rows equal the single-call forward over the whole sequence.
    from densecore_b200.ring import zigzag_unshard
    world, shape = 2, (1, 4, 4096, 128)
    mp.start_processes(_native_worker, args=(world, _free_port(), shape, causal, str(tmp_path)), nprocs=world,
                       join=True, start_method="spawn")
    parts = [torch.load(tmp_path / f"r{r}.pt") for r in range(world)]
    assert all(p["status"] == 0 for p in parts)
    out = zigzag_unshard([p["out"] for p in parts]).numpy()
    lse = zigzag_unshard([p["lse"] for p in parts]).numpy()
    q, k, v = _inputs(shape, seed=4)
    ref_out, ref_lse = dc._flash_attention(q, k, v, causal)
    assert rel_err(out, ref_out.cpu().numpy()) <= 1e-5
    assert rel_err(lse, ref_lse.cpu().numpy()) <= 1e-5


def test_c_abi_ring_one_rank_communicator_equals_forward():
    # A one-rank communicator: dc_ring_sdpa_fwd is then the local causal forward (step 0 only).
    from densecore_b200.ring import NativeRingAttention, NcclCommunicator
    q, k, v = _inputs((2, 4, 1024, 64), seed=5)
    comm = NcclCommunicator(device=torch.device(DEV))
    try:
        out, lse = NativeRingAttention(q.shape, k.shape, q.device, comm)(q, k, v)
        ref_out, ref_lse = dc._flash_attention(q, k, v, True)
        torch.cuda.synchronize()
        assert torch.equal(out, ref_out) and torch.equal(lse, ref_lse)
    finally:
        comm.destroy()
