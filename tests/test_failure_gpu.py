"""Failure detection on the GPU, in the forms that leave the device usable.

The tensor-core kernels wait on mbarriers with a bound; a wait that runs out records
DEV_WAIT_TIMEOUT (1) in the library's device status word and its CTA frees its tensor memory and
returns. ``dc_debug_wait_probe`` runs that same bounded wait on a barrier nothing arrives at,
with the bound shortened to microseconds. These tests check that the wait gives up no earlier
than its bound, that the call returns and the status reads 1 (and clears), and that the next
normal call -- which allocates every TMEM column of an SM -- is clean and matches the oracle.
The reference's analogue is its kernels' error slots (torch_attention.rs:163, :274-276) raised
as RuntimeError (lib.rs:633, :677).
"""
import ctypes

import numpy as np
import pytest
import torch

import densecore_b200 as dc
import oracle
from conftest import rel_err

pytestmark = pytest.mark.gpu

DEV = "cuda:0"


def _probe(timeout_ns, blocks):
    L = dc._lib.load()
    s = torch.cuda.current_stream(torch.device(DEV))
    t0, t1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    t0.record(s)
    st = L.dc_debug_wait_probe(ctypes.c_uint64(timeout_ns), blocks, ctypes.c_void_p(s.cuda_stream))
    t1.record(s)
    dc._lib.check(st, "wait probe")
    torch.cuda.synchronize()
    return t0.elapsed_time(t1)


def _normal_call_matches_oracle():
    rng = np.random.default_rng(40)
    q, k, v, g = (rng.normal(size=(2, 4, 384, 64)).astype(np.float32) for _ in range(4))
    tq, tk, tv = (torch.from_numpy(a).to(DEV).requires_grad_(True) for a in (q, k, v))
    y = dc.scaled_dot_product_attention(tq, tk, tv, is_causal=True)
    y.backward(torch.from_numpy(g).to(DEV))
    torch.cuda.synchronize()
    out, lse = oracle.flash_forward(q, k, v, causal=True)
    refs = [out, *oracle.flash_backward(g, q, k, v, out, lse, causal=True)]
    for name, a, r in zip(("out", "dq", "dk", "dv"), (y, tq.grad, tk.grad, tv.grad), refs):
        err = rel_err(a.detach().cpu().numpy(), r)
        assert err <= 1e-5, f"{name} after the probe: {err:.2e}"


@pytest.mark.parametrize("timeout_us,blocks", [(20, 1), (200, 296), (5000, 1024)])
def test_bounded_wait_gives_up_and_the_next_call_is_clean(timeout_us, blocks):
    L = dc._lib.load()
    L.dc_device_status(1)
    assert L.dc_device_status(0) == 0
    ms = _probe(timeout_us * 1000, blocks)
    # Each CTA waited at least its bound before giving up (the last wave ends no earlier).
    assert ms >= timeout_us / 1000.0 * 0.999, f"the wait gave up after {ms:.4f} ms, bound {timeout_us} us"
    assert L.dc_device_status(0) == 1  # DEV_WAIT_TIMEOUT
    assert L.dc_device_status(1) == 1
    assert L.dc_device_status(0) == 0  # cleared
    _normal_call_matches_oracle()
    assert L.dc_device_status(0) == 0


def test_probe_arguments_are_checked():
    L = dc._lib.load()
    s = ctypes.c_void_p(torch.cuda.current_stream(torch.device(DEV)).cuda_stream)
    for timeout, blocks in ((999, 1), (2_000_000_000, 1), (10_000, 0), (10_000, 1025)):
        assert L.dc_debug_wait_probe(ctypes.c_uint64(timeout), blocks, s) == dc._lib.DC_ERR_VALUE
    assert L.dc_device_status(0) == 0
