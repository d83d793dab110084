"""dc_sdpa_decode_noalloc: split-KV decode with its partials in the library's static device
scratch instead of a workspace. Called through the C ABI and compared with dc_sdpa_decode
(the workspace entry point) on the same inputs and split count.

Tolerance: the two entry points run the same kernels on the same split count, so their
results should agree bit for bit; the test allows max|delta| <= 1e-6 * max|ref|. The file is
named to be collected last, so the scratch is exercised both alone and after every other
GPU test in the same process.
"""
import ctypes

import numpy as np
import pytest
import torch

from densecore_b200 import _lib, _native
from conftest import rel_err

pytestmark = pytest.mark.gpu

DEV = "cuda:0"
TOL = 1e-6
SCRATCH_BYTES = 8 << 20  # DC_DECODE_NOALLOC_SCRATCH_BYTES


def _inputs(seed, B, H, Hkv, S, D):
    g = torch.Generator().manual_seed(seed)
    q = torch.randn(B, H, 1, D, generator=g).to(DEV)
    k = torch.randn(B, Hkv, S, D, generator=g).to(DEV)
    v = torch.randn(B, Hkv, S, D, generator=g).to(DEV)
    return q, k, v


def _noalloc(q, k, v, mask=None, num_splits=0, scale=None, out=None, lse=None):
    L = _lib.load()
    B, H = q.shape[:2]
    if out is None:
        out = torch.empty(B, H, 1, v.shape[3], device=DEV)
    if lse is None:
        lse = torch.empty(B, H, 1, device=DEV)
    views = [_lib.view(t) for t in (q, k, v, mask, out, lse)]
    has, sc = (0, 0.0) if scale is None else (1, float(scale))
    st = L.dc_sdpa_decode_noalloc(*[_lib.ref(x) for x in views[:4]], has, sc, num_splits,
                                  _lib.ref(views[4]), _lib.ref(views[5]), _lib.stream_of(q))
    return st, out, lse


def _splits(q, k, num_splits):
    if num_splits > 0:
        return num_splits
    return _lib.load().dc_sdpa_decode_default_splits(q.shape[0], q.shape[1], k.shape[2])


CASES = [
    # B, H, Hkv, S, D, num_splits, masked
    (2, 8, 2, 1000, 64, 0, False),
    (1, 32, 8, 16384, 128, 0, False),
    (4, 4, 4, 777, 128, 5, True),
    (3, 2, 1, 4096, 64, 64, False),
]


@pytest.mark.parametrize("case", CASES, ids=[f"B{c[0]}H{c[1]}kv{c[2]}S{c[3]}D{c[4]}sp{c[5]}m{int(c[6])}" for c in CASES])
def test_noalloc_matches_workspace_decode_twice(case):
    B, H, Hkv, S, D, num_splits, masked = case
    q, k, v = _inputs(1000 + S, B, H, Hkv, S, D)
    mask = None
    if masked:
        m = torch.rand(B, 1, 1, S, generator=torch.Generator().manual_seed(S)) > 0.3
        m[0, :, :, :] = False  # one batch fully masked: out 0, lse 0
        mask = m.to(DEV)
    splits = _splits(q, k, num_splits)
    ref_out, ref_lse = _native._decode(q, k, v, mask=mask, num_splits=splits)
    for call in range(2):  # two calls in a row reuse the same scratch
        st, out, lse = _noalloc(q, k, v, mask=mask, num_splits=num_splits)
        torch.cuda.synchronize()
        assert st == _lib.DC_OK, _lib.load().dc_last_error()
        assert _lib.load().dc_device_status(0) == 0
        assert rel_err(out.cpu().numpy(), ref_out.cpu().numpy()) <= TOL, f"out, call {call}"
        assert rel_err(lse.cpu().numpy(), ref_lse.cpu().numpy()) <= TOL, f"lse, call {call}"
    if masked:
        assert torch.all(out[0] == 0) and torch.all(lse[0] == 0)


def test_noalloc_back_to_back_different_shapes():
    """Two different problems back to back on one stream: the second must not see the
    first one's partials."""
    a = _inputs(7, 2, 4, 4, 3000, 128)
    b = _inputs(8, 1, 2, 2, 300, 64)
    ra = _native._decode(*a, num_splits=9)
    rb = _native._decode(*b, num_splits=3)
    st_a, oa, la = _noalloc(*a, num_splits=9)
    st_b, ob, lb = _noalloc(*b, num_splits=3)
    torch.cuda.synchronize()
    assert st_a == _lib.DC_OK and st_b == _lib.DC_OK
    for got, ref in ((oa, ra[0]), (la, ra[1]), (ob, rb[0]), (lb, rb[1])):
        assert rel_err(got.cpu().numpy(), ref.cpu().numpy()) <= TOL


def test_noalloc_rejects_oversized_request_without_launching():
    # 64*32 rows * 8 splits * (128 + 2) floats * 4 bytes = 8.5 MB > 8 MiB.
    B, H, S, D = 64, 32, 16, 128
    q, k, v = _inputs(9, B, H, H, S, D)
    need = _lib.load().dc_sdpa_decode_workspace_size(B, H, D, 8)
    assert need > SCRATCH_BYTES
    out = torch.full((B, H, 1, D), float("nan"), device=DEV)
    lse = torch.full((B, H, 1), float("nan"), device=DEV)
    st, out, lse = _noalloc(q, k, v, num_splits=8, out=out, lse=lse)
    torch.cuda.synchronize()
    assert st == _lib.DC_ERR_VALUE
    msg = _lib.load().dc_last_error().decode()
    assert "scratch" in msg and str(need) in msg
    assert torch.isnan(out).all() and torch.isnan(lse).all()  # nothing was written
    # One split fits (64*32*130*4 = 1.06 MB) and runs.
    st, out, lse = _noalloc(q, k, v, num_splits=1)
    torch.cuda.synchronize()
    assert st == _lib.DC_OK
    ref = _native._decode(q, k, v, num_splits=1)
    assert rel_err(out.cpu().numpy(), ref[0].cpu().numpy()) <= TOL


def _pool_high_water():
    """(reset, read) of the current device memory pool's used-memory high watermark, the pool
    cudaMallocAsync draws from; None when cuda-python cannot reach it."""
    try:
        from cuda.bindings import driver as cu
        from cuda.bindings import runtime as rt
    except ImportError:
        return None
    err, pool = rt.cudaDeviceGetMemPool(torch.cuda.current_device())
    if err != rt.cudaError_t.cudaSuccess:
        return None
    attr = rt.cudaMemPoolAttr.cudaMemPoolAttrUsedMemHigh

    def reset():
        (e,) = rt.cudaMemPoolSetAttribute(pool, attr, cu.cuuint64_t(0))
        return e == rt.cudaError_t.cudaSuccess

    def read():
        e, val = rt.cudaMemPoolGetAttribute(pool, attr)
        return int(val) if e == rt.cudaError_t.cudaSuccess else None

    return reset, read


def test_noalloc_draws_nothing_from_the_stream_ordered_pool():
    hw = _pool_high_water()
    if hw is None:
        pytest.skip("cuda-python cannot read the memory pool")
    reset, read = hw
    q, k, v = _inputs(11, 2, 8, 8, 2048, 128)
    B, H = q.shape[:2]
    L = _lib.load()
    # Control: dc_sdpa_decode without a workspace takes its scratch from that pool.
    out = torch.empty(B, H, 1, 128, device=DEV)
    lse = torch.empty(B, H, 1, device=DEV)
    torch.cuda.synchronize()
    if not reset():
        pytest.skip("cannot reset the pool's watermark")
    views = [_lib.view(t) for t in (q, k, v, None, out, lse)]
    st = L.dc_sdpa_decode(*[_lib.ref(x) for x in views[:4]], 0, 0.0, 4, _lib.ref(views[4]),
                          _lib.ref(views[5]), None, 0, _lib.stream_of(q))
    torch.cuda.synchronize()
    assert st == _lib.DC_OK
    control = read()
    if not control:
        pytest.skip("the pool's watermark does not register stream-ordered allocations")
    assert reset()
    st, out2, lse2 = _noalloc(q, k, v, num_splits=4)
    torch.cuda.synchronize()
    assert st == _lib.DC_OK
    assert read() == 0
    assert rel_err(out2.cpu().numpy(), out.cpu().numpy()) <= TOL
