"""The C-ABI library on a machine without a GPU: it loads, exports every symbol the header
declares, and its validation (which runs before any CUDA call) maps to the reference's
exception types (src/lib.rs:562-570, :601-605, :658-662). No compute call is made here."""
import ctypes
import os
import re

import pytest
import torch

from densecore_b200 import _lib

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def _declared():
    names = set()
    for fn in os.listdir(os.path.join(ROOT, "include")):
        if fn.endswith(".h"):
            text = open(os.path.join(ROOT, "include", fn)).read()
            names |= set(re.findall(r"DC_API\s+[\w\s\*]+?\b(dc_\w+)\s*\(", text))
    return names


def test_library_exports_every_declared_symbol():
    L = _lib.load()
    declared = _declared()
    assert declared, "no declarations found"
    assert declared == set(_lib.EXPORTS)
    for name in declared:
        assert hasattr(L, name), name
    assert L.dc_abi_version() == 1


def test_library_exports_nothing_undeclared():
    """Every exported dc_* symbol is declared in the header: nothing is exported that the header does not document."""
    import subprocess
    try:
        out = subprocess.run(["nm", "-D", "--defined-only", _lib.LIB_PATH], capture_output=True, text=True,
                             check=True).stdout
    except (OSError, subprocess.CalledProcessError):
        pytest.skip("nm is unavailable")
    exported = {line.split()[-1] for line in out.splitlines() if line.split() and line.split()[-1].startswith("dc_")}
    assert exported == _declared()


def _fake(shape, dtype=_lib.DC_F32, ptr=0x1000):
    v = _lib.DcTensor()
    v.data, v.dtype, v.ndim = ptr, dtype, len(shape)
    stride = 1
    for i in reversed(range(len(shape))):
        v.sizes[i] = shape[i]
        v.strides[i] = stride
        stride *= max(shape[i], 1)
    return v


def _fwd(q, k, v, mask=None, out=None, lse=None):
    L = _lib.load()
    B, H, Lq = q.sizes[0], q.sizes[1], q.sizes[2]
    out = out or _fake((B, H, Lq, v.sizes[3]))
    lse = lse or _fake((B, H, Lq))
    r = lambda x: None if x is None else ctypes.byref(x)
    return L.dc_sdpa_fwd(r(q), r(k), r(v), r(mask), 0, 0, 0.0, 0, r(out), r(lse), None)


def test_shape_errors_are_value_errors():
    L = _lib.load()
    st = _fwd(_fake((1, 3, 4, 8)), _fake((1, 2, 4, 8)), _fake((1, 2, 4, 8)))
    assert st == _lib.DC_ERR_VALUE and b"shapes do not match" in L.dc_last_error()
    st = _fwd(_fake((1, 2, 4, 8)), _fake((1, 2, 5, 8)), _fake((1, 2, 4, 8)))
    assert st == _lib.DC_ERR_VALUE
    st = _fwd(_fake((1, 2, 4, 8)), _fake((1, 2, 5, 8)), _fake((1, 2, 5, 8)), mask=_fake((3, 5), _lib.DC_BOOL))
    assert st == _lib.DC_ERR_VALUE and b"broadcast" in L.dc_last_error()
    st = _fwd(_fake((1, 2, 4, 8)), _fake((1, 2, 5, 8)), _fake((1, 2, 5, 8)), out=_fake((1, 2, 4, 7)))
    assert st == _lib.DC_ERR_VALUE
    q3 = _fake((2, 4, 8))
    st = _fwd(q3, q3, q3, out=_fake((2, 4, 8, 1)), lse=_fake((2, 4, 8)))
    assert st == _lib.DC_ERR_VALUE and b"(B, H, L, E)" in L.dc_last_error()
    with pytest.raises(ValueError, match="shapes do not match"):
        _lib.check(_fwd(_fake((1, 3, 4, 8)), _fake((1, 2, 4, 8)), _fake((1, 2, 4, 8))), "x")


def test_valid_call_without_device_is_a_cuda_error_not_a_fallback():
    if torch.cuda.is_available():
        pytest.skip("a device is present")
    st = _fwd(_fake((1, 2, 4, 8)), _fake((1, 2, 5, 8)), _fake((1, 2, 5, 8)), mask=_fake((4, 5), _lib.DC_BOOL))
    assert st == _lib.DC_ERR_CUDA
    with pytest.raises(RuntimeError):
        _lib.check(st, "forward")


def test_workspace_sizes():
    L = _lib.load()
    assert L.dc_sdpa_bwd_workspace_size(8, 12, 1024) >= 8 * 12 * 1024 * 4
    assert L.dc_sdpa_bwd_workspace_size(8, 12, 1024) % 256 == 0
    assert L.dc_sdpa_decode_workspace_size(64, 32, 128, 3) == 64 * 32 * 3 * 130 * 4
    assert L.dc_sdpa_decode_workspace_size(0, 32, 128, 3) == 0


def test_cpu_tensors_are_refused_loudly():
    import densecore_b200 as dc
    q = torch.zeros(1, 2, 4, 8)
    with pytest.raises(RuntimeError, match="CUDA"):
        dc.scaled_dot_product_attention(q, q, q)


def test_ring_entry_validates_before_any_device_work():
    L = _lib.load()
    q, k, v = _fake((1, 2, 64, 64)), _fake((1, 2, 64, 64)), _fake((1, 2, 64, 64))
    out, lse = _fake((1, 2, 64, 64)), _fake((1, 2, 64))
    need = L.dc_ring_sdpa_fwd_workspace_size(1, 2, 2, 64, 64)
    assert need == ((2 * 2 * 2 * 64 * 64 + 2 * 64 * 65) * 4 + 255) // 256 * 256
    ws = 0x100000

    def call(q_=q, k_=k, comm=0x2000, nbytes=need, wsp=ws):
        return L.dc_ring_sdpa_fwd(ctypes.byref(q_), ctypes.byref(k_), ctypes.byref(v), 1, 0, 0.0, 0, comm,
                                  ctypes.byref(out), ctypes.byref(lse), wsp, nbytes, None)

    assert call(comm=None) == _lib.DC_ERR_VALUE                # no communicator
    assert call(nbytes=need - 1) == _lib.DC_ERR_VALUE          # workspace too small
    assert call(wsp=ws + 16) == _lib.DC_ERR_VALUE              # workspace not 256-byte aligned
    odd = _fake((1, 2, 63, 64))
    assert call(q_=odd, k_=odd) == _lib.DC_ERR_VALUE           # local length must be even
    strided = _fake((1, 2, 64, 64))
    strided.strides[2] = 128                                    # k not contiguous
    assert call(k_=strided) == _lib.DC_ERR_VALUE
    assert b"contiguous" in L.dc_last_error()


def test_batch_or_heads_beyond_grid_limits_are_refused_before_any_launch():
    """Every kernel family's grid carries the batch and head counts in its y / z dimensions
    (at most 65535): a larger count is refused with DC_ERR_UNSUPPORTED by the shared
    validation, for the q_len == 1 (decode) shapes as for the rest, before anything launches."""
    L = _lib.load()
    for B, H in ((70000, 1), (1, 70000)):
        for Lq in (1, 8):
            q, k = _fake((B, H, Lq, 64)), _fake((B, H, 16, 64))
            out, lse = _fake((B, H, Lq, 64)), _fake((B, H, Lq))
            st = L.dc_sdpa_fwd(ctypes.byref(q), ctypes.byref(k), ctypes.byref(k), None, 0, 0, 0.0, 0,
                               ctypes.byref(out), ctypes.byref(lse), None)
            assert st == _lib.DC_ERR_UNSUPPORTED, (B, H, Lq, st)
            assert b"65535" in L.dc_last_error()
