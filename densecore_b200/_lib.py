"""ctypes binding of ``libdensecore_sdpa.so`` (the C ABI in include/densecore_sdpa.h).

The library is built in-tree (``densecore_b200/build.py``). There is no fallback: if the
shared library is missing or cannot be loaded, every call raises ``RuntimeError`` naming the
path and the loader's message.
"""
from __future__ import annotations

import ctypes
import os
import threading

import torch

HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(HERE, "libdensecore_sdpa.so")

DC_OK, DC_ERR_VALUE, DC_ERR_RUNTIME, DC_ERR_CUDA, DC_ERR_UNSUPPORTED = 0, 1, 2, 3, 4
DC_F32, DC_BOOL = 0, 1
DC_PREC_3XTF32, DC_PREC_TF32, DC_PREC_FP32 = 0, 1, 2

# Every entry point include/densecore_sdpa.h declares.
EXPORTS = ("dc_sdpa_fwd", "dc_sdpa_bwd_workspace_size", "dc_sdpa_bwd", "dc_sdpa_decode_workspace_size",
           "dc_sdpa_decode_default_splits", "dc_sdpa_decode", "dc_sdpa_decode_noalloc", "dc_attn_merge", "dc_attn_probs",
           "dc_last_error", "dc_abi_version", "dc_sdpa_fwd_path", "dc_kernel_timing", "dc_kernel_timing_report", "dc_device_status",
           "dc_dropout_keep_bits", "dc_rng_skip", "dc_sdpa_fwd_dropout", "dc_sdpa_bwd_dropout", "dc_attn_probs_dropout",
           "dc_debug_wait_probe", "dc_ring_sdpa_fwd_workspace_size", "dc_ring_sdpa_fwd")


class DcTensor(ctypes.Structure):
    _fields_ = [("data", ctypes.c_void_p), ("dtype", ctypes.c_int32), ("ndim", ctypes.c_int32),
                ("sizes", ctypes.c_int64 * 4), ("strides", ctypes.c_int64 * 4)]


_P = ctypes.POINTER(DcTensor)
_lock = threading.Lock()
_lib = None


def load():
    """Load the shared library once; raise RuntimeError if it is absent or broken."""
    global _lib
    with _lock:
        if _lib is not None:
            return _lib
        if not os.path.exists(LIB_PATH):
            raise RuntimeError(f"densecore_b200: CUDA library not built: {LIB_PATH} is missing "
                               "(run densecore_b200.build.build())")
        try:
            L = ctypes.CDLL(LIB_PATH)
        except OSError as e:
            raise RuntimeError(f"densecore_b200: cannot load {LIB_PATH}: {e}") from e
        i, d, sz, vp = ctypes.c_int, ctypes.c_double, ctypes.c_size_t, ctypes.c_void_p
        i64 = ctypes.c_int64
        L.dc_sdpa_fwd.argtypes = [_P, _P, _P, _P, i, i, d, i, _P, _P, vp]
        L.dc_sdpa_fwd.restype = i
        L.dc_sdpa_bwd_workspace_size.argtypes = [i64, i64, i64]
        L.dc_sdpa_bwd_workspace_size.restype = sz
        L.dc_sdpa_bwd.argtypes = [_P] * 7 + [i, i, d, i, _P, _P, _P, vp, sz, vp]
        L.dc_sdpa_bwd.restype = i
        L.dc_sdpa_decode_workspace_size.argtypes = [i64, i64, i64, i]
        L.dc_sdpa_decode_workspace_size.restype = sz
        L.dc_sdpa_decode_default_splits.argtypes = [i64, i64, i64]
        L.dc_sdpa_decode_default_splits.restype = i
        L.dc_sdpa_decode.argtypes = [_P, _P, _P, _P, i, d, i, _P, _P, vp, sz, vp]
        L.dc_sdpa_decode.restype = i
        L.dc_sdpa_decode_noalloc.argtypes = [_P, _P, _P, _P, i, d, i, _P, _P, vp]
        L.dc_sdpa_decode_noalloc.restype = i
        L.dc_attn_merge.argtypes = [_P, _P, _P, _P, vp]
        L.dc_attn_merge.restype = i
        L.dc_attn_probs.argtypes = [_P, _P, _P, _P, i, i, d, i, _P, vp]
        L.dc_attn_probs.restype = i
        u32p, f = ctypes.POINTER(ctypes.c_uint32), ctypes.c_float
        L.dc_dropout_keep_bits.argtypes = [vp, vp, i64, d, vp, vp]
        L.dc_dropout_keep_bits.restype = i
        L.dc_rng_skip.argtypes = [u32p, ctypes.c_uint64, u32p]
        L.dc_rng_skip.restype = i
        L.dc_sdpa_fwd_dropout.argtypes = [_P, _P, _P, _P, i, i, d, i, vp, f, _P, _P, vp]
        L.dc_sdpa_fwd_dropout.restype = i
        L.dc_sdpa_bwd_dropout.argtypes = [_P] * 7 + [i, i, d, i, vp, f, _P, _P, _P, vp, sz, vp]
        L.dc_sdpa_bwd_dropout.restype = i
        L.dc_attn_probs_dropout.argtypes = [_P, _P, _P, _P, i, i, d, vp, f, i, _P, vp]
        L.dc_attn_probs_dropout.restype = i
        L.dc_last_error.argtypes = []
        L.dc_last_error.restype = ctypes.c_char_p
        L.dc_abi_version.argtypes = []
        L.dc_abi_version.restype = i
        L.dc_sdpa_fwd_path.argtypes = [_P, _P, _P, _P, i, i]
        L.dc_sdpa_fwd_path.restype = i
        L.dc_device_status.argtypes = [i]
        L.dc_device_status.restype = i
        L.dc_ring_sdpa_fwd_workspace_size.argtypes = [i64, i64, i64, i64, i64]
        L.dc_ring_sdpa_fwd_workspace_size.restype = sz
        L.dc_ring_sdpa_fwd.argtypes = [_P, _P, _P, i, i, d, i, vp, _P, _P, vp, sz, vp]
        L.dc_ring_sdpa_fwd.restype = i
        L.dc_debug_wait_probe.argtypes = [ctypes.c_uint64, i, vp]
        L.dc_debug_wait_probe.restype = i
        L.dc_kernel_timing.argtypes = [i]
        L.dc_kernel_timing.restype = i
        L.dc_kernel_timing_report.argtypes = [ctypes.c_char_p, sz, i]
        L.dc_kernel_timing_report.restype = i
        if L.dc_abi_version() != 1:
            raise RuntimeError(f"densecore_b200: {LIB_PATH} has ABI {L.dc_abi_version()}, expected 1")
        _lib = L
        return L


def view(t: torch.Tensor | None):
    """A DcTensor describing ``t`` (no copy); None stays None (a NULL pointer)."""
    if t is None:
        return None
    if t.dtype == torch.float32:
        dt = DC_F32
    elif t.dtype in (torch.bool, torch.uint8):
        dt = DC_BOOL
    else:
        raise TypeError(f"densecore_b200: unsupported tensor dtype {t.dtype}")
    if t.dim() > 4:
        raise ValueError("densecore_b200: tensors have at most 4 dims")
    v = DcTensor()
    v.data = t.data_ptr() if t.numel() else 0
    v.dtype = dt
    v.ndim = t.dim()
    for n, (s, st) in enumerate(zip(t.shape, t.stride())):
        v.sizes[n] = s
        v.strides[n] = st
    return v


def ref(v):
    return None if v is None else ctypes.byref(v)


def check(status: int, what: str):
    """Map a status code to the exception the reference raises for it."""
    if status == DC_OK:
        return
    msg = (_lib.dc_last_error() or b"").decode(errors="replace")
    if status == DC_ERR_VALUE:
        raise ValueError(msg or what)
    if status == DC_ERR_UNSUPPORTED:
        raise NotImplementedError(msg or what)
    raise RuntimeError(f"{what}: {msg}" if msg else what)


def stream_of(t: torch.Tensor):
    return ctypes.c_void_p(torch.cuda.current_stream(t.device).cuda_stream)


def kernel_timing(enable: bool) -> None:
    """Turn the library's per-kernel CUDA-event tracing on or off."""
    load().dc_kernel_timing(int(bool(enable)))


def kernel_timing_report(reset: bool = True) -> dict:
    """{kernel: (launches, total_ms)} of the launches traced since the last reset."""
    import json
    buf = ctypes.create_string_buffer(1 << 16)
    n = load().dc_kernel_timing_report(buf, len(buf), int(bool(reset)))
    if n < 0:
        raise RuntimeError("kernel timing report failed: " + (_lib.dc_last_error() or b"").decode())
    return {k: (int(v[0]), float(v[1])) for k, v in json.loads(buf.value.decode()).items()}
