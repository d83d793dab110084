"""The native entry points, under the names DenseCore's pyo3 module exports.

``_flash_attention`` and ``_flash_attention_backward`` keep the signatures of
src/lib.rs:609-638 and :640-683 (``(q, k, v, causal, scale=None, mask=None)`` and
``(grad_out, q, k, v, out, lse, causal, scale=None, mask=None)``), their ValueError /
RuntimeError behaviour, and their outputs: fresh tensors (out, lse) and (grad_q, grad_k,
grad_v). The tensors are CUDA ``torch.Tensor`` (torch is used for device memory and streams
only); the work runs in libdensecore_sdpa.so. ``mask`` may be any float32/bool tensor that
broadcasts to (B, H, L, S) -- for a bool mask True means "may attend" -- so DenseCore's
materialised (B, H, L, S) float mask is accepted as one case of it.
"""
from __future__ import annotations

import torch

from . import _lib
from .backends import precision_code


def _require_cuda(*ts):
    dev = None
    for t in ts:
        if t is None:
            continue
        if not isinstance(t, torch.Tensor):
            raise TypeError("flash attention takes torch.Tensor arguments")
        if not t.is_cuda:
            raise RuntimeError("densecore_b200 runs on CUDA tensors; got a tensor on " + str(t.device))
        if dev is None:
            dev = t.device
        elif t.device != dev:
            raise RuntimeError(f"flash attention tensors are on different devices ({dev}, {t.device})")
    return dev


def _scale_args(scale):
    return (0, 0.0) if scale is None else (1, float(scale))


def _flash_attention(q, k, v, causal, scale=None, mask=None, precision=None):
    """Forward: (out (B,H,L,Ev), lse (B,H,L)). src/lib.rs:609-638."""
    L = _lib.load()
    dev = _require_cuda(q, k, v, mask)
    if q.dim() != 4 or k.dim() != 4 or v.dim() != 4:
        raise ValueError("flash attention takes (B, H, L, E) tensors")
    B, H, Lq = q.shape[:3]
    out = torch.empty((B, H, Lq, v.shape[3]), device=dev, dtype=torch.float32)
    lse = torch.empty((B, H, Lq), device=dev, dtype=torch.float32)
    prec = precision_code() if precision is None else precision
    has, sc = _scale_args(scale)
    with torch.cuda.device(dev):
        vq, vk, vv, vm, vo, vl = (_lib.view(t) for t in (q, k, v, mask, out, lse))
        path = L.dc_sdpa_fwd_path(_lib.ref(vq), _lib.ref(vk), _lib.ref(vv), _lib.ref(vm), int(bool(causal)), prec)
        if path == 2:
            splits = L.dc_sdpa_decode_default_splits(B, H, k.shape[2])
            ws = torch.empty(max(L.dc_sdpa_decode_workspace_size(B, H, v.shape[3], splits), 1),
                             dtype=torch.uint8, device=dev)
            st = L.dc_sdpa_decode(_lib.ref(vq), _lib.ref(vk), _lib.ref(vv), _lib.ref(vm), has, sc, splits,
                                  _lib.ref(vo), _lib.ref(vl), ws.data_ptr(), ws.numel(), _lib.stream_of(q))
        else:
            st = L.dc_sdpa_fwd(_lib.ref(vq), _lib.ref(vk), _lib.ref(vv), _lib.ref(vm), int(bool(causal)), has, sc,
                               prec, _lib.ref(vo), _lib.ref(vl), _lib.stream_of(q))
    _lib.check(st, "flash attention forward failed")
    return out, lse


def _flash_attention_backward(grad_out, q, k, v, out, lse, causal, scale=None, mask=None, precision=None):
    """Backward: (grad_q, grad_k, grad_v). src/lib.rs:640-683."""
    L = _lib.load()
    dev = _require_cuda(grad_out, q, k, v, out, lse, mask)
    if q.dim() != 4 or k.dim() != 4 or v.dim() != 4:
        raise ValueError("flash attention takes (B, H, L, E) tensors")
    gq = torch.empty(q.shape, device=dev, dtype=torch.float32)
    gk = torch.empty(k.shape, device=dev, dtype=torch.float32)
    gv = torch.empty(v.shape, device=dev, dtype=torch.float32)
    prec = precision_code() if precision is None else precision
    has, sc = _scale_args(scale)
    with torch.cuda.device(dev):
        nbytes = L.dc_sdpa_bwd_workspace_size(q.shape[0], q.shape[1], q.shape[2])
        ws = torch.empty(max(nbytes, 1), dtype=torch.uint8, device=dev)
        views = [_lib.view(t) for t in (grad_out, q, k, v, out, lse, mask, gq, gk, gv)]
        st = L.dc_sdpa_bwd(*[_lib.ref(x) for x in views[:7]], int(bool(causal)), has, sc, prec,
                           *[_lib.ref(x) for x in views[7:]], ws.data_ptr(), ws.numel(), _lib.stream_of(q))
    _lib.check(st, "flash attention backward failed")
    return gq, gk, gv


def _flash_attention_dropout(q, k, v, causal, scale, mask, keep, keep_scale, precision=None):
    """Forward with dropout on the weights (dc_sdpa_fwd_dropout): (out, lse). ``keep`` holds
    the packed keep bits of the (B, H, L, S) weights, ``keep_scale`` = float32(1/(1-p))."""
    L = _lib.load()
    dev = _require_cuda(q, k, v, mask, keep)
    if q.dim() != 4 or k.dim() != 4 or v.dim() != 4:
        raise ValueError("flash attention takes (B, H, L, E) tensors")
    B, H, Lq = q.shape[:3]
    out = torch.empty((B, H, Lq, v.shape[3]), device=dev, dtype=torch.float32)
    lse = torch.empty((B, H, Lq), device=dev, dtype=torch.float32)
    prec = precision_code() if precision is None else precision
    has, sc = _scale_args(scale)
    with torch.cuda.device(dev):
        vs = [_lib.view(t) for t in (q, k, v, mask, out, lse)]
        st = L.dc_sdpa_fwd_dropout(*[_lib.ref(x) for x in vs[:4]], int(bool(causal)), has, sc, prec, keep.data_ptr(),
                                   float(keep_scale), _lib.ref(vs[4]), _lib.ref(vs[5]), _lib.stream_of(q))
    _lib.check(st, "flash attention forward failed")
    return out, lse


def _flash_attention_dropout_backward(grad_out, q, k, v, out, lse, causal, scale, mask, keep, keep_scale,
                                      precision=None):
    """Backward of :func:`_flash_attention_dropout` (dc_sdpa_bwd_dropout): (grad_q, grad_k, grad_v)."""
    L = _lib.load()
    dev = _require_cuda(grad_out, q, k, v, out, lse, mask, keep)
    gq = torch.empty(q.shape, device=dev, dtype=torch.float32)
    gk = torch.empty(k.shape, device=dev, dtype=torch.float32)
    gv = torch.empty(v.shape, device=dev, dtype=torch.float32)
    prec = precision_code() if precision is None else precision
    has, sc = _scale_args(scale)
    with torch.cuda.device(dev):
        nbytes = L.dc_sdpa_bwd_workspace_size(q.shape[0], q.shape[1], q.shape[2])
        ws = torch.empty(max(nbytes, 1), dtype=torch.uint8, device=dev)
        views = [_lib.view(t) for t in (grad_out, q, k, v, out, lse, mask, gq, gk, gv)]
        st = L.dc_sdpa_bwd_dropout(*[_lib.ref(x) for x in views[:7]], int(bool(causal)), has, sc, prec,
                                   keep.data_ptr(), float(keep_scale), *[_lib.ref(x) for x in views[7:]],
                                   ws.data_ptr(), ws.numel(), _lib.stream_of(q))
    _lib.check(st, "flash attention backward failed")
    return gq, gk, gv


def _decode(q, k, v, scale=None, mask=None, num_splits=0, workspace=None):
    """Split-KV decode for q_len == 1 (dc_sdpa_decode): (out, lse)."""
    L = _lib.load()
    dev = _require_cuda(q, k, v, mask)
    B, H, Lq = q.shape[:3]
    out = torch.empty((B, H, Lq, v.shape[3]), device=dev, dtype=torch.float32)
    lse = torch.empty((B, H, Lq), device=dev, dtype=torch.float32)
    has, sc = _scale_args(scale)
    with torch.cuda.device(dev):
        splits = num_splits if num_splits > 0 else L.dc_sdpa_decode_default_splits(B, H, k.shape[2])
        need = L.dc_sdpa_decode_workspace_size(B, H, v.shape[3], splits)
        ws = workspace if workspace is not None else torch.empty(max(need, 1), dtype=torch.uint8, device=dev)
        vs = [_lib.view(t) for t in (q, k, v, mask, out, lse)]
        st = L.dc_sdpa_decode(*[_lib.ref(x) for x in vs[:4]], has, sc, splits, _lib.ref(vs[4]), _lib.ref(vs[5]),
                              ws.data_ptr(), ws.numel(), _lib.stream_of(q))
    _lib.check(st, "decode attention failed")
    return out, lse


def _attn_merge(out_acc, lse_acc, out_part, lse_part):
    """In-place logsumexp merge of (out_part, lse_part) into (out_acc, lse_acc)."""
    L = _lib.load()
    _require_cuda(out_acc, lse_acc, out_part, lse_part)
    with torch.cuda.device(out_acc.device):
        vs = [_lib.view(t) for t in (out_acc, lse_acc, out_part, lse_part)]
        st = L.dc_attn_merge(*[_lib.ref(x) for x in vs], _lib.stream_of(out_acc))
    _lib.check(st, "attention merge failed")
    return out_acc, lse_acc


def _ring_attention(q, k, v, comm_ptr, causal=True, scale=None, precision=None, workspace=None):
    """Ring attention forward of this rank's zig-zag shards over an NCCL communicator
    (dc_ring_sdpa_fwd): (out, lse) of the local query rows against the whole sequence."""
    L = _lib.load()
    dev = _require_cuda(q, k, v)
    B, H, Lq = q.shape[:3]
    out = torch.empty((B, H, Lq, v.shape[3]), device=dev, dtype=torch.float32)
    lse = torch.empty((B, H, Lq), device=dev, dtype=torch.float32)
    prec = precision_code() if precision is None else precision
    has, sc = _scale_args(scale)
    with torch.cuda.device(dev):
        need = L.dc_ring_sdpa_fwd_workspace_size(B, H, k.shape[1], Lq, q.shape[3])
        ws = workspace if workspace is not None else torch.empty(max(need, 1), dtype=torch.uint8, device=dev)
        vs = [_lib.view(t) for t in (q, k, v, out, lse)]
        st = L.dc_ring_sdpa_fwd(*[_lib.ref(x) for x in vs[:3]], int(bool(causal)), has, sc, prec, comm_ptr,
                                _lib.ref(vs[3]), _lib.ref(vs[4]), ws.data_ptr(), ws.numel(), _lib.stream_of(q))
    _lib.check(st, "ring attention failed")
    return out, lse


def _attn_probs(q, k, lse, causal, scale=None, mask=None, average_heads=True, keep=None, keep_scale=0.0):
    """softmax(scale q k^T + mask) from the forward's lse; (B,L,S) head mean or (B,H,L,S).
    With ``keep`` (packed dropout keep bits) each probability is times its dropout factor."""
    L = _lib.load()
    dev = _require_cuda(q, k, lse, mask, keep)
    B, H, Lq = q.shape[:3]
    S = k.shape[2]
    shape = (B, Lq, S) if average_heads else (B, H, Lq, S)
    probs = torch.empty(shape, device=dev, dtype=torch.float32)
    has, sc = _scale_args(scale)
    with torch.cuda.device(dev):
        vs = [_lib.view(t) for t in (q, k, lse, mask, probs)]
        if keep is None:
            st = L.dc_attn_probs(*[_lib.ref(x) for x in vs[:4]], int(bool(causal)), has, sc,
                                 int(bool(average_heads)), _lib.ref(vs[4]), _lib.stream_of(q))
        else:
            st = L.dc_attn_probs_dropout(*[_lib.ref(x) for x in vs[:4]], int(bool(causal)), has, sc, keep.data_ptr(),
                                         float(keep_scale), int(bool(average_heads)), _lib.ref(vs[4]),
                                         _lib.stream_of(q))
    _lib.check(st, "attention probabilities failed")
    return probs


def _fwd_path(q, k, v, mask=None, causal=False, precision=None):
    """0 = CUDA-core kernels, 1 = tcgen05 tensor cores, 2 = split-KV decode."""
    L = _lib.load()
    prec = precision_code() if precision is None else precision
    vs = [_lib.view(t) for t in (q, k, v, mask)]
    return L.dc_sdpa_fwd_path(*[_lib.ref(x) for x in vs], int(bool(causal)), prec)
