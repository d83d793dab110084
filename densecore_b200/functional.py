"""``scaled_dot_product_attention`` and ``multi_head_attention_forward`` on CUDA tensors.

The signatures, argument checks and error types mirror DenseCore's
python/densecore/functional.py (SDPA :276-340, ``_flash_mask`` :343-364, ``_flash_attention``
:367-388, MHA :400-461). The work runs in libdensecore_sdpa.so: every SDPA call -- rank 3 or
4, any mask DenseCore accepts, grouped-query heads, Ev != E -- goes to one of its kernels; there
is no CPU or composed-op fallback. Differences from the reference are listed where they occur.
"""
from __future__ import annotations

import math
import numbers

import numpy as np
import torch

from . import _native
from . import random as _random


def _as_mask(attn_mask, device):
    """The mask as a CUDA tensor (NumPy arrays are copied over), or None."""
    if attn_mask is None:
        return None
    if not isinstance(attn_mask, torch.Tensor):
        attn_mask = torch.from_numpy(np.ascontiguousarray(attn_mask))
    if attn_mask.device != device:
        attn_mask = attn_mask.to(device)
    return attn_mask


def _flash_mask(attn_mask, rank):
    """``_flash_mask`` (functional.py:343-364) without materialising: a bool mask (True may
    attend) or float32 additive mask, viewed with 4 dims that broadcast to (B, H, L, S).
    For rank-3 inputs (N, L, E) the mask broadcasts against (N, L, S) and gains the head dim.
    The kernel checks the broadcast and raises ValueError otherwise."""
    if attn_mask is None:
        return None
    if attn_mask.requires_grad:
        raise NotImplementedError("attention masks that require grad are not supported on CUDA")
    if attn_mask.dtype not in (torch.bool, torch.float32):
        raise TypeError(f"attn_mask must be bool or float32, got {attn_mask.dtype}")
    m = attn_mask
    if rank == 3:
        if m.dim() > 3:
            raise ValueError("attn_mask for rank-3 attention has at most 3 dims")
        while m.dim() < 3:
            m = m.unsqueeze(0)
        m = m.unsqueeze(1)
    else:
        if m.dim() > 4:
            raise ValueError("attn_mask has at most 4 dims")
        while m.dim() < 4:
            m = m.unsqueeze(0)
    return m


class _FlashAttention(torch.autograd.Function):
    """``_flash_attention``'s Function (functional.py:367-388): saves q, k, v, out, lse."""

    @staticmethod
    def forward(ctx, q, k, v, causal, scale, mask):
        out, lse = _native._flash_attention(q, k, v, causal, scale, mask)
        ctx.save_for_backward(q, k, v, out, lse)
        ctx.causal, ctx.scale, ctx.mask = causal, scale, mask
        ctx.mark_non_differentiable(lse)
        return out, lse

    @staticmethod
    def backward(ctx, grad, _grad_lse):
        q, k, v, out, lse = ctx.saved_tensors
        gq, gk, gv = _native._flash_attention_backward(grad.contiguous() if grad.stride(-1) != 1 else grad,
                                                       q, k, v, out, lse, ctx.causal, ctx.scale, ctx.mask)
        return gq, gk, gv, None, None, None


def _dropout_probability(p):
    """functional.py:219-226: a real number in [0, 1] (bools are refused)."""
    if isinstance(p, (bool, np.bool_)) or not isinstance(p, numbers.Real):
        raise TypeError("dropout probability must be real")
    p = float(p)
    if not 0.0 <= p <= 1.0:
        raise ValueError("dropout probability must be in [0, 1]")
    return p


def _keep_mask(n, p, device, generator=None):
    """The dropout keep bits of n weights and the survivors' factor, as ``_dropout_noise``
    (functional.py:638-641) draws them: bernoulli(1 - p) from the generator, survivors times
    float32(1) / float32(1 - p). p == 1 draws nothing and zeroes every weight (``dropout``
    multiplies by 0 there, functional.py:242-243)."""
    if p == 1.0:
        return torch.zeros(max((n + 31) // 32, 1), dtype=torch.int32, device=device), 0.0
    keep = _random.dropout_keep_bits(n, 1.0 - p, device, generator)
    return keep, float(np.float32(1.0) / np.float32(1.0 - p))


class _FlashAttentionDropout(torch.autograd.Function):
    """The fused kernels with dropout on the weights; saves q, k, v, out, lse and the keep bits."""

    @staticmethod
    def forward(ctx, q, k, v, causal, scale, mask, p):
        _native._require_cuda(q, k, v, mask)  # before the draw, so a refused call consumes nothing
        n = q.shape[0] * q.shape[1] * q.shape[2] * k.shape[2]
        keep, keep_scale = _keep_mask(n, p, q.device)
        out, lse = _native._flash_attention_dropout(q, k, v, causal, scale, mask, keep, keep_scale)
        ctx.save_for_backward(q, k, v, out, lse, keep)
        ctx.causal, ctx.scale, ctx.mask, ctx.keep_scale = causal, scale, mask, keep_scale
        return out

    @staticmethod
    def backward(ctx, grad):
        q, k, v, out, lse, keep = ctx.saved_tensors
        gq, gk, gv = _native._flash_attention_dropout_backward(
            grad.contiguous() if grad.stride(-1) != 1 else grad, q, k, v, out, lse, ctx.causal, ctx.scale, ctx.mask,
            keep, ctx.keep_scale)
        return gq, gk, gv, None, None, None, None


def flash_attention(q, k, v, causal=False, scale=None, mask=None):
    """(out, lse) of the fused kernel on (B,H,L,E) / (B,Hkv,S,E) / (B,Hkv,S,Ev) CUDA tensors,
    differentiable in q, k and v."""
    return _FlashAttention.apply(q, k, v, causal, scale, mask)


def scaled_dot_product_attention(query, key, value, attn_mask=None, dropout_p=0.0, is_causal=False, scale=None,
                                 enable_gqa=False):
    """softmax(query @ key^T * scale + mask) @ value for rank-3 (N, L, E) or rank-4 (N, H, L, E).

    As DenseCore's: a boolean mask is True where attention is allowed, a float mask is added to
    the scores; is_causal applies a top-left lower-triangular mask and cannot be combined with
    attn_mask; scale defaults to 1/sqrt(E). Fully masked rows give 0 (and zero gradients).
    dropout_p > 0 draws the keep bits from the default generator's stream, exactly as
    DenseCore's math path draws them (functional.py:318-340, :638-641).
    Differences: dropout runs in the fused kernels instead of the math path; grouped-query
    heads run natively instead of widening K/V.
    """
    for name, t in (("query", query), ("key", key), ("value", value)):
        if not isinstance(t, torch.Tensor):
            raise TypeError(f"attention {name} must be a Tensor")
    rank = query.dim()
    if enable_gqa and rank == 4 and key.dim() == 4 and key.shape[1] != query.shape[1]:
        if key.shape[1] == 0 or query.shape[1] % key.shape[1]:
            raise ValueError("attention shapes must be (..., L, E), (..., S, E), (..., S, Ev)")
        gqa = True
    else:
        gqa = False
    if rank not in (3, 4) or key.dim() != rank or value.dim() != rank:
        raise ValueError("attention query, key and value must all be rank 3 or all rank 4")
    lead, (length, embed) = tuple(query.shape[:-2]), tuple(query.shape[-2:])
    source = key.shape[-2]
    klead = tuple(key.shape[:-2]) if not gqa else (key.shape[0], query.shape[1])
    vlead = tuple(value.shape[:-2]) if not gqa else (value.shape[0], query.shape[1])
    if gqa and value.shape[1] != key.shape[1]:
        vlead = None
    if klead != lead or vlead != lead or key.shape[-1] != embed or value.shape[-2] != source:
        raise ValueError("attention shapes must be (..., L, E), (..., S, E), (..., S, Ev)")
    if type(is_causal) is not bool:
        raise TypeError("is_causal must be a bool")
    if is_causal and attn_mask is not None:
        raise ValueError("attn_mask and is_causal cannot both be set")
    if scale is None:
        scale = 1.0 / math.sqrt(embed) if embed else 1.0
    elif isinstance(scale, (bool, np.bool_)) or not isinstance(scale, numbers.Real):
        raise TypeError("scale must be real")
    p = _dropout_probability(dropout_p) if dropout_p else 0.0
    for t in (query, key, value):
        if t.dtype != torch.float32:
            raise TypeError(f"attention tensors must be float32, got {t.dtype}")
    mask = _flash_mask(_as_mask(attn_mask, query.device), rank)
    if rank == 3:
        q, k, v = query.unsqueeze(1), key.unsqueeze(1), value.unsqueeze(1)
    else:
        q, k, v = query, key, value
    if p:
        out = _FlashAttentionDropout.apply(q, k, v, is_causal, float(scale), mask, p)
    else:
        out, _lse = flash_attention(q, k, v, is_causal, float(scale), mask)
    return out.squeeze(1) if rank == 3 else out


def _float_mask(mask):
    """MHA masks (functional.py:391-397): bool True means NOT allowed (-inf); float adds."""
    if mask is None:
        return None
    if mask.dtype == torch.bool:
        return torch.zeros(mask.shape, dtype=torch.float32, device=mask.device).masked_fill_(mask, float("-inf"))
    return mask.to(torch.float32)


def multi_head_attention_forward(query, key, value, embed_dim_to_check, num_heads, in_proj_weight, in_proj_bias,
                                 bias_k, bias_v, add_zero_attn, dropout_p, out_proj_weight, out_proj_bias,
                                 training=True, key_padding_mask=None, need_weights=True, attn_mask=None,
                                 use_separate_proj_weight=False, q_proj_weight=None, k_proj_weight=None,
                                 v_proj_weight=None, static_k=None, static_v=None, average_attn_weights=True,
                                 is_causal=False):
    """DenseCore's MHA (functional.py:400-461) with the attention core on the fused kernels.

    Inputs are (L, N, E), or (L, E) unbatched. Projections are plain library GEMMs
    (``torch.nn.functional.linear``); scores, masking, softmax and the weighted sum run in one
    fused kernel with strided (N, H, L, D) views of the projections -- no transposed copies.
    As in the reference, a query row whose keys are all masked yields NaN (output and
    gradients); ``need_weights`` returns the softmax probabilities (head-averaged by default),
    which are not differentiable here. In training, dropout_p > 0 drops the probabilities with
    DenseCore's masks (functional.py:450-451); the returned weights are the dropped ones, as
    there.
    """
    F = torch.nn.functional
    if is_causal and attn_mask is None:
        raise RuntimeError("Need attn_mask if specifying the is_causal hint")
    batched = query.dim() == 3
    if not batched:
        query, key, value = query.unsqueeze(1), key.unsqueeze(1), value.unsqueeze(1)
        if key_padding_mask is not None:
            key_padding_mask = key_padding_mask.unsqueeze(0)
    tgt_len, bsz, embed_dim = query.shape
    if embed_dim != embed_dim_to_check:
        raise ValueError(f"was expecting embedding dimension of {embed_dim_to_check}, but got {embed_dim}")
    p = _dropout_probability(dropout_p) if training and dropout_p > 0 else 0.0
    head_dim = embed_dim // num_heads
    biases = (None, None, None) if in_proj_bias is None else in_proj_bias.chunk(3)
    weights = (q_proj_weight, k_proj_weight, v_proj_weight) if use_separate_proj_weight else in_proj_weight.chunk(3)
    q, k, v = (F.linear(x, w, b) for x, w, b in zip((query, key, value), weights, biases))
    attn_mask = _float_mask(attn_mask)
    if attn_mask is not None and attn_mask.dim() == 2:
        attn_mask = attn_mask.unsqueeze(0)
    kpm = key_padding_mask
    if bias_k is not None and bias_v is not None:
        k = torch.cat([k, bias_k.expand(1, bsz, embed_dim)])
        v = torch.cat([v, bias_v.expand(1, bsz, embed_dim)])
        attn_mask = None if attn_mask is None else F.pad(attn_mask, (0, 1))
        kpm = None if kpm is None else F.pad(kpm, (0, 1))
    src_len = k.shape[0] if static_k is None else static_k.shape[1]
    # (L, N, E) -> (N, H, L, D) strided views (the reference's reshape + transpose).
    qh = q.view(tgt_len, bsz, num_heads, head_dim).permute(1, 2, 0, 3)
    kh = (static_k.view(bsz, num_heads, src_len, head_dim) if static_k is not None
          else k.view(k.shape[0], bsz, num_heads, head_dim).permute(1, 2, 0, 3))
    vh = (static_v.view(bsz, num_heads, src_len, head_dim) if static_v is not None
          else v.view(v.shape[0], bsz, num_heads, head_dim).permute(1, 2, 0, 3))
    if add_zero_attn:
        kh = torch.cat([kh, kh.new_zeros(bsz, num_heads, 1, head_dim)], 2)
        vh = torch.cat([vh, vh.new_zeros(bsz, num_heads, 1, head_dim)], 2)
        attn_mask = None if attn_mask is None else F.pad(attn_mask, (0, 1))
        kpm = None if kpm is None else F.pad(kpm, (0, 1))
    S = kh.shape[2]
    # One broadcastable mask: key padding (N,1,1,S) and/or attn_mask (1 or N*H, L, S).
    mask = None
    if kpm is not None:
        if kpm.dtype == torch.bool:
            mask = (~kpm).reshape(bsz, 1, 1, S)  # the kernel's bool mask: True may attend
        else:
            mask = kpm.to(torch.float32).reshape(bsz, 1, 1, S)
    if attn_mask is not None:
        am = attn_mask.reshape(-1, tgt_len, S)
        am = am.unsqueeze(0) if am.shape[0] == 1 else am.reshape(bsz, num_heads, tgt_len, S)
        if mask is None:
            mask = am
        else:
            mask = (_float_mask(~mask) if mask.dtype == torch.bool else mask) + am
    dead = None
    if mask is not None:
        # Rows whose every key is masked: NaN in the reference's math path.
        allowed = mask if mask.dtype == torch.bool else mask != float("-inf")
        dead = ~allowed.expand(bsz, num_heads, tgt_len, S).any(-1)
        if not bool(dead.any()):
            dead = None
    keep, keep_scale = (None, 0.0)
    if p:
        _native._require_cuda(qh, kh, vh, mask)
        keep, keep_scale = _keep_mask(bsz * num_heads * tgt_len * S, p, qh.device)
    out, lse = _MHACore.apply(qh, kh, vh, float(math.sqrt(1.0 / head_dim)), mask, dead, keep, keep_scale)
    out = out.permute(2, 0, 1, 3).reshape(tgt_len * bsz, embed_dim)
    out = F.linear(out, out_proj_weight, out_proj_bias).reshape(tgt_len, bsz, -1)
    if not batched:
        out = out.squeeze(1)
    if not need_weights:
        return out, None
    with torch.no_grad():
        probs = _native._attn_probs(qh, kh, lse, False, float(math.sqrt(1.0 / head_dim)), mask,
                                    average_heads=average_attn_weights, keep=keep, keep_scale=keep_scale)
        if dead is not None:
            d = dead.any(1) if average_attn_weights else dead
            probs = probs.masked_fill(d.unsqueeze(-1), float("nan"))
    return out, probs if batched else probs.squeeze(0)


class _MHACore(torch.autograd.Function):
    """The fused MHA core, with the reference math path's NaN for fully masked rows: such a
    row's output is NaN and, through the softmax and bmm VJPs, so are its query gradient and
    the key/value gradients of its (batch, head)."""

    @staticmethod
    def forward(ctx, qh, kh, vh, scale, mask, dead, keep, keep_scale):
        if keep is None:
            out, lse = _native._flash_attention(qh, kh, vh, False, scale, mask)
        else:
            out, lse = _native._flash_attention_dropout(qh, kh, vh, False, scale, mask, keep, keep_scale)
        ctx.save_for_backward(qh, kh, vh, out, lse)
        ctx.scale, ctx.mask, ctx.dead, ctx.keep, ctx.keep_scale = scale, mask, dead, keep, keep_scale
        ctx.mark_non_differentiable(lse)
        if dead is not None:
            out = out.masked_fill(dead.unsqueeze(-1), float("nan"))
        return out, lse

    @staticmethod
    def backward(ctx, grad, _g):
        qh, kh, vh, out, lse = ctx.saved_tensors
        grad = grad.contiguous()
        if ctx.dead is not None:
            grad = grad.masked_fill(ctx.dead.unsqueeze(-1), 0.0)
        if ctx.keep is None:
            gq, gk, gv = _native._flash_attention_backward(grad, qh, kh, vh, out, lse, False, ctx.scale, ctx.mask)
        else:
            gq, gk, gv = _native._flash_attention_dropout_backward(grad, qh, kh, vh, out, lse, False, ctx.scale,
                                                                   ctx.mask, ctx.keep, ctx.keep_scale)
        if ctx.dead is not None:
            nan = float("nan")
            gq = gq.masked_fill(ctx.dead.unsqueeze(-1), nan)
            bh = ctx.dead.any(-1)[..., None, None]
            gk = gk.masked_fill(bh, nan)
            gv = gv.masked_fill(bh, nan)
        return gq, gk, gv, None, None, None, None, None
