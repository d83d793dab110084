"""``MultiheadAttention`` whose attention core runs on the fused CUDA kernels.

Same constructor, parameter names, initialisation and forward as DenseCore's
python/densecore/nn.py:595-640 (itself torch.nn.MultiheadAttention's), as a torch.nn.Module so
parameters live in CUDA memory. The forward calls
:func:`densecore_b200.functional.multi_head_attention_forward`.
"""
from __future__ import annotations

import torch
from torch import nn

from .functional import multi_head_attention_forward


class MultiheadAttention(nn.Module):
    def __init__(self, embed_dim, num_heads, dropout=0.0, bias=True, add_bias_kv=False, add_zero_attn=False,
                 kdim=None, vdim=None, batch_first=False, device=None, dtype=None):
        super().__init__()
        if embed_dim <= 0 or num_heads <= 0:
            raise ValueError("embed_dim and num_heads must be greater than 0")
        if embed_dim % num_heads:
            raise AssertionError("embed_dim must be divisible by num_heads")
        kw = dict(device=device, dtype=dtype or torch.float32)
        self.embed_dim, self.num_heads, self.dropout, self.batch_first = embed_dim, num_heads, dropout, batch_first
        self.kdim, self.vdim = kdim or embed_dim, vdim or embed_dim
        self._qkv_same_embed_dim = self.kdim == embed_dim and self.vdim == embed_dim
        self.head_dim, self.add_zero_attn = embed_dim // num_heads, add_zero_attn
        empty = lambda *shape: nn.Parameter(torch.zeros(shape, **kw))
        if self._qkv_same_embed_dim:
            self.in_proj_weight = empty(3 * embed_dim, embed_dim)
            self.register_parameter("q_proj_weight", None)
            self.register_parameter("k_proj_weight", None)
            self.register_parameter("v_proj_weight", None)
        else:
            self.q_proj_weight = empty(embed_dim, embed_dim)
            self.k_proj_weight = empty(embed_dim, self.kdim)
            self.v_proj_weight = empty(embed_dim, self.vdim)
            self.register_parameter("in_proj_weight", None)
        if bias:
            self.in_proj_bias = empty(3 * embed_dim)
        else:
            self.register_parameter("in_proj_bias", None)
        self.out_proj = nn.Linear(embed_dim, embed_dim, bias=bias, **kw)
        if add_bias_kv:
            self.bias_k, self.bias_v = empty(1, 1, embed_dim), empty(1, 1, embed_dim)
        else:
            self.bias_k = self.bias_v = None
        for weight in (self.in_proj_weight, self.q_proj_weight, self.k_proj_weight, self.v_proj_weight):
            if weight is not None:
                nn.init.xavier_uniform_(weight)
        if bias:
            nn.init.zeros_(self.out_proj.bias)
        for extra in (self.bias_k, self.bias_v):
            if extra is not None:
                nn.init.xavier_normal_(extra)

    def forward(self, query, key, value, key_padding_mask=None, need_weights=True, attn_mask=None,
                average_attn_weights=True, is_causal=False):
        batched = query.dim() == 3
        if self.batch_first and batched:
            query, key, value = (x.transpose(1, 0) for x in (query, key, value))
        out, weights = multi_head_attention_forward(
            query, key, value, self.embed_dim, self.num_heads, self.in_proj_weight, self.in_proj_bias,
            self.bias_k, self.bias_v, self.add_zero_attn, self.dropout, self.out_proj.weight, self.out_proj.bias,
            training=self.training, key_padding_mask=key_padding_mask, need_weights=need_weights,
            attn_mask=attn_mask, use_separate_proj_weight=not self._qkv_same_embed_dim,
            q_proj_weight=self.q_proj_weight, k_proj_weight=self.k_proj_weight, v_proj_weight=self.v_proj_weight,
            average_attn_weights=average_attn_weights, is_causal=is_causal)
        return (out.transpose(1, 0) if self.batch_first and batched else out), weights
