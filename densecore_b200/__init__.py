"""densecore_b200 -- DenseCore's scaled-dot-product-attention path, B200-native.

A drop-in for DenseCore's flash-attention path (src/torch_attention.rs reached through
``functional.scaled_dot_product_attention``, ``nn.MultiheadAttention`` and the pyo3 functions
``_flash_attention`` / ``_flash_attention_backward``) on CUDA tensors. The kernels are
hand-written for sm_100a and live in ``libdensecore_sdpa.so`` behind the C ABI of
``include/densecore_sdpa.h``; torch provides device memory, streams and torch.distributed.
"""
from . import backends, functional, nn
from ._native import _attn_merge, _attn_probs, _decode, _flash_attention, _flash_attention_backward
from .backends import set_sdpa_precision
from .functional import flash_attention, multi_head_attention_forward, scaled_dot_product_attention

__all__ = ["backends", "functional", "nn", "scaled_dot_product_attention", "multi_head_attention_forward",
           "flash_attention", "set_sdpa_precision", "_flash_attention", "_flash_attention_backward", "_decode",
           "_attn_merge", "_attn_probs"]
