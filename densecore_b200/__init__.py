"""densecore_b200 -- DenseCore's scaled-dot-product-attention path, B200-native.

A drop-in for DenseCore's flash-attention path (src/torch_attention.rs reached through
``functional.scaled_dot_product_attention``, ``nn.MultiheadAttention`` and the pyo3 functions
``_flash_attention`` / ``_flash_attention_backward``) on CUDA tensors. The kernels are
hand-written for sm_100a and live in ``libdensecore_sdpa.so`` behind the C ABI of
``include/densecore_sdpa.h``; torch provides device memory, streams and torch.distributed.
Dropout masks come from ``densecore_b200.random``, DenseCore's generator (same seeding, same
stream), drawn on the device.
"""
from . import backends, functional, nn, random
from ._native import _attn_merge, _attn_probs, _decode, _flash_attention, _flash_attention_backward
from .backends import set_sdpa_precision
from .functional import flash_attention, multi_head_attention_forward, scaled_dot_product_attention
from .random import Generator, default_generator, get_rng_state, initial_seed, manual_seed, seed, set_rng_state

__all__ = ["backends", "functional", "nn", "scaled_dot_product_attention", "multi_head_attention_forward",
           "flash_attention", "set_sdpa_precision", "_flash_attention", "_flash_attention_backward", "_decode",
           "_attn_merge", "_attn_probs", "random", "Generator", "default_generator", "manual_seed", "initial_seed",
           "seed", "get_rng_state", "set_rng_state"]
