"""Argument checks of scaled_dot_product_attention, ported from the reference's
tests/test_attention.py:50-63; they raise before any device work, so they run on CPU."""
import numpy as np
import pytest
import torch

import densecore_b200 as dc

RNG = np.random.default_rng(21)


def _t(*shape):
    return torch.from_numpy(RNG.normal(size=shape).astype(np.float32))


def test_rejections_match_reference():
    q, k, v = _t(1, 2, 4), _t(1, 3, 4), _t(1, 3, 5)
    sdpa = dc.functional.scaled_dot_product_attention
    with pytest.raises(ValueError, match="both"):
        sdpa(q, k, v, attn_mask=np.ones((2, 3), bool), is_causal=True)
    with pytest.raises(ValueError, match="shapes"):
        sdpa(q, _t(1, 3, 3), v)
    with pytest.raises(ValueError, match="rank"):
        sdpa(q.reshape(2, 4), k, v)
    with pytest.raises(TypeError):
        sdpa(q, k, v, is_causal=1)
    with pytest.raises(TypeError):
        sdpa(q, k, v, scale="x")
    with pytest.raises(TypeError):
        sdpa(q.numpy(), k, v)
    # functional.py:219-226 (dropout's own checks), then the device check before any draw.
    with pytest.raises(ValueError, match=r"\[0, 1\]"):
        sdpa(q, k, v, dropout_p=1.5)
    with pytest.raises(TypeError, match="real"):
        sdpa(q, k, v, dropout_p=True)
    with pytest.raises(TypeError, match="real"):
        sdpa(q, k, v, dropout_p="x")
    state = dc.get_rng_state()
    with pytest.raises(RuntimeError, match="CUDA"):
        sdpa(q, k, v, dropout_p=0.1)
    assert torch.equal(dc.get_rng_state(), state)  # the refused call drew nothing
    with pytest.raises(TypeError):
        sdpa(q.double(), k, v)


def test_precision_switch():
    from densecore_b200 import backends
    assert backends.precision_name() == "3xtf32"
    backends.cuda.matmul.allow_tf32 = True
    try:
        assert backends.precision_name() == "tf32"
    finally:
        backends.cuda.matmul.allow_tf32 = False
    dc.set_sdpa_precision("fp32")
    try:
        assert backends.precision_code() == 2
    finally:
        dc.set_sdpa_precision(None)
    with pytest.raises(ValueError):
        dc.set_sdpa_precision("fp16")


def test_mha_module_parameters_follow_torch():
    m = dc.nn.MultiheadAttention(16, 4)
    t = torch.nn.MultiheadAttention(16, 4)
    assert sorted(n for n, _ in m.named_parameters()) == sorted(n for n, _ in t.named_parameters())
    m2 = dc.nn.MultiheadAttention(8, 2, kdim=5, vdim=3, add_bias_kv=True)
    t2 = torch.nn.MultiheadAttention(8, 2, kdim=5, vdim=3, add_bias_kv=True)
    assert sorted(n for n, _ in m2.named_parameters()) == sorted(n for n, _ in t2.named_parameters())
    with pytest.raises(AssertionError):
        dc.nn.MultiheadAttention(10, 4)
