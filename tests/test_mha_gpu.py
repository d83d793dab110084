"""nn.MultiheadAttention on the fused kernels against PyTorch's module on CPU, with the
reference's own four configurations and tolerances (tests/test_multihead_attention.py:19-54),
plus config 2's shape (batch_first, E=512, 8 heads, key padding lengths in [16, 128])."""
import numpy as np
import pytest
import torch

import densecore_b200 as dc

pytestmark = pytest.mark.gpu


def pair(**kwargs):
    theirs = torch.nn.MultiheadAttention(**kwargs)
    ours = dc.nn.MultiheadAttention(**kwargs).cuda()
    names = dict(theirs.named_parameters())
    with torch.no_grad():
        for name, p in ours.named_parameters():
            p.copy_(names[name].detach())
    assert sorted(dict(ours.named_parameters())) == sorted(names)
    return ours, theirs


@pytest.mark.parametrize('kwargs,call', [
    (dict(embed_dim=8, num_heads=2), {}),
    (dict(embed_dim=8, num_heads=4, batch_first=True), {'average_attn_weights': False}),
    (dict(embed_dim=8, num_heads=2, kdim=5, vdim=3, add_bias_kv=True, add_zero_attn=True), {}),
    (dict(embed_dim=8, num_heads=2, bias=False), {'need_weights': False}),
])
def test_multihead_attention_matches_torch(kwargs, call):
    ours, theirs = pair(**kwargs)
    rng = np.random.default_rng(0)
    first = (2, 4) if kwargs.get('batch_first') else (4, 2)
    q = rng.normal(size=first + (8,)).astype(np.float32)
    k = rng.normal(size=(first[0], first[1] + 1) + (kwargs.get('kdim', 8),) if kwargs.get('batch_first') else
                   (first[0] + 1, first[1], kwargs.get('kdim', 8))).astype(np.float32)
    v = rng.normal(size=k.shape[:2] + (kwargs.get('vdim', 8),)).astype(np.float32)
    src = k.shape[1] if kwargs.get('batch_first') else k.shape[0]
    padding = np.zeros((2, src), bool)
    padding[1, -1] = True
    mask = np.triu(np.ones((4, src), bool), 2)
    tq = torch.tensor(q, requires_grad=True)
    out, weights = theirs(tq, torch.tensor(k), torch.tensor(v), key_padding_mask=torch.tensor(padding),
                          attn_mask=torch.tensor(mask), **call)
    dq = torch.tensor(q, device="cuda", requires_grad=True)
    got, got_weights = ours(dq, torch.tensor(k, device="cuda"), torch.tensor(v, device="cuda"),
                            key_padding_mask=torch.tensor(padding, device="cuda"),
                            attn_mask=torch.tensor(mask, device="cuda"), **call)
    np.testing.assert_allclose(got.detach().cpu().numpy(), out.detach().numpy(), rtol=1e-5, atol=1e-6)
    if weights is None:
        assert got_weights is None
    else:
        np.testing.assert_allclose(got_weights.cpu().numpy(), weights.detach().numpy(), rtol=1e-5, atol=1e-6)
    w = rng.normal(size=out.shape).astype(np.float32)
    (out * torch.tensor(w)).sum().backward()
    (got * torch.tensor(w, device="cuda")).sum().backward()
    np.testing.assert_allclose(dq.grad.cpu().numpy(), tq.grad.numpy(), rtol=1e-4, atol=1e-5)
    grads = dict(theirs.named_parameters())
    for name, p in ours.named_parameters():
        np.testing.assert_allclose(p.grad.cpu().numpy(), grads[name].grad.numpy(), rtol=1e-4, atol=1e-5,
                                   err_msg=name)


def test_config2_shape_matches_torch():
    torch.manual_seed(0)
    B, L, E, H = 32, 128, 512, 8
    ours, theirs = pair(embed_dim=E, num_heads=H, batch_first=True)
    rng = np.random.default_rng(1)
    x = rng.normal(size=(B, L, E)).astype(np.float32)
    lengths = rng.integers(16, 129, size=B)
    pad = np.arange(L)[None, :] >= lengths[:, None]
    tx = torch.tensor(x, requires_grad=True)
    out, wts = theirs(tx, tx, tx, key_padding_mask=torch.tensor(pad))
    cx = torch.tensor(x, device="cuda", requires_grad=True)
    got, gw = ours(cx, cx, cx, key_padding_mask=torch.tensor(pad, device="cuda"))
    scale = float(out.abs().max())
    assert float((got.detach().cpu() - out.detach()).abs().max()) <= 1e-5 * scale + 1e-6
    assert float((gw.cpu() - wts.detach()).abs().max()) <= 1e-5
    g = rng.normal(size=out.shape).astype(np.float32)
    out.backward(torch.tensor(g))
    got.backward(torch.tensor(g, device="cuda"))
    ref = tx.grad.numpy()
    assert np.abs(cx.grad.cpu().numpy() - ref).max() <= 1e-5 * np.abs(ref).max() + 1e-6
    grads = dict(theirs.named_parameters())
    for name, p in ours.named_parameters():
        r = grads[name].grad.numpy()
        assert np.abs(p.grad.cpu().numpy() - r).max() <= 1e-5 * np.abs(r).max() + 1e-6, name


def test_fully_masked_rows_are_nan_like_the_reference():
    ours, _ = pair(embed_dim=16, num_heads=2, batch_first=True)
    x = torch.randn(2, 5, 16, device="cuda", requires_grad=True)
    pad = torch.zeros(2, 5, dtype=torch.bool, device="cuda")
    pad[1] = True  # batch 1 sees no key at all
    out, w = ours(x, x, x, key_padding_mask=pad)
    assert torch.isnan(out[1]).all() and not torch.isnan(out[0]).any()
    assert torch.isnan(w[1]).all() and not torch.isnan(w[0]).any()
