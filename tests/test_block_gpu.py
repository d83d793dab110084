"""The drop-in case of the north star: a GPT-style causal self-attention block whose attention
call is ``densecore_b200.scaled_dot_product_attention`` on CUDA tensors, against the same
block in float64 on the CPU with PyTorch's SDPA. The block is written here the way GPT-2 /
nanoGPT-shaped models lay it out: one fused q/k/v projection, heads split by view + transpose
(non-contiguous (B, H, T, D) views that the kernels read in place), causal attention, heads
merged, output projection. Forward output, the input gradient and every weight gradient must
match within the 3xTF32 tolerance, max|delta| <= 1e-5 * max|ref|, also after a few SGD steps.
"""
import numpy as np
import pytest
import torch
import torch.nn as nn

import densecore_b200 as dc
from conftest import rel_err

pytestmark = pytest.mark.gpu


class Block(nn.Module):
    def __init__(self, n_embd, n_head, attention):
        super().__init__()
        self.n_head = n_head
        self.qkv = nn.Linear(n_embd, 3 * n_embd)
        self.proj = nn.Linear(n_embd, n_embd)
        self.attention = attention

    def forward(self, x):
        B, T, C = x.shape
        q, k, v = self.qkv(x).split(C, dim=2)
        heads = lambda t: t.view(B, T, self.n_head, C // self.n_head).transpose(1, 2)
        y = self.attention(heads(q), heads(k), heads(v), is_causal=True)
        return self.proj(y.transpose(1, 2).contiguous().view(B, T, C))


def _pair(n_embd, n_head, seed):
    torch.manual_seed(seed)
    ref = Block(n_embd, n_head, torch.nn.functional.scaled_dot_product_attention).double()
    ours = Block(n_embd, n_head, dc.scaled_dot_product_attention).cuda()
    with torch.no_grad():
        for (_, a), (_, b) in zip(ours.named_parameters(), ref.named_parameters()):
            a.copy_(b.float())
    return ours, ref


@pytest.mark.parametrize("B,T,n_embd,n_head", [(4, 256, 384, 6), (2, 300, 768, 12), (2, 128, 1024, 8)])
def test_causal_self_attention_block_forward_backward(B, T, n_embd, n_head):
    ours, ref = _pair(n_embd, n_head, 0)
    rng = np.random.default_rng(1)
    x = rng.normal(size=(B, T, n_embd)).astype(np.float32)
    g = rng.normal(size=(B, T, n_embd)).astype(np.float32)
    xo = torch.tensor(x, device="cuda", requires_grad=True)
    xr = torch.tensor(x, dtype=torch.float64, requires_grad=True)
    yo, yr = ours(xo), ref(xr)
    yo.backward(torch.tensor(g, device="cuda"))
    yr.backward(torch.tensor(g, dtype=torch.float64))
    assert rel_err(yo.detach().cpu().numpy(), yr.detach().numpy()) <= 1e-5
    assert rel_err(xo.grad.cpu().numpy(), xr.grad.numpy()) <= 1e-5
    for (name, a), (_, b) in zip(ours.named_parameters(), ref.named_parameters()):
        assert rel_err(a.grad.cpu().numpy(), b.grad.numpy()) <= 1e-5, name


def test_block_training_steps_track_the_float64_reference():
    ours, ref = _pair(384, 6, 3)
    opt_o = torch.optim.SGD(ours.parameters(), lr=0.05)
    opt_r = torch.optim.SGD(ref.parameters(), lr=0.05)
    rng = np.random.default_rng(4)
    for _ in range(3):
        x = rng.normal(size=(2, 256, 384)).astype(np.float32)
        t = rng.normal(size=(2, 256, 384)).astype(np.float32)
        for model, opt, dev, dt in ((ours, opt_o, "cuda", torch.float32), (ref, opt_r, "cpu", torch.float64)):
            opt.zero_grad()
            y = model(torch.tensor(x, device=dev, dtype=dt))
            loss = ((y - torch.tensor(t, device=dev, dtype=dt)) ** 2).mean()
            loss.backward()
            opt.step()
    for (name, a), (_, b) in zip(ours.named_parameters(), ref.named_parameters()):
        assert rel_err(a.detach().cpu().numpy(), b.detach().numpy()) <= 1e-5, name
