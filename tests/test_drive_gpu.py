"""The drive path of the north star: a PyTorch program's ``import torch`` resolved to
``densecore_b200.as_torch`` (the counterpart of DenseCore's scripts/run_as_torch.py:15-22),
so that its ``F.scaled_dot_product_attention`` runs this library's kernels on CUDA tensors.

A one-block nanoGPT-shaped model (tests/gpt_block.py) trains a few SGD steps on CUDA in
float32 through the stand-in modules, against the same model and steps with PyTorch's own SDPA
in float64. The losses and the trained weights must agree to float32 accuracy; the library's
kernels must have run (per-launch tracing). Two shapes: DenseCore's tiny GPT (vocab 17, width
16, 2 heads of 8 -- the CUDA-core kernels) and nanoGPT-char's attention shape (width 384,
6 heads of 64, block 256 -- the tensor-core kernels, config 1's per-head shape).
"""
import os
import subprocess
import sys

import numpy as np
import pytest
import torch

import densecore_b200 as dc
from conftest import ROOT
from gpt_block import make_gpt

pytestmark = pytest.mark.gpu


def _train(T, F, model, steps, batches, device, dtype):
    model = model.to(device=device, dtype=dtype)
    opt = T.optim.SGD(model.parameters(), lr=0.1)
    losses = []
    for x, y in batches[:steps]:
        loss = model(T.tensor(x, device=device), T.tensor(y, device=device))
        opt.zero_grad()
        loss.backward()
        opt.step()
        losses.append(loss.item())
    return losses, {k: p.detach().double().cpu() for k, p in model.named_parameters()}


@pytest.mark.parametrize("vocab,n,heads,block,batch,kernel", [
    (17, 16, 2, 12, 3, "simt"),          # DenseCore's tiny GPT: head dim 8
    (65, 384, 6, 256, 4, "tc"),          # nanoGPT-char's attention: head dim 64
])
def test_tiny_gpt_trains_through_the_torch_stand_in(vocab, n, heads, block, batch, kernel):
    from densecore_b200 import as_torch
    rng = np.random.default_rng(1)
    batches = [(rng.integers(0, vocab, (batch, block)), rng.integers(0, vocab, (batch, block))) for _ in range(4)]
    T = as_torch.install()
    try:
        import torch as T2
        import torch.nn.functional as F
        assert T2 is T and F is as_torch.functional
        assert F.scaled_dot_product_attention is dc.functional.scaled_dot_product_attention
        T.manual_seed(0)
        ours = make_gpt(T, F, vocab, n, heads, block)
        dc._lib.kernel_timing_report(reset=True)
        dc._lib.kernel_timing(True)
        got_losses, got = _train(T, F, ours, 4, batches, "cuda", torch.float32)
        dc._lib.kernel_timing(False)
        launched = dc._lib.kernel_timing_report(reset=True)
    finally:
        as_torch.uninstall()
    assert sys.modules["torch"] is torch
    names = set(launched)
    if kernel == "tc":
        assert {"fwd_tc_d64", "bwd_dkdv_tc", "bwd_dq_tc"} <= names, names
    else:
        assert {"fwd_simt", "bwd_dkdv_simt", "bwd_dq_simt"} <= names, names

    torch.manual_seed(0)
    ref = make_gpt(torch, torch.nn.functional, vocab, n, heads, block)
    ref_losses, want = _train(torch, torch.nn.functional, ref, 4, batches, "cuda", torch.float64)
    np.testing.assert_allclose(got_losses, ref_losses, rtol=2e-5)
    for k in want:
        scale = float(want[k].abs().max())
        err = float((got[k] - want[k]).abs().max()) / scale
        assert err <= 1e-4, f"{k}: max|delta|/max|ref| = {err:.2e}"


def test_run_module_drives_a_script(tmp_path):
    # ``python -m densecore_b200.run script.py``: the script imports torch as usual.
    script = tmp_path / "train.py"
    script.write_text(
        "import sys\n"
        "import torch\n"
        "import torch.nn.functional as F\n"
        "from gpt_block import make_gpt\n"
        "import densecore_b200\n"
        "assert F.scaled_dot_product_attention is densecore_b200.functional.scaled_dot_product_attention\n"
        "torch.manual_seed(0)\n"
        "m = make_gpt(torch, F, 65, 128, 2, 64).cuda()\n"
        "opt = torch.optim.SGD(m.parameters(), lr=0.1)\n"
        "x = torch.randint(0, 65, (2, 64), device='cuda')\n"
        "y = torch.randint(0, 65, (2, 64), device='cuda')\n"
        "losses = []\n"
        "for _ in range(3):\n"
        "    loss = m(x, y)\n"
        "    opt.zero_grad(); loss.backward(); opt.step(); losses.append(loss.item())\n"
        "assert losses[-1] < losses[0], losses\n"
        "print('trained', sys.argv[1:], losses)\n")
    env = dict(os.environ, PYTHONPATH=os.pathsep.join([ROOT, os.path.join(ROOT, "tests")]))
    r = subprocess.run([sys.executable, "-m", "densecore_b200.run", str(script), "--flag"], capture_output=True,
                       text=True, env=env, cwd=str(tmp_path), timeout=300)
    assert r.returncode == 0, r.stderr[-2000:]
    assert "trained ['--flag']" in r.stdout
