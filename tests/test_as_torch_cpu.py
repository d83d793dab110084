"""The torch stand-in of densecore_b200.as_torch on the CPU (no kernel runs): which names it
swaps for this library's, that everything else is PyTorch's own object, that the usual import
forms resolve to it, and that uninstall puts torch back. The counterpart of DenseCore's
scripts/run_as_torch.py:15-22."""
import os
import subprocess
import sys

import torch

import densecore_b200 as dc
from conftest import ROOT


def test_stand_in_swaps_only_the_attention_path():
    from densecore_b200 import as_torch
    T = as_torch.torch
    assert T.nn.functional.scaled_dot_product_attention is dc.functional.scaled_dot_product_attention
    assert T.nn.functional.multi_head_attention_forward is dc.functional.multi_head_attention_forward
    assert T.nn.MultiheadAttention is dc.nn.MultiheadAttention
    assert T.Tensor is torch.Tensor and T.optim is torch.optim and T.nn.Linear is torch.nn.Linear
    assert T.nn.functional.gelu is torch.nn.functional.gelu
    assert T.cuda is torch.cuda and T.float32 is torch.float32
    T.manual_seed(5)
    a = torch.rand(3)
    torch.manual_seed(5)
    assert torch.equal(a, torch.rand(3))
    assert dc.random.initial_seed() == 5  # DenseCore's generator is seeded too


def test_import_forms_resolve_to_the_stand_in_and_uninstall_restores():
    from densecore_b200 import as_torch
    real = sys.modules["torch"]
    as_torch.install()
    try:
        import torch as t1
        import torch.nn as nn1
        import torch.nn.functional as f1
        from torch.nn import functional as f2
        from torch import nn as nn2
        assert t1 is as_torch.torch and nn1 is as_torch.nn and nn2 is as_torch.nn
        assert f1 is as_torch.functional and f2 is as_torch.functional
    finally:
        as_torch.uninstall()
    assert sys.modules["torch"] is real and sys.modules["torch.nn.functional"] is torch.nn.functional


def test_run_module_resolves_the_script_imports(tmp_path):
    script = tmp_path / "probe.py"
    script.write_text("import sys, torch, torch.nn.functional as F\n"
                      "import densecore_b200\n"
                      "assert F.scaled_dot_product_attention is densecore_b200.functional.scaled_dot_product_attention\n"
                      "assert getattr(torch, '__densecore_b200__', False)\n"
                      "print('argv', sys.argv)\n")
    env = dict(os.environ, PYTHONPATH=ROOT)
    r = subprocess.run([sys.executable, "-m", "densecore_b200.run", str(script), "a", "b"], capture_output=True,
                       text=True, env=env, cwd=str(tmp_path), timeout=300)
    assert r.returncode == 0, r.stderr[-2000:]
    assert f"argv ['{script}', 'a', 'b']" in r.stdout
