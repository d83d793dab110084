"""A ``torch`` that runs DenseCore's attention path on this library.

DenseCore drives unmodified PyTorch scripts (nanoGPT) by making ``import torch`` resolve to
itself: ``scripts/run_as_torch.py:15-22`` puts ``densecore``, ``densecore.nn``,
``densecore.nn.functional``, ... into ``sys.modules`` under torch's names and runs the script.
DenseCore's tensors live on the CPU (``src/tensor.rs``; ``python/densecore/tensor.py:374-390``
refuses ``.to('cuda')``). Here the same switch keeps PyTorch's device tensors, autograd engine
and optimisers -- CUDA tensors, ``.to('cuda')`` and ``backward()`` work as in torch -- and swaps
in this library exactly where DenseCore's hot path is:

- ``torch.nn.functional.scaled_dot_product_attention`` -> :func:`densecore_b200.functional.
  scaled_dot_product_attention` (DenseCore's ``functional.py:276-340``), which nanoGPT's
  ``CausalSelfAttention`` calls when ``hasattr(F, 'scaled_dot_product_attention')``;
- ``torch.nn.functional.multi_head_attention_forward`` and ``torch.nn.MultiheadAttention`` ->
  this package's (``functional.py:400-461``, ``nn.py:595-640``);
- ``torch.manual_seed`` also seeds DenseCore's generator (:mod:`densecore_b200.random`), from
  which the fused kernels draw dropout masks, as ``densecore.manual_seed`` does.

Everything else is PyTorch's own object, reached through the stand-in modules. Use
:func:`install` / :func:`uninstall` around code that imports torch, or run a script with
``python -m densecore_b200.run script.py [args]``.
"""
from __future__ import annotations

import sys
import types

import torch as _torch
import torch.nn as _nn
import torch.nn.functional as _F

from . import functional as _dc_functional
from . import nn as _dc_nn
from . import random as _dc_random

_NAMES = ("torch", "torch.nn", "torch.nn.functional")


class _StandIn(types.ModuleType):
    """A module object that answers with its own overrides first, then the real module's."""

    def __init__(self, name, real, overrides):
        super().__init__(name, getattr(real, "__doc__", None))
        self.__dict__["_real"] = real
        self.__dict__.update(overrides)
        self.__dict__["__densecore_b200__"] = True

    def __getattr__(self, attr):
        return getattr(self.__dict__["_real"], attr)

    def __dir__(self):
        return sorted(set(dir(self.__dict__["_real"])) | set(self.__dict__))


def _manual_seed(seed):
    _dc_random.manual_seed(seed)
    return _torch.manual_seed(seed)


functional = _StandIn("torch.nn.functional", _F, {
    "scaled_dot_product_attention": _dc_functional.scaled_dot_product_attention,
    "multi_head_attention_forward": _dc_functional.multi_head_attention_forward,
})
nn = _StandIn("torch.nn", _nn, {"functional": functional, "MultiheadAttention": _dc_nn.MultiheadAttention})
torch = _StandIn("torch", _torch, {"nn": nn, "manual_seed": _manual_seed})

_saved = None


def install():
    """Make ``import torch`` (and ``torch.nn``, ``torch.nn.functional``) resolve to the
    stand-ins until :func:`uninstall`. Modules imported before keep what they imported."""
    global _saved
    if _saved is None:
        _saved = {n: sys.modules.get(n) for n in _NAMES}
    sys.modules.update({"torch": torch, "torch.nn": nn, "torch.nn.functional": functional})
    return torch


def uninstall():
    """Put PyTorch's own modules back under their names."""
    global _saved
    if _saved is None:
        return
    for n, m in _saved.items():
        if m is None:
            sys.modules.pop(n, None)
        else:
            sys.modules[n] = m
    _saved = None
