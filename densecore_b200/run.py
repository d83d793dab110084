"""Run a PyTorch script with DenseCore's attention path on this library.

    python -m densecore_b200.run script.py [script args...]

The counterpart of DenseCore's ``scripts/run_as_torch.py`` (:15-22, the prototype of
``densecore run``): the script's ``import torch`` resolves to :mod:`densecore_b200.as_torch`,
so that its ``scaled_dot_product_attention`` and ``MultiheadAttention`` calls run the sm_100a
kernels, while tensors, autograd, optimisers and torch.distributed stay PyTorch's (unlike
DenseCore, which has no device tensors and stubs out distributed training).
"""
from __future__ import annotations

import runpy
import sys


def main(argv=None):
    argv = list(sys.argv[1:] if argv is None else argv)
    if not argv:
        print(__doc__.strip().splitlines()[2].strip(), file=sys.stderr)
        return 2
    from . import as_torch
    as_torch.install()
    script = argv[0]
    sys.argv = argv
    sys.path.insert(0, ".")
    try:
        runpy.run_path(script, run_name="__main__")
    finally:
        as_torch.uninstall()
    return 0


if __name__ == "__main__":
    sys.exit(main())
