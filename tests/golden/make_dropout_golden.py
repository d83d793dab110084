"""Generate the golden fixtures for attention dropout (run once; the .npz is committed).

DenseCore's dropout is PyTorch's, bit for bit (python/densecore/_random.py:1-7): the mask is
``noise.bernoulli_(1 - p)`` drawn from the mt19937 CPU generator seeded by ``manual_seed``
(src/torch_random.rs:242-254), divided by float32(1 - p) (functional.py:638-641), and
``scaled_dot_product_attention`` with ``dropout_p > 0`` takes the math path
(functional.py:312-340). DenseCore's own test of that path compares against PyTorch's CPU
SDPA (tests/test_random_exact.py:90-103); these fixtures record the same thing with the same
case list and seeds:

  * ``stream_<seed>``   -- torch.rand(n, dtype=float64) after manual_seed(seed): the 53-bit
                           uniforms the bernoulli draw compares against ``1 - p``;
  * ``noise_<seed>``    -- torch.nn.functional.dropout(ones, p) after manual_seed(seed): the
                           keep mask times 1/float32(1 - p), in (B, H, L, S) element order;
  * ``attn_<i>``        -- test_random_exact.py:90-103: shapes (2,4,64,32), (1,2,7,5),
                           (2,3,9,4) x (causal, scale) in ((True, None), (False, 0.3),
                           (False, -0.5)), inputs from default_rng(0), manual_seed(5),
                           dropout_p 0.2; output and the gradients of q, k, v.

Usage: ``python tests/golden/make_dropout_golden.py`` (writes tests/golden/dropout_golden.npz).
"""
from __future__ import annotations

import json
import os

import numpy as np
import torch

HERE = os.path.dirname(os.path.abspath(__file__))

STREAM_SEEDS = [0, 5, 1337, 2**40 + 7, -5]
NOISE = [(3, (2, 3, 17, 33), 0.2), (11, (1, 2, 64, 64), 0.5), (7, (4, 5, 9), 0.9)]
ATTN_SHAPES = [(2, 4, 64, 32), (1, 2, 7, 5), (2, 3, 9, 4)]
ATTN_MODES = [(True, None), (False, 0.3), (False, -0.5)]


def main():
    torch.set_num_threads(1)
    arrays, index = {}, []
    for seed in STREAM_SEEDS:
        torch.manual_seed(seed)
        arrays[f"stream_{seed}"] = torch.rand(4099, dtype=torch.float64).numpy()
        index.append(dict(name=f"stream_{seed}", seed=seed, n=4099))
    for seed, shape, p in NOISE:
        torch.manual_seed(seed)
        arrays[f"noise_{seed}"] = torch.nn.functional.dropout(torch.ones(shape), p, True).numpy()
        index.append(dict(name=f"noise_{seed}", seed=seed, shape=list(shape), p=p))
    case = 0
    for shape in ATTN_SHAPES:
        for causal, scale in ATTN_MODES:
            r = np.random.default_rng(0)
            q, k, v, g = (r.normal(size=shape).astype(np.float32) for _ in range(4))
            torch.manual_seed(5)
            ts = [torch.tensor(a, requires_grad=True) for a in (q, k, v)]
            y = torch.nn.functional.scaled_dot_product_attention(*ts, dropout_p=0.2, is_causal=causal, scale=scale)
            y.backward(torch.tensor(g))
            name = f"attn_{case}"
            for key, val in dict(q=q, k=k, v=v, g=g, out=y.detach().numpy(), dq=ts[0].grad.numpy(),
                                 dk=ts[1].grad.numpy(), dv=ts[2].grad.numpy()).items():
                arrays[f"{name}/{key}"] = val
            index.append(dict(name=name, shape=list(shape), causal=causal, scale=scale, seed=5, p=0.2))
            case += 1
    np.savez_compressed(os.path.join(HERE, "dropout_golden.npz"), **arrays)
    with open(os.path.join(HERE, "dropout_golden.json"), "w") as f:
        json.dump({"generator": "tests/golden/make_dropout_golden.py", "torch": torch.__version__, "cases": index},
                  f, indent=1)
    print(f"{len(index)} cases, {sum(a.nbytes for a in arrays.values()) / 1e6:.2f} MB raw")


if __name__ == "__main__":
    main()
