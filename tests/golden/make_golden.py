"""Generate the golden fixtures for the SDPA path (run once; the .npz is committed).

DenseCore's own SDPA tests compare against PyTorch (tests/test_sdpa_exact.py,
tests/test_attention.py); DenseCore's flash path is a port of PyTorch's CPU flash attention
(src/torch_attention.rs:1-5). These fixtures therefore record PyTorch's CPU flash-attention
kernel (``aten::_scaled_dot_product_flash_attention_for_cpu`` and its backward), fed exactly
the way DenseCore's gate feeds its native kernel: the mask converted by ``_flash_mask``
(python/densecore/functional.py:343-364) into a contiguous (B,H,L,S) additive float mask.

Case lists and seeds follow the reference's tests:
  * ``bits_*``   -- tests/test_sdpa_exact.py:10-29, rng = default_rng(L*31+S)
  * ``mask_*``   -- tests/test_sdpa_exact.py:32-51, rng = default_rng(L+S); every mask kind
                    of the dict literal is drawn in order, as the reference's dict does
  * ``tol_*``    -- tests/test_attention.py:12-39 shapes and mask modes. The reference draws
                    from one module-level default_rng(21) in test order; here each case uses
                    default_rng(21 + case index) so the fixtures do not depend on test order.
                    Rank-3 and Ev != E cases take the reference's math path, so their outputs
                    come from torch.nn.functional.scaled_dot_product_attention (its oracle).

Usage: ``python tests/golden/make_golden.py`` (writes tests/golden/sdpa_golden.npz).
"""
from __future__ import annotations

import json
import os

import numpy as np
import torch

HERE = os.path.dirname(os.path.abspath(__file__))

BITS = [(2, 2, 7, 7, 5, False, None), (2, 2, 7, 7, 5, True, None), (1, 3, 33, 33, 16, True, None),
        (1, 2, 100, 37, 12, False, None), (1, 1, 200, 200, 8, True, None),
        (1, 1, 600, 600, 8, False, None), (1, 1, 800, 800, 4, True, None),
        (1, 2, 9, 1030, 6, False, None), (1, 2, 64, 64, 16, True, 0.3)]
MASKED = [(2, 2, 7, 7, 5), (1, 2, 200, 37, 12), (1, 1, 9, 1030, 6), (2, 3, 64, 64, 16)]
KINDS = ["bool2d", "float2d", "bool4d_b1", "float4d_1h", "row"]
TOL_SHAPES = [((2, 4, 3), (2, 5, 3), (2, 5, 2)), ((2, 3, 4, 8), (2, 3, 4, 8), (2, 3, 4, 8))]
TOL_MODES = ["none", "causal", "bool", "float"]


def flash_mask(values, qshape, source):
    """functional._flash_mask (functional.py:343-364)."""
    if values is None:
        return None
    batch, heads, length = qshape[:3]
    if values.dtype == np.bool_:
        values = np.where(values, np.float32(0.0), np.float32(-np.inf))
    return np.ascontiguousarray(np.broadcast_to(values, (batch, heads, length, source)), np.float32)


def torch_flash(q, k, v, g, mask, causal, scale):
    tq, tk, tv, tg = (torch.from_numpy(a) for a in (q, k, v, g))
    tm = None if mask is None else torch.from_numpy(mask)
    out, lse = torch.ops.aten._scaled_dot_product_flash_attention_for_cpu(
        tq, tk, tv, 0.0, causal, attn_mask=tm, scale=scale)
    gq, gk, gv = torch.ops.aten._scaled_dot_product_flash_attention_for_cpu_backward(
        tg, tq, tk, tv, out, lse, 0.0, causal, attn_mask=tm, scale=scale)
    return [t.contiguous().numpy() for t in (out, lse, gq, gk, gv)]


def torch_math(q, k, v, g, mask, causal, scale):
    ts = [torch.tensor(a, requires_grad=True) for a in (q, k, v)]
    tm = None if mask is None else torch.from_numpy(mask)
    y = torch.nn.functional.scaled_dot_product_attention(*ts, attn_mask=tm, is_causal=causal, scale=scale)
    y.backward(torch.from_numpy(g))
    return [y.detach().numpy(), None] + [t.grad.numpy() for t in ts]


def main():
    torch.set_num_threads(1)
    arrays, index = {}, []

    def put(name, meta, q, k, v, g, mask, results):
        out, lse, gq, gk, gv = results
        meta = dict(meta, name=name)
        index.append(meta)
        for key, val in dict(q=q, k=k, v=v, g=g, mask=mask, out=out, lse=lse, dq=gq, dk=gk, dv=gv).items():
            if val is not None:
                arrays[f"{name}/{key}"] = val

    for i, (B, H, L, S, E, causal, scale) in enumerate(BITS):
        rng = np.random.default_rng(L * 31 + S)
        q, g = (rng.normal(size=(B, H, L, E)).astype(np.float32) for _ in range(2))
        k, v = (rng.normal(size=(B, H, S, E)).astype(np.float32) for _ in range(2))
        put(f"bits_{i}", dict(kind="none", causal=causal, scale=scale, path="flash"), q, k, v, g, None,
            torch_flash(q, k, v, g, None, causal, scale))

    for (B, H, L, S, E) in MASKED:
        for kind in KINDS:
            rng = np.random.default_rng(L + S)
            q, g = (rng.normal(size=(B, H, L, E)).astype(np.float32) for _ in range(2))
            k, v = (rng.normal(size=(B, H, S, E)).astype(np.float32) for _ in range(2))
            masks = {"bool2d": rng.random((L, S)) > 0.3, "float2d": rng.normal(size=(L, S)).astype(np.float32),
                     "bool4d_b1": rng.random((B, 1, L, S)) > 0.5,
                     "float4d_1h": rng.normal(size=(1, H, 1, S)).astype(np.float32),
                     "row": np.zeros((L, S), bool)}
            mask = masks[kind]
            put(f"mask_{L}x{S}_{kind}", dict(kind=kind, causal=False, scale=None, path="flash"), q, k, v, g,
                mask, torch_flash(q, k, v, g, flash_mask(mask, q.shape, S), False, None))

    case = 0
    for shapes in TOL_SHAPES:
        for mode in TOL_MODES:
            rng = np.random.default_rng(21 + case)
            q, k, v = (rng.normal(size=s).astype(np.float32) for s in shapes)
            L, S = shapes[0][-2], shapes[1][-2]
            causal, mask = False, None
            if mode == "causal":
                if L != S:
                    case += 1
                    continue
                causal = True
            elif mode == "bool":
                mask = rng.random((L, S)) > .3
                mask[:, 0] = True
            elif mode == "float":
                mask = rng.normal(size=(L, S)).astype(np.float32)
            g = rng.normal(size=shapes[0][:-1] + (shapes[2][-1],)).astype(np.float32)
            flash_ok = len(shapes[0]) == 4 and shapes[2][-1] == shapes[0][-1]
            if flash_ok:
                res = torch_flash(q, k, v, g, flash_mask(mask, q.shape, S), causal, None)
            else:
                res = torch_math(q, k, v, g, mask, causal, None)
            put(f"tol_{case}", dict(kind=mode if mode in ("none", "causal") else mode + "2d", causal=causal,
                                    scale=None, path="flash" if flash_ok else "math"), q, k, v, g, mask, res)
            case += 1

    np.savez_compressed(os.path.join(HERE, "sdpa_golden.npz"), **arrays)
    with open(os.path.join(HERE, "sdpa_golden.json"), "w") as f:
        json.dump({"generator": "tests/golden/make_golden.py", "torch": torch.__version__, "cases": index}, f,
                  indent=1)
    print(f"{len(index)} cases, {sum(a.nbytes for a in arrays.values()) / 1e6:.2f} MB raw")


if __name__ == "__main__":
    main()
