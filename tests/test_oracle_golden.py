"""The CPU oracle against the golden fixtures (PyTorch's CPU flash kernel on the reference's
own test case lists), at the reference's own tolerances (tests/test_attention.py:34, :39)."""
import numpy as np
import pytest

import oracle
from conftest import load_golden

CASES = [c for c in load_golden() if c[0]["path"] == "flash"]


@pytest.mark.parametrize("meta,arr", CASES, ids=[c[0]["name"] for c in CASES])
def test_oracle_matches_golden(meta, arr):
    q, k, v, g = arr["q"], arr["k"], arr["v"], arr["g"]
    mask = oracle.flash_mask(arr.get("mask"), q.shape, k.shape[2])
    out, lse = oracle.flash_forward(q, k, v, mask, meta["causal"], meta["scale"])
    np.testing.assert_allclose(out, arr["out"], rtol=1e-5, atol=1e-6)
    np.testing.assert_allclose(lse, arr["lse"], rtol=1e-5, atol=1e-6)
    gq, gk, gv = oracle.flash_backward(g, q, k, v, out, lse, mask, meta["causal"], meta["scale"])
    for mine, ref in ((gq, arr["dq"]), (gk, arr["dk"]), (gv, arr["dv"])):
        np.testing.assert_allclose(mine, ref, rtol=1e-4, atol=1e-5)
    if meta["kind"] == "row":
        # Every row fully masked: out = 0, lse = 0 and zero gradients, exactly
        # (torch_attention.rs:223-226, :258-271).
        for a in (out, lse, gq, gk, gv):
            assert not np.any(a), "fully masked rows must give exact zeros"


def test_oracle_threads_do_not_change_bits():
    rng = np.random.default_rng(3)
    q, k, v, g = (rng.normal(size=(2, 3, 70, 16)).astype(np.float32) for _ in range(4))
    a = oracle.flash_forward(q, k, v, causal=True, threads=1)
    b = oracle.flash_forward(q, k, v, causal=True, threads=5)
    for x, y in zip(a, b):
        assert x.tobytes() == y.tobytes()
    ga = oracle.flash_backward(g, q, k, v, *a, causal=True, threads=1)
    gb = oracle.flash_backward(g, q, k, v, *a, causal=True, threads=4)
    for x, y in zip(ga, gb):
        assert x.tobytes() == y.tobytes()


def test_oracle_task_subset_matches_full_run():
    rng = np.random.default_rng(4)
    q, k, v = (rng.normal(size=(2, 4, 40, 8)).astype(np.float32) for _ in range(3))
    full = oracle.flash_forward(q, k, v, causal=True)
    part = oracle.flash_forward_tasks(q, k, v, [1, 6], causal=True)
    for t in (1, 6):
        b, h = divmod(t, 4)
        assert full[0][b, h].tobytes() == part[0][b, h].tobytes()
        assert full[1][b, h].tobytes() == part[1][b, h].tobytes()


def test_oracle_grouped_query_heads_equal_widened_heads():
    # torch_attention.rs:159-167: kv head h / repeat serves query head h.
    rng = np.random.default_rng(5)
    q, g = (rng.normal(size=(2, 4, 33, 8)).astype(np.float32) for _ in range(2))
    k, v = (rng.normal(size=(2, 2, 45, 8)).astype(np.float32) for _ in range(2))
    wide = lambda t: np.repeat(t, 2, axis=1)
    out, lse = oracle.flash_forward(q, k, v)
    ow, lw = oracle.flash_forward(q, wide(k), wide(v))
    assert out.tobytes() == ow.tobytes() and lse.tobytes() == lw.tobytes()
    gq, gk, gv = oracle.flash_backward(g, q, k, v, out, lse)
    gqw, gkw, gvw = oracle.flash_backward(g, q, wide(k), wide(v), ow, lw)
    np.testing.assert_allclose(gq, gqw, rtol=1e-6, atol=1e-6)
    np.testing.assert_allclose(gk, gkw.reshape(2, 2, 2, 45, 8).sum(2), rtol=1e-5, atol=1e-6)
    np.testing.assert_allclose(gv, gvw.reshape(2, 2, 2, 45, 8).sum(2), rtol=1e-5, atol=1e-6)


def test_oracle_rejects_bad_shapes():
    q = np.zeros((1, 3, 4, 8), np.float32)
    k = np.zeros((1, 2, 4, 8), np.float32)
    with pytest.raises(ValueError, match="shapes"):
        oracle.flash_forward(q, k, k)
    with pytest.raises(ValueError, match=r"\(B, H, L, E\)"):
        oracle.flash_forward(q[0], k[0], k[0])
