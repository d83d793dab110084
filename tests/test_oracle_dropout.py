"""The oracle's generator and dropout math path, pinned on the CPU.

* mt19937 against the reference's own known answer (src/torch_random.rs:313-323: seed 5489,
  the 10000th output is 4123659995);
* the bernoulli keep draw against PyTorch's float64 uniform stream and dropout noise
  (tests/golden/dropout_golden.npz, made by make_dropout_golden.py);
* the dropout SDPA math path (functional.py:318-340) against PyTorch's CPU SDPA with dropout
  on the reference's case list (tests/test_random_exact.py:90-103), at the reference's
  tolerances (tests/test_attention.py:34, :39).
"""
import json
import os

import numpy as np
import pytest

import oracle

HERE = os.path.dirname(os.path.abspath(__file__))
_GOLD = np.load(os.path.join(HERE, "golden", "dropout_golden.npz"))
_META = json.load(open(os.path.join(HERE, "golden", "dropout_golden.json")))["cases"]


def _cases(prefix):
    return [m for m in _META if m["name"].startswith(prefix)]


def test_mt19937_known_answer():
    g = oracle.MtGenerator(5489)
    assert int(g.random(10000)[-1]) == 4123659995


def test_state_layout_follows_the_reference():
    # manual_seed leaves left = 1, next = 0 (torch_random.rs:53-54); after one output the
    # engine has twisted: left = 624, next = 1.
    g = oracle.MtGenerator(7)
    assert g.state[624] == 1 and g.state[625] == 0
    g.random(1)
    assert g.state[624] == 624 and g.state[625] == 1
    g.random(623)
    assert g.state[624] == 1 and g.state[625] == 624


@pytest.mark.parametrize("meta", _cases("stream_"), ids=lambda m: m["name"])
def test_keep_draw_matches_torch_uniform_stream(meta):
    u = _GOLD[meta["name"]]
    for p_keep in (0.8, 0.5, 0.1, 1.0, 0.0):
        g = oracle.MtGenerator(meta["seed"])
        bits = g.keep_bits(u.size, p_keep)
        assert np.array_equal(oracle.unpack_bits(bits, u.size), u < p_keep)


@pytest.mark.parametrize("meta", _cases("noise_"), ids=lambda m: m["name"])
def test_dropout_noise_matches_torch(meta):
    noise = _GOLD[meta["name"]]
    n, p = noise.size, meta["p"]
    keep = oracle.unpack_bits(oracle.MtGenerator(meta["seed"]).keep_bits(n, 1 - p), n)
    mine = oracle.dropout_noise(keep, p).reshape(noise.shape)
    assert mine.tobytes() == noise.tobytes()


def test_draws_continue_across_calls():
    a = oracle.MtGenerator(9)
    one = oracle.unpack_bits(a.keep_bits(1000, 0.7), 1000)
    b = oracle.MtGenerator(9)
    x = oracle.unpack_bits(b.keep_bits(333, 0.7), 333)
    y = oracle.unpack_bits(b.keep_bits(667, 0.7), 667)
    assert np.array_equal(one, np.concatenate([x, y]))
    assert np.array_equal(a.state, b.state)


@pytest.mark.parametrize("meta", _cases("attn_"), ids=lambda m: m["name"])
def test_dropout_math_path_matches_torch(meta):
    arr = {k: _GOLD[f"{meta['name']}/{k}"] for k in ("q", "k", "v", "g", "out", "dq", "dk", "dv")}
    B, H, L, E = arr["q"].shape
    n = B * H * L * arr["k"].shape[2]
    keep = oracle.unpack_bits(oracle.MtGenerator(meta["seed"]).keep_bits(n, 1 - meta["p"]), n)
    noise = oracle.dropout_noise(keep, meta["p"])
    out, saved = oracle.sdpa_math_forward(arr["q"], arr["k"], arr["v"], causal=meta["causal"], scale=meta["scale"],
                                          noise=noise)
    np.testing.assert_allclose(out, arr["out"], rtol=1e-5, atol=1e-6)
    dq, dk, dv = oracle.sdpa_math_backward(arr["g"], arr["v"], saved)
    for mine, ref in ((dq, arr["dq"]), (dk, arr["dk"]), (dv, arr["dv"])):
        np.testing.assert_allclose(mine, ref, rtol=1e-4, atol=1e-5)
