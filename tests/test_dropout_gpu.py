"""Dropout on the device against the oracle and PyTorch's CPU values.

* dc_dropout_keep_bits: the packed keep mask and the advanced engine state are bit-identical
  to the oracle's sequential mt19937 + bernoulli (src/torch_random.rs:43-110, :242-254), from
  seeded, part-used and block-end states, for sizes from one element to several chunks of the
  parallel walk per CTA (one and two jump levels);
* scaled_dot_product_attention with dropout_p > 0: the reference's case list
  (tests/test_random_exact.py:90-103, fixtures from PyTorch's CPU SDPA) at the reference's
  tolerances (tests/test_attention.py:34, :39), and masks, grouped-query heads, rank 3 and
  Ev != E against the oracle's math path (functional.py:318-340) at 1e-5 * max|ref|;
* nn.MultiheadAttention training with dropout against PyTorch's CPU module;
* the stream: consecutive calls continue it, manual_seed repeats it, p == 1 draws nothing.
"""
import ctypes
import json
import os

import numpy as np
import pytest
import torch

import densecore_b200 as dc
import oracle
from conftest import rel_err
from densecore_b200 import _lib

pytestmark = pytest.mark.gpu

HERE = os.path.dirname(os.path.abspath(__file__))
CHUNK_ELEMS = 624 * 210 // 2  # elements per chunk of the parallel walk


def _device_bits(state, n, keep_prob, in_place=False):
    st_in = torch.from_numpy(state.view(np.int32).copy()).cuda()
    st_out = st_in if in_place else torch.zeros_like(st_in)
    bits = torch.full((max((n + 31) // 32, 1),), -1, dtype=torch.int32, device="cuda")
    L = _lib.load()
    st = L.dc_dropout_keep_bits(st_in.data_ptr(), st_out.data_ptr(), n, keep_prob, bits.data_ptr(),
                                torch.cuda.current_stream().cuda_stream)
    _lib.check(st, "keep bits")
    torch.cuda.synchronize()
    return bits.cpu().numpy().view(np.uint32)[:(n + 31) // 32], st_out.cpu().numpy().view(np.uint32)


@pytest.mark.parametrize("seed,pre,n", [
    (5, 0, 1), (5, 0, 31), (5, 0, 32), (5, 0, 33), (7, 1, 1000), (9, 623, 4099), (11, 624, 100_000),
    (13, 300, CHUNK_ELEMS - 3), (2, 0, 3 * CHUNK_ELEMS + 77), (4, 17, 35 * CHUNK_ELEMS + 5),
    # more chunks than SMs: CTAs own runs of several chunks (the last: config 3's weights)
    (6, 400, 160 * CHUNK_ELEMS + 11), (3, 0, 8 * 12 * 1024 * 1024)])
@pytest.mark.parametrize("keep_prob", [0.8, 0.5])
def test_keep_bits_match_oracle(seed, pre, n, keep_prob):
    g = oracle.MtGenerator(seed).discard(pre)
    bits, state = _device_bits(g.state.copy(), n, keep_prob)
    ref = g.keep_bits(n, keep_prob)
    assert np.array_equal(bits, ref)
    assert np.array_equal(state, g.state)


@pytest.mark.parametrize("keep_prob", [1.0, 0.0])
def test_keep_bits_edge_probabilities(keep_prob):
    g = oracle.MtGenerator(3)
    n = 1000
    bits, state = _device_bits(g.state.copy(), n, keep_prob)
    assert np.array_equal(bits, g.keep_bits(n, keep_prob))
    assert np.array_equal(state, g.state)
    full = oracle.unpack_bits(bits, n)
    assert full.all() if keep_prob == 1.0 else not full.any()


@pytest.mark.parametrize("e0", [5, 700, 3 * CHUNK_ELEMS + 17])
def test_keep_bits_threshold_ties(e0):
    # The device decides most draws on the high 21 bits alone and tempers the low word only
    # when those equal the threshold's: put the threshold on draw e0 (just above and exactly
    # at it), so e0 takes that path, in the first chunk and past a jump.
    g = oracle.MtGenerator(17).discard(3)
    n = 4 * CHUNK_ELEMS
    words = oracle.MtGenerator(17).discard(3).random(2 * e0 + 2)
    m = (int(words[2 * e0]) & 0x1FFFFF) << 32 | int(words[2 * e0 + 1])
    for thresh, kept in ((m + 1, True), (m, False)):
        keep_prob = thresh / 2.0 ** 53  # exact: thresh < 2^53
        bits, state = _device_bits(g.state.copy(), n, keep_prob)
        gg = oracle.MtGenerator(17).discard(3)
        ref = gg.keep_bits(n, keep_prob)
        assert np.array_equal(bits, ref)
        assert np.array_equal(state, gg.state)
        assert bool((bits[e0 // 32] >> (e0 % 32)) & 1) == kept


def test_keep_bits_in_place_state():
    g = oracle.MtGenerator(8).discard(5)
    n = 2 * CHUNK_ELEMS + 1
    bits, state = _device_bits(g.state.copy(), n, 0.7, in_place=True)
    assert np.array_equal(bits, g.keep_bits(n, 0.7))
    assert np.array_equal(state, g.state)


def test_keep_bits_across_launches():
    # Past (2048 - 2) chunks of words one call takes a second launch, which starts from the
    # first launch's end state (in place: through the library's temporary state copies).
    g = oracle.MtGenerator(12).discard(77)
    n = 2046 * CHUNK_ELEMS + 12_345
    bits, state = _device_bits(g.state.copy(), n, 0.75, in_place=True)
    assert np.array_equal(bits, g.keep_bits(n, 0.75))
    assert np.array_equal(state, g.state)


def test_invalid_state_is_reported_not_used():
    L = _lib.load()
    L.dc_device_status(1)
    bad = oracle.MtGenerator(1).state.copy()
    bad[624] = 0
    st_in = torch.from_numpy(bad.view(np.int32).copy()).cuda()
    st_out = torch.full_like(st_in, 7)
    bits = torch.full((4,), 5, dtype=torch.int32, device="cuda")
    _lib.check(L.dc_dropout_keep_bits(st_in.data_ptr(), st_out.data_ptr(), 100, 0.5, bits.data_ptr(),
                                      torch.cuda.current_stream().cuda_stream), "keep bits")
    assert L.dc_device_status(1) == 2
    assert L.dc_device_status(0) == 0
    assert (st_out == 7).all() and (bits == 5).all()
    with pytest.raises(ValueError, match=r"\[0, 1\]"):
        _lib.check(L.dc_dropout_keep_bits(st_in.data_ptr(), st_out.data_ptr(), 100, 1.5, bits.data_ptr(), None), "x")


def test_generator_stream_continues_across_calls():
    dc.manual_seed(9)
    a = dc.random.dropout_keep_bits(1000, 0.6, torch.device("cuda"))
    b = dc.random.dropout_keep_bits(777, 0.6, torch.device("cuda"))
    g = oracle.MtGenerator(9)
    assert np.array_equal(a.cpu().numpy().view(np.uint32), g.keep_bits(1000, 0.6))
    assert np.array_equal(b.cpu().numpy().view(np.uint32), g.keep_bits(777, 0.6))
    w = dc.get_rng_state().numpy().view(np.uint64)
    assert list(w[1:3]) == list(g.state[624:]) and np.array_equal(w[7:].astype(np.uint32), g.state[:624])


_GOLD = np.load(os.path.join(HERE, "golden", "dropout_golden.npz"))
_META = [m for m in json.load(open(os.path.join(HERE, "golden", "dropout_golden.json")))["cases"]
         if m["name"].startswith("attn_")]


@pytest.mark.parametrize("meta", _META, ids=lambda m: m["name"])
def test_sdpa_dropout_matches_torch_cases(meta):
    arr = {k: _GOLD[f"{meta['name']}/{k}"] for k in ("q", "k", "v", "g", "out", "dq", "dk", "dv")}
    dc.manual_seed(meta["seed"])
    t = [torch.tensor(arr[x], device="cuda", requires_grad=True) for x in ("q", "k", "v")]
    y = dc.functional.scaled_dot_product_attention(*t, dropout_p=meta["p"], is_causal=meta["causal"],
                                                   scale=meta["scale"])
    y.backward(torch.tensor(arr["g"], device="cuda"))
    # The reference's tolerances (rtol 1e-5 / 1e-4), with the absolute term raised to the
    # north star's 1e-5 * max|ref|: PyTorch's math path scales q and k by sqrt|scale| before
    # the product, the fused kernels scale the product, so single small outputs can differ by
    # a few ulps of the row's largest terms.
    out = arr["out"]
    np.testing.assert_allclose(y.detach().cpu().numpy(), out, rtol=1e-5, atol=max(1e-6, 1e-5 * np.abs(out).max()))
    for tt, key in zip(t, ("dq", "dk", "dv")):
        np.testing.assert_allclose(tt.grad.cpu().numpy(), arr[key], rtol=1e-4, atol=1e-5)


def _oracle_case(q, k, v, mask, causal, scale, p, seed):
    B, H, L = q.shape[:3]
    n = B * H * L * k.shape[2]
    keep = oracle.unpack_bits(oracle.MtGenerator(seed).keep_bits(n, 1 - p), n)
    return oracle.sdpa_math_forward(q, k, v, mask=mask, causal=causal, scale=scale,
                                    noise=oracle.dropout_noise(keep, p))


@pytest.mark.parametrize("shape,kind,causal,scale", [
    ((2, 3, 40, 24, 16, 16), "bool", False, None), ((1, 2, 33, 70, 8, 8), "float", False, 0.7),
    ((2, 2, 64, 64, 32, 32), None, True, None), ((1, 4, 19, 27, 12, 20), "bool4", False, -0.4),
    ((1, 2, 1024, 1024, 64, 64), None, True, None),
    # head dims the tensor-core kernels take: keep bits at unaligned offsets (S not a multiple
    # of 32), masks, and the D = 128 forward
    ((2, 3, 200, 173, 64, 64), "bool", False, None), ((2, 2, 130, 257, 64, 64), "float", False, 0.2),
    ((1, 2, 300, 300, 128, 128), None, True, 0.3), ((1, 2, 97, 200, 64, 64), None, True, None)])
def test_sdpa_dropout_matches_oracle(shape, kind, causal, scale):
    B, H, L, S, E, Ev = shape
    rng = np.random.default_rng(L + S)
    q, g = rng.normal(size=(B, H, L, E)).astype(np.float32), rng.normal(size=(B, H, L, Ev)).astype(np.float32)
    k, v = rng.normal(size=(B, H, S, E)).astype(np.float32), rng.normal(size=(B, H, S, Ev)).astype(np.float32)
    mask = {"bool": rng.random((L, S)) > 0.3, "float": rng.normal(size=(L, S)).astype(np.float32),
            "bool4": rng.random((B, 1, L, S)) > 0.5, None: None}[kind]
    if kind in ("bool", "bool4"):
        mask[..., 0, :] = False  # one fully masked row: output and gradients 0 there
    p = 0.3
    ref, saved = _oracle_case(q, k, v, mask, causal, scale, p, 11)
    dq, dk, dv = oracle.sdpa_math_backward(g, v, saved)
    dc.manual_seed(11)
    t = [torch.tensor(a, device="cuda", requires_grad=True) for a in (q, k, v)]
    m = None if mask is None else torch.tensor(mask, device="cuda")
    y = dc.functional.scaled_dot_product_attention(*t, attn_mask=m, dropout_p=p, is_causal=causal, scale=scale)
    y.backward(torch.tensor(g, device="cuda"))
    assert rel_err(y.detach().cpu().numpy(), ref) <= 1e-5
    for tt, r in zip(t, (dq, dk, dv)):
        assert rel_err(tt.grad.cpu().numpy(), r) <= 1e-5
    if kind in ("bool", "bool4"):
        row = y.detach().cpu().numpy()[..., 0, :]
        assert not row.any()


def test_sdpa_dropout_rank3_and_grouped_heads():
    rng = np.random.default_rng(4)
    # rank 3: (N, L, E) -- the reference's weights are (N, L, S), the same element order.
    q, k, v = (rng.normal(size=(3, 21, 8)).astype(np.float32) for _ in range(3))
    ref, _ = _oracle_case(q[:, None], k[:, None], v[:, None], None, False, None, 0.25, 6)
    dc.manual_seed(6)
    y = dc.functional.scaled_dot_product_attention(*(torch.tensor(a, device="cuda") for a in (q, k, v)),
                                                   dropout_p=0.25)
    assert rel_err(y.cpu().numpy(), ref[:, 0]) <= 1e-5
    # grouped-query heads: the reference widens K/V (functional.py:292-297).
    q = rng.normal(size=(2, 4, 17, 8)).astype(np.float32)
    k, v = (rng.normal(size=(2, 2, 23, 8)).astype(np.float32) for _ in range(2))
    wide = lambda a: np.repeat(a, 2, axis=1)
    ref, _ = _oracle_case(q, wide(k), wide(v), None, False, None, 0.4, 7)
    dc.manual_seed(7)
    y = dc.functional.scaled_dot_product_attention(*(torch.tensor(a, device="cuda") for a in (q, k, v)),
                                                   dropout_p=0.4, enable_gqa=True)
    assert rel_err(y.cpu().numpy(), ref) <= 1e-5


def test_sdpa_dropout_grouped_heads_tensor_cores():
    # Head dim 64: the tensor-core kernels, with four query heads over two kv heads.
    rng = np.random.default_rng(8)
    q, g = (rng.normal(size=(2, 4, 150, 64)).astype(np.float32) for _ in range(2))
    k, v = (rng.normal(size=(2, 2, 150, 64)).astype(np.float32) for _ in range(2))
    wide = lambda a: np.repeat(a, 2, axis=1)
    ref, saved = _oracle_case(q, wide(k), wide(v), None, True, None, 0.2, 9)
    dq, dk, dv = oracle.sdpa_math_backward(g, wide(v), saved)
    dk = dk.reshape(2, 2, 2, 150, 64).sum(axis=2)
    dv = dv.reshape(2, 2, 2, 150, 64).sum(axis=2)
    dc.manual_seed(9)
    t = [torch.tensor(a, device="cuda", requires_grad=True) for a in (q, k, v)]
    y = dc.functional.scaled_dot_product_attention(*t, dropout_p=0.2, is_causal=True, enable_gqa=True)
    y.backward(torch.tensor(g, device="cuda"))
    assert rel_err(y.detach().cpu().numpy(), ref) <= 1e-5
    for tt, r in zip(t, (dq, dk, dv)):
        assert rel_err(tt.grad.cpu().numpy(), r) <= 1e-5


def test_dropout_one_draws_nothing_and_zeroes():
    q = torch.randn(2, 3, 9, 8, device="cuda", requires_grad=True)
    dc.manual_seed(1)
    before = dc.get_rng_state()
    y = dc.functional.scaled_dot_product_attention(q, q, q, dropout_p=1.0)
    assert not y.detach().any()
    y.sum().backward()
    assert not q.grad.any()
    assert torch.equal(dc.get_rng_state(), before)


def test_dropout_is_reproducible_and_advances():
    q = torch.randn(2, 3, 16, 8, device="cuda")
    dc.manual_seed(3)
    a = dc.functional.scaled_dot_product_attention(q, q, q, dropout_p=0.5, is_causal=True)
    b = dc.functional.scaled_dot_product_attention(q, q, q, dropout_p=0.5, is_causal=True)
    dc.manual_seed(3)
    c = dc.functional.scaled_dot_product_attention(q, q, q, dropout_p=0.5, is_causal=True)
    assert torch.equal(a, c) and not torch.equal(a, b)
    plain = dc.functional.scaled_dot_product_attention(q, q, q, is_causal=True)
    assert not torch.equal(a, plain)


def _mha_pair(**kwargs):
    theirs = torch.nn.MultiheadAttention(**kwargs)
    ours = dc.nn.MultiheadAttention(**kwargs).cuda()
    names = dict(theirs.named_parameters())
    with torch.no_grad():
        for name, p in ours.named_parameters():
            p.copy_(names[name].detach())
    return ours, theirs


@pytest.mark.parametrize("need_weights", [True, False])
def test_mha_training_dropout_matches_torch(need_weights):
    torch.manual_seed(0)
    ours, theirs = _mha_pair(embed_dim=16, num_heads=4, dropout=0.3)
    rng = np.random.default_rng(2)
    x = rng.normal(size=(7, 3, 16)).astype(np.float32)
    padding = np.zeros((3, 7), bool)
    padding[1, -2:] = True
    tx = torch.tensor(x, requires_grad=True)
    torch.manual_seed(13)
    out, weights = theirs(tx, tx, tx, key_padding_mask=torch.tensor(padding), need_weights=need_weights)
    dx = torch.tensor(x, device="cuda", requires_grad=True)
    dc.manual_seed(13)
    got, got_weights = ours(dx, dx, dx, key_padding_mask=torch.tensor(padding, device="cuda"),
                            need_weights=need_weights)
    np.testing.assert_allclose(got.detach().cpu().numpy(), out.detach().numpy(), rtol=1e-5, atol=1e-6)
    if need_weights:
        np.testing.assert_allclose(got_weights.cpu().numpy(), weights.detach().numpy(), rtol=1e-5, atol=1e-6)
    w = rng.normal(size=out.shape).astype(np.float32)
    (out * torch.tensor(w)).sum().backward()
    (got * torch.tensor(w, device="cuda")).sum().backward()
    np.testing.assert_allclose(dx.grad.cpu().numpy(), tx.grad.numpy(), rtol=1e-4, atol=1e-5)
