"""GPU parity of the SDPA path: the CUDA kernels (through the C ABI) against the CPU oracle
and the golden fixtures, on the same seeded inputs.

Tolerances (the north star's): max|delta| <= 1e-5 * max|ref| for out, lse, dq, dk, dv in the
3xTF32 and fp32 modes; <= 5e-3 relative in the opt-in TF32 mode. Fully masked rows must give
exactly 0 output, 0 lse and 0 gradients (torch_attention.rs:223-226, :258-271).
"""
import numpy as np
import pytest
import torch

import densecore_b200 as dc
import oracle
from conftest import load_golden, rel_err

pytestmark = pytest.mark.gpu

TOL = {"3xtf32": 1e-5, "fp32": 1e-5, "tf32": 5e-3}
DEV = "cuda:0"


@pytest.fixture(params=["3xtf32", "fp32", "tf32"])
def precision(request):
    dc.set_sdpa_precision(request.param)
    yield request.param
    dc.set_sdpa_precision(None)


def _cuda(a, grad=False):
    t = torch.from_numpy(np.ascontiguousarray(a)).to(DEV)
    return t.requires_grad_(grad) if grad else t


def _run(q, k, v, g, mask=None, causal=False, scale=None, rank=4, enable_gqa=False):
    tq, tk, tv = (_cuda(a, True) for a in (q, k, v))
    tm = None if mask is None else _cuda(mask)
    y = dc.scaled_dot_product_attention(tq, tk, tv, attn_mask=tm, is_causal=causal, scale=scale,
                                        enable_gqa=enable_gqa)
    y.backward(_cuda(g))
    torch.cuda.synchronize()
    return [y.detach().cpu().numpy()] + [t.grad.cpu().numpy() for t in (tq, tk, tv)]


def _lse(q, k, v, mask=None, causal=False, scale=None):
    tm = None if mask is None else _cuda(mask)
    m = dc.functional._flash_mask(tm, 4)
    out, lse = dc._flash_attention(_cuda(q), _cuda(k), _cuda(v), causal, scale, m)
    return out.cpu().numpy(), lse.cpu().numpy()


def _assert_close(name, got, ref, tol):
    err = rel_err(got, ref)
    assert err <= tol, f"{name}: max|delta|/max|ref| = {err:.3e} > {tol:.0e}"


GOLDEN = load_golden()


@pytest.mark.parametrize("meta,arr", GOLDEN, ids=[c[0]["name"] for c in GOLDEN])
def test_golden_cases(meta, arr, precision):
    tol = TOL[precision]
    q, k, v, g = arr["q"], arr["k"], arr["v"], arr["g"]
    mask = arr.get("mask")
    got = _run(q, k, v, g, mask, meta["causal"], meta["scale"], rank=q.ndim)
    names = ("out", "dq", "dk", "dv")
    if meta["path"] == "flash":
        fm = oracle.flash_mask(mask, q.shape, k.shape[2])
        ref_out, ref_lse = oracle.flash_forward(q, k, v, fm, meta["causal"], meta["scale"])
        refs = [ref_out, *oracle.flash_backward(g, q, k, v, ref_out, ref_lse, fm, meta["causal"], meta["scale"])]
        _, lse = _lse(q, k, v, mask, meta["causal"], meta["scale"])
        _assert_close("lse", lse, ref_lse, tol)
    else:
        refs = [arr["out"], arr["dq"], arr["dk"], arr["dv"]]
    for name, a, r in zip(names, got, refs):
        _assert_close(name, a, r, tol)
    # Against PyTorch's own CPU kernel (the golden values) at the same bound.
    for name, a, key in zip(names, got, ("out", "dq", "dk", "dv")):
        _assert_close("golden " + name, a, arr[key], max(tol, 2e-5))
    if meta["kind"] == "row":
        for a in got:
            assert not np.any(a), "fully masked rows must give exact zeros"
        _, lse = _lse(q, k, v, mask)
        assert not np.any(lse)


def _inputs(seed, qshape, kshape, vshape=None, scale=1.0):
    rng = np.random.default_rng(seed)
    q = (rng.normal(size=qshape) * scale).astype(np.float32)
    k = (rng.normal(size=kshape) * scale).astype(np.float32)
    v = (rng.normal(size=vshape or kshape) * scale).astype(np.float32)
    g = rng.normal(size=qshape[:-1] + ((vshape or kshape)[-1],)).astype(np.float32)
    return q, k, v, g


CONFIG_CASES = {
    # (q shape, k shape, causal, mask kind, input scale): the five configs, reduced in batch/heads
    # (and sequence for cfg4) so the oracle finishes in seconds.
    "cfg1_nanogpt": ((2, 6, 256, 64), (2, 6, 256, 64), True, None, 1.0),
    "cfg3_gpt2": ((1, 2, 1024, 64), (1, 2, 1024, 64), True, None, 1.0),
    "cfg3_gpt2_floatmask": ((1, 2, 1024, 64), (1, 2, 1024, 64), False, "float", 1.0),
    "cfg4_long_d128": ((1, 1, 2048, 128), (1, 1, 2048, 128), True, None, 0.5),
    "odd_tiles": ((2, 3, 333, 64), (2, 3, 517, 64), False, "bool", 1.0),
    "causal_l_ne_s": ((1, 2, 300, 128), (1, 2, 200, 128), True, None, 1.0),
    "d128_floatmask": ((1, 2, 384, 128), (1, 2, 512, 128), False, "float", 1.0),
}


@pytest.mark.parametrize("name", sorted(CONFIG_CASES))
def test_config_shapes_against_oracle(name, precision):
    qs, ks, causal, mkind, sc = CONFIG_CASES[name]
    q, k, v, g = _inputs(sum(name.encode()), qs, ks, scale=sc)
    L, S = qs[2], ks[2]
    rng = np.random.default_rng(7)
    mask = None
    if mkind == "float":
        mask = (rng.normal(size=(L, S)) * 0.1).astype(np.float32)
    elif mkind == "bool":
        mask = rng.random((qs[0], 1, L, S)) > 0.2
    got = _run(q, k, v, g, mask, causal)
    fm = oracle.flash_mask(mask, q.shape, S)
    out, lse = oracle.flash_forward(q, k, v, fm, causal)
    ref = [out, *oracle.flash_backward(g, q, k, v, out, lse, fm, causal)]
    for nm, a, r in zip(("out", "dq", "dk", "dv"), got, ref):
        _assert_close(nm, a, r, TOL[precision])
    _, glse = _lse(q, k, v, mask, causal)
    _assert_close("lse", glse, lse, TOL[precision])


PERSISTENT_CASES = {
    # More tiles than a B200 has SMs (several waves of CTAs): ragged lengths with grouped-query
    # heads (dQ 5 x 80 = 400 tiles, dK/dV 6 x 40 = 240), keys past the last query under causal
    # masking (dK/dV tiles without query rows), a per-batch bool mask; and the same at head dim
    # 128, where two CTAs share each tile (one per 64-column half of the gradients).
    "many_tiles_ragged_gqa": ((4, 20, 640, 64), (4, 10, 700, 64), True, None),
    "keys_past_queries": ((4, 8, 256, 64), (4, 8, 1024, 64), True, None),
    "many_tiles_bool_mask": ((2, 24, 512, 64), (2, 24, 512, 64), False, "bool"),
    "d128_many_tiles_causal": ((2, 16, 512, 128), (2, 16, 512, 128), True, None),
    "d128_gqa_bool_mask_ragged": ((2, 8, 400, 128), (2, 4, 333, 128), False, "bool"),
    "d128_keys_past_queries": ((1, 4, 200, 128), (1, 4, 700, 128), True, None),
}


@pytest.mark.parametrize("name", sorted(PERSISTENT_CASES))
def test_many_tiles_per_cta_against_oracle(name, precision):
    qs, ks, causal, mkind = PERSISTENT_CASES[name]
    q, k, v, g = _inputs(sum(name.encode()), qs, ks)
    mask = None
    if mkind == "bool":
        mask = np.random.default_rng(3).random((qs[0], 1, qs[2], ks[2])) > 0.2
    got = _run(q, k, v, g, mask, causal, enable_gqa=qs[1] != ks[1])
    fm = oracle.flash_mask(mask, q.shape, ks[2])
    out, lse = oracle.flash_forward(q, k, v, fm, causal)
    ref = [out, *oracle.flash_backward(g, q, k, v, out, lse, fm, causal)]
    for nm, a, r in zip(("out", "dq", "dk", "dv"), got, ref):
        _assert_close(nm, a, r, TOL[precision])
    assert dc._lib.load().dc_device_status(0) == 0


def test_mha_core_key_padding_against_oracle(precision):
    # cfg2's core: (B*H, L, D) with a per-batch key-padding length in [16, 128].
    B, H, L, D = 4, 8, 128, 64
    q, k, v, g = _inputs(11, (B, H, L, D), (B, H, L, D))
    lengths = np.random.default_rng(12).integers(16, 129, size=B)
    pad = np.arange(L)[None, :] >= lengths[:, None]  # True = masked (MHA convention)
    keep = ~pad
    got = _run(q, k, v, g, keep[:, None, None, :])
    fm = oracle.flash_mask(keep[:, None, None, :], q.shape, L)
    out, lse = oracle.flash_forward(q, k, v, fm)
    ref = [out, *oracle.flash_backward(g, q, k, v, out, lse, fm)]
    for nm, a, r in zip(("out", "dq", "dk", "dv"), got, ref):
        _assert_close(nm, a, r, TOL[precision])


def test_grouped_query_heads(precision):
    q, k, v, g = _inputs(13, (2, 8, 96, 64), (2, 2, 130, 64))
    got = _run(q, k, v, g, enable_gqa=True)
    out, lse = oracle.flash_forward(q, k, v)
    ref = [out, *oracle.flash_backward(g, q, k, v, out, lse)]
    for nm, a, r in zip(("out", "dq", "dk", "dv"), got, ref):
        _assert_close(nm, a, r, TOL[precision])


def test_value_dim_differs_and_rank3():
    rng = np.random.default_rng(14)
    q = rng.normal(size=(3, 40, 24)).astype(np.float32)
    k = rng.normal(size=(3, 50, 24)).astype(np.float32)
    v = rng.normal(size=(3, 50, 40)).astype(np.float32)
    g = rng.normal(size=(3, 40, 40)).astype(np.float32)
    got = _run(q, k, v, g, rank=3)
    tq, tk, tv = (torch.tensor(a, requires_grad=True) for a in (q, k, v))
    y = torch.nn.functional.scaled_dot_product_attention(tq, tk, tv)
    y.backward(torch.from_numpy(g))
    for nm, a, r in zip(("out", "dq", "dk", "dv"), got, (y.detach(), tq.grad, tk.grad, tv.grad)):
        _assert_close(nm, a, r.numpy(), 1e-5)


@pytest.mark.parametrize("D", [64, 128])
def test_strided_views_need_no_copy(precision, D):
    # nanoGPT's layout: (B, T, H, D) viewed as (B, H, T, D).
    rng = np.random.default_rng(15)
    B, T, H = 2, 200, 4
    base = [rng.normal(size=(B, T, H, D)).astype(np.float32) for _ in range(3)]
    g = rng.normal(size=(B, H, T, D)).astype(np.float32)
    ts = [_cuda(a).transpose(1, 2).requires_grad_(True) for a in base]
    assert not ts[0].is_contiguous()
    y = dc.scaled_dot_product_attention(*ts, is_causal=True)
    y.backward(_cuda(g))
    q, k, v = (np.ascontiguousarray(a.transpose(0, 2, 1, 3)) for a in base)
    out, lse = oracle.flash_forward(q, k, v, causal=True)
    ref = [out, *oracle.flash_backward(g, q, k, v, out, lse, causal=True)]
    for nm, a, r in zip(("out", "dq", "dk", "dv"), [y.detach()] + [t.grad for t in ts], ref):
        _assert_close(nm, a.cpu().numpy(), r, TOL[precision])


@pytest.mark.parametrize("D", [64, 128])
def test_decode_split_kv_against_oracle(D):
    B, H, S = 2, 4, 8192
    q, k, v, _ = _inputs(16, (B, H, 1, D), (B, H, S, D))
    out, lse = oracle.flash_forward(q, k, v)
    assert dc._native._fwd_path(_cuda(q), _cuda(k), _cuda(v)) == 2
    for splits in (0, 1, 7):
        o, l = dc._decode(_cuda(q), _cuda(k), _cuda(v), num_splits=splits)
        _assert_close(f"out splits={splits}", o.cpu().numpy(), out, 1e-5)
        _assert_close(f"lse splits={splits}", l.cpu().numpy(), lse, 1e-5)
    # Through the public API too (q_len == 1 routes to the decode kernel).
    y = dc.scaled_dot_product_attention(_cuda(q), _cuda(k), _cuda(v))
    _assert_close("sdpa out", y.cpu().numpy(), out, 1e-5)


def test_decode_with_mask_and_fully_masked_row():
    B, H, S, D = 2, 2, 1000, 128
    q, k, v, _ = _inputs(17, (B, H, 1, D), (B, H, S, D))
    mask = np.random.default_rng(18).random((B, 1, 1, S)) > 0.5
    mask[1] = False  # batch 1: every key masked
    fm = oracle.flash_mask(mask, q.shape, S)
    out, lse = oracle.flash_forward(q, k, v, fm)
    o, l = dc._decode(_cuda(q), _cuda(k), _cuda(v), mask=_cuda(mask), num_splits=3)
    _assert_close("out", o.cpu().numpy(), out, 1e-5)
    _assert_close("lse", l.cpu().numpy(), lse, 1e-5)
    assert not o[1].any() and not l[1].any()


def test_merge_of_kv_chunks_equals_full_attention():
    # The ring-attention building block: attention over K/V chunks merged by logsumexp.
    q, k, v, _ = _inputs(19, (2, 3, 160, 64), (2, 3, 300, 64))
    full_o, full_l = dc._flash_attention(_cuda(q), _cuda(k), _cuda(v), False)
    acc_o = torch.zeros_like(full_o)
    acc_l = torch.full_like(full_l, float("-inf"))
    for a, b in ((0, 120), (120, 300)):
        po, pl = dc._flash_attention(_cuda(q), _cuda(k[:, :, a:b]), _cuda(v[:, :, a:b]), False)
        dc._attn_merge(acc_o, acc_l, po, pl)
    _assert_close("merged out", acc_o.cpu().numpy(), full_o.cpu().numpy(), 1e-5)
    _assert_close("merged lse", acc_l.cpu().numpy(), full_l.cpu().numpy(), 1e-5)


def test_empty_inputs():
    z = torch.zeros
    q = z(1, 2, 0, 8, device=DEV)
    k = z(1, 2, 5, 8, device=DEV)
    assert dc.scaled_dot_product_attention(q, k, k).shape == (1, 2, 0, 8)
    q = torch.randn(1, 2, 3, 8, device=DEV)
    k0 = z(1, 2, 0, 8, device=DEV)
    out, lse = dc._flash_attention(q, k0, k0, False)
    assert not out.any() and not lse.any()


def test_full_size_gpt2_sampled_heads_against_oracle():
    # cfg3 at its full shape; two (batch, head) tasks checked against the oracle (tasks are
    # independent, so their bits do not depend on the rest).
    gen = torch.Generator(device=DEV).manual_seed(20)
    q, k, v = (torch.randn(8, 12, 1024, 64, device=DEV, generator=gen) for _ in range(3))
    out, lse = dc._flash_attention(q, k, v, True)
    qn, kn, vn = (t.cpu().numpy() for t in (q, k, v))
    tasks = [5, 90]
    ro, rl = oracle.flash_forward_tasks(qn, kn, vn, tasks, causal=True)
    for t in tasks:
        b, h = divmod(t, 12)
        _assert_close(f"out task {t}", out[b, h].cpu().numpy(), ro[b, h], 1e-5)
        _assert_close(f"lse task {t}", lse[b, h].cpu().numpy(), rl[b, h], 1e-5)


def test_full_size_long_context_prefix_property():
    # cfg4 at full length: causal rows < P depend only on the first P keys, so the first 1024
    # rows of the 32768-long run equal the oracle on the 1024-long prefix.
    gen = torch.Generator(device=DEV).manual_seed(21)
    q, k, v = (torch.randn(1, 2, 32768, 128, device=DEV, generator=gen) * 0.5 for _ in range(3))
    out, lse = dc._flash_attention(q, k, v, True)
    P = 1024
    pre = [t[:, :, :P].cpu().numpy() for t in (q, k, v)]
    ro, rl = oracle.flash_forward(*pre, causal=True)
    _assert_close("prefix out", out[:, :, :P].cpu().numpy(), ro, 1e-5)
    _assert_close("prefix lse", lse[:, :, :P].cpu().numpy(), rl, 1e-5)
    # Value linearity: out(V = 1) is the all-ones row for every visible row, up to the fp32
    # rounding of two sums of up to 32768 terms taken in different orders (~2^-24 * log2(n)
    # per level, bounded here by 64 ulp).
    ones = torch.ones_like(v)
    o1, _ = dc._flash_attention(q, k, ones, True)
    assert float((o1 - 1).abs().max()) < 64 * 2.0 ** -23


def test_full_size_decode_sampled_rows():
    # cfg5 at full size (K and V 8.6 GB each), rows sampled against the oracle.
    gen = torch.Generator(device=DEV).manual_seed(22)
    B, H, S, D = 64, 32, 8192, 128
    q = torch.randn(B, H, 1, D, device=DEV, generator=gen)
    k = torch.randn(B, H, S, D, device=DEV, generator=gen)
    v = torch.randn(B, H, S, D, device=DEV, generator=gen)
    out = dc.scaled_dot_product_attention(q, k, v)
    for b, h in ((0, 0), (37, 19), (63, 31)):
        ro, _ = oracle.flash_forward(*(t[b:b + 1, h:h + 1].cpu().numpy() for t in (q, k, v)))
        _assert_close(f"out {b},{h}", out[b:b + 1, h:h + 1].cpu().numpy(), ro, 1e-5)
    del k, v
    torch.cuda.empty_cache()


@pytest.mark.parametrize("layout", ["bthd", "unaligned"])
@pytest.mark.parametrize("D", [64, 128])
def test_forward_into_callers_strided_out(precision, D, layout):
    # dc_sdpa_fwd writes into the caller's out view: a (B, T, H, D) buffer seen as (B, H, T, D),
    # or rows of D floats inside rows of D + 1 at an odd offset (unaligned rows). 288 query
    # tiles: the persistent kernel runs several per CTA; the last tile of each head is partial
    # (300 rows), and nothing outside the view may be written.
    from densecore_b200 import _lib
    from densecore_b200.backends import precision_code
    rng = np.random.default_rng(31)
    B, H, L = 8, 12, 300
    q, k, v = (rng.normal(size=(B, H, L, D)).astype(np.float32) for _ in range(3))
    tq, tk, tv = (_cuda(a) for a in (q, k, v))
    if layout == "bthd":
        buf = torch.full((B, L, H, D), 7.0, device=DEV)
        o = buf.transpose(1, 2)
        outside = None
    else:
        buf = torch.full((B, H, L, D + 1), 7.0, device=DEV)
        o = buf[..., 1:]
        outside = buf[..., 0]
    lse = torch.empty((B, H, L), device=DEV)
    lib = _lib.load()
    vq, vk, vv, vo, vl = (_lib.view(t) for t in (tq, tk, tv, o, lse))
    st = lib.dc_sdpa_fwd(_lib.ref(vq), _lib.ref(vk), _lib.ref(vv), None, 1, 0, 0.0, precision_code(),
                         _lib.ref(vo), _lib.ref(vl), _lib.stream_of(tq))
    _lib.check(st, "forward")
    torch.cuda.synchronize()
    ro, rl = oracle.flash_forward(q, k, v, causal=True)
    _assert_close("out", o.cpu().numpy(), ro, TOL[precision])
    _assert_close("lse", lse.cpu().numpy(), rl, TOL[precision])
    if outside is not None:
        assert bool((outside == 7.0).all()), "a store left the caller's view"
    assert lib.dc_device_status(0) == 0


@pytest.mark.parametrize("D", [64, 128])
def test_backward_with_inputs_tma_cannot_read(precision, D):
    # Rows of D floats inside rows of D + 1: strides that are not 16-byte multiples and bases off
    # 16-byte boundaries. The tensor-core backward then copies its hi and lo operands (in the
    # 3xTF32 mode it otherwise reads hi from the inputs and copies lo only); both must agree with
    # the oracle.
    rng = np.random.default_rng(23)
    B, H, L = 2, 3, 300
    bases = [rng.normal(size=(B, H, L, D + 1)).astype(np.float32) for _ in range(4)]
    ts = [_cuda(a)[..., 1:] for a in bases]
    assert ts[0].stride(2) == D + 1
    q, k, v = (t.clone().requires_grad_(True) for t in ts[:3])  # contiguous leaves for the forward
    out, lse = dc._flash_attention(q.detach(), k.detach(), v.detach(), True)
    dq, dk, dv = dc._flash_attention_backward(ts[3], ts[0], ts[1], ts[2], out, lse, True)
    qn, kn, vn, gn = (np.ascontiguousarray(a[..., 1:]) for a in bases)
    ro, rl = oracle.flash_forward(qn, kn, vn, causal=True)
    ref = oracle.flash_backward(gn, qn, kn, vn, ro, rl, causal=True)
    for nm, a, r in zip(("dq", "dk", "dv"), (dq, dk, dv), ref):
        _assert_close(nm, a.cpu().numpy(), r, TOL[precision])
    assert dc._lib.load().dc_device_status(0) == 0
