"""The dropout generator on the CPU: DenseCore's Generator surface (python/densecore/_random.py)
and the library's skip-ahead (dc_rng_skip), checked against the oracle's sequential mt19937
(src/torch_random.rs restated in oracle/dc_oracle.c). No device is used."""
import ctypes

import numpy as np
import pytest
import torch

import densecore_b200 as dc
import oracle
from densecore_b200 import _lib

_U32P = ctypes.POINTER(ctypes.c_uint32)
CHUNK = 624 * 210  # words per chunk of the library's parallel walk


def _skip(state, outputs):
    out = np.zeros(626, np.uint32)
    st = _lib.load().dc_rng_skip(state.ctypes.data_as(_U32P), int(outputs), out.ctypes.data_as(_U32P))
    _lib.check(st, "skip")
    return out


def _words(gen_state):
    return gen_state.numpy().view(np.uint64)


@pytest.mark.parametrize("seed,pre,n", [
    (5, 0, 1), (5, 0, 2), (5, 0, 623), (5, 0, 624), (5, 0, 625), (7, 3, 1000), (9, 623, 5), (11, 624, 1),
    (13, 624, 624), (1, 0, CHUNK), (1, 0, 2 * CHUNK + 17), (2, 100, 3 * CHUNK + 624 * 5 + 3),
    (3, 0, 40 * CHUNK + 1), (4, 311, 33 * CHUNK - 1)])
def test_skip_matches_sequential_generation(seed, pre, n):
    g = oracle.MtGenerator(seed)
    g.discard(pre)
    got = _skip(g.state.copy(), n)
    g.discard(n)
    assert np.array_equal(got, g.state)


def test_skip_beyond_one_table_reach():
    # More chunks than the jump table holds (2048): the host walk chains its largest jump.
    g = oracle.MtGenerator(21)
    n = 2100 * CHUNK + 999
    got = _skip(g.state.copy(), n)
    g.discard(n)
    assert np.array_equal(got, g.state)


def test_skip_rejects_invalid_states():
    L = _lib.load()
    bad = oracle.MtGenerator(1).state.copy()
    for left, nxt in ((0, 0), (625, 0), (3, 625)):
        bad[624], bad[625] = left, nxt
        out = np.zeros(626, np.uint32)
        st = L.dc_rng_skip(bad.ctypes.data_as(_U32P), 10, out.ctypes.data_as(_U32P))
        assert st == _lib.DC_ERR_VALUE and b"invalid generator state" in L.dc_last_error()
    good = oracle.MtGenerator(1).state.copy()
    out = np.zeros(626, np.uint32)
    assert L.dc_rng_skip(good.ctypes.data_as(_U32P), (1 << 36) + 1, out.ctypes.data_as(_U32P)) == _lib.DC_ERR_VALUE


def test_generator_surface_follows_the_reference():
    g = dc.Generator()
    assert g.initial_seed() == 67_280_421_310_721  # torch_random.rs:16
    with pytest.raises(NotImplementedError):
        dc.Generator("cuda")
    g.manual_seed(-5)
    assert g.initial_seed() == 0xFFFF_FFFF_FFFF_FFFF - 4  # _random.py:17-24
    with pytest.raises(TypeError):
        g.manual_seed(True)
    with pytest.raises(RuntimeError, match="Overflow"):
        g.manual_seed(1 << 64)
    s = g.seed()
    assert g.initial_seed() == s and 0 <= s < 1 << 63


def test_state_layout_and_round_trip():
    dc.manual_seed(5)
    w = _words(dc.get_rng_state())
    assert w.size == 631
    assert list(w[:7]) == [5, 1, 0, 0xFFFF_FFFF_FFFF_FFFF, 0, 0, 0]  # torch_random.rs:276-288
    assert np.array_equal(w[7:].astype(np.uint32), oracle.MtGenerator(5).state[:624])
    saved = dc.get_rng_state()
    dc.default_generator._skip_host(1000)
    ref = oracle.MtGenerator(5).discard(1000)
    w = _words(dc.get_rng_state())
    assert list(w[1:3]) == list(ref.state[624:]) and np.array_equal(w[7:].astype(np.uint32), ref.state[:624])
    dc.set_rng_state(saved)
    assert torch.equal(dc.get_rng_state(), saved)


def test_set_state_validation():
    good = dc.get_rng_state().numpy()
    with pytest.raises(ValueError, match="invalid generator state"):
        dc.set_rng_state(good[:-3])
    for index, value in ((1, 0), (1, 625), (2, 625)):
        bad = good.view(np.uint64).copy()
        bad[index] = value
        with pytest.raises(ValueError, match="invalid generator state"):
            dc.set_rng_state(bad.view(np.uint8))
    bad = good.view(np.uint64).copy()
    bad[7] = 1 << 32
    with pytest.raises(ValueError, match="invalid generator state"):
        dc.set_rng_state(bad.view(np.uint8))


def test_generators_are_independent():
    a, b = dc.Generator().manual_seed(3), dc.Generator().manual_seed(3)
    a._skip_host(10)
    assert not torch.equal(a.get_state(), b.get_state())
    b._skip_host(10)
    assert torch.equal(a.get_state(), b.get_state())
