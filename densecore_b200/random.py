"""The generator behind attention dropout: DenseCore's ``Generator`` / ``manual_seed``.

DenseCore draws dropout masks from its CPU generator, PyTorch's mt19937 with PyTorch's
sampling transforms (python/densecore/_random.py:1-7, src/torch_random.rs). This module keeps
that generator's surface -- ``Generator`` with ``manual_seed`` / ``initial_seed`` / ``seed`` /
``get_state`` / ``set_state``, the module-level ``default_generator``, ``manual_seed``,
``initial_seed``, ``seed``, ``get_rng_state``, ``set_rng_state`` -- with the same seeding,
the same engine and the same state layout (src/torch_random.rs:276-311), so the same seed
gives DenseCore's (and PyTorch's CPU) dropout masks.

Only the engine state is used here (dropout draws bernoulli through uniform doubles and never
touches the cached normal samples, which are carried through get_state / set_state as they
are). The first dropout call moves the engine state to that call's device, where
``dc_dropout_keep_bits`` advances it on the current stream; ``get_state`` copies it back (and
synchronises with the device). Dropout calls on different streams of one device must be
ordered by the caller, as any two launches that share memory must.
"""
from __future__ import annotations

import ctypes
import operator
import os
import threading

import numpy as np
import torch

from . import _lib

DEFAULT_SEED = 67_280_421_310_721  # torch_random.rs:16, default_rng_seed_val
_N = 624
_NO_DOUBLE_NORMAL = 0xFFFF_FFFF_FFFF_FFFF


def _seed_value(seed):
    """torch.manual_seed's accepted range; negatives wrap to 0xffff_ffff_ffff_ffff + seed + 1
    (python/densecore/_random.py:17-24)."""
    if isinstance(seed, (bool, np.bool_)):
        raise TypeError("seed must be an integer")
    seed = operator.index(seed)
    if not -0x8000_0000_0000_0000 <= seed <= 0xFFFF_FFFF_FFFF_FFFF:
        raise RuntimeError("Overflow when unpacking long long")
    return seed & 0xFFFF_FFFF_FFFF_FFFF


def _seeded_engine(seed):
    """manual_seed's engine (torch_random.rs:43-56): 624 words, left = 1, next = 0."""
    st = np.zeros(_N + 2, np.uint32)
    x = seed & 0xFFFF_FFFF
    st[0] = x
    for j in range(1, _N):
        x = (1_812_433_253 * (x ^ (x >> 30)) + j) & 0xFFFF_FFFF
        st[j] = x
    st[_N] = 1
    return st


class Generator:
    """CPU generator with PyTorch's engine; a new one starts from PyTorch's default seed."""

    def __init__(self, device="cpu"):
        if str(device) != "cpu":
            raise NotImplementedError("only CPU generators are supported")
        self.device = "cpu"
        self._lock = threading.RLock()
        self._seed = DEFAULT_SEED
        self._normals = [_NO_DOUBLE_NORMAL, 0, 0, 0]  # to_words()[3:7]: no cached normal samples
        self._host = _seeded_engine(DEFAULT_SEED)
        self._dev = None  # int32 CUDA tensor of 626 words while the engine lives on a device

    # ---- DenseCore's Generator API ----
    def manual_seed(self, seed):
        seed = _seed_value(seed)
        with self._lock:
            self._seed = seed
            self._normals = [_NO_DOUBLE_NORMAL, 0, 0, 0]
            self._host, self._dev = _seeded_engine(seed), None
        return self

    def initial_seed(self):
        return self._seed

    def seed(self):
        """Reseed from the operating system and return the new seed (like torch)."""
        seed = int.from_bytes(os.urandom(8), "little") & 0x7FFF_FFFF_FFFF_FFFF
        self.manual_seed(seed)
        return seed

    def get_state(self):
        """Engine state as a uint8 tensor in DenseCore's layout (torch_random.rs:276-288):
        seed, left, next, the two cached normals with their flags, the 624 state words."""
        engine = self._engine_on_host()
        words = np.array([self._seed, int(engine[_N]), int(engine[_N + 1])] + self._normals, np.uint64)
        words = np.concatenate([words, engine[:_N].astype(np.uint64)])
        return torch.from_numpy(words.view(np.uint8).copy())

    def set_state(self, state):
        array = state.detach().cpu().numpy() if isinstance(state, torch.Tensor) else np.asarray(state)
        array = np.ascontiguousarray(array, np.uint8)
        if array.size % 8:
            raise ValueError("invalid generator state")
        w = array.view(np.uint64)
        # Generator::from_words (torch_random.rs:290-311)
        if w.size != 7 + _N or w[1] == 0 or w[1] > _N or w[2] > _N or np.any(w[7:] > 0xFFFF_FFFF):
            raise ValueError("invalid generator state")
        engine = np.zeros(_N + 2, np.uint32)
        engine[:_N] = w[7:].astype(np.uint32)
        engine[_N], engine[_N + 1] = int(w[1]), int(w[2])
        with self._lock:
            self._seed = int(w[0])
            self._normals = [int(x) for x in w[3:7]]
            self._host, self._dev = engine, None
        return self

    # ---- device residence ----
    def _engine_on_host(self):
        with self._lock:
            if self._dev is not None:
                torch.cuda.synchronize(self._dev.device)
                self._host = self._dev.cpu().numpy().view(np.uint32).copy()
                self._dev = None
            return self._host.copy()

    def _engine_on(self, device):
        """The engine state as a CUDA tensor on ``device`` (moved there if needed); the caller
        advances it in place on that device's current stream."""
        with self._lock:
            if self._dev is None:
                self._dev = torch.from_numpy(self._host.view(np.int32).copy()).to(device)
            elif self._dev.device != device:
                self._dev = self._dev.to(device)
            return self._dev

    def _skip_host(self, outputs):
        """Advance the engine by ``outputs`` 32-bit outputs without a device (dc_rng_skip)."""
        engine = self._engine_on_host()
        out = np.empty_like(engine)
        p = ctypes.POINTER(ctypes.c_uint32)
        _lib.check(_lib.load().dc_rng_skip(engine.ctypes.data_as(p), int(outputs), out.ctypes.data_as(p)),
                   "generator skip failed")
        with self._lock:
            self._host = out


default_generator = Generator()


def _gen(generator=None):
    if generator is None:
        return default_generator
    if not isinstance(generator, Generator):
        raise TypeError("generator must be a densecore_b200 Generator")
    return generator


def manual_seed(seed):
    """Seed the default generator; the same seed gives PyTorch's CPU values."""
    return default_generator.manual_seed(seed)


def initial_seed():
    return default_generator.initial_seed()


def seed():
    return default_generator.seed()


def get_rng_state():
    return default_generator.get_state()


def set_rng_state(new_state):
    default_generator.set_state(new_state)


def dropout_keep_bits(n, keep_prob, device, generator=None):
    """n bernoulli(keep_prob) draws of the generator as packed int32 words on ``device``
    (element e is bit e % 32 of word e // 32), advancing the generator by 2n outputs."""
    gen = _gen(generator)
    words = torch.empty(max((n + 31) // 32, 1), dtype=torch.int32, device=device)
    if n == 0:
        return words
    with gen._lock, torch.cuda.device(device):
        engine = gen._engine_on(device)
        st = _lib.load().dc_dropout_keep_bits(engine.data_ptr(), engine.data_ptr(), int(n), float(keep_prob),
                                              words.data_ptr(), torch.cuda.current_stream(device).cuda_stream)
    _lib.check(st, "dropout mask failed")
    return words
