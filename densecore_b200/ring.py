"""Sequence-parallel ring attention (forward) over torch.distributed.

DenseCore has no sequence parallelism: its flash forward (src/torch_attention.rs:146-284) runs
every (batch, head) task over the whole key range on one host. For the long-context causal
prefill, this module splits the sequence over P ranks and passes K/V blocks around a ring;
each rank's result equals the reference's forward on the full sequence, restricted to that
rank's query rows.

Layout (zig-zag, for causal balance): the sequence is cut into 2P chunks of C = S / 2P rows;
rank r holds query, key and value chunks r and 2P-1-r, stored back to back as its local
(B, H, 2C, D) shard. Causally, every rank then does the same amount of work at every step:

  step 0     local queries against local keys: exactly a top-left causal attention over the
             2C local rows (chunk r sees itself causally, chunk 2P-1-r sees chunk r fully and
             itself causally, chunk r never sees chunk 2P-1-r);
  step t>0   keys of source rank s = (r - t) mod P:
             s < r: both local query chunks see key chunk s fully and key chunk 2P-1-s not at
                    all -> non-causal attention of all 2C local rows against the first C keys;
             s > r: local query chunk 2P-1-r sees both key chunks fully, chunk r sees neither
                    -> non-causal attention of the last C local rows against all 2C keys.

Each partial (out, lse) is folded into the running result with the logsumexp merge
(dc_attn_merge). K and V travel packed in one (2, B, H, 2C, D) buffer; the send of the held
block and the receive of the next are issued (batch_isend_irecv) before the step's attention
call, so the transfer overlaps the compute; the next step waits on the receive.

The compute and merge functions are injectable so that the ring logic can be exercised with
CPU tensors over gloo; the defaults are this package's CUDA kernels. A user mask is not
supported (a row fully masked inside one block would yield the reference's out = 0, lse = 0
for that block, which a logsumexp merge cannot tell from a real contribution).
"""
from __future__ import annotations

import torch
import torch.distributed as dist


def zigzag_indices(seq_len: int, rank: int, world: int) -> tuple[slice, slice]:
    """The two sequence slices rank ``rank`` holds: chunks rank and 2*world-1-rank."""
    if world < 1 or not 0 <= rank < world:
        raise ValueError(f"rank {rank} is not in a world of {world}")
    if seq_len % (2 * world):
        raise ValueError(f"sequence length {seq_len} is not a multiple of 2 * world size ({2 * world})")
    c = seq_len // (2 * world)
    a, b = rank, 2 * world - 1 - rank
    return slice(a * c, (a + 1) * c), slice(b * c, (b + 1) * c)


def zigzag_shard(x: torch.Tensor, rank: int, world: int, dim: int = 2) -> torch.Tensor:
    """This rank's zig-zag shard of ``x`` along ``dim`` (a new contiguous tensor)."""
    s0, s1 = zigzag_indices(x.shape[dim], rank, world)
    return torch.cat([x.narrow(dim, s0.start, s0.stop - s0.start),
                      x.narrow(dim, s1.start, s1.stop - s1.start)], dim=dim).contiguous()


def zigzag_unshard(shards, dim: int = 2) -> torch.Tensor:
    """Inverse of :func:`zigzag_shard`: the full tensor from all ranks' shards in rank order."""
    world = len(shards)
    c = shards[0].shape[dim] // 2
    chunks = [None] * (2 * world)
    for r, sh in enumerate(shards):
        chunks[r] = sh.narrow(dim, 0, c)
        chunks[2 * world - 1 - r] = sh.narrow(dim, c, c)
    return torch.cat(chunks, dim=dim)


def _default_attn(q, k, v, causal, scale, precision):
    from ._native import _flash_attention
    return _flash_attention(q, k, v, causal, scale, None, precision)


def _default_merge(out_acc, lse_acc, out_part, lse_part):
    from ._native import _attn_merge
    _attn_merge(out_acc, lse_acc, out_part, lse_part)


def ring_step(attn, merge, q, kk, vv, out, lse, t, rank, world, causal):
    """Step ``t`` of rank ``rank``'s ring: attend the local queries q (B, H, 2C, D) to the K/V
    block kk, vv that rank (rank - t) mod world started with, and fold the result into
    (out, lse). Step 0 creates and returns (out, lse)."""
    C = q.shape[2] // 2
    if t == 0:
        o, l = attn(q, kk, vv, causal)
        return o.contiguous(), l.contiguous()
    s = (rank - t) % world
    if not causal:
        po, pl = attn(q, kk, vv, False)
        merge(out, lse, po, pl)
    elif s < rank:
        po, pl = attn(q, kk[:, :, :C], vv[:, :, :C], False)
        merge(out, lse, po, pl)
    else:
        po, pl = attn(q[:, :, C:], kk, vv, False)
        merge(out[:, :, C:], lse[:, :, C:], po, pl)
    return out, lse


class RingAttention:
    """Reusable ring-attention forward for one shard shape: the (2, B, H, 2C, D) K/V exchange
    buffers are allocated once and reused by every call."""

    def __init__(self, shape_q, shape_kv, device, group=None, causal=True, scale=None, precision=None,
                 attn_fn=None, merge_fn=None, dtype=torch.float32):
        self.group = group
        self.world = dist.get_world_size(group)
        self.rank = dist.get_rank(group)
        B, H, L2, D = shape_q
        Bk, Hk, S2, Dk = shape_kv
        if L2 != S2 or L2 % 2:
            raise ValueError("ring attention needs local query and key shards of the same even length")
        if B != Bk or D != Dk:
            raise ValueError("ring attention q/k shapes do not match")
        self.causal = causal
        self.attn = attn_fn or (lambda q, k, v, c: _default_attn(q, k, v, c, scale, precision))
        self.merge = merge_fn or _default_merge
        self.bufs = [torch.empty((2, Bk, Hk, S2, Dk), device=device, dtype=dtype) for _ in range(2)]
        # Global ranks of the ring neighbours (P2P ops address global ranks).
        nxt, prv = (self.rank + 1) % self.world, (self.rank - 1) % self.world
        self.peer_next = dist.get_global_rank(group, nxt) if group is not None else nxt
        self.peer_prev = dist.get_global_rank(group, prv) if group is not None else prv

    def _exchange(self, send_buf, recv_buf):
        ops = [dist.P2POp(dist.isend, send_buf, self.peer_next, self.group),
               dist.P2POp(dist.irecv, recv_buf, self.peer_prev, self.group)]
        return dist.batch_isend_irecv(ops)

    def __call__(self, q, k, v):
        """(out, lse) of this rank's query shard against the whole sequence."""
        cur = self.bufs[0]
        cur[0].copy_(k)
        cur[1].copy_(v)
        out = lse = None
        for t in range(self.world):
            reqs = self._exchange(cur, self.bufs[(t + 1) % 2]) if t + 1 < self.world else None
            out, lse = ring_step(self.attn, self.merge, q, cur[0], cur[1], out, lse, t, self.rank,
                                 self.world, self.causal)
            if reqs is not None:
                for req in reqs:
                    req.wait()
                cur = self.bufs[(t + 1) % 2]
        return out, lse


def ring_emulate(q, k, v, world, causal=True, attn_fn=None, merge_fn=None, scale=None, precision=None):
    """Every rank of a ``world``-rank ring, one after another in this process, on full
    (B, H, S, D) tensors: the same steps and merges as :class:`RingAttention` without the
    exchange. Returns the full (out, lse). For checking the ring's arithmetic on one device."""
    attn = attn_fn or (lambda q_, k_, v_, c: _default_attn(q_, k_, v_, c, scale, precision))
    merge = merge_fn or _default_merge
    qs = [zigzag_shard(q, r, world) for r in range(world)]
    ks = [zigzag_shard(k, r, world) for r in range(world)]
    vs = [zigzag_shard(v, r, world) for r in range(world)]
    outs, lses = [], []
    for r in range(world):
        out = lse = None
        for t in range(world):
            s = (r - t) % world
            out, lse = ring_step(attn, merge, qs[r], ks[s], vs[s], out, lse, t, r, world, causal)
        outs.append(out)
        lses.append(lse)
    return zigzag_unshard(outs), zigzag_unshard(lses)


def ring_attention_forward(q, k, v, group=None, causal=True, scale=None, precision=None,
                           attn_fn=None, merge_fn=None):
    """One ring-attention forward of zig-zag shards q, k, v (B, H, 2C, D) of this rank; see the
    module docstring. Returns (out, lse) for the local query rows."""
    ring = RingAttention(q.shape, k.shape, q.device, group, causal, scale, precision, attn_fn, merge_fn,
                         dtype=k.dtype)
    if v.shape != k.shape:
        raise ValueError("ring attention needs k and v of the same shape")
    return ring(q, k, v)


class NcclCommunicator:
    """An NCCL communicator over the ranks of a torch.distributed group, made through
    libnccl's own C API (ncclGetUniqueId on the group's first rank, broadcast over the group,
    ncclCommInitRank on every rank) -- the communicator a C or Rust host would hand to
    ``dc_ring_sdpa_fwd``. ``ptr`` is the ncclComm_t. Every rank of the group must construct it
    together, with its CUDA device current."""

    _nccl = None

    @classmethod
    def _lib(cls):
        import ctypes
        if cls._nccl is None:
            import torch.cuda.nccl  # noqa: F401  (makes torch load its libnccl first)
            cls._nccl = ctypes.CDLL("libnccl.so.2")
        return cls._nccl

    def __init__(self, group=None, device=None):
        import ctypes

        class UniqueId(ctypes.Structure):
            _fields_ = [("internal", ctypes.c_char * 128)]

        lib = self._lib()
        lib.ncclGetUniqueId.argtypes = [ctypes.POINTER(UniqueId)]
        lib.ncclCommInitRank.argtypes = [ctypes.POINTER(ctypes.c_void_p), ctypes.c_int, UniqueId, ctypes.c_int]
        lib.ncclCommDestroy.argtypes = [ctypes.c_void_p]
        lib.ncclGetErrorString.restype = ctypes.c_char_p
        single = group is None and not dist.is_initialized()  # a one-rank communicator needs no group
        world, rank = (1, 0) if single else (dist.get_world_size(group), dist.get_rank(group))
        uid = UniqueId()
        if rank == 0:
            r = lib.ncclGetUniqueId(ctypes.byref(uid))
            if r:
                raise RuntimeError("ncclGetUniqueId: " + lib.ncclGetErrorString(r).decode())
        if not single:
            # The id's raw 128 bytes (reading the c_char array field would stop at its first NUL).
            box = [ctypes.string_at(ctypes.addressof(uid), 128) if rank == 0 else None]
            src = dist.get_global_rank(group, 0) if group is not None else 0
            dist.broadcast_object_list(box, src=src, group=group)
            uid = UniqueId()
            if len(box[0]) != 128:
                raise RuntimeError("NCCL unique id broadcast returned a wrong size")
            ctypes.memmove(ctypes.addressof(uid), box[0], 128)
        comm = ctypes.c_void_p()
        with torch.cuda.device(device if device is not None else torch.cuda.current_device()):
            r = lib.ncclCommInitRank(ctypes.byref(comm), world, uid, rank)
        if r:
            raise RuntimeError("ncclCommInitRank: " + lib.ncclGetErrorString(r).decode())
        self.ptr = comm.value
        self.world, self.rank = world, rank

    def destroy(self):
        if self.ptr:
            self._lib().ncclCommDestroy(self.ptr)
            self.ptr = None


class NativeRingAttention:
    """Ring attention through the library's C entry point ``dc_ring_sdpa_fwd``: the same zig-zag
    ring as :class:`RingAttention`, with the ring loop, the NCCL send/recv of K/V blocks and the
    merges inside the library (NCCL on a side stream, overlapped with each step's attention).
    ``comm`` is an :class:`NcclCommunicator` (or anything with an ncclComm_t in ``.ptr``)."""

    def __init__(self, shape_q, shape_kv, device, comm, causal=True, scale=None, precision=None):
        from . import _lib
        B, H, L2, D = shape_q
        _, Hk, S2, _ = shape_kv
        self.comm, self.causal, self.scale, self.precision = comm, causal, scale, precision
        n = _lib.load().dc_ring_sdpa_fwd_workspace_size(B, H, Hk, L2, D)
        self.ws = torch.empty(max(n, 1), dtype=torch.uint8, device=device)
        self.shape_q = tuple(shape_q)

    def __call__(self, q, k, v):
        from ._native import _ring_attention
        return _ring_attention(q, k, v, self.comm.ptr, self.causal, self.scale, self.precision, self.ws)
