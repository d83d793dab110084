"""CUDA-graph capture of the library's calls: a training step's attention (forward, then
backward with the dQ kernel on the library's second stream, forked and joined with events) is
captured once into a CUDA graph and replayed on new inputs copied into the captured buffers;
the replays must reproduce eager calls exactly (same kernels, same inputs). A dropout mask draw
captured the same way must continue the generator stream on every replay."""
import numpy as np
import pytest
import torch

import densecore_b200 as dc
import oracle
from densecore_b200 import _native

pytestmark = pytest.mark.gpu


def _step(q, k, v, g, causal):
    out, lse = _native._flash_attention(q, k, v, causal)
    dq, dk, dv = _native._flash_attention_backward(g, q, k, v, out, lse, causal)
    return out, lse, dq, dk, dv


@pytest.mark.parametrize("shape,causal", [((2, 6, 256, 64), True), ((1, 4, 200, 128), False)])
def test_attention_step_replays_from_a_cuda_graph(shape, causal):
    torch.manual_seed(0)
    static = [torch.randn(shape, device="cuda") for _ in range(4)]
    side = torch.cuda.Stream()
    side.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(side):  # warm-up off the capture: pools, modules, tables
        for _ in range(2):
            _step(*static, causal)
    torch.cuda.current_stream().wait_stream(side)
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph):
        outs = _step(*static, causal)
    for trial in range(3):
        fresh = [torch.randn(shape, device="cuda") for _ in range(4)]
        for s, f in zip(static, fresh):
            s.copy_(f)
        graph.replay()
        torch.cuda.synchronize()
        ref = _step(*fresh, causal)
        torch.cuda.synchronize()
        for name, a, b in zip(("out", "lse", "dq", "dk", "dv"), outs, ref):
            assert torch.equal(a, b), f"{name} differs on replay {trial}"
    assert dc._lib.load().dc_device_status(1) == 0


def test_keep_bits_draw_replays_from_a_cuda_graph():
    # After a first (uncaptured) call, a dropout mask draw with the generator state advanced in
    # place is captured once; every replay must draw the next bits of the stream and advance
    # the device state, as consecutive eager calls do.
    n, keep = 100_000, 0.7
    gen = oracle.MtGenerator(31).discard(5)
    st = torch.from_numpy(gen.state.view(np.int32).copy()).cuda()
    bits = torch.zeros((n + 31) // 32, dtype=torch.int32, device="cuda")
    L = dc._lib.load()

    def draw():
        dc._lib.check(L.dc_dropout_keep_bits(st.data_ptr(), st.data_ptr(), n, keep, bits.data_ptr(),
                                             torch.cuda.current_stream().cuda_stream), "keep bits")

    side = torch.cuda.Stream()
    side.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(side):  # first call off the capture: jump tables, kernel attributes
        draw()
    torch.cuda.current_stream().wait_stream(side)
    torch.cuda.synchronize()
    assert np.array_equal(bits.cpu().numpy().view(np.uint32), gen.keep_bits(n, keep))
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph):
        draw()
    for _ in range(3):
        graph.replay()
        torch.cuda.synchronize()
        assert np.array_equal(bits.cpu().numpy().view(np.uint32), gen.keep_bits(n, keep))
    assert np.array_equal(st.cpu().numpy().view(np.uint32), gen.state)
    assert L.dc_device_status(1) == 0
