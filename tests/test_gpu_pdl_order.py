"""Stream order under programmatic dependent launch.

The FP4 QDQ, pack, amax, STE, shadow-QDQ and Q4_K kernels are launched so that the next kernel
on the stream may be scheduled before the previous one has finished; each kernel waits
(``griddepcontrol.wait``) before it reads memory.  A chain in which every launch consumes the
previous launch's output must therefore give exactly the results of the same chain with a host
synchronisation between the calls, eagerly and replayed from a CUDA graph.
"""

from __future__ import annotations

import pytest
import torch

from qatfactory_b200 import _native

pytestmark = pytest.mark.gpu
DEV = torch.device("cuda", 0)


def _chain(x: torch.Tensor, sync: bool) -> list[torch.Tensor]:
    """amax -> NVFP4 QDQ of x scaled -> amax of the result -> STE of it -> MXFP4 of that -> Q4_K
    of that, eight times over, each step reading what the previous one wrote."""

    outs = []
    for i in range(8):
        amax = _native.tensor_amax(x)
        y, mask = _native.nvfp4_qdq(x, amax)
        running = _native.tensor_amax(y)
        _native.tensor_amax_update(x, running)
        g = _native.ste_backward(y, mask)
        m, _ = _native.mxfp4_qdq_even(g)
        blocks, recon, _ = _native.q4k_encode(m, "minmax", mask=False)
        outs += [amax, y, running, g, m, blocks, recon]
        x = (recon * (1.0 + 0.01 * i)).to(torch.bfloat16)
        if sync:
            torch.cuda.synchronize()
    return outs


def test_dependent_chain_matches_a_synchronised_chain():
    g = torch.Generator().manual_seed(3)
    x = (torch.randn(512, 1024, generator=g) * 0.1).to(torch.bfloat16).to(DEV)
    want = _chain(x, sync=True)
    got = _chain(x, sync=False)
    torch.cuda.synchronize()
    for a, b in zip(got, want):
        assert torch.equal(a, b)


def test_dependent_chain_in_a_cuda_graph():
    g = torch.Generator().manual_seed(4)
    x = (torch.randn(256, 2048, generator=g) * 0.1).to(torch.bfloat16).to(DEV)
    want = _chain(x, sync=True)
    static_x = x.clone()
    stream = torch.cuda.Stream(DEV)
    stream.wait_stream(torch.cuda.current_stream(DEV))
    with torch.cuda.stream(stream):
        _chain(static_x, sync=False)  # warm up (allocations) outside the capture
    torch.cuda.current_stream(DEV).wait_stream(stream)
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph):
        captured = _chain(static_x, sync=False)
    for _ in range(3):
        graph.replay()
    torch.cuda.synchronize()
    for a, b in zip(captured, want):
        assert torch.equal(a, b)
