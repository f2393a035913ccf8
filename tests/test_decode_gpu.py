"""GPU: the decode kernels (the cooperative mode at n <= 8 tokens: windows of slots staged by TMA bulk copies,
programmatic dependent launch) through the C ABI, against the float64 oracle.

Layers of the benchmark plan's decode shapes and the irregular reference test layer, float32 (relative 1e-5, absolute
2e-5) and bfloat16 (relative 2e-2 against the oracle of the layer and input as the runtime holds them), every n from
1 to 8 that changes the kernel's planes or its token fill; the same bits on repeat and inside a CUDA graph; the decode
error flag stays 0. The C5 shape's down projection (its act table does not fit the kernel's shared-memory budget)
exercises the general cooperative kernel the launcher falls back to.
"""
import dataclasses

import numpy as np
import pytest
import torch

from hffn_b200 import synth
from oracle import forward64

pytestmark = pytest.mark.gpu

LAYERS = ("c4_1024_4096_k512", "irreg_512_2048", "c5_2048_8192_k410")
TOKENS = (1, 3, 4, 5, 8)


def kernel_layer(layer):
    from hffn_b200.runtime import HFFNLayer
    t = torch.from_numpy
    return HFFNLayer.from_hidden_major(layer.d_model, layer.d_ff, t(layer.b_up), t(layer.up_offsets), t(layer.up_idx),
                                       t(layer.up_val), t(layer.b_down), t(layer.down_offsets), t(layer.down_idx),
                                       t(layer.down_val))


def held(layer, dtype):
    if dtype == torch.float32:
        return layer
    r = lambda a: torch.from_numpy(a).to(torch.bfloat16).float().numpy()  # noqa: E731
    return dataclasses.replace(layer, up_val=r(layer.up_val), b_up=r(layer.b_up), down_val=r(layer.down_val),
                               b_down=r(layer.b_down))


@pytest.fixture(scope="module", params=LAYERS)
def layer_of(request):
    case = synth.CASES[request.param]
    return case, synth.make_layer(case)


@pytest.mark.parametrize("dtype", [torch.float32, torch.bfloat16])
def test_decode_against_oracle(layer_of, dtype):
    from hffn_b200.runtime import HFFNRuntime
    case, layer = layer_of
    runtime = HFFNRuntime([kernel_layer(layer)], "cuda", dtype, tensor_cores=False)
    runtime.force("coop", "coop")
    expected_layer = held(layer, dtype)
    for n in TOKENS:
        x = torch.from_numpy(synth.make_input(case, n)).to(dtype).cuda()
        first = runtime.forward(0, x).clone()
        assert torch.equal(first, runtime.forward(0, x)), n
        expected = forward64.forward(expected_layer, x.float().cpu().numpy())
        y = first.double().cpu().numpy()
        gap = np.abs(y - expected)
        relative = float(np.max(gap / np.maximum(1.0, np.abs(expected))))
        if dtype == torch.float32:
            assert float(gap.max()) <= 2e-5 and relative <= 1e-5, (case.name, n, relative)
        else:
            assert relative <= 2e-2, (case.name, n, relative)
    assert runtime.device_errors() == 0


def test_decode_graph_replay_same_bits():
    """Four layers of the C4 shape, 8 tokens each, eager and replayed from a CUDA graph (the programmatic
    dependencies between the launches are captured): the same bits."""
    from hffn_b200.runtime import PreparedRuntime
    case = synth.CASES["c4_1024_4096_k512"]
    layer = synth.make_layer(case)
    runtime = PreparedRuntime([kernel_layer(layer)] * 4, "cuda", torch.bfloat16)
    xs = torch.stack([torch.from_numpy(synth.make_input(case, 8)) * (k + 1) for k in range(4)]).to(torch.bfloat16).cuda()
    outs = torch.empty(4, 8, case.d_model, dtype=torch.bfloat16, device="cuda")

    def step():
        for k in range(4):
            outs[k].copy_(runtime.forward(k, xs[k]))

    step()
    eager = outs.clone()
    graph = torch.cuda.CUDAGraph()
    side = torch.cuda.Stream()
    side.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(side):
        step()
        with torch.cuda.graph(graph, stream=side):
            step()
    torch.cuda.current_stream().wait_stream(side)
    outs.zero_()
    graph.replay()
    torch.cuda.synchronize()
    assert torch.equal(outs, eager)
    assert runtime.device_errors() == 0
