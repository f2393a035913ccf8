"""GPU parity of the forward (through the C ABI) against the float64 oracle.

Mirrors the reference leaf check ``runtime/gpu/nvidia/ffn/inference/checks/parity.py``: every test layer, the
reference's batch sizes, the policy and the nine forced kernel pairs, same bits on a repeated call,
``max |y - y64| <= 2e-5`` (the leaf tolerance) and ``max |y - y64| / max(1, |y64|) <= 1e-5`` (the fp32 target).
bf16 storage: relative 2e-2. Full-size configs compare a subset of token rows (tokens are independent)."""
import numpy as np
import pytest
import torch

from hffn_b200 import synth
from oracle import forward64

pytestmark = pytest.mark.gpu

BATCHES = (1, 2, 4, 5, 7, 8, 32, 63, 64, 96, 128, 129, 256, 512)
ABS_TOLERANCE = 2e-5
REL_TOLERANCE = 1e-5
BF16_TOLERANCE = 2e-2


def kernel_layer(layer):
    from hffn_b200.runtime import HFFNLayer
    t = torch.from_numpy
    return HFFNLayer.from_hidden_major(layer.d_model, layer.d_ff, t(layer.b_up), t(layer.up_offsets), t(layer.up_idx),
                                       t(layer.up_val), t(layer.b_down), t(layer.down_offsets), t(layer.down_idx),
                                       t(layer.down_val))


def runtime_for(layer, dtype=torch.float32, tensor_cores=None):
    from hffn_b200.runtime import HFFNRuntime
    return HFFNRuntime([kernel_layer(layer)], "cuda", dtype, tensor_cores=tensor_cores)


@pytest.mark.parametrize("name", sorted(synth.TEST_CASES))
def test_reference_batches_all_pairs(name):
    from hffn_b200 import parity
    case = synth.TEST_CASES[name]
    layer = synth.make_layer(case)
    runtime = runtime_for(layer)
    for n in BATCHES:
        x_np = synth.make_input(case, n)
        expected = torch.from_numpy(forward64.forward(layer, x_np))
        result = parity.check(runtime, 0, torch.from_numpy(x_np).cuda(), expected)
        assert result.repeatable, (name, n)
        assert result.sequential_bits, (name, n)
        assert result.error <= ABS_TOLERANCE, (name, n, result.error)
        assert result.relative <= REL_TOLERANCE, (name, n, result.relative)
    assert set(runtime.calls) >= {("coop", "coop"), ("tile", "blocked")}


@pytest.mark.parametrize("name,n", [("homog_256_1024", 64), ("homog_512_2048", 5), ("irreg_512_2048", 33)])
def test_golden_outputs(golden, name, n):
    with np.load(golden / f"forward_{name}_n{n}.npz") as g:
        x, y_ref = g["x"], g["y"].astype(np.float64)
    runtime = runtime_for(synth.make_layer(synth.TEST_CASES[name]))
    y = runtime.forward(0, torch.from_numpy(x).cuda()).double().cpu().numpy()
    assert np.max(np.abs(y - y_ref)) <= ABS_TOLERANCE


def test_c1_config_all_pairs():
    from hffn_b200 import parity
    case = synth.CONFIGS["c1_512_2048_k128"]
    layer = synth.make_layer(case)
    x = synth.make_input(case, 256)
    result = parity.check(runtime_for(layer), 0, torch.from_numpy(x).cuda(), torch.from_numpy(forward64.forward(layer, x)))
    assert result.repeatable and result.relative <= REL_TOLERANCE, result


def rows_subset(n):
    return np.r_[0:24, n // 2:n // 2 + 8, n - 24:n]


@pytest.mark.parametrize("tensor_cores", [False, None])
@pytest.mark.parametrize("dtype", [torch.float32, torch.bfloat16])
def test_c2_config_full_size(dtype, tensor_cores):
    case = synth.CONFIGS["c2_1024_4096_k512"]
    layer = synth.make_layer(case)
    n = 4096
    x = synth.make_input(case, n)
    runtime = runtime_for(layer, dtype, tensor_cores)
    y = runtime.forward(0, torch.from_numpy(x).cuda().to(dtype)).float().cpu().numpy()
    rows = rows_subset(n)
    expected = forward64.forward(layer, x[rows])
    relative = np.max(np.abs(y[rows] - expected) / np.maximum(1.0, np.abs(expected)))
    assert relative <= (REL_TOLERANCE if dtype == torch.float32 else BF16_TOLERANCE), relative
    assert np.isfinite(y).all()
    assert runtime.modes(n)[0] == ("tc" if tensor_cores is None else "tile")
    assert runtime.device_errors() == 0


def test_side_stream_and_second_call_same_bits():
    case = synth.TEST_CASES["irreg_512_2048"]
    layer = synth.make_layer(case)
    runtime = runtime_for(layer)
    x = torch.from_numpy(synth.make_input(case, 300)).cuda()
    first = runtime.forward(0, x).clone()
    stream = torch.cuda.Stream()
    with torch.cuda.stream(stream):
        second = runtime.forward(0, x).clone()
    stream.synchronize()
    assert torch.equal(first, second)


def test_errors():
    case = synth.TEST_CASES["homog_256_1024"]
    runtime = runtime_for(synth.make_layer(case))
    with pytest.raises(ValueError):
        runtime.forward(0, torch.zeros(4, 256, dtype=torch.float64, device="cuda"))
    with pytest.raises(ValueError):
        runtime.forward(0, torch.zeros(4, 255, device="cuda"))
    with pytest.raises(ValueError):
        runtime.forward(0, torch.zeros(256, 8, device="cuda").T)
    with pytest.raises(ValueError):
        runtime.force("fast", None)


def test_device_layout_validation():
    from hffn_b200 import _native as native
    from hffn_b200.runtime import layer_struct
    case = synth.TEST_CASES["irreg_512_2048"]
    runtime = runtime_for(synth.make_layer(case))
    flag = torch.ones(1, dtype=torch.int32, device="cuda")
    stream = native.stream_handle(runtime.device)
    native.check(native.lib.hffn_validate_layout(runtime._structs[0], flag.data_ptr(), stream), "validate")
    assert int(flag) == 0
    bad = dict(runtime._tensors[0])
    bad["out_hidden"] = bad["out_hidden"].clone()
    bad["out_hidden"][7] = runtime.d_ff
    native.check(native.lib.hffn_validate_layout(layer_struct(bad, runtime.d_model, runtime.d_ff), flag.data_ptr(),
                                                 stream), "validate")
    assert int(flag) == 1


def test_prepared_runtime_and_cuda_graph():
    """The decode fast path gives the bits of the plain runtime, and a prepared call replays inside a CUDA graph."""
    from hffn_b200.runtime import PreparedRuntime
    case = synth.TEST_CASES["homog_512_2048"]
    layer = synth.make_layer(case)
    plain = runtime_for(layer)
    prepared = PreparedRuntime([kernel_layer(layer)], "cuda")
    for n in (1, 4, 8, 9):
        x = torch.from_numpy(synth.make_input(case, n)).cuda()
        expected = plain.forward(0, x).clone()
        assert torch.equal(prepared.forward(0, x).clone(), expected)
        assert torch.equal(prepared.forward(0, x).clone(), expected)      # second call: the prepared entry
    x = torch.from_numpy(synth.make_input(case, 4)).cuda()
    static_x = x.clone()
    prepared.forward(0, static_x)
    graph = torch.cuda.CUDAGraph()
    stream = torch.cuda.Stream()
    stream.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(stream):
        with torch.cuda.graph(graph, stream=stream):
            y_graph = prepared.forward(0, static_x)
    torch.cuda.current_stream().wait_stream(stream)
    x2 = torch.from_numpy(synth.make_input(case, 7)[:4]).cuda()
    static_x.copy_(x2)
    graph.replay()
    torch.cuda.synchronize()
    assert torch.equal(y_graph, plain.forward(0, x2))


@pytest.mark.parametrize("name", ["irreg_512_2048", "homog_512_2048"])
def test_bf16_decode_sizes(name):
    """bfloat16 runtimes at the decode sizes (the cooperative kernels, n <= 8, irregular row starts included): within
    the bf16 bar of the oracle on the layer and input the runtime holds (values rounded to bf16), same bits on
    repeat."""
    import dataclasses
    case = synth.TEST_CASES[name]
    layer = synth.make_layer(case)
    r = lambda a: torch.from_numpy(a).to(torch.bfloat16).float().numpy()  # noqa: E731
    held = dataclasses.replace(layer, up_val=r(layer.up_val), b_up=r(layer.b_up), down_val=r(layer.down_val),
                               b_down=r(layer.b_down))
    runtime = runtime_for(layer, torch.bfloat16, None)
    runtime.force("coop", "coop")
    for n in (1, 2, 3, 4, 5, 7, 8):
        x = torch.from_numpy(synth.make_input(case, n)).to(torch.bfloat16)
        first = runtime.forward(0, x.cuda()).clone()
        assert torch.equal(first, runtime.forward(0, x.cuda())), n
        expected = forward64.forward(held, x.float().numpy())
        y = first.float().cpu().numpy()
        relative = np.max(np.abs(y - expected) / np.maximum(1.0, np.abs(expected)))
        assert relative <= BF16_TOLERANCE, (n, relative)
    assert runtime.device_errors() == 0
