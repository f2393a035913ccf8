"""GPU parity of the tensor-core (tcgen05) forward against the float64 oracle, through the C ABI.

float32 runs in both operand formats, the fp16x3 split (the default) and the 3xTF32 split, and must meet the float32
bar in each (relative 1e-5 with floor 1, absolute 2e-5); bfloat16 storage relative 2e-2. The kernels' bounded waits
must never fire (error flag 0)."""
import numpy as np
import pytest
import torch

from hffn_b200 import synth
from oracle import forward64

pytestmark = pytest.mark.gpu


def kernel_layer(layer):
    from hffn_b200.runtime import HFFNLayer
    t = torch.from_numpy
    return HFFNLayer.from_hidden_major(layer.d_model, layer.d_ff, t(layer.b_up), t(layer.up_offsets), t(layer.up_idx),
                                       t(layer.up_val), t(layer.b_down), t(layer.down_offsets), t(layer.down_idx),
                                       t(layer.down_val))


FORMATS = ("f16x3", "tf32x3")


def tc_runtime(layer, dtype=torch.float32, tc_format=None):
    from hffn_b200.runtime import HFFNRuntime
    runtime = HFFNRuntime([kernel_layer(layer)], "cuda", dtype, tensor_cores=True, tc_format=tc_format)
    runtime.force("tc", "tc")
    return runtime


def relative(y, expected):
    return float(np.max(np.abs(y - expected) / np.maximum(1.0, np.abs(expected))))


@pytest.mark.parametrize("tc_format", FORMATS)
@pytest.mark.parametrize("n", [1, 7, 128, 129, 300])
def test_small_layer(n, tc_format):
    case = synth.TEST_CASES["homog_256_1024"]
    layer = synth.make_layer(case)
    runtime = tc_runtime(layer, tc_format=tc_format)
    x = synth.make_input(case, n)
    y = runtime.forward(0, torch.from_numpy(x).cuda()).double().cpu().numpy()
    expected = forward64.forward(layer, x)
    assert runtime.device_errors() == 0
    assert np.max(np.abs(y - expected)) <= 2e-5 and relative(y, expected) <= 1e-5, relative(y, expected)
    assert runtime.calls[("tc", "tc")] == 1


@pytest.mark.parametrize("tc_format", FORMATS)
def test_irregular_layer_repeatable(tc_format):
    case = synth.TEST_CASES["irreg_512_2048"]
    layer = synth.make_layer(case)
    runtime = tc_runtime(layer, tc_format=tc_format)
    x = torch.from_numpy(synth.make_input(case, 333)).cuda()
    first = runtime.forward(0, x).clone()
    assert torch.equal(first, runtime.forward(0, x))
    assert relative(first.double().cpu().numpy(), forward64.forward(layer, x.cpu().numpy())) <= 1e-5
    assert runtime.device_errors() == 0


@pytest.mark.parametrize("dtype,tc_format", [(torch.float32, "f16x3"), (torch.float32, "tf32x3"),
                                             (torch.bfloat16, None)])
def test_c1_and_c2(dtype, tc_format):
    for name, n in (("c1_512_2048_k128", 256), ("c2_1024_4096_k512", 4096)):
        case = synth.CONFIGS[name]
        layer = synth.make_layer(case)
        runtime = tc_runtime(layer, dtype, tc_format)
        x = synth.make_input(case, n)
        y = runtime.forward(0, torch.from_numpy(x).cuda().to(dtype)).float().cpu().numpy()
        rows = np.r_[0:16, n - 16:n]
        rel = relative(y[rows], forward64.forward(layer, x[rows]))
        assert rel <= (1e-5 if dtype == torch.float32 else 2e-2), (name, dtype, rel)
        assert np.isfinite(y).all() and runtime.device_errors() == 0


def test_policy_picks_tensor_cores_for_large_batches():
    from hffn_b200.runtime import HFFNRuntime, TC_MIN_TOKENS
    case = synth.TEST_CASES["homog_512_2048"]
    runtime = HFFNRuntime([kernel_layer(synth.make_layer(case))], "cuda")
    assert runtime.modes(TC_MIN_TOKENS) == ("tc", "tc")
    assert runtime.modes(8) == ("coop", "coop")
    assert runtime.modes(TC_MIN_TOKENS, hidden_major=True)[0] != "tc"


def test_dense_operands_follow_optimizer_steps():
    """After a training step updates the compact values, the tensor-core forward sees the new values."""
    from hffn_b200.runtime import HFFNRuntime
    from hffn_b200.train_runtime import HFFNTrainRuntime
    case = synth.TEST_CASES["homog_256_1024"]
    layer = synth.make_layer(case)
    runtime = HFFNRuntime([kernel_layer(layer)], "cuda", tensor_cores=True)
    train = HFFNTrainRuntime(runtime)
    x = torch.from_numpy(synth.make_input(case, 300)).cuda()
    gy = torch.from_numpy(synth.make_upstream(case, 300, 0)).cuda()
    runtime.force("tc", "tc")
    before = runtime.forward(0, x).clone()
    train.step(0, x, gy)
    after_tc = runtime.forward(0, x).clone()
    runtime.force("tile", "blocked")
    after_cuda_cores = runtime.forward(0, x).clone()
    assert not torch.equal(before, after_tc)
    assert float((after_tc - after_cuda_cores).abs().max()) <= 2e-5
    assert runtime.device_errors() == 0


def bf16_layer(layer):
    """The layer a bfloat16 runtime holds: every value and bias rounded to bfloat16."""
    import dataclasses
    r = lambda a: torch.from_numpy(a).to(torch.bfloat16).float().numpy()  # noqa: E731
    return dataclasses.replace(layer, up_val=r(layer.up_val), b_up=r(layer.b_up), down_val=r(layer.down_val),
                               b_down=r(layer.b_down))


@pytest.mark.parametrize("dtype,tc_format", [(torch.float32, "f16x3"), (torch.float32, "tf32x3"),
                                             (torch.bfloat16, None)])
def test_forced_tile_widths(dtype, tc_format):
    """Every token width of the forward GEMMs' tiles (forced process-wide, then back to the automatic choice) on ragged
    token counts, irregular supports: the same bits at every width (token columns are independent), within tolerance
    of the oracle on the layer and input the kernel holds (bfloat16: rounded)."""
    from hffn_b200 import _native as native
    case = synth.TEST_CASES["irreg_512_2048"]
    layer = synth.make_layer(case)
    held = layer if dtype == torch.float32 else bf16_layer(layer)
    runtime = tc_runtime(layer, dtype, tc_format)
    try:
        for n in (1, 65, 200, 777):
            x = torch.from_numpy(synth.make_input(case, n)).to(dtype)
            outputs = {}
            for width in (256, 128, 64):
                native.check(native.lib.hffn_set_tc_tile_tokens(width), "hffn_set_tc_tile_tokens")
                outputs[width] = runtime.forward(0, x.cuda()).clone()
            for width in (128, 64):
                assert torch.equal(outputs[width], outputs[256]), (width, n)
            rel = relative(outputs[256].float().cpu().numpy(), forward64.forward(held, x.float().numpy()))
            assert rel <= (1e-5 if dtype == torch.float32 else 2e-2), (n, rel)
    finally:
        native.check(native.lib.hffn_set_tc_tile_tokens(0), "hffn_set_tc_tile_tokens")
    assert runtime.device_errors() == 0
