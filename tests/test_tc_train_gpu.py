"""GPU parity of the MSE training step on the tensor cores (hffn_train_step_tc) through the C ABI.

Against the float64 oracle on the reference's test layers: y, gx and the four compact gradients within 1e-5 of each
group's scale, the loss within 1e-5 relative, AdamW against its float64 closed form on the conditioned entries
(relative 1e-5, the reference's gate 3), the same bits twice from the same state. At the training benchmark's layer
shape, where the oracle is too slow, the step is checked against the CUDA-core step (itself checked against the
oracle at that shape). 3xTF32: the dense tf32 pairs stay equal to a fresh densification of the updated compact values;
fp16x3: the step leaves the dense operands to be rebuilt, and the next forward sees the updated values."""
import numpy as np
import pytest
import torch

from hffn_b200 import synth
from oracle import train64

pytestmark = pytest.mark.gpu


def kernel_layer(layer):
    from hffn_b200.runtime import HFFNLayer
    t = torch.from_numpy
    return HFFNLayer.from_hidden_major(layer.d_model, layer.d_ff, t(layer.b_up), t(layer.up_offsets), t(layer.up_idx),
                                       t(layer.up_val), t(layer.b_down), t(layer.down_offsets), t(layer.down_idx),
                                       t(layer.down_val))


def make_train(layer, n, tensor_cores, tc_format=None):
    from hffn_b200.runtime import HFFNRuntime
    from hffn_b200.train_runtime import HFFNTrainRuntime
    runtime = HFFNRuntime([kernel_layer(layer)], "cuda", tensor_cores=True, tc_format=tc_format)
    return HFFNTrainRuntime(runtime, **train64.HYPER, max_tokens=n, tensor_cores=tensor_cores)


def perm_of(layer):
    return np.argsort(layer.down_idx.astype(np.int64), kind="stable")


@pytest.mark.parametrize("name,n", [("homog_512_2048", 300), ("irreg_512_2048", 257), ("homog_256_1024", 1)])
def test_against_oracle(name, n):
    case = synth.CASES[name]
    layer = synth.make_layer(case)
    x_np, t_np = synth.make_input(case, n), synth.make_target(case, n)
    ref = train64.step_groups(layer, x_np, train64.mse_upstream(t_np, n))
    train = make_train(layer, n, tensor_cores=True)
    before = {k: v.double().cpu().numpy() for k, v in train.parameters(0).items()}
    loss = float(train.step_mse(0, torch.from_numpy(x_np).cuda(), torch.from_numpy(t_np).cuda()))
    assert train.calls[("tc", "tc")] == 1 and train.runtime.device_errors() == 0
    assert abs(loss - train64.mse_loss(ref["y"], t_np)) <= 1e-5 * train64.mse_loss(ref["y"], t_np)
    perm = perm_of(layer)
    got = {"y": train.runtime._y[:n].double().cpu().numpy(), "gx": train._gx[:n].double().cpu().numpy()}
    grads = {k: v.double().cpu().numpy() for k, v in train.gradients(0).items()}
    got.update(g_up=grads["up_val"], gb_up=grads["b_up"], g_down=grads["out_val"], gb_down=grads["b_down"])
    expected = dict(ref, g_down=ref["g_down"][perm])
    for key in ("y", "gx", "g_up", "gb_up", "g_down", "gb_down"):
        scale = max(1.0 if key == "y" else 0.0, float(np.abs(expected[key]).max()))
        error = float(np.max(np.abs(got[key] - expected[key])))
        assert error <= 1e-5 * scale, (name, n, key, error, scale)
    after = {k: v.double().cpu().numpy() for k, v in train.parameters(0).items()}
    for g_name, p_name in (("g_up", "up_val"), ("gb_up", "b_up"), ("g_down", "out_val"), ("gb_down", "b_down")):
        p1, _, _ = train64.adamw_closed_form(before[p_name], grads[p_name], 0.0, 0.0, 1, **train64.HYPER)
        mask = np.abs(expected[g_name]) >= 1e-3 * np.abs(expected[g_name]).max()
        scale = np.maximum(np.abs(p1), np.abs(before[p_name]))
        if mask.any():
            assert np.max((np.abs(after[p_name] - p1) / np.maximum(scale, 1e-30))[mask]) <= 1e-5, p_name


@pytest.mark.parametrize("tc_format", ["tf32x3", "f16x3"])
def test_repeatable_and_dense_consistent(tc_format):
    """Three steps, twice from the same state: the same bits. 3xTF32: the dense tf32 pairs refreshed in place by the
    update equal a rebuild from the compact values. fp16x3: the step refreshes no dense operand and leaves both formats
    marked for a rebuild, and the next forward (fp16x3 operands rebuilt from the updated values) equals the CUDA-core
    forward of the same values."""
    case = synth.TEST_CASES["irreg_512_2048"]
    layer = synth.make_layer(case)
    n = 300
    x = torch.from_numpy(synth.make_input(case, n)).cuda()
    target = torch.from_numpy(synth.make_target(case, n)).cuda()
    states = []
    for _ in range(2):
        train = make_train(layer, n, tensor_cores=True, tc_format=tc_format)
        for _ in range(3):
            train.step_mse(0, x, target)
        states.append({k: v.clone() for k, v in train.parameters(0).items()})
        runtime = train.runtime
        if tc_format == "tf32x3":
            dense = {k: v.clone() for k, v in runtime._dense[0].items()}
            runtime._densify(0)
            for k, v in runtime._dense[0].items():
                assert torch.equal(v, dense[k]), k      # refreshed in place = rebuilt from the compact values
        else:
            assert runtime._dense_stale[0] and runtime._dense16_stale[0]
            runtime.force("tc", "tc")
            y_tc = runtime.forward(0, x).clone()
            runtime.force("tile", "blocked")
            y_cc = runtime.forward(0, x).clone()
            runtime.force(None, None)
            assert float((y_tc - y_cc).abs().max()) <= 2e-5
    for k in states[0]:
        assert torch.equal(states[0][k], states[1][k]), k


def test_c3_shape_against_cuda_cores():
    """The training benchmark's layer (d 2048, d_ff 8192, 80 %) at 256 tokens: tensor cores against CUDA cores."""
    case = synth.CONFIGS["c3_2048_8192_k1638"]
    layer = synth.make_layer(case)
    n = 256
    x = torch.from_numpy(synth.make_input(case, n)).cuda()
    target = torch.from_numpy(synth.make_target(case, n)).cuda()
    results = []
    for tensor_cores in (True, False):
        train = make_train(layer, n, tensor_cores=tensor_cores)
        loss = float(train.step_mse(0, x, target))
        grads = {k: v.double().cpu() for k, v in train.gradients(0).items()}
        results.append((loss, train._gx[:n].double().cpu(), grads, train.runtime.device_errors()))
    (loss_tc, gx_tc, g_tc, err_tc), (loss_cc, gx_cc, g_cc, _) = results
    assert err_tc == 0
    assert abs(loss_tc - loss_cc) <= 1e-5 * loss_cc
    assert float((gx_tc - gx_cc).abs().max()) <= 2e-5 * float(gx_cc.abs().max())
    for k in g_cc:
        assert float((g_tc[k] - g_cc[k]).abs().max()) <= 2e-5 * float(g_cc[k].abs().max()), k
