"""GPU: gates 1 and 5 and the workspace guards of the reference's training check, on this build.

Mirrors ``runtime/gpu/nvidia/ffn/training/check.py:1-12,57-120`` with the criteria of
``runtime/gpu/nvidia/ffn/training/train_step.py:18-25,234-364``, in this repository's code:

- gate 1: the training runtime's forward without ``z`` equals the inference runtime's forward bit for bit, under the
  policy and every forced pair (the nine CUDA-core pairs and the tensor-core pair), for N in ``GATE1_N``;
- gate 5, pass A: five consecutive steps, each update against the float64 AdamW closed form started from the build's
  own pre-update parameters and moments and fed the build's own gradient of that step, on the conditioned entries
  (value relative to max(|ref|, |pre|, lr), m relative to max(|m_ref|, beta1 |m_pre|, (1 - beta1) |g|), v relative to
  |v_ref|), tolerance 1e-5; the step counter must advance by one per step;
- gate 5, pass B: from the same initial state, five steps whose upstream gradient is zero (decoupled decay only),
  the parameters after the last step against the float64 chain fed the build's gradients, relative to
  max(|ref|, |initial|), tolerance 1e-5;
- guards: a partial workspace beyond 32-bit indexing is refused, the same N does not grow any buffer, a larger N is
  counted as a growth.

Both step paths run gate 5: the CUDA-core step (``step`` on a given upstream gradient) and the tensor-core MSE step
(``step_mse_tc``), whose dense operands are refreshed in place by each update. The tensor-core pass reads the state
through the runtime's tensors, which leaves the dense operands as the last update left them, so a stale operand would
show in the next step's update. Its upstream gradient is the MSE gradient, ``2 (y - target) / (N d)``: pass A uses
five seeded targets, pass B the target equal to the current output (the forward of the same operands), whose
gradients must be negligible (<= 1e-6 of pass A's) rather than exactly zero, since the step's output is computed by
another GEMM configuration than the forward's.
"""
import numpy as np
import pytest
import torch

from hffn_b200 import synth
from oracle import train64
from test_train_gpu import dense_control, dist, kernel_layer, perm_of

pytestmark = pytest.mark.gpu

LAYER = "homog_256_1024"
CASES = (1, 33, 100, 128, 257, 300, 512, 1024, 2100)
GATE1_N = (1, 2, 4, 5, 63, 64, 128, 129, 512)
GATE3_CONDITIONING = 100.0
GATE5_RELATIVE = 1e-5
STEPS = 5
PARAM_OF = {"g_up": "up_val", "gb_up": "b_up", "g_down": "out_val", "gb_down": "b_down"}
JUDGED = ("g_up", "g_down")


def new_train(layer, n, **kw):
    from hffn_b200.runtime import HFFNRuntime
    from hffn_b200.train_runtime import HFFNTrainRuntime
    train = HFFNTrainRuntime(HFFNRuntime([kernel_layer(layer)], "cuda"), **train64.HYPER, max_tokens=max(n, 2048), **kw)
    train.reserve(n)
    return train


def read_state(train) -> dict:
    """Parameters and moments of layer 0 in the runtime's order (out_val output-major), float64 CPU; read through the
    runtime's tensors, which does not invalidate the dense tensor-core operands."""
    values, moments = train.runtime._tensors[0], train.moments(0)
    return {p: tuple(t.double().cpu() for t in (values[p], *moments[p])) for p in PARAM_OF.values()}


def snapshot(train) -> dict:
    return {"state": {p: tuple(t.clone() for t in (train.runtime._tensors[0][p], *train.moments(0)[p]))
                      for p in PARAM_OF.values()}, "steps": train.steps[0]}


def restore(train, saved) -> None:
    """Write a saved state back the way the reference's checks do: through ``parameters()`` and ``moments()``."""
    params, moments = train.parameters(0), train.moments(0)
    for p, (value, m, v) in saved["state"].items():
        params[p].copy_(value)
        moments[p][0].copy_(m)
        moments[p][1].copy_(v)
    train.steps[0] = saved["steps"]


def build_gradients(train) -> dict:
    grads = train.gradients(0)
    return {g: grads[p].double().cpu() for g, p in PARAM_OF.items()}


def rel(a, b, scale, mask) -> float:
    return float(((a - b).abs() / scale.clamp_min(1e-30))[mask].max())


def closed_form(p, g, m, v, k):
    out = train64.adamw_closed_form(p.numpy(), g.numpy(), m.numpy(), v.numpy(), k, **train64.HYPER)
    return tuple(torch.from_numpy(np.asarray(a, np.float64)) for a in out)


def conditioned_masks(layer, x_np, gy_np, x, gy) -> dict:
    """Entries whose float64 |gradient| >= 100 x the dense float32 control's distance (the gate-3 masks), in the
    runtime's order."""
    ref = {k: torch.from_numpy(np.asarray(v)) for k, v in train64.step_groups(layer, x_np, gy_np).items()}
    control = dense_control(layer, x, gy)
    perm = perm_of(layer)
    masks = {}
    for g in PARAM_OF:
        mask = ref[g].abs() >= GATE3_CONDITIONING * dist(control[g], ref[g])
        masks[g] = mask[perm] if g == "g_down" else mask
    return masks


def gate5(train, masks: dict, step, zero_step) -> dict:
    """Pass A (``step(k)`` for k = 1..5) and pass B (``zero_step()`` five times) from the same initial state; the
    worst error of each judged group and pass, and the largest |gradient| read in pass B. Leaves the initial state."""
    beta1 = train64.HYPER["betas"][0]
    lr = train64.HYPER["lr"]
    initial = snapshot(train)
    start = read_state(train)
    k0 = train.steps[0]
    worst = {g: 0.0 for g in JUDGED}
    counters, pass_a_scale = [], 0.0
    for k in range(1, STEPS + 1):
        pre = read_state(train)
        step(k)
        counters.append(train.steps[0] - k0)
        post, grads = read_state(train), build_gradients(train)
        for g in JUDGED:
            p = PARAM_OF[g]
            p_pre, m_pre, v_pre = pre[p]
            ref_p, ref_m, ref_v = closed_form(p_pre, grads[g], m_pre, v_pre, k0 + k)
            got_p, got_m, got_v = post[p]
            mask = masks[g]
            assert mask.any(), g
            pass_a_scale = max(pass_a_scale, float(grads[g].abs().max()))
            errors = (rel(got_p, ref_p, torch.maximum(ref_p.abs(), p_pre.abs()).clamp_min(lr), mask),
                      rel(got_m, ref_m, torch.maximum(torch.maximum(ref_m.abs(), beta1 * m_pre.abs()),
                                                      (1 - beta1) * grads[g].abs()), mask),
                      rel(got_v, ref_v, ref_v.abs(), mask))
            worst[g] = max(worst[g], *errors)
            assert all(bool(torch.isfinite(t).all()) for t in post[p])
    restore(train, initial)
    chain = {g: start[PARAM_OF[g]] for g in JUDGED}
    decay_gradient = 0.0
    for k in range(1, STEPS + 1):
        zero_step()
        grads = build_gradients(train)
        for g in JUDGED:
            decay_gradient = max(decay_gradient, float(grads[g].abs().max()))
            chain[g] = closed_form(*chain[g][:1], grads[g], *chain[g][1:], k0 + k)
    after = read_state(train)
    decay = {g: rel(after[PARAM_OF[g]][0], chain[g][0],
                    torch.maximum(chain[g][0].abs(), start[PARAM_OF[g]][0].abs()), masks[g]) for g in JUDGED}
    restore(train, initial)
    return {"local": worst, "decay": decay, "counters": counters, "decay_gradient": decay_gradient,
            "pass_a_gradient": pass_a_scale}


def test_gate1_inference_identity():
    from hffn_b200.parity import PAIRS
    from hffn_b200.runtime import HFFNRuntime
    case = synth.TEST_CASES[LAYER]
    layer = synth.make_layer(case)
    baseline = HFFNRuntime([kernel_layer(layer)], "cuda")
    train = new_train(layer, 1)
    pairs = [(None, None), *PAIRS, ("tc", "tc")]
    with torch.no_grad():
        for m in GATE1_N:
            x = torch.from_numpy(synth.make_input(case, m)).cuda()
            for pair in pairs:
                baseline.force(*pair)
                train.runtime.force(*pair)
                assert torch.equal(baseline.forward(0, x).clone(), train.forward(0, x).clone()), (m, pair)
    baseline.force(None, None)
    train.runtime.force(None, None)


@pytest.mark.parametrize("n", CASES)
def test_gate5_cuda_cores(n):
    case = synth.TEST_CASES[LAYER]
    layer = synth.make_layer(case)
    x_np = synth.make_input(case, n)
    x = torch.from_numpy(x_np).cuda()
    gy1 = synth.make_upstream(case, n, 1)
    masks = conditioned_masks(layer, x_np, gy1, x, torch.from_numpy(gy1).cuda())
    train = new_train(layer, n)
    upstream = {k: torch.from_numpy(synth.make_upstream(case, n, k)).cuda() for k in range(1, STEPS + 1)}
    zero = torch.zeros(n, case.d_model, device="cuda")
    result = gate5(train, masks, lambda k: train.step(0, x, upstream[k]), lambda: train.step(0, x, zero))
    assert result["counters"] == list(range(1, STEPS + 1))
    assert result["decay_gradient"] == 0.0                 # pass B read no gradient: decay only
    for g in JUDGED:
        assert result["local"][g] <= GATE5_RELATIVE, (n, g, result)
        assert result["decay"][g] <= GATE5_RELATIVE, (n, g, result)


def seeded_target(case, n, k) -> np.ndarray:
    rng = np.random.default_rng([case.seed, n, 7919, 100 + k])
    return np.ascontiguousarray(rng.standard_normal((n, case.d_model)).astype(np.float32))


@pytest.mark.parametrize("n", (257, 300, 1024, 2100))
def test_gate5_tensor_cores(n):
    case = synth.TEST_CASES[LAYER]
    layer = synth.make_layer(case)
    x_np = synth.make_input(case, n)
    x = torch.from_numpy(x_np).cuda()
    targets = {k: seeded_target(case, n, k) for k in range(1, STEPS + 1)}
    y64 = train64.step_groups(layer, x_np, np.zeros((n, case.d_model)))["y"]
    gy1 = np.asarray(train64.mse_upstream(targets[1], n)(y64, 0, n), np.float32)
    masks = conditioned_masks(layer, x_np, gy1, x, torch.from_numpy(gy1).cuda())
    train = new_train(layer, n, tensor_cores=True)
    target_dev = {k: torch.from_numpy(t).cuda() for k, t in targets.items()}

    def zero_step():
        train.runtime.force("tc", "tc")
        y = train.runtime.forward(0, x).clone()          # the current operands' output: the MSE gradient vanishes
        train.runtime.force(None, None)
        train.step_mse_tc(0, x, y)

    result = gate5(train, masks, lambda k: train.step_mse_tc(0, x, target_dev[k]), zero_step)
    assert train.runtime.device_errors() == 0
    assert result["counters"] == list(range(1, STEPS + 1))
    assert result["decay_gradient"] <= 1e-6 * result["pass_a_gradient"], result
    for g in JUDGED:
        assert result["local"][g] <= GATE5_RELATIVE, (n, g, result)
        assert result["decay"][g] <= GATE5_RELATIVE, (n, g, result)


def test_workspace_guards():
    case = synth.TEST_CASES[LAYER]
    layer = synth.make_layer(case)
    train = new_train(layer, 1)
    stride = max(c[3] for c in train._columns)
    assert train._columns[0] == (layer.down_val.size, layer.down_val.size + case.d_model,
                                 layer.down_val.size + case.d_model + layer.up_val.size,
                                 layer.down_val.size + case.d_model + layer.up_val.size + case.d_ff)
    with pytest.raises(ValueError):
        train._reserve_partials(2 ** 32 // stride * 256 + 256)
    before = train.growths
    train.reserve(train._tokens)
    assert train.growths == before
    train.reserve(train._tokens + 1)
    assert train.growths > before
