"""GPU parity of the training step (through the C ABI) against the float64 oracle, in the form of the reference's
gates (``runtime/gpu/nvidia/ffn/training/check.py:1-12``, ``train_step.py:174-231``):
 2 every group within 10x the distance of a dense float32 control (PyTorch, TF32 off), floor 1e-7 x scale;
 3 one AdamW update against its float64 closed form on the conditioned entries, relative 1e-5;
 4 the same bits twice from the same state; the fused backward + AdamW gives the bits of backward then adamw;
plus the MSE step of the training benchmark and the no-growth guard."""
import numpy as np
import pytest
import torch
import torch.nn.functional as F

from hffn_b200 import synth
from oracle import train64

pytestmark = pytest.mark.gpu

LAYER = "homog_256_1024"
CASES = (1, 33, 100, 128, 257, 300, 512, 1024, 2100)
GATE2_FACTOR, GATE2_FLOOR = 10.0, 1e-7
GATE3_CONDITIONING, GATE3_RELATIVE = 100.0, 1e-5


def kernel_layer(layer):
    from hffn_b200.runtime import HFFNLayer
    t = torch.from_numpy
    return HFFNLayer.from_hidden_major(layer.d_model, layer.d_ff, t(layer.b_up), t(layer.up_offsets), t(layer.up_idx),
                                       t(layer.up_val), t(layer.b_down), t(layer.down_offsets), t(layer.down_idx),
                                       t(layer.down_val))


def make_train(layer, n, **kw):
    from hffn_b200.runtime import HFFNRuntime
    from hffn_b200.train_runtime import HFFNTrainRuntime
    train = HFFNTrainRuntime(HFFNRuntime([kernel_layer(layer)], "cuda"), **train64.HYPER, max_tokens=n, **kw)
    train.reserve(n)
    return train


def perm_of(layer):
    return torch.from_numpy(np.argsort(layer.down_idx.astype(np.int64), kind="stable"))


def groups_of(train, layer, n):
    """The seven groups, hidden-major slot order (g_down mapped back from output-major), float64 CPU."""
    perm = perm_of(layer)
    grads, acts = train.gradients(0), train.activations(n)
    g_down = torch.empty(grads["out_val"].numel(), dtype=torch.float64)
    g_down[perm] = grads["out_val"].double().cpu()
    return {"y": train.runtime._y[:n].double().cpu(), "gb_down": grads["b_down"].double().cpu(), "g_down": g_down,
            "gz": acts["gz"].double().cpu(), "g_up": grads["up_val"].double().cpu(),
            "gb_up": grads["b_up"].double().cpu(), "gx": acts["gx"].double().cpu()}


def dense_control(layer, x, gy):
    """Dense float32 iso-support step with autograd (TF32 off): the control arm of the reference's gate 2."""
    torch.backends.cuda.matmul.allow_tf32 = False
    d, f = layer.d_model, layer.d_ff
    up_h = np.repeat(np.arange(f), np.diff(layer.up_offsets))
    dn_h = np.repeat(np.arange(f), np.diff(layer.down_offsets))
    w_up = torch.zeros(f, d, device="cuda")
    w_up[up_h, layer.up_idx.astype(np.int64)] = torch.from_numpy(layer.up_val).cuda()
    w_dn = torch.zeros(d, f, device="cuda")
    w_dn[layer.down_idx.astype(np.int64), dn_h] = torch.from_numpy(layer.down_val).cuda()
    w_up.requires_grad_()
    w_dn.requires_grad_()
    b_up = torch.from_numpy(layer.b_up.copy()).cuda().requires_grad_()
    b_dn = torch.from_numpy(layer.b_down.copy()).cuda().requires_grad_()
    xg = x.clone().requires_grad_()
    z = F.linear(xg, w_up, b_up)
    z.retain_grad()
    y = F.linear(F.gelu(z, approximate="none"), w_dn, b_dn)
    y.backward(gy)
    return {"y": y.detach().double().cpu(), "gz": z.grad.T.double().cpu(), "gx": xg.grad.double().cpu(),
            "g_up": w_up.grad[up_h, layer.up_idx.astype(np.int64)].double().cpu(), "gb_up": b_up.grad.double().cpu(),
            "g_down": w_dn.grad[layer.down_idx.astype(np.int64), dn_h].double().cpu(), "gb_down": b_dn.grad.double().cpu()}


def dist(a, b):
    return float((torch.as_tensor(a).double() - torch.as_tensor(b).double()).abs().max())


@pytest.mark.parametrize("n", CASES)
def test_gates(n):
    case = synth.TEST_CASES[LAYER]
    layer = synth.make_layer(case)
    x_np, gy_np = synth.make_input(case, n), synth.make_upstream(case, n, 0)
    x, gy = torch.from_numpy(x_np).cuda(), torch.from_numpy(gy_np).cuda()
    ref = {k: torch.from_numpy(np.asarray(v)) for k, v in train64.step_groups(layer, x_np, gy_np).items()}
    control = dense_control(layer, x, gy)

    # separate phases: forward(z), backward, adamw
    train = make_train(layer, n)
    growths = train.growths
    before = {k: v.clone() for k, v in train.parameters(0).items()}
    train.forward(0, x, train._z)
    train.backward(0, gy)
    hffn = groups_of(train, layer, n)
    for name in train64.GROUPS:
        scale = float(ref[name].abs().max())
        tolerance = GATE2_FACTOR * max(dist(control[name], ref[name]), GATE2_FLOOR * scale)
        assert dist(hffn[name], ref[name]) <= tolerance, (n, name, dist(hffn[name], ref[name]), tolerance)
    separate_grads = {k: v.clone() for k, v in train.gradients(0).items()}
    train.adamw(0)
    separate = {k: v.clone() for k, v in train.parameters(0).items()}
    separate_m = {k: (a.clone(), b.clone()) for k, (a, b) in train.moments(0).items()}

    # gate 3: the update against the float64 closed form fed the build's own gradient
    perm = perm_of(layer)
    for g_name, p_name in (("g_up", "up_val"), ("gb_up", "b_up"), ("g_down", "out_val"), ("gb_down", "b_down")):
        mask = ref[g_name].abs() >= GATE3_CONDITIONING * dist(control[g_name], ref[g_name])
        g_build = separate_grads[p_name].double().cpu()
        p0 = before[p_name].double().cpu()
        p1, m1, v1 = train64.adamw_closed_form(p0.numpy(), g_build.numpy(), 0.0, 0.0, 1, **train64.HYPER)
        got_p, (got_m, got_v) = separate[p_name].double().cpu(), separate_m[p_name]
        if p_name == "out_val":   # compare in the runtime's output-major order
            mask = mask[perm]
        p1, m1, v1 = (torch.from_numpy(np.asarray(a)) for a in (p1, m1, v1))
        if mask.any():
            scale = torch.maximum(p1.abs(), p0.abs())
            assert float(((got_p - p1).abs() / scale.clamp_min(1e-30))[mask].max()) <= GATE3_RELATIVE, p_name
            assert float(((got_m.double().cpu() - m1).abs() / m1.abs().clamp_min(1e-30))[mask].max()) <= GATE3_RELATIVE
            assert float(((got_v.double().cpu() - v1).abs() / v1.abs().clamp_min(1e-30))[mask].max()) <= GATE3_RELATIVE

    # gate 4: the fused step from the same initial state gives the bits of the separate phases, twice
    for _ in range(2):
        fused = make_train(layer, n)
        fused.step(0, x, gy)
        for k in separate:
            assert torch.equal(fused.parameters(0)[k], separate[k]), (n, k)
            assert torch.equal(fused.gradients(0)[k], separate_grads[k]), (n, k)
            assert torch.equal(fused.moments(0)[k][0], separate_m[k][0]) and torch.equal(fused.moments(0)[k][1], separate_m[k][1])
        assert torch.equal(fused.activations(n)["gx"], train.activations(n)["gx"])
    assert train.growths == growths


def test_step_sizes_its_own_buffers():
    """A runtime built for one token and stepped at N sizes its z / gz / gx buffers itself."""
    from hffn_b200.runtime import HFFNRuntime
    from hffn_b200.train_runtime import HFFNTrainRuntime
    case = synth.TEST_CASES[LAYER]
    layer = synth.make_layer(case)
    train = HFFNTrainRuntime(HFFNRuntime([kernel_layer(layer)], "cuda"))
    x = torch.from_numpy(synth.make_input(case, 37)).cuda()
    gy = torch.from_numpy(synth.make_upstream(case, 37, 0)).cuda()
    gx = train.step(0, x, gy)
    assert gx.shape == (37, layer.d_model) and bool(torch.isfinite(gx).all())


def test_backward_order_refused():
    case = synth.TEST_CASES[LAYER]
    layer = synth.make_layer(case)
    train = make_train(layer, 16)
    x = torch.from_numpy(synth.make_input(case, 16)).cuda()
    with pytest.raises(RuntimeError):
        train.backward(0, x)
    train.forward(0, x, train._z)
    train.runtime.forward(0, x)
    with pytest.raises(RuntimeError):
        train.backward(0, x)


@pytest.mark.parametrize("name,n", [("irreg_512_2048", 300), ("c1_512_2048_k128", 256)])
def test_mse_step(name, n):
    case = synth.CASES[name]
    layer = synth.make_layer(case)
    x_np, t_np = synth.make_input(case, n), synth.make_target(case, n)
    ref = train64.step_groups(layer, x_np, train64.mse_upstream(t_np, n))
    train = make_train(layer, n)
    before = {k: v.double().cpu().numpy() for k, v in train.parameters(0).items()}
    loss = float(train.step_mse(0, torch.from_numpy(x_np).cuda(), torch.from_numpy(t_np).cuda()))
    assert abs(loss - train64.mse_loss(ref["y"], t_np)) <= 1e-5 * train64.mse_loss(ref["y"], t_np)
    perm = perm_of(layer).numpy()
    grads = {k: v.double().cpu().numpy() for k, v in train.gradients(0).items()}
    for g_name, p_name in (("g_up", "up_val"), ("g_down", "out_val")):
        g_ref = ref[g_name] if p_name == "up_val" else ref[g_name][perm]
        scale = np.abs(g_ref).max()
        assert np.max(np.abs(grads[p_name] - g_ref)) <= 1e-4 * scale, g_name
        p1, _, _ = train64.adamw_closed_form(before[p_name], grads[p_name], 0.0, 0.0, 1, **train64.HYPER)
        got = train.parameters(0)[p_name].double().cpu().numpy()
        assert np.max(np.abs(got - p1) / np.maximum(np.abs(p1), 1e-3)) <= 1e-5


def test_c3_shape_small_batch():
    """The training benchmark's layer shape (d 2048, d_ff 8192, 80 % density) at a batch the oracle finishes."""
    case = synth.CONFIGS["c3_2048_8192_k1638"]
    layer = synth.make_layer(case)
    n = 6
    x_np, t_np = synth.make_input(case, n), synth.make_target(case, n)
    ref = train64.step_groups(layer, x_np, train64.mse_upstream(t_np, n), chunk=3)
    train = make_train(layer, n)
    train.runtime.force("tile", "blocked")   # the staged-tile kernels at this shape (the policy picks coop at N <= 8)
    train.step_mse(0, torch.from_numpy(x_np).cuda(), torch.from_numpy(t_np).cuda())
    got = groups_of(train, layer, n)
    for name in ("y", "g_up", "g_down", "gx", "gb_up", "gb_down"):
        r = torch.from_numpy(np.asarray(ref[name]))
        scale = max(1.0 if name == "y" else 0.0, float(r.abs().max()))
        assert dist(got[name], r) <= 1e-5 * scale, (name, dist(got[name], r), scale)
