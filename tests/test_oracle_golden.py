"""CPU: the oracle and the generator pinned against the reference's own outputs (tests/golden, made by running the
reference's Python oracles) and against the reference's x86 kernel compiled from its sources (oracle/_ref)."""
import hashlib
import json

import numpy as np
import pytest

from hffn_b200 import synth
from oracle import forward64, layout, train64, x86ref, x86train


def load(golden, name):
    with np.load(golden / name) as data:
        return {k: data[k] for k in data.files}


@pytest.mark.parametrize("name", sorted(synth.TEST_CASES))
def test_generator_matches_pinned_fingerprint(golden, name):
    pinned = json.loads((golden / "fingerprints.json").read_text())["fingerprints"]
    case = synth.TEST_CASES[name]
    assert synth.fingerprint(synth.make_layer(case), case) == pinned[name]


FORWARD = [("homog_256_1024", 1), ("homog_256_1024", 7), ("homog_256_1024", 64), ("homog_512_2048", 1),
           ("homog_512_2048", 5), ("irreg_512_2048", 1), ("irreg_512_2048", 9), ("irreg_512_2048", 33)]


@pytest.mark.parametrize("name,n", FORWARD)
def test_forward64_matches_reference_oracle(golden, name, n):
    case = synth.TEST_CASES[name]
    layer = synth.make_layer(case)
    g = load(golden, f"forward_{name}_n{n}.npz")
    x = synth.make_input(case, n)
    assert np.array_equal(x, g["x"])
    y = forward64.forward(layer, x)
    # golden outputs are stored as float32: agreement to float32 rounding pins the algorithm
    assert np.max(np.abs(y - g["y"]) / np.maximum(1.0, np.abs(y))) < 1e-6


@pytest.mark.parametrize("name,n", [("homog_256_1024", 1), ("homog_256_1024", 7), ("irreg_512_2048", 3)])
def test_train64_matches_reference_oracle(golden, name, n):
    case = synth.TEST_CASES[name]
    layer = synth.make_layer(case)
    g = load(golden, f"train_{name}_n{n}.npz")
    assert np.array_equal(synth.make_upstream(case, n, 0), g["gy"])
    out = train64.step_groups(layer, g["x"], g["gy"])
    for key in train64.GROUPS:
        ref = g[key].astype(np.float64)
        scale = max(1.0, float(np.abs(ref).max()))
        assert np.max(np.abs(out[key] - ref)) <= 1e-6 * scale, key
    p, m, v = train64.adamw_closed_form(layer.up_val.astype(np.float64), out["g_up"], 0.0, 0.0, 1, **train64.HYPER)
    k = g["adamw_up_val"].size
    assert np.allclose(p[:k], g["adamw_up_val"], rtol=1e-6, atol=1e-9)
    assert np.allclose(m[:k], g["adamw_m"], rtol=1e-5, atol=1e-12)
    assert np.allclose(v[:k], g["adamw_v"], rtol=1e-5, atol=1e-18)


def test_layout_matches_reference_functions(golden):
    digests = json.loads((golden / "layout_digests.json").read_text())
    for name in ("homog_256_1024", "irreg_512_2048"):
        layer = synth.make_layer(synth.TEST_CASES[name])
        om = layout.out_major(layer.d_model, layer.d_ff, layer.down_offsets, layer.down_idx, layer.down_val)
        sup = layout.transposed_supports(layer.d_model, layer.d_ff, layer.up_offsets, layer.up_idx,
                                         om["out_offsets"], om["out_hidden"])
        arrays = {"out_offsets": om["out_offsets"], "out_hidden": om["out_hidden"], "out_val": om["out_val"], **sup}
        for key, digest in digests[name].items():
            assert hashlib.sha256(np.ascontiguousarray(arrays[key]).tobytes()).hexdigest() == digest, (name, key)
    g = load(golden, "layout_homog_256_1024.npz")
    layer = synth.make_layer(synth.TEST_CASES["homog_256_1024"])
    om = layout.out_major(layer.d_model, layer.d_ff, layer.down_offsets, layer.down_idx, layer.down_val)
    assert np.array_equal(om["out_hidden"], g["out_hidden"]) and np.array_equal(om["out_offsets"], g["out_offsets"])


def test_negative_control_detected(golden):
    """A planted mistake in the oracle (one weight scaled) must be seen by the golden comparison."""
    case = synth.TEST_CASES["homog_256_1024"]
    layer = synth.make_layer(case)
    g = load(golden, "forward_homog_256_1024_n7.npz")
    bad = layer.up_val.copy()
    bad[100] *= 1.5
    tampered = synth.CompactLayer(**{**layer.__dict__, "up_val": bad})
    y = forward64.forward(tampered, g["x"])
    assert np.max(np.abs(y - g["y"])) > 1e-4


@pytest.mark.skipif(not x86ref.available(), reason="oracle/_ref not built (make -C oracle)")
@pytest.mark.parametrize("name,n", [("homog_512_2048", 1), ("homog_512_2048", 5), ("irreg_512_2048", 96),
                                    ("irreg_512_2048", 130)])
def test_reference_x86_kernel_matches_forward64(name, n):
    case = synth.TEST_CASES[name]
    layer = synth.make_layer(case)
    x = synth.make_input(case, n)
    y = x86ref.X86Kernel(layer, threads=4).forward(x)
    assert np.max(np.abs(y - forward64.forward(layer, x))) <= 2e-5


@pytest.mark.skipif(not x86train.available(), reason="oracle/_ref not built (make -C oracle)")
@pytest.mark.parametrize("name,n", [("homog_256_1024", 64), ("irreg_512_2048", 40)])
def test_reference_g4_training_step_matches_train64(name, n):
    """The reference's own CPU training step (forward, backward, AdamW of the G4 kernel) against the float64 oracle:
    every gradient group within 2e-5 of its scale, the updated values against the AdamW closed form."""
    case = synth.TEST_CASES[name]
    layer = synth.make_layer(case)
    x, target = synth.make_input(case, n), synth.make_target(case, n)
    step = x86train.G4Step(layer, n, **train64.HYPER)
    before = step.up_val.copy()
    loss = step.step_mse(x, target)
    ref = train64.step_groups(layer, x, train64.mse_upstream(target, n))
    assert abs(loss - train64.mse_loss(ref["y"], target)) <= 1e-5 * train64.mse_loss(ref["y"], target)
    got = step.gradients()
    for key in ("g_up", "g_down", "gb_up", "gb_down", "gx"):
        expected = np.asarray(ref[key])
        assert np.max(np.abs(got[key] - expected)) <= 2e-5 * np.abs(expected).max(), key
    p1, _, _ = train64.adamw_closed_form(before.astype(np.float64), got["g_up"].astype(np.float64), 0.0, 0.0, 1,
                                         **train64.HYPER)
    mask = np.abs(ref["g_up"]) >= 1e-3 * np.abs(ref["g_up"]).max()
    scale = np.maximum(np.abs(p1), np.abs(before))
    assert np.max((np.abs(step.up_val - p1) / scale)[mask]) <= 1e-5
