"""CPU: the product's host layouts (HFFNLayer.from_hidden_major, transposed_supports) equal the oracle's bit for bit,
and malformed layers are refused."""
import numpy as np
import pytest
import torch

from hffn_b200 import synth
from oracle import layout


def kernel_layer(layer):
    from hffn_b200.runtime import HFFNLayer
    t = torch.from_numpy
    return HFFNLayer.from_hidden_major(layer.d_model, layer.d_ff, t(layer.b_up), t(layer.up_offsets), t(layer.up_idx),
                                       t(layer.up_val), t(layer.b_down), t(layer.down_offsets), t(layer.down_idx),
                                       t(layer.down_val))


@pytest.mark.parametrize("name", ["homog_256_1024", "irreg_512_2048", "c1_512_2048_k128"])
def test_layouts_bit_exact(name):
    from hffn_b200.train_runtime import transposed_supports
    layer = synth.make_layer(synth.CASES[name])
    kl = kernel_layer(layer)
    om = layout.out_major(layer.d_model, layer.d_ff, layer.down_offsets, layer.down_idx, layer.down_val)
    for key in ("out_offsets", "out_hidden", "out_val"):
        assert np.array_equal(getattr(kl, key).numpy(), om[key]), key
    ts = transposed_supports(kl)
    ref = layout.transposed_supports(layer.d_model, layer.d_ff, layer.up_offsets, layer.up_idx, om["out_offsets"],
                                     om["out_hidden"])
    for key, value in ref.items():
        assert ts[key].dtype == torch.from_numpy(value).dtype and np.array_equal(ts[key].numpy(), value), key
    kl.validate()


def test_malformed_layers_refused():
    import dataclasses
    layer = kernel_layer(synth.make_layer(synth.TEST_CASES["homog_256_1024"]))
    bad_offsets = layer.up_offsets.clone()
    bad_offsets[-1] += 1
    with pytest.raises(ValueError):
        dataclasses.replace(layer, up_offsets=bad_offsets).validate()
    bad_idx = layer.up_idx.clone()
    bad_idx[3] = layer.d_model
    with pytest.raises(ValueError):
        dataclasses.replace(layer, up_idx=bad_idx).validate()
    dec = layer.out_offsets.clone()
    dec[5], dec[6] = dec[6], dec[5] - 1
    with pytest.raises(ValueError):
        dataclasses.replace(layer, out_offsets=dec).validate()


def test_runtime_refuses_cpu_device():
    from hffn_b200.runtime import HFFNRuntime
    layer = kernel_layer(synth.make_layer(synth.TEST_CASES["homog_256_1024"]))
    with pytest.raises(ValueError):
        HFFNRuntime([layer], "cpu")
