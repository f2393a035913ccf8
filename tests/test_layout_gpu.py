"""GPU: the device-side layout build (hffn_build_out_major, hffn_build_supports) through the C ABI.

The output-major down edges and the two transposed supports, built on the device from CUDA tensors, must carry the
SHA-256 digests of the reference's own ``HFFNLayer.from_hidden_major`` and ``transposed_supports`` run on the test
layers (``tests/golden/layout_digests.json``, written by ``tests/golden/make_golden.py``), and equal the host stable
sorts bit for bit at the training benchmark's layer size (13.4 M edges per projection). An index out of range is
refused (ValueError) without any out-of-range access (the kernels skip and flag it). A runtime built from a
device-laid-out layer gives the bits of the host-laid-out one.
"""
import hashlib
import json
from pathlib import Path

import numpy as np
import pytest
import torch

from hffn_b200 import synth

pytestmark = pytest.mark.gpu

GOLDEN = Path(__file__).resolve().parent / "golden"
ARRAYS = ("out_offsets", "out_hidden", "out_val", "in_offsets", "in_pos", "in_hidden", "hid_offsets", "hid_pos",
          "hid_output")


def device_layout(layer, device="cuda"):
    from hffn_b200.runtime import HFFNLayer
    from hffn_b200.train_runtime import transposed_supports
    t = lambda a: torch.from_numpy(np.ascontiguousarray(a)).to(device)  # noqa: E731
    kl = HFFNLayer.from_hidden_major(layer.d_model, layer.d_ff, t(layer.b_up), t(layer.up_offsets), t(layer.up_idx),
                                     t(layer.up_val), t(layer.b_down), t(layer.down_offsets), t(layer.down_idx),
                                     t(layer.down_val))
    return kl, transposed_supports(kl)


def host_layout(layer):
    from hffn_b200.runtime import HFFNLayer
    from hffn_b200.train_runtime import transposed_supports
    t = torch.from_numpy
    kl = HFFNLayer.from_hidden_major(layer.d_model, layer.d_ff, t(layer.b_up), t(layer.up_offsets), t(layer.up_idx),
                                     t(layer.up_val), t(layer.b_down), t(layer.down_offsets), t(layer.down_idx),
                                     t(layer.down_val))
    return kl, transposed_supports(kl)


def arrays_of(kl, sup) -> dict:
    out = {"out_offsets": kl.out_offsets, "out_hidden": kl.out_hidden, "out_val": kl.out_val, **sup}
    return {k: v.cpu().contiguous().numpy() for k, v in out.items()}


@pytest.mark.parametrize("name", ["homog_256_1024", "irreg_512_2048"])
def test_device_layout_matches_reference_digests(name):
    digests = json.loads((GOLDEN / "layout_digests.json").read_text())[name]
    kl, sup = device_layout(synth.make_layer(synth.TEST_CASES[name]))
    assert kl.out_hidden.is_cuda and sup["hid_pos"].is_cuda
    arrays = arrays_of(kl, sup)
    for key in ARRAYS:
        assert hashlib.sha256(arrays[key].tobytes()).hexdigest() == digests[key], (name, key)


def test_device_layout_equals_host_at_training_size():
    layer = synth.make_layer(synth.CONFIGS["c3_2048_8192_k1638"])
    device = arrays_of(*device_layout(layer))
    host = arrays_of(*host_layout(layer))
    for key in ARRAYS:
        assert device[key].dtype == host[key].dtype and np.array_equal(device[key], host[key]), key


def test_bf16_values_and_runtime_from_device_layer():
    from hffn_b200.runtime import HFFNRuntime
    case = synth.TEST_CASES["irreg_512_2048"]
    layer = synth.make_layer(case)
    x = torch.from_numpy(synth.make_input(case, 37)).cuda()
    y_host = HFFNRuntime([host_layout(layer)[0]], "cuda").forward(0, x).clone()
    y_dev = HFFNRuntime([device_layout(layer)[0]], "cuda").forward(0, x).clone()
    assert torch.equal(y_host, y_dev)
    from hffn_b200 import layout_device
    t = lambda a: torch.from_numpy(np.ascontiguousarray(a)).cuda()  # noqa: E731
    _, _, val16 = layout_device.out_major(layer.d_model, layer.d_ff, t(layer.down_offsets), t(layer.down_idx),
                                          t(layer.down_val).to(torch.bfloat16))
    _, _, val32 = layout_device.out_major(layer.d_model, layer.d_ff, t(layer.down_offsets), t(layer.down_idx),
                                          t(layer.down_val))
    assert torch.equal(val16, val32.to(torch.bfloat16))


def test_out_of_range_index_refused():
    from hffn_b200 import layout_device
    layer = synth.make_layer(synth.TEST_CASES["homog_256_1024"])
    bad = layer.down_idx.copy()
    bad[100] = layer.d_model + 5                    # one edge to an output that does not exist
    t = lambda a: torch.from_numpy(np.ascontiguousarray(a)).cuda()  # noqa: E731
    with pytest.raises(ValueError):
        layout_device.out_major(layer.d_model, layer.d_ff, t(layer.down_offsets), t(bad), t(layer.down_val))
    # the context stays usable: a valid build right after
    offsets, _, _ = layout_device.out_major(layer.d_model, layer.d_ff, t(layer.down_offsets), t(layer.down_idx),
                                            t(layer.down_val))
    assert int(offsets[-1]) == layer.down_idx.size
