"""GPU: the fp16x3 operand format of the float32 tensor-core forward (``hffn_densify_f16x3``, ``hffn_forward_f16x3``,
``hffn_up_f16x3`` / ``hffn_down_f16x3``) through the C ABI, against the float64 oracle.

- The operands: (hi + lo) x 2^-e_r gives every weight back within 2^-22 of its row's largest |value|, each row's
  largest scaled |value| lies in [2^14, 2^15), and ``up_bound`` holds the largest row L1 norm and the largest |b_up|.
- Token scales: tokens whose x rows are scaled by powers of two from 2^-60 to 2^40, an all-zero row and rows mixing
  magnitudes 1e-4 to 1e3 meet the float32 bar per token relative to that token's largest output (the same bar the
  3xTF32 format meets on the same inputs).
- Weight row scales: neurons' up rows and outputs' down rows scaled by powers of two from 2^-12 to 2^12, all-zero
  rows among them: the same bar.
- The split entries: ``hffn_up_f16x3`` stores z (token-major) within the bar of the oracle's z, and up then down gives
  the bits of ``hffn_forward_f16x3``.
- After an optimiser step on the tensor cores (which refreshes the tf32 pairs in place), the next fp16x3 forward sees
  the new values.
- Token packets (``hffn_split_f16x3``, ``hffn_forward_f16x3_packets``): packets split in parts and concatenated give
  the forward's bits, and two neuron shards of one layer, each running on the packets the other split (the exchange
  of the sharded forward, emulated on one GPU), sum to the whole layer within the bar.
"""
import ctypes
import dataclasses

import numpy as np
import pytest
import torch

from hffn_b200 import synth
from oracle import forward64

pytestmark = pytest.mark.gpu

BAR = 1e-5


def kernel_layer(layer):
    from hffn_b200.runtime import HFFNLayer
    t = torch.from_numpy
    return HFFNLayer.from_hidden_major(layer.d_model, layer.d_ff, t(layer.b_up), t(layer.up_offsets), t(layer.up_idx),
                                       t(layer.up_val), t(layer.b_down), t(layer.down_offsets), t(layer.down_idx),
                                       t(layer.down_val))


def runtime_of(layer, tc_format="f16x3"):
    from hffn_b200.runtime import HFFNRuntime
    runtime = HFFNRuntime([kernel_layer(layer)], "cuda", torch.float32, tensor_cores=True, tc_format=tc_format)
    runtime.force("tc", "tc")
    return runtime


def token_relative(y: np.ndarray, expected: np.ndarray) -> float:
    """max over tokens of max_j |y - expected| / max(1, max_j |expected|) (the float32 bar per token)."""
    scale = np.maximum(1.0, np.abs(expected).max(axis=1, keepdims=True))
    return float((np.abs(y - expected) / scale).max())


def test_operands_reconstruct_the_weights():
    case = synth.TEST_CASES["irreg_512_2048"]
    layer = synth.make_layer(case)
    runtime = runtime_of(layer)
    runtime.forward_operands(0)
    dense = runtime._dense16[0]
    kl = runtime.layers[0]
    for side, rows, cols, offsets, idx, val in (
            ("up", case.d_ff, case.d_model, kl.up_offsets, kl.up_idx, kl.up_val),
            ("down", case.d_model, case.d_ff, kl.out_offsets, kl.out_hidden, kl.out_val)):
        w = torch.zeros(rows, cols, dtype=torch.float64)
        owner = torch.repeat_interleave(torch.arange(rows), offsets.diff().long())
        w[owner, idx.long()] = val.double()
        hi, lo = dense[f"{side}_hi"].double().cpu(), dense[f"{side}_lo"].double().cpu()
        scale = dense[f"{side}_scale"].double().cpu()[:, None]
        row_max = w.abs().max(dim=1, keepdim=True).values
        assert float(((hi + lo) * scale - w).abs().div(row_max.clamp_min(1e-300)).max()) <= 2.0 ** -22, side
        scaled_max = (hi.abs().max(dim=1).values)[row_max[:, 0] > 0]
        assert bool(((scaled_max >= 2.0 ** 14) & (scaled_max <= 2.0 ** 15)).all()), side
    l1 = torch.zeros(case.d_ff, dtype=torch.float64).index_add_(
        0, torch.repeat_interleave(torch.arange(case.d_ff), kl.up_offsets.diff().long()), kl.up_val.double().abs())
    bound = dense["up_bound"].double().cpu()
    assert abs(float(bound[0]) - float(l1.max())) <= 1e-5 * float(l1.max())
    assert float(bound[1]) == float(kl.b_up.abs().max())


def scaled_tokens(case, n) -> np.ndarray:
    x = synth.make_input(case, n).astype(np.float64)
    powers = [-60, -30, -10, 0, 10, 30, 40]
    for t in range(n):
        x[t] *= 2.0 ** powers[t % len(powers)]
    x[3] = 0.0
    rng = np.random.default_rng(11)
    for t in (5, 9):
        x[t] *= 10.0 ** rng.uniform(-4, 3, size=case.d_model)
    return x.astype(np.float32)


@pytest.mark.parametrize("tc_format", ["f16x3", "tf32x3"])
def test_token_scales(tc_format):
    case = synth.TEST_CASES["irreg_512_2048"]
    layer = synth.make_layer(case)
    runtime = runtime_of(layer, tc_format)
    x = scaled_tokens(case, 300)
    y = runtime.forward(0, torch.from_numpy(x).cuda()).double().cpu().numpy()
    expected = forward64.forward(layer, x)
    assert np.isfinite(y).all()
    assert token_relative(y, expected) <= BAR, (tc_format, token_relative(y, expected))
    assert runtime.device_errors() == 0


def scaled_rows(layer):
    """Up rows (neurons) scaled by 2^k, k cycling over -12 .. 12, neuron 7 all zero; down rows (outputs) likewise,
    output 4 all zero."""
    powers = np.arange(-12, 13, 3)
    up_val = layer.up_val.astype(np.float64).copy()
    for r in range(layer.d_ff):
        lo, hi = layer.up_offsets[r], layer.up_offsets[r + 1]
        up_val[lo:hi] *= 0.0 if r == 7 else 2.0 ** powers[r % len(powers)]
    down_scale = np.array([0.0 if o == 4 else 2.0 ** powers[(o * 5) % len(powers)] for o in range(layer.d_model)])
    down_val = layer.down_val.astype(np.float64) * down_scale[layer.down_idx.astype(np.int64)]
    return dataclasses.replace(layer, up_val=up_val.astype(np.float32), down_val=down_val.astype(np.float32))


@pytest.mark.parametrize("tc_format", ["f16x3", "tf32x3"])
def test_weight_row_scales(tc_format):
    case = synth.TEST_CASES["homog_512_2048"]
    layer = scaled_rows(synth.make_layer(case))
    runtime = runtime_of(layer, tc_format)
    x = synth.make_input(case, 257)
    y = runtime.forward(0, torch.from_numpy(x).cuda()).double().cpu().numpy()
    expected = forward64.forward(layer, x)
    assert token_relative(y, expected) <= BAR, (tc_format, token_relative(y, expected))
    assert runtime.device_errors() == 0


def test_split_entries_and_z():
    from hffn_b200 import _native as native
    case = synth.TEST_CASES["irreg_512_2048"]
    layer = synth.make_layer(case)
    runtime = runtime_of(layer)
    n = 333
    x_np = synth.make_input(case, n)
    x = torch.from_numpy(x_np).cuda()
    y_whole = runtime.forward(0, x).clone()
    _, dense = runtime.forward_operands(0)
    struct = runtime._structs[0]
    work = torch.empty(int(native.lib.hffn_forward_f16x3_workspace(struct, n)), dtype=torch.uint8, device="cuda")
    z = torch.empty(n, case.d_ff, device="cuda")
    y = torch.empty(n, case.d_model, device="cuda")
    err = torch.zeros(1, dtype=torch.int32, device="cuda")
    stream = native.stream_handle(runtime.device)
    native.check(native.lib.hffn_up_f16x3(x.data_ptr(), ctypes.byref(dense), struct.b_up, z.data_ptr(),
                                          work.data_ptr(), err.data_ptr(), case.d_model, case.d_ff, n, stream),
                 "hffn_up_f16x3")
    native.check(native.lib.hffn_down_f16x3(work.data_ptr(), ctypes.byref(dense), struct.b_down, y.data_ptr(),
                                            err.data_ptr(), case.d_model, case.d_ff, n, stream), "hffn_down_f16x3")
    assert torch.equal(y, y_whole)
    z64 = forward64.hidden(layer, x_np)
    gap = np.abs(z.double().cpu().numpy() - z64)
    assert float((gap / np.maximum(1.0, np.abs(z64))).max()) <= BAR
    assert int(err.item()) == 0


def test_forward_follows_tensor_core_training_steps():
    from hffn_b200.train_runtime import HFFNTrainRuntime
    case = synth.TEST_CASES["homog_256_1024"]
    layer = synth.make_layer(case)
    runtime = runtime_of(layer)
    train = HFFNTrainRuntime(runtime, lr=1e-2, tensor_cores=True)
    n = 300
    x = torch.from_numpy(synth.make_input(case, n)).cuda()
    target = torch.from_numpy(synth.make_input(case, n)).cuda()
    before = runtime.forward(0, x).clone()
    train.step_mse_tc(0, x, target)
    after = runtime.forward(0, x).clone()
    runtime.force("tile", "blocked")
    cuda_cores = runtime.forward(0, x).clone()
    assert not torch.equal(before, after)
    assert float((after - cuda_cores).abs().max()) <= 2e-5
    assert runtime.device_errors() == 0


def test_packets_concatenate_and_match_the_forward():
    """Packets split in two token halves and concatenated give the bits of the forward from x (tokens are
    independent), through ``forward_packets`` (the entry the neuron-sharded forward calls on gathered packets)."""
    case = synth.TEST_CASES["irreg_512_2048"]
    layer = synth.make_layer(case)
    runtime = runtime_of(layer)
    n = 600
    x = torch.from_numpy(synth.make_input(case, n)).cuda()
    y = runtime.forward(0, x).clone()
    packets = torch.empty(n, runtime.packet_bytes(), dtype=torch.uint8, device="cuda")
    runtime.split_packets(0, x[:250].contiguous(), packets[:250])
    runtime.split_packets(0, x[250:].contiguous(), packets[250:])
    out = torch.empty(n, case.d_model, device="cuda")
    runtime.forward_packets(0, packets, out)
    assert torch.equal(out, y)
    assert runtime.packet_bytes() == 4 * ((case.d_model + 31) // 32 * 32) + 64
    assert runtime.device_errors() == 0


def test_neuron_shards_read_each_others_packets():
    """Two neuron shards of one layer on one GPU, each with the whole layer's up bound (as ``sharded_runtime`` sets
    it): every shard runs on the packets the other shard split, and the sum of the partial outputs meets the float32
    bar against the oracle of the whole layer (the exchange of the two-GPU sharded forward, emulated)."""
    from hffn_b200.distributed import neuron_partition, shard_hidden_major
    from hffn_b200.runtime import HFFNLayer, HFFNRuntime
    case = synth.TEST_CASES["irreg_512_2048"]
    layer = synth.make_layer(case)
    arrays = {k: torch.from_numpy(getattr(layer, k)) for k in ("b_up", "up_offsets", "up_idx", "up_val", "b_down",
                                                                 "down_offsets", "down_idx", "down_val")}
    bounds = neuron_partition(arrays, 2)
    l1 = np.add.reduceat(np.abs(layer.up_val.astype(np.float64)), layer.up_offsets[:-1])
    floor = torch.tensor([l1.max(), np.abs(layer.b_up).max()], dtype=torch.float32)
    shards = []
    for rank in range(2):
        s = shard_hidden_major(case.d_model, arrays, bounds[rank], bounds[rank + 1], with_bias=rank == 0)
        kl = HFFNLayer.from_hidden_major(s["d_model"], s["d_ff"], s["b_up"], s["up_offsets"], s["up_idx"],
                                         s["up_val"], s["b_down"], s["down_offsets"], s["down_idx"], s["down_val"])
        rt = HFFNRuntime([kl], "cuda", torch.float32, tensor_cores=True)
        rt.force("tc", "tc")
        rt.up_bound_floor = floor
        shards.append(rt)
    n = 300
    x_np = synth.make_input(case, n)
    x = torch.from_numpy(x_np).cuda()
    packets = [torch.empty(n, shards[0].packet_bytes(), dtype=torch.uint8, device="cuda") for _ in range(2)]
    for rank in range(2):
        shards[rank].split_packets(0, x, packets[rank])
    partial = [torch.empty(n, case.d_model, device="cuda") for _ in range(2)]
    for rank in range(2):
        shards[rank].forward_packets(0, packets[1 - rank], partial[rank])
    y = (partial[0] + partial[1]).double().cpu().numpy()
    expected = forward64.forward(layer, x_np)
    assert token_relative(y, expected) <= BAR, token_relative(y, expected)
    assert all(rt.device_errors() == 0 for rt in shards)
