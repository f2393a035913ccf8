"""GPU: the forward entry that allocates nothing (hffn_forward_noalloc), through the C ABI.

It exists for callers that can pass the library only their input and output device buffers and cannot allocate
device memory themselves, for instance a plugin whose host framework owns all device memory. The entry keeps the
hidden activations in a fixed array inside the library, so the caller passes no workspace. Checked here against the
existing entry (hffn_forward with a caller-provided workspace) on two calls in a row, within the forward tolerance of
the other tests (float32; bf16 within the bf16 tolerance), at the largest token count the array admits (computed from
the entry's own limit, so the last row of the array stays covered if the limit changes), and the size limit is
refused before any launch in both storage types. This file is collected last on purpose.
"""
import numpy as np
import pytest
import torch

from hffn_b200 import synth

pytestmark = pytest.mark.gpu

ABS_TOLERANCE = 2e-5
REL_TOLERANCE = 1e-5
BF16_REL_TOLERANCE = 2e-2
ELEMENT = {torch.float32: 4, torch.bfloat16: 2}


def kernel_layer(layer):
    from hffn_b200.runtime import HFFNLayer
    t = torch.from_numpy
    return HFFNLayer.from_hidden_major(layer.d_model, layer.d_ff, t(layer.b_up), t(layer.up_offsets), t(layer.up_idx),
                                       t(layer.up_val), t(layer.b_down), t(layer.down_offsets), t(layer.down_idx),
                                       t(layer.down_val))


def largest_n(case, dtype) -> int:
    from hffn_b200 import _native as native
    return int(native.lib.hffn_forward_noalloc_max_bytes()) // (ELEMENT[dtype] * case.d_ff)


def compare_two_calls(name, n, dtype):
    from hffn_b200 import _native as native
    from hffn_b200.runtime import DTYPES, HFFNRuntime
    case = synth.CASES[name]
    runtime = HFFNRuntime([kernel_layer(synth.make_layer(case))], "cuda", dtype, tensor_cores=False)
    n = largest_n(case, dtype) if n is None else n
    x = torch.from_numpy(synth.make_input(case, n)).to(dtype).cuda()
    expected = runtime.forward(0, x).double().clone()      # hffn_forward, caller-provided act workspace
    stream = native.stream_handle(runtime.device)
    scale = expected.abs().clamp(min=1.0)
    for _ in range(2):
        y = torch.full((n, case.d_model), float("nan"), device="cuda", dtype=dtype)
        status = native.lib.hffn_forward_noalloc(DTYPES[dtype], runtime._structs[0], x.data_ptr(), y.data_ptr(), n,
                                                 stream)
        native.check(status, "hffn_forward_noalloc")
        torch.cuda.synchronize()
        distance = (y.double() - expected).abs()
        if dtype == torch.float32:
            assert float(distance.max()) <= ABS_TOLERANCE
            assert float((distance / scale).max()) <= REL_TOLERANCE
        else:
            assert float((distance / scale).max()) <= BF16_REL_TOLERANCE


@pytest.mark.parametrize("name,n", [("irreg_512_2048", 300), ("c2_1024_4096_k512", None), ("homog_256_1024", 3)])
def test_noalloc_matches_forward_on_two_calls(name, n):
    compare_two_calls(name, n, torch.float32)


@pytest.mark.parametrize("name,n", [("homog_256_1024", 3), ("irreg_512_2048", 300), ("c2_1024_4096_k512", None)])
def test_noalloc_bf16_matches_forward_on_two_calls(name, n):
    compare_two_calls(name, n, torch.bfloat16)


@pytest.mark.parametrize("dtype", [torch.float32, torch.bfloat16])
def test_noalloc_refuses_beyond_its_scratch(dtype):
    from hffn_b200 import _native as native
    from hffn_b200.runtime import DTYPES, HFFNRuntime
    case = synth.CONFIGS["c2_1024_4096_k512"]
    runtime = HFFNRuntime([kernel_layer(synth.make_layer(case))], "cuda", dtype, tensor_cores=False)
    n_max = largest_n(case, dtype)
    x = torch.zeros(n_max + 1, case.d_model, device="cuda", dtype=dtype)
    y = torch.zeros_like(x)
    status = native.lib.hffn_forward_noalloc(DTYPES[dtype], runtime._structs[0], x.data_ptr(), y.data_ptr(),
                                             n_max + 1, native.stream_handle(runtime.device))
    assert status == native.HFFN_ERR_ARGUMENT
    assert b"scratch" in native.lib.hffn_last_error()
    assert np.all(y.float().cpu().numpy() == 0)
