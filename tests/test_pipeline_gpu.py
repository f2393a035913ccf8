"""GPU: the host pipeline (host batches in, host outputs back, copies overlapped with the kernels) gives, batch by
batch, the bits of a plain device call, for ragged batch sizes, both forward paths and several pipeline depths."""
import pytest
import torch

from hffn_b200 import synth
from hffn_b200.pipeline import HostPipeline, runtime_forward

pytestmark = pytest.mark.gpu


def runtime_for(layer, dtype, tensor_cores):
    from hffn_b200.runtime import HFFNLayer, HFFNRuntime
    t = torch.from_numpy
    kl = HFFNLayer.from_hidden_major(layer.d_model, layer.d_ff, t(layer.b_up), t(layer.up_offsets), t(layer.up_idx),
                                     t(layer.up_val), t(layer.b_down), t(layer.down_offsets), t(layer.down_idx),
                                     t(layer.down_val))
    return HFFNRuntime([kl], "cuda", dtype, tensor_cores=tensor_cores)


@pytest.mark.parametrize("depth", [1, 2, 3])
@pytest.mark.parametrize("dtype,tensor_cores", [(torch.float32, True), (torch.bfloat16, True), (torch.float32, False)])
def test_pipeline_matches_plain_calls(depth, dtype, tensor_cores):
    case = synth.TEST_CASES["irreg_512_2048"]
    runtime = runtime_for(synth.make_layer(case), dtype, tensor_cores)
    sizes = [300, 7, 1024, 300, 513, 1, 700]
    xs = [torch.from_numpy(synth.make_input(case, n + k)[:n]).to(dtype).pin_memory() for k, n in enumerate(sizes)]
    ys = [torch.empty(n, case.d_model, dtype=dtype).pin_memory() for n in sizes]
    pipe = HostPipeline(runtime_forward(runtime, 0), case.d_model, case.d_model, max(sizes), dtype, "cuda", depth)
    for _ in range(2):                                          # a second run reuses the buffers and events
        for y in ys:
            y.zero_()
        pipe.run(xs, ys)
        for x, y in zip(xs, ys):
            assert torch.equal(y, runtime.forward(0, x.cuda()).cpu())
    assert runtime.device_errors() == 0


def test_pipeline_rejects_bad_batches():
    case = synth.TEST_CASES["homog_256_1024"]
    runtime = runtime_for(synth.make_layer(case), torch.float32, True)
    pipe = HostPipeline(runtime_forward(runtime, 0), 256, 256, 64, torch.float32, "cuda")
    good_x, good_y = torch.zeros(8, 256).pin_memory(), torch.zeros(8, 256).pin_memory()
    with pytest.raises(ValueError):
        pipe.run([torch.zeros(8, 256)], [good_y])                # not pinned
    with pytest.raises(ValueError):
        pipe.run([torch.zeros(65, 256).pin_memory()], [torch.zeros(65, 256).pin_memory()])   # above max_tokens
    with pytest.raises(ValueError):
        pipe.run([good_x], [torch.zeros(8, 255).pin_memory()])   # output shape
    with pytest.raises(ValueError):
        pipe.run([good_x], [])
