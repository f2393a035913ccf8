"""Device-side layout build: the output-major down edges and the transposed supports of a layer computed on the GPU by
stable counting sorts (``hffn_build_out_major``, ``hffn_build_supports`` of ``libhffn_b200.so``), equal bit for bit
to the host stable sorts of ``HFFNLayer.from_hidden_major`` (``runtime/gpu/nvidia/common/kernels/hffn_cuda/
runtime.py:55-67``) and ``transposed_supports`` (``runtime/gpu/nvidia/ffn/training/train_runtime.py:39-56``).

``HFFNLayer.from_hidden_major`` and ``transposed_supports`` take this path when their arrays are CUDA tensors, so a
model loaded onto a GPU needs no host argsort. Each call allocates its outputs and a workspace with torch and
synchronises once (the check of the layout flag: an offset or an index out of range raises ``ValueError``).
"""
from __future__ import annotations

import torch

from . import _native as native

DTYPES = {torch.float32: native.F32, torch.bfloat16: native.BF16}


def _workspace(d_model: int, d_ff: int, nnz_up: int, nnz_down: int, device) -> torch.Tensor:
    size = int(native.lib.hffn_build_layout_workspace(d_model, d_ff, nnz_up, nnz_down))
    if size < 0:
        raise ValueError("invalid layer dimensions")
    return torch.empty(max(size, 1), dtype=torch.uint8, device=device)


def _check(flag: torch.Tensor, what: str) -> None:
    if int(flag.item()):
        raise ValueError(f"{what}: an offset or an index of the layer is out of range")


def out_major(d_model: int, d_ff: int, down_offsets: torch.Tensor, down_idx: torch.Tensor,
              down_val: torch.Tensor) -> tuple[torch.Tensor, torch.Tensor, torch.Tensor]:
    """(out_offsets int32 [d_model + 1], out_hidden int16 [nnz], out_val [nnz]) on the arrays' device."""
    device = down_idx.device
    if down_val.dtype not in DTYPES:
        raise ValueError("down_val must be float32 or bfloat16")
    down_offsets = down_offsets.to(device, torch.int32).contiguous()
    down_idx = down_idx.to(device, torch.int16).contiguous()
    down_val = down_val.to(device).contiguous()
    nnz = down_idx.numel()
    out_offsets = torch.empty(d_model + 1, dtype=torch.int32, device=device)
    out_hidden = torch.empty(nnz, dtype=torch.int16, device=device)
    out_val = torch.empty(nnz, dtype=down_val.dtype, device=device)
    flag = torch.empty(1, dtype=torch.int32, device=device)
    work = _workspace(d_model, d_ff, 0, nnz, device)
    native.check(native.lib.hffn_build_out_major(DTYPES[down_val.dtype], d_model, d_ff, down_offsets.data_ptr(),
                                                 down_idx.data_ptr(), down_val.data_ptr(), nnz, out_offsets.data_ptr(),
                                                 out_hidden.data_ptr(), out_val.data_ptr(), work.data_ptr(),
                                                 flag.data_ptr(), native.stream_handle(device)), "hffn_build_out_major")
    _check(flag, "hffn_build_out_major")
    return out_offsets, out_hidden, out_val


def supports(d_model: int, d_ff: int, up_offsets: torch.Tensor, up_idx: torch.Tensor, out_offsets: torch.Tensor,
             out_hidden: torch.Tensor) -> dict[str, torch.Tensor]:
    """The six transposed-support arrays (``SUPPORTS`` of the training runtime) on the arrays' device."""
    device = out_hidden.device
    up_offsets = up_offsets.to(device, torch.int32).contiguous()
    up_idx = up_idx.to(device, torch.int16).contiguous()
    out_offsets = out_offsets.to(device, torch.int32).contiguous()
    out_hidden = out_hidden.to(device, torch.int16).contiguous()
    nnz_up, nnz_down = up_idx.numel(), out_hidden.numel()
    i32 = lambda n: torch.empty(n, dtype=torch.int32, device=device)  # noqa: E731
    i16 = lambda n: torch.empty(n, dtype=torch.int16, device=device)  # noqa: E731
    out = {"in_offsets": i32(d_model + 1), "in_pos": i32(nnz_up), "in_hidden": i16(nnz_up),
           "hid_offsets": i32(d_ff + 1), "hid_pos": i32(nnz_down), "hid_output": i16(nnz_down)}
    flag = torch.empty(1, dtype=torch.int32, device=device)
    work = _workspace(d_model, d_ff, nnz_up, nnz_down, device)
    native.check(native.lib.hffn_build_supports(d_model, d_ff, up_offsets.data_ptr(), up_idx.data_ptr(), nnz_up,
                                                out_offsets.data_ptr(), out_hidden.data_ptr(), nnz_down,
                                                *(out[k].data_ptr() for k in ("in_offsets", "in_pos", "in_hidden",
                                                                              "hid_offsets", "hid_pos", "hid_output")),
                                                work.data_ptr(), flag.data_ptr(), native.stream_handle(device)),
                 "hffn_build_supports")
    _check(flag, "hffn_build_supports")
    return out
