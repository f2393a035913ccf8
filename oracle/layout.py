"""TEST INFRASTRUCTURE ONLY. Integer layouts of the kernel arrays, restated with numpy stable sorts.

- ``out_major`` restates ``HFFNLayer.from_hidden_major`` (``runtime/gpu/nvidia/common/kernels/hffn_cuda/runtime.py:55-67``):
  the down slots permuted to output-major order by a stable argsort of ``down_idx``; ``out_offsets`` by
  bincount + cumsum; ``out_hidden`` the owning neuron of each edge (int16).
- ``transposed_supports`` restates ``runtime/gpu/nvidia/ffn/training/train_runtime.py:39-56``: the up slots
  input-major (``in_offsets``, ``in_pos`` positions into ``up_*``, ``in_hidden``) and the output-major down edges
  hidden-major (``hid_offsets``, ``hid_pos`` positions into ``out_*``, ``hid_output``), both by stable sorts.
The product's layouts must equal these arrays bit for bit.
"""
from __future__ import annotations

import numpy as np


def _offsets(keys: np.ndarray, count: int) -> np.ndarray:
    offsets = np.zeros(count + 1, dtype=np.int32)
    offsets[1:] = np.cumsum(np.bincount(keys, minlength=count))
    return offsets


def out_major(d_model: int, d_ff: int, down_offsets, down_idx, down_val) -> dict:
    output = np.asarray(down_idx).astype(np.int64)
    order = np.argsort(output, kind="stable")
    hidden = np.repeat(np.arange(d_ff), np.diff(np.asarray(down_offsets)))
    return {"out_offsets": _offsets(output, d_model), "out_hidden": hidden[order].astype(np.int16),
            "out_val": np.asarray(down_val)[order], "perm": order.astype(np.int64)}


def transposed_supports(d_model: int, d_ff: int, up_offsets, up_idx, out_offsets, out_hidden) -> dict:
    up_idx = np.asarray(up_idx).astype(np.int64)
    out_hidden = np.asarray(out_hidden).astype(np.int64)
    up_hidden = np.repeat(np.arange(d_ff), np.diff(np.asarray(up_offsets)))
    by_input = np.argsort(up_idx, kind="stable")
    out_output = np.repeat(np.arange(d_model), np.diff(np.asarray(out_offsets)))
    by_hidden = np.argsort(out_hidden, kind="stable")
    return {"in_offsets": _offsets(up_idx, d_model), "in_pos": by_input.astype(np.int32),
            "in_hidden": up_hidden[by_input].astype(np.int16),
            "hid_offsets": _offsets(out_hidden, d_ff), "hid_pos": by_hidden.astype(np.int32),
            "hid_output": out_output[by_hidden].astype(np.int16)}
