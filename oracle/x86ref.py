"""TEST INFRASTRUCTURE ONLY. The reference's own x86 AVX2 inference kernel, driven as its ctypes loader drives it.

The library is the reference source ``runtime/cpu/x86/common/kernels/hffn_compact_g4_inference.cpp`` compiled with the
reference's flags by ``oracle/Makefile`` into ``oracle/_ref/libhffn_x86_inference.so``. This module follows
``runtime/cpu/x86/ffn/inference/hffn/compact.py:107-217`` (``CompactKernel``): the ``dual`` route for N >= 2 and the
``decode`` route for N = 1, batches above 96 tokens in balanced chunks that are multiples of 8
(``compact.py:63-69``), T threads each owning one group of hidden neurons (``hidden_partition``, ``compact.py:87-89``)
and one group of output features balanced by edge count (``dual_route``, ``compact.py:92-105``), work buffers on
64-byte boundaries (``compact.py:43-48``).

It serves two roles: a cross-check of ``forward64`` (float32 within 2e-5 of float64, the reference leaf's
tolerance) and the timed CPU baseline of ``bench.py``.
"""
from __future__ import annotations

import ctypes
import os
from pathlib import Path

import numpy as np

LIB = Path(__file__).resolve().parent / "_ref" / "libhffn_x86_inference.so"
MAX_BATCH = 96
WORK_ALIGNMENT = 64


def available() -> bool:
    return LIB.exists()


def aligned_empty(size: int) -> np.ndarray:
    raw = np.empty(size * 4 + WORK_ALIGNMENT, np.uint8)
    start = -raw.ctypes.data % WORK_ALIGNMENT
    return raw[start:start + size * 4].view(np.float32)


def batch_chunks(n: int, max_batch: int) -> list[tuple[int, int]]:
    if n <= max_batch:
        return [(0, n)]
    count = -(-n // max_batch)
    size = -(-(-(-n // count)) // 8) * 8
    return [(start, min(size, n - start)) for start in range(0, n, size)]


def _balanced(cost: np.ndarray, threads: int) -> np.ndarray:
    total, bounds, cumulative, target = int(cost.sum()), [0], 0, 1
    for feature, value in enumerate(cost.tolist()):
        cumulative += int(value)
        while target < threads and cumulative >= round(total * target / threads):
            bounds.append(feature + 1)
            target += 1
    while len(bounds) < threads:
        bounds.append(bounds[-1])
    bounds.append(cost.size)
    return np.array(bounds, dtype=np.int32)


class X86Kernel:
    """The reference kernel on one layer, ``threads`` host threads (default: the process affinity, at most 64)."""

    def __init__(self, layer, threads: int | None = None, max_batch: int = MAX_BATCH) -> None:
        if not LIB.exists():
            raise FileNotFoundError(f"{LIB} is missing: run `make -C oracle` where the reference sources exist")
        self._lib = ctypes.CDLL(str(LIB))
        self.threads = max(1, min(threads or len(os.sched_getaffinity(0)), 64))
        self.max_batch = max_batch
        self.layer = layer
        t = self.threads
        self._hidden_groups = np.array([(g * layer.d_ff) // t for g in range(t + 1)], dtype=np.int32)
        output = layer.down_idx.astype(np.int64)
        count = np.bincount(output, minlength=layer.d_model).astype(np.int32)
        self._out_offsets = np.zeros(layer.d_model + 1, np.int32)
        self._out_offsets[1:] = np.cumsum(count)
        order = np.argsort(output, kind="stable")
        self._out_hidden = np.ascontiguousarray(np.repeat(np.arange(layer.d_ff), np.diff(layer.down_offsets))[order].astype(np.int16))
        self._out_val = np.ascontiguousarray(layer.down_val[order])
        self._output_groups = _balanced(count, t)
        p, i = ctypes.c_void_p, ctypes.c_int
        self._dual = self._lib.hffn_compact_forward_dual_nt_f32
        self._dual.argtypes = [i] + [p] * 11 + [i, i, i] + [p] * 6
        self._dual.restype = None
        self._decode = self._lib.hffn_compact_forward_decode_nt_f32
        self._decode.argtypes = [i] + [p] * 11 + [i, i] + [p] * 3
        self._decode.restype = None
        self._work: dict[str, np.ndarray] = {}
        self._timing = np.zeros(4, np.int64)

    def _buffer(self, role: str, size: int) -> np.ndarray:
        if role not in self._work or self._work[role].size < size:
            self._work[role] = aligned_empty(size)
        return self._work[role]

    def forward(self, x: np.ndarray) -> np.ndarray:
        """``y[N, d_model]`` float32 for a C-contiguous float32 ``x[N, d_model]``."""
        layer, a = self.layer, (lambda array: array.ctypes.data)
        x = np.ascontiguousarray(x, dtype=np.float32)
        n = x.shape[0]
        y = np.empty_like(x)
        up = [a(self._hidden_groups), a(layer.b_up), a(layer.up_offsets), a(layer.up_idx), a(layer.up_val)]
        reverse = [a(layer.b_down), a(self._out_offsets), a(self._out_hidden), a(self._out_val), a(self._output_groups)]
        if n == 1:
            act = self._buffer("act", layer.d_ff)
            self._decode(self.threads, a(x), *up, *reverse, layer.d_model, layer.d_ff, a(y), a(act), a(self._timing))
            return y
        for start, size in batch_chunks(n, self.max_batch):
            x_t = self._buffer("x_t", layer.d_model * size)
            act = self._buffer("act", layer.d_ff * size)
            self._dual(self.threads, a(x) + start * x.strides[0], *up, *reverse, size, layer.d_model, layer.d_ff,
                       a(x_t), a(y) + start * y.strides[0], a(x_t), a(act), a(act), a(self._timing))
        return y
