"""TEST INFRASTRUCTURE ONLY. The reference's own CPU training step of one FFN layer (the G4 ``Step``), driven as its
Python driver drives it.

Libraries (built by ``oracle/Makefile`` from the reference sources, with the reference's flags, into ``oracle/_ref``):
the x86 inference kernel (forward, dual route with z stored: ``hffn_compact_forward_dual_slots_nt_f32``) and the G4
training kernel (``hffn_compact_g4_backward_dual_nt_f32``, ``hffn_compact_g4_adamw_f32``). This module follows
``runtime/cpu/common/ffn/training/hffn_ffn_training/step.py:66-157`` (``Step``: buffers reserved once for N tokens,
forward with the G4 hidden partition and 4 workers, the dual backward from ``DUAL_MIN_N`` = 32 tokens, AdamW with the
step counter) and ``layer.py:18-38`` (the reverse schedules: features' slots by a stable sort, the owner of each slot,
four groups balanced by slot count). The G4 kernel's worker count is fixed at 4 (``g4_contract.h:3``).

Used as the timed CPU baseline of the training workload in ``bench.py`` and cross-checked against ``train64`` in
``tests/test_oracle_golden.py``. The MSE loss gradient of the training benchmark, ``gy = 2 (y - target) / (N d)``,
is computed here in numpy between the forward and the backward (the reference's step takes gy from its caller).
"""
from __future__ import annotations

import ctypes
from pathlib import Path

import numpy as np

from .x86ref import aligned_empty

HERE = Path(__file__).resolve().parent
INFERENCE_LIB = HERE / "_ref" / "libhffn_x86_inference.so"
TRAINING_LIB = HERE / "_ref" / "libhffn_g4_training.so"
GROUPS = 4
DUAL_MIN_N = 32


def available() -> bool:
    return INFERENCE_LIB.exists() and TRAINING_LIB.exists()


def balanced_groups(cost: np.ndarray, groups: int = GROUPS) -> np.ndarray:
    """Cut the features into ``groups`` contiguous ranges of about equal slot count (layer.py:18-29)."""
    total, bounds, cumulative, target = int(cost.sum()), [0], 0, 1
    for feature, value in enumerate(cost.tolist()):
        cumulative += int(value)
        while target < groups and cumulative >= round(total * target / groups):
            bounds.append(feature + 1)
            target += 1
    while len(bounds) < groups:
        bounds.append(bounds[-1])
    bounds.append(cost.size)
    return np.array(bounds, dtype=np.int32)


def reverse_schedule(offsets: np.ndarray, index: np.ndarray, d_ff: int, d_model: int):
    """Per feature: the offsets of its slots, the slots (stable order), their owning neurons, the balanced groups."""
    count = np.bincount(index.astype(np.int64), minlength=d_model)
    by_feature = np.zeros(d_model + 1, np.int32)
    by_feature[1:] = np.cumsum(count)
    slots = np.argsort(index.astype(np.int64), kind="stable")
    owner = np.repeat(np.arange(d_ff), np.diff(offsets))
    return (by_feature, np.ascontiguousarray(slots.astype(np.int32)),
            np.ascontiguousarray(owner[slots].astype(np.int16)), balanced_groups(count))


def _aligned_copy(array: np.ndarray) -> np.ndarray:
    """A copy of ``array`` (flattened) on a 64-byte boundary, as the reference's work buffers are."""
    raw = np.empty(array.nbytes + 64, np.uint8)
    start = -raw.ctypes.data % 64
    out = raw[start:start + array.nbytes].view(array.dtype)
    out[:] = array.ravel()
    return out


class G4Step:
    """One FFN layer's training step on the host: forward (z stored), MSE gradient, backward, AdamW, for N tokens."""

    def __init__(self, layer, n: int, lr: float = 1e-3, betas: tuple[float, float] = (0.9, 0.999), eps: float = 1e-8,
                 weight_decay: float = 1e-2) -> None:
        if not available():
            raise FileNotFoundError("oracle/_ref kernels missing: run `make -C oracle` where the reference exists")
        if n < DUAL_MIN_N:
            raise ValueError(f"the host step is driven on the dual route, N >= {DUAL_MIN_N}")
        self.n, self.d, self.f = n, layer.d_model, layer.d_ff
        self.lr, self.betas, self.eps, self.weight_decay = lr, betas, eps, weight_decay
        p, i, fl, l64 = ctypes.c_void_p, ctypes.c_int, ctypes.c_float, ctypes.c_int64
        inference, training = ctypes.CDLL(str(INFERENCE_LIB)), ctypes.CDLL(str(TRAINING_LIB))
        self._forward = inference.hffn_compact_forward_dual_slots_nt_f32
        self._forward.argtypes, self._forward.restype = [i] + [p] * 12 + [i] * 3 + [p] * 6, None
        self._backward = training.hffn_compact_g4_backward_dual_nt_f32
        self._backward.argtypes, self._backward.restype = [p] * 15 + [i] * 3 + [p] * 9, None
        self._adamw = training.hffn_compact_g4_adamw_f32
        self._adamw.argtypes, self._adamw.restype = ([p] * 4 + [i]) * 4 + [fl] * 5 + [l64], None
        a = _aligned_copy
        self.groups = a(np.asarray(layer.groups, np.int32))
        self.up_offsets, self.up_idx = a(layer.up_offsets.astype(np.int32)), a(layer.up_idx.astype(np.int16))
        self.down_offsets, self.down_idx = a(layer.down_offsets.astype(np.int32)), a(layer.down_idx.astype(np.int16))
        self.up_val, self.b_up = a(layer.up_val.astype(np.float32)), a(layer.b_up.astype(np.float32))
        self.down_val, self.b_down = a(layer.down_val.astype(np.float32)), a(layer.b_down.astype(np.float32))
        down = reverse_schedule(layer.down_offsets, layer.down_idx, self.f, self.d)
        up = reverse_schedule(layer.up_offsets, layer.up_idx, self.f, self.d)
        self.down_by_output, self.down_slots, self.down_hidden, self.output_groups = (a(t) for t in down)
        self.up_by_input, self.up_slots, self.up_hidden, self.input_groups = (a(t) for t in up)
        empty = aligned_empty
        d, f = self.d, self.f
        self.x_t, self.y_t, self.y_nt = empty(d * n), empty(d * n), empty(d * n)
        self.z, self.act, self.gz = empty(f * n), empty(f * n), empty(f * n)
        self.gy_nt, self.gy_t, self.gx_nt, self.gx_t = empty(d * n), empty(d * n), empty(d * n), empty(d * n)
        e_up, e_down = self.up_val.size, self.down_val.size
        self.g_up, self.g_down, self.g_b_up, self.g_b_down = empty(e_up), empty(e_down), empty(f), empty(d)
        self.moments = [empty(e_up), empty(e_up), empty(e_down), empty(e_down), empty(f), empty(f), empty(d), empty(d)]
        for m in self.moments:
            m[:] = 0.0
        self.timing = np.zeros(8, np.int64)
        self.steps = 0

    def forward(self, x: np.ndarray) -> np.ndarray:
        """y [N, d_model] (a view of the step's buffer) for C-contiguous float32 x [N, d_model]; z and act stored."""
        x = np.ascontiguousarray(x, np.float32)
        if x.shape != (self.n, self.d):
            raise ValueError("x must be [N, d_model] for the step's N")
        c = lambda array: array.ctypes.data  # noqa: E731
        self._forward(GROUPS, c(x), c(self.groups), c(self.b_up), c(self.up_offsets), c(self.up_idx), c(self.up_val),
                      c(self.b_down), c(self.down_by_output), c(self.down_hidden), c(self.down_val), c(self.down_slots),
                      c(self.output_groups), self.n, self.d, self.f, c(self.x_t), c(self.y_nt), c(self.y_t), c(self.z),
                      c(self.act), c(self.timing))
        return self.y_nt.reshape(self.n, self.d)

    def backward(self, gy: np.ndarray) -> None:
        self.gy_nt[:] = np.ascontiguousarray(gy, np.float32).ravel()
        c = lambda array: array.ctypes.data  # noqa: E731
        self._backward(c(self.gy_nt), c(self.x_t), c(self.z), c(self.act), c(self.groups), c(self.up_offsets),
                       c(self.up_idx), c(self.up_val), c(self.down_offsets), c(self.down_idx), c(self.down_val),
                       c(self.up_by_input), c(self.up_slots), c(self.up_hidden), c(self.input_groups), self.n, self.d,
                       self.f, c(self.gy_t), c(self.gx_nt), c(self.gx_t), c(self.gz), c(self.g_up), c(self.g_down),
                       c(self.g_b_up), c(self.g_b_down), self.timing[4:].ctypes.data)

    def update(self) -> None:
        c, m = (lambda array: array.ctypes.data), self.moments
        self.steps += 1
        self._adamw(c(self.up_val), c(self.g_up), c(m[0]), c(m[1]), self.up_val.size,
                    c(self.down_val), c(self.g_down), c(m[2]), c(m[3]), self.down_val.size,
                    c(self.b_up), c(self.g_b_up), c(m[4]), c(m[5]), self.f,
                    c(self.b_down), c(self.g_b_down), c(m[6]), c(m[7]), self.d,
                    self.lr, self.betas[0], self.betas[1], self.eps, self.weight_decay, self.steps)

    def step_mse(self, x: np.ndarray, target: np.ndarray) -> float:
        """Forward, loss ``mean((y - target)^2)`` and its gradient ``2 (y - target) / (N d)``, backward, AdamW.
        Returns the loss of the parameters before the update."""
        y = self.forward(x)
        diff = y - np.asarray(target, np.float32)
        loss = float(np.mean(np.square(diff, dtype=np.float64)))
        self.backward(diff * np.float32(2.0 / (self.n * self.d)))
        self.update()
        return loss

    def gradients(self) -> dict:
        """This step's gradients, hidden-major slot order (the canonical order of both value arrays)."""
        return {"g_up": self.g_up.copy(), "g_down": self.g_down.copy(), "gb_up": self.g_b_up.copy(),
                "gb_down": self.g_b_down.copy(), "gx": self.gx_nt.reshape(self.n, self.d).copy(),
                "gz": self.gz.reshape(self.f, self.n).copy()}
