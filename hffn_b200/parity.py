"""Parity of the runtime on one FFN against a float64 expectation, under every kernel pair the runtime offers.

Drop-in names of the reference's ``runtime/gpu/nvidia/common/kernels/hffn_cuda/parity.py``: ``PAIRS`` (the policy,
then the nine forced (up, down) pairs), ``Parity`` (its four summary fields) and ``check(runtime, index, x,
expected)``. The body is this repository's: every pair is measured into a table row, and the summary is folded from
the table, so a caller also learns which pair was worst (the tensor-core pair ("tc", "tc"), added when the runtime
holds dense operands, is the one most likely to be).

Per pair: two calls on the same input (same bits required), the largest absolute distance to the float64 output and
the largest distance relative to ``max(1, |y_float64|)``. Reported without a threshold: whether the four pairs of the
tiled kernels (up lane / tile x down tiled / blocked) agree bit for bit, which holds here because they share one
summation order.
"""
from __future__ import annotations

from dataclasses import dataclass, field

import torch

from .runtime import DOWN_MODES, TC, UP_MODES, HFFNRuntime

PAIRS = [(None, None)] + [(up, down) for up in UP_MODES for down in DOWN_MODES]
TILED_UP, TILED_DOWN = ("lane", "tile"), ("tiled", "blocked")


@dataclass
class PairResult:
    error: float        # largest |y - y_float64|
    relative: float     # largest |y - y_float64| / max(1, |y_float64|)
    repeatable: bool    # the second call gave the bits of the first


@dataclass
class Parity:
    error: float
    relative: float
    repeatable: bool
    sequential_bits: bool
    pairs: dict = field(default_factory=dict)    # (up, down) -> PairResult
    worst: tuple | None = None                   # the pair with the largest relative distance


def _measure(runtime: HFFNRuntime, index: int, x: torch.Tensor, expected: torch.Tensor,
             scale: torch.Tensor) -> tuple[PairResult, torch.Tensor]:
    first = runtime.forward(index, x).clone()
    again = runtime.forward(index, x)
    gap = (first.double() - expected).abs()
    return PairResult(float(gap.max()), float((gap / scale).max()), bool(torch.equal(first, again))), first


def check(runtime: HFFNRuntime, index: int, x: torch.Tensor, expected: torch.Tensor) -> Parity:
    """``x`` [N, d_model] on the runtime's device, ``expected`` its float64 output (any device). The runtime's
    forcing is cleared on return."""
    expected = expected.to(device=x.device, dtype=torch.float64)
    scale = expected.abs().clamp(min=1.0)
    candidates = list(PAIRS)
    if getattr(runtime, "tensor_cores", False):
        candidates.append((TC, TC))
    table: dict = {}
    tiled_outputs = []
    try:
        for pair in candidates:
            runtime.force(*pair)
            table[pair], y = _measure(runtime, index, x, expected, scale)
            if pair[0] in TILED_UP and pair[1] in TILED_DOWN:
                tiled_outputs.append(y)
    finally:
        runtime.force(None, None)
    worst = max(table, key=lambda pair: table[pair].relative)
    same_tiled = all(torch.equal(y, tiled_outputs[0]) for y in tiled_outputs[1:])
    return Parity(error=max(r.error for r in table.values()), relative=table[worst].relative,
                  repeatable=all(r.repeatable for r in table.values()), sequential_bits=same_tiled,
                  pairs=table, worst=worst)
