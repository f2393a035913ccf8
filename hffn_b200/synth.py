"""Seeded synthetic HFFN layers in the canonical compact hidden-major layout, and their inputs.

The generator follows the reference's ``runtime/common/ffn/hffn_ffn_layers/synth.py:53-86``: numpy's PCG64 generator
(``np.random.default_rng(seed)``) draws, in this order, the up degrees and the down degrees (irregular cases only),
then per hidden neuron a sorted choice of ``degree`` distinct input features, the up values
``standard_normal * (1 / sqrt(nominal degree))`` as float32, the same for the down side, then ``b_up`` and ``b_down``.
The draw order is what the reference's pinned SHA-256 fingerprints fix (``runtime/common/ffn/reference/
fingerprints.json``), so it is kept as it is; the tests check the fingerprints of the three reference test layers.

Inputs: ``np.random.default_rng([seed, n]).standard_normal((n, d_model))`` as float32, token-major
(``synth.py:83-86``).

Besides the three reference test layers, ``CONFIGS`` holds the five benchmark shapes of this build (d_model, d_ff,
per-neuron support size, seed). They use the same draw order with a bias standard deviation of 0.02.
"""
from __future__ import annotations

from dataclasses import dataclass

import numpy as np

N_GROUPS = 4


@dataclass(frozen=True)
class Case:
    name: str
    d_model: int
    d_ff: int
    up_degree: int
    down_degree: int
    irregular: bool
    seed: int
    bias_std: float = 0.1     # the reference test layers use 0.1 (synth.py:80-81)


@dataclass(frozen=True)
class CompactLayer:
    """Canonical hidden-major storage: neuron r owns up slots and down slots ``[offsets[r], offsets[r + 1])``."""
    d_model: int
    d_ff: int
    groups: np.ndarray        # int32[5], hidden partition of the four CPU groups (kept for the fingerprint)
    up_offsets: np.ndarray    # int32[d_ff + 1]
    up_idx: np.ndarray        # int16[nnz_up], input feature of each slot
    up_val: np.ndarray        # float32[nnz_up]
    b_up: np.ndarray          # float32[d_ff]
    down_offsets: np.ndarray  # int32[d_ff + 1]
    down_idx: np.ndarray      # int16[nnz_down], output feature of each slot
    down_val: np.ndarray      # float32[nnz_down]
    b_down: np.ndarray        # float32[d_model]


# The reference's three fingerprinted test layers (synth.py:28-35).
TEST_CASES = {
    case.name: case
    for case in (
        Case("homog_256_1024", 256, 1024, 26, 26, False, 1001),
        Case("homog_512_2048", 512, 2048, 51, 51, False, 1002),
        Case("irreg_512_2048", 512, 2048, 51, 51, True, 1003),
    )
}

# The benchmark shapes: C1 fp32 forward, C2 Pythia-410M FFN shape, C3 training step, C4 / C5 the FFNs of the
# Pythia-410M and Pythia-1B shapes (one layer each; a model draws layer l with seed + 100 * l).
CONFIGS = {
    case.name: case
    for case in (
        Case("c1_512_2048_k128", 512, 2048, 128, 128, False, 3001, 0.02),
        Case("c2_1024_4096_k512", 1024, 4096, 512, 512, False, 3002, 0.02),
        Case("c3_2048_8192_k1638", 2048, 8192, 1638, 1638, False, 3003, 0.02),
        Case("c4_1024_4096_k512", 1024, 4096, 512, 512, False, 3004, 0.02),
        Case("c5_2048_8192_k410", 2048, 8192, 410, 410, False, 3005, 0.02),
    )
}

CASES = {**TEST_CASES, **CONFIGS}


def _degrees(rng: np.random.Generator, d_ff: int, degree: int, d_model: int, irregular: bool) -> np.ndarray:
    if not irregular:
        return np.full(d_ff, degree, dtype=np.int64)
    # Degrees 0 .. min(2 degree, d_model): empty neurons and heavy neurons, as a pruned support has.
    return rng.integers(0, min(2 * degree, d_model) + 1, size=d_ff, dtype=np.int64)


def _projection(rng: np.random.Generator, degrees: np.ndarray, d_model: int, scale: float):
    offsets = np.zeros(degrees.size + 1, dtype=np.int32)
    offsets[1:] = np.cumsum(degrees)
    idx = np.empty(int(offsets[-1]), dtype=np.int16)
    for hidden, degree in enumerate(degrees.tolist()):
        idx[offsets[hidden]:offsets[hidden + 1]] = np.sort(rng.choice(d_model, size=int(degree), replace=False))
    val = (rng.standard_normal(idx.size) * scale).astype(np.float32)
    return offsets, idx, val


def make_layer(case: Case) -> CompactLayer:
    rng = np.random.default_rng(case.seed)
    up_deg = _degrees(rng, case.d_ff, case.up_degree, case.d_model, case.irregular)
    down_deg = _degrees(rng, case.d_ff, case.down_degree, case.d_model, case.irregular)
    up_offsets, up_idx, up_val = _projection(rng, up_deg, case.d_model, 1.0 / np.sqrt(case.up_degree))
    down_offsets, down_idx, down_val = _projection(rng, down_deg, case.d_model, 1.0 / np.sqrt(case.down_degree))
    b_up = (rng.standard_normal(case.d_ff) * case.bias_std).astype(np.float32)
    b_down = (rng.standard_normal(case.d_model) * case.bias_std).astype(np.float32)
    groups = np.array([(g * case.d_ff) // N_GROUPS for g in range(N_GROUPS + 1)], dtype=np.int32)
    return CompactLayer(case.d_model, case.d_ff, groups, up_offsets, up_idx, up_val, b_up,
                        down_offsets, down_idx, down_val, b_down)


def make_input(case: Case, n: int) -> np.ndarray:
    """Token-major float32 input ``[n, d_model]`` (PCG64 seeded by ``[case.seed, n]``)."""
    rng = np.random.default_rng([case.seed, n])
    return np.ascontiguousarray(rng.standard_normal((n, case.d_model)).astype(np.float32))


def make_target(case: Case, n: int) -> np.ndarray:
    """Token-major float32 regression target ``[n, d_model]`` for the MSE training step (seed ``[seed, n, 7919]``)."""
    rng = np.random.default_rng([case.seed, n, 7919])
    return np.ascontiguousarray(rng.standard_normal((n, case.d_model)).astype(np.float32))


def make_upstream(case: Case, n: int, salt: int) -> np.ndarray:
    """Upstream gradient ``[n, d_model]`` float32 x 0.1 (PCG64 seeded by ``[seed, n, 7919, salt]``), the form of the
    reference's ``runtime/gpu/nvidia/ffn/training/train_step.py:28-32``."""
    rng = np.random.Generator(np.random.PCG64([case.seed, n, 7919, salt]))
    return (rng.standard_normal((n, case.d_model)).astype(np.float32) * 0.1)


FINGERPRINT_FIELDS = ("groups", "up_offsets", "up_idx", "up_val", "b_up", "down_offsets", "down_idx", "down_val", "b_down")
FINGERPRINT_N = (1, 2, 4, 7, 8, 16, 32, 64, 96, 128)


def fingerprint(layer: CompactLayer, case: Case) -> str:
    """SHA-256 of the layer arrays then of the inputs for ``FINGERPRINT_N`` (``layers.py:37-45`` of the reference)."""
    import hashlib
    digest = hashlib.sha256()
    for name in FINGERPRINT_FIELDS:
        digest.update(getattr(layer, name).tobytes())
    for n in FINGERPRINT_N:
        digest.update(make_input(case, n).tobytes())
    return digest.hexdigest()
