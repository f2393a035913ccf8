"""TEST INFRASTRUCTURE ONLY. Float64 forward of one compact HFFN layer (the checker of the CUDA forward).

Restates ``runtime/common/ffn/hffn_ffn_layers/reference.py:21-38`` of the reference: the pre-activation of neuron r
is ``b_up[r] + sum over its up slots of up_val[e] * x[t, up_idx[e]]``, ``h = gelu(z)`` with the exact erf form
(``reference.py:17-18``), and ``y[t, o] = b_down[o] + sum over the down slots of output o of down_val * h``.
Sums are per-neuron segment sums over the hidden-major slots (numpy ``add.reduceat``), in float64; at the float32
tolerances of the tests the float64 summation order does not matter.
"""
from __future__ import annotations

import math

import numpy as np

_erf = np.vectorize(math.erf, otypes=[np.float64])
TOKEN_CHUNK = 16


def gelu(z: np.ndarray) -> np.ndarray:
    """Exact GELU, ``0.5 z (1 + erf(z / sqrt 2))`` (reference.py:17-18), float64."""
    return 0.5 * z * (1.0 + _erf(z * 0.7071067811865476))


def gelu_grad(z: np.ndarray) -> np.ndarray:
    """``0.5 (1 + erf(z / sqrt 2)) + z phi(z)`` (train_step.py:51-52 of the training leaf), float64."""
    return 0.5 * (1.0 + _erf(z * 0.7071067811865476)) + z * np.exp(-0.5 * z * z) * 0.3989422804014327


def segment_sum(values: np.ndarray, offsets: np.ndarray) -> np.ndarray:
    """Sum of ``values[:, offsets[k]:offsets[k + 1]]`` for every k (zero for an empty segment)."""
    offsets = np.asarray(offsets, dtype=np.int64)
    count = offsets.size - 1
    out = np.zeros(values.shape[:-1] + (count,), dtype=np.float64)
    nonempty = np.flatnonzero(np.diff(offsets) > 0)
    if nonempty.size:
        out[..., nonempty] = np.add.reduceat(values, offsets[nonempty], axis=-1)
    return out


def hidden(layer, x: np.ndarray, up_val=None, b_up=None) -> np.ndarray:
    """Pre-activations ``z[N, d_ff]`` in float64."""
    x = np.asarray(x, dtype=np.float64)
    w = np.asarray(layer.up_val if up_val is None else up_val, dtype=np.float64)
    b = np.asarray(layer.b_up if b_up is None else b_up, dtype=np.float64)
    idx = layer.up_idx.astype(np.int64)
    z = np.empty((x.shape[0], layer.d_ff), dtype=np.float64)
    for lo in range(0, x.shape[0], TOKEN_CHUNK):
        hi = min(x.shape[0], lo + TOKEN_CHUNK)
        z[lo:hi] = b + segment_sum(x[lo:hi][:, idx] * w, layer.up_offsets)
    return z


def down(layer, h: np.ndarray, down_val=None, b_down=None) -> np.ndarray:
    """``y[N, d_model]`` from ``h[N, d_ff]`` in float64, summed per output over its down slots."""
    v = np.asarray(layer.down_val if down_val is None else down_val, dtype=np.float64)
    b = np.asarray(layer.b_down if b_down is None else b_down, dtype=np.float64)
    output = layer.down_idx.astype(np.int64)
    order = np.argsort(output, kind="stable")
    offsets = np.zeros(layer.d_model + 1, dtype=np.int64)
    offsets[1:] = np.cumsum(np.bincount(output, minlength=layer.d_model))
    hid = np.repeat(np.arange(layer.d_ff), np.diff(layer.down_offsets))[order]
    v = v[order]
    y = np.empty((h.shape[0], layer.d_model), dtype=np.float64)
    for lo in range(0, h.shape[0], TOKEN_CHUNK):
        hi = min(h.shape[0], lo + TOKEN_CHUNK)
        y[lo:hi] = b + segment_sum(h[lo:hi][:, hid] * v, offsets)
    return y


def forward(layer, x: np.ndarray) -> np.ndarray:
    """``y[N, d_model]`` in float64 for ``x[N, d_model]`` (reference.py:21-38)."""
    return down(layer, gelu(hidden(layer, x)))
