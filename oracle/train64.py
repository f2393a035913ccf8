"""TEST INFRASTRUCTURE ONLY. Float64 training step of one compact HFFN layer (the checker of the CUDA backward/AdamW).

Restates ``runtime/gpu/nvidia/ffn/training/train_step.py:56-82`` (every group of the step, hidden-major slot order)
and ``train_step.py:85-91`` (AdamW closed form, the form of ``torch.optim.AdamW``):

    z = b_up + W_up x,  h = gelu(z),  y = b_down + W_down h
    gb_down = sum_t gy,   g_down[q] = sum_t gy[t, o_q] h[t, r_q]
    dh[t, r] = sum_q down_val[q] gy[t, o_q],   gz = dh * gelu'(z)
    gb_up = sum_t gz,     g_up[e] = sum_t gz[t, r_e] x[t, i_e]
    gx[t, i] = sum_e up_val[e] gz[t, r_e]

The MSE loss of the training benchmark (not in the reference, which takes gy from the caller):
``L = mean((y - target)^2)`` over all N x d_model entries, so ``gy = 2 (y - target) / (N d_model)``, the
convention of ``torch.nn.functional.mse_loss(reduction="mean")``.
"""
from __future__ import annotations

import numpy as np

from . import forward64

HYPER = dict(lr=1e-3, betas=(0.9, 0.999), eps=1e-8, weight_decay=1e-2)
GROUPS = ("y", "gb_down", "g_down", "gz", "g_up", "gb_up", "gx")


def hidden_of_slot(offsets: np.ndarray) -> np.ndarray:
    return np.repeat(np.arange(offsets.size - 1), np.diff(offsets))


def step_groups(layer, x: np.ndarray, gy: np.ndarray, params: dict | None = None, chunk: int = 64) -> dict:
    """Every group of one step in float64, hidden-major slot order for ``g_up`` and ``g_down`` (train_step.py:56-82).

    ``gy`` may be a callable ``gy(y_chunk, lo, hi)`` returning the upstream gradient of a token chunk from its
    output (the MSE loss uses it). ``params`` (float64 ``up_val``, ``b_up``, ``down_val``, ``b_down``, hidden-major)
    overrides the layer's values."""
    p = params or {"up_val": layer.up_val, "b_up": layer.b_up, "down_val": layer.down_val, "b_down": layer.b_down}
    up_val, b_up = np.asarray(p["up_val"], np.float64), np.asarray(p["b_up"], np.float64)
    down_val, b_down = np.asarray(p["down_val"], np.float64), np.asarray(p["b_down"], np.float64)
    up_hidden, up_input = hidden_of_slot(layer.up_offsets), layer.up_idx.astype(np.int64)
    down_hidden, down_output = hidden_of_slot(layer.down_offsets), layer.down_idx.astype(np.int64)
    n, d, f = x.shape[0], layer.d_model, layer.d_ff
    # scatters over outputs (y) and inputs (gx) as segment sums over the slots sorted by their target feature
    by_output = np.argsort(down_output, kind="stable")
    output_offsets = np.concatenate([[0], np.cumsum(np.bincount(down_output, minlength=d))])
    by_input = np.argsort(up_input, kind="stable")
    input_offsets = np.concatenate([[0], np.cumsum(np.bincount(up_input, minlength=d))])
    out = {"y": np.empty((n, d)), "gz": np.empty((f, n)), "gx": np.empty((n, d)),
           "g_up": np.zeros(up_val.size), "g_down": np.zeros(down_val.size),
           "gb_up": np.zeros(f), "gb_down": np.zeros(d)}
    for lo in range(0, n, chunk):
        hi = min(n, lo + chunk)
        xc = np.asarray(x[lo:hi], np.float64)
        z = b_up + forward64.segment_sum(xc[:, up_input] * up_val, layer.up_offsets)
        h = forward64.gelu(z)
        y = b_down + forward64.segment_sum(h[:, down_hidden[by_output]] * down_val[by_output], output_offsets)
        out["y"][lo:hi] = y
        gc = np.asarray(gy(y, lo, hi) if callable(gy) else gy[lo:hi], np.float64)
        out["gb_down"] += gc.sum(0)
        out["g_down"] += (gc[:, down_output] * h[:, down_hidden]).sum(0)
        dh = forward64.segment_sum(gc[:, down_output] * down_val, layer.down_offsets)
        gz = dh * forward64.gelu_grad(z)
        out["gz"][:, lo:hi] = gz.T
        out["gb_up"] += gz.sum(0)
        out["g_up"] += (gz[:, up_hidden] * xc[:, up_input]).sum(0)
        out["gx"][lo:hi] = forward64.segment_sum(gz[:, up_hidden[by_input]] * up_val[by_input], input_offsets)
    return out


def mse_upstream(target: np.ndarray, n_total: int):
    """The ``gy`` callable of the MSE loss ``mean((y - target)^2)`` over ``n_total x d_model`` entries."""
    def gy(y, lo, hi):
        return 2.0 * (y - np.asarray(target[lo:hi], np.float64)) / (n_total * y.shape[1])
    return gy


def mse_loss(y: np.ndarray, target: np.ndarray) -> float:
    diff = np.asarray(y, np.float64) - np.asarray(target, np.float64)
    return float((diff * diff).mean())


def adamw_closed_form(p, g, m, v, step: int, lr, betas, eps, weight_decay):
    """One AdamW update in float64: decoupled decay, bias correction (train_step.py:85-91)."""
    b1, b2 = betas
    m = b1 * m + (1 - b1) * g
    v = b2 * v + (1 - b2) * g * g
    p = p * (1 - lr * weight_decay) - lr * (m / (1 - b1 ** step)) / (np.sqrt(v / (1 - b2 ** step)) + eps)
    return p, m, v
