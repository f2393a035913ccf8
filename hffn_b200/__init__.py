"""HFFN fixed-support sparse FFN on B200 (sm_100a): hand-written CUDA kernels behind a C ABI, with the reference's
Python layer API (``HFFNLayer``, ``HFFNRuntime``, ``HFFNTrainRuntime``, ``parity.check``).

Submodules load ``lib/libhffn_b200.so`` on first use; ``hffn_b200.build`` and ``hffn_b200.synth`` import without it.
"""
from __future__ import annotations

_LAZY = {
    "HFFNLayer": "runtime", "HFFNRuntime": "runtime", "UP_MODES": "runtime", "DOWN_MODES": "runtime",
    "MAX_TOKENS": "runtime", "up_mode": "runtime", "down_mode": "runtime",
    "HFFNTrainRuntime": "train_runtime", "transposed_supports": "train_runtime",
}


def __getattr__(name: str):
    if name in _LAZY:
        import importlib
        return getattr(importlib.import_module(f".{_LAZY[name]}", __name__), name)
    raise AttributeError(name)
