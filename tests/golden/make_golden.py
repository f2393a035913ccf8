"""Generates the golden fixtures of this directory by running the reference's own Python code.

Run where the reference tree exists (``python tests/golden/make_golden.py [reference_root]``); the GPU box and the
tests only read the committed ``.npz`` / ``.json`` outputs.

- ``fingerprints.json``: the reference's pinned SHA-256 of its three test layers and inputs
  (``runtime/common/ffn/reference/fingerprints.json``), which pin the seeded generator.
- ``forward_<layer>_n<N>.npz``: ``x`` and the float64 oracle output ``y`` of ``runtime/common/ffn/hffn_ffn_layers/
  reference.py:21-38`` (stored as float32: the pin is the algorithm, not the last bits).
- ``train_<layer>_n<N>.npz``: every group of ``runtime/gpu/nvidia/ffn/training/train_step.py:56-82`` for the upstream
  gradient ``make_gy(case, N, 0)`` (float32 storage), and one AdamW closed form (``train_step.py:85-91``).
- ``layout_homog_256_1024.npz`` and ``layout_digests.json`` (SHA-256 of each array, both layers): the kernel arrays of ``HFFNLayer.from_hidden_major`` (``runtime/gpu/nvidia/common/kernels/
  hffn_cuda/runtime.py:55-67``) and ``transposed_supports`` (``runtime/gpu/nvidia/ffn/training/train_runtime.py:39-56``).
  Both modules import CuPy at their top, which is absent here, so the two functions are taken from the reference
  source by ``ast`` and executed unchanged with torch.
"""
from __future__ import annotations

import ast
import hashlib
import json
import os
import sys
from dataclasses import dataclass
from pathlib import Path

import numpy as np
import torch

HERE = Path(__file__).resolve().parent
REFERENCE = Path(sys.argv[1] if len(sys.argv) > 1 else os.environ.get("HFFN_REFERENCE", "/root/reference"))
FFN_COMMON = REFERENCE / "runtime/common/ffn"
TRAINING = REFERENCE / "runtime/gpu/nvidia/ffn/training"
RUNTIME_PY = REFERENCE / "runtime/gpu/nvidia/common/kernels/hffn_cuda/runtime.py"
TRAIN_RUNTIME_PY = TRAINING / "train_runtime.py"

FORWARD_CASES = (("homog_256_1024", (1, 7, 64)), ("homog_512_2048", (1, 5)), ("irreg_512_2048", (1, 9, 33)))
TRAIN_CASES = (("homog_256_1024", (1, 7)), ("irreg_512_2048", (3,)))
ADAMW_SLICE = 2048


def _extract(path: Path, name: str, namespace: dict):
    """Execute the top-level definition ``name`` of ``path`` in ``namespace`` and return it."""
    tree = ast.parse(path.read_text())
    node = next(n for n in tree.body if isinstance(n, (ast.FunctionDef, ast.ClassDef)) and n.name == name)
    code = compile(ast.Module(body=[node], type_ignores=[]), str(path), "exec")
    exec(code, namespace)
    return namespace[name]


def main() -> int:
    sys.path.insert(0, str(FFN_COMMON))
    sys.path.insert(0, str(TRAINING))
    from hffn_ffn_layers import layers, reference  # the reference's own modules
    import train_step as ts

    pinned = json.loads((FFN_COMMON / "reference/fingerprints.json").read_text())["fingerprints"]
    (HERE / "fingerprints.json").write_text(json.dumps({"source": "runtime/common/ffn/reference/fingerprints.json",
                                                        "fingerprints": pinned}, indent=1) + "\n")
    namespace = {"torch": torch, "dataclass": dataclass, "annotations": None}
    hffn_layer = _extract(RUNTIME_PY, "HFFNLayer", namespace)
    transposed = _extract(TRAIN_RUNTIME_PY, "transposed_supports", namespace)

    for name, ns in FORWARD_CASES:
        layer, case = layers.load(name)
        for n in ns:
            x = layers.make_input(case, n)
            y = reference.forward(layer, x)
            np.savez_compressed(HERE / f"forward_{name}_n{n}.npz", x=x, y=y.astype(np.float32))

    for name, ns in TRAIN_CASES:
        layer, case = layers.load(name)
        for n in ns:
            x = torch.from_numpy(layers.make_input(case, n))
            gy = ts.make_gy(case, n, 0)
            out = ts.oracle(layer, x, gy)
            g = out["g_up"]
            p1, m1, v1 = ts.adamw_closed_form(torch.from_numpy(layer.up_val).double(), g, torch.zeros_like(g),
                                              torch.zeros_like(g), 1, **ts.HYPER)
            keep = slice(0, ADAMW_SLICE)
            np.savez_compressed(HERE / f"train_{name}_n{n}.npz", x=x.numpy(), gy=gy.numpy(),
                                **{k: v.numpy().astype(np.float32) for k, v in out.items()},
                                adamw_up_val=p1.numpy()[keep], adamw_m=m1.numpy()[keep], adamw_v=v1.numpy()[keep])

    digests = {}
    for name in ("homog_256_1024", "irreg_512_2048"):
        layer, _ = layers.load(name)
        t = torch.from_numpy
        kl = hffn_layer.from_hidden_major(layer.d_model, layer.d_ff, t(layer.b_up), t(layer.up_offsets), t(layer.up_idx),
                                          t(layer.up_val), t(layer.b_down), t(layer.down_offsets), t(layer.down_idx),
                                          t(layer.down_val))
        sup = transposed(kl)
        arrays = {"out_offsets": kl.out_offsets.numpy(), "out_hidden": kl.out_hidden.numpy(),
                  "out_val": kl.out_val.numpy(), **{k: v.numpy() for k, v in sup.items()}}
        digests[name] = {k: hashlib.sha256(np.ascontiguousarray(v).tobytes()).hexdigest() for k, v in arrays.items()}
        if name == "homog_256_1024":
            np.savez_compressed(HERE / f"layout_{name}.npz", **arrays)
    (HERE / "layout_digests.json").write_text(json.dumps(digests, indent=1) + "\n")
    print("golden fixtures written to", HERE)
    return 0


if __name__ == "__main__":
    raise SystemExit(main())
