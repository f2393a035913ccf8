"""Golden logits of the reference's own Pythia dense arm, for pinning ``oracle/pythia_dense.py``.

Run where the reference tree exists (``$HFFN_REFERENCE``, else the conventional mount point, or the first argument):
it writes a tiny seeded random-init GPT-NeoX checkpoint and seeded synthetic exports with this repository's
``hffn_b200.pythia.make_random_pythia`` (the reference's export format), loads them through the reference's
``hffn_pythia.model.load_pythia(model_dir, export_dir, "dense", None, "cpu")``
(``runtime/common/pythia/hffn_pythia/model.py:82-111``, float32 on the CPU, imported unchanged), and records its
prefill logits on seeded token ids and its greedy tokens over a cached decode. The fixture also holds the SHA-256 of
the generated checkpoint and exports, so a test that regenerates the model can tell generator drift from a parity
failure. Output: ``tests/golden/pythia_dense_tiny.npz``.
"""
from __future__ import annotations

import hashlib
import json
import os
import sys
import tempfile
from pathlib import Path

import numpy as np
import torch

HERE = Path(__file__).resolve().parent
ROOT = HERE.parents[1]
sys.path.insert(0, str(ROOT))

from hffn_b200 import pythia  # noqa: E402

ARCH = dict(pythia.PYTHIA_410M, hidden_size=64, num_hidden_layers=2, num_attention_heads=4, intermediate_size=256,
            vocab_size=512, max_position_embeddings=128)
SUPPORT, SEED = 32, 17
BATCH, PROMPT, DECODE = 2, 16, 8
OUT = HERE / "pythia_dense_tiny.npz"


def files_digest(model_dir: Path, export_dir: Path) -> str:
    h = hashlib.sha256()
    for path in [model_dir / "model.safetensors", *sorted(export_dir.rglob("*.pt"))]:
        h.update(path.read_bytes())
    return h.hexdigest()


def prompt_ids() -> torch.Tensor:
    return torch.randint(0, ARCH["vocab_size"], (BATCH, PROMPT), generator=torch.Generator().manual_seed(23))


@torch.no_grad()
def run(model, ids: torch.Tensor) -> tuple[np.ndarray, np.ndarray]:
    """Prefill logits [B, T, V] (float32) and the greedy tokens of a cached decode [B, DECODE]."""
    out = model(input_ids=ids, use_cache=True)
    logits = out.logits.float().numpy()
    tokens, cache, token = [], out.past_key_values, out.logits[:, -1:].argmax(-1)
    for _ in range(DECODE):
        tokens.append(token)
        out = model(input_ids=token, past_key_values=cache, use_cache=True)
        cache, token = out.past_key_values, out.logits[:, -1:].argmax(-1)
    return logits, torch.cat(tokens, dim=1).numpy()


def main() -> int:
    reference = Path(sys.argv[1] if len(sys.argv) > 1 else os.environ.get("HFFN_REFERENCE", "/root/reference"))
    sys.path.insert(0, str(reference / "runtime/common/pythia"))
    from hffn_pythia.model import load_pythia  # the reference's loader, unchanged
    with tempfile.TemporaryDirectory() as tmp:
        model_dir, export_dir = Path(tmp) / "model", Path(tmp) / "export"
        pythia.make_random_pythia(model_dir, export_dir, ARCH, support=SUPPORT, seed=SEED)
        model = load_pythia(model_dir, export_dir, "dense", None, "cpu")
        logits, tokens = run(model, prompt_ids())
        digest = files_digest(model_dir, export_dir)
    np.savez_compressed(OUT, logits=logits, tokens=tokens, ids=prompt_ids().numpy(), digest=np.array(digest),
                        config=np.array(json.dumps({"arch": ARCH, "support": SUPPORT, "seed": SEED})))
    print(f"wrote {OUT}: logits {logits.shape}, tokens {tokens.tolist()}, digest {digest[:16]}")
    return 0


if __name__ == "__main__":
    raise SystemExit(main())
