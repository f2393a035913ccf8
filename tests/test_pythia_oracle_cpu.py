"""CPU: the Pythia token oracle pinned to the reference's own dense arm.

``tests/golden/pythia_dense_tiny.npz`` holds the prefill logits and the greedy tokens of the reference's
``load_pythia(model_dir, export_dir, "dense", None, "cpu")`` (``runtime/common/pythia/hffn_pythia/model.py:82-111``,
run unchanged by ``tests/golden/make_pythia_golden.py``) on a tiny seeded random-init model. Here the same model is
regenerated (its files' digest must match the fixture's, so generator drift is told apart from a parity failure) and
``oracle/pythia_dense.dense_pythia`` (the token oracle of the GPU tests), and this repository's own loader's dense arm,
must reproduce the reference's logits within float32 rounding (1e-5 relative to max(1, |logit|): the host's BLAS may
sum in another order than the machine that wrote the fixture) and its greedy tokens exactly.
"""
import json
import sys
from pathlib import Path

import numpy as np
import pytest
import torch

from hffn_b200 import pythia
from oracle import pythia_dense

GOLDEN = Path(__file__).resolve().parent / "golden"
sys.path.insert(0, str(GOLDEN))
import make_pythia_golden as golden  # noqa: E402


@pytest.fixture(scope="module")
def tiny(tmp_path_factory):
    fixture = np.load(GOLDEN / "pythia_dense_tiny.npz")
    config = json.loads(str(fixture["config"]))
    root = tmp_path_factory.mktemp("pythia_tiny")
    pythia.make_random_pythia(root / "model", root / "export", config["arch"], support=config["support"],
                              seed=config["seed"])
    assert golden.files_digest(root / "model", root / "export") == str(fixture["digest"]), "generator drift"
    return root, fixture


def check(model, fixture):
    logits, tokens = golden.run(model, torch.from_numpy(fixture["ids"]))
    expected = fixture["logits"].astype(np.float64)
    relative = float(np.max(np.abs(logits - expected) / np.maximum(1.0, np.abs(expected))))
    assert relative <= 1e-5, relative
    assert np.array_equal(tokens, fixture["tokens"]), (tokens, fixture["tokens"])


def test_oracle_dense_arm_matches_reference_loader(tiny):
    root, fixture = tiny
    check(pythia_dense.dense_pythia(root / "model", root / "export", "cpu"), fixture)


def test_product_dense_arm_matches_reference_loader(tiny):
    root, fixture = tiny
    check(pythia.load_pythia(root / "model", root / "export", "dense", "cpu"), fixture)


def test_negative_control_detected(tiny):
    """An attention weight of the oracle scaled by 1.5 (the reference's negative control, planted in the oracle on
    the CPU) moves the logits far past the bound."""
    root, fixture = tiny
    model = pythia_dense.dense_pythia(root / "model", root / "export", "cpu")
    with torch.no_grad():
        model.gpt_neox.layers[1].attention.dense.weight.mul_(1.5)
    with pytest.raises(AssertionError):
        check(model, fixture)
