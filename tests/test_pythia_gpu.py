"""GPU: the Pythia FFN swap-in (HFFNMLP / load_pythia) against the dense arm, with the reference's token criterion.

Random-init GPT-NeoX checkpoints with seeded synthetic HFFN exports (no checkpoint or text is available offline;
token ids are drawn uniformly). The dense arm (``oracle/pythia_dense``) is pinned to the reference's own loader by
``tests/test_pythia_oracle_cpu.py``. The HFFN arm's greedy tokens must equal the dense control's or be explained by
the float64 arbiter within the control's own error band (the reference's criterion); in float32 they must be
identical; a fault planted in the HFFN arm (one attention weight scaled by 1.5, the reference's negative control)
must be detected. Float32 on a small model,
bfloat16 on the Pythia-410M architecture of the benchmark plan (24 layers, d_model 1024, d_ff 4096, 50 % supports).
"""
import pytest
import torch

from hffn_b200 import pythia
from oracle import pythia_dense

pytestmark = pytest.mark.gpu

SMALL = dict(pythia.PYTHIA_410M, hidden_size=256, num_hidden_layers=4, num_attention_heads=4, intermediate_size=1024,
             vocab_size=2048)


@pytest.fixture(scope="module")
def small_model(tmp_path_factory):
    root = tmp_path_factory.mktemp("pythia_small")
    pythia.make_random_pythia(root / "model", root / "export", SMALL, support=128, seed=11)
    return root


def prompts(vocab: int, shapes, seed: int):
    g = torch.Generator().manual_seed(seed)
    return [torch.randint(0, vocab, (b, t), generator=g).cuda() for b, t in shapes]


def test_small_float32_token_parity_and_negative_control(small_model):
    dense = pythia_dense.dense_pythia(small_model / "model", small_model / "export", "cuda")
    arbiter = pythia_dense.dense_pythia(small_model / "model", small_model / "export", "cuda", torch.float64)
    hffn = pythia.load_pythia(small_model / "model", small_model / "export", "hffn", "cuda")
    assert hffn.hffn_runtime is not None and not any(".mlp." in n for n, _ in hffn.named_parameters())
    ps = prompts(SMALL["vocab_size"], ((1, 32), (4, 32), (1, 300)), 5)
    result = pythia_dense.check_arm(dense, hffn, arbiter, ps)
    print(f"pythia-small float32: {result}")
    assert result["unexplained"] == 0, result
    assert result["differs"] == 0, result
    assert hffn.hffn_runtime.device_errors() == 0
    # prefill of 300 tokens used the tensor-core pair, decode the cooperative kernels
    calls = hffn.hffn_runtime.calls
    assert calls[("tc", "tc")] > 0 and calls[("coop", "coop")] > 0, calls
    with torch.no_grad():
        hffn.gpt_neox.layers[1].attention.dense.weight.mul_(1.5)
    faulty = pythia_dense.check_arm(dense, hffn, arbiter, ps)
    assert faulty["unexplained"] > 0, faulty


def test_load_pythia_dense_arm_matches_oracle(small_model):
    ours = pythia.load_pythia(small_model / "model", small_model / "export", "dense", "cuda")
    ref = pythia_dense.dense_pythia(small_model / "model", small_model / "export", "cuda")
    ids = prompts(SMALL["vocab_size"], ((2, 24),), 9)[0]
    with torch.no_grad():
        assert torch.equal(ours(input_ids=ids).logits, ref(input_ids=ids).logits)


@pytest.fixture(scope="module")
def pythia_410m(tmp_path_factory):
    root = tmp_path_factory.mktemp("pythia_410m")
    pythia.make_random_pythia(root / "model", root / "export", pythia.PYTHIA_410M, support=512, seed=3004)
    return root


@pytest.mark.parametrize("dtype", [torch.float32, torch.bfloat16])
def test_pythia_410m_tokens(pythia_410m, dtype):
    """The benchmark model as the plan runs it: prefill of 8 x 512 tokens, then 128 greedy steps (arbiter-driven).
    float32: the reference's criterion as it is (its loader path is float32); bfloat16: the same criterion with the
    control's global band. The counts of positions where the HFFN token differs from the dense control's are printed
    beside it."""
    dense = pythia_dense.dense_pythia(pythia_410m / "model", pythia_410m / "export", "cuda", dtype)
    arbiter = pythia_dense.dense_pythia(pythia_410m / "model", pythia_410m / "export", "cuda", torch.float64)
    hffn = pythia.load_pythia(pythia_410m / "model", pythia_410m / "export", "hffn", "cuda", dtype)
    ps = prompts(50277, ((8, 512),), 3004)
    band = "pointwise" if dtype == torch.float32 else "global"
    result = pythia_dense.check_arm(dense, hffn, arbiter, ps, steps=128, band=band)
    print(f"pythia-410m {dtype}: {result}")
    assert result["unexplained"] == 0, result
    if dtype == torch.float32:                  # identical greedy tokens (measured: 0 of 5120 positions differ)
        assert result["differs"] == 0, result
    assert hffn.hffn_runtime.device_errors() == 0
    with torch.no_grad():
        hffn.gpt_neox.layers[3].attention.dense.weight.mul_(1.5)
    faulty = pythia_dense.check_arm(dense, hffn, arbiter, ps, steps=8, band=band)
    assert faulty["unexplained"] > 0, faulty
