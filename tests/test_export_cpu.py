"""CPU: the hffn_training_compact_g4_v2 export format (write / read round trip, refusals) and the dense arm of the
Pythia loader against the oracle's dense arm on a tiny random-init model."""
import pytest
import torch

from hffn_b200 import export, pythia, synth


def test_round_trip_and_refusals(tmp_path):
    layer = export.from_compact(synth.make_layer(synth.TEST_CASES["irreg_512_2048"]))
    path = export.layer_path(tmp_path, 0)
    export.write_layer(path, layer)
    back = export.read_layer(path)
    for key in export.TYPES:
        assert torch.equal(back[key], layer[key]), key
    assert torch.equal(back["group_hidden_offsets"], layer["group_hidden_offsets"])
    bad = dict(layer, up_idx=layer["up_idx"].clone())
    bad["up_idx"][0] = 600
    with pytest.raises(ValueError):
        export.write_layer(tmp_path / "bad.pt", bad)
    bad = dict(layer, down_row_offsets=layer["down_row_offsets"].clone())
    bad["down_row_offsets"][-1] += 1
    with pytest.raises(ValueError):
        export.validate(bad)
    bad = dict(layer, up_val=layer["up_val"].double())
    with pytest.raises(ValueError):
        export.validate(bad)
    torch.save({"format": "other"}, tmp_path / "other.pt")
    with pytest.raises(ValueError):
        export.read_layer(tmp_path / "other.pt")


def test_dense_arm_matches_oracle_on_cpu(tmp_path):
    from oracle import pythia_dense
    arch = dict(pythia.PYTHIA_410M, hidden_size=64, num_hidden_layers=2, num_attention_heads=4, intermediate_size=256,
                vocab_size=512)
    pythia.make_random_pythia(tmp_path / "model", tmp_path / "export", arch, support=32, seed=5)
    ours = pythia.load_pythia(tmp_path / "model", tmp_path / "export", "dense", "cpu")
    ref = pythia_dense.dense_pythia(tmp_path / "model", tmp_path / "export", "cpu")
    ids = torch.randint(0, 512, (2, 12), generator=torch.Generator().manual_seed(0))
    with torch.no_grad():
        assert torch.equal(ours(input_ids=ids).logits, ref(input_ids=ids).logits)
    with pytest.raises(ValueError):
        pythia.load_pythia(tmp_path / "model", tmp_path / "export", "sparse", "cpu")
