"""GPU: one cell of the request-level harness on a small GPT-NeoX architecture: the gates hold (the second HFFN
runtime gives the first's logits bit for bit, HFFN within the guard of dense) and every arm is timed."""
import pytest

from hffn_b200 import request_bench as rb

pytestmark = pytest.mark.gpu

TINY = {1: {"hidden_size": 256, "num_hidden_layers": 2, "num_attention_heads": 4, "intermediate_size": 1024}}


@pytest.mark.parametrize("shape", ["prefill_b1", "decode_b4"])
def test_one_cell(tmp_path_factory, shape):
    assets = tmp_path_factory.getbasetemp() / "request_assets"
    rb.make_assets(assets, sizes=(1,), densities=(50,), architectures=TINY)
    row = rb.run_cell({"size": 1, "density": 50, "shape": shape, "session": 0, "parity": 0, "blocks": 1,
                       "window_ms": 20.0, "assets": str(assets)})
    assert row["gate_passed"] and row["bitwise_copy"], row
    assert row["hffn_vs_dense_relative_gap"] <= rb.GUARD
    assert all(len(row["samples_ms"][arm]) == 2 and min(row["samples_ms"][arm]) > 0 for arm in rb.ARMS)
    assert row["runtime"]["device_errors"] == 0
