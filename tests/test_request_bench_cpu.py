"""CPU: the request-level harness's bookkeeping (cells, per-cell summary, the A/A verdict) and the sharing of the
non-FFN modules between arms."""
import pytest
import torch

from hffn_b200 import request_bench as rb


def row(size, density, shape, hffn, dense, copy):
    return {"size": size, "density": density, "shape": shape,
            "samples_ms": {"hffn": [hffn, hffn * 1.01], "dense": [dense, dense], "hffn_copy": [copy, copy]}}


def test_cells_cover_the_grid():
    grid = rb.GRIDS["run"]
    cells = rb.cells_of(grid)
    assert len(cells) == len(grid["sizes"]) * len(grid["densities"]) * len(grid["shapes"])
    assert len({(c["size"], c["density"], c["shape"]) for c in cells}) == len(cells)


def test_summary_and_admissible_verdict():
    rows = [row(70, 20, "decode_b1", 2.0, 4.0, 2.02), row(70, 20, "decode_b1", 2.1, 4.1, 2.1)]
    summary = rb.summarize(rows)
    assert len(summary) == 1 and summary[0]["sessions"] == 2
    assert summary[0]["hffn_over_dense"] == pytest.approx((2.01 / 4.0 + 2.1105 / 4.1) / 2)
    verdict = rb.verdict(summary, complete=True, gate_passed=True)
    assert verdict["admissible"] and verdict["aa_values"] == 2


def test_verdict_rejects_a_failed_aa_control_or_incomplete_runs():
    rows = [row(70, 20, "prefill_b1", 2.0, 4.0, 2.5)]          # A/A ratio 1.24: outside 3 %
    assert not rb.verdict(rb.summarize(rows), complete=True, gate_passed=True)["admissible"]
    assert not rb.verdict(rb.summarize([row(70, 20, "prefill_b1", 2, 4, 2)]), complete=True,
                          gate_passed=False)["admissible"]
    assert rb.verdict([], complete=False, gate_passed=True) == {"admissible": False, "reason": "incomplete coverage"}


def test_share_non_ffn_keeps_only_the_ffns_distinct():
    from transformers import GPTNeoXConfig, GPTNeoXForCausalLM
    config = GPTNeoXConfig(vocab_size=128, hidden_size=64, num_hidden_layers=2, num_attention_heads=4,
                           intermediate_size=256)
    torch.manual_seed(0)
    source, target = GPTNeoXForCausalLM(config).eval(), GPTNeoXForCausalLM(config).eval()
    target.load_state_dict({k: v for k, v in source.state_dict().items() if ".mlp." in k}, strict=False)
    rb.share_non_ffn(target, source)
    assert target.embed_out is source.embed_out and target.gpt_neox.embed_in is source.gpt_neox.embed_in
    for tb, sb in zip(target.gpt_neox.layers, source.gpt_neox.layers):
        assert tb.attention is sb.attention and tb.mlp is not sb.mlp
    ids = torch.randint(0, 128, (1, 9))
    with torch.no_grad():
        assert torch.equal(target(input_ids=ids).logits, source(input_ids=ids).logits)
