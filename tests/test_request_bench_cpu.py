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


class _Worker:
    """Stands in for the fresh worker process of a cell: one JSON row per call, gate held or not."""

    def __init__(self, gate_fails_at=None):
        self.calls, self.gate_fails_at = [], gate_fails_at

    def __call__(self, command, text, capture_output, cwd):
        import json
        import types
        job = json.loads(command[command.index("--worker") + 1])
        self.calls.append(job)
        passed = len(self.calls) != self.gate_fails_at
        row = {**{k: v for k, v in job.items() if k != "assets"}, "repeats": 3, "bitwise_copy": passed,
               "hffn_vs_dense_relative_gap": 1e-6, "gate_passed": passed,
               "samples_ms": {"hffn": [1.0, 1.0], "dense": [2.0, 2.0], "hffn_copy": [1.01, 1.01]}}
        return types.SimpleNamespace(returncode=0 if passed else 4, stdout=json.dumps(row) + "\n", stderr="")


def test_orchestrate_runs_every_cell_in_alternating_order(tmp_path, monkeypatch):
    import json
    worker = _Worker()
    monkeypatch.setattr(rb.subprocess, "run", worker)
    grid = {"sizes": (70,), "densities": (20, 50), "shapes": ("prefill_b1", "decode_b1"), "sessions": 2, "blocks": 1,
            "window_ms": 10.0}
    assert rb.orchestrate("smoke", tmp_path / "assets", tmp_path / "run", grid=grid) == 0
    cells = [(c["density"], c["shape"]) for c in worker.calls]
    assert len(cells) == 8 and cells[4:] == cells[:4][::-1]          # the second session runs in reverse order
    summary = json.loads((tmp_path / "run" / "summary.json").read_text())
    assert summary["verdict"]["admissible"] and len(summary["cells"]) == 4
    assert all(c["hffn_over_dense"] == pytest.approx(0.5) for c in summary["cells"])
    assert (tmp_path / "run" / "REPORT.md").read_text().count("| 70M |") == 4


def test_orchestrate_stops_at_a_failed_gate(tmp_path, monkeypatch):
    import json
    monkeypatch.setattr(rb.subprocess, "run", _Worker(gate_fails_at=2))
    grid = {"sizes": (70,), "densities": (20,), "shapes": ("prefill_b1", "decode_b1"), "sessions": 1, "blocks": 1,
            "window_ms": 10.0}
    assert rb.orchestrate("smoke", tmp_path / "assets", tmp_path / "run", grid=grid) == 1
    summary = json.loads((tmp_path / "run" / "summary.json").read_text())
    assert summary["failure"]["returncode"] == 4 and not summary["verdict"]["admissible"]
