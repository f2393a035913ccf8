"""Request-level timing of Pythia with HFFN FFNs against the dense model, with an A/A control: the protocol of the
reference's shared harness (``runtime/common/pythia/hffn_pythia/bench_request.py:1-15``, ``:52-61`` for the shapes
and grids, ``:123-176`` for a cell, ``:180-205`` for the verdict), implemented for this runtime.

A cell is one (architecture size, FFN density, request shape) in one fresh process. The process loads three arms
through ``load_pythia``: ``dense``, ``hffn`` and ``hffn_copy`` (a second, independent HFFN runtime), the HFFN arms
reusing the dense model's embedding, attention, norm and head modules so that the arms differ by their FFNs only.
A request is the prompt call followed by the cached decode steps of the shape, fed with the dense arm's greedy
tokens. Gates before any timing: ``hffn_copy``'s logits equal ``hffn``'s bit for bit, and ``hffn`` stays within
``GUARD`` x max|logit| of ``dense``. A window is ``repeats`` back-to-back requests between two synchronisations,
``repeats`` fixed per cell so that a dense window lasts at least ``window_ms``; every timed window follows an
untimed window of the same arm, and the arm order alternates between blocks and between sessions. A run is
admissible when at least ``AA_SHARE`` of the A/A ratios (``hffn_copy / hffn``, one per cell and session) lie within
1 +- ``AA_TOLERANCE``; only then is ``hffn / dense`` read.

Random-init checkpoints and seeded synthetic exports stand in for the reference's Pythia checkpoints and exports (no
checkpoint is available offline): ``make_assets`` writes them; token ids are drawn uniformly from the tokenizer's
range.

    python -m hffn_b200.request_bench --mode smoke|run --assets DIR --out DIR [--sessions N] [--densities 10,50]
    python -m hffn_b200.request_bench --worker '<cell json>'      (one cell; one JSON line on stdout)
"""
from __future__ import annotations

import argparse
import json
import statistics
import subprocess
import sys
import time
from pathlib import Path

ARMS = ("hffn", "dense", "hffn_copy")
SHAPES = {   # batch, prompt tokens, cached decode steps after the prompt call
    "prefill_b1": {"batch": 1, "prompt": 128, "steps": 0},
    "prefill_b4": {"batch": 4, "prompt": 128, "steps": 0},
    "decode_b1": {"batch": 1, "prompt": 32, "steps": 16},
    "decode_b4": {"batch": 4, "prompt": 32, "steps": 16},
}
ARCHITECTURES = {   # GPT-NeoX shapes of the Pythia sizes the grid names (vocabulary 50304, parallel residual)
    70: {"hidden_size": 512, "num_hidden_layers": 6, "num_attention_heads": 8, "intermediate_size": 2048},
    160: {"hidden_size": 768, "num_hidden_layers": 12, "num_attention_heads": 12, "intermediate_size": 3072},
    410: {"hidden_size": 1024, "num_hidden_layers": 24, "num_attention_heads": 16, "intermediate_size": 4096},
}
GRIDS = {
    "run": {"sizes": (70, 160, 410), "densities": (10, 20, 50, 80), "shapes": tuple(SHAPES), "sessions": 3,
            "blocks": 2, "window_ms": 300.0},
    "smoke": {"sizes": (70,), "densities": (20,), "shapes": ("prefill_b1", "decode_b1"), "sessions": 1, "blocks": 1,
              "window_ms": 60.0},
}
GUARD = 1e-3
AA_TOLERANCE, AA_SHARE = 0.03, 0.95
MAX_REPEATS = 200
VOCAB_DRAWN = 50277


def asset_dirs(root: str | Path, size: int, density: int) -> tuple[Path, Path]:
    base = Path(root) / f"pythia{size}m_d{density}"
    return base / "model", base / "export"


def make_assets(root: str | Path, sizes, densities, seed: int = 7, architectures: dict | None = None) -> None:
    """Random-init checkpoints and synthetic exports for every (size, density) (support = density % of d_model)."""
    from .pythia import PYTHIA_410M, make_random_pythia
    architectures = architectures or ARCHITECTURES
    for size in sizes:
        arch = dict(PYTHIA_410M, **architectures[size])
        for density in densities:
            model_dir, export_dir = asset_dirs(root, size, density)
            if (model_dir / "model.safetensors").exists() and (export_dir / "layer0").exists():
                continue
            support = max(1, round(arch["hidden_size"] * density / 100))
            make_random_pythia(model_dir, export_dir, arch, support=support, seed=seed + size)


def share_non_ffn(target, source) -> None:
    """Make ``target`` use ``source``'s modules everywhere but the FFNs (``block.mlp``): one copy of those weights
    in the process, read by every arm."""
    target.embed_out = source.embed_out
    t, s = target.gpt_neox, source.gpt_neox
    t.embed_in, t.final_layer_norm, t.rotary_emb = s.embed_in, s.final_layer_norm, s.rotary_emb
    if len(t.layers) != len(s.layers):
        raise ValueError("the arms have different depths")
    for tb, sb in zip(t.layers, s.layers):
        tb.input_layernorm, tb.post_attention_layernorm, tb.attention = \
            sb.input_layernorm, sb.post_attention_layernorm, sb.attention


def run_cell(cell: dict) -> dict:
    """One cell in this process: gates, then the timed windows of every arm."""
    import torch

    from .pythia import load_pythia
    model_dir, export_dir = asset_dirs(cell["assets"], cell["size"], cell["density"])
    dtype = getattr(torch, cell.get("dtype", "float32"))
    device = cell.get("device", "cuda")
    models = {"dense": load_pythia(model_dir, export_dir, "dense", device, dtype),
              "hffn": load_pythia(model_dir, export_dir, "hffn", device, dtype),
              "hffn_copy": load_pythia(model_dir, export_dir, "hffn", device, dtype)}
    for arm in ("hffn", "hffn_copy"):
        share_non_ffn(models[arm], models["dense"])
    shape = SHAPES[cell["shape"]]
    g = torch.Generator().manual_seed(cell.get("seed", 11))
    prompt = torch.randint(0, VOCAB_DRAWN, (shape["batch"], shape["prompt"]), generator=g).to(device)

    def request(arm, tokens, keep=False):
        model = models[arm]
        out = model(input_ids=prompt, use_cache=True)
        kept = [out.logits[:, -1].clone()] if keep else None
        for token in tokens:
            out = model(input_ids=token, past_key_values=out.past_key_values, use_cache=True)
            if keep:
                kept.append(out.logits[:, -1].clone())
        return kept

    def window(arm, tokens, repeats):
        torch.cuda.synchronize()
        start = time.perf_counter_ns()
        for _ in range(repeats):
            request(arm, tokens)
        torch.cuda.synchronize()
        return (time.perf_counter_ns() - start) / repeats / 1e6

    with torch.inference_mode():
        out = models["dense"](input_ids=prompt, use_cache=True)
        tokens = []
        for _ in range(shape["steps"]):
            tokens.append(out.logits[:, -1:].argmax(-1))
            out = models["dense"](input_ids=tokens[-1], past_key_values=out.past_key_values, use_cache=True)
        del out
        logits = {arm: request(arm, tokens, keep=True) for arm in ARMS}
        bitwise = all(bool(torch.equal(a, b)) for a, b in zip(logits["hffn_copy"], logits["hffn"]))
        scale = max(float(b.abs().max()) for b in logits["dense"])
        gap = max(float((a - b).abs().max()) for a, b in zip(logits["hffn"], logits["dense"])) / scale
        differ = sum(int((a.argmax(-1) != b.argmax(-1)).sum()) for a, b in zip(logits["hffn"], logits["dense"]))
        del logits
        passed = bitwise and gap <= GUARD
        samples, repeats = {arm: [] for arm in ARMS}, None
        if passed:
            for arm in ARMS:
                window(arm, tokens, 2)
            once = min(window("dense", tokens, 1) for _ in range(3))
            repeats = max(1, min(MAX_REPEATS, int(cell["window_ms"] / once) + 1))
            orders = (ARMS + ARMS[::-1], ARMS[::-1] + ARMS)
            for block in range(cell["blocks"]):
                for arm in orders[(cell["parity"] + block) % 2]:
                    window(arm, tokens, repeats)
                    samples[arm].append(window(arm, tokens, repeats))
    runtime = models["hffn"].hffn_runtime
    return {**{k: v for k, v in cell.items() if k != "assets"}, "samples_ms": samples, "repeats": repeats,
            "bitwise_copy": bitwise, "hffn_vs_dense_relative_gap": gap, "argmax_differing_positions": differ,
            "gate_passed": passed, "runtime": {"calls": {f"{u}/{d}": c for (u, d), c in runtime.calls.items()},
                                               "device_errors": runtime.device_errors()}}


def cells_of(grid: dict) -> list[dict]:
    return [{"size": s, "density": d, "shape": shape} for s in grid["sizes"] for d in grid["densities"]
            for shape in grid["shapes"]]


def summarize(rows: list[dict]) -> list[dict]:
    """Per cell over its sessions: median ms per arm, median hffn / dense with its range, the A/A ratios."""
    cells: dict = {}
    for row in rows:
        cells.setdefault((row["size"], row["density"], row["shape"]), []).append(
            {arm: statistics.median(row["samples_ms"][arm]) for arm in ARMS})
    summary = []
    for (size, density, shape), sessions in sorted(cells.items()):
        ratios = [s["hffn"] / s["dense"] for s in sessions]
        summary.append({"size": size, "density": density, "shape": shape, "sessions": len(sessions),
                        "ms": {arm: statistics.median(s[arm] for s in sessions) for arm in ARMS},
                        "hffn_over_dense": statistics.median(ratios), "min": min(ratios), "max": max(ratios),
                        "aa": [s["hffn_copy"] / s["hffn"] for s in sessions]})
    return summary


def verdict(summary: list[dict], complete: bool, gate_passed: bool) -> dict:
    """Admissible when every cell ran, the gates held and at least AA_SHARE of the A/A ratios are within tolerance."""
    if not complete:
        return {"admissible": False, "reason": "incomplete coverage"}
    aa = [a for cell in summary for a in cell["aa"]]
    inside = sum(abs(a - 1) <= AA_TOLERANCE for a in aa)
    return {"admissible": gate_passed and inside >= AA_SHARE * len(aa), "gate_passed": gate_passed,
            "aa_values": len(aa), "aa_within_tolerance": inside, "aa_share": inside / len(aa),
            "aa_median": statistics.median(aa), "aa_min": min(aa), "aa_max": max(aa)}


def orchestrate(mode: str, assets: Path, out: Path, sessions: int | None = None, densities=None,
                grid: dict | None = None, extra: dict | None = None) -> int:
    """Every cell of the grid in its own process, sessions in alternating cell order; writes raw.jsonl,
    summary.json and REPORT.md under ``out``. Returns 0 when every cell ran."""
    grid = dict(grid or GRIDS[mode])
    if sessions:
        grid["sessions"] = sessions
    if densities:
        grid["densities"] = tuple(densities)
    out.mkdir(parents=True, exist_ok=True)
    cells = cells_of(grid)
    (out / "config.json").write_text(json.dumps({"mode": mode, **grid, "arms": ARMS, "shapes": SHAPES, "guard": GUARD,
                                                 "aa_tolerance": AA_TOLERANCE, "aa_share": AA_SHARE}, indent=1) + "\n")
    rows, failure = [], None
    with (out / "raw.jsonl").open("w") as raw:
        for session in range(grid["sessions"]):
            order = list(enumerate(cells)) if session % 2 == 0 else list(enumerate(cells))[::-1]
            for index, cell in order:
                job = {**cell, **(extra or {}), "session": session, "parity": (session + index) % 2,
                       "blocks": grid["blocks"], "window_ms": grid["window_ms"], "assets": str(assets)}
                result = subprocess.run([sys.executable, "-m", "hffn_b200.request_bench", "--worker", json.dumps(job)],
                                        text=True, capture_output=True, cwd=Path(__file__).resolve().parents[1])
                lines = [line for line in result.stdout.splitlines() if line.startswith("{")]
                if result.returncode not in (0, 4) or not lines:
                    failure = {"cell": cell, "session": session, "returncode": result.returncode,
                               "stderr": result.stderr[-4000:]}
                    break
                row = json.loads(lines[-1])
                raw.write(json.dumps(row) + "\n")
                rows.append(row)
                if result.returncode == 4:
                    failure = {"cell": cell, "session": session, "returncode": 4, "gate": {
                        k: row[k] for k in ("bitwise_copy", "hffn_vs_dense_relative_gap")}}
                    break
            if failure:
                break
    complete = len(rows) == len(cells) * grid["sessions"] and failure is None
    summary = summarize(rows) if complete else []
    judged = verdict(summary, complete, failure is None or failure["returncode"] != 4)
    (out / "summary.json").write_text(json.dumps({"cells": summary, "verdict": judged, "failure": failure},
                                                 indent=1) + "\n")
    report = [f"# Request-level timing, {mode}", "", f"{len(rows)} of {len(cells) * grid['sessions']} cell runs.", "",
              "Milliseconds per request; `hffn/dense` is read only when the verdict is admissible.", "",
              "| model | density | shape | dense | hffn | hffn/dense [min-max] | A/A per session |",
              "|---|---:|---|---:|---:|---|---|"]
    for c in summary:
        report.append(f"| {c['size']}M | {c['density']} % | {c['shape']} | {c['ms']['dense']:.3f} | "
                      f"{c['ms']['hffn']:.3f} | {c['hffn_over_dense']:.3f} [{c['min']:.3f}-{c['max']:.3f}] | "
                      + " ".join(f"{a:.3f}" for a in c["aa"]) + " |")
    report += ["", "```json", json.dumps(judged, indent=1), "```"]
    if failure:
        report += ["", "Failure:", "```", json.dumps(failure, indent=1)[:4000], "```"]
    (out / "REPORT.md").write_text("\n".join(report) + "\n")
    print("\n".join(report), flush=True)
    return 0 if complete else 1


def main() -> int:
    parser = argparse.ArgumentParser()
    parser.add_argument("--worker")
    parser.add_argument("--mode", choices=sorted(GRIDS))
    parser.add_argument("--assets", type=Path)
    parser.add_argument("--out", type=Path)
    parser.add_argument("--sessions", type=int)
    parser.add_argument("--densities", type=lambda text: tuple(int(v) for v in text.split(",")))
    parser.add_argument("--dtype", default="float32", choices=("float32", "bfloat16"))
    args = parser.parse_args()
    if args.worker:
        row = run_cell(json.loads(args.worker))
        print(json.dumps(row), flush=True)
        return 0 if row["gate_passed"] else 4
    if not (args.mode and args.assets and args.out):
        parser.error("--mode, --assets and --out are required")
    grid = dict(GRIDS[args.mode])
    make_assets(args.assets, grid["sizes"], args.densities or grid["densities"])
    return orchestrate(args.mode, args.assets, args.out, args.sessions, args.densities, extra={"dtype": args.dtype})


if __name__ == "__main__":
    sys.exit(main())
