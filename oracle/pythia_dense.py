"""TEST INFRASTRUCTURE ONLY. The dense arm of the Pythia checks and the reference's token-parity criterion.

``dense_pythia`` restates the reference's dense arm (``runtime/common/pythia/hffn_pythia/model.py:39-61`` and
``:82-111`` with ``ffn="dense"``): the GPT-NeoX model of ``config.json`` with every tensor of ``model.safetensors``
and, per FFN, the model's own MLP whose weights carry the export's values on the support and zero elsewhere. It is
built here independently of the product's loader (numpy scatter of the export into the dense matrices).

``check_arm`` restates the criterion of ``runtime/common/pythia/hffn_pythia/parity_model.py:1-21,86-126``: every
HFFN token equals the dense control's token or, failing that, the float64 arbiter's, or, failing that, its float64
margin (arbiter's logit of its token minus that of the chosen token) is within the larger of one float32 step and
the dense control's own error at that position; the arbiter drives a cached greedy decode that all arms follow.
"""
from __future__ import annotations

from pathlib import Path

import numpy as np
import torch

DECODE_STEPS = 16


def dense_pythia(model_dir: str | Path, export_dir: str | Path, device, dtype=torch.float32):
    from safetensors.torch import load_file
    from transformers import AutoConfig, AutoModelForCausalLM
    config = AutoConfig.from_pretrained(model_dir)
    model = AutoModelForCausalLM.from_config(config, dtype=torch.float32, attn_implementation="sdpa")
    state = load_file(str(Path(model_dir) / "model.safetensors"))
    for index, block in enumerate(model.gpt_neox.layers):
        raw = torch.load(Path(export_dir) / f"layer{index}" / "hffn_training_compact_g4_v2.pt", weights_only=True)
        d, f = int(raw["d_model"]), int(raw["d_ff"])
        w_up = np.zeros((f, d), np.float32)
        w_dn = np.zeros((d, f), np.float32)
        up_owner = np.repeat(np.arange(f), np.diff(raw["up_row_offsets"].numpy()))
        dn_owner = np.repeat(np.arange(f), np.diff(raw["down_row_offsets"].numpy()))
        w_up[up_owner, raw["up_idx"].numpy().astype(np.int64)] = raw["up_val"].numpy()
        w_dn[raw["down_idx"].numpy().astype(np.int64), dn_owner] = raw["down_val"].numpy()
        prefix = f"gpt_neox.layers.{index}.mlp."
        state[prefix + "dense_h_to_4h.weight"] = torch.from_numpy(w_up)
        state[prefix + "dense_h_to_4h.bias"] = raw["b_up"]
        state[prefix + "dense_4h_to_h.weight"] = torch.from_numpy(w_dn)
        state[prefix + "dense_4h_to_h.bias"] = raw["b_down"]
    missing, unexpected = model.load_state_dict(state, strict=False)
    if [k for k in missing if not k.endswith("inv_freq")] or unexpected:
        raise ValueError(f"dense arm: missing {missing}, unexpected {unexpected}")
    return model.to(device=device, dtype=dtype).eval().requires_grad_(False)


@torch.inference_mode()
def all_logits(models: list, prompt: torch.Tensor, steps: int = DECODE_STEPS) -> list[torch.Tensor]:
    """Per model its logits [B, T + steps, vocabulary] (float64); ``models[-1]`` (the arbiter) drives the decode."""
    outputs = [model(input_ids=prompt, use_cache=True) for model in models]
    kept = [[o.logits.double()] for o in outputs]
    for _ in range(steps):
        fed = outputs[-1].logits[:, -1:].argmax(-1)
        outputs = [model(input_ids=fed, past_key_values=o.past_key_values, use_cache=True)
                   for model, o in zip(models, outputs)]
        for k, o in zip(kept, outputs):
            k.append(o.logits.double())
    return [torch.cat(k, dim=1) for k in kept]


def float32_step(value: torch.Tensor) -> torch.Tensor:
    magnitude = value.abs().float()
    return (torch.nextafter(magnitude, torch.full_like(magnitude, float("inf"))) - magnitude).double()


def check_arm(dense, hffn, arbiter, prompts, steps: int = DECODE_STEPS, band: str = "pointwise") -> dict:
    """Counts over all prompts: tokens, HFFN != dense, unexplained (the criterion's failures).

    ``band="pointwise"`` is the reference's criterion (the control's error at the same position). ``band="global"``
    uses the control's largest error over all positions of the prompt instead: the form of the criterion for
    bfloat16 arms, whose rounding noise (~2^-8 relative) makes the two arms' errors at one near-tie position
    independent draws of the same size (still set by the control alone, no free constant)."""
    total = differs_total = unexplained = 0
    for prompt in prompts:
        dense_l, hffn_l, arb_l = all_logits([dense, hffn, arbiter], prompt, steps)
        dense_t, hffn_t, arb_t = dense_l.argmax(-1), hffn_l.argmax(-1), arb_l.argmax(-1)
        differs = hffn_t != dense_t
        moved = differs & (hffn_t != arb_t)
        best = arb_l.gather(-1, arb_t.unsqueeze(-1)).squeeze(-1)
        chosen = arb_l.gather(-1, hffn_t.unsqueeze(-1)).squeeze(-1)
        control = ((dense_l.gather(-1, arb_t.unsqueeze(-1)).squeeze(-1) - best).abs()
                   + (dense_l.gather(-1, hffn_t.unsqueeze(-1)).squeeze(-1) - chosen).abs())
        if band == "global":
            control = torch.full_like(control, float(control.max()))
        band_value = torch.maximum(float32_step(best).to(best.device), control)
        unexplained += int((moved & (best - chosen > band_value)).sum())
        differs_total += int(differs.sum())
        total += hffn_t.numel()
    return {"tokens": total, "differs": differs_total, "unexplained": unexplained}
