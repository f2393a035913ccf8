"""Reader and writer of the ``hffn_training_compact_g4_v2`` exports (one file per FFN of a model).

The format is the reference's on-disk contract (``runtime/common/pythia/hffn_pythia/export.py:13-57``): a ``torch.save``
dict with ``format``, ``d_model``, ``d_ff`` and, per hidden neuron r, its up slots ``up_idx / up_val[
up_row_offsets[r]:up_row_offsets[r + 1]]`` (int16 / float32, offsets int32), ``b_up`` [d_ff], its down slots
``down_idx / down_val`` over ``down_row_offsets`` and ``b_down`` [d_model]; optionally ``group_hidden_offsets`` (int32[5],
the CPU runtimes' four-group partition). The reader refuses a file whose types, sizes, offsets or indices are
inconsistent, as the reference's does. Files sit at ``<export_dir>/layer<i>/hffn_training_compact_g4_v2.pt``.
"""
from __future__ import annotations

from pathlib import Path

import torch

FORMAT = "hffn_training_compact_g4_v2"
TYPES = {"up_row_offsets": torch.int32, "up_idx": torch.int16, "up_val": torch.float32, "b_up": torch.float32,
         "down_row_offsets": torch.int32, "down_idx": torch.int16, "down_val": torch.float32, "b_down": torch.float32}


def layer_path(export_dir: str | Path, index: int) -> Path:
    return Path(export_dir) / f"layer{index}" / f"{FORMAT}.pt"


def validate(layer: dict, where: str = "layer") -> None:
    d, f = layer["d_model"], layer["d_ff"]
    for name, dtype in TYPES.items():
        if layer[name].dtype != dtype:
            raise ValueError(f"{where}: {name} must be {dtype}")
    if layer["b_up"].numel() != f or layer["b_down"].numel() != d:
        raise ValueError(f"{where}: bias dimensions do not match d_model / d_ff")
    for side in ("up", "down"):
        offsets, index, values = layer[f"{side}_row_offsets"], layer[f"{side}_idx"], layer[f"{side}_val"]
        if offsets.numel() != f + 1 or int(offsets[0]) != 0 or int(offsets[-1]) != values.numel() \
                or index.numel() != values.numel():
            raise ValueError(f"{where}: invalid {side} hidden-major storage")
        if bool((offsets.diff() < 0).any()) or (index.numel() and (int(index.min()) < 0 or int(index.max()) >= d)):
            raise ValueError(f"{where}: invalid {side} offsets or feature index")
    groups = layer.get("group_hidden_offsets")
    if groups is not None and (groups.dtype != torch.int32 or tuple(groups.shape) != (5,) or int(groups[0]) != 0
                               or int(groups[-1]) != f or bool((groups.diff() < 0).any())):
        raise ValueError(f"{where}: invalid group_hidden_offsets")


def read_layer(path: str | Path) -> dict:
    """The validated arrays of one export file as contiguous CPU tensors."""
    raw = torch.load(path, map_location="cpu", weights_only=True)
    if raw.get("format") != FORMAT:
        raise ValueError(f"{path}: expected a {FORMAT} export")
    layer = {"d_model": int(raw["d_model"]), "d_ff": int(raw["d_ff"])}
    for name in TYPES:
        layer[name] = raw[name].contiguous()
    if "group_hidden_offsets" in raw:
        layer["group_hidden_offsets"] = raw["group_hidden_offsets"].contiguous()
    validate(layer, str(path))
    return layer


def read_layers(export_dir: str | Path, count: int) -> list[dict]:
    return [read_layer(layer_path(export_dir, index)) for index in range(count)]


def write_layer(path: str | Path, layer: dict) -> None:
    validate(layer, str(path))
    Path(path).parent.mkdir(parents=True, exist_ok=True)
    record = {"format": FORMAT, "d_model": int(layer["d_model"]), "d_ff": int(layer["d_ff"])}
    record.update({name: layer[name].contiguous() for name in TYPES})
    if "group_hidden_offsets" in layer:
        record["group_hidden_offsets"] = layer["group_hidden_offsets"].contiguous()
    torch.save(record, path)


def hidden_of_slot(layer: dict, side: str) -> torch.Tensor:
    """The hidden neuron owning each compact slot of one side (int64[nnz])."""
    return torch.repeat_interleave(torch.arange(layer["d_ff"]), layer[f"{side}_row_offsets"].diff().long())


def from_compact(compact) -> dict:
    """An export dict from a ``synth.CompactLayer``."""
    t = lambda a: torch.from_numpy(a.copy())  # noqa: E731
    return {"d_model": compact.d_model, "d_ff": compact.d_ff, "up_row_offsets": t(compact.up_offsets),
            "up_idx": t(compact.up_idx), "up_val": t(compact.up_val), "b_up": t(compact.b_up),
            "down_row_offsets": t(compact.down_offsets), "down_idx": t(compact.down_idx),
            "down_val": t(compact.down_val), "b_down": t(compact.b_down),
            "group_hidden_offsets": t(compact.groups)}


def kernel_layer(layer: dict, device=None):
    """The runtime's ``HFFNLayer`` of one export layer (output-major down edges). With a CUDA ``device`` the arrays
    are moved there first and the output-major order is built on the device (no host sort)."""
    from .runtime import HFFNLayer
    names = ("b_up", "up_row_offsets", "up_idx", "up_val", "b_down", "down_row_offsets", "down_idx", "down_val")
    arrays = {k: layer[k] for k in names}
    if device is not None and torch.device(device).type == "cuda":
        arrays = {k: v.to(device) for k, v in arrays.items()}
    return HFFNLayer.from_hidden_major(layer["d_model"], layer["d_ff"], arrays["b_up"], arrays["up_row_offsets"],
                                       arrays["up_idx"], arrays["up_val"], arrays["b_down"], arrays["down_row_offsets"],
                                       arrays["down_idx"], arrays["down_val"])
