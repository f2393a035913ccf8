"""Pythia (GPT-NeoX) with its FFNs executed by the HFFN runtime: the drop-in of the reference's loader
(``runtime/common/pythia/hffn_pythia/model.py:27-111``, bound by ``runtime/gpu/nvidia/llm/inference/hffn_pythia_cuda/
model.py:11-28``).

``load_pythia(model_dir, export_dir, ffn, device, dtype)`` builds the GPT-NeoX model of ``model_dir/config.json``,
loads every non-FFN tensor of ``model_dir/model.safetensors`` and reads the compact FFNs of ``export_dir``
(``hffn_training_compact_g4_v2``). ``ffn="hffn"``: every ``block.mlp`` is an ``HFFNMLP`` that hands its activations to
one shared ``PreparedRuntime`` (decode-sized calls prepared once; no dense FFN weight is ever allocated); ``ffn="dense"``: the model's own MLP with its
weights set from the export on the support and zero elsewhere (the control arm of the checks). Embeddings,
attention (PyTorch SDPA), LayerNorm, KV cache and head stay PyTorch in both arms. The HFFN arm exposes its runtime
as ``model.hffn_runtime``. ``dtype`` float32 (the reference's only type) or bfloat16.

``make_random_pythia`` writes a seeded random-init checkpoint and seeded synthetic exports of a given architecture
(the benchmark models: no checkpoint is available offline).
"""
from __future__ import annotations

import json
from contextlib import contextmanager
from pathlib import Path

import torch
from torch import nn

from . import export

# Buffers of older GPT-NeoX checkpoints that the model classes rebuild themselves.
_LEGACY = (".attention.bias", ".attention.masked_bias", ".attention.rotary_emb.inv_freq")

PYTHIA_410M = dict(vocab_size=50304, hidden_size=1024, num_hidden_layers=24, num_attention_heads=16,
                   intermediate_size=4096, max_position_embeddings=2048, use_parallel_residual=True,
                   hidden_act="gelu", layer_norm_eps=1e-5, tie_word_embeddings=False)
PYTHIA_1B = dict(PYTHIA_410M, hidden_size=2048, num_hidden_layers=16, num_attention_heads=8, intermediate_size=8192)


class HFFNMLP(nn.Module):
    """Replacement of ``block.mlp``: ``runtime.forward(index, h.view(-1, d))``. Its output is a view of the runtime's
    output buffer, which the block consumes (residual sum) before the next FFN call overwrites it."""

    def __init__(self, runtime, index: int) -> None:
        super().__init__()
        self.runtime, self.index = runtime, index

    def forward(self, hidden_states: torch.Tensor) -> torch.Tensor:
        shape = hidden_states.shape
        return self.runtime.forward(self.index, hidden_states.reshape(-1, shape[-1]).contiguous()).view(shape)


class ShardedHFFNMLP(nn.Module):
    """``block.mlp`` of a neuron-sharded model (one process per GPU, every rank running the same tokens through the
    rest of the model): this rank's shard of the FFN's hidden neurons (``b_down`` on rank 0 only), its partial output
    all-reduced (sum) over ``group``. The output is a view of the runtime's output buffer, consumed by the block
    before the next FFN call overwrites it."""

    def __init__(self, runtime, index: int, group) -> None:
        super().__init__()
        self.runtime, self.index, self.group = runtime, index, group

    def forward(self, hidden_states: torch.Tensor) -> torch.Tensor:
        import torch.distributed as dist
        shape = hidden_states.shape
        y = self.runtime.forward(self.index, hidden_states.reshape(-1, shape[-1]).contiguous())
        dist.all_reduce(y, op=dist.ReduceOp.SUM, group=self.group)
        return y.view(shape)


class TrainableHFFNMLP(nn.Module):
    """Replacement of ``block.mlp`` for training: the layer ``index`` of an ``HFFNTrainRuntime`` as a torch autograd
    function (``HFFNFunction``): gradients flow to the model's other parameters through gx, the FFN's compact
    gradients stay in the training runtime (``model.hffn_train``), whose ``adamw`` updates them."""

    def __init__(self, train, index: int) -> None:
        super().__init__()
        self.train_runtime, self.index = train, index

    def forward(self, hidden_states: torch.Tensor) -> torch.Tensor:
        from .train_runtime import HFFNFunction
        shape = hidden_states.shape
        y = HFFNFunction.apply(hidden_states.reshape(-1, shape[-1]).contiguous(), self.train_runtime, self.index)
        return y.view(shape)


def shard_layers(layers: list[dict], rank: int, world: int) -> list[dict]:
    """This rank's neuron shard of every export layer (hidden ranges balanced by edge count, multiples of 8; down
    edges restricted to the shard; ``b_down`` kept on rank 0 only): canonical hidden-major arrays."""
    from .distributed import neuron_partition, shard_hidden_major
    shards = []
    for layer in layers:
        arrays = {"b_up": layer["b_up"], "up_offsets": layer["up_row_offsets"], "up_idx": layer["up_idx"],
                  "up_val": layer["up_val"], "b_down": layer["b_down"], "down_offsets": layer["down_row_offsets"],
                  "down_idx": layer["down_idx"], "down_val": layer["down_val"]}
        bounds = neuron_partition(arrays, world)
        if bounds[rank + 1] <= bounds[rank]:
            raise ValueError(f"rank {rank} owns no hidden neuron of a layer (d_ff {layer['d_ff']}, {world} ranks)")
        shards.append(shard_hidden_major(layer["d_model"], arrays, bounds[rank], bounds[rank + 1],
                                         with_bias=rank == 0))
    return shards


class _NoFFN(nn.Module):
    """Parameterless stand-in for ``GPTNeoXMLP`` while the HFFN arm is built: no dense FFN is allocated."""

    def __init__(self, config) -> None:
        super().__init__()


@contextmanager
def _without_dense_ffn():
    from transformers.models.gpt_neox import modeling_gpt_neox
    original = modeling_gpt_neox.GPTNeoXMLP
    modeling_gpt_neox.GPTNeoXMLP = _NoFFN
    try:
        yield
    finally:
        modeling_gpt_neox.GPTNeoXMLP = original


@torch.no_grad()
def set_dense_mlp(mlp: nn.Module, layer: dict) -> None:
    """The dense control: the model's own MLP with the export's values on the support, zeros elsewhere."""
    up, down = mlp.dense_h_to_4h, mlp.dense_4h_to_h
    if tuple(up.weight.shape) != (layer["d_ff"], layer["d_model"]):
        raise ValueError("export and model dimensions differ")
    up.weight.zero_()
    up.weight[export.hidden_of_slot(layer, "up"), layer["up_idx"].long()] = layer["up_val"].to(up.weight.dtype)
    up.bias.copy_(layer["b_up"])
    down.weight.zero_()
    down.weight[layer["down_idx"].long(), export.hidden_of_slot(layer, "down")] = layer["down_val"].to(down.weight.dtype)
    down.bias.copy_(layer["b_down"])


@torch.no_grad()
def _load_non_ffn(model: nn.Module, checkpoint: Path) -> None:
    from safetensors import safe_open
    targets = {name: tensor for name, tensor in model.state_dict().items() if ".mlp." not in name}
    with safe_open(str(checkpoint), framework="pt", device="cpu") as source:
        names = [name for name in source.keys() if ".mlp." not in name and (name in targets or not name.endswith(_LEGACY))]
        if set(names) != set(targets):
            raise ValueError(f"checkpoint and model tensors differ: {sorted(set(names) ^ set(targets))}")
        for name in names:
            targets[name].copy_(source.get_tensor(name))


def load_pythia(model_dir: str | Path, export_dir: str | Path, ffn: str, device: str | torch.device = "cuda",
                dtype: torch.dtype = torch.float32, tensor_cores: bool | None = None, group=None,
                trainable: bool = False, **train_options) -> nn.Module:
    """Pythia in eval mode (``dtype``, on ``device``) with its FFNs from ``export_dir``, executed dense or by HFFN.

    ``group`` (a process group of more than one rank, HFFN arm): every FFN neuron-sharded over the group's ranks
    (``ShardedHFFNMLP``), the rest of the model replicated; every rank runs the same tokens and gets the whole
    model's output. ``model.hffn_runtimes`` holds the rank's runtimes (one per distinct shard width).

    ``trainable=True`` (HFFN arm, float32, one GPU): every FFN is a ``TrainableHFFNMLP`` over one
    ``HFFNTrainRuntime`` (``model.hffn_train``; ``train_options``: its lr, betas, eps, weight_decay), the model is in
    train mode and its other parameters require gradients: ``loss.backward()`` leaves the FFNs' compact gradients in
    ``model.hffn_train.gradients(index)``, and ``model.hffn_train.adamw(index)`` applies them. The layers' layouts
    are built on the device."""
    from transformers import AutoConfig, AutoModelForCausalLM
    if ffn not in ("dense", "hffn"):
        raise ValueError("ffn must be 'dense' or 'hffn'")
    config = AutoConfig.from_pretrained(model_dir)
    if ffn == "hffn":
        with _without_dense_ffn():
            model = AutoModelForCausalLM.from_config(config, dtype=torch.float32, attn_implementation="sdpa")
        if any(".mlp." in name for name, _ in model.named_parameters()):
            raise RuntimeError("dense FFN parameters were allocated in the HFFN arm")
    else:
        model = AutoModelForCausalLM.from_config(config, dtype=torch.float32, attn_implementation="sdpa")
    _load_non_ffn(model, Path(model_dir) / "model.safetensors")
    blocks = model.gpt_neox.layers
    layers = export.read_layers(export_dir, len(blocks))
    runtime = None
    if ffn == "dense":
        for block, layer in zip(blocks, layers):
            set_dense_mlp(block.mlp, layer)
    elif trainable:
        if dtype != torch.float32 or (group is not None and _world(group) > 1):
            raise ValueError("trainable HFFN Pythia: float32 on one GPU")
        from .runtime import HFFNRuntime
        from .train_runtime import HFFNTrainRuntime
        runtime = HFFNRuntime([export.kernel_layer(layer, device) for layer in layers], device, dtype,
                              tensor_cores=tensor_cores)
        model.hffn_train = HFFNTrainRuntime(runtime, **train_options)
        for index, block in enumerate(blocks):
            block.mlp = TrainableHFFNMLP(model.hffn_train, index)
    elif group is None or _world(group) == 1:
        from .runtime import PreparedRuntime
        runtime = PreparedRuntime([export.kernel_layer(layer, device) for layer in layers], device, dtype,
                                  tensor_cores=tensor_cores)
        for index, block in enumerate(blocks):
            block.mlp = HFFNMLP(runtime, index)
    else:
        import torch.distributed as dist

        from .runtime import HFFNLayer, PreparedRuntime
        shards = shard_layers(layers, dist.get_rank(group), dist.get_world_size(group))
        by_width: dict = {}
        for index, shard in enumerate(shards):
            by_width.setdefault(shard["d_ff"], []).append(index)
        runtimes = []
        for width, indices in by_width.items():
            kls = [HFFNLayer.from_hidden_major(shards[i]["d_model"], width, shards[i]["b_up"], shards[i]["up_offsets"],
                                               shards[i]["up_idx"], shards[i]["up_val"], shards[i]["b_down"],
                                               shards[i]["down_offsets"], shards[i]["down_idx"], shards[i]["down_val"])
                   for i in indices]
            shard_runtime = PreparedRuntime(kls, device, dtype, tensor_cores=tensor_cores)
            runtimes.append(shard_runtime)
            for local, index in enumerate(indices):
                blocks[index].mlp = ShardedHFFNMLP(shard_runtime, local, group)
        runtime = runtimes[0]
        model.hffn_runtimes = runtimes
    model = model.to(device=device, dtype=dtype)
    model = model.train().requires_grad_(True) if trainable else model.eval().requires_grad_(False)
    model.hffn_runtime = runtime
    if runtime is not None and not hasattr(model, "hffn_runtimes"):
        model.hffn_runtimes = [runtime]
    return model


def _world(group) -> int:
    import torch.distributed as dist
    return dist.get_world_size(group)


def make_random_pythia(model_dir: str | Path, export_dir: str | Path, architecture: dict, support: int,
                       seed: int, bias_std: float = 0.02) -> None:
    """A seeded random-init GPT-NeoX checkpoint (``config.json`` + ``model.safetensors``, non-FFN tensors from the
    model's own initialisation under ``torch.manual_seed(seed)``) and per-layer synthetic exports (support ``support``
    of d_model per neuron on both sides, weights N(0, 1 / sqrt(support)), biases N(0, bias_std); layer l drawn with seed
    ``seed + 100 l`` by the seeded generator)."""
    from safetensors.torch import save_file
    from transformers import GPTNeoXConfig, GPTNeoXForCausalLM

    from . import synth
    model_dir, export_dir = Path(model_dir), Path(export_dir)
    model_dir.mkdir(parents=True, exist_ok=True)
    config = GPTNeoXConfig(**architecture)
    torch.manual_seed(seed)
    with _without_dense_ffn():
        model = GPTNeoXForCausalLM(config)
    config.save_pretrained(model_dir)
    state = {k: v.contiguous() for k, v in model.state_dict().items() if ".mlp." not in k}
    save_file(state, str(model_dir / "model.safetensors"))
    d, f = architecture["hidden_size"], architecture["intermediate_size"]
    for index in range(architecture["num_hidden_layers"]):
        case = synth.Case(f"pythia_layer{index}", d, f, support, support, False, seed + 100 * index, bias_std)
        export.write_layer(export.layer_path(export_dir, index), export.from_compact(synth.make_layer(case)))
    (model_dir / "hffn_random_init.json").write_text(json.dumps({"seed": seed, "support": support,
                                                                 "architecture": architecture}, indent=1))
