"""CPU, gloo, world size 2: the neuron-sharded forward's partition and collectives (hffn_b200.distributed).

Each rank runs its neuron shard through the float64 oracle (standing in for the GPU kernels, which need a B200);
the collectives are the product's. The sum over ranks of the shard outputs must equal the whole layer's output,
for a replicated batch (all-reduce) and for per-rank batches (the gather / reduce-scatter pipeline, and the own-first
schedule's point-to-point exchange at 2 and 3 ranks)."""
import os
import socket
import types

import numpy as np
import pytest
import torch
import torch.multiprocessing as mp

from hffn_b200 import synth
from hffn_b200.distributed import balanced_partition, neuron_partition, shard_hidden_major


def canonical(layer) -> dict:
    t = torch.from_numpy
    return {k: t(getattr(layer, k).copy()) for k in ("b_up", "up_offsets", "up_idx", "up_val", "b_down",
                                                       "down_offsets", "down_idx", "down_val")}


def as_layer(shard: dict):
    return types.SimpleNamespace(d_model=shard["d_model"], d_ff=shard["d_ff"],
                                 **{k: v.numpy() for k, v in shard.items() if isinstance(v, torch.Tensor)})


def test_balanced_partition():
    cost = torch.tensor([5, 1, 1, 1, 9, 0, 0, 3] * 16)
    bounds = balanced_partition(cost, 4)
    assert bounds[0] == 0 and bounds[-1] == cost.numel() and bounds == sorted(bounds)
    assert all(b % 8 == 0 for b in bounds[:-1])
    shares = [int(cost[a:b].sum()) for a, b in zip(bounds, bounds[1:])]
    assert max(shares) - min(shares) <= 2 * 20      # within one granule of cost of each other


@pytest.mark.parametrize("world", [2, 3, 8])
def test_shards_sum_to_layer(world):
    from oracle import forward64
    case = synth.TEST_CASES["irreg_512_2048"]
    layer = synth.make_layer(case)
    arrays = canonical(layer)
    bounds = neuron_partition(arrays, world)
    x = synth.make_input(case, 5)
    total = sum(forward64.forward(as_layer(shard_hidden_major(layer.d_model, arrays, lo, hi, k == 0)), x)
                for k, (lo, hi) in enumerate(zip(bounds, bounds[1:])))
    assert np.allclose(total, forward64.forward(layer, x), rtol=0, atol=1e-12)


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _worker(rank: int, world: int, port: int, results) -> None:
    import torch.distributed as dist

    from hffn_b200.distributed import ShardedFFN
    from oracle import forward64
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        case = synth.TEST_CASES["homog_256_1024"]
        layer = synth.make_layer(case)
        arrays = canonical(layer)
        bounds = neuron_partition(arrays, world)
        shard = as_layer(shard_hidden_major(layer.d_model, arrays, bounds[rank], bounds[rank + 1], rank == 0))
        local = lambda x, out: out.copy_(torch.from_numpy(forward64.forward(shard, x.numpy())))  # noqa: E731
        ffn = ShardedFFN(local, layer.d_model, segments=3)
        x_shared = torch.from_numpy(synth.make_input(case, 6)).double()
        y_rep = ffn.forward_replicated(x_shared)
        x_own = torch.from_numpy(synth.make_input(case, 7 + 100 * rank)[:7]).double()
        y_own = ffn.forward(x_own)
        ok_rep = np.allclose(y_rep.numpy(), forward64.forward(layer, x_shared.numpy()), atol=1e-12, rtol=0)
        ok_own = np.allclose(y_own.numpy(), forward64.forward(layer, x_own.numpy()), atol=1e-12, rtol=0)
        # the own-first schedule (point-to-point exchange, partials summed in rank order), twice: buffers reused
        first = ShardedFFN(local, layer.d_model, schedule="own_first")
        ok_first = True
        for call in range(2):
            x_k = torch.from_numpy(synth.make_input(case, 9 + 100 * rank + call)[:9]).double()
            ok_first &= np.allclose(first.forward(x_k).numpy(), forward64.forward(layer, x_k.numpy()), atol=1e-12,
                                    rtol=0)
        results[rank] = (ok_rep, ok_own, bool(ok_first))
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("world", [2, 3])
def test_gloo_ranks(world):
    ctx = mp.get_context("spawn")
    manager = ctx.Manager()
    results = manager.dict()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(rank, world, port, results)) for rank in range(world)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout=240)
        if p.is_alive():
            p.kill()
    assert all(p.exitcode == 0 for p in procs), [p.exitcode for p in procs]
    assert dict(results) == {rank: (True, True, True) for rank in range(world)}


def test_peer_forward_requires_tensor_cores_and_checks_push():
    """The peer-memory sharded forward refuses a runtime without the tensor-core path and an unknown delivery mode
    before touching the process group (its exchange is exercised on GPUs)."""
    import types

    from hffn_b200.distributed import PeerShardedFFN
    assert callable(getattr(PeerShardedFFN, "forward_many", None))
    with pytest.raises(ValueError):
        PeerShardedFFN(types.SimpleNamespace(tensor_cores=False), 64)
    with pytest.raises(ValueError):
        PeerShardedFFN(types.SimpleNamespace(tensor_cores=True), 64, push="broadcast")


def test_pythia_shard_layers_partition_every_ffn():
    """``pythia.shard_layers``: the ranks' shards of every export layer hold its hidden neurons once each, in order,
    with their own up slots and down edges, and b_down on rank 0 only."""
    from hffn_b200 import export, pythia
    layers = [export.from_compact(synth.make_layer(synth.TEST_CASES[name]))
              for name in ("irreg_512_2048", "homog_512_2048")]
    world = 4
    shards = [pythia.shard_layers(layers, rank, world) for rank in range(world)]
    for index, layer in enumerate(layers):
        parts = [shards[rank][index] for rank in range(world)]
        assert sum(p["d_ff"] for p in parts) == layer["d_ff"]
        assert torch.equal(torch.cat([p["b_up"] for p in parts]), layer["b_up"])
        assert torch.equal(torch.cat([p["up_val"] for p in parts]), layer["up_val"])
        assert torch.equal(torch.cat([p["up_idx"] for p in parts]), layer["up_idx"])
        assert sum(int(p["down_val"].numel()) for p in parts) == layer["down_val"].numel()
        assert torch.equal(parts[0]["b_down"], layer["b_down"])
        assert all(not p["b_down"].any() for p in parts[1:])


def _mlp_worker(rank: int, world: int, port: int, results) -> None:
    import torch.distributed as dist

    from hffn_b200.pythia import ShardedHFFNMLP
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        class Partial:                      # stands in for the rank's shard runtime: partial output = (rank + 1) x
            def forward(self, index, x):
                return x * (rank + 1) + index

        mlp = ShardedHFFNMLP(Partial(), 2, None)
        h = torch.arange(24, dtype=torch.float32).view(2, 3, 4)
        results[rank] = mlp(h)
    finally:
        dist.destroy_process_group()


def test_sharded_mlp_all_reduces_the_partials():
    ctx = mp.get_context("spawn")
    manager = ctx.Manager()
    results = manager.dict()
    port = _free_port()
    procs = [ctx.Process(target=_mlp_worker, args=(rank, 2, port, results)) for rank in range(2)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout=120)
    assert all(p.exitcode == 0 for p in procs)
    h = torch.arange(24, dtype=torch.float32).view(2, 3, 4)
    for rank in range(2):
        assert torch.equal(results[rank], h * 3 + 4)
