"""GPU, NCCL, 2 and 4 ranks (each skipped with fewer GPUs): the neuron-sharded forward and the data-parallel training
step against one GPU.

Sharded forward (the replicated and the per-rank-batch forms, tensor cores and CUDA cores, and the peer-memory form
on tensor cores) equals the single-GPU runtime's output within the forward tolerance (the partial sums are added in
another order). The data-parallel MSE
step of the ranks gives the gradients (all-reduced mean) and the loss of a single-GPU step on the concatenation of
their batches within float32 tolerance (the update itself is AdamW of those gradients, tested on one GPU)."""
import os
import socket

import numpy as np
import pytest
import torch
import torch.multiprocessing as mp

pytestmark = pytest.mark.gpu


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _kernel_layer(layer):
    from hffn_b200.runtime import HFFNLayer
    t = torch.from_numpy
    return HFFNLayer.from_hidden_major(layer.d_model, layer.d_ff, t(layer.b_up), t(layer.up_offsets), t(layer.up_idx),
                                       t(layer.up_val), t(layer.b_down), t(layer.down_offsets), t(layer.down_idx),
                                       t(layer.down_val))


def _worker(rank: int, world: int, port: int, results) -> None:
    import datetime

    import torch.distributed as dist

    from hffn_b200 import synth
    from hffn_b200.distributed import DataParallelTrainer, sharded_runtime
    from hffn_b200.runtime import HFFNRuntime
    from hffn_b200.train_runtime import HFFNTrainRuntime
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    torch.cuda.set_device(rank)
    device = torch.device("cuda", rank)
    dist.init_process_group("nccl", rank=rank, world_size=world, device_id=device,
                            timeout=datetime.timedelta(seconds=120))
    out = {}
    try:
        case = synth.TEST_CASES["irreg_512_2048"]
        layer = synth.make_layer(case)
        arrays = {k: torch.from_numpy(getattr(layer, k).copy()) for k in
                  ("b_up", "up_offsets", "up_idx", "up_val", "b_down", "down_offsets", "down_idx", "down_val")}
        full = HFFNRuntime([_kernel_layer(layer)], device)
        for tensor_cores in (True, False):
            runtime, ffn, _ = sharded_runtime(layer.d_model, arrays, device, tensor_cores=tensor_cores)
            x_shared = torch.from_numpy(synth.make_input(case, 300)).to(device)
            y_rep = ffn.forward_replicated(x_shared)
            expected = full.forward(0, x_shared).double()
            rel_rep = float(((y_rep.double() - expected).abs() / expected.abs().clamp(min=1)).max())
            x_own = torch.from_numpy(synth.make_input(case, 260 + rank)[:260]).to(device)
            y_own = ffn.forward(x_own)
            expected = full.forward(0, x_own).double()
            rel_own = float(((y_own.double() - expected).abs() / expected.abs().clamp(min=1)).max())
            out[f"sharded_tc{int(tensor_cores)}"] = max(rel_rep, rel_own)
            out[f"errors_tc{int(tensor_cores)}"] = runtime.device_errors()

        # the peer-memory form (tensor cores), both delivery modes: single batches of two sizes, then a stream of
        # five different batches (the pipeline across batches; buffers reused within and across calls)
        worst, errors = 0.0, 0
        for push in ("copy", "store"):
            runtime, peer, _ = sharded_runtime(layer.d_model, arrays, device, tensor_cores=True, transport="peer",
                                               push=push)
            for n_own in (260, 1000):
                x_own = torch.from_numpy(synth.make_input(case, n_own + rank)[:n_own]).to(device)
                expected = full.forward(0, x_own).double()
                for _ in range(2):
                    y_peer = peer.forward(x_own)
                    worst = max(worst, float(((y_peer.double() - expected).abs() / expected.abs().clamp(min=1)).max()))
            xs = [torch.from_numpy(synth.make_input(case, 300 + 7 * k + rank)[:300]).to(device) for k in range(5)]
            for x_k, y_k in zip(xs, peer.forward_many(xs)):
                expected = full.forward(0, x_k).double()
                worst = max(worst, float(((y_k.double() - expected).abs() / expected.abs().clamp(min=1)).max()))
            errors += runtime.device_errors()
        out["sharded_peer"] = worst
        out["errors_peer"] = errors

        # data-parallel training: world x 64 tokens against one GPU on the concatenated tokens
        n = 64
        xs = [synth.make_input(case, world * n)[k * n:(k + 1) * n] for k in range(world)]
        ts = [synth.make_target(case, world * n)[k * n:(k + 1) * n] for k in range(world)]
        dp_train = HFFNTrainRuntime(HFFNRuntime([_kernel_layer(layer)], device, tensor_cores=False), max_tokens=n)
        dp = DataParallelTrainer(dp_train)
        loss = float(dp.step_mse(0, torch.from_numpy(xs[rank]).to(device), torch.from_numpy(ts[rank]).to(device)))
        one = HFFNTrainRuntime(HFFNRuntime([_kernel_layer(layer)], device, tensor_cores=False), max_tokens=world * n)
        loss_one = float(one.step_mse(0, torch.from_numpy(np.concatenate(xs)).to(device),
                                      torch.from_numpy(np.concatenate(ts)).to(device)))
        worst = 0.0
        for name, g in dp_train.gradients(0).items():    # the all-reduced mean gradient against one GPU's
            h = one.gradients(0)[name]
            worst = max(worst, float((g - h).abs().max() / h.abs().max()))
        out["dp_param_rel"] = worst
        out["dp_loss_rel"] = abs(loss - loss_one) / loss_one
        results[rank] = out
    finally:
        dist.barrier()
        dist.destroy_process_group()


@pytest.mark.parametrize("world", [2, 4])
def test_ranks(world):
    if torch.cuda.device_count() < world:
        pytest.skip(f"needs {world} GPUs")
    ctx = mp.get_context("spawn")
    manager = ctx.Manager()
    results = manager.dict()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(rank, world, port, results)) for rank in range(world)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout=300)
        if p.is_alive():
            p.kill()
    assert all(p.exitcode == 0 for p in procs), [p.exitcode for p in procs]
    for rank in range(world):
        r = results[rank]
        assert r["sharded_tc1"] <= 1e-5 and r["sharded_tc0"] <= 1e-5, r
        assert r["errors_tc1"] == 0 and r["errors_tc0"] == 0, r
        assert r["sharded_peer"] <= 1e-5 and r["errors_peer"] == 0, r
        assert r["dp_param_rel"] <= 1e-5 and r["dp_loss_rel"] <= 1e-5, r


def _pythia_worker(rank: int, world: int, port: int, root: str, results) -> None:
    import datetime

    import torch.distributed as dist

    from hffn_b200 import pythia
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    torch.cuda.set_device(rank)
    device = torch.device("cuda", rank)
    dist.init_process_group("nccl", rank=rank, world_size=world, device_id=device,
                            timeout=datetime.timedelta(seconds=120))
    try:
        sharded = pythia.load_pythia(f"{root}/model", f"{root}/export", "hffn", device, group=dist.group.WORLD)
        single = pythia.load_pythia(f"{root}/model", f"{root}/export", "hffn", device)
        ids = torch.randint(0, 2048, (2, 300), generator=torch.Generator().manual_seed(5)).to(device)
        with torch.no_grad():
            a = sharded(input_ids=ids, use_cache=True)
            b = single(input_ids=ids, use_cache=True)
            nxt = b.logits[:, -1:].argmax(-1)
            a2 = sharded(input_ids=nxt, past_key_values=a.past_key_values, use_cache=True)
            b2 = single(input_ids=nxt, past_key_values=b.past_key_values, use_cache=True)
        results[rank] = {
            "prefill": float((a.logits - b.logits).abs().max() / b.logits.abs().max()),
            "decode": float((a2.logits - b2.logits).abs().max() / b2.logits.abs().max()),
            "errors": sum(r.device_errors() for r in sharded.hffn_runtimes)}
    finally:
        dist.barrier()
        dist.destroy_process_group()


@pytest.mark.parametrize("world", [2, 4])
def test_pythia_with_sharded_ffns(world, tmp_path):
    """Every FFN of a small random-init GPT-NeoX neuron-sharded over the ranks (``load_pythia(group=...)``): the
    logits of a 300-token prefill (tensor cores) and of one cached decode step (decode kernels) equal the single-GPU
    HFFN model's within 1e-4 of max|logit| (the partial outputs are summed in another order)."""
    if torch.cuda.device_count() < world:
        pytest.skip(f"needs {world} GPUs")
    from hffn_b200 import pythia
    small = dict(pythia.PYTHIA_410M, hidden_size=256, num_hidden_layers=4, num_attention_heads=4,
                 intermediate_size=1024, vocab_size=2048)
    pythia.make_random_pythia(tmp_path / "model", tmp_path / "export", small, support=128, seed=11)
    ctx = mp.get_context("spawn")
    manager = ctx.Manager()
    results = manager.dict()
    port = _free_port()
    procs = [ctx.Process(target=_pythia_worker, args=(rank, world, port, str(tmp_path), results))
             for rank in range(world)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout=300)
        if p.is_alive():
            p.kill()
    assert all(p.exitcode == 0 for p in procs), [p.exitcode for p in procs]
    for rank in range(world):
        r = results[rank]
        assert r["prefill"] <= 1e-4 and r["decode"] <= 1e-4 and r["errors"] == 0, r
