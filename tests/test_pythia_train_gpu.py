"""GPU: a Pythia model trained end to end with its FFNs executed by HFFN (``load_pythia(..., trainable=True)``).

Every FFN is an autograd function over the training runtime (its forward keeps the call's own activations, its
backward runs ``hffn_backward``), so ``loss.backward()`` through the whole model gives: gradients of the attention,
embedding and LayerNorm parameters equal to those of the dense arm (the model's own MLP holding the export's values on
the support, zero elsewhere, float32 autograd) within 1e-4 of their scale, and the FFNs' compact gradients equal to
the dense arm's weight gradients read on the supports. Then a few steps (the FFNs' compact AdamW, torch's AdamW for the
other parameters) lower the loss on a fixed batch.
"""
import pytest
import torch
import torch.nn.functional as F

from hffn_b200 import export, pythia

pytestmark = pytest.mark.gpu

SMALL = dict(pythia.PYTHIA_410M, hidden_size=128, num_hidden_layers=2, num_attention_heads=4, intermediate_size=512,
             vocab_size=1024, max_position_embeddings=128)
TOLERANCE = 1e-4


@pytest.fixture(scope="module")
def tiny(tmp_path_factory):
    root = tmp_path_factory.mktemp("pythia_train")
    pythia.make_random_pythia(root / "model", root / "export", SMALL, support=64, seed=21)
    return root


def batch():
    return torch.randint(0, SMALL["vocab_size"], (2, 24), generator=torch.Generator().manual_seed(5)).cuda()


def lm_loss(model, ids):
    logits = model(input_ids=ids).logits
    return F.cross_entropy(logits[:, :-1].reshape(-1, logits.shape[-1]), ids[:, 1:].reshape(-1))


def relative(a: torch.Tensor, b: torch.Tensor) -> float:
    return float((a.double() - b.double()).abs().max() / max(float(b.double().abs().max()), 1e-30))


def test_gradients_match_dense_arm(tiny):
    hffn = pythia.load_pythia(tiny / "model", tiny / "export", "hffn", "cuda", trainable=True)
    dense = pythia.load_pythia(tiny / "model", tiny / "export", "dense", "cuda").train().requires_grad_(True)
    ids = batch()
    loss_h, loss_d = lm_loss(hffn, ids), lm_loss(dense, ids)
    assert abs(float(loss_h.detach()) - float(loss_d.detach())) <= 1e-5 * abs(float(loss_d.detach()))
    loss_h.backward()
    loss_d.backward()
    named_d = dict(dense.named_parameters())
    compared = 0
    for name, p in hffn.named_parameters():
        assert ".mlp." not in name
        assert relative(p.grad, named_d[name].grad) <= TOLERANCE, name
        compared += 1
    assert compared > 10
    layers = export.read_layers(tiny / "export", SMALL["num_hidden_layers"])
    train = hffn.hffn_train
    for index, (block, layer) in enumerate(zip(dense.gpt_neox.layers, layers)):
        grads = train.gradients(index)
        kl = train.runtime.layers[index]
        up_owner = torch.repeat_interleave(torch.arange(layer["d_ff"]), layer["up_row_offsets"].diff().long()).cuda()
        g_up = block.mlp.dense_h_to_4h.weight.grad[up_owner, layer["up_idx"].long().cuda()]
        out_owner = torch.repeat_interleave(torch.arange(layer["d_model"]).cuda(), kl.out_offsets.diff().long())
        g_down = block.mlp.dense_4h_to_h.weight.grad[out_owner, kl.out_hidden.long()]
        assert relative(grads["up_val"], g_up) <= TOLERANCE, index
        assert relative(grads["b_up"], block.mlp.dense_h_to_4h.bias.grad) <= TOLERANCE, index
        assert relative(grads["out_val"], g_down) <= TOLERANCE, index
        assert relative(grads["b_down"], block.mlp.dense_4h_to_h.bias.grad) <= TOLERANCE, index
    assert train.runtime.device_errors() == 0


def test_training_steps_lower_the_loss(tiny):
    hffn = pythia.load_pythia(tiny / "model", tiny / "export", "hffn", "cuda", trainable=True, lr=1e-3)
    optimizer = torch.optim.AdamW(hffn.parameters(), lr=1e-3)
    ids = batch()
    losses = []
    for _ in range(6):
        optimizer.zero_grad()
        loss = lm_loss(hffn, ids)
        loss.backward()
        optimizer.step()
        for index in range(SMALL["num_hidden_layers"]):
            hffn.hffn_train.adamw(index)
        losses.append(float(loss.detach()))
    assert losses[-1] < losses[0] - 0.05, losses
    assert all(s == 6 for s in hffn.hffn_train.steps)
