"""Synthetic PrunePath decoder (config 4 building blocks): CUDA-graph decode matches eager
decode token for token, MoE and dense MLP variants both run."""
import importlib

import pytest
import torch

from conftest import pkg

pytestmark = pytest.mark.gpu


def _dec(mlp, cuda):
    D = importlib.import_module(pkg().__name__ + ".decoder")
    cfg = D.DecoderConfig(layers=2, hidden=256, heads=2, head_dim=128, vocab=1000, experts=16, group=32,
                          max_seq=64, mlp=mlp)
    return D.SyntheticDecoder(cfg, cuda, seed=3, max_batch=4)


@pytest.mark.parametrize("mlp", ["moe", "dense"])
@pytest.mark.parametrize("batch", [1, 4])
def test_graph_decode_matches_eager(cuda, mlp, batch):
    d = _dec(mlp, cuda)
    ids = torch.randint(0, 1000, (batch, 20), generator=torch.Generator().manual_seed(1)).to(cuda)
    t_graph, _, _ = d.generate(ids, 12, use_graph=True)
    t_graph2, _, _ = d.generate(ids, 12, use_graph=True)  # replays the captured graph
    t_eager, _, _ = d.generate(ids, 12, use_graph=False)
    assert torch.equal(t_graph, t_eager) and torch.equal(t_graph2, t_eager)
    assert t_graph.shape == (batch, 12)


def test_decoder_moe_layer_vs_oracle(cuda):
    """One MoE layer inside the decoder, checked against the oracle on the hidden states the
    decoder actually fed it (captured by forward hooks, as the reference's evaluation scripts
    attach hooks to the module, src/evaluation_triton.py:134-170): router logits, selection,
    output, end-to-end masks against the literal reference."""
    import types
    from gpu_helpers import check_against_oracle
    D = importlib.import_module(pkg().__name__ + ".decoder")
    cfg = D.DecoderConfig(layers=2, hidden=1536, heads=12, head_dim=128, vocab=1000, experts=64, group=96,
                          max_seq=64, mlp="moe", tau=0.70)
    d = D.SyntheticDecoder(cfg, cuda, seed=5, max_batch=4)
    m = d.layers[1]["moe"]
    seen = []
    h = m.register_forward_hook(lambda mod, inp, out: seen.append((inp[0].detach().clone(), out.detach().clone())))
    ids = torch.randint(0, 1000, (4, 12), generator=torch.Generator().manual_seed(2)).to(cuda)
    d.generate(ids, 3, use_graph=False)
    h.remove()
    decode_calls = [(x, y) for x, y in seen if x.shape[1] == 1]  # [B, 1, H]: decode steps
    assert decode_calls
    x, y = decode_calls[-1]
    x = x.reshape(-1, 1536)
    lg = torch.empty(x.shape[0], 64, dtype=torch.bfloat16, device=cuda)
    w = torch.empty_like(lg)
    y2 = m.forward_decode(x.contiguous(), logits_out=lg, weights_out=w)
    assert torch.equal(y2, y.reshape(-1, 1536))  # deterministic: the hooked output
    G = 96
    layer = types.SimpleNamespace(gate_w=m.W_gate.t().cpu(), up_w=m.W_up.t().cpu(), down_w=m.W_down.t().cpu(),
                                  router_w=m.router.t().cpu(), experts=64,
                                  experts_id=torch.arange(64 * G) // G)
    check_against_oracle(layer, x.cpu(), 0.70, y2.cpu(), lg.cpu(), w.cpu(), what="decoder layer 1")
