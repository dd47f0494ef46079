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
