"""Training-mode router outputs (softmax probabilities for the regularisers) and the
auxiliary losses of src/openpangu_moe.py:282-307."""
import math

import pytest
import torch

from conftest import oracle, pkg
from gpu_helpers import assert_selection_matches, ulp_diff_bf16


def _reference_losses(probs_list, mask, E, gamma, lb_gamma):
    """The loop of src/openpangu_moe.py:291-305, written out for the test."""
    ent = lb = 0.0
    valid = mask.sum()
    for p in probs_list:
        p = p.float()
        e = torch.special.entr(p).sum(-1)
        ent += ((e * mask).sum() / (valid + 1e-6) * gamma).item()
        avg = (p * mask.unsqueeze(-1)).reshape(-1, E).sum(0) / (valid + 1e-6)
        lb += ((avg ** 2).sum() * E * lb_gamma).item()
    return ent / len(probs_list), lb / len(probs_list)


def test_aux_losses_known_values_and_mask():
    tr = pkg().training
    E = 8
    uni = torch.full((2, 3, E), 1.0 / E)
    ent, lb = tr.moe_aux_losses([uni], E, gamma=1.0)
    assert abs(ent.item() - math.log(E)) < 1e-5 and abs(lb.item() - 1.0) < 1e-5
    one = torch.zeros(2, 3, E)
    one[..., 0] = 1.0  # every token on expert 0: no entropy, maximal imbalance
    ent, lb = tr.moe_aux_losses([one], E, gamma=1.0, lb_gamma=0.5)
    assert abs(ent.item()) < 1e-6 and abs(lb.item() - 0.5 * E) < 1e-4
    g = torch.Generator().manual_seed(0)
    layers = [torch.softmax(torch.randn(2, 5, E, generator=g), -1).to(torch.bfloat16) for _ in range(3)]
    mask = torch.tensor([[1, 1, 1, 0, 0], [1, 1, 1, 1, 1]], dtype=torch.float32)
    ent, lb = tr.moe_aux_losses(layers, E, gamma=3e-4, lb_gamma=1e-3, attention_mask=mask)
    r_ent, r_lb = _reference_losses(layers, mask, E, 3e-4, 1e-3)
    assert abs(ent.item() - r_ent) <= 1e-9 + 1e-5 * abs(r_ent)
    assert abs(lb.item() - r_lb) <= 1e-9 + 1e-5 * abs(r_lb)
    with pytest.raises(ValueError):
        tr.moe_aux_losses([], E, gamma=1.0)


@pytest.mark.gpu
@pytest.mark.parametrize("E", [16, 64, 192])
def test_route_training_outputs(cuda, E):
    """y_soft equals the oracle's bf16 softmax within 1 ulp (exp implementation); y_gated
    equals the inference selection on the same logits."""
    lib = pkg()._lib
    g = torch.Generator().manual_seed(E)
    lg = (torch.randn(3, 700, E, generator=g) * 2.0).to(torch.bfloat16)
    w, p = pkg().training.route_training(lg.to(cuda), 0.7)
    ref_soft = torch.softmax(lg, dim=-1)  # bf16 CPU softmax, as softmax_thresholding computes it
    assert int(ulp_diff_bf16(p.cpu(), ref_soft).max()) <= 1
    assert (p.cpu() == ref_soft).float().mean().item() > 0.99
    w_inf = torch.empty(2100, E, dtype=torch.bfloat16, device=cuda)
    lib.call("ppmoe_route_logits", lg.to(cuda).data_ptr(), 2100, E, 0.7, w_inf.data_ptr(), None,
             torch.cuda.current_stream().cuda_stream)
    assert torch.equal(w.view(2100, E), w_inf)


@pytest.mark.gpu
def test_training_branch_against_reference_math(cuda):
    """IntegratedOpenPanguMoEMLP in training mode (src/openpangu_moe.py:98-123): the selection
    comes from the GPU kernel, y_gated / y_soft / the masked down projection and the router
    gradient equal the reference's formulas (src/MoEBlock.py:49-95, 164-208) evaluated with
    the oracle's selection on the same bf16 logits."""
    import types
    import torch.nn as nn
    P = pkg()
    H, I, G = 256, 512, 32
    E = I // G
    g = torch.Generator().manual_seed(5)
    mlp = types.SimpleNamespace(gate_proj=nn.Linear(H, I, bias=False), up_proj=nn.Linear(H, I, bias=False),
                                down_proj=nn.Linear(I, H, bias=False), act_fn=nn.SiLU())
    for lin in (mlp.gate_proj, mlp.up_proj, mlp.down_proj):
        lin.weight.data = (torch.randn(lin.weight.shape, generator=g) * 0.05)
    cfg = types.SimpleNamespace(hidden_size=H, intermediate_size=I)
    targs = types.SimpleNamespace(group_size=G, tau=0.7)
    probs = []
    m = P.IntegratedOpenPanguMoEMLP(cfg, targs, mlp, probs)
    m.moelayer.mlp_router[0].weight.data = torch.randn(E, H, generator=g) * 0.2
    m = m.to(device=cuda, dtype=torch.bfloat16).train()
    x = torch.randn(2, 300, H, generator=g).to(torch.bfloat16).to(cuda)
    y = m(x)
    assert len(probs) == 1 and probs[0].shape == (2, 300, E)
    y.float().square().mean().backward()
    gr = m.moelayer.mlp_router[0].weight.grad.clone()

    # the reference formulas with the oracle's selection
    W = m.moelayer.mlp_router[0].weight.detach().clone().requires_grad_(True)
    score = torch.nn.functional.linear(x, W)
    w_k, _ = pkg().training.route_training(score.detach(), 0.7)
    assert_selection_matches(w_k.cpu().reshape(-1, E), score.detach().cpu().reshape(-1, E), 0.7, "training mask")
    sel = w_k > 0
    y_g = torch.sigmoid(torch.where(sel, score, torch.full_like(score, torch.finfo(score.dtype).min)))
    inter = m.act_fn(m.gate_proj(x)) * m.up_proj(x)
    y_ref = m.down_proj(inter * (y_g @ m.moelayer.experts_masks))
    assert torch.equal(y.detach(), y_ref.detach())
    assert torch.equal(probs[0].detach(), torch.softmax(score.detach(), -1))
    y_ref.float().square().mean().backward()
    assert torch.allclose(gr.float(), W.grad.float(), rtol=1e-2, atol=1e-6)
    # eval mode goes through the fused path and records nothing
    m.eval()
    assert len(probs) == 1
