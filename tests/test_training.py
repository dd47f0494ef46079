"""Training-mode router outputs (softmax probabilities for the regularisers) and the
auxiliary losses of src/openpangu_moe.py:282-307."""
import math

import pytest
import torch

from conftest import oracle, pkg
from gpu_helpers import ulp_diff_bf16


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
