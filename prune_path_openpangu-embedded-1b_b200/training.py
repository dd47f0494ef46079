"""Training-mode outputs of the router: the softmax probabilities and the auxiliary losses.

In training mode the reference's ``softmax_thresholding`` returns, besides the gate weights,
``y_soft = softmax(logits)`` (``src/MoEBlock.py:68, 93-94``); ``MoELayer`` hands it up
(``src/MoEBlock.py:205-208``) and ``CustomOpenPangu.forward`` turns the collected tensors into
an entropy regulariser and a load-balance term (``src/openpangu_moe.py:282-307``).

:func:`route_training` produces both router outputs on the GPU (``ppmoe_route_logits_train``:
the probabilities are exactly the ones the selection ranked).  :func:`moe_aux_losses` is the
host-side loss arithmetic, restated from the reference.
"""
from __future__ import annotations

from typing import Iterable, Optional, Tuple

import torch

import torch.nn as nn
import torch.nn.functional as F

from . import _lib

__all__ = ["route_training", "moe_aux_losses", "TrainingMoELayer"]


def route_training(logits: torch.Tensor, tau: float) -> Tuple[torch.Tensor, torch.Tensor]:
    """``softmax_thresholding(logits, tau, training=True)`` on the GPU.

    ``logits [..., E]`` bf16 on a CUDA device -> ``(y_gated, y_soft)``, both bf16 of the same
    shape: sigmoid(logit) on the selected experts (0 elsewhere) and the softmax probabilities.
    """
    if not logits.is_cuda:
        raise RuntimeError("route_training runs on CUDA only")
    shape = logits.shape
    E = shape[-1]
    lg = logits.reshape(-1, E).to(torch.bfloat16).contiguous()
    n = lg.shape[0]
    w = torch.empty_like(lg)
    p = torch.empty_like(lg)
    _lib.call("ppmoe_route_logits_train", lg.data_ptr(), n, E, float(tau), w.data_ptr(), None, p.data_ptr(),
              torch.cuda.current_stream(lg.device).cuda_stream)
    return w.view(shape), p.view(shape)


def moe_aux_losses(probs_list: Iterable[torch.Tensor], num_experts: int, gamma: float,
                   lb_gamma: Optional[float] = None,
                   attention_mask: Optional[torch.Tensor] = None) -> Tuple[torch.Tensor, torch.Tensor]:
    """Entropy regulariser and load-balance loss over the recorded layers
    (``src/openpangu_moe.py:282-307``).

    ``probs_list``: one ``[B, L, E]`` softmax tensor per layer (``y_soft``); ``attention_mask``
    ``[B, L]`` (1 = valid token; all ones if omitted).  Per layer: the masked mean token
    entropy times ``gamma`` and ``E * sum_e(mean_prob_e^2)`` times ``lb_gamma`` (default
    ``gamma``, as in the reference); both averaged over the layers.  Returns
    ``(entropy_loss, load_balance_loss)`` as fp32 scalars.
    """
    probs_list = list(probs_list)
    if not probs_list:
        raise ValueError("no router probabilities recorded")
    lb_gamma = gamma if lb_gamma is None else lb_gamma
    dev = probs_list[0].device
    ent = torch.zeros((), dtype=torch.float32, device=dev)
    lb = torch.zeros((), dtype=torch.float32, device=dev)
    eps = 1e-6
    for probs in probs_list:
        pf = probs.float()
        mask = (torch.ones(pf.shape[:-1], dtype=torch.float32, device=dev) if attention_mask is None
                else attention_mask.to(device=dev, dtype=torch.float32))
        valid = mask.sum()
        entropy = torch.special.entr(pf).sum(dim=-1)
        ent = ent + (entropy * mask).sum() / (valid + eps) * gamma
        avg = (pf * mask.unsqueeze(-1)).reshape(-1, num_experts).sum(dim=0) / (valid + eps)
        lb = lb + (avg ** 2).sum() * num_experts * lb_gamma
    n = len(probs_list)
    return ent / n, lb / n


class TrainingMoELayer(nn.Module):
    """Training-mode router and neuron mask of one MLP (``MoELayer``, src/MoEBlock.py:105-208).

    Same parameters and buffers as the reference, so checkpoints load by key:
    ``mlp_router.0.weight [E, H]`` (zero-initialised, ``router_weights_init``),
    ``experts_masks [E, I]`` (neuron -> expert one-hot; contiguous groups when ``experts_id``
    is None) and ``activated_statistics [E]``.

    ``forward(hidden_states, intermediate) -> (intermediate * (y_gated @ experts_masks), y_soft)``
    in training mode.  The selection (softmax, descending sort, cumulative mass < tau, top-1
    guard) runs on the GPU (``ppmoe_route_logits_train``) on the detached bf16 router logits;
    the differentiable outputs are then formed with autograd from the same logits:
    ``y_gated = sigmoid(where(selected, logits, finfo.min))`` and ``y_soft = softmax(logits)``
    (src/MoEBlock.py:68, 89-94), so gradients reach the router as in the reference.  In eval
    mode it updates ``activated_statistics`` and returns ``(masked intermediate, None)``."""

    def __init__(self, hidden_size: int, intermediate_size: int, experts: int, tau: float = 0.95,
                 experts_id: Optional[torch.Tensor] = None):
        super().__init__()
        if intermediate_size % experts:
            raise ValueError(f"intermediate_size={intermediate_size} not divisible by experts={experts}")
        self.experts, self.tau = experts, tau
        self.mlp_router = nn.Sequential(nn.Linear(hidden_size, experts, bias=False))
        nn.init.zeros_(self.mlp_router[0].weight)
        if experts_id is None:
            experts_id = torch.arange(intermediate_size) // (intermediate_size // experts)
        masks = F.one_hot(torch.as_tensor(experts_id, dtype=torch.long), num_classes=experts).t()
        self.register_buffer("experts_masks", masks.to(self.mlp_router[0].weight.dtype))
        self.register_buffer("activated_statistics", torch.zeros(experts, dtype=torch.long))

    def forward(self, hidden_states: torch.Tensor, intermediate: torch.Tensor):
        score = self.mlp_router(hidden_states)
        with torch.no_grad():
            y_sel, _ = route_training(score.detach(), self.tau)
        selected = y_sel > 0
        y_gated = torch.sigmoid(torch.where(selected, score, torch.full_like(score, torch.finfo(score.dtype).min)))
        if not self.training:
            self.activated_statistics.add_(selected.reshape(-1, self.experts).long().sum(0))
        out = intermediate * (y_gated @ self.experts_masks.to(y_gated.dtype))
        if not self.training:
            return out, None
        return out, torch.softmax(score, dim=-1)
