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

from . import _lib

__all__ = ["route_training", "moe_aux_losses"]


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
