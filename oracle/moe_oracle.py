"""CPU oracle for the PrunePath sparse-MoE MLP -- TEST INFRASTRUCTURE ONLY.

Only ``tests/``, ``__graft_entry__.smoke()`` and ``bench.py``'s CPU-baseline / reference arm
may import this module, and only as the checker or the timed CPU baseline.  The product
path (the CUDA library behind ``TauSparseMoE``) never calls into it.

It restates, with the same torch CPU bf16 operators, the reference's dense-then-mask MoE
MLP path, which is the numerics the B200 kernels must reproduce:

* ``softmax_thresholding``  <- ``src/MoEBlock.py:49-95``
* ``MoELayer.forward``      <- ``src/MoEBlock.py:164-208`` (router ``:178``, gate weights
  ``:181-185``, activation counter ``:189-191``, neuron mask ``:200``, masking ``:203``)
* ``IntegratedOpenPanguMoEMLP.forward`` <- ``src/openpangu_moe_origin.py:83-121``
  (``act_fn(gate_proj(x)) * up_proj(x)`` then ``down_proj``)
* ``physical_reorder_for_inference``    <- ``src/openpangu_moe.py:212-256`` (layout only)

Rounding points this implies (every op stores bf16, computes fp32 inside):
``g=bf16(x.Wg)``, ``u=bf16(x.Wu)``, ``s=bf16(silu(g))``, ``a=bf16(s*u)``,
``logit=bf16(x.R)``, ``p=bf16(softmax_fp32(logit))``, ``c_j=bf16(sum_{i<=j} p_sorted_i)``
(sequential fp32), select ``c_j < bf16(tau)`` with a forced top-1,
``w=bf16(sigmoid(logit))`` on selected experts and 0 elsewhere, ``a2=bf16(a*w)``,
``out=bf16(sum a2*Wd)``.

``torch.sort`` on CPU is not stable for 64 elements, so the reference's tie order among
equal bf16 probabilities is implementation-defined.  ``stable=True`` (the default here)
breaks ties by lower expert index, which is the contract the kernels implement and the
one the reference Triton decode kernel also uses (lowest index among equal maxima,
``src/tl_kernel_optimized_Ultimate_PanGU.py:369``).  ``stable=False`` is the literal
reference call.

Parity pin: the functions here are checked bit-for-bit against the reference modules
imported from the reference checkout on golden cases (``tests/golden/make_golden.py``
writes the fixtures, ``tests/test_oracle.py`` replays them).
"""
from __future__ import annotations

from dataclasses import dataclass
from typing import Optional

import torch
import torch.nn.functional as F

__all__ = ["softmax_thresholding", "router_logits", "moe_mlp", "MoEResult",
           "reference_layout", "activation_counts"]

BF16 = torch.bfloat16


def softmax_thresholding(logits: torch.Tensor, tau: float, stable: bool = True):
    """Gate weights and selection mask for bf16 router logits ``[..., E]``.

    Returns ``(w, mask)``: ``w`` bf16 = sigmoid(logit) on selected experts, exactly 0 on
    the rest; ``mask`` bool.  Follows ``src/MoEBlock.py:68-91``.
    """
    shape = logits.shape
    lg = logits.reshape(-1, 1, shape[-1])  # the reference indexes dims (B, L, E)
    y_soft = torch.softmax(lg, dim=-1)
    sorted_prob, sorted_idx = torch.sort(y_soft, dim=-1, descending=True, stable=stable)
    cum_prob = torch.cumsum(sorted_prob, dim=-1)
    keep_sorted = cum_prob < tau
    mask = torch.zeros_like(keep_sorted)
    mask.scatter_(dim=2, index=sorted_idx, src=keep_sorted)
    none = mask.sum(dim=-1) == 0
    if none.any():  # forced top-1 (src/MoEBlock.py:81-86)
        b, l = torch.where(none)
        mask[b, l, sorted_idx[b, l, 0]] = True
    floor = torch.full_like(lg, torch.finfo(lg.dtype).min)
    w = torch.sigmoid(torch.where(mask, lg, floor))
    return w.reshape(shape), mask.reshape(shape)


def router_logits(x: torch.Tensor, router_w: torch.Tensor,
                  bias: Optional[torch.Tensor] = None) -> torch.Tensor:
    """bf16 ``x @ router_w.T`` (``src/MoEBlock.py:178``); optional fp32 prior added then
    rounded to bf16 (an extension for skewed-routing benchmarks; the reference router has
    no bias)."""
    lg = F.linear(x, router_w)
    if bias is not None:
        lg = (lg.float() + bias.float()).to(lg.dtype)
    return lg


@dataclass
class MoEResult:
    out: torch.Tensor  # [..., H] bf16
    logits: torch.Tensor  # [..., E] bf16
    weights: torch.Tensor  # [..., E] bf16 (0 where unselected)
    mask: torch.Tensor  # [..., E] bool


def moe_mlp(x: torch.Tensor, layer, tau: float, stable: bool = True,
            logits: Optional[torch.Tensor] = None,
            bias: Optional[torch.Tensor] = None) -> MoEResult:
    """Dense-then-mask MoE MLP on CPU bf16 (``src/openpangu_moe_origin.py:96-115`` +
    ``src/MoEBlock.py:178-203``).

    ``layer`` is a ``synth.LayerWeights`` (reference ``nn.Linear`` layouts).  ``logits``
    overrides the router output (teacher forcing, to score a kernel's expert computation
    independently of 1-ulp router rounding differences).
    """
    x = x.to(BF16)
    gate = F.silu(F.linear(x, layer.gate_w))
    up = F.linear(x, layer.up_w)
    inter = gate * up
    lg = router_logits(x, layer.router_w, bias) if logits is None else logits.to(BF16)
    w, mask = softmax_thresholding(lg, tau, stable=stable)
    experts_masks = F.one_hot(layer.experts_id, num_classes=layer.experts).t().to(BF16)
    neuron_mask = w @ experts_masks
    out = F.linear(inter * neuron_mask, layer.down_w)
    return MoEResult(out, lg, w, mask)


def activation_counts(weights: torch.Tensor) -> torch.Tensor:
    """Per-expert count of tokens with a positive gate weight (``src/MoEBlock.py:189-191``)."""
    return (weights.reshape(-1, weights.shape[-1]) > 0).long().sum(dim=0)


def reference_layout(layer):
    """The buffers ``physical_reorder_for_inference`` mounts on ``TauSparseMoE``
    (``src/openpangu_moe.py:229-243``): neurons sorted by expert id.

    Returns ``(W_gate [H,I], W_up [H,I], W_down [I,H], router [H,E])`` bf16, contiguous.
    """
    experts_masks = F.one_hot(layer.experts_id, num_classes=layer.experts).t()
    expert_ids = torch.argmax(experts_masks.to(torch.int32), dim=0)
    sort_idx = torch.argsort(expert_ids, stable=True)  # reference: unstable argsort; any
    # within-expert neuron order is equivalent, stable keeps the oracle deterministic
    W_gate = layer.gate_w[sort_idx, :].t().contiguous()
    W_up = layer.up_w[sort_idx, :].t().contiguous()
    W_down = layer.down_w[:, sort_idx].t().contiguous()
    router = layer.router_w.t().contiguous()
    return W_gate, W_up, W_down, router
