"""Seeded synthetic PrunePath MoE-MLP layers (weights, cluster assignment, activations).

The reference ships no dataset or checkpoint for this path, so every test and benchmark
runs on synthetic inputs drawn here.  The recipe is fixed so that the GPU box, the CPU
baseline and the committed golden fixtures all see bit-identical tensors:

* one CPU ``torch.Generator`` seeded with ``seed`` draws, in this order,
  ``gate.weight [I,H]``, ``up.weight [I,H]``, ``down.weight [H,I]``, ``router [E,H]``
  (the ``nn.Linear`` layouts of ``src/openpangu_moe_origin.py:59-62`` and
  ``src/MoEBlock.py:125-127``), each ``N(0,1) * 0.02`` in fp32 then cast to bf16; the
  router is additionally multiplied by ``router_scale`` before the cast so that roughly
  10-30% of experts are active (scale 3.5 at tau 0.95, 1.75 at tau 0.70);
* the same generator then draws a balanced neuron->expert assignment
  (``randperm(I) // G`` scattered, i.e. every expert owns exactly G neurons), the form
  ``MoELayer(experts_id=...)`` accepts (``src/MoEBlock.py:116,138-139``);
* activations come from a second generator seeded with ``seed * 7919 + 17 + stream`` so
  different token batches can be drawn for the same weights: ``N(0,1)`` cast to bf16.

The optional Zipf(alpha) router-logit prior ``b_e = -alpha * ln(e + 1)`` models skewed
routing for the expert-parallel prefill configuration; the reference router has no bias,
so the oracle applies it as ``bf16(logit + b)`` before ``softmax_thresholding``.
"""
from __future__ import annotations

import math
from dataclasses import dataclass

import torch

__all__ = ["LayerWeights", "make_layer", "make_tokens", "zipf_bias", "router_scale_for_tau"]


def router_scale_for_tau(tau: float) -> float:
    """Router weight scale that keeps ~20% of experts active at this tau (seeded measurement)."""
    return 3.5 if tau >= 0.9 else 1.75


@dataclass
class LayerWeights:
    """One MoE MLP layer in the reference's dense (``nn.Linear``) layouts, bf16 on CPU."""

    gate_w: torch.Tensor  # [I, H]  gate_proj.weight
    up_w: torch.Tensor  # [I, H]  up_proj.weight
    down_w: torch.Tensor  # [H, I]  down_proj.weight
    router_w: torch.Tensor  # [E, H]  mlp_router[0].weight
    experts_id: torch.Tensor  # [I] int64, neuron -> expert
    hidden: int
    inter: int
    experts: int
    group: int

    def to(self, device) -> "LayerWeights":
        return LayerWeights(self.gate_w.to(device), self.up_w.to(device), self.down_w.to(device),
                            self.router_w.to(device), self.experts_id.to(device),
                            self.hidden, self.inter, self.experts, self.group)


def make_layer(seed: int, hidden: int = 1536, experts: int = 64, group: int = 96,
               router_scale: float = 1.0, inter: int | None = None) -> LayerWeights:
    inter = experts * group if inter is None else inter
    if inter != experts * group:
        raise ValueError("intermediate size must equal experts * group")
    g = torch.Generator().manual_seed(int(seed))

    def draw(*shape, scale=1.0):
        return (torch.randn(*shape, generator=g, dtype=torch.float32) * (0.02 * scale)).to(torch.bfloat16)

    gate_w = draw(inter, hidden)
    up_w = draw(inter, hidden)
    down_w = draw(hidden, inter)
    router_w = draw(experts, hidden, scale=router_scale)
    perm = torch.randperm(inter, generator=g)
    experts_id = torch.empty(inter, dtype=torch.long)
    experts_id[perm] = torch.arange(inter, dtype=torch.long) // group
    return LayerWeights(gate_w, up_w, down_w, router_w, experts_id, hidden, inter, experts, group)


def make_tokens(seed: int, n: int, hidden: int = 1536, stream: int = 0) -> torch.Tensor:
    """``[n, hidden]`` bf16 activations ~N(0,1)."""
    g = torch.Generator().manual_seed(int(seed) * 7919 + 17 + int(stream))
    return torch.randn(n, hidden, generator=g, dtype=torch.float32).to(torch.bfloat16)


def zipf_bias(experts: int, alpha: float = 1.2) -> torch.Tensor:
    """fp32 ``[E]`` log-prior ``-alpha * ln(e + 1)``: expert 0 is the most popular."""
    return torch.tensor([-alpha * math.log(e + 1.0) for e in range(experts)], dtype=torch.float32)
