"""Real-weight ingestion: checkpoint state_dict + cluster assignment files -> TauSparseMoE layers.

Mirrors the reference's inference preparation of ``CustomOpenPangu``:

* ``load_state_dict(torch.load(checkpoint), strict=False)`` (``src/evaluation_triton.py:524``)
  onto the adapter whose MLPs are ``IntegratedOpenPanguMoEMLP`` (``src/openpangu_moe.py:163-176``),
  i.e. per layer ``i`` the keys ``{prefix}.{i}.mlp.gate_proj.weight [I,H]``,
  ``.up_proj.weight [I,H]``, ``.down_proj.weight [H,I]``,
  ``.moelayer.mlp_router.0.weight [E,H]`` and the buffer ``.moelayer.experts_masks [E,I]``
  (``src/MoEBlock.py:125-143``);
* ``custom_post_init`` (``src/openpangu_moe.py:180-209``): when the masks come from the
  cluster files ``Pangu_Clusters/layer_{i}_k{G}.txt`` (one expert id per neuron, written by
  ``np.savetxt`` as floats), ``mask[j] = (ids == j)``;
* ``physical_reorder_for_inference(tau)`` (``src/openpangu_moe.py:212-256``): neurons grouped
  by expert and mounted on ``tau_moe`` (here :func:`tau_moe.physical_reorder_for_inference`).

A checkpoint saved after the reorder carries ``{prefix}.{i}.mlp.tau_moe.{W_gate, W_up,
W_down, router}`` instead; those are mounted as they are.
"""
from __future__ import annotations

import os
import re
from typing import Dict, List, Mapping, Optional

import numpy as np
import torch

from .tau_moe import TauSparseMoE, physical_reorder_for_inference

__all__ = ["load_cluster_ids", "masks_from_ids", "layer_indices", "moe_layers_from_state_dict"]

DEFAULT_PREFIX = "model.model.layers"


def load_cluster_ids(path: str) -> torch.Tensor:
    """Neuron -> expert ids from a cluster file (``np.loadtxt`` of one float per line, as
    ``custom_post_init`` reads it with ``dtype=np.int32``)."""
    ids = np.loadtxt(path, dtype=np.float64).reshape(-1)
    if not np.all(ids == np.round(ids)) or ids.min() < 0:
        raise ValueError(f"{path}: expert ids must be non-negative integers")
    return torch.from_numpy(ids.astype(np.int64))


def masks_from_ids(ids: torch.Tensor, num_experts: int) -> torch.Tensor:
    """``experts_masks [E, I]`` (bool) with ``mask[j, n] = (ids[n] == j)``."""
    ids = torch.as_tensor(ids, dtype=torch.long)
    if int(ids.max()) >= num_experts:
        raise ValueError(f"expert id {int(ids.max())} out of range for {num_experts} experts")
    return ids.unsqueeze(0) == torch.arange(num_experts, dtype=torch.long).unsqueeze(1)


def layer_indices(state_dict: Mapping[str, torch.Tensor], prefix: str = DEFAULT_PREFIX) -> List[int]:
    """Sorted layer indices that have MLP weights under ``prefix``."""
    pat = re.compile(re.escape(prefix) + r"\.(\d+)\.mlp\.")
    return sorted({int(m.group(1)) for k in state_dict for m in [pat.match(k)] if m})


def _take(sd: Mapping[str, torch.Tensor], key: str) -> Optional[torch.Tensor]:
    t = sd.get(key)
    return None if t is None else t.detach()


def moe_layers_from_state_dict(state_dict: Mapping[str, torch.Tensor], group_size: int, tau: float,
                               device: torch.device | str = "cuda", prefix: str = DEFAULT_PREFIX,
                               cluster_dir: Optional[str] = None,
                               layers: Optional[List[int]] = None) -> Dict[int, TauSparseMoE]:
    """Build one :class:`TauSparseMoE` per layer found in ``state_dict``.

    Expert masks come, in this order, from the checkpoint's ``moelayer.experts_masks`` buffer
    or from ``cluster_dir/layer_{i}_k{group_size}.txt``.  Raises ``KeyError`` naming the first
    missing tensor.  Returns ``{layer index: module}``; on a CUDA device the weights are
    packed for the kernels right away.
    """
    out: Dict[int, TauSparseMoE] = {}
    for i in (layers if layers is not None else layer_indices(state_dict, prefix)):
        base = f"{prefix}.{i}.mlp."
        post = {n: _take(state_dict, base + "tau_moe." + n) for n in ("W_gate", "W_up", "W_down", "router")}
        if all(v is not None for v in post.values()):
            H, I = post["W_gate"].shape
            E = post["router"].shape[1]
            m = TauSparseMoE(H, I, E, group_size, tau).to(device)
            for n, v in post.items():
                getattr(m, n).data = v.to(device=device, dtype=torch.bfloat16).contiguous()
            if torch.device(device).type == "cuda":
                m.packed()
            out[i] = m
            continue
        gate = _take(state_dict, base + "gate_proj.weight")
        up = _take(state_dict, base + "up_proj.weight")
        down = _take(state_dict, base + "down_proj.weight")
        router = _take(state_dict, base + "moelayer.mlp_router.0.weight")
        for name, t in (("gate_proj.weight", gate), ("up_proj.weight", up), ("down_proj.weight", down),
                        ("moelayer.mlp_router.0.weight", router)):
            if t is None:
                raise KeyError(base + name)
        I, H = gate.shape
        E = router.shape[0]
        if I != E * group_size:
            raise ValueError(f"layer {i}: intermediate {I} != experts {E} x group {group_size}")
        masks = _take(state_dict, base + "moelayer.experts_masks")
        if masks is None:
            if cluster_dir is None:
                raise KeyError(base + "moelayer.experts_masks (and no cluster_dir given)")
            masks = masks_from_ids(load_cluster_ids(os.path.join(cluster_dir, f"layer_{i}_k{group_size}.txt")), E)
        m = TauSparseMoE(H, I, E, group_size, tau).to(device)
        physical_reorder_for_inference(m, gate, up, down, router, masks, tau)
        if torch.device(device).type == "cuda":
            m.packed()
        out[i] = m
    return out
