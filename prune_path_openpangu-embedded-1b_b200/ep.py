"""Expert-parallel prefill over P GPUs (one process per GPU, torch.distributed / NCCL).

The reference runs on one device only; this is the sharded form of its prefill path
(``TauSparseMoE.forward_prefill``, src/tl_kernel_optimized_Ultimate_PanGU.py:532-604) for
large token counts:

* rank r owns experts ``r, r + P, r + 2P, ...`` (their packed gate/up/down records) and a
  shard of the tokens; the strided assignment spreads popular low-index experts (skewed
  routing) over all ranks instead of piling them on rank 0;
* every rank routes its own tokens (``ppmoe_prefill_route``: tcgen05 router GEMM + selection);
* a token row is sent once to each rank that owns at least one of its selected experts,
  together with its gate weights for that rank's experts: a count exchange
  (``all_to_all_single`` of int64 counts) then the payload ``all_to_all_single`` (bf16 rows,
  bf16 gate weights);
* each rank runs its local experts on the received rows (``ppmoe_prefill_experts``: grouped
  tcgen05 GEMMs) and returns fp32 partial sums with a second ``all_to_all_single``;
* the source adds the partials in rank order (deterministic) and rounds to bf16 once.

Routing and expert compute are injectable so the distributed logic can be exercised on CPU
ranks (gloo) with a CPU stand-in for the kernels.
"""
from __future__ import annotations

from typing import Callable, Optional

import torch
import torch.distributed as dist

from . import _lib
from .tau_moe import TauSparseMoE, _stream_handle

__all__ = ["ExpertParallelMoE", "dispatch_plan", "combine_partials"]


def owned_experts(E: int, world: int, rank: int) -> torch.Tensor:
    """Experts of ``rank`` under the strided assignment: rank, rank + P, ..."""
    return torch.arange(rank, E, world)


def dispatch_plan(weights: torch.Tensor, world: int):
    """Per-destination send lists from gate weights ``[n, E]`` (0 = not selected).

    Returns ``(send_tok [n_send] int64, send_w [n_send, E/P], send_counts [P] int64)``:
    rows grouped by destination rank in rank order, tokens ascending within a destination;
    ``send_w`` holds the row's gate weights for the destination's own experts, in the order
    of ``owned_experts(E, P, destination)``."""
    n, E = weights.shape
    if E % world:
        raise ValueError(f"experts={E} not divisible by world size {world}")
    el = E // world
    wv = weights.view(n, el, world).transpose(1, 2)  # [n, P, E/P]: expert d + P*j at [:, d, j]
    sel = (wv > 0).any(-1)  # [n, P]
    counts = sel.sum(0).to(torch.int64)
    # stable order: destination major, token minor
    dest, tok = torch.nonzero(sel.t(), as_tuple=True)
    send_w = wv[tok, dest]
    return tok, send_w.contiguous(), counts


def combine_partials(back: torch.Tensor, send_tok: torch.Tensor, send_counts, n: int) -> torch.Tensor:
    """Sum fp32 partial rows into their tokens in rank order and round once to bf16.

    On CUDA this is ``ppmoe_ep_combine`` over a ``[P, n]`` row table; elsewhere (CPU ranks in
    tests) destination-by-destination scatters with the same order."""
    if back.is_cuda:
        P = len(send_counts)
        dest = torch.repeat_interleave(torch.arange(P, device=back.device),
                                       torch.as_tensor(send_counts, device=back.device))
        row_of = torch.full((P, n), -1, dtype=torch.int32, device=back.device)
        row_of[dest, send_tok] = torch.arange(back.shape[0], dtype=torch.int32, device=back.device)
        out = torch.empty(n, back.shape[1], dtype=torch.bfloat16, device=back.device)
        _lib.call("ppmoe_ep_combine", back.data_ptr(), row_of.data_ptr(), P, n, back.shape[1], out.data_ptr(),
                  torch.cuda.current_stream(back.device).cuda_stream)
        return out
    acc = torch.zeros(n, back.shape[1], dtype=torch.float32, device=back.device)
    off = 0
    for c in send_counts:
        c = int(c)
        if c:
            acc.index_add_(0, send_tok[off:off + c], back[off:off + c])
        off += c
    return acc.to(torch.bfloat16)


class ExpertParallelMoE:
    """One MoE MLP layer sharded by expert over the ranks of ``group``.

    ``W_gate [H,I]``, ``W_up [H,I]``, ``W_down [I,H]``, ``router [H,E]`` are the reference
    layout buffers (neurons grouped by expert, ``physical_reorder_for_inference``).  Every
    rank keeps the full router and its own slice of experts."""

    def __init__(self, W_gate, W_up, W_down, router, num_experts: int, group_size: int, tau: float,
                 group=None, logit_bias: Optional[torch.Tensor] = None,
                 route_fn: Optional[Callable] = None, expert_fn: Optional[Callable] = None):
        self.group = group
        self.world = dist.get_world_size(group) if dist.is_initialized() else 1
        self.rank = dist.get_rank(group) if dist.is_initialized() else 0
        H = W_gate.shape[0]
        E, G = num_experts, group_size
        if E % self.world:
            raise ValueError(f"experts={E} not divisible by world size {self.world}")
        self.H, self.E, self.G, self.tau = H, E, G, tau
        self.el = E // self.world
        own = owned_experts(E, self.world, self.rank)
        neurons = (own[:, None] * G + torch.arange(G)[None]).reshape(-1).to(W_gate.device if W_gate is not None else "cpu")
        self.route_fn = route_fn
        self.expert_fn = expert_fn
        self.full = self.local = None
        if route_fn is None or expert_fn is None:
            dev = W_gate.device
            self.full = TauSparseMoE(H, E * G, E, G, tau).to(dev)
            self.full.W_gate, self.full.W_up, self.full.W_down, self.full.router = W_gate, W_up, W_down, router
            self.full.logit_bias = logit_bias
            self.local = TauSparseMoE(H, self.el * G, self.el, G, tau).to(dev)
            self.local.W_gate = W_gate[:, neurons].contiguous()
            self.local.W_up = W_up[:, neurons].contiguous()
            self.local.W_down = W_down[neurons].contiguous()
            self.local.router = torch.zeros(H, self.el, dtype=torch.bfloat16, device=dev)
        self.last_stats = {}
        self.profile = False  # record per-phase device times (ms) into last_stats

    # ------------------------------------------------------------------ kernels
    def _route(self, x):
        if self.route_fn is not None:
            return self.route_fn(x)
        m = self.full
        n = x.shape[0]
        w = torch.empty(n, self.E, dtype=torch.bfloat16, device=x.device)
        ws = m.prefill_workspace(n)
        bias = m.logit_bias
        if bias is not None:
            bias = bias.to(device=x.device, dtype=torch.float32).contiguous()
        _lib.call("ppmoe_prefill_route", x.data_ptr(), n, m.packed().data_ptr(), self.H, self.E, self.G,
                  float(self.tau), _lib.ptr(bias), None, w.data_ptr(), ws.data_ptr(), ws.numel(),
                  _stream_handle(x.device))
        return w

    def _experts(self, xr, wr):
        if self.expert_fn is not None:
            return self.expert_fn(xr, wr, owned_experts(self.E, self.world, self.rank))
        n = xr.shape[0]
        out = torch.empty(n, self.H, dtype=torch.float32, device=xr.device)
        if n == 0:
            return out
        m = self.local
        ws = m.prefill_workspace(n)
        _lib.call("ppmoe_prefill_experts", xr.data_ptr(), n, m.packed().data_ptr(), self.H, self.el, self.G,
                  wr.data_ptr(), out.data_ptr(), None, ws.data_ptr(), ws.numel(), _stream_handle(xr.device))
        return out

    # ------------------------------------------------------------------ forward
    def __call__(self, x: torch.Tensor) -> torch.Tensor:
        """``x [n, H]`` bf16 (this rank's tokens) -> ``[n, H]`` bf16."""
        ev = []

        def mark():
            if getattr(self, "profile", False) and x.is_cuda:
                e = torch.cuda.Event(enable_timing=True)
                e.record()
                ev.append(e)
        x = x.to(torch.bfloat16).contiguous()
        n = x.shape[0]
        mark()
        w = self._route(x)
        send_tok, send_w, send_counts = dispatch_plan(w, self.world)
        send_x = x.index_select(0, send_tok)
        mark()
        if self.world == 1:
            recv_x, recv_w, recv_counts = send_x, send_w, send_counts
        else:
            recv_counts = torch.empty_like(send_counts)
            dist.all_to_all_single(recv_counts, send_counts, group=self.group)
            sc, rc = send_counts.tolist(), recv_counts.tolist()
            recv_x = torch.empty(sum(rc), self.H, dtype=x.dtype, device=x.device)
            recv_w = torch.empty(sum(rc), self.el, dtype=send_w.dtype, device=x.device)
            dist.all_to_all_single(recv_x, send_x, rc, sc, group=self.group)
            dist.all_to_all_single(recv_w, send_w, rc, sc, group=self.group)
        mark()
        part = self._experts(recv_x, recv_w)
        mark()
        if self.world == 1:
            back = part
        else:
            back = torch.empty(int(send_counts.sum()), self.H, dtype=torch.float32, device=x.device)
            dist.all_to_all_single(back, part, sc, rc, group=self.group)
        mark()
        y = combine_partials(back, send_tok, send_counts.tolist(), n)
        mark()
        self.last_stats = {"sent_rows": int(send_counts.sum()), "recv_rows": int(recv_x.shape[0])}
        if ev:
            torch.cuda.synchronize()
            names = ["route_plan", "dispatch_a2a", "experts", "combine_a2a", "combine_add"]
            self.last_stats.update({k: ev[i].elapsed_time(ev[i + 1]) for i, k in enumerate(names)})
        return y
