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
  tcgen05 GEMMs) and returns fp32 partial sums with a second ``all_to_all_single`` (or bf16
  partials in the optional reduced-traffic mode, ``partials="bf16"``);
* the source adds the partials in rank order (deterministic) and rounds to bf16 once;
* the tokens go through in chunks so that the all-to-all transfers of one chunk overlap the
  grouped GEMMs of its neighbours (see ``ExpertParallelMoE.__call__``).

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


def plan_counts(weights: torch.Tensor, world: int):
    """Device-side half of the dispatch plan: ``sel [n, P]`` (token goes to destination) and
    ``counts [P]`` int64 from gate weights ``[n, E]`` (0 = not selected).  No host sync."""
    n, E = weights.shape
    if E % world:
        raise ValueError(f"experts={E} not divisible by world size {world}")
    wv = weights.view(n, E // world, world).transpose(1, 2)  # [n, P, E/P]: expert d + P*j at [:, d, j]
    sel = (wv > 0).any(-1)
    return sel, sel.sum(0).to(torch.int64)


def plan_lists(weights: torch.Tensor, sel: torch.Tensor, counts_host, world: int):
    """Send lists for the counts already known on the host (no further host sync): rows
    grouped by destination rank in rank order, tokens ascending within a destination.
    Returns ``(send_tok [total] int64, send_w [total, E/P], row_of [P, n] int32)``; ``send_w``
    holds each row's gate weights for the destination's own experts, in ``owned_experts``
    order; ``row_of[d, t]`` is the row of (token t, destination d), -1 if t is not sent to d."""
    n, E = weights.shape
    el = E // world
    total = int(sum(counts_host))
    wv = weights.view(n, el, world).transpose(1, 2)
    nz = torch.nonzero_static(sel.t(), size=total)  # destination-major, token-minor
    dest, send_tok = nz[:, 0], nz[:, 1]
    send_w = wv[send_tok, dest]
    row_of = torch.full((world, n), -1, dtype=torch.int32, device=weights.device)
    row_of[dest, send_tok] = torch.arange(total, dtype=torch.int32, device=weights.device)
    return send_tok, send_w.contiguous(), row_of


def dispatch_plan(weights: torch.Tensor, world: int):
    """Per-destination send lists from gate weights ``[n, E]`` (0 = not selected).

    Returns ``(send_tok [n_send] int64, send_w [n_send, E/P], send_counts [P] int64)`` as
    :func:`plan_lists` orders them (one host read of the counts)."""
    sel, counts = plan_counts(weights, world)
    tok, sw, _ = plan_lists(weights, sel, counts.tolist(), world)
    return tok, sw, counts


def combine_partials(back: torch.Tensor, send_tok: torch.Tensor, send_counts, n: int,
                     row_of: Optional[torch.Tensor] = None) -> torch.Tensor:
    """Sum fp32 partial rows into their tokens in rank order and round once to bf16.

    On CUDA this is ``ppmoe_ep_combine`` over the ``[P, n]`` row table (from
    :func:`plan_lists`, or built here); elsewhere (CPU ranks in tests)
    destination-by-destination scatters with the same order."""
    if back.is_cuda:
        P = len(send_counts)
        if row_of is None:
            dest = torch.repeat_interleave(torch.arange(P, device=back.device),
                                           torch.as_tensor(send_counts, device=back.device))
            row_of = torch.full((P, n), -1, dtype=torch.int32, device=back.device)
            row_of[dest, send_tok] = torch.arange(back.shape[0], dtype=torch.int32, device=back.device)
        out = torch.empty(n, back.shape[1], dtype=torch.bfloat16, device=back.device)
        fn = "ppmoe_ep_combine_bf16" if back.dtype == torch.bfloat16 else "ppmoe_ep_combine"
        _lib.call(fn, back.data_ptr(), row_of.data_ptr(), P, n, back.shape[1], out.data_ptr(),
                  torch.cuda.current_stream(back.device).cuda_stream)
        return out
    acc = torch.zeros(n, back.shape[1], dtype=torch.float32, device=back.device)
    off = 0
    for c in send_counts:
        c = int(c)
        if c:
            acc.index_add_(0, send_tok[off:off + c], back[off:off + c].float())
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
        self.local = None
        self.router_rows = None
        self.logit_bias = logit_bias
        self._route_ws = None
        if route_fn is None or expert_fn is None:
            dev = W_gate.device
            # routing reads only the router section of a packed blob (router_eh [E][H]): keep
            # just those rows, not a second copy of every expert's weights
            buf = torch.empty(E * H * 2 + 1024, dtype=torch.uint8, device=dev)
            off = (-buf.data_ptr()) % 1024
            self.router_rows = buf[off:off + E * H * 2]
            self.router_rows.view(torch.bfloat16).view(E, H).copy_(router.t())
            self.local = TauSparseMoE(H, self.el * G, self.el, G, tau).to(dev)
            self.local.W_gate = W_gate[:, neurons].contiguous()
            self.local.W_up = W_up[:, neurons].contiguous()
            self.local.W_down = W_down[neurons].contiguous()
            self.local.router = torch.zeros(H, self.el, dtype=torch.bfloat16, device=dev)
        self.last_stats = {}
        self.profile = False  # record per-phase device times (ms) into last_stats
        self.chunks = 2 if self.world > 1 else 1  # pipeline depth (measured best at 2 on 2 GPUs)
        # "fp32": partial sums cross the network in fp32 and the only bf16 rounding is the final
        # one (the single-device numerics).  "bf16": each rank rounds its partial once before
        # sending (half the combine traffic, a second rounding: looser tolerance).
        self.partials = "fp32"

    # ------------------------------------------------------------------ kernels
    def _route(self, x):
        if self.route_fn is not None:
            return self.route_fn(x)
        n = x.shape[0]
        w = torch.empty(n, self.E, dtype=torch.bfloat16, device=x.device)
        nbytes = _lib.load().ppmoe_route_workspace_bytes(n, self.H, self.E, self.G)
        if self._route_ws is None or self._route_ws.numel() < nbytes:
            buf = torch.empty(nbytes + 1024, dtype=torch.uint8, device=x.device)
            self._route_ws = buf[(-buf.data_ptr()) % 1024:][:nbytes]
        ws = self._route_ws
        bias = self.logit_bias
        if bias is not None:
            bias = bias.to(device=x.device, dtype=torch.float32).contiguous()
        _lib.call("ppmoe_prefill_route", x.data_ptr(), n, self.router_rows.data_ptr(), self.H, self.E, self.G,
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
        """``x [n, H]`` bf16 (this rank's tokens) -> ``[n, H]`` bf16.

        The tokens are processed in ``self.chunks`` consecutive chunks (default 2 on more than
        one rank).  One routing call covers all of them, and one count exchange carries every
        chunk's per-destination counts (the only host synchronisation).  Then every chunk's
        dispatch all-to-all is enqueued asynchronously; chunk c's expert GEMMs wait only for
        its own rows, and its combine all-to-all is enqueued right after them.  NCCL transfers
        of neighbouring chunks therefore run under the grouped GEMMs.  Each token's partials
        live in exactly one chunk, so the result equals the unchunked path bit for bit."""
        ev = []

        def mark():
            if getattr(self, "profile", False) and x.is_cuda:
                e = torch.cuda.Event(enable_timing=True)
                e.record()
                ev.append(e)
        x = x.to(torch.bfloat16).contiguous()
        n = x.shape[0]
        P = self.world
        C = max(1, min(getattr(self, "chunks", 2 if P > 1 else 1), n))
        bounds = [(n * c) // C for c in range(C + 1)]
        mark()
        w = self._route(x)
        cnts = [plan_counts(w[bounds[c]:bounds[c + 1]], P) for c in range(C)]
        send_counts = torch.stack([k for _, k in cnts], 1).contiguous()  # [P dest, C]
        if P == 1:
            sc = send_counts.t().tolist()  # the one host synchronisation
            rc = sc
        else:
            recv_counts = torch.empty_like(send_counts)                   # [P src, C]
            dist.all_to_all_single(recv_counts, send_counts, group=self.group)
            both = torch.stack([send_counts, recv_counts]).cpu()         # the one host synchronisation
            sc, rc = both[0].t().tolist(), both[1].t().tolist()           # [C][P]
        plans = [plan_lists(w[bounds[c]:bounds[c + 1]], cnts[c][0], sc[c], P) for c in range(C)]
        mark()
        # dispatch: rows and gate weights of every chunk, asynchronously
        recv, works = [], []
        for c, (tok, sw, _) in enumerate(plans):
            sx = x[bounds[c]:bounds[c + 1]].index_select(0, tok)
            if P == 1:
                recv.append((sx, sw))
                continue
            rx = torch.empty(sum(rc[c]), self.H, dtype=x.dtype, device=x.device)
            rw = torch.empty(sum(rc[c]), self.el, dtype=sw.dtype, device=x.device)
            works.append((dist.all_to_all_single(rx, sx, rc[c], sc[c], group=self.group, async_op=True),
                          dist.all_to_all_single(rw, sw, rc[c], sc[c], group=self.group, async_op=True)))
            recv.append((rx, rw))
        mark()
        # experts per chunk, each followed by its combine transfer
        backs, bworks = [], []
        for c in range(C):
            if P > 1:
                for wk in works[c]:
                    wk.wait()
            part = self._experts(*recv[c])
            if getattr(self, "partials", "fp32") == "bf16":
                part = part.to(torch.bfloat16)
            if P == 1:
                backs.append(part)
                continue
            back = torch.empty(sum(sc[c]), self.H, dtype=part.dtype, device=x.device)
            bworks.append(dist.all_to_all_single(back, part, sc[c], rc[c], group=self.group, async_op=True))
            backs.append(back)
        mark()
        y = torch.empty(n, self.H, dtype=torch.bfloat16, device=x.device)
        for c in range(C):
            if P > 1:
                bworks[c].wait()
            y[bounds[c]:bounds[c + 1]] = combine_partials(backs[c], plans[c][0], sc[c], bounds[c + 1] - bounds[c],
                                                          row_of=plans[c][2])
        mark()
        self.last_stats = {"sent_rows": sum(sum(v) for v in sc), "recv_rows": sum(sum(v) for v in rc),
                           "chunks": C}
        if ev:
            torch.cuda.synchronize()
            names = ["route_plan", "count_exchange_and_dispatch_enqueue", "experts_and_transfers", "combine"]
            self.last_stats.update({k: ev[i].elapsed_time(ev[i + 1]) for i, k in enumerate(names)})
        return y
