"""Expert-parallel prefill over P GPUs (one process per GPU, torch.distributed / NCCL).

The reference runs on one device only; this is the sharded form of its prefill path
(``TauSparseMoE.forward_prefill``, src/tl_kernel_optimized_Ultimate_PanGU.py:532-604) for
large token counts:

* rank r owns one expert of every group of P consecutive experts in snake order
  (``owned_experts``: their packed gate/up/down records) and a shard of the tokens; the snake
  order balances skewed routing that favours low expert indices;
* every rank routes its own tokens (``ppmoe_prefill_route``: tcgen05 router GEMM + selection);
* a token row is sent once to each rank that owns at least one of its selected experts,
  together with its gate weights for that rank's experts, as one payload row: the send rows
  are built on the device (``ppmoe_ep_dispatch``: per-block counts, a scan, a scatter copy),
  then a count exchange (``all_to_all_single`` of int64 counts, the one host synchronisation)
  and one payload ``all_to_all_single`` per chunk;
* each rank runs its local experts on the received payload rows as they are
  (``ppmoe_ep_experts``: grouped tcgen05 GEMMs) and returns its partial sums with a second
  ``all_to_all_single``: scaled-fp16 rows by default (``partials="f16s"``), or fp32 / bf16
  rows (``partials="fp32"`` / ``"bf16"``);
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

__all__ = ["ExpertParallelMoE", "owned_experts", "dispatch_reference", "combine_partials", "chunk_bounds", "row_pitch",
           "f16s_pitch", "f16s_encode", "f16s_decode"]


def owned_experts(E: int, world: int, rank: int) -> torch.Tensor:
    """Experts of ``rank`` under the snake assignment: in expert group g (experts g P ..
    g P + P - 1) rank r owns g P + r for even g and g P + P - 1 - r for odd g.  Against a
    router prior that falls with the expert index (the Zipf skew of the benchmark) every rank
    gets one popular and one unpopular expert of each pair of groups, where a plain stride
    (r, r + P, ...) gives rank 0 the most popular expert of every group."""
    return torch.tensor([g * world + (rank if g % 2 == 0 else world - 1 - rank) for g in range(E // world)],
                        dtype=torch.long)


def chunk_bounds(n: int, chunks: int) -> list:
    """Token bounds of the dispatch chunks: whole 256-token blocks, chunk c = blocks
    [nb c / C, nb (c + 1) / C) (the split ``ppmoe_ep_dispatch`` uses)."""
    nb = (n + 255) // 256
    return [min(n, 256 * ((nb * c) // chunks)) for c in range(chunks + 1)]


def row_pitch(H: int, el: int) -> int:
    """Bytes per payload row: H bf16 activations + el bf16 gate weights, 16-byte multiple."""
    return ((H + el) * 2 + 15) // 16 * 16


def dispatch_reference(x: torch.Tensor, weights: torch.Tensor, world: int, chunks: int, pitch: int):
    """Torch restatement of ``ppmoe_ep_dispatch`` (CPU ranks, and the checker of the GPU
    kernel): returns ``(send [rows, pitch] uint8, counts [P, C] int64, row_of [P, n] int32)``.
    Rows chunk-major, destination-major, tokens ascending; a row is the token's activations then
    its gate weights for the destination's experts (``owned_experts`` order); pad bytes 0."""
    n, E = weights.shape
    H = x.shape[1]
    if E % world:
        raise ValueError(f"experts={E} not divisible by world size {world}")
    el = E // world
    b = chunk_bounds(n, chunks)
    perm = torch.stack([owned_experts(E, world, d) for d in range(world)]).to(weights.device)  # [P, el]
    wv = weights[:, perm]  # [n, P, el]: destination d's experts in owned order
    sel = (wv > 0).any(-1)
    counts = torch.zeros(world, chunks, dtype=torch.int64)
    row_of = torch.full((world, n), -1, dtype=torch.int32)
    segs, pos = [], 0
    for c in range(chunks):
        for d in range(world):
            toks = torch.nonzero(sel[b[c]:b[c + 1], d]).flatten() + b[c]
            counts[d, c] = len(toks)
            row_of[d, toks] = torch.arange(pos, pos + len(toks), dtype=torch.int32)
            segs.append((toks, d))
            pos += len(toks)
    send = torch.zeros(pos, pitch, dtype=torch.uint8)
    r = 0
    for toks, d in segs:
        k = len(toks)
        if k:
            send[r:r + k, :2 * H] = x[toks].contiguous().view(torch.uint8)
            send[r:r + k, 2 * H:2 * (H + el)] = wv[toks, d].contiguous().view(torch.uint8)
        r += k
    return send, counts, row_of


def f16s_pitch(H: int) -> int:
    """Bytes per scaled-fp16 partial row (``ppmoe_ep_partial_pitch``)."""
    return (2 * H + H // 64 + 15) // 16 * 16


def f16s_encode(rows: torch.Tensor) -> torch.Tensor:
    """Torch restatement of the scaled-fp16 row format (CPU ranks): per 64-column slice
    s = 14 - exponent(max |v|) clamped to [-126, 126], fp16(v * 2^s), then the int8 exponents."""
    n, H = rows.shape
    v = rows.float().view(n, H // 64, 64)
    m = v.abs().amax(-1)
    e = torch.frexp(m)[1] - 1  # exponent of m (m = f 2^e, 1 <= f < 2)
    sc = torch.where(m > 0, 14 - e, torch.zeros_like(e)).clamp(-126, 126)
    h = (v * torch.exp2(sc.float())[..., None]).to(torch.float16).view(n, H)
    out = torch.zeros(n, f16s_pitch(H), dtype=torch.uint8)
    out[:, :2 * H] = h.view(torch.uint8)
    out[:, 2 * H:2 * H + H // 64] = sc.to(torch.int8).view(torch.uint8)
    return out


def f16s_decode(rows: torch.Tensor, H: int) -> torch.Tensor:
    """fp32 values of scaled-fp16 rows (exact rescaling)."""
    n = rows.shape[0]
    h = rows[:, :2 * H].contiguous().view(torch.float16).float().view(n, H // 64, 64)
    sc = rows[:, 2 * H:2 * H + H // 64].contiguous().view(torch.int8).float()
    return (h * torch.exp2(-sc)[..., None]).view(n, H)


def combine_partials(back: torch.Tensor, row_of: torch.Tensor, n: int, H: Optional[int] = None) -> torch.Tensor:
    """Sum the partial rows of every token in rank order (fp32 additions) and round once to
    bf16: ``out[t] = bf16(sum_d back[row_of[d, t]])`` over the rows that exist (``ppmoe_ep_combine``
    on CUDA; the same order with torch operations on CPU ranks).  uint8 ``back`` holds
    scaled-fp16 rows of hidden size ``H`` (``ppmoe_ep_combine_f16s``)."""
    P = row_of.shape[0]
    if back.dtype == torch.uint8:
        if back.is_cuda:
            out = torch.empty(n, H, dtype=torch.bfloat16, device=back.device)
            _lib.call("ppmoe_ep_combine_f16s", back.data_ptr(), back.shape[1], row_of.data_ptr(), P, n, H,
                      out.data_ptr(), torch.cuda.current_stream(back.device).cuda_stream)
            return out
        back = f16s_decode(back, H)
    if back.is_cuda:
        out = torch.empty(n, back.shape[1], dtype=torch.bfloat16, device=back.device)
        fn = "ppmoe_ep_combine_bf16" if back.dtype == torch.bfloat16 else "ppmoe_ep_combine"
        _lib.call(fn, back.data_ptr(), row_of.data_ptr(), P, n, back.shape[1], out.data_ptr(),
                  torch.cuda.current_stream(back.device).cuda_stream)
        return out
    acc = torch.zeros(n, back.shape[1], dtype=torch.float32)
    for d in range(P):
        rows = row_of[d].long()
        has = rows >= 0
        acc[has] += back[rows[has]].float()
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
        # Format of the partial sums that cross the network on the way back:
        # "f16s" (default): fp16 with a power-of-two scale per 64-column slice, the prefill's
        #   pair-row format (relative error <= 2^-11 per rank's partial, half the fp32 bytes);
        # "fp32": the only rounding is the final bf16 one;
        # "bf16": each rank rounds its partial once to bf16 (looser tolerance).
        self.partials = "f16s"

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

    def _experts(self, payload, fmt: int = 0):
        """Partial sums of this rank's experts over received payload rows: ``[rows, H]`` fp32
        (``fmt`` 0), or rows of ``ppmoe_ep_partial_pitch(H)`` bytes in the scaled-fp16 format
        (``fmt`` 1, uint8 ``[rows, pitch]``)."""
        n = payload.shape[0]
        if self.expert_fn is not None:
            v = payload.view(torch.bfloat16)
            part = self.expert_fn(v[:, :self.H], v[:, self.H:self.H + self.el],
                                  owned_experts(self.E, self.world, self.rank))
            return part if fmt == 0 else f16s_encode(part)
        if fmt == 0:
            out = torch.empty(n, self.H, dtype=torch.float32, device=payload.device)
        else:
            out = torch.empty(n, _lib.load().ppmoe_ep_partial_pitch(self.H), dtype=torch.uint8, device=payload.device)
        if n == 0:
            return out
        m = self.local
        ws = m.prefill_workspace(n)
        _lib.call("ppmoe_ep_experts", payload.data_ptr(), n, payload.shape[1], m.packed().data_ptr(), self.H,
                  self.el, self.G, fmt, out.data_ptr(), ws.data_ptr(), ws.numel(), _stream_handle(payload.device))
        return out

    def _dispatch(self, x, w, C, pitch):
        if not x.is_cuda:
            return dispatch_reference(x, w, self.world, C, pitch)
        n, P = x.shape[0], self.world
        dev = x.device
        cache = getattr(self, "_dispatch_bufs", None)
        key = (n, P, C, pitch, dev)
        if cache is None or cache[0] != key:
            lib = _lib.load()
            nbytes = lib.ppmoe_ep_dispatch_workspace_bytes(n, P)
            cache = (key, torch.empty(max(1, n * P), pitch, dtype=torch.uint8, device=dev),
                     torch.empty(P, C, dtype=torch.int64, device=dev),
                     torch.empty(P, n, dtype=torch.int32, device=dev),
                     torch.empty(nbytes, dtype=torch.uint8, device=dev))
            self._dispatch_bufs = cache
        _, send, counts, row_of, ws = cache
        _lib.call("ppmoe_ep_dispatch", x.data_ptr(), w.data_ptr(), n, self.H, self.E, P, C, send.data_ptr(), pitch,
                  counts.data_ptr(), row_of.data_ptr(), ws.data_ptr(), ws.numel(), _stream_handle(dev))
        return send, counts, row_of

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
        C = max(1, min(getattr(self, "chunks", 2 if P > 1 else 1), (n + 255) // 256, 8))
        pitch = row_pitch(self.H, self.el)
        mark()
        w = self._route(x)
        send, counts, row_of = self._dispatch(x, w, C, pitch)   # device-side send rows, no sync
        if P == 1:
            sc = counts.t().tolist()                               # the one host synchronisation
            rc = sc
        else:
            recv_counts = torch.empty_like(counts)                  # [P src, C]
            dist.all_to_all_single(recv_counts, counts, group=self.group)
            both = torch.stack([counts, recv_counts]).cpu()        # the one host synchronisation
            sc, rc = both[0].t().tolist(), both[1].t().tolist()     # [C][P]
        sbase = [0]
        for c in range(C):
            sbase.append(sbase[-1] + sum(sc[c]))
        mark()
        # dispatch: one payload all-to-all per chunk (rows and gate weights together)
        recv, works = [], []
        for c in range(C):
            sx = send[sbase[c]:sbase[c + 1]]
            if P == 1:
                recv.append(sx)
                continue
            rx = torch.empty(sum(rc[c]), pitch, dtype=torch.uint8, device=x.device)
            works.append(dist.all_to_all_single(rx, sx, rc[c], sc[c], group=self.group, async_op=True))
            recv.append(rx)
        mark()
        # experts per chunk, each followed by its return transfer into the chunk's rows of `back`
        mode = getattr(self, "partials", "f16s")
        fmt = 1 if mode == "f16s" else 0
        if fmt:
            back = torch.empty(sbase[C], f16s_pitch(self.H), dtype=torch.uint8, device=x.device)
        else:
            back = torch.empty(sbase[C], self.H, dtype=torch.bfloat16 if mode == "bf16" else torch.float32,
                               device=x.device)
        bworks = []
        for c in range(C):
            if P > 1:
                works[c].wait()
            part = self._experts(recv[c], fmt)
            if mode == "bf16":
                part = part.to(torch.bfloat16)
            if P == 1:
                back[sbase[c]:sbase[c + 1]] = part
                continue
            bworks.append(dist.all_to_all_single(back[sbase[c]:sbase[c + 1]], part, sc[c], rc[c],
                                                 group=self.group, async_op=True))
        for wk in bworks:
            wk.wait()
        mark()
        y = combine_partials(back, row_of, n, self.H)
        mark()
        self.last_stats = {"sent_rows": sum(sum(v) for v in sc), "recv_rows": sum(sum(v) for v in rc),
                           "chunks": C}
        if ev:
            torch.cuda.synchronize()
            names = ["route_plan", "count_exchange_and_dispatch_enqueue", "experts_and_transfers", "combine"]
            self.last_stats.update({k: ev[i].elapsed_time(ev[i + 1]) for i, k in enumerate(names)})
        return y
