"""Drop-in ``TauSparseMoE`` backed by the sm_100a kernels of libppmoe.

Mirrors the reference module ``TauSparseMoE``
(src/tl_kernel_optimized_Ultimate_PanGU.py:468-615):

* constructor ``TauSparseMoE(hidden_size, intermediate_size, num_experts, group_size, tau)``;
* persistent bf16 buffers ``W_gate [H,I]``, ``W_up [H,I]``, ``W_down [I,H]``,
  ``router [H,E]`` (tl:483-486) -- the state-dict keys ``...mlp.tau_moe.{W_gate,W_up,W_down,
  router}`` and the tensors ``physical_reorder_for_inference`` assigns through ``.data``
  (src/openpangu_moe.py:239-243);
* mutable attribute ``tau`` (src/openpangu_moe.py:226);
* ``forward(x [B,L,H]) -> [B,L,H]`` bf16 (tl:606-615): up to 16 tokens go through the
  fused single-launch decode kernel, more tokens through the tcgen05 prefill path.

The packed layout the kernels read is derived on the device from those four buffers and
rebuilt automatically whenever one of them is replaced or modified in place.  Every call is
enqueued on the current CUDA stream without host synchronisation.
"""
from __future__ import annotations

import torch
import torch.nn as nn

from . import _lib

__all__ = ["TauSparseMoE", "IntegratedOpenPanguMoEMLP", "physical_reorder_for_inference"]


def _stream_handle(device) -> int:
    """Raw handle of the current CUDA stream of ``device`` (no Stream object is built)."""
    return torch._C._cuda_getCurrentRawStream(device.index if device.index is not None else torch.cuda.current_device())


class TauSparseMoE(nn.Module):
    """B200 tau-sparse MoE MLP with the reference module's interface."""

    def __init__(self, hidden_size: int, intermediate_size: int, num_experts: int,
                 group_size: int, tau: float):
        super().__init__()
        if intermediate_size != num_experts * group_size:
            raise ValueError("intermediate_size must equal num_experts * group_size")
        self.hidden_size = hidden_size
        self.intermediate_size = intermediate_size
        self.num_experts = num_experts
        self.group_size = group_size
        self.tau = tau
        self.logit_bias = None  # optional fp32 [E] prior (skewed-routing benchmarks)
        self.track_statistics = False
        self.register_buffer("W_gate", torch.empty(hidden_size, intermediate_size, dtype=torch.bfloat16))
        self.register_buffer("W_up", torch.empty(hidden_size, intermediate_size, dtype=torch.bfloat16))
        self.register_buffer("W_down", torch.empty(intermediate_size, hidden_size, dtype=torch.bfloat16))
        self.register_buffer("router", torch.empty(hidden_size, num_experts, dtype=torch.bfloat16))
        # per-expert count of tokens with a positive gate weight (src/MoEBlock.py:146,189-191)
        self.register_buffer("activated_statistics", torch.zeros(num_experts, dtype=torch.long),
                             persistent=False)
        self._packed = None
        self._packed_key = None
        self._ws = None
        self._ws_tokens = 0
        self._pws = None
        self._pws_tokens = 0
        # persistent decode output (the reference's decode_out, tl:491, returned as a view at
        # tl:530): forward() of <= 16 tokens returns a view of it that the next decode call
        # of this module overwrites
        self._dec_out = None
        self._dec_views = {}
        self._bias_src = None
        self._bias_ver = -1
        self._bias_dev = None

    # ------------------------------------------------------------------ packing
    def _weights_key(self):
        # identity of the four buffers' storage and their in-place version counters (a
        # reassignment of .data changes the pointer, an in-place edit bumps _version)
        b = self._buffers
        g, u, d, r = b["W_gate"], b["W_up"], b["W_down"], b["router"]
        return (g.data_ptr(), g._version, u.data_ptr(), u._version, d.data_ptr(), d._version,
                r.data_ptr(), r._version)

    def packed(self) -> torch.Tensor:
        """The packed weight blob (uint8, 1 KiB aligned), rebuilt if any buffer changed."""
        key = self._weights_key()
        if self._packed is None or self._packed_key != key:
            dev = self.W_gate.device
            if dev.type != "cuda":
                raise RuntimeError("TauSparseMoE runs on CUDA only; move the module to a GPU")
            H, E, G = self.hidden_size, self.num_experts, self.group_size
            nbytes = _lib.load().ppmoe_packed_bytes(H, E, G)
            if nbytes == 0:
                raise _lib.PPMoEError("ppmoe_packed_bytes", -2, _lib.load().ppmoe_last_error().decode())
            blob = torch.empty(nbytes + 1024, dtype=torch.uint8, device=dev)
            off = (-blob.data_ptr()) % 1024
            blob = blob[off:off + nbytes]
            ws = [t.contiguous() for t in (self.W_gate, self.W_up, self.W_down, self.router)]
            _lib.call("ppmoe_pack", *[t.data_ptr() for t in ws], H, E, G, blob.data_ptr(),
                      _stream_handle(dev))
            self._packed = blob
            self._packed_key = key
        return self._packed

    def workspace(self, tokens: int) -> torch.Tensor:
        dev = self.W_gate.device
        tokens = min(max(tokens, 1), _lib.DECODE_MAX_TOKENS)
        if self._ws is None or self._ws_tokens < tokens or self._ws.device != dev:
            n = _lib.load().ppmoe_workspace_bytes(tokens, self.hidden_size, self.num_experts,
                                                  self.group_size)
            buf = torch.empty(n + 256, dtype=torch.uint8, device=dev)
            off = (-buf.data_ptr()) % 256
            ws = buf[off:off + n]
            _lib.call("ppmoe_workspace_init", ws.data_ptr(), n, _stream_handle(dev))
            self._ws, self._ws_tokens = ws, tokens
        return self._ws

    def check_device_status(self) -> None:
        """Synchronise and raise if a kernel recorded a device-side error (bounded wait ran
        out); clears the status words."""
        for ws in (self._ws, self._pws):
            if ws is not None:
                _lib.call("ppmoe_workspace_status", ws.data_ptr(), _stream_handle(ws.device))

    # ------------------------------------------------------------------ forward
    def forward_decode(self, x_flat: torch.Tensor, *, logits_out=None, weights_out=None,
                       pdl: bool = False) -> torch.Tensor:
        N, H = x_flat.shape
        out = torch.empty(N, H, dtype=torch.bfloat16, device=x_flat.device)
        ws = self.workspace(N)
        bias = self._device_bias(x_flat.device)
        counts = self.activated_statistics if self.track_statistics else None
        _lib.call("ppmoe_decode", x_flat.data_ptr(), N, self.packed().data_ptr(), H,
                  self.num_experts, self.group_size, float(self.tau), _lib.ptr(bias),
                  out.data_ptr(), _lib.ptr(logits_out), _lib.ptr(weights_out), _lib.ptr(counts),
                  ws.data_ptr(), ws.numel(), int(pdl), _stream_handle(x_flat.device))
        return out

    def prefill_workspace(self, tokens: int) -> torch.Tensor:
        """Worst-case-sized prefill workspace (grown on demand, zeroed once)."""
        dev = self.W_gate.device
        if self._pws is None or self._pws_tokens < tokens or self._pws.device != dev:
            n = _lib.load().ppmoe_prefill_workspace_bytes(tokens, self.hidden_size, self.num_experts,
                                                          self.group_size)
            if n == 0:
                raise _lib.PPMoEError("ppmoe_prefill_workspace_bytes", -2, _lib.load().ppmoe_last_error().decode())
            buf = torch.empty(n + 1024, dtype=torch.uint8, device=dev)
            off = (-buf.data_ptr()) % 1024
            ws = buf[off:off + n]
            _lib.call("ppmoe_workspace_init", ws.data_ptr(), n, _stream_handle(dev))
            self._pws, self._pws_tokens = ws, tokens
        return self._pws

    def forward_prefill(self, x_flat: torch.Tensor, *, logits_out=None, weights_out=None) -> torch.Tensor:
        N, H = x_flat.shape
        out = torch.empty(N, H, dtype=torch.bfloat16, device=x_flat.device)
        ws = self.prefill_workspace(N)
        bias = self._device_bias(x_flat.device)
        counts = self.activated_statistics if self.track_statistics else None
        _lib.call("ppmoe_prefill", x_flat.data_ptr(), N, self.packed().data_ptr(), H, self.num_experts,
                  self.group_size, float(self.tau), _lib.ptr(bias), out.data_ptr(), _lib.ptr(logits_out),
                  _lib.ptr(weights_out), _lib.ptr(counts), ws.data_ptr(), ws.numel(),
                  _stream_handle(x_flat.device))
        return out

    def route(self, x_flat: torch.Tensor, *, mask_out=None):
        """Compact active-expert lists for ``x_flat [N,H]`` (``ppmoe_route``): returns
        ``(ids [N,E] int32, weights [N,E] bf16, n_active [N] int32)``, each row's selected
        experts in descending probability with -1 / 0 past ``n_active`` -- the decode router
        outputs of the reference (tl:488-490, tl:502-509) for any token count."""
        N, H = x_flat.shape
        dev = x_flat.device
        E = self.num_experts
        ids = torch.empty(N, E, dtype=torch.int32, device=dev)
        w = torch.empty(N, E, dtype=torch.bfloat16, device=dev)
        n = torch.empty(N, dtype=torch.int32, device=dev)
        nbytes = _lib.load().ppmoe_route_workspace_bytes(N, H, E, self.group_size)
        buf = torch.empty(nbytes + 1024, dtype=torch.uint8, device=dev)
        ws = buf[(-buf.data_ptr()) % 1024:][:nbytes]
        bias = self.logit_bias
        if bias is not None:
            bias = bias.to(device=dev, dtype=torch.float32).contiguous()
        x_flat = x_flat.to(torch.bfloat16).contiguous()
        _lib.call("ppmoe_route", x_flat.data_ptr(), N, self.packed().data_ptr(), H, E, self.group_size,
                  float(self.tau), _lib.ptr(bias), ids.data_ptr(), w.data_ptr(), n.data_ptr(),
                  _lib.ptr(mask_out), ws.data_ptr(), nbytes, _stream_handle(dev))
        return ids, w, n

    def _device_bias(self, dev):
        b = self.logit_bias
        if b is None:
            return None
        if b is not self._bias_src or b._version != self._bias_ver or self._bias_dev.device != dev:
            self._bias_src, self._bias_ver = b, b._version
            self._bias_dev = b.to(device=dev, dtype=torch.float32).contiguous()
        return self._bias_dev

    def _decode_into_persistent(self, x, B, L, H):
        """forward() for <= 16 tokens: one ctypes call into ppmoe_decode writing the persistent
        output buffer; the view returned aliases it (as the reference's decode_out does)."""
        dev = x.device
        key = self._weights_key()
        if self._packed is None or self._packed_key != key:
            self.packed()
        out = self._dec_out
        if out is None or out.device != dev:
            out = self._dec_out = torch.empty(_lib.DECODE_MAX_TOKENS, H, dtype=torch.bfloat16, device=dev)
            self._dec_views = {}
        ws = self._ws
        if ws is None or self._ws_tokens < _lib.DECODE_MAX_TOKENS or ws.device != dev:
            ws = self.workspace(_lib.DECODE_MAX_TOKENS)
        view = self._dec_views.get((B, L))
        if view is None:
            view = self._dec_views[(B, L)] = out[:B * L].view(B, L, H)
        bias = self._device_bias(dev)
        counts = self._buffers["activated_statistics"] if self.track_statistics else None
        rc = _lib.load().ppmoe_decode(x.data_ptr(), B * L, self._packed.data_ptr(), H, self.num_experts,
                                      self.group_size, float(self.tau),
                                      None if bias is None else bias.data_ptr(), out.data_ptr(), None, None,
                                      None if counts is None else counts.data_ptr(), ws.data_ptr(), ws.numel(), 0,
                                      _stream_handle(dev))
        if rc:
            raise _lib.PPMoEError("ppmoe_decode", rc, _lib.load().ppmoe_last_error().decode())
        return view

    def forward(self, x: torch.Tensor, **kw) -> torch.Tensor:
        """``[B,L,H] -> [B,L,H]`` bf16 (tl:606-615).  Up to 16 tokens: the fused decode
        kernel, returning a view of a persistent per-module output buffer (overwritten by the
        module's next decode call, like the reference's decode_out); more tokens: prefill into
        a fresh tensor."""
        B, L, H = x.shape
        N = B * L
        if x.device.type != "cuda":
            raise RuntimeError("TauSparseMoE runs on CUDA only; got a tensor on " + str(x.device))
        if x.dtype is not torch.bfloat16:
            x = x.to(torch.bfloat16)
        if not x.is_contiguous():
            x = x.contiguous()
        if N == 0:
            return torch.empty(B, L, H, dtype=torch.bfloat16, device=x.device)
        if N <= _lib.DECODE_MAX_TOKENS and not kw:
            return self._decode_into_persistent(x, B, L, H)
        x_flat = x.view(N, H)
        if N <= _lib.DECODE_MAX_TOKENS:
            return self.forward_decode(x_flat, **kw).view(B, L, H)
        return self.forward_prefill(x_flat, **kw).view(B, L, H)


class IntegratedOpenPanguMoEMLP(nn.Module):
    """The reference MLP wrapper (src/openpangu_moe.py:43-130).

    Eval mode: ``forward`` routes hidden states through ``self.tau_moe`` (the fused CUDA path)
    and unwraps a tuple as the reference does (:125-130).  Training mode (:98-123): the dense
    gate/up projections of ``original_mlp``, the training router ``self.moelayer``
    (:class:`~.training.TrainingMoELayer`: GPU selection, autograd through the gate weights
    and softmax), the neuron mask, the down projection; the softmax probabilities are
    appended to ``penalize_logits_list`` for the entropy and load-balance losses
    (:func:`~.training.moe_aux_losses`)."""

    def __init__(self, config, train_args, original_mlp=None, penalize_logits_list=None):
        super().__init__()
        from .training import TrainingMoELayer
        hidden = getattr(config, "hidden_size", 1536)
        inter = getattr(config, "intermediate_size", hidden * 4)
        experts = inter // train_args.group_size
        self.config, self.train_args = config, train_args
        self.gate_proj = getattr(original_mlp, "gate_proj", None)
        self.up_proj = getattr(original_mlp, "up_proj", None)
        self.down_proj = getattr(original_mlp, "down_proj", None)
        self.act_fn = getattr(original_mlp, "act_fn", None) or nn.SiLU()
        self.penalize_logits_list = penalize_logits_list if penalize_logits_list is not None else []
        self.moelayer = TrainingMoELayer(hidden, inter, experts, getattr(train_args, "tau", 0.95))
        self.tau_moe = TauSparseMoE(hidden, inter, experts, train_args.group_size,
                                    getattr(train_args, "tau", 0.5))

    def forward(self, hidden_states, *args, **kwargs):
        if self.training:
            if self.gate_proj is None or self.up_proj is None or self.down_proj is None:
                raise NotImplementedError("training mode needs gate_proj, up_proj and down_proj")
            inter = self.act_fn(self.gate_proj(hidden_states)) * self.up_proj(hidden_states)
            inter, probs = self.moelayer(hidden_states, inter)
            if probs is not None:
                self.penalize_logits_list.append(probs)
            return self.down_proj(inter)
        out = self.tau_moe(hidden_states)
        return out[0] if isinstance(out, tuple) else out


@torch.no_grad()
def physical_reorder_for_inference(tau_moe: TauSparseMoE, gate_w, up_w, down_w, router_w,
                                   experts_masks, tau: float) -> None:
    """One layer of ``CustomOpenPangu.physical_reorder_for_inference``
    (src/openpangu_moe.py:222-243): group neurons by expert and mount the transposed
    projections on ``tau_moe``'s buffers.  ``gate_w/up_w [I,H]``, ``down_w [H,I]``,
    ``router_w [E,H]`` are the ``nn.Linear`` weights, ``experts_masks [E,I]``."""
    dev = tau_moe.W_gate.device
    tau_moe.tau = tau
    expert_ids = torch.argmax(experts_masks.to(torch.int32), dim=0)
    sort_idx = torch.argsort(expert_ids, stable=True)
    tau_moe.W_gate.data = gate_w[sort_idx, :].t().contiguous().to(device=dev, dtype=torch.bfloat16)
    tau_moe.W_up.data = up_w[sort_idx, :].t().contiguous().to(device=dev, dtype=torch.bfloat16)
    tau_moe.W_down.data = down_w[:, sort_idx].t().contiguous().to(device=dev, dtype=torch.bfloat16)
    tau_moe.router.data = router_w.t().contiguous().to(device=dev, dtype=torch.bfloat16)
