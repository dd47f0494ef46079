"""Synthetic PrunePath decoder for end-to-end decode measurement (26 layers, prompt 512, 128 new tokens).

26 pre-norm decoder layers, hidden 1536, 12 attention heads x 128 (multi-head attention: the
openPangu KV-head count is not given in the reference, which loads the HF model remotely,
src/openpangu_moe.py:154-159), RMSNorm, rotary position embedding, vocabulary 153,600,
random-init bf16 weights.  Every MLP is either the PrunePath MoE MLP (``TauSparseMoE``, 64 x
96 experts, tau 0.70; the reference injects it at src/openpangu_moe.py:163-178) or the dense
SwiGLU MLP it replaces (same weights, all 6144 neurons, cuBLAS GEMMs) for the baseline.

Prompt prefill runs the prefill path; greedy decode runs one token per step through a CUDA
graph of the whole 26-layer step (the fused single-launch decode kernel per MoE layer).
Attention, norms, RoPE and the LM head use PyTorch operators: they are not part of the
hot path this library rebuilds.
"""
from __future__ import annotations

from dataclasses import dataclass

import torch
import torch.nn.functional as F

from .tau_moe import TauSparseMoE

__all__ = ["DecoderConfig", "SyntheticDecoder"]


@dataclass
class DecoderConfig:
    layers: int = 26
    hidden: int = 1536
    heads: int = 12
    head_dim: int = 128
    vocab: int = 153600
    experts: int = 64
    group: int = 96
    tau: float = 0.70
    router_scale: float = 1.75
    max_seq: int = 640
    mlp: str = "moe"  # or "dense"
    eps: float = 1e-6
    rope_theta: float = 10000.0


def _rms(x, w, eps):
    xf = x.float()
    return (xf * torch.rsqrt(xf.pow(2).mean(-1, keepdim=True) + eps)).to(x.dtype) * w


class SyntheticDecoder:
    def __init__(self, cfg: DecoderConfig, device, seed: int = 0, max_batch: int = 16):
        self.cfg = cfg
        self.dev = torch.device(device)
        g = torch.Generator(device=self.dev).manual_seed(seed)
        H, I = cfg.hidden, cfg.experts * cfg.group

        def w(*shape, scale=0.02):
            return (torch.randn(*shape, generator=g, device=self.dev) * scale).to(torch.bfloat16)

        self.embed = w(cfg.vocab, H)
        self.lm_head = w(cfg.vocab, H)
        self.norm_w = torch.ones(H, dtype=torch.bfloat16, device=self.dev)
        self.layers = []
        for _ in range(cfg.layers):
            L = {"ln1": torch.ones(H, dtype=torch.bfloat16, device=self.dev),
                 "ln2": torch.ones(H, dtype=torch.bfloat16, device=self.dev),
                 "wqkv": w(3 * H, H), "wo": w(H, H)}
            # neurons already grouped by expert (identity clustering): reference layout directly
            W_gate, W_up, W_down = w(H, I), w(H, I), w(I, H)
            router = w(H, cfg.experts, scale=0.02 * cfg.router_scale)
            if cfg.mlp == "moe":
                m = TauSparseMoE(H, I, cfg.experts, cfg.group, cfg.tau).to(self.dev)
                m.W_gate, m.W_up, m.W_down, m.router = W_gate, W_up, W_down, router
                m.packed()
                m.workspace(max_batch)
                L["moe"] = m
            else:
                L["gate_up"] = torch.cat([W_gate.t(), W_up.t()], 0).contiguous()  # [2I, H]
                L["down"] = W_down.t().contiguous()  # [H, I]
            self.layers.append(L)
        half = cfg.head_dim // 2
        inv = 1.0 / (cfg.rope_theta ** (torch.arange(half, device=self.dev, dtype=torch.float32) / half))
        ang = torch.arange(cfg.max_seq, device=self.dev, dtype=torch.float32)[:, None] * inv[None]
        self.cos, self.sin = ang.cos(), ang.sin()
        self.kv = None
        self.graph = None

    # ------------------------------------------------------------------ pieces
    def _rope(self, x, pos):  # x [B, h, L, d]; pos [L] int64 (device)
        c, s = self.cos[pos][None, None], self.sin[pos][None, None]
        x1, x2 = x.float().chunk(2, -1)
        return torch.cat([x1 * c - x2 * s, x2 * c + x1 * s], -1).to(x.dtype)

    def _mlp(self, L, h):
        if self.cfg.mlp == "moe":
            return L["moe"](h)
        gu = F.linear(h, L["gate_up"])
        gate, up = gu.chunk(2, -1)
        return F.linear(F.silu(gate) * up, L["down"])

    def _layer(self, i, L, x, pos, prefill: bool):
        cfg = self.cfg
        B, T, H = x.shape
        h = _rms(x, L["ln1"], cfg.eps)
        q, k, v = F.linear(h, L["wqkv"]).view(B, T, 3, cfg.heads, cfg.head_dim).permute(2, 0, 3, 1, 4)
        q, k = self._rope(q, pos), self._rope(k, pos)
        kc, vc = self.kv[i]
        kc.index_copy_(2, pos, k)
        vc.index_copy_(2, pos, v)
        if prefill:
            o = F.scaled_dot_product_attention(q, k, v, is_causal=True)
        else:
            mask = (torch.arange(cfg.max_seq, device=self.dev) <= pos[0])[None, None, None]
            o = F.scaled_dot_product_attention(q, kc, vc, attn_mask=mask)
        x = x + F.linear(o.transpose(1, 2).reshape(B, T, H), L["wo"])
        return x + self._mlp(L, _rms(x, L["ln2"], cfg.eps))

    def _logits_next(self, x):
        return F.linear(_rms(x[:, -1], self.norm_w, self.cfg.eps), self.lm_head).argmax(-1)

    # ------------------------------------------------------------------ API
    @torch.no_grad()
    def prefill(self, ids):
        cfg = self.cfg
        B, T = ids.shape
        if self.kv is None or self.kv[0][0].shape[0] != B:  # persistent: captured graphs read them
            self.kv = [(torch.zeros(B, cfg.heads, cfg.max_seq, cfg.head_dim, dtype=torch.bfloat16, device=self.dev),
                        torch.zeros(B, cfg.heads, cfg.max_seq, cfg.head_dim, dtype=torch.bfloat16, device=self.dev))
                       for _ in range(cfg.layers)]
            self.graph = None
        x = self.embed[ids]
        pos = torch.arange(T, device=self.dev)
        for i, L in enumerate(self.layers):
            x = self._layer(i, L, x, pos, True)
        return self._logits_next(x)

    @torch.no_grad()
    def _step(self, tok, pos):
        x = self.embed[tok][:, None]
        for i, L in enumerate(self.layers):
            x = self._layer(i, L, x, pos, False)
        return self._logits_next(x)

    @torch.no_grad()
    def generate(self, ids, new_tokens: int, use_graph: bool = True):
        """Greedy decode; returns (tokens [B, new_tokens], prefill_ms, decode_ms)."""
        B, T = ids.shape
        if T + new_tokens > self.cfg.max_seq:
            raise ValueError(f"prompt {T} + {new_tokens} new tokens exceed max_seq {self.cfg.max_seq}")
        e0, e1, e2 = (torch.cuda.Event(enable_timing=True) for _ in range(3))
        e0.record()
        tok = self.prefill(ids)
        e1.record()
        out = [tok]
        if use_graph and (self.graph is None or self._gB != B):
            self._pos = torch.zeros(1, dtype=torch.long, device=self.dev)  # graph inputs: fixed tensors
            self._tok = torch.zeros(B, dtype=torch.long, device=self.dev)
        elif not use_graph:
            self._pos = torch.zeros(1, dtype=torch.long, device=self.dev)
            self._tok = torch.zeros(B, dtype=torch.long, device=self.dev)
        self._pos.fill_(T)
        self._tok.copy_(tok)
        if use_graph:
            if self.graph is None or self._gB != B:
                s = torch.cuda.Stream(self.dev)
                s.wait_stream(torch.cuda.current_stream(self.dev))
                with torch.cuda.stream(s):
                    self._next = self._step(self._tok, self._pos)  # warm-up outside capture
                torch.cuda.current_stream(self.dev).wait_stream(s)
                self.graph = torch.cuda.CUDAGraph()
                with torch.cuda.graph(self.graph):
                    self._next = self._step(self._tok, self._pos)
                self._gB = B
                # the warm-up wrote position T into the caches: harmless, rewritten below
        for _ in range(new_tokens - 1):
            if use_graph:
                self.graph.replay()
                nxt = self._next
            else:
                nxt = self._step(self._tok, self._pos)
            out.append(nxt.clone())
            self._tok.copy_(nxt)
            self._pos += 1
        e2.record()
        torch.cuda.synchronize()
        return torch.stack(out, 1), e0.elapsed_time(e1), e1.elapsed_time(e2)
