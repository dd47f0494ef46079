"""Oracle pinned against the reference's own outputs (golden vectors made by running the
reference modules, tests/golden/make_golden.py).  CPU only."""
import hashlib

import numpy as np
import pytest
import torch

from conftest import oracle, pkg


def _layer(c):
    synth = pkg().synth
    L = synth.make_layer(c["seed"], c["hidden"], c["experts"], c["group"], router_scale=c["router_scale"])
    if "experts_id" in c:
        L.experts_id = c["experts_id"].long()
    return L


def _digest(L):
    h = hashlib.sha256()
    for t in (L.gate_w, L.up_w, L.down_w, L.router_w):
        h.update(t.contiguous().view(torch.int16).numpy().tobytes())
    h.update(L.experts_id.numpy().astype(np.int64).tobytes())
    return h.hexdigest()


def test_synth_reproduces_golden_inputs(golden):
    synth = pkg().synth
    for c in golden["cases"]:
        L = _layer(c)
        assert _digest(L) == c["digest"], c["name"]
        x = synth.make_tokens(c["seed"], c["tokens"], c["hidden"])
        assert hashlib.sha256(x.view(torch.int16).numpy().tobytes()).hexdigest() == c["x_digest"]


@pytest.mark.parametrize("idx", range(9))
def test_oracle_matches_reference_bit_exact(golden, idx):
    c = golden["cases"][idx]
    L = _layer(c)
    x = pkg().synth.make_tokens(c["seed"], c["tokens"], c["hidden"])
    r = oracle().moe_mlp(x, L, c["tau"], stable=False)
    assert torch.equal(r.logits, c["logits"])
    assert torch.equal(r.weights, c["weights"])
    assert torch.equal(r.out, c["out"])
    assert torch.equal(oracle().activation_counts(r.weights), c["counts"])


def test_oracle_selection_ties(golden):
    T = golden["ties"]
    for tau, d in T["taus"].items():
        w_lit, _ = oracle().softmax_thresholding(T["logits"], float(tau), stable=False)
        w_st, m_st = oracle().softmax_thresholding(T["logits"], float(tau), stable=True)
        assert torch.equal(w_lit, d["literal"])
        assert torch.equal(w_st, d["stable"])
        assert bool(m_st.any(-1).all())  # forced top-1


def test_stable_selection_properties():
    """Stable contract: kept set is a prefix of the (p desc, index asc) order; the forced
    top-1 always holds; sigmoid weights are positive exactly where selected (or underflow)."""
    O = oracle()
    g = torch.Generator().manual_seed(7)
    lg = (torch.randn(512, 64, generator=g) * 3).to(torch.bfloat16)
    for tau in (0.3, 0.7, 0.95, 1.0):
        w, m = O.softmax_thresholding(lg, tau)
        p = torch.softmax(lg, -1)
        order = torch.sort(p, dim=-1, descending=True, stable=True).indices
        ms = torch.gather(m, 1, order)
        k = ms.sum(-1)
        assert bool((k >= 1).all())
        assert torch.equal(ms, torch.arange(64).expand(512, 64) < k[:, None])
        assert bool(((w > 0) <= m).all())


def test_reference_layout_groups_experts():
    synth = pkg().synth
    L = synth.make_layer(3, 128, 16, 32, router_scale=1.0)
    Wg, Wu, Wd, R = oracle().reference_layout(L)
    order = torch.argsort(L.experts_id, stable=True)
    assert torch.equal(Wg, L.gate_w[order].t())
    assert torch.equal(Wd, L.down_w[:, order].t())
    assert torch.equal(R, L.router_w.t())
    assert torch.equal(L.experts_id[order], torch.arange(16).repeat_interleave(32))
