"""Generate golden vectors by running the reference's own PyTorch MoE path on CPU.

Run from the repository root, in a checkout that has the reference sources available::

    python tests/golden/make_golden.py --ref <reference-checkout>/src

It imports ``MoEBlock_origin`` and ``openpangu_moe_origin`` unchanged (with a stand-in
``k_means_constrained`` module, needed only by the offline clustering helper that this
path never calls), builds ``IntegratedOpenPanguMoEMLP`` in eval mode around synthetic
``nn.Linear`` projections, and records for each case the reference's output, router logits,
gate weights and selection mask.  Weights are regenerated from the seed at test time
(``synth.make_layer``); each case stores the SHA-256 of the weight bytes so a test can
confirm the regenerated tensors are the ones the reference saw.

Cases: two small shapes (H=128, E=16, G=32) at tau 0.70/0.95; the benchmark shape
(H=1536, E=64, G=96) at batch 1 (seeds 0-3, tau 0.95) and batch 16 (tau 0.70); the
reference's shipped configuration (E=192, G=32) using the real cluster assignment of
layer 0 (``src/Pangu_Clusters/layer_0_k32.txt``); and router-only tie cases for
``softmax_thresholding`` with both the literal (unstable) and the stable-sort behaviour.
"""
from __future__ import annotations

import argparse
import hashlib
import importlib
import os
import sys
import types
from types import SimpleNamespace

import numpy as np
import torch
import torch.nn as nn

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(os.path.dirname(HERE))
sys.path.insert(0, ROOT)
synth = importlib.import_module("prune_path_openpangu-embedded-1b_b200.synth")


def weight_digest(layer) -> str:
    h = hashlib.sha256()
    for t in (layer.gate_w, layer.up_w, layer.down_w, layer.router_w):
        h.update(t.contiguous().view(torch.int16).numpy().tobytes())
    h.update(layer.experts_id.numpy().astype(np.int64).tobytes())
    return h.hexdigest()


def build_reference_mlp(OM, layer, tau):
    cfg = SimpleNamespace(hidden_size=layer.hidden, intermediate_size=layer.inter)
    targs = SimpleNamespace(group_size=layer.group, tau=tau)
    mlp = SimpleNamespace(gate_proj=nn.Linear(layer.hidden, layer.inter, bias=False),
                          up_proj=nn.Linear(layer.hidden, layer.inter, bias=False),
                          down_proj=nn.Linear(layer.inter, layer.hidden, bias=False),
                          act_fn=nn.SiLU())
    m = OM.IntegratedOpenPanguMoEMLP(cfg, targs, mlp, [])
    with torch.no_grad():
        m.gate_proj.weight.data = layer.gate_w.clone()
        m.up_proj.weight.data = layer.up_w.clone()
        m.down_proj.weight.data = layer.down_w.clone()
        m.moelayer.mlp_router[0].weight.data = layer.router_w.clone()
        masks = torch.nn.functional.one_hot(layer.experts_id, layer.experts).t()
        m.moelayer.experts_masks = masks.to(torch.bfloat16)
    return m.eval()


def run_case(MB, OM, name, seed, hidden, experts, group, tokens, tau, scale, experts_id=None):
    layer = synth.make_layer(seed, hidden, experts, group, router_scale=scale)
    if experts_id is not None:
        layer.experts_id = torch.as_tensor(experts_id, dtype=torch.long)
    x = synth.make_tokens(seed, tokens, hidden)
    m = build_reference_mlp(OM, layer, tau)
    with torch.no_grad():
        out = m(x.view(1, tokens, hidden)).view(tokens, hidden)
        logits = m.moelayer.mlp_router(x.view(1, tokens, hidden))
        w, _ = MB.softmax_thresholding(logits, tau, training=False)
    rec = dict(name=name, seed=seed, hidden=hidden, experts=experts, group=group, tokens=tokens,
               tau=tau, router_scale=scale, digest=weight_digest(layer),
               out=out.clone(), logits=logits.view(tokens, experts).clone(),
               weights=w.view(tokens, experts).clone(),
               x_digest=hashlib.sha256(x.view(torch.int16).numpy().tobytes()).hexdigest(),
               counts=m.moelayer.activated_statistics.clone())
    if experts_id is not None:
        rec["experts_id"] = layer.experts_id.to(torch.int16).clone()
    return rec


def tie_cases(MB):
    """Router logits with exact bf16 ties straddling the tau cutoff."""
    g = torch.Generator().manual_seed(1234)
    rows = []
    for t in range(48):
        lg = torch.randn(64, generator=g) * 2.0
        k = t % 6 + 2  # make k experts share the maximum (or a near-top value)
        base = lg.max() if t % 2 == 0 else lg.sort(descending=True).values[3]
        idx = torch.randperm(64, generator=g)[:k]
        lg[idx] = base
        rows.append(lg)
    rows.append(torch.zeros(64))  # all equal: forced top-1 then ties
    rows.append(torch.full((64,), -3.0))
    one = torch.full((64,), -20.0); one[17] = 10.0  # single dominant expert (forced top-1)
    rows.append(one)
    logits = torch.stack(rows).to(torch.bfloat16)
    out = {}
    for tau in (0.5, 0.7, 0.95):
        w_lit, _ = MB.softmax_thresholding(logits.view(1, -1, 64), tau, training=False)
        orig_sort = torch.sort

        def stable_sort(*a, **k):
            k["stable"] = True
            return orig_sort(*a, **k)
        torch.sort = stable_sort
        try:
            w_st, _ = MB.softmax_thresholding(logits.view(1, -1, 64), tau, training=False)
        finally:
            torch.sort = orig_sort
        out[str(tau)] = dict(literal=w_lit.view(-1, 64).clone(), stable=w_st.view(-1, 64).clone())
    return dict(logits=logits, taus=out)


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--ref", required=True, help="reference src/ directory")
    ap.add_argument("--out", default=os.path.join(HERE, "golden.pt"))
    args = ap.parse_args()
    sys.modules.setdefault("k_means_constrained", types.SimpleNamespace(KMeansConstrained=None))
    sys.path.insert(0, args.ref)
    MB = importlib.import_module("MoEBlock_origin")
    OM = importlib.import_module("openpangu_moe_origin")
    torch.set_num_threads(os.cpu_count() or 1)

    cases = [
        run_case(MB, OM, "small_t70", 1, 128, 16, 32, 32, 0.70, 1.75),
        run_case(MB, OM, "small_t95", 2, 128, 16, 32, 32, 0.95, 3.5),
    ]
    for s in range(4):
        cases.append(run_case(MB, OM, f"base_bs1_t95_s{s}", s, 1536, 64, 96, 1, 0.95, 3.5))
    cases.append(run_case(MB, OM, "base_b16_t70", 0, 1536, 64, 96, 16, 0.70, 1.75))
    cases.append(run_case(MB, OM, "base_b64_t95", 3, 1536, 64, 96, 64, 0.95, 3.5))
    ids = np.loadtxt(os.path.join(args.ref, "Pangu_Clusters", "layer_0_k32.txt")).astype(np.int64)
    cases.append(run_case(MB, OM, "pangu_e192_t70", 5, 1536, 192, 32, 4, 0.70, 1.75, experts_id=ids))
    torch.save(dict(cases=cases, ties=tie_cases(MB)), args.out)
    print(f"wrote {args.out}: {[c['name'] for c in cases]}")


if __name__ == "__main__":
    main()
