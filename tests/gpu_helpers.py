"""Helpers shared by the GPU parity tests (builds modules through the package's own
drop-in path: physical_reorder_for_inference -> TauSparseMoE buffers -> packed blob)."""
import torch
import torch.nn.functional as F

from conftest import oracle, pkg


def make_layer(seed, hidden=1536, experts=64, group=96, tau=0.95, scale=None, experts_id=None):
    synth = pkg().synth
    if scale is None:
        scale = synth.router_scale_for_tau(tau)
    L = synth.make_layer(seed, hidden, experts, group, router_scale=scale)
    if experts_id is not None:
        L.experts_id = torch.as_tensor(experts_id, dtype=torch.long)
    return L


def make_module(L, tau, device):
    P = pkg()
    m = P.TauSparseMoE(L.hidden, L.inter, L.experts, L.group, tau).to(device)
    masks = F.one_hot(L.experts_id, L.experts).t()
    P.physical_reorder_for_inference(m, L.gate_w, L.up_w, L.down_w, L.router_w, masks, tau)
    return m


def run_decode(m, x, device, bias=None):
    N = x.shape[0]
    E = m.num_experts
    xd = x.to(device)
    lg = torch.empty(N, E, dtype=torch.bfloat16, device=device)
    w = torch.empty(N, E, dtype=torch.bfloat16, device=device)
    m.logit_bias = bias
    out = m.forward_decode(xd, logits_out=lg, weights_out=w)
    m.check_device_status()
    return out.cpu(), lg.cpu(), w.cpu()


def ulp_diff_bf16(a, b):
    """Per-element |a - b| in units of one bf16 ulp of max(|a|, |b|), floored at the ulp of
    2^-10: near-zero logits carry fp32 summation-order error of a few 1e-6 absolute."""
    a = a.float()
    b = b.float()
    m = torch.maximum(a.abs(), b.abs()).clamp_min(2.0 ** -10)
    ulp = torch.exp2(torch.floor(torch.log2(m)) - 7)
    return ((a - b).abs() / ulp).ceil()


def _near_bf16_midpoint(v, tol=2e-4):
    """True where a positive float64 value lies within `tol` bf16-ulps of a rounding midpoint
    (so a few-ulp fp32 difference in how it was computed can flip its bf16 rounding)."""
    v = v.double()
    pos = v > 0
    e = torch.floor(torch.log2(torch.where(pos, v, torch.ones_like(v))))
    ulp = torch.exp2(e - 7)
    frac = torch.remainder(v / ulp, 1.0)
    return pos & ((frac - 0.5).abs() < tol)


def ambiguous_tokens(lg):
    """Tokens whose reference selection or gate weights hinge on fp32 rounding inside
    softmax or sigmoid (exp implementation / summation order): a probability or a sigmoid
    sits on a bf16 rounding midpoint to within fp32 precision."""
    l64 = lg.double()
    return (_near_bf16_midpoint(torch.softmax(l64, -1)) | _near_bf16_midpoint(torch.sigmoid(l64))).any(-1)


def assert_selection_matches(w, lg, tau, what=""):
    """Selection contract: given the same bf16 logits, the kernel's gate weights equal the
    oracle's (stable tie order) on every token, except tokens whose result hinges on fp32
    rounding inside softmax/sigmoid (CPU and GPU use different exp implementations and
    summation orders); those must be rare and explained."""
    w_ref, _ = oracle().softmax_thresholding(lg, tau)
    bad = (w != w_ref).any(-1)
    if bool(bad.any()):
        amb = ambiguous_tokens(lg[bad])
        assert bool(amb.all()), f"{what}: {int((~amb).sum())} selection mismatches not explained by rounding"
        assert int(bad.sum()) <= max(2, lg.shape[0] // 500), f"{what}: {int(bad.sum())} ambiguous mismatches"
    return int(bad.sum())


# Per-test end-to-end mask agreement with the literal reference (collected for the summary
# printed at the end of the session by conftest.py)
L2_STATS = []


def assert_mask_l2(x, L, tau, lg, w, bias=None, what="", ref_logits=None):
    """End-to-end selection parity with the LITERAL reference path (unstable CPU sort on the
    oracle's own router logits, src/MoEBlock.py:68-86).  Every token whose mask differs must
    be explained by one of:
      * "logit": the GPU's router logits of that token differ from the oracle's (<= 1 bf16 ulp,
        fp32 summation order) and the GPU mask equals the oracle's selection on the GPU's
        logits;
      * "tie": the oracle's stable and unstable selections differ on its own logits (equal
        bf16 probabilities straddle the cutoff) and the GPU mask equals the stable one;
      * "rounding": a probability or sigmoid of the token sits on a bf16 rounding midpoint to
        fp32 precision (CPU and GPU exp implementations differ there).
    Returns (tokens, mismatches, counts by cause) and records them in L2_STATS."""
    O = oracle()
    ref_lg = O.router_logits(x, L.router_w, bias) if ref_logits is None else ref_logits
    _, lit = O.softmax_thresholding(ref_lg, tau, stable=False)
    _, st = O.softmax_thresholding(ref_lg, tau, stable=True)
    _, st_gpu = O.softmax_thresholding(lg, tau, stable=True)
    gm = (w > 0).reshape(lit.shape)
    diff = (gm != lit).any(-1).flatten()
    n = int(diff.numel())
    causes = {"logit": 0, "tie": 0, "rounding": 0}
    if bool(diff.any()):
        lg2, rl2 = lg.reshape(n, -1), ref_lg.reshape(n, -1)
        gm2, st2, stg2, lit2 = gm.reshape(n, -1), st.reshape(n, -1), st_gpu.reshape(n, -1), lit.reshape(n, -1)
        for t in diff.nonzero().flatten().tolist():
            if not torch.equal(lg2[t], rl2[t]) and torch.equal(gm2[t], stg2[t]):
                causes["logit"] += 1
            elif not torch.equal(st2[t], lit2[t]) and torch.equal(gm2[t], st2[t]):
                causes["tie"] += 1
            elif bool(ambiguous_tokens(lg2[t:t + 1]).all()):
                causes["rounding"] += 1
            else:
                raise AssertionError(f"{what}: token {t} selects {gm2[t].nonzero().flatten().tolist()}, the "
                                     f"reference {lit2[t].nonzero().flatten().tolist()}: unexplained")
    mism = int(diff.sum())
    L2_STATS.append((what, n, mism, dict(causes)))
    return n, mism, causes


def check_against_oracle(L, x, tau, out, lg, w, bias=None, what=""):
    """Router logits within 1 bf16 ulp of the oracle's; selection bit-exact given the GPU's
    logits (stable contract); output within tolerance of the oracle teacher-forced with the
    GPU's logits.  Returns (#logit mismatches, #tokens whose selection differs from the
    oracle's own end to end)."""
    from conftest import assert_close_out
    O = oracle()
    ref = O.moe_mlp(x, L, tau, bias=bias)
    nd = ulp_diff_bf16(lg, ref.logits)
    if int(nd.max()) > 1:
        i = int(nd.flatten().argmax())
        raise AssertionError(f"{what}: router logit {i} differs by {int(nd.max())} ulp: "
                             f"gpu={lg.flatten()[i].item()} cpu={ref.logits.flatten()[i].item()}")
    assert_selection_matches(w, lg, tau, what)
    tf = O.moe_mlp(x, L, tau, logits=lg)
    assert_close_out(out, tf.out, what)
    assert_mask_l2(x, L, tau, lg, w, bias=bias, what=what, ref_logits=ref.logits)
    # end to end against the oracle's own output on the tokens whose selection agrees
    agree = ~((w > 0) != (ref.weights > 0)).any(-1)
    if bool(agree.any()):
        assert_close_out(out[agree], ref.out[agree], what + " (end to end)")
    sel_diff = int((~agree).sum())
    return int((nd > 0).sum()), sel_diff
