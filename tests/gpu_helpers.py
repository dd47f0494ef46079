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
    sel_diff = int(((w > 0) != (ref.weights > 0)).any(-1).sum())
    if sel_diff == 0:
        assert_close_out(out, ref.out, what + " (end to end)")
    return int((nd > 0).sum()), sel_diff
