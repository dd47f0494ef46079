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
    """Per-element distance in bf16 units-in-the-last-place (same-sign values)."""
    ai = a.view(torch.int16).int()
    bi = b.view(torch.int16).int()
    return (ai - bi).abs()


def check_against_oracle(L, x, tau, out, lg, w, bias=None, what=""):
    """Router logits within 1 bf16 ulp of the oracle's; selection bit-exact given the GPU's
    logits (stable contract); output within tolerance of the oracle teacher-forced with the
    GPU's logits.  Returns (#logit mismatches, #tokens whose selection differs from the
    oracle's own end to end)."""
    from conftest import assert_close_out
    O = oracle()
    ref = O.moe_mlp(x, L, tau, bias=bias)
    nd = ulp_diff_bf16(lg, ref.logits)
    assert int(nd.max()) <= 1, f"{what}: router logits differ by >1 ulp"
    w_ref, _ = O.softmax_thresholding(lg, tau)
    assert torch.equal(w, w_ref), f"{what}: selection/gate weights differ from the oracle on identical logits"
    tf = O.moe_mlp(x, L, tau, logits=lg)
    assert_close_out(out, tf.out, what)
    sel_diff = int(((w > 0) != (ref.weights > 0)).any(-1).sum())
    if sel_diff == 0:
        assert_close_out(out, ref.out, what + " (end to end)")
    return int((nd > 0).sum()), sel_diff
