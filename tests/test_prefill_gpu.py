"""GPU parity of the tcgen05 prefill path (batch 64 and 8 x 2048 tokens) against the
CPU oracle, plus consistency with the fused decode kernel."""
import pytest
import torch

from conftest import assert_close_out, oracle, pkg
from gpu_helpers import assert_mask_l2, assert_selection_matches, make_layer, make_module, ulp_diff_bf16

pytestmark = pytest.mark.gpu


def run_prefill(m, x, cuda, bias=None):
    N = x.shape[0]
    lg = torch.empty(N, m.num_experts, dtype=torch.bfloat16, device=cuda)
    w = torch.empty(N, m.num_experts, dtype=torch.bfloat16, device=cuda)
    m.logit_bias = bias
    out = m.forward_prefill(x.to(cuda), logits_out=lg, weights_out=w)
    m.check_device_status()
    return out.cpu(), lg.cpu(), w.cpu()


def check(L, x, tau, out, lg, w, bias=None, what=""):
    O = oracle()
    ref_lg = O.router_logits(x, L.router_w, bias)
    assert int(ulp_diff_bf16(lg, ref_lg).max()) <= 1, what
    assert_selection_matches(w, lg, tau, what)
    tf = O.moe_mlp(x, L, tau, logits=lg)
    assert_close_out(out, tf.out, what)
    assert_mask_l2(x, L, tau, lg, w, bias=bias, what=what, ref_logits=ref_lg)


@pytest.mark.parametrize("shape", [(256, 16, 32, 300, 0.7), (1536, 64, 96, 64, 0.95), (1536, 64, 96, 17, 0.7),
                                   (1536, 192, 32, 200, 0.7), (2048, 32, 128, 129, 0.95), (1536, 64, 96, 2048, 0.7)])
def test_prefill_vs_oracle(cuda, shape):
    H, E, G, N, tau = shape
    L = make_layer(7, H, E, G, tau)
    x = pkg().synth.make_tokens(7, N, H)
    m = make_module(L, tau, cuda)
    out, lg, w = run_prefill(m, x, cuda)
    check(L, x, tau, out, lg, w, what=str(shape))


def test_prefill_config3_full_size(cuda):
    """Prefill of 8 x 2048 tokens, tau 0.70, against the teacher-forced oracle."""
    H, E, G, tau = 1536, 64, 96, 0.70
    L = make_layer(3, H, E, G, tau)
    x = pkg().synth.make_tokens(3, 16384, H)
    m = make_module(L, tau, cuda)
    m.track_statistics = True
    out, lg, w = run_prefill(m, x, cuda)
    check(L, x, tau, out, lg, w, what="config3")
    assert torch.equal(m.activated_statistics.cpu(), oracle().activation_counts(w))
    # the module forward takes the same path for [8, 2048, H]
    y = m(x.view(8, 2048, H).to(cuda)).view(16384, H).cpu()
    assert_close_out(y, out, "forward vs forward_prefill")


def test_prefill_matches_decode_and_reuses_workspace(cuda):
    H, E, G, tau = 1536, 64, 96, 0.95
    L = make_layer(9, H, E, G, tau)
    m = make_module(L, tau, cuda)
    x_big = pkg().synth.make_tokens(9, 1000, H)
    run_prefill(m, x_big, cuda)  # sizes the workspace for 1000 tokens
    x = pkg().synth.make_tokens(9, 12, H, stream=2)
    out_p, lg_p, w_p = run_prefill(m, x, cuda)  # smaller call in the same workspace
    out_d = m.forward_decode(x.to(cuda)).cpu()
    assert_close_out(out_p, out_d, "prefill vs decode")
    check(L, x, tau, out_p, lg_p, w_p, what="reuse")


def test_prefill_zipf_bias(cuda):
    H, E, G, tau = 1536, 64, 96, 0.70
    L = make_layer(4, H, E, G, tau)
    m = make_module(L, tau, cuda)
    b = pkg().synth.zipf_bias(E, 1.2)
    x = pkg().synth.make_tokens(4, 700, H)
    out, lg, w = run_prefill(m, x, cuda, bias=b.to(cuda))
    check(L, x, tau, out, lg, w, bias=b, what="zipf")
    out2, lg2, w2 = run_prefill(m, x, cuda, bias=b.to(cuda))  # fixed-order sums: bit-reproducible
    assert torch.equal(out2, out) and torch.equal(w2, w) and torch.equal(lg2, lg)


@pytest.mark.parametrize("tau", [0.70, 0.95])
def test_batch64_sweep(cuda, tau):
    """Config 2 at 64 tokens (the module sends more than 16 tokens to the prefill path):
    seeds 0-3 at both taus, full layer shape, against the oracle (logits, selection, output,
    end-to-end masks against the literal reference)."""
    H, E, G = 1536, 64, 96
    for seed in range(4):
        L = make_layer(seed, H, E, G, tau)
        x = pkg().synth.make_tokens(seed, 64, H, stream=1)
        m = make_module(L, tau, cuda)
        out, lg, w = run_prefill(m, x, cuda)
        check(L, x, tau, out, lg, w, what=f"b64 tau{tau} s{seed}")
        y = m(x.view(1, 64, H).to(cuda)).view(64, H).cpu()  # the module takes the same path
        assert torch.equal(y, out)
