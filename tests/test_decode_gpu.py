"""GPU parity of the fused decode kernel and the selection kernel against the CPU oracle
and the reference's golden vectors (decode at batch 1..16)."""
import pytest
import torch
import torch.nn.functional as F

from conftest import MAX_ABS, MEAN_REL, assert_close_out, oracle, pkg
from gpu_helpers import (assert_mask_l2, assert_selection_matches, check_against_oracle, make_layer,
                         make_module, run_decode)

pytestmark = pytest.mark.gpu


def _align(v, a):
    return (v + a - 1) // a * a


def test_pack_layout(cuda):
    L = make_layer(3, hidden=256, experts=16, group=32, tau=0.7)
    m = make_module(L, 0.7, cuda)
    blob = m.packed().cpu()
    H, E, G = 256, 16, 32
    Wg, Wu, Wd, R = oracle().reference_layout(L)
    off = 0
    def take(n):
        nonlocal off
        t = blob[off:off + n * 2].view(torch.bfloat16)
        off = _align(off + n * 2, 1024)
        return t
    assert torch.equal(take(H * E).view(E, H), R.t())
    ex = take(E * G * 3 * H).view(E * G, 3, H)
    assert torch.equal(ex[:, 0], Wg.t())
    assert torch.equal(ex[:, 1], Wu.t())
    assert torch.equal(ex[:, 2], Wd)
    dt = take(E * G * H).view(E, H, G)
    assert torch.equal(dt, Wd.view(E, G, H).transpose(1, 2))
    assert off == pkg()._lib.load().ppmoe_packed_bytes(H, E, G)


def test_decode_golden_cases(golden, cuda):
    """Every golden case of <= 16 tokens: the reference's own outputs."""
    synth = pkg().synth
    for c in golden["cases"]:
        if c["tokens"] > 16:
            continue
        L = make_layer(c["seed"], c["hidden"], c["experts"], c["group"], c["tau"], c["router_scale"],
                       c.get("experts_id"))
        x = synth.make_tokens(c["seed"], c["tokens"], c["hidden"])
        m = make_module(L, c["tau"], cuda)
        out, lg, w = run_decode(m, x, cuda)
        check_against_oracle(L, x, c["tau"], out, lg, w, what=c["name"])
        # against the reference's own recorded selection (literal unstable sort on its own
        # logits): every differing token explained, the others' outputs within tolerance
        assert_mask_l2(x, L, c["tau"], lg, w, what=c["name"] + " vs reference golden", ref_logits=c["logits"])
        agree = ~((w > 0) != (c["weights"] > 0)).any(-1)
        if bool(agree.any()):
            assert_close_out(out[agree], c["out"][agree], c["name"] + " vs reference golden")


@pytest.mark.parametrize("tau", [0.70, 0.95])
@pytest.mark.parametrize("batch", [1, 4, 16])
def test_decode_sweep(cuda, batch, tau):
    """Batched decode (batch 1/4/16 x tau, seeds 0-3) at the full layer shape."""
    synth = pkg().synth
    stats = []
    for seed in range(4):
        L = make_layer(seed, tau=tau)
        x = synth.make_tokens(seed, batch, 1536, stream=1)
        m = make_module(L, tau, cuda)
        out, lg, w = run_decode(m, x, cuda)
        stats.append(check_against_oracle(L, x, tau, out, lg, w, what=f"b{batch} tau{tau} s{seed}"))
    # 1-ulp router rounding differences are rare (fp32 summation order only)
    assert sum(s[0] for s in stats) <= max(2, batch * 64 * 4 // 100)


def test_decode_small_and_pangu_shapes(cuda):
    synth = pkg().synth
    for (H, E, G, N, tau) in [(128, 16, 32, 3, 0.7), (256, 8, 128, 16, 0.95), (1536, 192, 32, 5, 0.7),
                              (2048, 64, 128, 2, 0.7), (4096, 32, 256, 1, 0.95), (1536, 256, 24, 7, 0.5)]:
        L = make_layer(11, H, E, G, tau)
        x = synth.make_tokens(11, N, H)
        m = make_module(L, tau, cuda)
        out, lg, w = run_decode(m, x, cuda)
        check_against_oracle(L, x, tau, out, lg, w, what=f"H{H} E{E} G{G} N{N}")


def test_decode_deterministic_and_counts(cuda):
    synth = pkg().synth
    L = make_layer(2, tau=0.7)
    m = make_module(L, 0.7, cuda)
    m.track_statistics = True
    x = synth.make_tokens(2, 9, 1536)
    o1, l1, w1 = run_decode(m, x, cuda)
    o2, l2, w2 = run_decode(m, x, cuda)
    assert torch.equal(o1, o2) and torch.equal(w1, w2)
    counts = m.activated_statistics.cpu()
    assert torch.equal(counts, 2 * oracle().activation_counts(w1))


def test_decode_zipf_bias(cuda):
    synth = pkg().synth
    L = make_layer(4, tau=0.7)
    m = make_module(L, 0.7, cuda)
    b = synth.zipf_bias(64, 1.2)
    x = synth.make_tokens(4, 8, 1536)
    out, lg, w = run_decode(m, x, cuda, bias=b.to(cuda))
    check_against_oracle(L, x, 0.7, out, lg, w, bias=b, what="zipf")


def test_repack_after_inplace_update(cuda):
    synth = pkg().synth
    L = make_layer(5, tau=0.95)
    m = make_module(L, 0.95, cuda)
    x = synth.make_tokens(5, 1, 1536)
    run_decode(m, x, cuda)
    with torch.no_grad():
        L.gate_w.mul_(-1.0)
        L.down_w.mul_(0.5)
        masks = F.one_hot(L.experts_id, 64).t()
        pkg().physical_reorder_for_inference(m, L.gate_w, L.up_w, L.down_w, L.router_w, masks, 0.95)
        m.W_up.data.mul_(2.0)  # in-place edit after mounting: must be picked up too
        L.up_w.mul_(2.0)
    out, lg, w = run_decode(m, x, cuda)
    check_against_oracle(L, x, 0.95, out, lg, w, what="repacked")


def test_module_forward_api(cuda):
    """TauSparseMoE.forward keeps the reference's [B,L,H] -> [B,L,H] bf16 contract."""
    synth = pkg().synth
    L = make_layer(6, tau=0.7)
    m = make_module(L, 0.7, cuda)
    x = synth.make_tokens(6, 6, 1536)
    y = m(x.view(2, 3, 1536).to(cuda).float())  # non-bf16 input is cast like tl:610
    assert y.shape == (2, 3, 1536) and y.dtype == torch.bfloat16
    out, lg, w = run_decode(m, x, cuda)
    assert torch.equal(y.view(6, 1536).cpu(), out)
    check_against_oracle(L, x, 0.7, out, lg, w, what="forward")
    with pytest.raises(RuntimeError):
        m(x.view(1, 6, 1536))  # CPU input


@pytest.mark.parametrize("E", [16, 64, 192, 256])
def test_route_logits_random(cuda, E):
    lib = pkg()._lib
    g = torch.Generator().manual_seed(E)
    lg = (torch.randn(2048, E, generator=g) * 2.5).to(torch.bfloat16)
    lg[::7, 1] = lg[::7, 0]  # exact ties
    for tau in (0.3, 0.7, 0.95, 1.0):
        w = torch.empty(2048, E, dtype=torch.bfloat16, device=cuda)
        mk = torch.empty(2048, E, dtype=torch.uint8, device=cuda)
        lgd = lg.to(cuda)
        lib.call("ppmoe_route_logits", lgd.data_ptr(), 2048, E, tau, w.data_ptr(), mk.data_ptr(),
                 torch.cuda.current_stream().cuda_stream)
        assert_selection_matches(w.cpu(), lg, tau, f"E{E} tau{tau}")
        w_ref, m_ref = oracle().softmax_thresholding(lg, tau)
        agree = (w.cpu() == w_ref).all(-1)
        assert torch.equal(mk.cpu().bool()[agree], m_ref[agree])


def test_route_logits_golden_ties(golden, cuda):
    lib = pkg()._lib
    T = golden["ties"]
    lg = T["logits"]
    n = lg.shape[0]
    for tau, d in T["taus"].items():
        w = torch.empty(n, 64, dtype=torch.bfloat16, device=cuda)
        lgd = lg.to(cuda)
        lib.call("ppmoe_route_logits", lgd.data_ptr(), n, 64, float(tau), w.data_ptr(), None,
                 torch.cuda.current_stream().cuda_stream)
        assert torch.equal(w.cpu(), d["stable"]), tau


@pytest.mark.parametrize("pinned", [True, False])
@pytest.mark.parametrize("batch", [1, 5])
def test_decode_host_buffers(cuda, batch, pinned):
    """ppmoe_decode_host returns exactly what ppmoe_decode returns for the same activations:
    pinned host buffers (the kernel reads and writes them over the host link) and pageable
    ones (staging copies on the stream)."""
    lib = pkg()._lib
    synth = pkg().synth
    L = make_layer(8, tau=0.95)
    m = make_module(L, 0.95, cuda)
    x = synth.make_tokens(8, batch, 1536)
    ref = m.forward_decode(x.to(cuda)).cpu()
    xh = x.pin_memory() if pinned else x.clone()
    oh = torch.empty(batch, 1536, dtype=torch.bfloat16)
    if pinned:
        oh = oh.pin_memory()
    xd = torch.empty(batch, 1536, dtype=torch.bfloat16, device=cuda)
    od = torch.empty_like(xd)
    ws = m.workspace(batch)
    s = torch.cuda.current_stream()
    lib.call("ppmoe_decode_host", xh.data_ptr(), batch, m.packed().data_ptr(), 1536, 64, 96, 0.95, None,
             oh.data_ptr(), xd.data_ptr(), od.data_ptr(), ws.data_ptr(), ws.numel(), s.cuda_stream)
    s.synchronize()
    m.check_device_status()
    assert torch.equal(oh, ref)


@pytest.mark.parametrize("tau", [0.3, 1.0])
@pytest.mark.parametrize("batch", [1, 2, 9])
def test_decode_extreme_tau(cuda, batch, tau):
    """tau 1.0 selects (nearly) every expert: one token then overflows the 24-slot
    single-token path and runs the CUDA-core path; tau 0.3 leaves mostly the forced top-1."""
    synth = pkg().synth
    L = make_layer(21, tau=0.95, scale=1.0)
    x = synth.make_tokens(21, batch, 1536)
    m = make_module(L, tau, cuda)
    out, lg, w = run_decode(m, x, cuda)
    check_against_oracle(L, x, tau, out, lg, w, what=f"b{batch} tau{tau}")
    if tau == 1.0:
        assert int((w > 0).sum(-1).min()) > 30


def test_decode_hidden_not_multiple_of_384(cuda):
    """H = 1152 (H % 384 != 0 for the batched tensor-core rounds): CUDA-core multi-token path."""
    synth = pkg().synth
    L = make_layer(22, 1152, 32, 64, 0.7)
    for n in (1, 6):
        x = synth.make_tokens(22, n, 1152)
        m = make_module(L, 0.7, cuda)
        out, lg, w = run_decode(m, x, cuda)
        check_against_oracle(L, x, 0.7, out, lg, w, what=f"H1152 N{n}")


@pytest.mark.parametrize("scale", [0.5, 1.0])
def test_decode_one_token_broad_selection(cuda, scale):
    """One token selecting most experts (flat router at tau 0.95): each CTA holds more neurons
    than the ring has slots, so the windowed path with slot refills runs."""
    L = make_layer(17, tau=0.95, scale=scale)
    m = make_module(L, 0.95, cuda)
    for s in range(3):
        x = pkg().synth.make_tokens(17 + s, 1, 1536)
        out, lg, w = run_decode(m, x, cuda)
        assert int((w > 0).sum()) > 30  # > 24 neurons per CTA: the windowed path
        check_against_oracle(L, x, 0.95, out, lg, w, what=f"broad s{scale} {s}")
