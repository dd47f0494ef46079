"""Expert-parallel prefill with the real kernels: one rank on one GPU (against the
single-device prefill), and 2 ranks over NCCL when two GPUs are visible."""
import datetime
import os
import sys

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from conftest import ROOT, assert_close_out, oracle, pkg
from gpu_helpers import assert_selection_matches, make_layer, make_module

pytestmark = pytest.mark.gpu


def _ep_module(L, tau, dev, bias=None):
    from importlib import import_module
    ep = import_module(pkg().__name__ + ".ep")
    m = make_module(L, tau, dev)
    return ep.ExpertParallelMoE(m.W_gate, m.W_up, m.W_down, m.router, L.experts, L.group, tau,
                                logit_bias=bias), m


# bf16 partials (optional reduced-traffic mode) round each rank's partial once more before
# the cross-rank sum: a looser, stated tolerance
BF16_PARTIALS_MAX_ABS, BF16_PARTIALS_MEAN_REL = 3e-2, 4e-3


def _close_loose(got, ref, what):
    d = (got.float() - ref.float()).abs()
    mean_rel = (d.sum() / ref.float().abs().sum()).item()
    assert d.max().item() <= BF16_PARTIALS_MAX_ABS and mean_rel <= BF16_PARTIALS_MEAN_REL, \
        f"{what}: max_abs={d.max().item():.3e} mean_rel={mean_rel:.3e}"


def test_ep_single_rank_matches_prefill(cuda):
    L = make_layer(12, 1536, 64, 96, 0.7)
    epm, m = _ep_module(L, 0.7, cuda)
    x = pkg().synth.make_tokens(12, 3000, 1536).to(cuda)
    y = epm(x).cpu()
    ref = m.forward_prefill(x).cpu()
    assert_close_out(y, ref, "ep(1) vs prefill")
    epm.chunks = 3  # chunking never changes a token's sum
    assert torch.equal(epm(x).cpu(), y)
    epm.partials = "bf16"
    _close_loose(epm(x).cpu(), ref, "ep(1) bf16 partials vs prefill")


@pytest.mark.parametrize("n,world,chunks", [(3000, 1, 1), (3000, 2, 2), (3000, 4, 3), (17, 8, 1), (4096, 8, 8)])
def test_ep_dispatch_kernel_matches_reference(cuda, n, world, chunks):
    """ppmoe_ep_dispatch (device send rows, counts, row table) equals its torch restatement
    byte for byte on the defined bytes of every row."""
    from importlib import import_module
    ep = import_module(pkg().__name__ + ".ep")
    L = make_layer(21, 1536, 64, 96, 0.7)
    x = pkg().synth.make_tokens(21, n, 1536)
    w, _ = oracle().softmax_thresholding(oracle().router_logits(x, L.router_w), 0.7)
    pitch = ep.row_pitch(1536, 64 // world)
    send_r, cnt_r, row_r = ep.dispatch_reference(x, w, world, chunks, pitch)
    m = ep.ExpertParallelMoE.__new__(ep.ExpertParallelMoE)
    m.world, m.H, m.E = world, 1536, 64
    send, cnt, row_of = m._dispatch(x.to(cuda), w.to(cuda), chunks, pitch)
    torch.cuda.synchronize()
    assert torch.equal(cnt.cpu(), cnt_r)
    assert torch.equal(row_of.cpu(), row_r)
    k = send_r.shape[0]
    used = 2 * (1536 + 64 // world)
    assert torch.equal(send[:k, :used].cpu(), send_r[:, :used])


def test_ep_single_rank_against_oracle(cuda):
    """Expert-parallel path (device dispatch, payload experts, combine) against the oracle on
    the first 256 tokens, logits teacher-forced from the routing call."""
    L = make_layer(14, 1536, 64, 96, 0.7)
    epm, m = _ep_module(L, 0.7, cuda)
    x = pkg().synth.make_tokens(14, 1024, 1536)
    y = epm(x.to(cuda)).cpu()
    xs = x[:256]
    lg = torch.empty(256, 64, dtype=torch.bfloat16, device=cuda)
    w = torch.empty(256, 64, dtype=torch.bfloat16, device=cuda)
    m.forward_prefill(xs.to(cuda), logits_out=lg, weights_out=w)
    ref = oracle().moe_mlp(xs, L, 0.7, logits=lg.cpu())
    assert_selection_matches(w.cpu(), lg.cpu(), 0.7, "ep(1) selection")
    assert_close_out(y[:256], ref.out, "ep(1) vs oracle")


def _nccl_worker(rank, world, port, q):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    sys.path.insert(0, ROOT)
    sys.path.insert(0, os.path.join(ROOT, "tests"))
    try:
        torch.cuda.set_device(rank)
        dev = torch.device("cuda", rank)
        dist.init_process_group("nccl", rank=rank, world_size=world, device_id=dev,
                                timeout=datetime.timedelta(seconds=60))
        P = pkg()
        L = make_layer(13, 1536, 64, 96, 0.7)
        b = P.synth.zipf_bias(64, 1.2)
        epm, single = _ep_module(L, 0.7, dev, bias=b.to(dev))
        x = P.synth.make_tokens(13, 4096, 1536)
        n = 4096 // world
        xs = x[rank * n:(rank + 1) * n].to(dev)
        y = epm(xs)
        epm.chunks = 1
        same = torch.equal(epm(xs), y)  # the chunked pipeline equals the unchunked path exactly
        epm.chunks, epm.partials = 2, "bf16"
        yb = epm(xs)
        outs = [torch.empty_like(y) for _ in range(world)]
        dist.all_gather(outs, y)
        outs_b = [torch.empty_like(yb) for _ in range(world)]
        dist.all_gather(outs_b, yb)
        ref = None
        if rank == 0:  # the single-device prefill on the whole batch, same router numerics
            single.logit_bias = b.to(dev)
            ref = single.forward_prefill(x.to(dev)).cpu()
        torch.cuda.synchronize()
        q.put((rank, "ok" if same else "chunked path differs",
               (torch.cat(outs).cpu(), ref, torch.cat(outs_b).cpu()) if rank == 0 else None))
    except Exception as e:  # noqa: BLE001
        q.put((rank, "err", repr(e)[:300]))
    finally:
        if dist.is_initialized():
            dist.destroy_process_group()


@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs 2 GPUs")
def test_ep_two_gpus_nccl():
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = 31000 + os.getpid() % 2000
    procs = [ctx.Process(target=_nccl_worker, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    res = dict((r, (s, v)) for r, s, v in (q.get(timeout=300) for _ in range(2)))
    for p in procs:
        p.join(timeout=60)
    assert res[0][0] == "ok" and res[1][0] == "ok", res
    y, ref, yb = res[0][1]
    assert_close_out(y, ref, "ep(2) vs single-device prefill")
    _close_loose(yb, ref, "ep(2) bf16 partials vs single-device prefill")


def test_ep_partial_formats(cuda):
    """The expert side's scaled-fp16 partial rows decode to the fp32 partial rows within fp16
    precision of each 64-column slice's maximum, and the source-side combine of those rows
    (ppmoe_ep_combine_f16s) equals the torch restatement bit for bit."""
    from importlib import import_module
    ep = import_module(pkg().__name__ + ".ep")
    L = make_layer(15, 1536, 64, 96, 0.7)
    epm, _ = _ep_module(L, 0.7, cuda)
    x = pkg().synth.make_tokens(15, 700, 1536).to(cuda)
    w = epm._route(x)
    send, cnt, row_of = epm._dispatch(x, w, 1, ep.row_pitch(1536, 64))
    rows = int(cnt.sum())
    p32 = epm._experts(send[:rows], 0)
    p16 = epm._experts(send[:rows], 1)
    assert p16.shape[1] == ep.f16s_pitch(1536) == pkg()._lib.load().ppmoe_ep_partial_pitch(1536)
    dec = ep.f16s_decode(p16.cpu(), 1536).view(rows, 24, 64)
    ref = p32.cpu().view(rows, 24, 64)
    bound = ref.abs().amax(-1, keepdim=True) * 2.0 ** -11
    assert bool(((dec - ref).abs() <= bound).all())
    used = 2 * 1536 + 1536 // 64  # defined bytes of a row (the 16-byte padding is not written)
    assert torch.equal(ep.f16s_encode(p32.cpu())[:, :used], p16.cpu()[:, :used])  # restatement == kernel
    y = ep.combine_partials(p16, row_of, 700, 1536).cpu()
    y_ref = ep.combine_partials(p16.cpu(), row_of.cpu(), 700, 1536)
    assert torch.equal(y, y_ref)


@pytest.mark.parametrize("experts", [8, 16])
def test_ep_local_layer_sizes_of_8_and_4_ranks(cuda, experts):
    """A rank of 8-way (4-way) expert parallelism at E = 64 holds 8 (16) experts: the same
    expert-side kernels on a layer of that many experts, against the oracle."""
    L = make_layer(16, 1536, experts, 96, 0.7)
    epm, m = _ep_module(L, 0.7, cuda)
    x = pkg().synth.make_tokens(16, 600, 1536)
    y = epm(x.to(cuda)).cpu()
    lg = torch.empty(600, experts, dtype=torch.bfloat16, device=cuda)
    w = torch.empty(600, experts, dtype=torch.bfloat16, device=cuda)
    m.forward_prefill(x.to(cuda), logits_out=lg, weights_out=w)
    ref = oracle().moe_mlp(x, L, 0.7, logits=lg.cpu())
    assert_selection_matches(w.cpu(), lg.cpu(), 0.7, f"E={experts} selection")
    assert_close_out(y, ref.out, f"ep(1) E={experts} vs oracle")
