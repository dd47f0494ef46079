"""Expert-parallel prefill host logic on CPU ranks (gloo, world size 2 and 4): dispatch plan, count
and payload exchange, partial return, deterministic combine.  Kernels are replaced by CPU
stand-ins built from the oracle; the GPU path is covered by tests/test_ep_gpu.py."""
import datetime
import os
import sys

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp
import torch.nn.functional as F

from conftest import MAX_ABS, MEAN_REL, ROOT, oracle, pkg


def _cpu_route(L, tau):
    O = oracle()

    def route(x):
        w, _ = O.softmax_thresholding(O.router_logits(x, L.router_w), tau)
        return w
    return route


def _cpu_experts(L):
    masks = F.one_hot(L.experts_id, L.experts).t().to(torch.bfloat16)  # [E, I]

    def experts(xr, wr, own):
        inter = F.silu(F.linear(xr, L.gate_w)) * F.linear(xr, L.up_w)
        nm = wr @ masks[own]
        return F.linear((inter * nm).float(), L.down_w.float())
    return experts


def _worker(rank, world, port, q, mode):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    sys.path.insert(0, ROOT)
    sys.path.insert(0, os.path.join(ROOT, "tests"))
    try:
        dist.init_process_group("gloo", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=15))
        P = pkg()
        from importlib import import_module
        ep = import_module(P.__name__ + ".ep")
        L = P.synth.make_layer(8, 128, 16, 32, router_scale=1.75)
        x = P.synth.make_tokens(8, 96, 128)
        n = 96 // world
        shard = x[rank * n:(rank + 1) * n]
        # with injected kernels the layer only needs its shapes (no device weights)
        m = ep.ExpertParallelMoE.__new__(ep.ExpertParallelMoE)
        m.group, m.world, m.rank = None, world, rank
        m.H, m.E, m.G, m.tau, m.el = 128, 16, 32, 0.7, 16 // world
        m.route_fn, m.expert_fn, m.local, m.last_stats = _cpu_route(L, 0.7), _cpu_experts(L), None, {}
        if mode == "fail" and rank == 1:
            raise RuntimeError("injected failure before dispatch")
        y = m(shard)
        outs = [torch.empty_like(y) for _ in range(world)]
        dist.all_gather(outs, y)
        q.put((rank, "ok", torch.cat(outs) if rank == 0 else None))
    except Exception as e:  # noqa: BLE001 - reported to the parent
        q.put((rank, "err", repr(e)[:200]))
    finally:
        if dist.is_initialized():
            try:
                dist.destroy_process_group()
            except Exception:  # noqa: BLE001
                pass


def _run(mode, world=2):
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = 29500 + (os.getpid() % 2000)
    procs = [ctx.Process(target=_worker, args=(r, world, port, q, mode)) for r in range(world)]
    for p in procs:
        p.start()
    res = {}
    for _ in range(world):
        r, status, payload = q.get(timeout=120)
        res[r] = (status, payload)
    for p in procs:
        p.join(timeout=60)
    return res


@pytest.mark.parametrize("world", [2, 4])
def test_ep_ranks_match_oracle(world):
    res = _run("ok", world)
    assert all(res[r][0] == "ok" for r in range(world)), res
    y = res[0][1]
    P = pkg()
    L = P.synth.make_layer(8, 128, 16, 32, router_scale=1.75)
    x = P.synth.make_tokens(8, 96, 128)
    ref = oracle().moe_mlp(x, L, 0.7).out
    d = (y.float() - ref.float()).abs()
    assert d.max() <= MAX_ABS and d.sum() / ref.float().abs().sum() <= MEAN_REL


def test_ep_rank_failure_surfaces_as_error():
    res = _run("fail")
    assert res[1][0] == "err" and "injected" in res[1][1]
    assert res[0][0] == "err"  # the surviving rank's collective fails instead of hanging


def test_dispatch_reference_and_combine_single_process():
    ep = __import__(pkg().__name__ + ".ep", fromlist=["x"])
    w = torch.zeros(5, 8, dtype=torch.bfloat16)
    w[0, 1] = 0.5; w[0, 6] = 0.25; w[2, 5] = 1.0; w[3, 0] = 0.75; w[4, 7] = 0.5; w[4, 4] = 0.5
    x = torch.arange(5 * 8, dtype=torch.float32).view(5, 8).to(torch.bfloat16)
    pitch = ep.row_pitch(8, 4)
    assert pitch == 32
    # snake assignment at 2 ranks: rank 0 owns experts 0, 3, 4, 7; rank 1 owns 1, 2, 5, 6
    assert ep.owned_experts(8, 2, 0).tolist() == [0, 3, 4, 7] and ep.owned_experts(8, 2, 1).tolist() == [1, 2, 5, 6]
    send, cnt, row_of = ep.dispatch_reference(x, w, 2, 1, pitch)
    assert cnt.tolist() == [[2], [2]]
    assert row_of.tolist() == [[-1, -1, -1, 0, 1], [2, -1, 3, -1, -1]]
    v = send.view(torch.bfloat16)
    assert torch.equal(v[:, :8], x[[3, 4, 0, 2]])
    sw = v[:, 8:12].float()
    assert sw[0].tolist() == [0.75, 0.0, 0.0, 0.0] and sw[1].tolist() == [0.0, 0.0, 0.5, 0.5]
    assert sw[2].tolist() == [0.5, 0.0, 0.0, 0.25] and sw[3].tolist() == [0.0, 0.0, 1.0, 0.0]
    back = torch.arange(4 * 3, dtype=torch.float32).view(4, 3)
    out = ep.combine_partials(back, row_of, 5)
    assert out[0].float().tolist() == back[2].tolist()
    assert out[4].float().tolist() == back[1].tolist()
    assert out[3].float().tolist() == back[0].tolist()
    assert out[1].float().abs().sum() == 0


def test_dispatch_reference_chunks():
    """Chunks are whole 256-token blocks; rows chunk-major, then destination-major."""
    ep = __import__(pkg().__name__ + ".ep", fromlist=["x"])
    assert ep.chunk_bounds(600, 2) == [0, 256, 600] and ep.chunk_bounds(600, 3) == [0, 256, 512, 600]
    g = torch.Generator().manual_seed(3)
    w = (torch.rand(600, 16, generator=g) > 0.7).to(torch.bfloat16) * 0.5
    x = torch.randn(600, 64, generator=g).to(torch.bfloat16)
    send, cnt, row_of = ep.dispatch_reference(x, w, 4, 3, ep.row_pitch(64, 4))
    b = ep.chunk_bounds(600, 3)
    pos = 0
    for c in range(3):
        for d in range(4):
            k = int(cnt[d, c])
            toks = [t for t in range(b[c], b[c + 1]) if bool((w[t, ep.owned_experts(16, 4, d)] > 0).any())]
            assert len(toks) == k
            assert row_of[d, toks].tolist() == list(range(pos, pos + k))
            pos += k
    assert send.shape[0] == pos


def test_snake_assignment_partitions_and_balances():
    """Every expert has exactly one owner; against a load falling with the expert index the
    snake order spreads the load more evenly than a plain stride."""
    ep = __import__(pkg().__name__ + ".ep", fromlist=["x"])
    for E, P in [(64, 2), (64, 4), (64, 8), (16, 4), (192, 8)]:
        owned = torch.cat([ep.owned_experts(E, P, r) for r in range(P)])
        assert sorted(owned.tolist()) == list(range(E))
    load = torch.exp(-1.2 * torch.log(torch.arange(1, 65, dtype=torch.float64)))  # Zipf(1.2) prior
    for P in (2, 4, 8):
        snake = torch.stack([load[ep.owned_experts(64, P, r)].sum() for r in range(P)])
        stride = torch.stack([load[r::P].sum() for r in range(P)])
        assert (snake.max() / snake.min()) < (stride.max() / stride.min())


def test_f16s_round_trip_bound():
    """Scaled-fp16 partial rows: every value within 2^-11 of its 64-column slice's maximum,
    zeros and all-zero slices exact, and magnitudes far outside fp16's range survive."""
    ep = __import__(pkg().__name__ + ".ep", fromlist=["x"])
    g = torch.Generator().manual_seed(4)
    x = torch.randn(37, 256, generator=g) * torch.logspace(-20, 20, 37)[:, None]
    x[3] = 0.0
    x[5, :64] = 0.0
    enc = ep.f16s_encode(x)
    assert enc.shape == (37, ep.f16s_pitch(256)) and ep.f16s_pitch(256) % 16 == 0
    dec = ep.f16s_decode(enc, 256)
    bound = x.abs().view(37, 4, 64).amax(-1, keepdim=True) * 2.0 ** -11
    assert bool(((dec - x).view(37, 4, 64).abs() <= bound).all())
    assert bool((dec[3] == 0).all()) and bool((dec[5, :64] == 0).all())
    assert bool(torch.isfinite(dec).all())
