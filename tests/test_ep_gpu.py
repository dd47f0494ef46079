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
from gpu_helpers import make_layer, make_module

pytestmark = pytest.mark.gpu


def _ep_module(L, tau, dev, bias=None):
    from importlib import import_module
    ep = import_module(pkg().__name__ + ".ep")
    m = make_module(L, tau, dev)
    return ep.ExpertParallelMoE(m.W_gate, m.W_up, m.W_down, m.router, L.experts, L.group, tau,
                                logit_bias=bias), m


def test_ep_single_rank_matches_prefill(cuda):
    L = make_layer(12, 1536, 64, 96, 0.7)
    epm, m = _ep_module(L, 0.7, cuda)
    x = pkg().synth.make_tokens(12, 3000, 1536).to(cuda)
    y = epm(x).cpu()
    ref = m.forward_prefill(x).cpu()
    assert_close_out(y, ref, "ep(1) vs prefill")


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
        y = epm(x[rank * n:(rank + 1) * n].to(dev))
        outs = [torch.empty_like(y) for _ in range(world)]
        dist.all_gather(outs, y)
        ref = None
        if rank == 0:  # the single-device prefill on the whole batch, same router numerics
            single.logit_bias = b.to(dev)
            ref = single.forward_prefill(x.to(dev)).cpu()
        torch.cuda.synchronize()
        q.put((rank, "ok", (torch.cat(outs).cpu(), ref) if rank == 0 else None))
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
    y, ref = res[0][1]
    assert_close_out(y, ref, "ep(2) vs single-device prefill")
