"""GradSync host logic on CPU ranks (gloo, world 2).

The layer's backward needs a B200; here a stand-in backward writes known
values into the destinations GradSync hands out and calls its two callbacks
at the points the real backward does (expert gradients final, then the
router gradient).  Checked: the parameters' .grad is the flat buffer's view;
after wait() every rank holds the average over ranks (DDP's reduction);
a second backward without zero_grad is told to accumulate; no_sync() reduces
nothing and the next synced backward reduces the accumulated sum; a .grad
replaced by a foreign tensor is refused."""

import os
import socket
from types import SimpleNamespace

import torch
import torch.distributed as dist
import torch.multiprocessing as mp
import torch.nn as nn


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _layer():
    m = nn.Module()
    m.gate = nn.Module()
    m.gate.weight = nn.Parameter(torch.zeros(4, 8))
    m.experts = nn.Module()
    m.experts.gate_up_proj = nn.Parameter(torch.zeros(4, 6, 8))
    m.experts.down_proj = nn.Parameter(torch.zeros(4, 8, 3))
    return m


def _fake_backward(sync, scale):
    g = sync.begin()
    for t, v, a in ((g.gate_up, 1.0, g.accumulate[1]), (g.down, 2.0, g.accumulate[2])):
        t.add_(v * scale) if a else t.fill_(v * scale)
    beside = g.experts_ready()
    assert beside is None  # no SM limit on CPU
    (g.router.add_ if g.accumulate[0] else g.router.fill_)(3.0 * scale)
    g.router_ready()
    return g.accumulate


def _worker(rank, world, port, results):
    from datetime import timedelta
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=timedelta(seconds=20))
    try:
        from spark_gpt_b200.grad_sync import GradSync
        m = _layer()
        sync = GradSync(m)
        out = {}
        acc = _fake_backward(sync, rank + 1)
        sync.wait()
        out["first_acc"] = acc
        out["is_view"] = all(p.grad.data_ptr() == v.data_ptr()
                             for p, v in zip(sync.params, sync.views))
        out["avg"] = [float(m.experts.gate_up_proj.grad.mean()),
                      float(m.experts.down_proj.grad.mean()), float(m.gate.weight.grad.mean())]
        for p in m.parameters():
            p.grad = None
        with sync.no_sync():
            _fake_backward(sync, rank + 1)
            sync.wait()
            out["local"] = float(m.experts.gate_up_proj.grad.mean())
        out["second_acc"] = _fake_backward(sync, rank + 1)   # accumulates, then reduces
        sync.wait()
        out["accumulated"] = [float(m.experts.gate_up_proj.grad.mean()),
                              float(m.gate.weight.grad.mean())]
        m.gate.weight.grad = torch.zeros(4, 8)
        try:
            sync.begin()
            out["foreign"] = None
        except RuntimeError as e:
            out["foreign"] = str(e)
        results[rank] = out
    finally:
        dist.destroy_process_group()


def test_grad_sync_averages_accumulates_and_defers():
    mgr = mp.get_context("spawn").Manager()
    results = mgr.dict()
    mp.start_processes(_worker, args=(2, _free_port(), results), nprocs=2, join=True,
                       start_method="spawn")
    for rank in range(2):
        r = results[rank]
        assert r["first_acc"] == (False, False, False)
        assert r["is_view"]
        assert r["avg"] == [1.5, 3.0, 4.5]           # mean of rank 1 and rank 2 scales
        assert r["local"] == 1.0 * (rank + 1)        # no_sync: nothing reduced
        assert r["second_acc"] == (True, True, True)
        # local sum of two backward passes, averaged over ranks: (2*1 + 2*2) / 2
        assert r["accumulated"] == [3.0, 9.0]
        assert r["foreign"] is not None and "replaced" in r["foreign"]
