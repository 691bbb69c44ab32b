"""Expert-parallel orchestration on CPU ranks (gloo, world sizes 2 and 4).

spark_gpt_b200.ep.ExpertParallelMoE is driven with an oracle-backed ops
object in place of the device kernels, so the routing, the per-(token, rank)
send plan, the all_to_all_single exchanges, the owner-side partial combine and
the backward's reverse exchanges are checked on CPU: every rank's output and
input gradient must equal the single-process oracle layer on that rank's
tokens, and each rank's expert-shard gradients must equal the oracle's
gradients of those experts summed over all ranks' tokens.  Also: ranks with
different token counts (one with none), and a rank that fails before its
first exchange (its peer gets an error, not a hang).  Test infrastructure
only: the product path runs the CUDA kernels.
"""

import contextlib
import os
import socket
from types import SimpleNamespace

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from oracle import moe_oracle as O


class OracleOps:
    """CPU stand-in for spark_gpt_b200.ep.CudaExpertOps (fp32 oracle math).

    Same send plan as the device path: one row per (token, destination rank)
    in rank-major, token order, with the row's k slots marked by local expert
    id (or -1) and routing weight; slot words are fp32 pairs here."""

    @staticmethod
    def router(x, w_router, num_experts, top_k, norm):
        logits = x.float() @ w_router.float().t()
        probs, w, sel = O.router_select(logits, top_k, norm)
        return logits, w_router.float(), sel, w

    @staticmethod
    def router_bwd(x, wr, logits_buf, sel, d_rw, d_logits, num_experts, top_k, norm):
        probs = O.softmax_fp32(logits_buf)
        _, dx, dwr = O.router_backward(x, wr, probs, None, sel, d_rw, norm,
                                       d_logits_extra=d_logits)
        return dx, dwr

    @staticmethod
    def send_plan(sel, rw, experts_per_rank, ranks):
        T, k = sel.shape
        dest = torch.div(sel, experts_per_rank, rounding_mode="floor")
        mask = torch.zeros(T, ranks, dtype=torch.bool)
        mask[torch.arange(T).unsqueeze(1).expand(T, k), dest] = True
        pairs = mask.t().nonzero()                     # (rank, token), rank-major
        rank_of, tok = pairs[:, 0], pairs[:, 1]
        inv = torch.full((T, ranks), -1, dtype=torch.int64)
        inv[tok, rank_of] = torch.arange(len(tok))
        mine = dest[tok] == rank_of.unsqueeze(1)       # (rows, k)
        ids = torch.where(mine, sel[tok] % experts_per_rank, torch.full_like(sel[tok], -1))
        w = torch.where(mine, rw[tok].float(), torch.zeros(()))
        meta = torch.cat([ids.float(), w], 1)
        sizes = torch.stack([mask.sum(0), torch.bincount(dest.reshape(-1), minlength=ranks)], 1)
        plan = SimpleNamespace(tok=tok, inv=inv, k=k, experts_per_rank=experts_per_rank,
                               meta=meta)
        return plan, sizes.to(torch.int64)

    @staticmethod
    def pack_rows(src, plan):
        return src.float()[plan.tok]

    @staticmethod
    def unpack(meta):
        k = meta.shape[1] // 2
        return meta[:, :k].long(), meta[:, k:]

    @staticmethod
    def experts_fwd(rows, sel_loc, w_loc, w_gu, w_d, slots):
        row_of, slot_of = (sel_loc >= 0).nonzero(as_tuple=True)
        ids = sel_loc[row_of, slot_of]
        n = len(ids)
        d = O.dispatch(ids.view(n, 1), w_gu.shape[0])
        perm = torch.from_numpy(d.permutation)
        xs = rows.float()[row_of][perm]
        gu, h = O.swiglu_forward(xs, w_gu, d.offsets)
        y = O.grouped_linear_forward(h, w_d, d.offsets)[torch.from_numpy(d.inverse)]
        w = w_loc[row_of, slot_of].unsqueeze(1)
        part = torch.zeros(rows.shape[0], rows.shape[1]).index_add_(0, row_of, y * w)
        return part, (d, row_of, slot_of, w, xs, gu, h, y, w_gu, w_d)

    @staticmethod
    def experts_dgrad(ctx, d_rows, k, device):
        d, row_of, slot_of, w, xs, gu, h, y, w_gu, w_d = ctx
        g = d_rows.float()[row_of]
        dw = torch.zeros(d_rows.shape[0], k)
        dw[row_of, slot_of] = (g * y).sum(-1)
        perm = torch.from_numpy(d.permutation)
        dy = (g * w)[perm]
        dh, dwd = O.grouped_linear_backward(h, w_d, dy, d.offsets)
        dxs, dwgu, _ = O.swiglu_backward(xs, w_gu, gu, dh, d.offsets)
        dxs = dxs[torch.from_numpy(d.inverse)]
        dx = torch.zeros(d_rows.shape[0], d_rows.shape[1]).index_add_(0, row_of, dxs)
        return dx, dw, (dwgu, dwd)

    @staticmethod
    def experts_wgrad(state, g_gu, g_d, E, H, I, device):
        dwgu, dwd = state
        if g_gu is None:
            return dwgu, dwd
        return g_gu + dwgu, g_d + dwd

    @staticmethod
    def reduce_rows(rows_back, plan, addend=None, out=None):
        T, P = plan.inv.shape
        res = torch.zeros(T, rows_back.shape[1])
        has = plan.inv >= 0
        t_idx, r_idx = has.nonzero(as_tuple=True)
        res.index_add_(0, t_idx, rows_back.float()[plan.inv[t_idx, r_idx]])
        if addend is not None:
            res = res + addend
        if out is None:
            return res
        out.copy_(res)
        return out

    @staticmethod
    def weight_grad(dw_back, plan, sel, out=None):
        T, k = sel.shape
        r = torch.div(sel, plan.experts_per_rank, rounding_mode="floor")
        rows = plan.inv[torch.arange(T).unsqueeze(1), r]
        res = dw_back[rows, torch.arange(k).unsqueeze(0)]
        if out is None:
            return res
        out.copy_(res)
        return out

    @staticmethod
    def overlap(comm_sms):
        return contextlib.nullcontext()

    @staticmethod
    def cast(w):
        return w.float()


T, H, E, K, I = 48, 32, 8, 3, 16


def full_weights():
    g = torch.Generator().manual_seed(7)
    return (torch.randn(E, H, generator=g) * 0.5, torch.randn(E, 2 * I, H, generator=g) * 0.2,
            torch.randn(E, H, I, generator=g) * 0.2)


def rank_inputs(rank, tokens=T):
    g = torch.Generator().manual_seed(100 + rank)
    return torch.randn(tokens, H, generator=g), torch.randn(tokens, H, generator=g)


def _worker(rank, world, port, results, chunks, tokens=None):
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        from spark_gpt_b200.ep import ExpertParallelMoE
        cfg = SimpleNamespace(hidden_size=H, num_experts=E, num_experts_per_tok=K,
                              moe_intermediate_size=I, norm_topk_prob=True)
        m = ExpertParallelMoE(cfg, backend=OracleOps, chunks=chunks, comm_sms=8)
        w_r, w_gu, w_d = full_weights()
        lo, hi = m.expert_offset, m.expert_offset + m.local_experts
        with torch.no_grad():
            m.gate.weight.copy_(w_r)
            m.experts.gate_up_proj.copy_(w_gu[lo:hi])
            m.experts.down_proj.copy_(w_d[lo:hi])
        x, d_out = rank_inputs(rank, tokens[rank] if tokens else T)
        xin = x.clone().requires_grad_(True)
        out, logits, sel = m(xin)
        out.backward(d_out)
        results[rank] = {
            "out": out.detach(), "sel": sel, "dx": xin.grad, "dW_router": m.gate.weight.grad,
            "dW_gu": m.experts.gate_up_proj.grad, "dW_d": m.experts.down_proj.grad,
            "lo": lo, "hi": hi}
    finally:
        dist.destroy_process_group()


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


@pytest.mark.parametrize("world,chunks", [(2, 1), (4, 1), (2, 3)])
def test_expert_parallel_matches_single_process_oracle(world, chunks):
    mgr = mp.get_context("spawn").Manager()
    results = mgr.dict()
    mp.start_processes(_worker, args=(world, _free_port(), results, chunks), nprocs=world,
                       join=True, start_method="spawn")
    w_r, w_gu, w_d = full_weights()
    sum_gu = torch.zeros_like(w_gu)
    sum_d = torch.zeros_like(w_d)
    for rank in range(world):
        r = results[rank]
        x, d_out = rank_inputs(rank)
        ref = O.layer_forward_backward(x, w_r, w_gu, w_d, K, d_out)
        assert torch.equal(r["sel"], ref["selected"])
        torch.testing.assert_close(r["out"], ref["out"], rtol=1e-5, atol=1e-6)
        torch.testing.assert_close(r["dx"], ref["dx"], rtol=1e-5, atol=1e-6)
        torch.testing.assert_close(r["dW_router"], ref["dW_router"], rtol=1e-5, atol=1e-6)
        sum_gu += ref["dW_gate_up"]
        sum_d += ref["dW_down"]
    for rank in range(world):
        r = results[rank]
        torch.testing.assert_close(r["dW_gu"], sum_gu[r["lo"]:r["hi"]], rtol=1e-5, atol=1e-6)
        torch.testing.assert_close(r["dW_d"], sum_d[r["lo"]:r["hi"]], rtol=1e-5, atol=1e-6)
    # every expert received rows from both ranks in this routing
    assert np.all(np.bincount(torch.cat([results[r]["sel"].reshape(-1) for r in range(world)]),
                              minlength=E) > 0)


def _ckpt_worker(rank, world, port, results):
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        from spark_gpt_b200.ep import ExpertParallelMoE
        cfg = SimpleNamespace(hidden_size=H, num_experts=E, num_experts_per_tok=K,
                              moe_intermediate_size=I, norm_topk_prob=True)
        w_r, w_gu, w_d = full_weights()
        full = {"gate.weight": w_r, "experts.gate_up_proj": w_gu, "experts.down_proj": w_d}
        m = ExpertParallelMoE(cfg, backend=OracleOps)
        m.load_full_state_dict(full)
        got = m.full_state_dict()
        sd = m.state_dict()
        m2 = ExpertParallelMoE(cfg, backend=OracleOps)
        m2.load_state_dict(sd)                      # same layout: loads
        mismatch = None
        try:
            bad = dict(sd)
            bad["_extra_state"] = {**sd["_extra_state"], "expert_parallel_ranks": world * 2}
            m2.load_state_dict(bad)
        except ValueError as e:
            mismatch = str(e)
        results[rank] = {"full": {k: v.clone() for k, v in got.items()},
                         "shard_gu": sd["experts.gate_up_proj"].clone(),
                         "m2_gu": m2.experts.gate_up_proj.detach().clone(),
                         "keys": sorted(sd.keys()), "mismatch": mismatch,
                         "lo": m.expert_offset, "hi": m.expert_offset + m.local_experts}
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("world", [2, 4])
def test_expert_shards_round_trip_to_the_full_layout(world):
    """full_state_dict gathers the reference's (E,2I,H)/(E,H,I) tensors from the
    shards; load_full_state_dict slices them back; a shard's state dict carries
    its layout and refuses to load into another one."""
    mgr = mp.get_context("spawn").Manager()
    results = mgr.dict()
    mp.start_processes(_ckpt_worker, args=(world, _free_port(), results), nprocs=world,
                       join=True, start_method="spawn")
    w_r, w_gu, w_d = full_weights()
    for rank in range(world):
        r = results[rank]
        assert torch.equal(r["full"]["gate.weight"], w_r)
        assert torch.equal(r["full"]["experts.gate_up_proj"], w_gu)
        assert torch.equal(r["full"]["experts.down_proj"], w_d)
        assert sorted(r["full"]) == ["experts.down_proj", "experts.gate_up_proj", "gate.weight"]
        assert torch.equal(r["shard_gu"], w_gu[r["lo"]:r["hi"]])
        assert torch.equal(r["m2_gu"], w_gu[r["lo"]:r["hi"]])
        assert "_extra_state" in r["keys"]
        assert r["mismatch"] is not None and "cannot load" in r["mismatch"]


@pytest.mark.parametrize("tokens", [(48, 17), (0, 48), (31, 48, 5, 0)])
def test_expert_parallel_ranks_with_different_token_counts(tokens):
    """Ranks holding different numbers of tokens (one of them none): the counts
    exchange sizes every buffer, and each rank's results still equal the
    single-process oracle on its own tokens."""
    world = len(tokens)
    mgr = mp.get_context("spawn").Manager()
    results = mgr.dict()
    mp.start_processes(_worker, args=(world, _free_port(), results, 1, list(tokens)),
                       nprocs=world, join=True, start_method="spawn")
    w_r, w_gu, w_d = full_weights()
    sum_gu = torch.zeros_like(w_gu)
    sum_d = torch.zeros_like(w_d)
    for rank in range(world):
        r = results[rank]
        assert r["out"].shape == (tokens[rank], H) and r["dx"].shape == (tokens[rank], H)
        if tokens[rank] == 0:
            continue
        x, d_out = rank_inputs(rank, tokens[rank])
        ref = O.layer_forward_backward(x, w_r, w_gu, w_d, K, d_out)
        torch.testing.assert_close(r["out"], ref["out"], rtol=1e-5, atol=1e-6)
        torch.testing.assert_close(r["dx"], ref["dx"], rtol=1e-5, atol=1e-6)
        sum_gu += ref["dW_gate_up"]
        sum_d += ref["dW_down"]
    for rank in range(world):
        r = results[rank]
        torch.testing.assert_close(r["dW_gu"], sum_gu[r["lo"]:r["hi"]], rtol=1e-5, atol=1e-6)
        torch.testing.assert_close(r["dW_d"], sum_d[r["lo"]:r["hi"]], rtol=1e-5, atol=1e-6)


def _failing_worker(rank, world, port, results):
    """Rank 1 raises before its first exchange; rank 0 must get an error from
    the process group (its short timeout, or the closed connection) instead of
    waiting for good."""
    import time
    from datetime import timedelta
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=timedelta(seconds=5))
    from spark_gpt_b200.ep import ExpertParallelMoE
    cfg = SimpleNamespace(hidden_size=H, num_experts=E, num_experts_per_tok=K,
                          moe_intermediate_size=I, norm_topk_prob=True)
    m = ExpertParallelMoE(cfg, backend=OracleOps)
    w_r, w_gu, w_d = full_weights()
    with torch.no_grad():
        m.gate.weight.copy_(w_r)
        m.experts.gate_up_proj.copy_(w_gu[m.expert_offset:m.expert_offset + m.local_experts])
        m.experts.down_proj.copy_(w_d[m.expert_offset:m.expert_offset + m.local_experts])
    if rank == 1:
        results[rank] = {"error": "planted failure before the first exchange", "seconds": 0.0}
        return  # leaves without joining any collective (no destroy, no barrier)
    t0 = time.monotonic()
    try:
        m(rank_inputs(rank)[0])
        results[rank] = {"error": None, "seconds": time.monotonic() - t0}
    except Exception as e:  # noqa: BLE001 - the failure is the point
        results[rank] = {"error": f"{type(e).__name__}: {e}", "seconds": time.monotonic() - t0}


def test_a_rank_that_fails_surfaces_as_an_error_not_a_hang():
    mgr = mp.get_context("spawn").Manager()
    results = mgr.dict()
    mp.start_processes(_failing_worker, args=(2, _free_port(), results), nprocs=2, join=True,
                       start_method="spawn")
    assert results[1]["error"].startswith("planted")
    assert results[0]["error"] is not None, "rank 0 finished an exchange its peer never joined"
    assert results[0]["seconds"] < 60


def _mismatch_worker(rank, world, port, results):
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    from datetime import timedelta
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=timedelta(seconds=20))
    try:
        from spark_gpt_b200.ep import ExpertParallelMoE
        experts = E if rank == 0 else 2 * E     # rank 1 is configured differently
        cfg = SimpleNamespace(hidden_size=H, num_experts=experts, num_experts_per_tok=K,
                              moe_intermediate_size=I, norm_topk_prob=True)
        m = ExpertParallelMoE(cfg, backend=OracleOps)
        g = torch.Generator().manual_seed(rank)
        with torch.no_grad():
            for p in m.parameters():
                p.copy_(torch.randn(p.shape, generator=g) * 0.1)
        try:
            m(rank_inputs(rank)[0])
            results[rank] = None
        except ValueError as e:
            results[rank] = str(e)
    finally:
        dist.destroy_process_group()


def test_ranks_with_different_layer_configurations_all_raise():
    """A rank built with a different number of experts (so a different expert
    -> rank map): every rank sees it in the counts exchange and raises the same
    error before any row moves, instead of routing rows to experts that are
    not there."""
    mgr = mp.get_context("spawn").Manager()
    results = mgr.dict()
    mp.start_processes(_mismatch_worker, args=(2, _free_port(), results), nprocs=2, join=True,
                       start_method="spawn")
    for rank in range(2):
        assert results[rank] is not None and "disagree on the layer configuration" in results[rank]


def test_construction_rejects_what_a_transport_cannot_run():
    """Checked on the host before any collective: experts that do not split
    over the ranks, and the peer-memory transport at a hidden size its
    combine-and-return kernel does not take."""
    from datetime import timedelta
    from spark_gpt_b200.ep import ExpertParallelMoE
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(_free_port())
    dist.init_process_group("gloo", rank=0, world_size=1, timeout=timedelta(seconds=20))
    try:
        cfg = SimpleNamespace(hidden_size=768, num_experts=8, num_experts_per_tok=2,
                              moe_intermediate_size=384, norm_topk_prob=True)
        with pytest.raises(ValueError, match="transport='nccl'"):
            ExpertParallelMoE(cfg, transport="p2p")
        m = ExpertParallelMoE(cfg, transport="nccl")
        assert m.local_experts == 8
        with pytest.raises(ValueError, match="transport must be"):
            ExpertParallelMoE(cfg, transport="shm")
    finally:
        dist.destroy_process_group()


def test_peer_transports_are_kept_per_group_shape_and_chunk():
    """One transport per (group, H, k, device, chunk slot), found again by the
    group's name; creating one allocates nothing (buffers come with the first
    forward)."""
    from datetime import timedelta
    from spark_gpt_b200.ep import PeerTransport
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(_free_port())
    dist.init_process_group("gloo", rank=0, world_size=1, timeout=timedelta(seconds=20))
    try:
        sub = dist.new_group([0])
        a = PeerTransport.get(None, 1024, 8, "cpu")
        assert PeerTransport.get(dist.group.WORLD, 1024, 8, "cpu") is a
        assert PeerTransport.get(None, 1024, 8, "cpu", slot=1) is not a
        assert PeerTransport.get(None, 2048, 8, "cpu") is not a
        b = PeerTransport.get(sub, 1024, 8, "cpu")
        assert b is not a and PeerTransport.get(sub, 1024, 8, "cpu") is b
        assert a.cap == 0 and a.P == 1 and a.me == 0
    finally:
        PeerTransport._cache.clear()
        dist.destroy_process_group()


def test_peer_transport_is_rebuilt_for_a_group_created_after_destroy():
    """torch restarts its group-name counter in destroy_process_group, so the
    WORLD group of a second init carries the name of the first one.  The cache
    must not hand back the first group's transport (its peer mappings belong
    to a destroyed group): get() returns a new transport bound to the new
    group object."""
    from datetime import timedelta
    from spark_gpt_b200.ep import PeerTransport
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    try:
        os.environ["MASTER_PORT"] = str(_free_port())
        dist.init_process_group("gloo", rank=0, world_size=1, timeout=timedelta(seconds=20))
        first = PeerTransport.get(None, 1024, 8, "cpu")
        first_pg = dist.group.WORLD
        dist.destroy_process_group()
        os.environ["MASTER_PORT"] = str(_free_port())
        dist.init_process_group("gloo", rank=0, world_size=1, timeout=timedelta(seconds=20))
        assert dist.group.WORLD is not first_pg
        second = PeerTransport.get(None, 1024, 8, "cpu")
        assert second is not first
        assert second.pg is dist.group.WORLD
        assert PeerTransport.get(None, 1024, 8, "cpu") is second
    finally:
        PeerTransport._cache.clear()
        if dist.is_initialized():
            dist.destroy_process_group()


class FaultingOps(OracleOps):
    """OracleOps whose fault hooks stand in for the device fault word: the
    snapshot at the end of rank 1's first forward "lands" bit 1 (a bounded
    wait that gave up), as b200moe_fault_snapshot would after a peer barrier
    timed out."""

    landed = 0
    rank = 0

    @classmethod
    def snapshot(cls, device):
        if cls.rank == 1:
            cls.landed = 1

    @classmethod
    def raise_pending(cls, device):
        from spark_gpt_b200.faults import DeviceFault
        if cls.landed:
            word, cls.landed = cls.landed, 0
            raise DeviceFault(word, device)


def _fault_worker(rank, world, port, results):
    import time
    from datetime import timedelta
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=timedelta(seconds=5))
    from spark_gpt_b200.ep import ExpertParallelMoE
    FaultingOps.rank = rank
    cfg = SimpleNamespace(hidden_size=H, num_experts=E, num_experts_per_tok=K,
                          moe_intermediate_size=I, norm_topk_prob=True)
    m = ExpertParallelMoE(cfg, backend=FaultingOps)
    w_r, w_gu, w_d = full_weights()
    with torch.no_grad():
        m.gate.weight.copy_(w_r)
        m.experts.gate_up_proj.copy_(w_gu[m.expert_offset:m.expert_offset + m.local_experts])
        m.experts.down_proj.copy_(w_d[m.expert_offset:m.expert_offset + m.local_experts])
    x = rank_inputs(rank)[0]
    m(x)  # the first step completes on both ranks; rank 1's snapshot records the fault
    t0 = time.monotonic()
    try:
        m(x)
        results[rank] = {"error": None, "type": None, "seconds": time.monotonic() - t0}
    except Exception as e:  # noqa: BLE001 - the failure is the point
        results[rank] = {"error": str(e), "type": type(e).__name__,
                         "seconds": time.monotonic() - t0}


def test_a_recorded_device_fault_raises_on_the_next_call():
    """A fault word recorded during one step raises DeviceFault (a
    RuntimeError naming the fault) at the start of that rank's next layer
    call, before it issues any collective; its peer then gets an error from
    the process group's short timeout instead of waiting for good."""
    mgr = mp.get_context("spawn").Manager()
    results = mgr.dict()
    mp.start_processes(_fault_worker, args=(2, _free_port(), results), nprocs=2, join=True,
                       start_method="spawn")
    assert results[1]["type"] == "DeviceFault"
    assert "bounded device wait gave up" in results[1]["error"]
    assert results[0]["error"] is not None, "rank 0 finished an exchange its peer never joined"
    assert results[0]["seconds"] < 60
