"""Expert-parallel orchestration on CPU ranks (gloo, world size 2).

spark_gpt_b200.ep.ExpertParallelMoE is driven with an oracle-backed ops
object in place of the device kernels, so the routing, the send order, the
all_to_all_single exchanges and the backward's reverse exchanges are checked
on CPU: every rank's output and input gradient must equal the single-process
oracle layer on that rank's tokens, and each rank's expert-shard gradients
must equal the oracle's gradients of those experts summed over both ranks'
tokens.  Test infrastructure only: the product path runs the CUDA kernels.
"""

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
    """CPU stand-in for spark_gpt_b200.ep.CudaExpertOps (fp32 oracle math)."""

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
    def row_map(order, inv, top_k):
        return SimpleNamespace(order=order, inv=inv, k=top_k)

    @staticmethod
    def experts_fwd(rows, ids, w_gu, w_d):
        n = rows.shape[0]
        d = O.dispatch(ids.view(n, 1).long(), w_gu.shape[0])
        xs = rows.float()[torch.from_numpy(d.permutation)]
        gu, h = O.swiglu_forward(xs, w_gu, d.offsets)
        y = O.grouped_linear_forward(h, w_d, d.offsets)
        return y[torch.from_numpy(d.inverse)], (d, xs, gu, h, w_gu, w_d)

    @staticmethod
    def experts_bwd(ctx, dy_rows, E, H, I, device):
        d, xs, gu, h, w_gu, w_d = ctx
        dy = dy_rows.float()[torch.from_numpy(d.permutation)]
        dh, dwd = O.grouped_linear_backward(h, w_d, dy, d.offsets)
        dxs, dwgu, _ = O.swiglu_backward(xs, w_gu, gu, dh, d.offsets)
        return dxs[torch.from_numpy(d.inverse)], dwgu, dwd

    @staticmethod
    def combine(y_sorted, rm, rw):
        rows = y_sorted.float()[rm.inv] * rw.reshape(-1, 1).float()
        return rows.view(-1, rm.k, rows.shape[-1]).sum(1)

    @staticmethod
    def combine_bwd(d_out, y_sorted, rm, rw):
        g = d_out.float()[torch.div(rm.order, rm.k, rounding_mode="floor")]
        dy = g * rw.reshape(-1)[rm.order].unsqueeze(-1).float()
        dw = torch.empty(rm.order.numel())
        dw[rm.order] = (g * y_sorted.float()).sum(-1)
        return dy, dw.view(-1, rm.k)

    @staticmethod
    def gather_bwd(dx_sorted, rm, addend):
        rows = dx_sorted.float()[rm.inv]
        return rows.view(-1, rm.k, rows.shape[-1]).sum(1) + addend

    @staticmethod
    def cast(w):
        return w.float()


T, H, E, K, I = 48, 32, 8, 3, 16


def full_weights():
    g = torch.Generator().manual_seed(7)
    return (torch.randn(E, H, generator=g) * 0.5, torch.randn(E, 2 * I, H, generator=g) * 0.2,
            torch.randn(E, H, I, generator=g) * 0.2)


def rank_inputs(rank):
    g = torch.Generator().manual_seed(100 + rank)
    return torch.randn(T, H, generator=g), torch.randn(T, H, generator=g)


def _worker(rank, world, port, results):
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        from spark_gpt_b200.ep import ExpertParallelMoE
        cfg = SimpleNamespace(hidden_size=H, num_experts=E, num_experts_per_tok=K,
                              moe_intermediate_size=I, norm_topk_prob=True)
        m = ExpertParallelMoE(cfg, backend=OracleOps)
        w_r, w_gu, w_d = full_weights()
        lo, hi = m.expert_offset, m.expert_offset + m.local_experts
        with torch.no_grad():
            m.gate.weight.copy_(w_r)
            m.experts.gate_up_proj.copy_(w_gu[lo:hi])
            m.experts.down_proj.copy_(w_d[lo:hi])
        x, d_out = rank_inputs(rank)
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


def test_expert_parallel_matches_single_process_oracle():
    world = 2
    mgr = mp.get_context("spawn").Manager()
    results = mgr.dict()
    mp.start_processes(_worker, args=(world, _free_port(), results), nprocs=world,
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
