"""Expert-parallel layer on 2 GPUs over NCCL against the single-GPU layer.

Each rank holds half of the experts; its routing must equal
spark_gpt_b200.SparseMoE's (all experts on one GPU) on the same tokens, and
its output, input gradient and router gradient, and each expert shard's weight
gradients summed over both ranks' tokens, must agree with it within the
layer's bf16 tolerance (the owner rounds its partial sum of a token's local
slots to bf16 before the source adds the two ranks' partial rows).  Runs as
two spawned processes; skipped where fewer than two GPUs are visible.
"""

import os
import socket
from types import SimpleNamespace

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from tests.helpers import assert_bf16_close

pytestmark = pytest.mark.gpu

T, H, E, K, I = 2048, 1024, 16, 4, 256
# NCCL all-to-all: one send plan per step, exchanges in sequence; 3 token
# chunks with the exchanges overlapped and 16 SMs left to NCCL; and the
# peer-memory transport (rows stored straight into the other rank's buffers),
# plain, with 2 token chunks pipelined on a copy stream, and pipelined per
# source rank with point-to-point completion flags
VARIANTS = {"plain": dict(chunks=1, comm_sms=0), "overlap": dict(chunks=3, comm_sms=16),
            "p2p": dict(transport="p2p"),
            "p2p_overlap": dict(transport="p2p", chunks=2, comm_sms=16),
            "p2p_pipe": dict(transport="p2p_pipe", comm_sms=16)}


def _cfg():
    return SimpleNamespace(hidden_size=H, num_experts=E, num_experts_per_tok=K,
                           moe_intermediate_size=I, norm_topk_prob=True)


def _weights():
    g = torch.Generator().manual_seed(3)
    return (torch.randn(E, H, generator=g) * 0.05, torch.randn(E, 2 * I, H, generator=g) * 0.01,
            torch.randn(E, H, I, generator=g) * 0.01)


def _inputs(rank):
    g = torch.Generator().manual_seed(40 + rank)
    return (torch.randn(T, H, generator=g).to(torch.bfloat16),
            (torch.randn(T, H, generator=g) * 1e-2).to(torch.bfloat16))


def _worker(rank, world, port, results):
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    torch.cuda.set_device(rank)
    dev = torch.device("cuda", rank)
    from datetime import timedelta
    dist.init_process_group("nccl", rank=rank, world_size=world, device_id=dev,
                            timeout=timedelta(seconds=60))
    try:
        from spark_gpt_b200 import SparseMoE
        from spark_gpt_b200.ep import ExpertParallelMoE
        w_r, w_gu, w_d = _weights()
        eps = {name: ExpertParallelMoE(_cfg(), **kw).to(dev) for name, kw in VARIANTS.items()}
        ep0 = next(iter(eps.values()))
        lo, hi = ep0.expert_offset, ep0.expert_offset + ep0.local_experts
        ref = SparseMoE(_cfg()).to(dev)
        with torch.no_grad():
            for m in (*eps.values(), ref):
                m.gate.weight.copy_(w_r)
            for ep in eps.values():
                ep.experts.gate_up_proj.copy_(w_gu[lo:hi])
                ep.experts.down_proj.copy_(w_d[lo:hi])
            ref.experts.gate_up_proj.copy_(w_gu)
            ref.experts.down_proj.copy_(w_d)
        x, d_out = _inputs(rank)
        x, d_out = x.to(dev), d_out.to(dev)
        outs = {}
        for name, m in (*eps.items(), ("ref", ref)):
            xin = x.clone().requires_grad_(True)
            out, logits, sel = m(xin)
            out.backward(d_out)
            outs[name] = (out.detach().cpu(), sel.cpu(), xin.grad.cpu(), m.gate.weight.grad.cpu())
        gu_sum = ref.experts.gate_up_proj.grad.clone()
        d_sum = ref.experts.down_proj.grad.clone()
        dist.all_reduce(gu_sum)
        dist.all_reduce(d_sum)
        torch.cuda.synchronize()
        results[rank] = {"outs": outs,
                         "ep_gu": {n: ep.experts.gate_up_proj.grad.cpu() for n, ep in eps.items()},
                         "ep_d": {n: ep.experts.down_proj.grad.cpu() for n, ep in eps.items()},
                         "ref_gu": gu_sum[lo:hi].cpu(), "ref_d": d_sum[lo:hi].cpu()}
    finally:
        dist.destroy_process_group()


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def test_expert_parallel_two_gpus_matches_single_gpu_layer():
    if torch.cuda.device_count() < 2:
        pytest.skip("needs two GPUs")
    mgr = mp.get_context("spawn").Manager()
    results = mgr.dict()
    mp.start_processes(_worker, args=(2, _free_port(), results), nprocs=2, join=True,
                       start_method="spawn")
    for rank in range(2):
        r = results[rank]
        o_ref, s_ref, dx_ref, dr_ref = r["outs"]["ref"]
        for name in VARIANTS:
            o_ep, s_ep, dx_ep, dr_ep = r["outs"][name]
            assert torch.equal(s_ep, s_ref)
            assert_bf16_close(o_ep, o_ref, f"{name} out")
            assert_bf16_close(dx_ep, dx_ref, f"{name} dx")
            assert_bf16_close(dr_ep, dr_ref, f"{name} dW_router")
            assert_bf16_close(r["ep_gu"][name], r["ref_gu"], f"{name} dW_gate_up")
            assert_bf16_close(r["ep_d"][name], r["ref_d"], f"{name} dW_down")
        # the chunked, overlapped schedule and the peer-memory transport compute
        # the same values as the plain NCCL schedule
        assert torch.equal(r["outs"]["plain"][0], r["outs"]["overlap"][0])
        assert torch.equal(r["outs"]["plain"][0], r["outs"]["p2p"][0])
        assert torch.equal(r["outs"]["plain"][2], r["outs"]["p2p"][2])
        assert torch.equal(r["outs"]["plain"][0], r["outs"]["p2p_overlap"][0])
        assert torch.equal(r["outs"]["plain"][2], r["outs"]["p2p_overlap"][2])
        # per-source chunks: every row's result is computed as without them
        assert torch.equal(r["outs"]["p2p"][0], r["outs"]["p2p_pipe"][0])
        assert torch.equal(r["outs"]["p2p"][2], r["outs"]["p2p_pipe"][2])
