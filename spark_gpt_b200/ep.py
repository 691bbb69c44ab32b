"""Expert-parallel MoE layer: experts sharded over a process group.

With P ranks, rank r owns experts [r*E/P, (r+1)*E/P) and keeps its own T
tokens.  Per forward:

  1. router on the local tokens (replicated router weight), top-k;
  2. send plan: each token goes ONCE to every rank that owns at least one of
     its k experts (one row per (token, destination rank), not one per slot),
     with k packed slot words (local expert id + bf16 routing weight, or "no
     expert here") beside the row; rank-major, token order within a rank;
  3. the rows and slot words cross the NVLink/NVSwitch fabric with NCCL
     all_to_all_single (one host read of the per-rank row and slot counts
     sizes the receive buffers);
  4. the owner runs its local experts on the received rows as a k-slot layer
     whose foreign slots are skipped (dispatch, gate_up GEMM + SwiGLU, down
     GEMM) and combines each row's local slots with their routing weights
     into one partial output row (fp32 sum, rounded to bf16);
  5. the partial rows travel back and the source sums each token's partial
     rows over the ranks it went to (fp32 sum, rounded once).

The backward mirrors it: d_out rows go to the owners along the same plan; the
owner computes the combine backward (slot gradients and routing-weight
gradients), its experts' backward (expert weight gradients stay local) and
sums each row's slot input-gradients into one row; rows and routing-weight
gradients travel back and the source adds them to the router's input
gradient.  The load-balancing counts are all-reduced by
global_load_balancing_loss as in the data-parallel layout (train.py:3162).

Each (token, rank) row crosses the fabric once per pass instead of once per
slot: with top-8 of 128 experts a token reaches about 5.3 of 8 ranks (2 of
2), so each of the four exchanges moves a third (three quarters) less than a
per-slot exchange.  Results agree with the single-GPU layer within bf16
rounding: the owner's partial sums are rounded to bf16 before the source adds
them (one extra rounding when a token's experts span ranks).

The reference trains data-parallel only (experts replicated, DDP); this module
is the expert-parallel layout of the same layer.  Expert parameters here are
this rank's shard: gate_up_proj (E/P, 2I, H), down_proj (E/P, H, I).
"""

from __future__ import annotations

from types import SimpleNamespace

import torch
import torch.distributed as dist
import torch.nn as nn

from . import ops
from .moe import BF16, TopKRouter, _as_bf16, _extra_logit_grad, _require_cuda

MAX_RANKS = 16  # the source-side sum over ranks reduces at most 16 rows per token


class CudaExpertOps:
    """The device kernels the expert-parallel path runs (libb200moe.so)."""

    @staticmethod
    def router(x, w_router, num_experts, top_k, norm):
        W = ops.router_width(num_experts)
        wr = ops.cast_bf16(w_router, W)
        logits_buf = ops.router_logits(x, wr)
        sel, rw = ops.router_topk(logits_buf, num_experts, top_k, norm)
        return logits_buf, wr, sel, rw

    @staticmethod
    def router_bwd(x, wr, logits_buf, sel, d_rw, d_logits, num_experts, top_k, norm):
        T, W = logits_buf.shape
        extra = _extra_logit_grad(d_logits, T, W)
        dl = ops.router_topk_bwd(logits_buf, sel, d_rw, extra, num_experts, top_k, norm)
        return ops.router_dgrad(dl, wr), ops.router_wgrad(x, dl, num_experts)

    @staticmethod
    def send_plan(sel, rw, experts_per_rank, ranks):
        """Send layout + slot words; sizes (P, 2) int64 = [rows, slots] per rank."""
        dest, slots = ops.ep_route(sel, experts_per_rank, ranks)
        send = ops.dispatch(dest, ranks)
        meta = ops.ep_pack(sel, rw, send, experts_per_rank)
        rows = send.pad_offsets[1:] - send.pad_offsets[:-1]
        sizes = torch.stack([rows.to(torch.int64), slots.to(torch.int64)], 1)
        return SimpleNamespace(send=send, meta=meta, experts_per_rank=experts_per_rank), sizes

    @staticmethod
    def pack_rows(src, plan):
        return ops.gather_rows(_as_bf16(src), plan.send)

    @staticmethod
    def unpack(meta):
        return ops.ep_unpack(meta)

    @staticmethod
    def experts_fwd(rows, sel_loc, w_loc, w_gu, w_d, slots):
        """partial[i] = sum over row i's local slots of bf16(expert(rows[i]) * w)."""
        E = w_gu.shape[0]
        if rows.shape[0] == 0 or slots == 0:
            return rows.new_zeros(rows.shape), None
        d = ops.dispatch(sel_loc, E, routed_slots=slots)
        xs = ops.gather_rows(rows, d)
        gu, h = ops.gate_up_fwd(xs, w_gu, d)
        y = ops.down_fwd(h, w_d, d)
        part = ops.combine(y, d, w_loc)
        return part, (d, w_loc, xs, gu, h, y, w_gu, w_d)

    @staticmethod
    def experts_bwd(ctx, d_rows, k, E, H, I, device):
        """-> (dx rows, d_weights (rows, k) fp32, dW_gate_up, dW_down)."""
        n = d_rows.shape[0]
        if ctx is None:
            z = torch.zeros(E, 2 * I, H, device=device), torch.zeros(E, H, I, device=device)
            return (d_rows.new_zeros(n, H), torch.zeros(n, k, device=device), z[0], z[1])
        d, w_loc, xs, gu, h, y, w_gu, w_d = ctx
        dy, dw = ops.combine_bwd(_as_bf16(d_rows), y, d, w_loc)
        d_gu = ops.down_dgrad_swiglu(dy, w_d, gu, d)
        g_down = ops.wgrad(dy, h, d, name="down_wgrad")
        dxs = ops.gate_up_dgrad(d_gu, w_gu, d)
        g_gu = ops.wgrad(d_gu, xs, d, name="gate_up_wgrad")
        return ops.gather_rows_bwd(dxs, d), dw, g_gu, g_down

    @staticmethod
    def reduce_rows(rows_back, plan, addend=None):
        """out[t] = sum over the ranks token t went to of its returned row (+ addend)."""
        return ops.gather_rows_bwd(rows_back, plan.send, addend=addend)

    @staticmethod
    def weight_grad(dw_back, plan, sel):
        return ops.ep_weight_grad(dw_back, plan.send, sel, plan.experts_per_rank)

    @staticmethod
    def cast(w):
        return ops.cast_bf16(w)


def _exchange(buf, send_counts, recv_counts, group):
    """all_to_all_single of row blocks; counts are host lists of row counts."""
    out = buf.new_empty((sum(recv_counts), *buf.shape[1:]))
    with ops.timed("all_to_all"):
        dist.all_to_all_single(out, buf[: sum(send_counts)].contiguous(), recv_counts,
                               send_counts, group=group)
    return out


class _EPMoEFn(torch.autograd.Function):
    @staticmethod
    def forward(ctx, x, w_router, w_gu, w_d, top_k, norm, num_experts, group, backend):
        P = dist.get_world_size(group)
        E_loc = w_gu.shape[0]
        T, H = x.shape
        xb = _as_bf16(x) if x.is_cuda else x
        logits_buf, wr, sel, rw = backend.router(xb, w_router, num_experts, top_k, norm)
        plan, sizes = backend.send_plan(sel, rw, E_loc, P)
        x_send = backend.pack_rows(xb, plan)
        recv_sizes = torch.empty_like(sizes)
        dist.all_to_all_single(recv_sizes, sizes, group=group)
        host = torch.cat([sizes, recv_sizes]).cpu()  # the one host read of the step
        send_rows = host[:P, 0].tolist()
        recv_rows = host[P:, 0].tolist()
        recv_slots = int(host[P:, 1].sum())
        x_recv = _exchange(x_send, send_rows, recv_rows, group)
        meta_recv = _exchange(plan.meta, send_rows, recv_rows, group)
        sel_loc, w_loc = backend.unpack(meta_recv)
        wgu_b, wd_b = backend.cast(w_gu), backend.cast(w_d)
        part, ectx = backend.experts_fwd(x_recv, sel_loc, w_loc, wgu_b, wd_b, recv_slots)
        back = _exchange(part, recv_rows, send_rows, group)
        out = backend.reduce_rows(back, plan)
        ctx.save_for_backward(xb, logits_buf, wr, sel)
        ctx.meta = (plan, ectx, send_rows, recv_rows, group, backend, top_k, norm, num_experts,
                    E_loc, H, w_gu.shape[1] // 2, x.dtype)
        ctx.mark_non_differentiable(sel)
        E = num_experts
        logits = logits_buf if logits_buf.shape[1] == E else logits_buf[:, :E]
        return out.to(x.dtype), logits, sel

    @staticmethod
    def backward(ctx, d_out, d_logits, _d_sel):
        xb, logits_buf, wr, sel = ctx.saved_tensors
        (plan, ectx, send_rows, recv_rows, group, backend, top_k, norm, num_experts, E_loc, H, I,
         xdtype) = ctx.meta
        if d_out is None:
            d_out = torch.zeros(xb.shape, device=xb.device, dtype=xb.dtype)
        d_send = backend.pack_rows(d_out, plan)
        d_recv = _exchange(d_send, send_rows, recv_rows, group)
        dx_rows, dw_rows, g_gu, g_d = backend.experts_bwd(ectx, d_recv, top_k, E_loc, H, I,
                                                          xb.device)
        dx_back = _exchange(dx_rows, recv_rows, send_rows, group)
        dw_back = _exchange(dw_rows, recv_rows, send_rows, group)
        d_rw = backend.weight_grad(dw_back, plan, sel)
        dx_router, g_router = backend.router_bwd(xb, wr, logits_buf, sel, d_rw, d_logits,
                                                 num_experts, top_k, norm)
        dx = backend.reduce_rows(dx_back, plan, addend=dx_router)
        return (dx.to(xdtype), g_router, g_gu, g_d, None, None, None, None, None)


class ExpertParallelMoE(nn.Module):
    """SparseMoE with experts sharded over `group`.

    Same call and outputs as SparseMoE: (out, router_logits, selected_experts).
    ``gate.weight`` is replicated (all-reduce its gradient like any other
    data-parallel parameter); ``experts.gate_up_proj`` / ``down_proj`` hold
    this rank's E/P experts."""

    def __init__(self, config, group=None, backend=CudaExpertOps):
        super().__init__()
        self.group = group
        P = dist.get_world_size(group)
        r = dist.get_rank(group)
        E = config.num_experts
        if E % P:
            raise ValueError(f"{E} experts do not split over {P} ranks")
        if P > MAX_RANKS:
            raise ValueError(f"expert parallelism supports at most {MAX_RANKS} ranks, got {P}")
        self.num_experts = E
        self.local_experts = E // P
        self.expert_offset = r * self.local_experts
        self.backend = backend
        self.gate = TopKRouter(config)
        self.experts = nn.Module()
        I, H = config.moe_intermediate_size, config.hidden_size
        self.experts.gate_up_proj = nn.Parameter(torch.empty(self.local_experts, 2 * I, H))
        self.experts.down_proj = nn.Parameter(torch.empty(self.local_experts, H, I))

    def forward(self, hidden_states):
        if self.backend is CudaExpertOps:
            _require_cuda(hidden_states)
        shape = hidden_states.shape
        x = hidden_states.reshape(-1, shape[-1])
        out, logits, sel = _EPMoEFn.apply(
            x, self.gate.weight, self.experts.gate_up_proj, self.experts.down_proj,
            self.gate.top_k, self.gate.norm_topk_prob, self.num_experts, self.group,
            self.backend)
        return out.view(shape), logits.view(*shape[:-1], -1), sel.view(*shape[:-1], -1)
