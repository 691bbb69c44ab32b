"""Expert-parallel MoE layer: experts sharded over a process group.

with P ranks, rank r owns experts [r*E/P, (r+1)*E/P) and
keeps its own T tokens.  Per forward:

  1. router on the local tokens (replicated router weight), top-k;
  2. the T*k routed slots are ordered stably by destination rank
     (owner = expert // (E/P)), and the token rows, the owners' local expert
     ids and the per-destination counts cross the NVLink/NVSwitch fabric with
     NCCL all_to_all_single (one host read of the counts sizes the buffers);
  3. each owner runs its local experts on the rows it received as a k=1
     problem (dispatch, gate_up GEMM + SwiGLU, down GEMM) and sends the
     results back the same way;
  4. the source combines its k results per token with the routing weights.

The backward mirrors it: combine backward on the source, the slot gradients
cross to the owners, the owners' expert backward yields the row gradients
(sent back) and the local expert weight gradients, and the source sums the
row gradients per token together with the router's input gradient.  The
load-balancing counts are all-reduced by global_load_balancing_loss as in the
data-parallel layout (train.py:3162).

The reference trains data-parallel only (experts replicated, DDP); this module
is the build's expert-parallel layout of the same layer.  Expert parameters
here are this rank's shard: gate_up_proj (E/P, 2I, H), down_proj (E/P, H, I).
"""

from __future__ import annotations

import torch
import torch.distributed as dist
import torch.nn as nn

from . import ops
from .moe import BF16, TopKRouter, _as_bf16, _extra_logit_grad, _require_cuda


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
    def row_map(order: torch.Tensor, inv: torch.Tensor, top_k: int):
        """A dispatch view whose 'padded rows' are the send-ordered slots."""
        R = order.numel()
        dev = order.device
        i32 = dict(device=dev, dtype=torch.int32)
        return ops.Dispatch(
            counts=torch.tensor([R], **i32), offsets=torch.tensor([R], **i32),
            pad_offsets=torch.tensor([0, R], **i32), row_flat=order.to(torch.int32),
            inv_pad=inv.to(torch.int32), tile_expert=torch.zeros(1, **i32), rows_cap=R,
            num_tokens=R // top_k, top_k=top_k, num_experts=1)

    @staticmethod
    def experts_fwd(rows, ids, w_gu, w_d):
        """y[i] = expert ids[i] applied to rows[i] (a k=1 layer with unit weights)."""
        E = w_gu.shape[0]
        n = rows.shape[0]
        if n == 0:
            return rows.new_zeros(0, rows.shape[1]), None
        d = ops.dispatch(ids.view(n, 1).to(torch.int64).contiguous(), E)
        ones = torch.ones(n, 1, device=rows.device, dtype=BF16)
        xs = ops.gather_rows(rows, d)
        gu, h = ops.gate_up_fwd(xs, w_gu, d)
        y = ops.down_fwd(h, w_d, d)
        out = ops.combine(y, d, ones)
        return out, (d, ones, xs, gu, h, y, w_gu, w_d)

    @staticmethod
    def experts_bwd(ctx, dy_rows, E, H, I, device):
        if ctx is None:
            z = torch.zeros(E, 2 * I, H, device=device), torch.zeros(E, H, I, device=device)
            return dy_rows.new_zeros(0, H), z[0], z[1]
        d, ones, xs, gu, h, y, w_gu, w_d = ctx
        dy, _ = ops.combine_bwd(_as_bf16(dy_rows), y, d, ones)
        d_gu = ops.down_dgrad_swiglu(dy, w_d, gu, d)
        g_down = ops.wgrad(dy, h, d, name="down_wgrad")
        dxs = ops.gate_up_dgrad(d_gu, w_gu, d)
        g_gu = ops.wgrad(d_gu, xs, d, name="gate_up_wgrad")
        return ops.gather_rows_bwd(dxs, d), g_gu, g_down

    @staticmethod
    def combine(y_sorted, rm, rw):
        return ops.combine(y_sorted, rm, rw)

    @staticmethod
    def combine_bwd(d_out, y_sorted, rm, rw):
        return ops.combine_bwd(d_out, y_sorted, rm, rw)

    @staticmethod
    def gather_bwd(dx_sorted, rm, addend):
        return ops.gather_rows_bwd(dx_sorted, rm, addend=addend)

    @staticmethod
    def cast(w):
        return ops.cast_bf16(w)


def _exchange(buf, send_counts, recv_counts, group):
    """all_to_all_single of row blocks; counts are host lists of row counts."""
    out = buf.new_empty((sum(recv_counts), *buf.shape[1:]))
    dist.all_to_all_single(out, buf.contiguous(), recv_counts, send_counts, group=group)
    return out


class _EPMoEFn(torch.autograd.Function):
    @staticmethod
    def forward(ctx, x, w_router, w_gu, w_d, top_k, norm, num_experts, group, backend):
        P = dist.get_world_size(group)
        E_loc = w_gu.shape[0]
        T, H = x.shape
        xb = _as_bf16(x) if x.is_cuda else x
        logits_buf, wr, sel, rw = backend.router(xb, w_router, num_experts, top_k, norm)
        flat = sel.reshape(-1)
        dest = torch.div(flat, E_loc, rounding_mode="floor")
        order = torch.sort(dest, stable=True).indices          # send order (stable)
        inv = torch.empty_like(order)
        inv[order] = torch.arange(order.numel(), device=order.device)
        send_counts_t = torch.bincount(dest, minlength=P)
        recv_counts_t = torch.empty_like(send_counts_t)
        dist.all_to_all_single(recv_counts_t, send_counts_t, group=group)
        send_counts = send_counts_t.tolist()
        recv_counts = recv_counts_t.tolist()
        x_send = xb[torch.div(order, top_k, rounding_mode="floor")]
        ids_send = (flat % E_loc)[order].to(torch.int32)
        x_recv = _exchange(x_send, send_counts, recv_counts, group)
        ids_recv = _exchange(ids_send, send_counts, recv_counts, group)
        wgu_b, wd_b = backend.cast(w_gu), backend.cast(w_d)
        y_recv, ectx = backend.experts_fwd(x_recv, ids_recv, wgu_b, wd_b)
        y_sorted = _exchange(y_recv, recv_counts, send_counts, group)
        rm = backend.row_map(order, inv, top_k)
        out = backend.combine(y_sorted, rm, rw)
        ctx.save_for_backward(xb, logits_buf, wr, sel, rw, y_sorted)
        ctx.meta = (rm, ectx, send_counts, recv_counts, group, backend, top_k, norm,
                    num_experts, E_loc, H, w_gu.shape[1] // 2, x.dtype)
        ctx.mark_non_differentiable(sel)
        E = num_experts
        logits = logits_buf if logits_buf.shape[1] == E else logits_buf[:, :E]
        return out.to(x.dtype), logits, sel

    @staticmethod
    def backward(ctx, d_out, d_logits, _d_sel):
        xb, logits_buf, wr, sel, rw, y_sorted = ctx.saved_tensors
        (rm, ectx, send_counts, recv_counts, group, backend, top_k, norm, num_experts, E_loc,
         H, I, xdtype) = ctx.meta
        if d_out is None:
            d_out = torch.zeros(xb.shape, device=xb.device, dtype=xb.dtype)
        d_out = _as_bf16(d_out) if d_out.is_cuda else d_out
        dy_sorted, d_rw = backend.combine_bwd(d_out, y_sorted, rm, rw)
        dy_recv = _exchange(dy_sorted, send_counts, recv_counts, group)
        dx_recv, g_gu, g_d = backend.experts_bwd(ectx, dy_recv, E_loc, H, I, xb.device)
        dx_sorted = _exchange(dx_recv, recv_counts, send_counts, group)
        dx_router, g_router = backend.router_bwd(xb, wr, logits_buf, sel, d_rw, d_logits,
                                                 num_experts, top_k, norm)
        dx = backend.gather_bwd(dx_sorted, rm, dx_router)
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
