"""Global load-balancing loss (spark-gpt train.py:3098-3197) on device kernels.

Same signature, value and gradient as the reference's
``global_load_balancing_loss``: per sparse layer the masked softmax sums, the
masked top-k counts, the entropy and the valid-row count are reduced on the
GPU (deterministic two-pass), summed over layers, all-reduced once over the
process group (one packed 2E+2 fp32 vector, train.py:3162), and turned into
``aux = E * <counts/rows, soft/rows>``.  The gradient is that of the local
proxy ``world * E / rows * <counts/rows, soft_local>`` (straight-through
value correction), written straight into each layer's bf16 logit gradient.
"""

from __future__ import annotations

import torch
import torch.distributed as dist

from . import ops

BF16 = torch.bfloat16


class _LoadBalanceFn(torch.autograd.Function):
    @staticmethod
    def forward(ctx, valid_u8, num_experts, top_k, n_layers, *tensors):
        logits_layers = tensors[:n_layers]
        selected_layers = tensors[n_layers:]
        dev = valid_u8.device
        packed = torch.zeros(2 * num_experts + 2, device=dev, dtype=torch.float32)
        for lg, sel in zip(logits_layers, selected_layers):
            ops.lb_stats(lg, sel, valid_u8, num_experts, top_k, packed)
        distributed = dist.is_available() and dist.is_initialized()
        world = dist.get_world_size() if distributed else 1
        if distributed:
            dist.all_reduce(packed, op=dist.ReduceOp.SUM)
        aux, stats, coef = ops.lb_finalize(packed, num_experts, top_k, world)
        ctx.save_for_backward(valid_u8, coef, *logits_layers)
        ctx.num_experts = num_experts
        ctx.mark_non_differentiable(stats, packed)
        return aux, stats, packed

    @staticmethod
    def backward(ctx, g_aux, _g_stats, _g_packed):
        valid_u8, coef, *logits_layers = ctx.saved_tensors
        E = ctx.num_experts
        g = g_aux.float().reshape(1).contiguous()
        grads = []
        for lg in logits_layers:
            d = ops.lb_grad(lg, valid_u8, coef, g, E)
            grads.append(d if d.shape[1] == E else d[:, :E])
        return (None, None, None, None, *grads, *([None] * len(logits_layers)))


def _check_logits(lg: torch.Tensor) -> torch.Tensor:
    if not lg.is_cuda or lg.dtype != BF16:
        raise RuntimeError("global_load_balancing_loss: expects the bf16 CUDA router logits of "
                           "the B200 layer (no CPU path)")
    if lg.stride(-1) != 1:
        lg = lg.contiguous()
    return lg


def global_load_balancing_loss(router_logits, selected_experts, valid_mask, *, num_experts,
                               top_k):
    """Qwen3 auxiliary router loss over all sparse layers and ranks.

    Returns (aux_loss, stats) like train.py:3098; aux_loss carries the
    gradient of the rank-local proxy and the value of the global loss."""
    if not router_logits:
        zero = valid_mask.sum(dtype=torch.float32) * 0.0
        return zero, {k: zero.detach() for k in (
            "aux_loss", "assignment_min_frac", "assignment_max_frac", "assignment_cv",
            "router_entropy", "unused_experts")}
    if len(router_logits) != len(selected_experts):
        raise ValueError("router logits and selected-expert layers do not match")
    T = valid_mask.numel()
    lgs, sels = [], []
    for lg, sel in zip(router_logits, selected_experts):
        if lg.shape[:-1] != valid_mask.shape or lg.shape[-1] != num_experts:
            raise ValueError("router-logit shape does not match the token mask/config")
        if sel.shape != (*valid_mask.shape, top_k):
            raise ValueError("selected-expert shape does not match the token mask/config")
        lgs.append(_check_logits(lg.reshape(T, num_experts)))
        sels.append(sel.reshape(T, top_k).to(torch.int64).contiguous())
    valid_u8 = valid_mask.reshape(T).to(torch.uint8).contiguous()
    aux, stats, _packed = _LoadBalanceFn.apply(valid_u8, num_experts, top_k, len(lgs),
                                               *lgs, *sels)
    s = stats.detach()
    return aux, {
        "aux_loss": aux.detach(),
        "assignment_min_frac": s[0],
        "assignment_max_frac": s[1],
        "assignment_cv": s[2],
        "router_entropy": s[3],
        "unused_experts": s[4],
    }
