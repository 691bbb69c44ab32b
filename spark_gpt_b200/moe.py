"""Drop-in B200 replacement for spark-gpt's Qwen3-MoE layer.

Same module tree, parameter names, shapes and call signatures as the
reference (train.py:2134-2334):

    SparseMoE(config)                      -> .gate (TopKRouter), .experts (Experts)
    SparseMoE.forward(h)                   -> (out, router_logits, selected_experts)
    TopKRouter.forward(h)                  -> (router_logits, routing_weights, selected)
    Experts.forward(h, selected, weights)  -> out

Parameters stay fp32 masters in the stock HF Qwen3-MoE layout
(``gate.weight`` (E,H), ``experts.gate_up_proj`` (E,2I,H),
``experts.down_proj`` (E,H,I)), so build_optimizer, apply_mup_init, export_hf
and checkpoints are untouched.  Every step of the forward and backward runs in
libb200moe.so; there is no CPU or torch fallback.
"""

from __future__ import annotations

import torch
import torch.nn as nn

from . import faults, fp8, ops
from .custom_ops import TOKEN_MAJOR, _dispatch_from, moe_backward, norm_sparse_moe, sparse_moe

BF16 = torch.bfloat16



def _require_cuda(*ts):
    for t in ts:
        if not t.is_cuda:
            raise RuntimeError("spark_gpt_b200: the MoE layer runs only on CUDA (sm_100a); "
                               "there is no CPU path")


def _as_bf16(x: torch.Tensor) -> torch.Tensor:
    x = x if x.dtype == BF16 else x.to(BF16)
    x = x.contiguous()
    if x.data_ptr() % 16:
        x = x.clone()
    return x


def _grad_like(g: torch.Tensor, p: torch.Tensor) -> torch.Tensor:
    return g if g.dtype == p.dtype else g.to(p.dtype)


def _extra_logit_grad(d_logits, T, W):
    """The gradient reaching router_logits (T,E), laid out with row stride W."""
    if d_logits is None:
        return None
    if d_logits.dtype == BF16 and d_logits.stride() == (W, 1) and d_logits.data_ptr() % 16 == 0:
        return d_logits
    buf = torch.zeros(T, W, device=d_logits.device, dtype=BF16)
    buf[:, : d_logits.shape[1]] = d_logits
    return buf


class _RouterFn(torch.autograd.Function):
    """TopKRouter.forward on its own (train.py:2144-2158)."""

    @staticmethod
    def forward(ctx, x, w_router, top_k, norm):
        _require_cuda(x, w_router)
        faults.raise_pending(x.device)
        E = w_router.shape[0]
        W = ops.router_width(E)
        xb = _as_bf16(x)
        wr = ops.cast_bf16(w_router, W)
        logits_buf = ops.router_logits(xb, wr)
        sel, rw = ops.router_topk(logits_buf, E, top_k, norm)
        faults.snapshot(x.device)
        ctx.save_for_backward(xb, wr, logits_buf, sel)
        ctx.cfg = (E, W, top_k, norm, x.dtype)
        ctx.mark_non_differentiable(sel)
        logits = logits_buf if W == E else logits_buf[:, :E]
        return logits, rw, sel

    @staticmethod
    def backward(ctx, d_logits, d_rw, _d_sel):
        xb, wr, logits_buf, sel = ctx.saved_tensors
        faults.raise_pending(xb.device)
        E, W, top_k, norm, xdtype = ctx.cfg
        T = xb.shape[0]
        if d_rw is None:
            d_rw = torch.zeros(T, top_k, device=xb.device, dtype=torch.float32)
        d_rw = d_rw.float().contiguous()
        extra = _extra_logit_grad(d_logits, T, W)
        dl = ops.router_topk_bwd(logits_buf, sel, d_rw, extra, E, top_k, norm)
        dx = ops.router_dgrad(dl, wr)
        g_router = ops.router_wgrad(xb, dl, E) if ctx.needs_input_grad[1] else None
        faults.snapshot(xb.device)
        return dx.to(xdtype), g_router, None, None


class _ExpertsFn(torch.autograd.Function):
    """Experts.forward with given routing (train.py:2262-2322)."""

    @staticmethod
    def forward(ctx, x, selected, weights, w_gate_up, w_down):
        _require_cuda(x, selected, weights, w_gate_up, w_down)
        faults.raise_pending(x.device)
        E = w_gate_up.shape[0]
        xb = _as_bf16(x)
        rw = _as_bf16(weights)
        sel = selected.to(torch.int64).contiguous()
        wgu = ops.cast_bf16(w_gate_up)
        wd = ops.cast_bf16(w_down)
        d = ops.dispatch(sel, E)
        xs = ops.gather_rows(xb, d)
        gu, h = ops.gate_up_fwd(xs, wgu, d)
        y = ops.down_fwd(h, wd, d, token_major=TOKEN_MAJOR)
        out = ops.combine(y, d, rw, token_major=TOKEN_MAJOR)
        faults.snapshot(x.device)
        ctx.save_for_backward(rw, wgu, wd, xs, gu, h, y)
        ctx.dispatch = d
        ctx.cfg = (x.dtype, weights.dtype)
        return out.to(x.dtype)

    @staticmethod
    def backward(ctx, d_out):
        rw, wgu, wd, xs, gu, h, y = ctx.saved_tensors
        faults.raise_pending(xs.device)
        d = ctx.dispatch
        xdtype, wdtype = ctx.cfg
        dy, d_rw = ops.combine_bwd(_as_bf16(d_out), y, d, rw, token_major=TOKEN_MAJOR)
        d_gu = ops.down_dgrad_swiglu(dy, wd, gu, d)
        g_down = ops.wgrad(dy, h, d, name="down_wgrad") if ctx.needs_input_grad[4] else None
        dxs = ops.gate_up_dgrad(d_gu, wgu, d, token_major=TOKEN_MAJOR)
        g_gu = ops.wgrad(d_gu, xs, d, name="gate_up_wgrad") if ctx.needs_input_grad[3] else None
        dx = ops.gather_rows_bwd(dxs, d, token_major=TOKEN_MAJOR)
        faults.snapshot(xs.device)
        return dx.to(xdtype), None, d_rw.to(wdtype), g_gu, g_down


class _GradSyncMoEFn(torch.autograd.Function):
    """The fused layer with its weight gradients handed to a GradSync
    (grad_sync.py): written or accumulated into the sync's flat buffer, the
    expert bucket's all-reduce started as soon as it is final.  The
    parameters' .grad is that buffer, so no gradient is returned for them."""

    @staticmethod
    def forward(ctx, x, w_router, w_gate_up, w_down, top_k, norm, sync):
        out, logits_buf, sel, *saved = torch.ops.b200moe.sparse_moe_fwd(
            x, w_router, w_gate_up, w_down, top_k, norm)
        ctx.save_for_backward(x, logits_buf, sel, *saved)
        ctx.set_materialize_grads(False)
        ctx.cfg = (top_k, norm, w_gate_up.shape[0], x.dtype)
        ctx.sync = sync
        ctx.mark_non_differentiable(sel)
        E = w_gate_up.shape[0]
        logits = logits_buf if logits_buf.shape[1] == E else logits_buf[:, :E]
        return out, logits, sel

    @staticmethod
    def backward(ctx, d_out, d_logits, _d_sel):
        x, logits_buf, sel, wr, wgu, wd, rw, xs, gu, h, y, counts, offsets, pad_offsets, \
            row_flat, inv_pad, tile_expert = ctx.saved_tensors
        top_k, norm, E, xdt = ctx.cfg
        xb = _as_bf16(x)
        faults.raise_pending(xb.device)
        if d_out is None:
            d_out = torch.zeros_like(xb)
        d = _dispatch_from(counts, offsets, pad_offsets, row_flat, inv_pad, tile_expert,
                           xb.shape[0], top_k, E)
        grads = ctx.sync.begin()
        dx, _, _, _ = moe_backward(d_out, d_logits, xb, logits_buf, sel, wr, wgu, wd, rw, xs, gu,
                                   h, y, d, top_k, norm, E, grads=grads)
        faults.snapshot(xb.device)
        return dx.to(xdt), None, None, None, None, None, None


class TopKRouter(nn.Module):
    """Qwen3-MoE router: bias-free logits, fp32 softmax, then top-k."""

    def __init__(self, config):
        super().__init__()
        self.num_experts = config.num_experts
        self.top_k = config.num_experts_per_tok
        self.norm_topk_prob = config.norm_topk_prob
        self.weight = nn.Parameter(torch.empty(config.num_experts, config.hidden_size))

    def forward(self, hidden_states: torch.Tensor):
        shape = hidden_states.shape
        x = hidden_states.reshape(-1, shape[-1])
        logits, rw, sel = _RouterFn.apply(x, self.weight, self.top_k, self.norm_topk_prob)
        lead = shape[:-1]
        return (logits.view(*lead, logits.shape[-1]), rw.view(*lead, rw.shape[-1]),
                sel.view(*lead, sel.shape[-1]))


class Experts(nn.Module):
    """Packed Qwen3-MoE experts in the stock HF checkpoint layout."""

    def __init__(self, config):
        super().__init__()
        self.num_experts = config.num_experts
        self.hidden_dim = config.hidden_size
        self.intermediate_dim = config.moe_intermediate_size
        self.gate_up_proj = nn.Parameter(torch.empty(
            self.num_experts, 2 * self.intermediate_dim, self.hidden_dim))
        self.down_proj = nn.Parameter(torch.empty(
            self.num_experts, self.hidden_dim, self.intermediate_dim))
        # the fp8 path's delayed scales and amax slots (x, gu, h, d_gu, dy),
        # train.py:2258-2260; see spark_gpt_b200.fp8
        self.register_buffer("fp8_scale", torch.ones(5), persistent=False)
        self.register_buffer("fp8_amax", torch.zeros(5), persistent=False)

    def forward(self, hidden_states, selected_experts, routing_weights):
        if fp8.use_fp8(self, hidden_states):  # train.py:2292-2300
            return fp8.FP8ExpertsFn.apply(hidden_states, selected_experts, routing_weights,
                                          self.gate_up_proj, self.down_proj, self.fp8_scale,
                                          self.fp8_amax)
        return _ExpertsFn.apply(hidden_states, selected_experts, routing_weights,
                                self.gate_up_proj, self.down_proj)


class SparseMoE(nn.Module):
    """out, router_logits, selected_experts = SparseMoE(config)(hidden)."""

    def __init__(self, config):
        super().__init__()
        self.gate = TopKRouter(config)
        self.experts = Experts(config)
        self._grad_sync = None  # set by grad_sync.GradSync

    def forward(self, hidden_states: torch.Tensor):
        shape = hidden_states.shape
        x = hidden_states.reshape(-1, shape[-1])
        _require_cuda(x)
        if fp8.use_fp8(self.experts, x):
            # router in bf16, experts on the fp8 path (train.py:2292-2300)
            logits, rw, sel = self.gate(x)
            out = self.experts(x, sel, rw)
        elif self._grad_sync is not None and torch.is_grad_enabled():
            out, logits, sel = _GradSyncMoEFn.apply(
                x, self.gate.weight, self.experts.gate_up_proj, self.experts.down_proj,
                self.gate.top_k, self.gate.norm_topk_prob, self._grad_sync)
        else:
            out, logits, sel = sparse_moe(
                x, self.gate.weight, self.experts.gate_up_proj, self.experts.down_proj,
                self.gate.top_k, self.gate.norm_topk_prob)
        lead = shape[:-1]
        return out.view(shape), logits.view(*lead, logits.shape[-1]), sel.view(*lead, sel.shape[-1])

    def forward_normed(self, hidden_states: torch.Tensor, norm: nn.Module):
        """self(norm(hidden_states)) with the block's post-attention RMSNorm
        (train.py:162-170, applied at :2370) folded into the layer: one pass
        writes the normalised rows and r per token, and the norm's backward
        (its input and weight gradients) runs inside the row-gather backward,
        so the normalised rows' gradient is never written.  `norm` is the
        reference's RMSNorm module (its .weight and .eps); its weight gets its
        gradient as with the unfused call.  Block.forward's
        `self.mlp(self.post_attention_layernorm(h))` becomes
        `self.mlp.forward_normed(h, self.post_attention_layernorm)`."""
        shape = hidden_states.shape
        x = hidden_states.reshape(-1, shape[-1])
        _require_cuda(x)
        H = shape[-1]
        if H % 32 or H > 4096 or H * self.gate.top_k > 18432 or self._grad_sync is not None:
            # beyond the fused backward's shared-memory row ring: the plain composition
            return self(norm(hidden_states))
        out, logits, sel = norm_sparse_moe(
            x, norm.weight, norm.eps, self.gate.weight, self.experts.gate_up_proj,
            self.experts.down_proj, self.gate.top_k, self.gate.norm_topk_prob)
        lead = shape[:-1]
        return out.view(shape), logits.view(*lead, logits.shape[-1]), sel.view(*lead, sel.shape[-1])
