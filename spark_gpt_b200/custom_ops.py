"""The fused MoE layer as torch.library custom ops (torch.compile-traceable).

spark-gpt compiles its model (train.py:3787).  The layer's forward and
backward are registered as opaque custom ops with fake (meta) implementations:
every output shape is static (the padded routed-row capacity depends only on
T*k and E), so the compiled graph holds them without graph breaks, and
register_autograd wires the backward op in.

    b200moe::sparse_moe_fwd(x, w_router, w_gate_up, w_down, top_k, norm)
        -> out, logits (T, W), selected, plus the tensors the backward needs
    b200moe::sparse_moe_bwd(d_out, d_logits?, saved..., top_k, norm, ...)
        -> dx, dW_router, dW_gate_up, dW_down
"""

from __future__ import annotations

from contextlib import nullcontext
from typing import Optional

import torch

from . import faults, ops

BF16 = torch.bfloat16

# Layout of the down-projection output y and of the gate_up input gradient
# dxs: token-major (slot t*k+s in row t*k+s, so the combine and the gather
# backward read each token's k rows as one contiguous block) or padded-row
# order (the GEMMs write rows sequentially).  Measured on B200 at config 2:
# the shared-memory row reduction reads scattered 2 KB rows as fast as
# contiguous ones, while scattered epilogue writes slow the two GEMMs, so the
# padded order is the default.
TOKEN_MAJOR = False


def _owned(t: torch.Tensor, src: torch.Tensor) -> torch.Tensor:
    """A custom op's outputs may not alias its inputs (bf16 masters pass through
    cast_bf16 unchanged)."""
    return t.clone() if t.data_ptr() == src.data_ptr() else t


def padded_capacity(routed_rows, num_experts: int):
    """b200moe_padded_rows in Python arithmetic, so that it also holds for the
    symbolic sizes of a traced graph: every expert's row block is rounded up
    to 128 rows."""
    r = routed_rows + num_experts * 127
    return (r + 127) // 128 * 128


def _dispatch_from(counts, offsets, pad_offsets, row_flat, inv_pad, tile_expert, T, k, E):
    return ops.Dispatch(counts, offsets, pad_offsets, row_flat, inv_pad, tile_expert,
                        row_flat.shape[0], T, k, E)


@torch.library.custom_op("b200moe::sparse_moe_fwd", mutates_args=(), device_types="cuda")
def sparse_moe_fwd(x: torch.Tensor, w_router: torch.Tensor, w_gate_up: torch.Tensor,
                   w_down: torch.Tensor, top_k: int, norm: bool) -> tuple[
                       torch.Tensor, torch.Tensor, torch.Tensor, torch.Tensor, torch.Tensor,
                       torch.Tensor, torch.Tensor, torch.Tensor, torch.Tensor, torch.Tensor,
                       torch.Tensor, torch.Tensor, torch.Tensor, torch.Tensor, torch.Tensor,
                       torch.Tensor, torch.Tensor]:
    """Router + experts + combine forward (train.py:2331-2334): router GEMM ->
    fp32 softmax/top-k -> dispatch -> row gather -> gate_up GEMM with SwiGLU in
    its epilogue -> down GEMM -> weighted combine.  (The tile::gather4 GEMM
    variants read x rows inside the GEMM instead of materialising xs; on B200
    their per-row TMA requests ran slower than the streaming gather kernel,
    so this path materialises.)"""
    faults.raise_pending(x.device)
    xb = x if x.dtype == BF16 else x.to(BF16)
    xb = xb.contiguous()
    if xb.data_ptr() % 16:
        xb = xb.clone()
    res = _layer_forward(xb, x.dtype, w_router, w_gate_up, w_down, top_k, norm)
    faults.snapshot(x.device)
    return res


def _layer_forward(xb, out_dtype, w_router, w_gate_up, w_down, top_k, norm):
    """The forward body on bf16, 16-byte aligned rows xb; returns the op's outputs."""
    E = w_gate_up.shape[0]
    W = ops.router_width(E)
    wr = _owned(ops.cast_bf16(w_router, W), w_router)
    wgu = _owned(ops.cast_bf16(w_gate_up), w_gate_up)
    wd = _owned(ops.cast_bf16(w_down), w_down)
    logits_buf = ops.router_logits(xb, wr)
    sel, rw = ops.router_topk(logits_buf, E, top_k, norm)
    d = ops.dispatch(sel, E)
    xs = ops.gather_rows(xb, d)
    gu, h = ops.gate_up_fwd(xs, wgu, d)
    y = ops.down_fwd(h, wd, d, token_major=TOKEN_MAJOR)
    out = ops.combine(y, d, rw, token_major=TOKEN_MAJOR).to(out_dtype)
    return (out, logits_buf, sel, wr, wgu, wd, rw, xs, gu, h, y, d.counts, d.offsets,
            d.pad_offsets, d.row_flat, d.inv_pad, d.tile_expert)


@sparse_moe_fwd.register_fake
def _(x, w_router, w_gate_up, w_down, top_k, norm):
    T, H = x.shape
    E, two_i, _ = w_gate_up.shape
    I = two_i // 2
    W = ops.router_width(E)
    cap = padded_capacity(T * top_k, E)
    e = lambda *s, dt=BF16: x.new_empty(s, dtype=dt)  # noqa: E731
    i32 = torch.int32
    return (e(T, H, dt=x.dtype), e(T, W), e(T, top_k, dt=torch.int64), e(W, H),
            e(E, two_i, H), e(E, H, I), e(T, top_k), e(cap, H), e(cap, two_i), e(cap, I),
            e(cap, H), e(E, dt=i32), e(E, dt=i32), e(E + 1, dt=i32), e(cap, dt=i32),
            e(T * top_k, dt=i32), e(cap // 128, dt=i32))


def moe_backward(d_out, d_logits, xb, logits_buf, sel, wr, wgu, wd, rw, xs, gu, h, y,
                 d: "ops.Dispatch", top_k: int, norm: bool, num_experts: int, grads=None,
                 rmsnorm=None):
    """Router + experts + combine backward: combine backward -> down dgrad with
    the SwiGLU backward in its epilogue -> both weight gradients -> gate_up
    dgrad -> top-k/softmax backward -> router dgrad, folded into the
    row-gather backward -> router wgrad (train.py:2331-2334 under autograd).

    `grads` (optional, grad_sync.GradSync) supplies the fp32 destinations of
    the three weight gradients, whether to accumulate into them, and two
    callbacks: one when the expert gradients are final (it may start their
    all-reduce on another stream and returns a context that limits the SMs of
    the GEMM running beside it) and one when the router gradient is.
    `rmsnorm` (optional: the norm's input, weight and per-token r) folds the
    post-attention RMSNorm's backward into the row-gather backward; the result
    then ends with the norm weight's gradient.  With
    `grads` the gate_up weight gradient runs before the gate_up dgrad, so that
    both expert gradients are final while the dgrad, the router backward and
    the row-gather backward still run; without it the dgrad runs first (its
    input, d_gu, is then partly still in L2)."""
    T = xb.shape[0]
    E = num_experts
    W = wr.shape[0]
    out_r = out_gu = out_d = None
    acc = (False, False, False)
    if grads is not None:
        out_r, out_gu, out_d = grads.router, grads.gate_up, grads.down
        acc = grads.accumulate
    d_out = d_out.to(BF16).contiguous()
    dy, d_rw = ops.combine_bwd(d_out, y, d, rw, token_major=TOKEN_MAJOR)
    d_gu = ops.down_dgrad_swiglu(dy, wd, gu, d)
    g_down = ops.wgrad(dy, h, d, name="down_wgrad", out=out_d, accumulate=acc[2])
    del dy
    if grads is None:
        dxs = ops.gate_up_dgrad(d_gu, wgu, d, token_major=TOKEN_MAJOR)
        g_gate_up = ops.wgrad(d_gu, xs, d, name="gate_up_wgrad")
    else:
        g_gate_up = ops.wgrad(d_gu, xs, d, name="gate_up_wgrad", out=out_gu, accumulate=acc[1])
        beside = grads.experts_ready()
        with beside if beside is not None else nullcontext():
            dxs = ops.gate_up_dgrad(d_gu, wgu, d, token_major=TOKEN_MAJOR)
    del d_gu
    extra = None
    if d_logits is not None:
        if (d_logits.dtype == BF16 and d_logits.stride() == (W, 1)
                and d_logits.data_ptr() % 16 == 0):
            extra = d_logits
        else:
            extra = torch.zeros(T, W, device=xb.device, dtype=BF16)
            extra[:, : d_logits.shape[1]] = d_logits
    dl = ops.router_topk_bwd(logits_buf, sel, d_rw, extra, E, top_k, norm)
    dx_router = ops.router_dgrad(dl, wr)
    if rmsnorm is None:
        dx = ops.gather_rows_bwd(dxs, d, addend=dx_router, token_major=TOKEN_MAJOR)
    else:
        dx, g_norm = ops.gather_rows_bwd_rmsnorm(dxs, d, dx_router, *rmsnorm,
                                                 token_major=TOKEN_MAJOR)
    g_router = ops.router_wgrad(xb, dl, E, out=out_r, accumulate=acc[0])
    if grads is not None:
        grads.router_ready()
    if rmsnorm is not None:
        return dx, g_router, g_gate_up, g_down, g_norm
    return dx, g_router, g_gate_up, g_down


@torch.library.custom_op("b200moe::sparse_moe_bwd", mutates_args=(), device_types="cuda")
def sparse_moe_bwd(d_out: torch.Tensor, d_logits: Optional[torch.Tensor], xb: torch.Tensor,
                   logits_buf: torch.Tensor, sel: torch.Tensor, wr: torch.Tensor,
                   wgu: torch.Tensor, wd: torch.Tensor, rw: torch.Tensor, xs: torch.Tensor,
                   gu: torch.Tensor, h: torch.Tensor, y: torch.Tensor, counts: torch.Tensor,
                   offsets: torch.Tensor, pad_offsets: torch.Tensor, row_flat: torch.Tensor,
                   inv_pad: torch.Tensor, tile_expert: torch.Tensor, top_k: int, norm: bool,
                   num_experts: int) -> tuple[torch.Tensor, torch.Tensor, torch.Tensor,
                                              torch.Tensor]:
    faults.raise_pending(xb.device)
    if xb.data_ptr() % 16:
        xb = xb.clone()
    d = _dispatch_from(counts, offsets, pad_offsets, row_flat, inv_pad, tile_expert,
                       xb.shape[0], top_k, num_experts)
    res = moe_backward(d_out, d_logits, xb, logits_buf, sel, wr, wgu, wd, rw, xs, gu, h, y, d,
                       top_k, norm, num_experts)
    faults.snapshot(xb.device)
    return res


@sparse_moe_bwd.register_fake
def _(d_out, d_logits, xb, logits_buf, sel, wr, wgu, wd, rw, xs, gu, h, y, counts, offsets,
      pad_offsets, row_flat, inv_pad, tile_expert, top_k, norm, num_experts):
    T, H = xb.shape
    E, two_i, _ = wgu.shape
    f32 = torch.float32
    return (xb.new_empty(T, H), xb.new_empty(num_experts, H, dtype=f32),
            xb.new_empty(E, two_i, H, dtype=f32), xb.new_empty(E, H, two_i // 2, dtype=f32))


def _setup_context(ctx, inputs, output):
    x, w_router, w_gate_up, w_down, top_k, norm = inputs
    (_out, logits_buf, sel, *saved) = output
    ctx.save_for_backward(x, logits_buf, sel, *saved)
    # the saved activations are outputs too; their (absent) gradients stay None
    ctx.set_materialize_grads(False)
    ctx.cfg = (top_k, norm, w_gate_up.shape[0], x.dtype, w_router.dtype, w_gate_up.dtype,
               w_down.dtype)


def _backward(ctx, d_out, d_logits, *_unused):
    """Router + experts + combine backward as one op: combine backward ->
    down dgrad with the SwiGLU backward in its epilogue -> both weight
    gradients -> gate_up dgrad -> top-k/softmax backward -> router dgrad,
    folded into the row-gather backward -> router wgrad (train.py:2331-2334
    under autograd)."""
    x, logits_buf, sel, wr, wgu, wd, rw, xs, gu, h, y, counts, offsets, pad_offsets, row_flat, \
        inv_pad, tile_expert = ctx.saved_tensors
    top_k, norm, E, xdt, rdt, gdt, ddt = ctx.cfg
    xb = x if x.dtype == BF16 else x.to(BF16)
    xb = xb.contiguous()
    if d_out is None:
        d_out = torch.zeros_like(xb)
    dx, g_r, g_gu, g_d = torch.ops.b200moe.sparse_moe_bwd(
        d_out, d_logits, xb, logits_buf, sel, wr, wgu, wd, rw, xs, gu, h, y, counts, offsets,
        pad_offsets, row_flat, inv_pad, tile_expert, top_k, norm, E)
    return dx.to(xdt), g_r.to(rdt), g_gu.to(gdt), g_d.to(ddt), None, None


torch.library.register_autograd("b200moe::sparse_moe_fwd", _backward,
                                setup_context=_setup_context)


def sparse_moe(x, w_router, w_gate_up, w_down, top_k, norm):
    """(out, router_logits (T, E), selected_experts) of the fused layer."""
    out, logits_buf, sel, *_ = torch.ops.b200moe.sparse_moe_fwd(x, w_router, w_gate_up, w_down,
                                                                 top_k, norm)
    E = w_gate_up.shape[0]
    logits = logits_buf if logits_buf.shape[1] == E else logits_buf[:, :E]
    return out, logits, sel


# --------------------------------------------------------------------------- #
# the layer with the block's post-attention RMSNorm folded in
# --------------------------------------------------------------------------- #
def _fake_forward(x, w_gate_up, top_k):
    T, H = x.shape
    E, two_i, _ = w_gate_up.shape
    I = two_i // 2
    W = ops.router_width(E)
    cap = padded_capacity(T * top_k, E)
    e = lambda *s, dt=BF16: x.new_empty(s, dtype=dt)  # noqa: E731
    i32 = torch.int32
    return (e(T, H, dt=x.dtype), e(T, W), e(T, top_k, dt=torch.int64), e(W, H),
            e(E, two_i, H), e(E, H, I), e(T, top_k), e(cap, H), e(cap, two_i), e(cap, I),
            e(cap, H), e(E, dt=i32), e(E, dt=i32), e(E + 1, dt=i32), e(cap, dt=i32),
            e(T * top_k, dt=i32), e(cap // 128, dt=i32))


@torch.library.custom_op("b200moe::norm_sparse_moe_fwd", mutates_args=(), device_types="cuda")
def norm_sparse_moe_fwd(h: torch.Tensor, norm_w: torch.Tensor, eps: float,
                        w_router: torch.Tensor, w_gate_up: torch.Tensor, w_down: torch.Tensor,
                        top_k: int, norm: bool) -> tuple[
                            torch.Tensor, torch.Tensor, torch.Tensor, torch.Tensor, torch.Tensor,
                            torch.Tensor, torch.Tensor, torch.Tensor, torch.Tensor, torch.Tensor,
                            torch.Tensor, torch.Tensor, torch.Tensor, torch.Tensor, torch.Tensor,
                            torch.Tensor, torch.Tensor, torch.Tensor, torch.Tensor]:
    """SparseMoE(RMSNorm(h)) forward (train.py:162-170, :2370-2372): one pass
    writes x_n = bf16(bf16(h * r) * bf16(w)) and r per token, then the layer
    runs on x_n.  Outputs: the layer's outputs, then x_n and r."""
    faults.raise_pending(h.device)
    hb = h if h.dtype == BF16 else h.to(BF16)
    hb = hb.contiguous()
    if hb.data_ptr() % 16:
        hb = hb.clone()
    x_n, rstd = ops.rmsnorm(hb, norm_w, eps)
    res = _layer_forward(x_n, h.dtype, w_router, w_gate_up, w_down, top_k, norm)
    faults.snapshot(h.device)
    return (*res, x_n, rstd)


@norm_sparse_moe_fwd.register_fake
def _(h, norm_w, eps, w_router, w_gate_up, w_down, top_k, norm):
    T, H = h.shape
    return (*_fake_forward(h, w_gate_up, top_k), h.new_empty(T, H, dtype=BF16),
            h.new_empty(T, dtype=torch.float32))


@torch.library.custom_op("b200moe::norm_sparse_moe_bwd", mutates_args=(), device_types="cuda")
def norm_sparse_moe_bwd(d_out: torch.Tensor, d_logits: Optional[torch.Tensor],
                        h: torch.Tensor, norm_w: torch.Tensor, rstd: torch.Tensor,
                        x_n: torch.Tensor, logits_buf: torch.Tensor, sel: torch.Tensor,
                        wr: torch.Tensor, wgu: torch.Tensor, wd: torch.Tensor, rw: torch.Tensor,
                        xs: torch.Tensor, gu: torch.Tensor, hh: torch.Tensor, y: torch.Tensor,
                        counts: torch.Tensor, offsets: torch.Tensor, pad_offsets: torch.Tensor,
                        row_flat: torch.Tensor, inv_pad: torch.Tensor, tile_expert: torch.Tensor,
                        top_k: int, norm: bool, num_experts: int) -> tuple[
                            torch.Tensor, torch.Tensor, torch.Tensor, torch.Tensor,
                            torch.Tensor]:
    """The layer's backward with the RMSNorm backward folded into the row-gather
    backward: d h, d norm weight, d router, d gate_up, d down."""
    faults.raise_pending(h.device)
    hb = h if h.dtype == BF16 else h.to(BF16)
    hb = hb.contiguous()
    if hb.data_ptr() % 16:
        hb = hb.clone()
    d = _dispatch_from(counts, offsets, pad_offsets, row_flat, inv_pad, tile_expert,
                       hb.shape[0], top_k, num_experts)
    dh, g_r, g_gu, g_d, g_norm = moe_backward(
        d_out, d_logits, x_n, logits_buf, sel, wr, wgu, wd, rw, xs, gu, hh, y, d, top_k, norm,
        num_experts, rmsnorm=(hb, norm_w.float().contiguous(), rstd))
    faults.snapshot(h.device)
    return dh, g_norm, g_r, g_gu, g_d


@norm_sparse_moe_bwd.register_fake
def _(d_out, d_logits, h, norm_w, rstd, x_n, logits_buf, sel, wr, wgu, wd, rw, xs, gu, hh, y,
      counts, offsets, pad_offsets, row_flat, inv_pad, tile_expert, top_k, norm, num_experts):
    T, H = h.shape
    E, two_i, _ = wgu.shape
    f32 = torch.float32
    return (h.new_empty(T, H, dtype=BF16), h.new_empty(H, dtype=f32),
            h.new_empty(num_experts, H, dtype=f32), h.new_empty(E, two_i, H, dtype=f32),
            h.new_empty(E, H, two_i // 2, dtype=f32))


def _norm_setup_context(ctx, inputs, output):
    h, norm_w, eps, w_router, w_gate_up, w_down, top_k, norm = inputs
    (_out, logits_buf, sel, *saved, x_n, rstd) = output
    ctx.save_for_backward(h, norm_w, rstd, x_n, logits_buf, sel, *saved)
    ctx.set_materialize_grads(False)
    ctx.cfg = (top_k, norm, w_gate_up.shape[0], h.dtype, norm_w.dtype, w_router.dtype,
               w_gate_up.dtype, w_down.dtype)


def _norm_backward(ctx, d_out, d_logits, *_unused):
    h, norm_w, rstd, x_n, logits_buf, sel, wr, wgu, wd, rw, xs, gu, hh, y, counts, offsets, \
        pad_offsets, row_flat, inv_pad, tile_expert = ctx.saved_tensors
    top_k, norm, E, hdt, ndt, rdt, gdt, ddt = ctx.cfg
    if d_out is None:
        d_out = torch.zeros_like(x_n)
    dh, g_n, g_r, g_gu, g_d = torch.ops.b200moe.norm_sparse_moe_bwd(
        d_out, d_logits, h, norm_w, rstd, x_n, logits_buf, sel, wr, wgu, wd, rw, xs, gu, hh, y,
        counts, offsets, pad_offsets, row_flat, inv_pad, tile_expert, top_k, norm, E)
    return (dh.to(hdt), g_n.to(ndt), None, g_r.to(rdt), g_gu.to(gdt), g_d.to(ddt), None, None)


torch.library.register_autograd("b200moe::norm_sparse_moe_fwd", _norm_backward,
                                setup_context=_norm_setup_context)


def norm_sparse_moe(h, norm_w, eps, w_router, w_gate_up, w_down, top_k, norm):
    """(out, router_logits (T, E), selected_experts) of SparseMoE(RMSNorm(h))."""
    out, logits_buf, sel, *_ = torch.ops.b200moe.norm_sparse_moe_fwd(
        h, norm_w, float(eps), w_router, w_gate_up, w_down, top_k, norm)
    E = w_gate_up.shape[0]
    logits = logits_buf if logits_buf.shape[1] == E else logits_buf[:, :E]
    return out, logits, sel
