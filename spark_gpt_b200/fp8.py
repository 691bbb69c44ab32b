"""The fp8 expert path: spark-gpt's ``--fp8-mlp`` on MoE layers.

The reference keeps the expert activations in fp8 while training when
``train.FP8_MLP`` is set (train.py:914, :1258-1264, :1543-1604): x, the gate/up
pre-activations and the SwiGLU output as e4m3, their gradient d_gu and the
expert rows' gradient dy as e5m2, the expert weights as per-expert e4m3 copies
of the fp32 masters; the router and the top-k combine stay bf16.  Scales are
delayed: each step quantizes with powers of two derived from the previous
step's amax (the ``fp8_scale`` / ``fp8_amax`` buffers of the Experts module,
five slots: x, gu, h, d_gu, dy), the kernels raise this step's amax, and
``fp8_update_scales`` rolls them after the optimizer step (train.py:938-946).

Here every piece runs in libb200moe.so: the gather fused with the x
quantization, the weight copies, the four fp8 GEMMs on tcgen05
``kind::f8f6f4`` (two-CTA tiles), the bf16 down-projection dgrad with the
SwiGLU backward and the e5m2 quantization in its epilogue.  The kernels read
the scales from device memory and write the amax slots with atomics, so a step
never waits for the host.

Use: set ``spark_gpt_b200.fp8.FP8_MLP = True`` alongside ``train.FP8_MLP`` and
call ``spark_gpt_b200.fp8_update_scales(model)`` where train.py calls its own
``fp8_update_scales`` (after the prewarm step and after every optimizer step).
The path is taken, as in the reference, only while the module is training,
for bf16 CUDA input, and for shapes the kernels take (H a multiple of 256 and
a power of two, I a multiple of 128, at most 256 experts); otherwise the layer
runs its bf16 path.
"""

from __future__ import annotations

import torch

from . import faults, ops

FP8_MLP = False

# per-site limits and headroom (train.py:921-924): x, gu, h (e4m3), d_gu, dy (e5m2)
FP8_SITE_MAX = (448.0, 448.0, 448.0, 57344.0, 57344.0)
FP8_HEADROOM_BINADES = 1


def use_fp8(experts, x: torch.Tensor) -> bool:
    """The reference's _use_fp8_moe (train.py:1258-1263) for this library's
    kernels."""
    if not (FP8_MLP and experts.training and x.is_cuda and x.dtype == torch.bfloat16):
        return False
    H, I, E = experts.hidden_dim, experts.intermediate_dim, experts.num_experts
    return H % 256 == 0 and H & (H - 1) == 0 and I % 128 == 0 and E <= 256


@torch.no_grad()
def fp8_update_scales(model: torch.nn.Module) -> None:
    """Roll every fp8 expert block's recorded amax into next step's scales
    (train.py:938-946): scale = 2^(floor(log2(max / amax)) - 1) where amax > 0,
    then amax = 0."""
    from .moe import Experts
    for m in model.modules():
        if isinstance(m, Experts):
            fmax = m.fp8_scale.new_tensor(FP8_SITE_MAX)
            new = torch.exp2(torch.floor(torch.log2(fmax / m.fp8_amax.clamp(min=1e-30)))
                             - FP8_HEADROOM_BINADES)
            m.fp8_scale.copy_(torch.where(m.fp8_amax > 0, new, m.fp8_scale))
            m.fp8_amax.zero_()


class FP8ExpertsFn(torch.autograd.Function):
    """Experts.forward on the fp8 path with given routing: dispatch, then the
    reference's _FP8Experts (train.py:1543-1604), then the bf16 top-k combine
    (train.py:2220-2241); out in the input dtype."""

    @staticmethod
    def forward(ctx, x, selected, weights, w_gate_up, w_down, scale, amax):
        from .moe import _as_bf16, _require_cuda
        _require_cuda(x, selected, weights, w_gate_up, w_down, scale, amax)
        faults.raise_pending(x.device)
        E = w_gate_up.shape[0]
        xb = _as_bf16(x)
        rw = _as_bf16(weights)
        sel = selected.to(torch.int64).contiguous()
        d = ops.dispatch(sel, E)
        x8 = ops.fp8_gather_quant(xb, d, scale, amax)
        w8, q_gu = ops.fp8_quantize_experts(w_gate_up)
        wd8, q_d = ops.fp8_quantize_experts(w_down)
        gu8, h8 = ops.fp8_gate_up_fwd(x8, w8, q_gu, d, scale, amax)
        y = ops.fp8_down_fwd(h8, wd8, q_d, d, scale)
        out = ops.combine(y, d, rw)
        wd = ops.cast_bf16(w_down)  # the down dgrad's bf16 operand (train.py:1573)
        faults.snapshot(x.device)
        ctx.save_for_backward(rw, x8, w8, q_gu, wd, gu8, h8, y, scale, amax)
        ctx.dispatch = d
        ctx.cfg = (x.dtype, weights.dtype)
        return out.to(x.dtype)

    @staticmethod
    def backward(ctx, d_out):
        from .moe import _as_bf16
        rw, x8, w8, q_gu, wd, gu8, h8, y, scale, amax = ctx.saved_tensors
        faults.raise_pending(y.device)
        d = ctx.dispatch
        xdtype, wdtype = ctx.cfg
        dy, d_rw, dy8 = ops.fp8_combine_bwd(_as_bf16(d_out), y, d, rw, scale[4:5], amax[4:5])
        d_gu8 = ops.fp8_down_dgrad_swiglu(dy, wd, gu8, d, scale, amax)
        dxs = ops.fp8_gate_up_dgrad(d_gu8, w8, q_gu, d, scale)
        g_gu = (ops.fp8_wgrad(d_gu8, x8, d, scale[3:4], scale[0:1], name="gate_up_wgrad")
                if ctx.needs_input_grad[3] else None)
        g_d = (ops.fp8_wgrad(dy8, h8, d, scale[4:5], scale[2:3], name="down_wgrad")
               if ctx.needs_input_grad[4] else None)
        dx = ops.gather_rows_bwd(dxs, d)
        faults.snapshot(y.device)
        return dx.to(xdtype), None, d_rw.to(wdtype), g_gu, g_d, None, None
