"""CPU oracle for spark-gpt's fp8 expert path (``--fp8-mlp`` on MoE layers).

TEST INFRASTRUCTURE ONLY.  Like ``moe_oracle``, this module is a parity
checker: only ``tests/``, ``__graft_entry__.smoke()`` and ``bench.py``'s CPU
arm may import it; the product path never does.

It restates in plain torch arithmetic (fp32 math on fp8-valued tensors) what
the reference's Triton kernels compute:

* fp8 state and delayed scales   train.py:914-946  (FP8_SITE_MAX, FP8_HEADROOM_BINADES,
                                                    fp8_update_scales)
* per-expert e4m3 weight copies  train.py:1536-1540 (_fp8_quantize_experts)
* gather + e4m3 quantization     train.py:1301-1313 (_fp8_moe_gather_quant_kernel)
* gate_up GEMM + SwiGLU epilogue train.py:1317-1354 (_fp8_moe_swiglu_fwd_kernel)
* down GEMM                      train.py:1357-1379 (_fp8_moe_down_fwd_kernel)
* down dgrad (bf16) + SwiGLU bwd train.py:1382-1423 (_fp8_moe_down_dgrad_swiglu_kernel)
* gate_up dgrad                  train.py:1426-1448 (_fp8_moe_dgrad_kernel)
* gate_up wgrad                  train.py:1451-1478 (_fp8_moe_wgrad_kernel)
* down wgrad (dy -> e5m2)        train.py:1504-1530 (_fp8_moe_wgrad_rows_kernel)
* autograd wiring                train.py:1543-1604 (_FP8Experts)

Quantization is ``clamp(v * scale, -max, max)`` then a round-to-nearest-even
cast (torch's ``.to(float8_e4m3fn / float8_e5m2)``), scales are powers of two,
and every dequantization divides by a product of powers of two (exact).  The
GEMMs multiply fp8 values exactly and accumulate in fp32, so a device result
differs from this restatement only by fp32 summation order (and, through it,
by an occasional one-step rounding flip of a quantized value).

Parity pin: ``tests/golden/make_golden.py --only fp8`` runs the reference's own
``_fp8_quantize_experts`` and ``fp8_update_scales`` (pure torch) on seeded and
edge-case inputs and stores the results under ``tests/golden/fp8_golden.pt``;
``tests/test_oracle_golden.py`` checks this file against them bit for bit.
The reference's Triton kernels cannot pin the rest here: this container has
no GPU, and Triton's CPU interpreter converts to e4m3 differently from the
device (in a probe it turned 7.9375 into 4.0 and 25.0 into 26.0, where the
device's round-to-nearest-even cast gives 8.0 and 24.0), so its outputs are
not the reference's.  The kernel arithmetic above is restated from the kernel
source and checked through the reference's own acceptance test
(tests/test_fp8_mlp.py:57-110 of the reference: relative error against fp32
below 0.12 after one prewarm step and a scale update), which the GPU tests
apply to both this oracle and the device path.
"""

from __future__ import annotations

import torch

E4M3 = torch.float8_e4m3fn
E5M2 = torch.float8_e5m2
E4M3_MAX = 448.0
E5M2_MAX = 57344.0
# per-site limits and headroom (train.py:921-922): x, gu, h (e4m3), d_gu, dy (e5m2)
SITE_MAX = (E4M3_MAX, E4M3_MAX, E4M3_MAX, E5M2_MAX, E5M2_MAX)
HEADROOM_BINADES = 1


def q_e4m3(v: torch.Tensor, s) -> torch.Tensor:
    return (v.float() * s).clamp(-E4M3_MAX, E4M3_MAX).to(E4M3)


def q_e5m2(v: torch.Tensor, s) -> torch.Tensor:
    return (v.float() * s).clamp(-E5M2_MAX, E5M2_MAX).to(E5M2)


def quantize_experts(w: torch.Tensor):
    """Per-expert pow2 scale q_e = 2^floor(log2(448 / amax_e)) and the e4m3
    copy of w * q_e (train.py:1536-1540)."""
    amax = w.detach().float().abs().amax(dim=(1, 2)).clamp(min=1e-30)
    q = torch.exp2(torch.floor(torch.log2(E4M3_MAX / amax)))
    return (w.detach().float() * q[:, None, None]).clamp(-E4M3_MAX, E4M3_MAX).to(E4M3), q


def update_scales(scale: torch.Tensor, amax: torch.Tensor) -> None:
    """fp8_update_scales for one module's buffers (train.py:938-946), in place."""
    fmax = scale.new_tensor(SITE_MAX)
    new = torch.exp2(torch.floor(torch.log2(fmax / amax.clamp(min=1e-30))) - HEADROOM_BINADES)
    scale.copy_(torch.where(amax > 0, new, scale))
    amax.zero_()


def _ranges(offsets):
    """(expert, start, end) of each expert's rows from inclusive offsets."""
    out, s = [], 0
    for e, end in enumerate([int(v) for v in offsets]):
        out.append((e, s, end))
        s = end
    return out


def experts_forward(x, w_gu, w_d, token_index, offsets, scale, amax):
    """_FP8Experts.forward: unweighted bf16 expert rows in expert order, plus
    what the backward keeps.  ``amax`` (5,) is raised in place (atomic max of
    the unquantized x, gu, h)."""
    E, twoI, _ = w_gu.shape
    I = twoI // 2
    rows = x.float()[token_index.long()]
    if rows.numel():
        amax[0] = torch.maximum(amax[0], rows.abs().max())
    x8 = q_e4m3(rows, scale[0])
    w8, q_gu = quantize_experts(w_gu)
    wd8, q_d = quantize_experts(w_d)
    R, D = rows.shape
    gu8 = torch.zeros(R, twoI, dtype=E4M3)
    h8 = torch.zeros(R, I, dtype=E4M3)
    out = torch.zeros(R, D, dtype=torch.bfloat16)
    for e, s, t in _ranges(offsets):
        if t == s:
            continue
        acc = x8[s:t].float() @ w8[e].float().t()
        deq = 1.0 / (scale[0] * q_gu[e])
        g = (acc[:, :I] * deq).to(torch.bfloat16).float()
        u = (acc[:, I:] * deq).to(torch.bfloat16).float()
        h = g * torch.sigmoid(g) * u
        gu8[s:t, :I] = q_e4m3(g, scale[1])
        gu8[s:t, I:] = q_e4m3(u, scale[1])
        h8[s:t] = q_e4m3(h, scale[2])
        amax[1] = torch.maximum(amax[1], torch.maximum(g.abs().max(), u.abs().max()))
        amax[2] = torch.maximum(amax[2], h.abs().max())
        y = h8[s:t].float() @ wd8[e].float().t()
        out[s:t] = (y / (scale[2] * q_d[e])).to(torch.bfloat16)
    saved = dict(x8=x8, w8=w8, q_gu=q_gu, wd=w_d.detach().to(torch.bfloat16), gu8=gu8, h8=h8)
    return out, saved


def experts_backward(d_rows, saved, offsets, scale, amax):
    """_FP8Experts.backward for the gradient of the expert rows (R, D) bf16
    (the combine's backward output).  Returns (dx_rows bf16 (R, D) in expert
    order, dW_gu fp32 (E, 2I, D), dW_d fp32 (E, D, I)); ``amax`` slots 3, 4
    are raised in place."""
    x8, w8, q_gu, wd, gu8, h8 = (saved[k] for k in ("x8", "w8", "q_gu", "wd", "gu8", "h8"))
    E, D, I = wd.shape
    R = d_rows.shape[0]
    dy = d_rows.float()
    if R:
        amax[4] = torch.maximum(amax[4], dy.abs().max())
    dgu8 = torch.zeros(R, 2 * I, dtype=E5M2)
    dx = torch.zeros(R, D, dtype=torch.bfloat16)
    dw_gu = torch.zeros(E, 2 * I, D)
    dw_d = torch.zeros(E, D, I)
    dy8 = q_e5m2(dy, scale[4])
    for e, s, t in _ranges(offsets):
        if t == s:
            continue
        dh = (dy[s:t] @ wd[e].float()).to(torch.bfloat16).float()
        g = gu8[s:t, :I].float() * (1.0 / scale[1])
        u = gu8[s:t, I:].float() * (1.0 / scale[1])
        sig = torch.sigmoid(g)
        d_gate = dh * u * (sig * (1.0 + g * (1.0 - sig)))
        d_up = dh * g * sig
        dgu8[s:t, :I] = q_e5m2(d_gate, scale[3])
        dgu8[s:t, I:] = q_e5m2(d_up, scale[3])
        amax[3] = torch.maximum(amax[3], torch.maximum(d_gate.abs().max(), d_up.abs().max()))
        acc = dgu8[s:t].float() @ w8[e].float()
        dx[s:t] = (acc / (scale[3] * q_gu[e])).to(torch.bfloat16)
        dw_gu[e] = (dgu8[s:t].float().t() @ x8[s:t].float()) / (scale[3] * scale[0])
        dw_d[e] = (dy8[s:t].float().t() @ h8[s:t].float()) / (scale[4] * scale[2])
    return dx, dw_gu, dw_d, dict(dgu8=dgu8, dy8=dy8)


def experts_layer(x, selected, weights, w_gu, w_d, d_out, scale, amax):
    """Experts.forward on the fp8 path with given routing (train.py:2262-2300:
    sort, _FP8Experts, then the bf16 _CombineTopK) and its backward for the
    output gradient ``d_out``.  Returns dict(out, dx, dW_gate_up, dW_down,
    d_weights) with the combine in bf16 as the reference runs it (each
    weighted row rounded to bf16, the k-sum in fp32 rounded once)."""
    from oracle import moe_oracle as O
    d = O.dispatch(selected, w_gu.shape[0])
    tok = torch.from_numpy(d.token_index)
    inv = torch.from_numpy(d.inverse)
    k = d.top_k
    rows, saved = experts_forward(x, w_gu, w_d, tok, d.offsets, scale, amax)
    w_sorted = weights.reshape(-1)[torch.from_numpy(d.permutation)].to(torch.bfloat16)
    weighted = (rows * w_sorted.unsqueeze(-1))                      # bf16 product
    out = weighted[inv].float().view(-1, k, rows.shape[-1]).sum(dim=1).to(torch.bfloat16)
    g = d_out.to(torch.bfloat16)[tok]
    dy = g * w_sorted.unsqueeze(-1)                                 # bf16 product
    dw_sorted = (g.float() * rows.float()).sum(dim=-1)
    dx_rows, dw_gu, dw_d, _ = experts_backward(dy, saved, d.offsets, scale, amax)
    dx = dx_rows[inv].float().view(-1, k, rows.shape[-1]).sum(dim=1).to(torch.bfloat16)
    d_weights = torch.empty_like(dw_sorted)
    d_weights[torch.from_numpy(d.permutation)] = dw_sorted
    return dict(out=out, dx=dx, dW_gate_up=dw_gu, dW_down=dw_d,
                d_weights=d_weights.view(selected.shape))
