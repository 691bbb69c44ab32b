"""The fp8 expert path (spark-gpt's --fp8-mlp on MoE layers) on the device.

Checked against the fp8 oracle (oracle/fp8_oracle.py, a restatement of the
reference's _FP8Experts, train.py:1543-1604) and against fp32:

* the per-expert e4m3 weight copies and their scales bit-exact;
* the gather + e4m3 quantization of x bit-exact, its amax exact;
* the e5m2 quantization of a bf16 matrix bit-exact, its amax exact;
* each fp8 GEMM against the oracle's arithmetic on the same fp8 operands:
  fp32 accumulation order is the only difference, so the bf16 outputs agree
  within the bf16 contract and the fp8 outputs differ in at most a few
  elements by one quantization step;
* the whole layer, two steps with a scale update between (the reference's
  own acceptance test, tests/test_fp8_mlp.py:57-110 of the reference): out,
  dx, dW_gate_up, dW_down within 0.12 relative (Frobenius) error of fp32,
  finite, zero gradients for an expert without rows; and within 0.03 of the
  fp8 oracle run with the device's routing and scales;
* the scale update from the device's amax slots equals the oracle's.
"""

import pytest
import torch
import torch.nn.functional as F

from oracle import fp8_oracle as F8
from tests.helpers import assert_bf16_close

pytestmark = pytest.mark.gpu

DEV = "cuda"
BF16 = torch.bfloat16


def _bytes(t):
    return t.view(torch.uint8)


def _dispatch(sel, E):
    from spark_gpt_b200 import ops
    return ops.dispatch(sel.to(DEV).contiguous(), E)


def _unpadded(d, t):
    """Rows of a padded-row tensor in the reference's expert order (valid rows
    only; rows past the padded total are spare capacity and hold nothing)."""
    total = int(d.pad_offsets[-1])
    rf = d.row_flat.cpu()[:total]
    keep = rf >= 0
    return t.cpu()[:total][keep], rf[keep]


def test_quantize_experts_bit_exact():
    from spark_gpt_b200 import ops
    g = torch.Generator().manual_seed(3)
    w = torch.randn(6, 256, 128, generator=g) * torch.tensor([0.02, 0.5, 3.0, 1e-4, 0.0, 7.0])[:, None, None]
    w8, q = ops.fp8_quantize_experts(w.to(DEV))
    r8, rq = F8.quantize_experts(w)
    assert torch.equal(q.cpu(), rq)
    assert torch.equal(_bytes(w8).cpu(), _bytes(r8))


@pytest.mark.parametrize("T,H,E,k", [(777, 256, 8, 2), (2048, 1024, 64, 8)])
def test_gather_quant_and_row_quant_bit_exact(T, H, E, k):
    from spark_gpt_b200 import ops
    torch.manual_seed(T)
    x = (torch.randn(T, H) * 3).to(BF16)
    sel = torch.stack([torch.randperm(E)[:k] for _ in range(T)])
    d = _dispatch(sel, E)
    scale = torch.tensor([16.0, 1, 1, 1, 0.25], device=DEV)
    amax = torch.zeros(5, device=DEV)
    x8 = ops.fp8_gather_quant(x.to(DEV), d, scale, amax)
    rows, rf = _unpadded(d, x8)
    ref = F8.q_e4m3(x.float()[rf.long() // k], 16.0)
    assert torch.equal(_bytes(rows), _bytes(ref))
    pad = d.row_flat.cpu() < 0
    pad[int(d.pad_offsets[-1]):] = False
    assert torch.count_nonzero(_bytes(x8.cpu()[pad])) == 0
    assert float(amax[0]) == float(x.float().abs().max())
    # e5m2 rows with amax in slot 4
    src = (torch.randn(1024, H) * 100).to(BF16)
    q8 = ops.fp8_quantize_rows(src.to(DEV), scale[4:5], amax[4:5], ops.E5M2)
    assert torch.equal(_bytes(q8).cpu(), _bytes(F8.q_e5m2(src.float(), 0.25)))
    assert float(amax[4]) == float(src.float().abs().max())


@pytest.mark.parametrize("T,H,E,k", [(777, 256, 8, 2), (2048, 1024, 64, 8), (512, 4096, 16, 4)])
def test_fused_combine_bwd_e5m2_bit_exact(T, H, E, k):
    """The combine backward with the e5m2 copy of its rows fused in equals the
    plain combine backward followed by the separate quantization, bit for bit
    (H = 4096 takes the unfused fallback inside the entry point)."""
    from spark_gpt_b200 import ops
    torch.manual_seed(T + H)
    sel = torch.stack([torch.randperm(E)[:k] for _ in range(T)])
    d = _dispatch(sel, E)
    y = (torch.randn(d.rows_cap, H, device=DEV) * 0.5).to(BF16)
    d_out = (torch.randn(T, H, device=DEV) * 30).to(BF16)
    w = torch.softmax(torch.randn(T, k, device=DEV), -1).to(BF16)
    scale = torch.tensor([1.0, 1, 1, 1, 512.0], device=DEV)
    am1, am2 = torch.zeros(5, device=DEV), torch.zeros(5, device=DEV)
    dy, dw, dy8 = ops.fp8_combine_bwd(d_out, y, d, w, scale[4:5], am1[4:5])
    dy_r, dw_r = ops.combine_bwd(d_out, y, d, w)
    dy8_r = ops.fp8_quantize_rows(dy_r, scale[4:5], am2[4:5], ops.E5M2, d)
    total = int(d.pad_offsets[-1])
    assert torch.equal(dy[:total], dy_r[:total])
    assert torch.equal(dw, dw_r)
    assert torch.equal(_bytes(dy8[:total]), _bytes(dy8_r[:total]))
    assert float(am1[4]) == float(am2[4]) > 0


def _layer_case(T, H, E, k, I, seed, unused=None):
    torch.manual_seed(seed)
    w_gu = torch.randn(E, 2 * I, H) * 0.05
    w_d = torch.randn(E, H, I) * 0.05
    x = torch.randn(T, H).to(BF16)
    if unused is None:
        sel = torch.stack([torch.randperm(E)[:k] for _ in range(T)])
    else:
        choices = torch.tensor([[0, 1], [1, 3], [0, 3]])
        sel = choices[torch.randint(0, 3, (T,))]
    weights = torch.softmax(torch.randn(T, k), -1).to(BF16)
    probe = torch.randn(T, H)
    return w_gu, w_d, x, sel, weights, probe


def _experts(H, E, I, w_gu, w_d):
    from types import SimpleNamespace
    from spark_gpt_b200 import Experts
    cfg = SimpleNamespace(hidden_size=H, num_experts=E, num_experts_per_tok=2,
                          moe_intermediate_size=I, norm_topk_prob=True)
    ex = Experts(cfg).to(DEV).train()
    with torch.no_grad():
        ex.gate_up_proj.copy_(w_gu)
        ex.down_proj.copy_(w_d)
    return ex


def _device_step(ex, x, sel, weights, probe):
    xx = x.to(DEV).clone().requires_grad_(True)
    out = ex(xx, sel.to(DEV), weights.to(DEV))
    grads = torch.autograd.grad((out.float() * probe.to(DEV)).sum(),
                                [xx, ex.gate_up_proj, ex.down_proj])
    torch.cuda.synchronize()
    return (out.detach(),) + tuple(g.detach() for g in grads)


def _fp32_layer(x, selected, weights, w_gu, w_d, probe):
    """The fp32 layer the reference's acceptance test compares with, written
    per expert (sum over slots of w * SwiGLU expert output) on the GPU."""
    x32 = x.float().to(DEV).requires_grad_(True)
    wgu = w_gu.float().to(DEV).requires_grad_(True)
    wd = w_d.float().to(DEV).requires_grad_(True)
    sel = selected.to(DEV)
    w = weights.float().to(DEV)
    y32 = torch.zeros(x.shape[0], x.shape[1], device=DEV)
    with _no_tf32():
        for e in range(w_gu.shape[0]):
            t, s = (sel == e).nonzero(as_tuple=True)
            if t.numel() == 0:
                continue
            g, u = (x32[t] @ wgu[e].t()).chunk(2, dim=-1)
            y32 = y32.index_add(0, t, w[t, s, None] * ((F.silu(g) * u) @ wd[e].t()))
        grads = torch.autograd.grad((y32 * probe.to(DEV)).sum(), [x32, wgu, wd])
    return (y32.detach(),) + grads


class _no_tf32:
    def __enter__(self):
        self.prev = torch.backends.cuda.matmul.allow_tf32
        torch.backends.cuda.matmul.allow_tf32 = False

    def __exit__(self, *exc):
        torch.backends.cuda.matmul.allow_tf32 = self.prev


def _rel(a, b):
    a = a.detach().float().cpu()
    b = b.detach().float().cpu()
    return float((a - b).norm() / b.norm().clamp_min(1e-30))


@pytest.mark.parametrize("T,H,E,k,I,unused", [
    (500, 256, 4, 2, 128, 2),         # the reference's acceptance shapes, expert 2 unused
    (4096, 1024, 64, 8, 256, None),   # cfg2 shapes
    (1024, 2048, 128, 8, 768, None),  # cfg3 shapes (I % 256 == 0 -> 3 N tiles of 256)
    (1024, 1024, 32, 4, 384, None),   # I % 256 == 128: half-empty last weight-gradient tile
])
def test_fp8_layer_two_steps(T, H, E, k, I, unused):
    from spark_gpt_b200 import _lib, fp8, fp8_update_scales
    w_gu, w_d, x, sel, weights, probe = _layer_case(T, H, E, k, I, seed=T + H, unused=unused)
    ex = _experts(H, E, I, w_gu, w_d)
    saved = fp8.FP8_MLP
    fp8.FP8_MLP = True
    try:
        _device_step(ex, x, sel, weights, probe)          # prewarm
        assert bool((ex.fp8_amax > 0).all()), ex.fp8_amax
        amax_dev = ex.fp8_amax.cpu().clone()
        scale_o, amax_o = torch.ones(5), amax_dev.clone()
        F8.update_scales(scale_o, amax_o)
        fp8_update_scales(ex)
        assert torch.equal(ex.fp8_scale.cpu(), scale_o)
        assert bool((ex.fp8_amax == 0).all())
        scale = ex.fp8_scale.cpu().clone()
        res = _device_step(ex, x, sel, weights, probe)
    finally:
        fp8.FP8_MLP = saved
    assert _lib.read_fault() == 0
    ref32 = _fp32_layer(x, sel, weights, w_gu, w_d, probe)
    amax_ref = torch.zeros(5)
    ref8 = F8.experts_layer(x, sel, weights, w_gu, w_d, probe, scale, amax_ref)
    names = ("out", "dx", "dW_gate_up", "dW_down")
    for n, a, r32, r8 in zip(names, res, ref32,
                             (ref8["out"], ref8["dx"], ref8["dW_gate_up"], ref8["dW_down"])):
        assert torch.isfinite(a.float()).all(), n
        e32, e8 = _rel(a, r32), _rel(a, r8)
        print(f"\nfp8 T={T} H={H} E={E} k={k} I={I} {n}: vs fp32 {e32:.3e}, vs fp8 oracle {e8:.3e}")
        assert e32 < 0.12, f"{n}: rel err vs fp32 {e32:.3e}"
        assert e8 < 0.03, f"{n}: rel err vs the fp8 oracle {e8:.3e}"
    # the device's amax of this step against the oracle's (same scales)
    am = ex.fp8_amax.cpu()
    torch.testing.assert_close(am, amax_ref, rtol=2e-2, atol=0)
    if unused is not None:
        assert torch.count_nonzero(res[2][unused]) == 0
        assert torch.count_nonzero(res[3][unused]) == 0


def test_fp8_gemms_match_oracle_arithmetic():
    """Each GEMM on the same fp8 operands as the oracle: the bf16 outputs
    within the bf16 contract, the fp8 outputs equal up to rare one-step
    rounding flips, the fp32 weight gradients to fp32 summation order."""
    from spark_gpt_b200 import ops
    T, H, E, k, I = 2048, 1024, 16, 4, 256
    w_gu, w_d, x, sel, weights, probe = _layer_case(T, H, E, k, I, seed=5)
    d = _dispatch(sel, E)
    scale = torch.tensor([32.0, 64.0, 32.0, 2.0 ** 14, 2.0 ** 12], device=DEV)
    amax = torch.zeros(5, device=DEV)
    x8 = ops.fp8_gather_quant(x.to(DEV), d, scale, amax)
    w8, q_gu = ops.fp8_quantize_experts(w_gu.to(DEV))
    wd8, q_d = ops.fp8_quantize_experts(w_d.to(DEV))
    gu8, h8 = ops.fp8_gate_up_fwd(x8, w8, q_gu, d, scale, amax)
    y = ops.fp8_down_fwd(h8, wd8, q_d, d, scale)
    rows_x8, rf = _unpadded(d, x8)
    offsets = torch.cumsum(torch.bincount(sel.reshape(-1), minlength=E), 0)
    sc = scale.cpu()
    # oracle forward on the device's x8 (bit-exact with the oracle's own, checked above)
    tok = rf.long() // k
    am_o = torch.zeros(5)
    out_o, saved = F8.experts_forward(x, w_gu, w_d, tok, offsets, sc, am_o)
    assert torch.equal(_bytes(saved["x8"]), _bytes(rows_x8))
    g8, _ = _unpadded(d, gu8)
    hh8, _ = _unpadded(d, h8)
    flips_gu = (_bytes(g8) != _bytes(saved["gu8"])).float().mean()
    flips_h = (_bytes(hh8) != _bytes(saved["h8"])).float().mean()
    assert float(flips_gu) < 2e-3 and float(flips_h) < 2e-3, (flips_gu, flips_h)
    yy, _ = _unpadded(d, y)
    assert_bf16_close(yy, out_o.float(), "fp8 down fwd y", max_rel=6e-2, mean_rel=4e-3)
    # backward GEMMs on the device's own fp8 intermediates
    dy = (torch.randn(d.rows_cap, H) * 0.01).to(BF16).to(DEV)
    dy[d.row_flat < 0] = 0
    dy[int(d.pad_offsets[-1]):] = float("nan")  # spare rows: never read
    wd = w_d.to(BF16).to(DEV)
    dgu8 = ops.fp8_down_dgrad_swiglu(dy, wd, gu8, d, scale, amax)
    dxs = ops.fp8_gate_up_dgrad(dgu8, w8, q_gu, d, scale)
    dy8 = ops.fp8_quantize_rows(dy, scale[4:5], amax[4:5], ops.E5M2, d)
    g_gu = ops.fp8_wgrad(dgu8, x8, d, scale[3:4], scale[0:1])
    g_d = ops.fp8_wgrad(dy8, h8, d, scale[4:5], scale[2:3])
    torch.cuda.synchronize()
    dyu, _ = _unpadded(d, dy)
    saved_dev = dict(x8=rows_x8, w8=w8.cpu(), q_gu=q_gu.cpu(), wd=w_d.to(BF16), gu8=g8, h8=hh8)
    am_b = torch.zeros(5)
    dx_o, dwgu_o, dwd_o, inter = F8.experts_backward(dyu, saved_dev, offsets, sc, am_b)
    dg8, _ = _unpadded(d, dgu8)
    flips_d = (_bytes(dg8) != _bytes(inter["dgu8"])).float().mean()
    assert float(flips_d) < 2e-3, flips_d
    dxu, _ = _unpadded(d, dxs)
    assert_bf16_close(dxu, dx_o.float(), "fp8 gate_up dgrad", max_rel=6e-2, mean_rel=4e-3)
    assert _rel(g_gu, dwgu_o) < 1e-2
    assert _rel(g_d, dwd_o) < 1e-3


def test_sparse_moe_takes_the_fp8_path_when_enabled():
    """SparseMoE.forward (router in bf16, experts on the fp8 path) with
    spark_gpt_b200.fp8.FP8_MLP set and the module training: the experts'
    amax slots are raised, the output and gradients stay within the fp8 bar of
    the same layer's bf16 path, and in eval mode (or with the flag off) the
    bf16 path runs and leaves the amax untouched."""
    from types import SimpleNamespace
    from spark_gpt_b200 import SparseMoE, fp8, fp8_update_scales
    torch.manual_seed(11)
    T, H, E, k, I = 2048, 1024, 32, 4, 256
    cfg = SimpleNamespace(hidden_size=H, num_experts=E, num_experts_per_tok=k,
                          moe_intermediate_size=I, norm_topk_prob=True)
    m = SparseMoE(cfg).to(DEV).train()
    with torch.no_grad():
        m.gate.weight.normal_(0.0, 0.02)
        m.experts.gate_up_proj.normal_(0.0, 0.05)
        m.experts.down_proj.normal_(0.0, 0.05)
    x = torch.randn(T, H, device=DEV).to(BF16)
    probe = torch.randn(T, H, device=DEV)

    def run():
        for p in m.parameters():
            p.grad = None
        xx = x.clone().requires_grad_(True)
        out, logits, sel = m(xx)
        (out.float() * probe).sum().backward()
        torch.cuda.synchronize()
        return out.detach(), sel, xx.grad, m.experts.gate_up_proj.grad.clone()

    ref = run()                                   # bf16 path (flag off)
    assert torch.count_nonzero(m.experts.fp8_amax) == 0
    saved = fp8.FP8_MLP
    fp8.FP8_MLP = True
    try:
        run()                                     # prewarm on the fp8 path
        assert bool((m.experts.fp8_amax > 0).all()), m.experts.fp8_amax
        fp8_update_scales(m)
        res = run()
        m.eval()
        amax0 = m.experts.fp8_amax.clone()
        with torch.no_grad():
            m(x)                                  # eval: the bf16 path
        assert torch.equal(m.experts.fp8_amax, amax0)
    finally:
        fp8.FP8_MLP = saved
        m.train()
    assert torch.equal(res[1], ref[1])            # the router stays bf16: same routing
    for n, a, b in (("out", res[0], ref[0]), ("dx", res[2], ref[2]), ("dW_gate_up", res[3], ref[3])):
        e = _rel(a, b)
        print(f"\nSparseMoE fp8 vs bf16 {n}: {e:.3e}")
        assert e < 0.12, f"{n}: {e:.3e}"
