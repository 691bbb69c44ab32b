"""Whole-layer parity: spark_gpt_b200.SparseMoE + global_load_balancing_loss
on the GPU against the CPU oracle (fp32, same bf16 operand values, routing
injected from the device so both sides route identically).

Tolerance (layer contract): max_rel <= 2e-2 and mean_rel <= 2e-3, errors
normalised by the reference tensor's scale (tests/helpers.py)."""

from types import SimpleNamespace

import pytest
import torch

from oracle import moe_oracle as O
from tests.helpers import assert_bf16_close

pytestmark = pytest.mark.gpu

DEV = "cuda"


def cfg(H, E, k, I, norm=True):
    return SimpleNamespace(hidden_size=H, num_experts=E, num_experts_per_tok=k,
                           moe_intermediate_size=I, norm_topk_prob=norm)


def build(H, E, k, I, seed, norm=True, router_std=0.02, zipf=None):
    from spark_gpt_b200 import SparseMoE
    torch.manual_seed(seed)
    m = SparseMoE(cfg(H, E, k, I, norm)).to(DEV)
    std_in, std_w = O.mup_std(H)
    with torch.no_grad():
        m.gate.weight.normal_(0.0, router_std)
        m.experts.gate_up_proj.normal_(0.0, std_in)
        m.experts.down_proj.normal_(0.0, std_w)
    return m


def run_layer(m, x, d_out, valid, coef=1e-3):
    from spark_gpt_b200 import global_load_balancing_loss
    xin = x.clone().requires_grad_(True)
    out, logits, sel = m(xin)
    E, k = m.gate.num_experts, m.gate.top_k
    aux, stats = global_load_balancing_loss((logits,), (sel,), valid, num_experts=E, top_k=k)
    torch.autograd.backward([out, aux], [d_out, torch.tensor(coef, device=DEV)])
    return out, logits, sel, aux, stats, xin.grad


def oracle_for(m, x, d_out, valid, logits, sel, rw, coef=1e-3):
    E, k = m.gate.num_experts, m.gate.top_k
    bf = lambda t: t.detach().to(torch.bfloat16).float().cpu()
    lg = logits.detach().float().cpu()
    aux, stats, g_aux = O.load_balancing_loss((lg,), (sel.cpu(),), valid.cpu(), num_experts=E,
                                              top_k=k)
    d_extra = (coef * g_aux[0]).to(torch.bfloat16).float()
    res = O.layer_forward_backward(
        bf(x), bf(m.gate.weight), bf(m.experts.gate_up_proj), bf(m.experts.down_proj), k,
        bf(d_out), norm_topk_prob=m.gate.norm_topk_prob, selected=sel.cpu(),
        weights=rw.detach().float().cpu(), d_logits_extra=d_extra, logits=lg)
    return res, aux, stats


LAYERS = [
    # T, H, E, k, I, norm, filler
    (4096, 256, 8, 2, 128, True, 0),       # config-1 shape
    (2048, 512, 16, 4, 192, False, 300),
    (8192, 1024, 64, 8, 256, True, 0),     # config-2 shape, fewer tokens
    (1024, 2048, 128, 8, 768, True, 64),   # config-3 shape, fewer tokens
]


@pytest.mark.parametrize("T,H,E,k,I,norm,filler", LAYERS)
def test_layer_matches_oracle(T, H, E, k, I, norm, filler):
    from spark_gpt_b200 import _lib
    m = build(H, E, k, I, seed=T + H)
    m.gate.norm_topk_prob = norm
    x = torch.randn(T, H, device=DEV).to(torch.bfloat16)
    d_out = (torch.randn(T, H, device=DEV) * 1e-2).to(torch.bfloat16)
    valid = torch.ones(T, dtype=torch.bool, device=DEV)
    if filler:
        valid[-filler:] = False
    out, logits, sel, aux, stats, dx = run_layer(m, x, d_out, valid)
    assert _lib.read_fault() == 0
    # router logits against fp32 logits of the same bf16 operands
    ref_logits = x.float() @ m.gate.weight.detach().to(torch.bfloat16).float().t()
    assert_bf16_close(logits, ref_logits, "logits")
    # routing: bit-exact top-k of the device logits
    ref_sel, ref_rw = O.router_select(logits.detach().float().cpu(), k, norm)[2], None
    assert torch.equal(sel.cpu(), ref_sel)
    from spark_gpt_b200 import ops
    rw = ops.router_topk(logits.detach().contiguous(), E, k, norm)[1]
    res, r_aux, r_stats = oracle_for(m, x, d_out, valid, logits, sel, rw)
    assert abs(float(aux) - float(r_aux)) <= 1e-5 * abs(float(r_aux))
    assert abs(float(stats["router_entropy"]) - float(r_stats["router_entropy"])) <= 1e-4
    errs = {
        "out": assert_bf16_close(out, res["out"], "out"),
        "dx": assert_bf16_close(dx, res["dx"], "dx"),
        "dW_gate_up": assert_bf16_close(m.experts.gate_up_proj.grad, res["dW_gate_up"], "dW_gate_up"),
        "dW_down": assert_bf16_close(m.experts.down_proj.grad, res["dW_down"], "dW_down"),
        "dW_router": assert_bf16_close(m.gate.weight.grad, res["dW_router"], "dW_router"),
    }
    print(f"\nlayer T={T} H={H} E={E} k={k} I={I}: " +
          ", ".join(f"{k_}: max {v['max_rel']:.2e} mean {v['mean_rel']:.2e}" for k_, v in errs.items()))
    assert m.experts.gate_up_proj.grad.dtype == torch.float32


@pytest.mark.parametrize("shape", [(0, 256), (2, 0, 256), (7, 256), (3, 5, 256)])
def test_empty_and_ragged_batches(shape):
    """An empty batch (a rank or micro-batch without tokens), a 3-D hidden
    state and batches smaller than one 128-row tile: outputs keep the input's
    leading shape, gradients are finite, the expert and router gradients of
    an empty batch are zero, and nothing sets the fault word."""
    from spark_gpt_b200 import SparseMoE, _lib
    torch.manual_seed(0)
    m = SparseMoE(cfg(256, 8, 2, 128)).to(DEV)
    with torch.no_grad():
        m.gate.weight.normal_(0, 0.05)
        m.experts.gate_up_proj.normal_(0, 0.02)
        m.experts.down_proj.normal_(0, 0.02)
    x = torch.randn(*shape, device=DEV).to(torch.bfloat16).requires_grad_(True)
    out, logits, sel = m(x)
    assert out.shape == x.shape
    assert logits.shape == (*shape[:-1], 8) and sel.shape == (*shape[:-1], 2)
    out.float().square().sum().backward()
    torch.cuda.synchronize()
    assert _lib.read_fault() == 0
    assert x.grad.shape == x.shape and torch.isfinite(x.grad.float()).all()
    for p in m.parameters():
        assert p.grad is not None and torch.isfinite(p.grad).all()
        if x.numel() == 0:
            assert torch.all(p.grad == 0)


def test_unused_experts_have_zero_finite_gradients():
    """Analogue of the reference's tests/test_moe.py:452-472."""
    from spark_gpt_b200 import Experts
    c = cfg(128, 4, 2, 64)
    ex = Experts(c).to(DEV)
    with torch.no_grad():
        ex.gate_up_proj.normal_(0.0, 0.02)
        ex.down_proj.normal_(0.0, 0.02)
    hidden = torch.randn(256, 128, device=DEV, dtype=torch.bfloat16, requires_grad=True)
    selected = torch.tensor([[0, 1]], device=DEV).expand(256, -1)
    weights = torch.full((256, 2), 0.5, device=DEV, dtype=torch.bfloat16)
    out = ex(hidden, selected, weights)
    out.float().square().mean().backward()
    for g in (ex.gate_up_proj.grad, ex.down_proj.grad):
        assert torch.isfinite(g).all()
        assert torch.all(g[2:] == 0)


def test_experts_module_matches_oracle_with_given_routing():
    from spark_gpt_b200 import Experts
    T, H, E, k, I = 1500, 256, 6, 3, 128
    c = cfg(H, E, k, I)
    torch.manual_seed(11)
    ex = Experts(c).to(DEV)
    with torch.no_grad():
        ex.gate_up_proj.normal_(0.0, 0.05)
        ex.down_proj.normal_(0.0, 0.05)
    x = torch.randn(T, H, device=DEV).to(torch.bfloat16).requires_grad_(True)
    sel = torch.stack([torch.randperm(E)[:k] for _ in range(T)]).to(DEV)
    w = torch.rand(T, k, device=DEV).to(torch.bfloat16).requires_grad_(True)
    out = ex(x, sel, w)
    probe = torch.randn(T, H, device=DEV).to(torch.bfloat16)
    out.backward(probe)
    bf = lambda t: t.detach().to(torch.bfloat16).float().cpu()
    d = O.dispatch(sel.cpu(), E)
    sw = w.detach().float().cpu().reshape(-1)[torch.from_numpy(d.permutation)]
    xs = O.gather_forward(bf(x), d)
    gu, h = O.swiglu_forward(xs, bf(ex.gate_up_proj), d.offsets)
    y = O.grouped_linear_forward(h, bf(ex.down_proj), d.offsets)
    ref_out = O.combine_forward(y, sw, d)
    dy, dw_sorted = O.combine_backward(y, sw, d, probe.float().cpu())
    dh, dwd = O.grouped_linear_backward(h, bf(ex.down_proj), dy, d.offsets)
    dxs, dwgu, _ = O.swiglu_backward(xs, bf(ex.gate_up_proj), gu, dh, d.offsets)
    assert_bf16_close(out, ref_out, "out")
    assert_bf16_close(x.grad, O.gather_backward(dxs, d), "dx")
    assert_bf16_close(ex.gate_up_proj.grad, dwgu, "dW_gate_up")
    assert_bf16_close(ex.down_proj.grad, dwd, "dW_down")
    dwf = torch.empty(T * k)
    dwf[torch.from_numpy(d.permutation)] = dw_sorted
    assert_bf16_close(w.grad, dwf.view(T, k), "d_routing_weights")


def test_router_module_and_determinism():
    from spark_gpt_b200 import TopKRouter
    T, H, E, k = 3000, 512, 32, 4
    r = TopKRouter(cfg(H, E, k, 64)).to(DEV)
    with torch.no_grad():
        r.weight.normal_(0.0, 0.05)
    x = torch.randn(T, H, device=DEV).to(torch.bfloat16)
    outs = []
    for _ in range(2):
        xin = x.clone().requires_grad_(True)
        r.weight.grad = None
        lg, w, sel = r(xin)
        (lg.float().square().sum() + (w.float() * torch.arange(k, device=DEV)).sum()).backward()
        outs.append((lg, w, sel, xin.grad, r.weight.grad))
    for a, b in zip(*outs):
        assert torch.equal(a, b)
    lg, w, sel, gx, gw = outs[0]
    ref = x.float() @ r.weight.detach().to(torch.bfloat16).float().t()
    assert_bf16_close(lg, ref, "router logits")
    assert torch.equal(sel.cpu(), O.router_select(lg.float().cpu(), k, True)[2])
    # gradient through softmax/top-k/renorm and the logits, against the oracle
    p = O.softmax_fp32(lg.detach().float().cpu())
    d_logits_direct = 2 * lg.detach().float().cpu()
    d_w = torch.arange(k).float().expand(T, k)
    dl, dx, dwr = O.router_backward(x.float().cpu(), r.weight.detach().to(torch.bfloat16).float().cpu(),
                                    p, w.float().cpu(), sel.cpu(), d_w, True,
                                    d_logits_extra=d_logits_direct.to(torch.bfloat16).float())
    assert_bf16_close(gx, dx, "router dx")
    assert_bf16_close(gw, dwr, "router dW")


def test_layer_is_deterministic():
    m = build(1024, 64, 8, 256, seed=3)
    x = torch.randn(4096, 1024, device=DEV).to(torch.bfloat16)
    d_out = (torch.randn(4096, 1024, device=DEV) * 1e-2).to(torch.bfloat16)
    valid = torch.ones(4096, dtype=torch.bool, device=DEV)
    r1 = run_layer(m, x, d_out, valid)
    g1 = [p.grad.clone() for p in m.parameters()]
    for p in m.parameters():
        p.grad = None
    r2 = run_layer(m, x, d_out, valid)
    g2 = [p.grad.clone() for p in m.parameters()]
    for a, b in zip(r1, r2):
        if isinstance(a, torch.Tensor):
            assert torch.equal(a, b)
    for a, b in zip(g1, g2):
        assert torch.equal(a, b)
