"""The fp8 expert oracle against fp32, with the reference's own acceptance
bar for its fp8 experts (tests/test_fp8_mlp.py:57-110 of the reference):
after one prewarm step and a scale update, out, dx, dW_gate_up and dW_down
within a relative (Frobenius) error of 0.12 of the fp32 layer, all finite,
and zero weight gradients for an expert that received no rows."""

import torch
import torch.nn.functional as F

from oracle import fp8_oracle as F8


def _fp32_layer(x, selected, weights, w_gu, w_d, probe):
    x32 = x.float().requires_grad_(True)
    wgu = w_gu.detach().float().requires_grad_(True)
    wd = w_d.detach().float().requires_grad_(True)
    y32 = torch.zeros(x.shape[0], x.shape[1])
    for s in range(selected.shape[1]):
        e = selected[:, s]
        g, u = torch.einsum("td,tod->to", x32, wgu[e]).chunk(2, dim=-1)
        y32 = y32 + weights[:, s, None].float() * torch.einsum(
            "ti,tdi->td", F.silu(g) * u, wd[e])
    grads = torch.autograd.grad((y32 * probe).sum(), [x32, wgu, wd])
    return (y32.detach(),) + grads


def test_fp8_oracle_tracks_fp32_after_prewarm():
    torch.manual_seed(0)
    T, H, I, E, k = 500, 256, 128, 4, 2
    w_gu = torch.randn(E, 2 * I, H) * 0.05
    w_d = torch.randn(E, H, I) * 0.05
    x = torch.randn(T, H).to(torch.bfloat16)
    choices = torch.tensor([[0, 1], [1, 3], [0, 3]])   # expert 2 gets no tokens
    selected = choices[torch.randint(0, 3, (T,))]
    weights = torch.softmax(torch.randn(T, k), -1).to(torch.bfloat16)
    probe = torch.randn(T, H)
    scale, amax = torch.ones(5), torch.zeros(5)
    F8.experts_layer(x, selected, weights, w_gu, w_d, probe, scale, amax)   # prewarm
    assert bool((amax > 0).all()), amax
    F8.update_scales(scale, amax)
    assert bool((amax == 0).all())
    res = F8.experts_layer(x, selected, weights, w_gu, w_d, probe, scale, amax)
    ref = _fp32_layer(x, selected, weights, w_gu, w_d, probe)
    for name, a, r in zip(("out", "dx", "dW_gate_up", "dW_down"),
                          (res["out"], res["dx"], res["dW_gate_up"], res["dW_down"]), ref):
        err = float((a.float() - r).norm() / r.norm())
        assert torch.isfinite(a.float()).all(), name
        assert err < 0.12, f"{name}: rel err {err:.3e}"
    assert torch.count_nonzero(res["dW_gate_up"][2]) == 0
    assert torch.count_nonzero(res["dW_down"][2]) == 0
