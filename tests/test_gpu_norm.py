"""The post-attention RMSNorm folded into the layer (SparseMoE.forward_normed).

The reference normalises the residual stream before the layer
(train.py:162-170, :2370); forward_normed does it in one pass and runs the
norm's backward inside the row-gather backward.  Checked on the device:

* the norm kernel against the oracle's RMSNorm (pinned to the reference's
  own module): x_n bit-exact except where the fp32 sum of squares, added in a
  different order, moves r by an ulp (then x_n by at most two bf16 units, on
  fewer than 0.1% of the elements);
* the whole fused layer, forward + load-balancing loss + backward, against
  the oracle composition RMSNorm -> layer -> layer backward -> RMSNorm
  backward, with the device's routing injected: out, d h, the norm weight's
  gradient and the three layer weight gradients within the bf16 contract
  (max 2e-2 / mean 2e-3 of the reference tensor's scale);
* the fused call against the unfused one on the device (a torch RMSNorm
  module with the reference's formula, then the layer).
"""

from types import SimpleNamespace

import pytest
import torch
import torch.nn as nn

from oracle import moe_oracle as O
from tests.helpers import assert_bf16_close

pytestmark = pytest.mark.gpu

DEV = "cuda"
BF16 = torch.bfloat16


class RefRMSNorm(nn.Module):
    """The reference's RMSNorm formula (train.py:162-170) as a torch module."""

    def __init__(self, dim, eps=1e-6):
        super().__init__()
        self.weight = nn.Parameter(torch.ones(dim))
        self.eps = eps

    def forward(self, x):
        out = x.float() * torch.rsqrt(x.float().pow(2).mean(dim=-1, keepdim=True) + self.eps)
        return out.to(dtype=x.dtype) * self.weight.to(dtype=x.dtype)


def _layer(H, E, k, I, seed):
    from spark_gpt_b200 import SparseMoE
    torch.manual_seed(seed)
    cfg = SimpleNamespace(hidden_size=H, num_experts=E, num_experts_per_tok=k,
                          moe_intermediate_size=I, norm_topk_prob=True)
    m = SparseMoE(cfg).to(DEV)
    std_in, std_w = O.mup_std(H)
    with torch.no_grad():
        m.gate.weight.normal_(0.0, 0.02)
        m.experts.gate_up_proj.normal_(0.0, std_in)
        m.experts.down_proj.normal_(0.0, std_w)
    norm = RefRMSNorm(H).to(DEV)
    with torch.no_grad():
        norm.weight.copy_(1.0 + 0.1 * torch.randn(H))
    return m, norm


@pytest.mark.parametrize("T,H", [(4096, 1024), (1000, 768), (2048, 2048)])
def test_norm_kernel_matches_oracle(T, H):
    from spark_gpt_b200 import ops
    x = (torch.randn(T, H, device=DEV) * 3.0).to(BF16)
    w = 1.0 + 0.1 * torch.randn(H, device=DEV)
    x_n, r = ops.rmsnorm(x, w, 1e-6)
    ref, ref_r = O.rmsnorm_forward(x, w, 1e-6)
    assert torch.allclose(r, ref_r, rtol=1e-6, atol=0)
    d = (x_n.float() - ref).abs()
    # where r differs by an ulp, x * r and then its product with w may each
    # round to the neighbouring bf16 value: at most two units, on few elements
    assert float((d > 0).float().mean()) < 1e-3
    assert bool((d <= 2 ** -6 * ref.abs().clamp_min(2 ** -100)).all())


LAYERS = [
    # T, H, E, k, I
    (8192, 1024, 64, 8, 256),      # cfg2 shape (1 column vector per lane)
    (4096, 768, 32, 4, 384),       # cfg4 shape (H not a power of two)
    (2048, 2048, 128, 8, 768),     # cfg3 shape (2 column vectors per lane)
]


@pytest.mark.parametrize("T,H,E,k,I", LAYERS)
def test_fused_norm_layer_matches_oracle(T, H, E, k, I):
    from spark_gpt_b200 import _lib, global_load_balancing_loss, ops
    m, norm = _layer(H, E, k, I, seed=T + H)
    h = (torch.randn(T, H, device=DEV) * 2.0).to(BF16)
    d_out = (torch.randn(T, H, device=DEV) * 1e-2).to(BF16)
    valid = torch.ones(T, dtype=torch.bool, device=DEV)
    hin = h.clone().requires_grad_(True)
    out, logits, sel = m.forward_normed(hin, norm)
    aux, _ = global_load_balancing_loss((logits,), (sel,), valid, num_experts=E, top_k=k)
    torch.autograd.backward([out, aux], [d_out, torch.tensor(1e-3, device=DEV)])
    torch.cuda.synchronize()
    assert _lib.read_fault() == 0

    # oracle: RMSNorm -> layer (routing from the device) -> backward -> RMSNorm backward
    x_n, r = O.rmsnorm_forward(h, norm.weight.detach(), norm.eps)
    lg = logits.detach().float()
    assert torch.equal(sel, O.router_select(lg, k, True)[2])
    rw = ops.router_topk(logits.detach().contiguous(), E, k, True)[1]
    bf = lambda t: t.detach().to(BF16).float()  # noqa: E731
    _, _, g_aux = O.load_balancing_loss((lg,), (sel,), valid, num_experts=E, top_k=k)
    res = O.layer_forward_backward(
        x_n, bf(m.gate.weight), bf(m.experts.gate_up_proj), bf(m.experts.down_proj), k,
        bf(d_out), selected=sel, weights=rw.float(), logits=lg,
        d_logits_extra=(1e-3 * g_aux[0]).to(BF16).float())
    dh, dw = O.rmsnorm_backward(h, norm.weight.detach(), r, res["dx"])
    errs = {
        "out": assert_bf16_close(out, res["out"], "out"),
        "dh": assert_bf16_close(hin.grad, dh, "dh"),
        "dW_norm": assert_bf16_close(norm.weight.grad, dw, "dW_norm"),
        "dW_gate_up": assert_bf16_close(m.experts.gate_up_proj.grad, res["dW_gate_up"],
                                        "dW_gate_up"),
        "dW_down": assert_bf16_close(m.experts.down_proj.grad, res["dW_down"], "dW_down"),
        "dW_router": assert_bf16_close(m.gate.weight.grad, res["dW_router"], "dW_router"),
    }
    assert norm.weight.grad.dtype == torch.float32
    print(f"\nnorm-fused T={T} H={H} E={E} k={k} I={I}: " +
          ", ".join(f"{n}: max {v['max_rel']:.2e} mean {v['mean_rel']:.2e}"
                    for n, v in errs.items()))


def test_fused_equals_unfused_on_device():
    """forward_normed and self(norm(h)) route identically and agree within the
    bf16 contract (the fused backward rounds the norm's intermediate product
    once; the unfused torch backward keeps more bf16 roundings).  The inputs
    are multiples of 1/8 in [-2, 2], so every sum of squares is exact in fp32
    whatever its order and both paths normalise with the same r."""
    T, H, E, k, I = 4096, 1024, 64, 8, 256
    m, norm = _layer(H, E, k, I, seed=9)
    h = (torch.randint(-16, 17, (T, H), device=DEV).float() / 8).to(BF16)
    d_out = (torch.randn(T, H, device=DEV) * 1e-2).to(BF16)
    res = []
    for fused in (True, False):
        for p in list(m.parameters()) + list(norm.parameters()):
            p.grad = None
        hin = h.clone().requires_grad_(True)
        out, logits, sel = m.forward_normed(hin, norm) if fused else m(norm(hin))
        out.backward(d_out)
        res.append((out.detach(), sel, hin.grad, norm.weight.grad.clone(),
                    m.experts.gate_up_proj.grad.clone()))
    (o1, s1, g1, n1, w1), (o2, s2, g2, n2, w2) = res
    assert torch.equal(s1, s2)
    assert_bf16_close(o1, o2, "out fused vs unfused")
    assert_bf16_close(g1, g2, "dh fused vs unfused")
    assert_bf16_close(n1, n2, "dW_norm fused vs unfused")
    assert_bf16_close(w1, w2, "dW_gate_up fused vs unfused")
