"""SparseMoE under torch.compile.

spark-gpt compiles its whole model (train.py:3787, mode="default",
dynamic=False).  The B200 layer is a pair of torch.library custom ops
(b200moe::sparse_moe_fwd / sparse_moe_bwd) with fake implementations, so a
model holding it traces into one graph (fullgraph=True: a graph break is an
error) and the compiled run launches the same kernels as eager mode: the
layer's outputs and gradients are identical bit for bit.
"""

import pytest
import torch
import torch.nn as nn

from tests.test_gpu_layer import DEV, build

pytestmark = pytest.mark.gpu


class Block(nn.Module):
    """Pre-norm residual MoE block (train.py's transformer block shape)."""

    def __init__(self, moe, H):
        super().__init__()
        self.norm = nn.RMSNorm(H, eps=1e-6).to(DEV)
        self.moe = moe

    def forward(self, x):
        out, logits, sel = self.moe(self.norm(x))
        return x + out, logits, sel


def _step(model, params, x, d_out, g_logits):
    xin = x.clone().requires_grad_(True)
    out, logits, sel = model(xin)
    loss = (out.float() * d_out).sum() + (logits.float() * g_logits).sum()
    loss.backward()
    grads = {n: p.grad.clone() for n, p in params.named_parameters()}
    for p in params.parameters():
        p.grad = None
    return out.detach(), logits.detach(), sel, xin.grad, grads


@pytest.mark.parametrize("H,E,k,I", [(256, 8, 2, 128), (512, 64, 8, 128)])
def test_compiled_layer_matches_eager(H, E, k, I):
    from spark_gpt_b200 import ops
    torch._dynamo.reset()
    m = build(H, E, k, I, seed=11)
    g = torch.Generator(device=DEV).manual_seed(5)
    x = torch.randn(2, 384, H, device=DEV, generator=g).to(torch.bfloat16)
    d_out = torch.randn(2, 384, H, device=DEV, generator=g) * 1e-2
    g_logits = torch.randn(2, 384, E, device=DEV, generator=g) * 1e-3
    eager = _step(m, m, x, d_out, g_logits)
    compiled = torch.compile(m, fullgraph=True, dynamic=False)
    _step(compiled, m, x, d_out, g_logits)  # compile
    n0 = ops.LAUNCHES["count"]
    comp = _step(compiled, m, x, d_out, g_logits)
    assert ops.LAUNCHES["count"] > n0, "compiled graph did not run the kernels"
    for a, b in zip(eager[:4], comp[:4]):
        assert a.shape == b.shape and torch.equal(a, b)
    for name, ga in eager[4].items():
        assert torch.equal(ga, comp[4][name]), name


def test_compiled_block_matches_eager():
    torch._dynamo.reset()
    H, E, k, I = 256, 16, 4, 128
    blk = Block(build(H, E, k, I, seed=12), H)
    g = torch.Generator(device=DEV).manual_seed(6)
    x = torch.randn(4, 256, H, device=DEV, generator=g).to(torch.bfloat16)
    d_out = torch.randn(4, 256, H, device=DEV, generator=g) * 1e-2
    g_logits = torch.zeros(4, 256, E, device=DEV)
    eager = _step(blk, blk, x, d_out, g_logits)
    compiled = torch.compile(blk, fullgraph=True, dynamic=False)
    comp = _step(compiled, blk, x, d_out, g_logits)
    # the RMSNorm may be fused differently by the compiler: bf16-rounding slack
    for a, b in zip(eager[:2], comp[:2]):
        torch.testing.assert_close(b.float(), a.float(), rtol=2e-2, atol=2e-2 * a.abs().max())
    assert (eager[2] == comp[2]).float().mean() > 0.99
    for name, ga in eager[4].items():
        gb = comp[4][name]
        torch.testing.assert_close(gb, ga, rtol=5e-2, atol=5e-2 * ga.abs().max().item() + 1e-12)
