"""GradSync on one GPU: the layer's backward writes its three weight
gradients straight into the sync's flat buffer (bit-identical to the
gradients autograd receives on the plain path), and a second backward
without zero_grad adds into that buffer in the GEMM epilogues, giving twice
the gradient (within fp32 rounding), as autograd's accumulation does.  The input
gradient and the forward outputs are unchanged.  The all-reduce across
ranks is covered on gloo CPU ranks and by the data-parallel bench run."""

from types import SimpleNamespace

import pytest
import torch

pytestmark = pytest.mark.gpu

DEV = "cuda"


def test_grad_sync_gradients_equal_autograd_and_accumulate_in_place():
    from spark_gpt_b200 import SparseMoE, check_faults
    from spark_gpt_b200.grad_sync import GradSync
    cfg = SimpleNamespace(hidden_size=1024, num_experts=64, num_experts_per_tok=8,
                          moe_intermediate_size=256, norm_topk_prob=True)
    torch.manual_seed(5)
    m = SparseMoE(cfg).to(DEV)
    with torch.no_grad():
        m.gate.weight.normal_(0, 0.02)
        m.experts.gate_up_proj.normal_(0, 0.01)
        m.experts.down_proj.normal_(0, 0.002)
    x = torch.randn(4096, 1024, device=DEV).to(torch.bfloat16)
    d_out = (torch.randn(4096, 1024, device=DEV) * 1e-2).to(torch.bfloat16)

    def run():
        xin = x.clone().requires_grad_(True)
        out, logits, sel = m(xin)
        (out.float() * d_out.float()).sum().backward()
        return out.detach(), xin.grad

    out0, dx0 = run()
    ref = [p.grad.clone() for p in m.parameters()]
    for p in m.parameters():
        p.grad = None
    sync = GradSync(m)
    out1, dx1 = run()
    sync.wait()
    assert torch.equal(out1, out0) and torch.equal(dx1, dx0)
    for p, r, v in zip(m.parameters(), ref, [sync.views[2], sync.views[0], sync.views[1]]):
        assert p.grad.data_ptr() == v.data_ptr()
        assert torch.equal(p.grad, r)
    run()  # no zero_grad: the GEMMs add into the buffer
    sync.wait()
    for p, r in zip(m.parameters(), ref):
        # the same sum as autograd's r + r up to the association of the fp32
        # adds (the router's split-K partials are added to the buffer in turn)
        torch.testing.assert_close(p.grad, 2 * r, rtol=1e-5, atol=1e-6 * float(r.abs().max()))
    sync.detach()
    for p in m.parameters():
        p.grad = None
    run()
    for p, r in zip(m.parameters(), ref):
        assert torch.equal(p.grad, r)
    torch.cuda.synchronize()
    check_faults()
