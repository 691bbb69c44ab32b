"""Muon on the packed expert tensors (spark_gpt_b200.muon) against the CPU
oracle, which is pinned to the reference's own MuonAdamWHybrid steps.

Tolerances: the momentum buffer within fp32 rounding (1e-6 relative); the
parameter updates within the layer's bf16 tolerance (max|d| / max|ref| <=
2e-2, mean <= 2e-3).  The bf16 Newton-Schulz iterate on its own gets
max <= 4e-2 (mean still <= 2e-3): five chained products, each rounded to bf16,
turn a one-ulp difference of one fp32 accumulation order into a few ulps at a
few elements (the oracle and the reference's own CPU path already differ by
1.9e-2 max on the golden cases).
"""

NS_MAX_REL = 4e-2

import pytest
import torch

from oracle import muon_oracle as M
from tests.helpers import assert_bf16_close

pytestmark = pytest.mark.gpu

DEV = "cuda"


@pytest.fixture(scope="module")
def muon():
    from spark_gpt_b200 import muon as _muon
    return _muon


def test_momentum_stage(muon):
    g = torch.Generator().manual_seed(5)
    grad = torch.randn(3, 256, 384, generator=g) * 1e-3
    v = torch.randn(3, 256, 384, generator=g) * 1e-3
    for nest, mom in ((True, 0.95), (False, 0.9), (True, 0.3)):
        ref_v, ref_u = M.momentum_stage(grad, v, mom, nest)
        vd = v.clone().to(DEV)
        u = muon.momentum_stage(grad.to(DEV), vd, mom, nest).cpu()
        # the kernel's lerps are FMAs, the oracle's separate multiply and add
        torch.testing.assert_close(vd.cpu(), ref_v, rtol=1e-6, atol=1e-6 * float(ref_v.abs().max()))
        diff = (u.float() - ref_u.float()).abs()
        assert float(diff.max()) <= 2 ** -8 * float(ref_u.float().abs().max())
        assert float((diff > 0).float().mean()) < 1e-3


@pytest.mark.parametrize("shape", [(4, 256, 512), (3, 512, 256), (2, 128, 128), (8, 512, 1024),
                                   (8, 1024, 256), (2, 1536, 2048), (2, 2048, 768)])
def test_newton_schulz_matches_oracle(muon, shape):
    from spark_gpt_b200 import _lib
    g = torch.Generator().manual_seed(shape[1] + shape[2])
    x = (torch.randn(*shape, generator=g) * 1e-3).to(torch.bfloat16)
    ref = M.newton_schulz(x, 5)
    out = muon.newton_schulz(x.to(DEV).clone(), 5).cpu()
    assert_bf16_close(out, ref, f"ns {shape}", max_rel=NS_MAX_REL)
    torch.cuda.synchronize()
    assert _lib.read_fault() == 0


@pytest.mark.parametrize("name", ["ns_wide", "ns_tall"])
def test_newton_schulz_matches_reference_golden(muon, name):
    from tests.conftest import ROOT
    from tests.golden.make_golden import NS_CASES, ns_case_input
    gold = torch.load(ROOT / "tests" / "golden" / "muon_golden.pt", weights_only=True)
    shape, seed = NS_CASES[name]
    out = muon.newton_schulz(ns_case_input(shape, seed).to(DEV), 5).cpu()
    assert_bf16_close(out, gold[name]["out"], name, max_rel=NS_MAX_REL)


@pytest.mark.parametrize("name", ["muon_wide", "muon_tall", "muon_square_plain"])
def test_two_muon_steps_match_reference(muon, name):
    from tests.conftest import ROOT
    from tests.golden.make_golden import MUON_CASES, muon_case_inputs
    gold = torch.load(ROOT / "tests" / "golden" / "muon_golden.pt", weights_only=True)[name]
    E, rows, cols, lr, mom, nest, seed = MUON_CASES[name]
    p0, grads = muon_case_inputs(E, rows, cols, seed)
    p = torch.nn.Parameter(p0.clone().to(DEV))
    opt = muon.PackedExpertMuon([p], lr=lr, momentum=mom, nesterov=nest)
    for gr in grads:
        p.grad = gr.to(DEV)
        opt.step()
    torch.testing.assert_close(opt.state[p]["v"].cpu(), gold["v2"], rtol=1e-6,
                               atol=1e-6 * float(gold["v2"].abs().max()))
    assert_bf16_close(p.detach().cpu() - p0, gold["delta2"], f"{name} update")


def test_muon_step_on_layer_expert_gradients(muon):
    """The drop-in use: one backward of the B200 layer, then a Muon step of its
    packed expert tensors, against the oracle step on the same gradients."""
    from types import SimpleNamespace
    from spark_gpt_b200 import SparseMoE
    T, H, E, k, I = 4096, 1024, 16, 4, 256
    cfg = SimpleNamespace(hidden_size=H, num_experts=E, num_experts_per_tok=k,
                          moe_intermediate_size=I, norm_topk_prob=True)
    torch.manual_seed(0)
    m = SparseMoE(cfg).to(DEV)
    with torch.no_grad():
        m.gate.weight.normal_(0, 0.02)
        m.experts.gate_up_proj.normal_(0, 0.01)
        m.experts.down_proj.normal_(0, 0.01)
    x = torch.randn(T, H, device=DEV).to(torch.bfloat16)
    out, _, _ = m(x)
    out.float().square().mean().backward()
    params = [m.experts.gate_up_proj, m.experts.down_proj]
    before = [p.detach().cpu().clone() for p in params]
    grads = [p.grad.detach().cpu().clone() for p in params]
    opt = muon.PackedExpertMuon(params, lr=0.02)
    opt.step()
    for p, p0, g in zip(params, before, grads):
        ref, _ = M.muon_step(p0, g, torch.zeros_like(p0), 0.02)
        assert_bf16_close(p.detach().cpu() - p0, ref - p0, f"muon {tuple(p.shape)}")


def test_newton_schulz_orthogonalises_full_size(muon):
    """Size-independent property at the Qwen3-30B-A3B expert shape: the NS5
    iterate has every singular value of the normalised input pushed into the
    band the quintic's coefficients target (about 0.7 to 1.2)."""
    g = torch.Generator(device=DEV).manual_seed(1)
    x = torch.randn(8, 1536, 2048, device=DEV, generator=g).to(torch.bfloat16)
    out = muon.newton_schulz(x, 5)
    s = torch.linalg.svdvals(out.float())
    assert float(s.min()) > 0.5 and float(s.max()) < 1.3


def test_muon_streams_match_single_stream(muon):
    """The parameters' updates on two streams equal the one-stream step bit for
    bit (the same kernels, only overlapped), over three steps at the cfg2
    expert shapes, and the caller's stream sees the finished parameters."""
    g = torch.Generator(device=DEV).manual_seed(11)
    shapes = [(64, 512, 1024), (64, 1024, 256)]
    init = [torch.randn(*s, device=DEV, generator=g) * 0.01 for s in shapes]
    grads = [[torch.randn(*s, device=DEV, generator=g) * 1e-3 for s in shapes] for _ in range(3)]
    results = []
    for streams in (1, 2):
        params = [torch.nn.Parameter(t.clone()) for t in init]
        opt = muon.PackedExpertMuon(params, lr=0.02, streams=streams)
        for step_grads in grads:
            for p, gr in zip(params, step_grads):
                p.grad = gr.clone()
            opt.step()
        results.append([p.detach().clone() for p in params])  # on the caller's stream
    torch.cuda.synchronize()
    for a, b in zip(*results):
        assert torch.equal(a, b)
