"""Layer parity at the sizes and on the inputs that bench.py times.

bench.py measures the layer on full-size synthetic inputs:

* cfg2: 65,536 tokens, hidden 1024, 64 experts, top-8, intermediate 256,
  near-uniform routing;
* cfg3: 16,384 tokens, hidden 2048, 128 experts, top-8, intermediate 768,
  router logits skewed by a Zipf(1.1) per-expert bias so that the busiest
  expert receives about 8x the mean rows;
* cfg4: the MoE layer of BASELINE configs[3]'s 12-layer model (hidden 768,
  32 experts, top-4, intermediate 384) at that config's 65,536-token batch.

Each test builds exactly those inputs (bench.make_weights / make_tokens,
seed 0), runs SparseMoE forward + global_load_balancing_loss + backward on
the GPU, and checks every output against the oracle (oracle/moe_oracle.py,
pinned to the reference's own outputs) evaluated in fp32 on the same GPU with
TF32 off, on the same bf16 operand values and with the device's routing
injected:

* routing (expert ids and their order) bit-exact against the oracle's top-k
  of the device's logits, and the per-expert row counts equal;
* out, dx and the three weight gradients: max|d|/max|ref| <= 2e-2 and
  mean|d|/max|ref| <= 2e-3 (the layer's bf16 contract);
* aux loss within 1e-5 relative.

A scheduling or indexing fault that shows only at hundreds of thousands of
routed rows, or with one expert holding 8x the mean, fails here.
"""

import numpy as np
import pytest
import torch

import bench
from oracle import moe_oracle as O
from tests.helpers import assert_bf16_close

pytestmark = pytest.mark.gpu

DEV = "cuda"
COEF = bench.AUX_COEF


def _layer(c):
    from types import SimpleNamespace

    from spark_gpt_b200 import SparseMoE
    cfg = SimpleNamespace(hidden_size=c["H"], num_experts=c["E"], num_experts_per_tok=c["k"],
                          moe_intermediate_size=c["I"], norm_topk_prob=True)
    m = SparseMoE(cfg).to(DEV)
    w_r, w_gu, w_d = bench.make_weights(c, 0)
    with torch.no_grad():
        m.gate.weight.copy_(w_r)
        m.experts.gate_up_proj.copy_(w_gu)
        m.experts.down_proj.copy_(w_d)
    return m


@pytest.mark.parametrize("name", ["cfg2", "cfg3", "cfg4"])
def test_layer_at_benchmarked_size(name):
    from spark_gpt_b200 import _lib, global_load_balancing_loss, ops
    assert not torch.backends.cuda.matmul.allow_tf32, "the fp32 oracle needs TF32 off"
    c = dict(bench.CONFIGS[name])
    T, E, k = c["T"], c["E"], c["k"]
    m = _layer(c)
    x_h, d_h = bench.make_tokens(c, T, 0)
    x = x_h.to(torch.bfloat16).to(DEV)
    d_out = d_h.to(torch.bfloat16).to(DEV)
    del x_h, d_h
    valid = torch.ones(T, dtype=torch.bool, device=DEV)

    xin = x.clone().requires_grad_(True)
    out, logits, sel = m(xin)
    aux, stats = global_load_balancing_loss((logits,), (sel,), valid, num_experts=E, top_k=k)
    torch.autograd.backward([out, aux], [d_out, torch.tensor(COEF, device=DEV)])
    torch.cuda.synchronize()
    assert _lib.read_fault() == 0

    # routing: bit-exact top-k of the device logits (ties toward the lower index)
    lg = logits.detach().float()
    ref_sel = O.router_select(lg, k, True)[2]
    assert torch.equal(sel, ref_sel), "expert ids differ from the oracle's top-k"
    counts = np.bincount(sel.cpu().numpy().reshape(-1), minlength=E)
    rw = ops.router_topk(logits.detach().contiguous(), E, k, True)[1]

    bf = lambda t: t.detach().to(torch.bfloat16).float()  # noqa: E731
    r_aux, _, g_aux = O.load_balancing_loss((lg,), (sel,), valid, num_experts=E, top_k=k)
    res = O.layer_forward_backward(
        bf(x), bf(m.gate.weight), bf(m.experts.gate_up_proj), bf(m.experts.down_proj), k,
        bf(d_out), selected=sel, weights=rw.float(), logits=lg,
        d_logits_extra=(COEF * g_aux[0]).to(torch.bfloat16).float())
    assert np.array_equal(counts, res["dispatch"].counts)
    assert abs(float(aux) - float(r_aux)) <= 1e-5 * abs(float(r_aux))
    errs = {
        "out": assert_bf16_close(out, res["out"], "out"),
        "dx": assert_bf16_close(xin.grad, res["dx"], "dx"),
        "dW_gate_up": assert_bf16_close(m.experts.gate_up_proj.grad, res["dW_gate_up"],
                                        "dW_gate_up"),
        "dW_down": assert_bf16_close(m.experts.down_proj.grad, res["dW_down"], "dW_down"),
        "dW_router": assert_bf16_close(m.gate.weight.grad, res["dW_router"], "dW_router"),
    }
    mean_rows = T * k / E
    print(f"\n{name}: T={T} routed rows {T * k}, busiest expert {counts.max()} rows "
          f"({counts.max() / mean_rows:.2f}x mean), least busy {counts.min()}; aux "
          f"{float(aux):.6f} vs {float(r_aux):.6f}; " +
          ", ".join(f"{n}: max {v['max_rel']:.2e} mean {v['mean_rel']:.2e}"
                    for n, v in errs.items()))
    if c["routing"].startswith("zipf"):
        # the skew bench.py times is really applied
        assert counts.max() >= 6 * mean_rows


def _tie_logits(T, E, k, seed):
    g = torch.Generator().manual_seed(seed)
    lg = (torch.randn(T, E, generator=g) * 0.9).to(torch.bfloat16)
    lg[:64] = lg[:64, :1].expand(-1, E).clone()  # every logit of the row equal
    # rows whose k-th and following logits are equal (ties across the cut)
    lg[64:128] = (torch.randn(64, E, generator=g) * 0.1 - 5.0).to(torch.bfloat16)
    lg[64:128, 3:3 + min(k + 2, E - 3)] = 1.0
    return lg


@pytest.mark.parametrize("E,k", [(64, 8), (128, 8), (256, 16), (32, 4), (8, 2)])
def test_topk_matches_torch_cuda(E, k):
    """The reference's router on CUDA is F.softmax(logits, dtype=float32)
    followed by torch.topk and the renormalisation (train.py:2145-2153).  On
    bf16 logits (many exact ties) the library's selection must equal it:
    the same expert ids in the same order, and routing weights within one
    bf16 unit in the last place (the fp32 softmax and renormalisation sum
    in a different order, which can move a weight across a bf16 rounding
    boundary)."""
    from spark_gpt_b200 import ops
    T = 65536
    lg = _tie_logits(T, E, k, E * 31 + k).to(DEV).contiguous()
    sel, w = ops.router_topk(lg, E, k, True)
    p = torch.softmax(lg, dim=-1, dtype=torch.float32)
    rv, rs = torch.topk(p, k, dim=-1)
    rw = (rv / rv.sum(dim=-1, keepdim=True)).to(torch.bfloat16)
    set_diff = int((sel.sort(-1).values != rs.sort(-1).values).any(-1).sum())
    order_diff = int((sel != rs).any(-1).sum())
    ulp = torch.finfo(torch.bfloat16).eps * rw.float().abs().clamp_min(2 ** -126)
    w_diff = (w.float() - rw.float()).abs()
    w_off = int((w_diff > 0).sum())
    print(f"\nE={E} k={k}: rows with another expert set {set_diff}, another order "
          f"{order_diff}; weights off by one bf16 ulp {w_off} of {T * k}")
    assert set_diff == 0
    assert order_diff == 0
    assert bool((w_diff <= ulp).all())
