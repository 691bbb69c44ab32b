"""Pin the CPU oracle against golden vectors made by the reference itself.

The fixtures come from tests/golden/make_golden.py, which runs spark-gpt's own
SparseMoE / global_load_balancing_loss (train.py:2325-2334, 3098-3197) and its
MuonAdamWHybrid / _newtonschulz5_batched (train.py:2877-3024).
"""

import numpy as np
import pytest
import torch

from oracle import moe_oracle as O


def close(a, b, rtol=1e-5, atol=1e-6):
    torch.testing.assert_close(a.float(), b.float(), rtol=rtol, atol=atol)


def test_router_known_case(golden):
    c = golden["router_known"]
    logits, probs, w, sel = O.router_forward(c["x"], c["w_router"], c["top_k"], c["norm"])
    close(logits, c["logits"])
    assert torch.equal(sel, c["selected"])
    close(w, c["weights"])


def test_experts_with_given_routing(golden):
    c = golden["experts_given_routing"]
    k = c["selected"].shape[1]
    d = O.dispatch(c["selected"], c["w_gate_up"].shape[0])
    sw = c["weights"].reshape(-1)[torch.from_numpy(d.permutation)]
    xs = O.gather_forward(c["x"], d)
    gu, h = O.swiglu_forward(xs, c["w_gate_up"], d.offsets)
    y = O.grouped_linear_forward(h, c["w_down"], d.offsets)
    out = O.combine_forward(y, sw, d)
    close(out, c["out"])
    dy, _ = O.combine_backward(y, sw, d, c["probe"])
    dh, dwd = O.grouped_linear_backward(h, c["w_down"], dy, d.offsets)
    dxs, dwgu, _ = O.swiglu_backward(xs, c["w_gate_up"], gu, dh, d.offsets)
    close(O.gather_backward(dxs, d), c["dx"])
    close(dwgu, c["dW_gate_up"])
    close(dwd, c["dW_down"])
    assert k == 2


def test_aux_loss_masked_and_filler(golden):
    c = golden["aux_masked"]
    aux, stats, grads = O.load_balancing_loss((c["logits"],), (c["selected"],), c["valid"],
                                              num_experts=4, top_k=2)
    close(aux, c["aux"])
    close(grads[0], c["d_logits"])
    for k, v in stats.items():
        close(v, c["stat_" + k])
    assert torch.all(grads[0][-1] == 0)
    c = golden["aux_all_filler"]
    aux, _, grads = O.load_balancing_loss((c["logits"],), (c["selected"],), c["valid"],
                                          num_experts=4, top_k=2)
    assert float(aux) == 0.0 and float(c["aux"]) == 0.0
    assert torch.all(grads[0] == 0)


def assert_same_dispatch(d, ref_perm, selected):
    """The reference sorts with torch.sort(stable=False) (train.py:2275): the
    order of rows inside one expert's segment is implementation-defined (torch
    CPU's small-size sort is not stable).  Pin what is defined: the segments
    hold the same flat indices, and our order inside them is the stable one
    (expert, flat index) that torch.sort(stable=True) gives."""
    flat = selected.reshape(-1)
    stable = torch.sort(flat, stable=True).indices.numpy()
    assert np.array_equal(d.permutation, stable)
    for e, s, t in O.expert_ranges(d.offsets):
        assert np.array_equal(np.sort(d.permutation[s:t]), np.sort(ref_perm[s:t])), e
    inv = np.empty_like(d.permutation)
    inv[d.permutation] = np.arange(d.permutation.size)
    assert np.array_equal(inv, d.inverse)


def _layer(c):
    T = c["x"].shape[0]
    aux, stats, g_aux = O.load_balancing_loss(
        None or (c["x"].float() @ c["w_router"].t(),), None or (c["selected"],), c["valid"],
        num_experts=c["w_gate_up"].shape[0], top_k=c["top_k"])
    res = O.layer_forward_backward(c["x"], c["w_router"], c["w_gate_up"], c["w_down"],
                                   c["top_k"], c["probe"], norm_topk_prob=c["norm"],
                                   d_logits_extra=1e-3 * g_aux[0])
    return res, aux, stats, T


def test_small_layers_match_reference(golden):
    for name in ("layer_small", "layer_nonorm_filler", "layer_wide_k8"):
        c = golden[name]
        res, aux, stats, _ = _layer(c)
        assert torch.equal(res["selected"], c["selected"]), name
        d = res["dispatch"]
        assert_same_dispatch(d, c["permutation"].numpy(), c["selected"]), name
        assert np.array_equal(d.offsets, c["offsets"].numpy()), name
        close(res["logits"], c["logits"])
        close(res["weights"], c["routing_weights"])
        close(res["out"], c["out"], rtol=1e-4, atol=1e-5)
        close(aux, c["aux"])
        for k, v in stats.items():
            close(v, c["stat_" + k])
        close(res["dx"], c["dx"], rtol=1e-4, atol=1e-5)
        close(res["dW_router"], c["dW_router"], rtol=1e-4, atol=1e-5)
        close(res["dW_gate_up"], c["dW_gate_up"], rtol=1e-4, atol=1e-5)
        close(res["dW_down"], c["dW_down"], rtol=1e-4, atol=1e-5)


def test_config1_matches_reference(golden):
    c = golden["config1"]
    T, H, E, k, I = c["shape"].tolist()
    from tests.golden.make_golden import seeded_inputs
    x, w_r, w_gu, w_d, probe = seeded_inputs(T, H, E, I, int(c["seed"]))
    sums = torch.stack([t.double().sum() for t in (x, w_r, w_gu, w_d, probe)])
    assert torch.allclose(sums, c["input_sums"], rtol=1e-12, atol=1e-9), "RNG drifted"
    valid = torch.ones(T, dtype=torch.bool)
    logits = x @ w_r.t()
    _, sel0 = O.topk_cuda_order(O.softmax_fp32(logits), k)
    aux, stats, g_aux = O.load_balancing_loss((logits,), (sel0,), valid, num_experts=E, top_k=k)
    res = O.layer_forward_backward(x, w_r, w_gu, w_d, k, probe, d_logits_extra=1e-3 * g_aux[0])
    assert torch.equal(res["selected"].to(torch.int8), c["selected"])
    assert_same_dispatch(res["dispatch"], c["permutation"].numpy().astype(np.int64), res["selected"])
    assert np.array_equal(res["dispatch"].offsets, c["offsets"].numpy())
    close(aux, c["aux"])
    for key in ("out", "logits", "dx"):
        close(res[key][:64], c[key + "_head"], rtol=1e-4, atol=1e-5)
        assert abs(float(res[key].double().norm()) / float(c[key + "_norm"]) - 1) < 1e-5
    close(res["weights"][:64], c["routing_weights_head"])
    for key in ("dW_router", "dW_gate_up", "dW_down"):
        close(res[key].reshape(-1)[:4096], c[key + "_head"], rtol=1e-4, atol=1e-6)
        assert abs(float(res[key].double().norm()) / float(c[key + "_norm"]) - 1) < 1e-5


# torch.topk of an all-equal row on a B200 (torch 2.11.0): the order its bitonic
# sort of the k winners leaves them in (the live comparison with torch.topk on
# tie-heavy logits is tests/test_gpu_fullsize.py::test_topk_matches_torch_cuda)
CUDA_ALL_TIE_ORDER = {
    2: [1, 0], 3: [2, 1, 0], 4: [1, 0, 2, 3], 8: [7, 6, 4, 5, 1, 0, 2, 3],
    16: [7, 6, 4, 5, 1, 0, 2, 3, 11, 10, 8, 9, 13, 12, 14, 15],
}


@pytest.mark.parametrize("k", sorted(CUDA_ALL_TIE_ORDER))
def test_topk_cuda_order_of_an_all_tie_row(k):
    for E in (k, 32, 256):
        if E >= k:
            _, i = O.topk_cuda_order(torch.ones(3, E), k)
            assert i.tolist() == [CUDA_ALL_TIE_ORDER[k]] * 3


def test_topk_tie_rule_set_and_order():
    # the set: lowest indices among the values equal to the k-th
    p = torch.tensor([[0.5, 1.0, 1.0, 1.0, 0.2]])
    v, i = O.topk_cuda_order(p, 2)
    assert sorted(i[0].tolist()) == [1, 2] and i.tolist() == [[2, 1]]
    v, i = O.topk_cuda_order(torch.tensor([[0.1, 0.3, 0.3, 0.2]]), 3)
    assert i.tolist() == [[2, 1, 3]]
    assert torch.allclose(v, torch.tensor([[0.3, 0.3, 0.2]]))
    # no ties: plain descending order
    v, i = O.topk_cuda_order(torch.tensor([[0.1, 0.4, 0.2, 0.3]]), 3)
    assert i.tolist() == [[1, 3, 2]]


def test_dispatch_empty_and_all_one_expert():
    sel = torch.tensor([[2, 0], [2, 0], [0, 2]])
    d = O.dispatch(sel, 4)
    assert d.counts.tolist() == [3, 0, 3, 0]
    assert d.offsets.tolist() == [3, 3, 6, 6]
    # rows ordered by (expert, token): expert 0 <- tokens 0,1,2 ; expert 2 <- tokens 0,1,2
    assert d.token_index.tolist() == [0, 1, 2, 0, 1, 2]


# --------------------------------------------------------------------------- #
# Muon on the packed expert tensors (train.py:2877-3024)
# --------------------------------------------------------------------------- #
@pytest.fixture(scope="module")
def muon_golden():
    from tests.conftest import ROOT
    return torch.load(ROOT / "tests" / "golden" / "muon_golden.pt", weights_only=True)


@pytest.mark.parametrize("name", ["muon_wide", "muon_tall", "muon_square_plain"])
def test_muon_oracle_matches_reference_steps(muon_golden, name):
    from oracle import muon_oracle as M
    from tests.golden.make_golden import MUON_CASES, muon_case_inputs
    from tests.helpers import assert_bf16_close
    E, rows, cols, lr, mom, nest, seed = MUON_CASES[name]
    p0, grads = muon_case_inputs(E, rows, cols, seed)
    c = muon_golden[name]
    assert torch.isclose(c["input_sum"], p0.double().sum() + sum(g.double().sum() for g in grads))
    p, v = p0.clone(), torch.zeros_like(p0)
    for g in grads:
        p, v = M.muon_step(p, g, v, lr, mom, nest)
    torch.testing.assert_close(v, c["v2"], rtol=1e-6, atol=1e-9)
    assert_bf16_close(p - p0, c["delta2"], f"{name} update")


@pytest.mark.parametrize("name", ["ns_wide", "ns_tall"])
def test_newton_schulz_oracle_matches_reference(muon_golden, name):
    from oracle import muon_oracle as M
    from tests.golden.make_golden import NS_CASES, ns_case_input
    from tests.helpers import assert_bf16_close
    shape, seed = NS_CASES[name]
    out = M.newton_schulz(ns_case_input(shape, seed), steps=5)
    assert out.dtype == torch.bfloat16 and out.shape == shape
    assert_bf16_close(out, muon_golden[name]["out"], name)


@pytest.mark.parametrize("case", ["norm_bf16", "norm_f32"])
def test_rmsnorm_oracle_matches_reference(case):
    """The oracle's RMSNorm against the reference's own RMSNorm module
    (tests/golden/norm_golden.pt, made by make_golden.py --only norm): the
    forward bit-exact; the backward, which the reference runs through bf16
    autograd ops for bf16 input, within the layer's bf16 contract (max 2e-2 /
    mean 2e-3 of the reference tensor's scale), and to fp32 rounding for fp32
    input."""
    from tests.conftest import ROOT
    from tests.helpers import assert_bf16_close
    c = torch.load(ROOT / "tests" / "golden" / "norm_golden.pt", weights_only=True)[case]
    bf = c["x"].dtype == torch.bfloat16
    x_n, r = O.rmsnorm_forward(c["x"], c["w"], float(c["eps"]))
    assert torch.equal(x_n, c["out"].float())
    dx, dw = O.rmsnorm_backward(c["x"], c["w"], r, c["probe"], bf16_io=bf)
    if bf:
        assert_bf16_close(dx, c["dx"].float(), "dx")
        assert_bf16_close(dw, c["dw"].float(), "dw")
    else:
        torch.testing.assert_close(dx, c["dx"], rtol=1e-5, atol=1e-6)
        torch.testing.assert_close(dw, c["dw"], rtol=1e-5, atol=1e-6)


def test_fp8_oracle_matches_reference_torch_pieces():
    """The fp8 oracle's per-expert e4m3 weight copies and delayed-scale update
    against the reference's own _fp8_quantize_experts and fp8_update_scales
    (tests/golden/fp8_golden.pt, made by make_golden.py --only fp8): bit-exact,
    including an all-zero expert, an amax that is an exact power of two, and
    amax slots that recorded nothing (the scale is kept)."""
    from oracle import fp8_oracle as F8
    from tests.conftest import ROOT
    c = torch.load(ROOT / "tests" / "golden" / "fp8_golden.pt", weights_only=True)
    q = c["quantize_experts"]
    w8, qe = F8.quantize_experts(q["w"])
    assert torch.equal(qe, q["q"])
    assert torch.equal(w8.view(torch.uint8), q["w8"])
    u = c["update_scales"]
    for a, s_out, a_out in zip(u["amax"], u["scale_out"], u["amax_out"]):
        s = u["scale_in"].clone()
        am = a.clone()
        F8.update_scales(s, am)
        assert torch.equal(s, s_out)
        assert torch.equal(am, a_out)
