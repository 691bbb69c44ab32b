"""GPU parity of the HBM-bound kernels: router top-k, dispatch, gather,
combine and the load-balancing statistics, against the CPU oracle (which is
pinned to the reference's golden vectors)."""

import numpy as np
import pytest
import torch

from oracle import moe_oracle as O
from tests.helpers import unpadded_permutation

pytestmark = pytest.mark.gpu

DEV = "cuda"


@pytest.fixture(scope="module")
def ops():
    from spark_gpt_b200 import ops as _ops
    return _ops


def _topk_ref(logits_cpu, k, norm):
    probs, w, sel = O.router_select(logits_cpu.float(), k, norm)
    return sel, w


@pytest.mark.parametrize("case", ["layer_small", "layer_nonorm_filler", "layer_wide_k8"])
def test_topk_bit_exact_on_reference_logits(ops, golden, case):
    """Expert indices equal the reference's, given the reference's fp32 logits."""
    c = golden[case]
    E = c["w_router"].shape[0]
    lg = c["logits"].float().contiguous().to(DEV)
    sel, w = ops.router_topk(lg, E, c["top_k"], c["norm"])
    assert torch.equal(sel.cpu(), c["selected"])
    ref_w = c["routing_weights"].float().to(torch.bfloat16).float()
    assert (w.float().cpu() - ref_w).abs().max() <= 2 ** -8 * ref_w.abs().max()


def test_topk_bit_exact_config1(ops, golden):
    c = golden["config1"]
    T, H, E, k, I = c["shape"].tolist()
    from tests.golden.make_golden import seeded_inputs
    x, w_r, *_ = seeded_inputs(T, H, E, I, int(c["seed"]))
    lg = (x @ w_r.t()).contiguous()
    sel, _ = ops.router_topk(lg.to(DEV), E, k, True)
    assert torch.equal(sel.cpu().to(torch.int8), c["selected"])


@pytest.mark.parametrize("E,k,dtype", [(128, 8, torch.float32), (128, 8, torch.bfloat16),
                                       (64, 8, torch.bfloat16), (8, 2, torch.bfloat16),
                                       (256, 16, torch.bfloat16), (40, 3, torch.float32)])
def test_topk_matches_oracle_with_ties(ops, E, k, dtype):
    """bf16 logits produce many exact ties; the selected set and order follow
    the stated rule (probability desc, lower index first)."""
    g = torch.Generator().manual_seed(E * 31 + k)
    T = 20000
    lg = (torch.randn(T, E, generator=g) * 0.9).to(dtype)
    # rows with deliberate ties at the k-th position
    lg[:50] = lg[:50, :1].expand(-1, E).clone()
    sel, w = ops.router_topk(lg.contiguous().to(DEV), E, k, True)
    ref_sel, ref_w = _topk_ref(lg.float(), k, True)
    assert torch.equal(sel.cpu(), ref_sel)
    assert (w.float().cpu() - ref_w.to(torch.bfloat16).float()).abs().max() <= 2 ** -8


@pytest.mark.parametrize("T,k,E,skew", [(1000, 2, 8, True), (20000, 8, 64, False),
                                        (7, 3, 5, False), (4096, 8, 128, True)])
def test_dispatch_bit_exact(ops, T, k, E, skew):
    g = torch.Generator().manual_seed(T + E)
    if skew:
        # experts 0..E/4 get nothing, the last expert gets most rows
        p = torch.zeros(E)
        p[E // 4:] = 1.0
        p[-1] = 20.0
        sel = torch.stack([torch.multinomial(p, k, replacement=False, generator=g)
                           for _ in range(T)])
    else:
        sel = torch.stack([torch.randperm(E, generator=g)[:k] for _ in range(T)])
    d = ops.dispatch(sel.to(DEV).contiguous(), E)
    ref = O.dispatch(sel, E)
    assert np.array_equal(d.counts.cpu().numpy(), ref.counts)
    assert np.array_equal(d.offsets.cpu().numpy(), ref.offsets)
    assert np.array_equal(unpadded_permutation(d.row_flat, d.pad_offsets), ref.permutation)
    pad = d.pad_offsets.cpu().numpy()
    counts = ref.counts
    assert pad[0] == 0 and np.all(pad % 128 == 0)
    assert np.array_equal(np.diff(pad), (counts + 127) // 128 * 128)
    rf = d.row_flat.cpu().numpy()
    inv = d.inv_pad.cpu().numpy()
    assert np.array_equal(rf[inv], np.arange(T * k))
    for e in range(E):
        assert np.all(rf[pad[e] + counts[e]:pad[e + 1]] == -1)
    te = d.tile_expert.cpu().numpy()[: pad[-1] // 128]
    assert np.array_equal(te, np.repeat(np.arange(E), np.diff(pad) // 128))
    from spark_gpt_b200 import _lib
    assert _lib.read_fault() == 0


def _routing(T, k, E, seed):
    g = torch.Generator().manual_seed(seed)
    return torch.stack([torch.randperm(E, generator=g)[:k] for _ in range(T)])


def test_gather_and_backward(ops):
    T, k, E, H = 3000, 4, 16, 256
    sel = _routing(T, k, E, 1)
    x = torch.randn(T, H).to(torch.bfloat16)
    d = ops.dispatch(sel.to(DEV), E)
    xs = ops.gather_rows(x.to(DEV), d)
    ref = O.dispatch(sel, E)
    perm = unpadded_permutation(d.row_flat, d.pad_offsets)
    rows = d.row_flat.cpu().numpy()[: int(d.pad_offsets[-1])]
    xs_c = xs.cpu()[: int(d.pad_offsets[-1])]
    assert torch.equal(xs_c[torch.from_numpy(rows >= 0)], x[torch.from_numpy(perm // k)])
    assert torch.all(xs_c[torch.from_numpy(rows < 0)] == 0)
    # backward: sum of the k slot rows (+ addend)
    dxs = torch.randn(d.rows_cap, H).to(torch.bfloat16)
    add = torch.randn(T, H).to(torch.bfloat16)
    dx = ops.gather_rows_bwd(dxs.to(DEV), d, addend=add.to(DEV)).cpu().float()
    inv = d.inv_pad.cpu().long().view(T, k)
    ref_dx = dxs.float()[inv].sum(1) + add.float()
    assert (dx - ref_dx).abs().max() <= 2 ** -7 * ref_dx.abs().max()
    assert ref.permutation.size == perm.size


def test_combine_and_backward(ops):
    T, k, E, H = 2500, 8, 64, 512
    sel = _routing(T, k, E, 2)
    d = ops.dispatch(sel.to(DEV), E)
    y = torch.randn(d.rows_cap, H).to(torch.bfloat16)
    w = torch.rand(T, k).to(torch.bfloat16)
    out = ops.combine(y.to(DEV), d, w.to(DEV)).cpu().float()
    inv = d.inv_pad.cpu().long().view(T, k)
    weighted = (y.float()[inv] * w.float().unsqueeze(-1)).to(torch.bfloat16).float()
    ref = weighted.sum(1)
    assert (out - ref).abs().max() <= 2 ** -7 * ref.abs().max()
    d_out = torch.randn(T, H).to(torch.bfloat16)
    dy, dw = ops.combine_bwd(d_out.to(DEV), y.to(DEV), d, w.to(DEV))
    dy, dw = dy.cpu().float(), dw.cpu()
    rf = d.row_flat.cpu().long()[: int(d.pad_offsets[-1])]
    valid = rf >= 0
    f = rf[valid]
    ref_dy = (d_out.float()[f // k] * w.float().view(-1)[f].unsqueeze(-1)).to(torch.bfloat16).float()
    assert torch.equal(dy[: len(rf)][valid], ref_dy)
    assert torch.all(dy[: len(rf)][~valid] == 0)
    ref_dw = (d_out.float()[f // k] * y.float()[: len(rf)][valid]).sum(-1)
    got = dw.view(-1)[f]
    assert (got - ref_dw).abs().max() <= 1e-4 * ref_dw.abs().max()


@pytest.mark.parametrize("E,k,filler", [(64, 8, 100), (8, 2, 0), (128, 8, 3000)])
def test_load_balance_stats_and_grad(ops, E, k, filler):
    T = 4096
    g = torch.Generator().manual_seed(E)
    lg = (torch.randn(T, E, generator=g) * 2).to(torch.bfloat16)
    sel, _ = _topk_ref(lg.float(), k, True)
    valid = torch.ones(T, dtype=torch.bool)
    if filler:
        valid[-filler:] = False
    W = ops.router_width(E)
    buf = torch.zeros(T, W, dtype=torch.bfloat16)
    buf[:, :E] = lg
    lg_dev = buf.to(DEV)[:, :E]
    packed = torch.zeros(2 * E + 2, device=DEV)
    v8 = valid.to(torch.uint8).to(DEV)
    ops.lb_stats(lg_dev, sel.to(DEV), v8, E, k, packed)
    aux, stats, coef = ops.lb_finalize(packed, E, k, 1)
    r_aux, r_stats, r_grads = O.load_balancing_loss((lg.float(),), (sel,), valid,
                                                    num_experts=E, top_k=k)
    assert abs(float(aux) - float(r_aux)) <= 1e-5 * abs(float(r_aux))
    for i, key in enumerate(["assignment_min_frac", "assignment_max_frac", "assignment_cv",
                             "router_entropy", "unused_experts"]):
        assert abs(float(stats[i]) - float(r_stats[key])) <= 1e-5 * abs(float(r_stats[key])) + 1e-7, key
    grad = torch.full((1,), 0.37, device=DEV)
    dl = ops.lb_grad(lg_dev, v8, coef, grad, E).cpu().float()[:, :E]
    ref = (0.37 * r_grads[0]).to(torch.bfloat16).float()
    assert (dl - ref).abs().max() <= 2 ** -7 * ref.abs().max() + 1e-12
    if filler:
        assert torch.all(dl[~valid] == 0)


@pytest.mark.parametrize("T,k,E,H", [(2500, 8, 64, 512), (3000, 4, 16, 256), (700, 2, 8, 128),
                                     (513, 8, 128, 2048)])
def test_token_major_combine_paths_equal_padded(ops, T, k, E, H):
    """The token-major layout (slot t*k+s in row t*k+s) gives the same results
    as the padded-row layout, bit for bit."""
    sel = _routing(T, k, E, 3)
    d = ops.dispatch(sel.to(DEV), E)
    n = int(d.pad_offsets[-1])
    y = torch.randn(d.rows_cap, H, device=DEV).to(torch.bfloat16)
    rf = d.row_flat[:n].long()
    y_tok = torch.empty(T * k, H, device=DEV, dtype=torch.bfloat16)
    y_tok[rf[rf >= 0]] = y[:n][rf >= 0]
    w = torch.rand(T, k, device=DEV).to(torch.bfloat16)
    assert torch.equal(ops.combine(y, d, w), ops.combine(y_tok, d, w, token_major=True))
    add = torch.randn(T, H, device=DEV).to(torch.bfloat16)
    assert torch.equal(ops.gather_rows_bwd(y, d, addend=add),
                       ops.gather_rows_bwd(y_tok, d, addend=add, token_major=True))
    d_out = torch.randn(T, H, device=DEV).to(torch.bfloat16)
    dy0, dw0 = ops.combine_bwd(d_out, y, d, w)
    dy1, dw1 = ops.combine_bwd(d_out, y_tok, d, w, token_major=True)
    assert torch.equal(dy0[:n], dy1[:n])
    assert torch.all(dy1[:n][rf < 0] == 0)
    torch.testing.assert_close(dw0, dw1, rtol=1e-6, atol=1e-6)
