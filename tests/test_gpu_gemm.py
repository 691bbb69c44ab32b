"""GPU parity of the tcgen05 grouped GEMMs (every contraction of the layer)
against fp32 per-expert products of the same bf16 operands."""

import pytest
import torch

from tests.helpers import assert_bf16_close, bf16_round

pytestmark = pytest.mark.gpu

DEV = "cuda"


@pytest.fixture(scope="module")
def ops():
    from spark_gpt_b200 import ops as _ops
    return _ops


def _skewed_routing(T, k, E, seed, empty=(1,)):
    """Routing with some empty experts and one heavy expert."""
    g = torch.Generator().manual_seed(seed)
    p = torch.ones(E)
    for e in empty:
        p[e] = 0.0
    p[-1] = 8.0
    return torch.stack([torch.multinomial(p, k, replacement=False, generator=g) for _ in range(T)])


def _setup(ops, T, k, E, H, I, seed):
    torch.manual_seed(seed)
    sel = _skewed_routing(T, k, E, seed)
    d = ops.dispatch(sel.to(DEV), E)
    x = torch.randn(T, H, device=DEV).to(torch.bfloat16)
    xs = ops.gather_rows(x, d)
    wgu = (torch.randn(E, 2 * I, H, device=DEV) * H ** -0.5).to(torch.bfloat16)
    wd = (torch.randn(E, H, I, device=DEV) * I ** -0.5).to(torch.bfloat16)
    return d, x, xs, wgu, wd


def _segments(d):
    pad = d.pad_offsets.cpu().tolist()
    for e in range(d.num_experts):
        yield e, pad[e], pad[e + 1]


SHAPES = [(1000, 2, 8, 256, 128), (600, 4, 6, 256, 192), (4096, 8, 64, 1024, 256),
          (512, 8, 16, 2048, 768)]


@pytest.mark.parametrize("T,k,E,H,I", SHAPES)
def test_gate_up_forward(ops, T, k, E, H, I):
    d, x, xs, wgu, wd = _setup(ops, T, k, E, H, I, 1)
    gu, h = ops.gate_up_fwd(xs, wgu, d)
    ref = torch.zeros(d.rows_cap, 2 * I, device=DEV)
    for e, s, t in _segments(d):
        if t > s:
            ref[s:t] = xs[s:t].float() @ wgu[e].float().t()
    n = int(d.pad_offsets[-1])
    assert_bf16_close(gu[:n], ref[:n], "gu", max_rel=1e-2, mean_rel=5e-4)
    g, u = gu[:n, :I].float(), gu[:n, I:].float()
    h_ref = bf16_round(g * torch.sigmoid(g) * u)
    assert_bf16_close(h[:n], h_ref, "h", max_rel=1e-2, mean_rel=2e-4)


@pytest.mark.parametrize("T,k,E,H,I", SHAPES)
def test_down_forward_and_dgrad_swiglu(ops, T, k, E, H, I):
    d, x, xs, wgu, wd = _setup(ops, T, k, E, H, I, 2)
    gu, h = ops.gate_up_fwd(xs, wgu, d)
    y = ops.down_fwd(h, wd, d)
    n = int(d.pad_offsets[-1])
    y_ref = torch.zeros(n, H, device=DEV)
    for e, s, t in _segments(d):
        if t > s:
            y_ref[s:t] = h[s:t].float() @ wd[e].float().t()
    assert_bf16_close(y[:n], y_ref, "y", max_rel=1e-2, mean_rel=5e-4)
    dy = torch.randn(d.rows_cap, H, device=DEV).to(torch.bfloat16)
    dy[n:] = 0
    d_gu = ops.down_dgrad_swiglu(dy, wd, gu, d)
    dh = torch.zeros(n, I, device=DEV)
    for e, s, t in _segments(d):
        if t > s:
            dh[s:t] = dy[s:t].float() @ wd[e].float()
    dh = bf16_round(dh)
    g, u = gu[:n, :I].float(), gu[:n, I:].float()
    sig = torch.sigmoid(g)
    ref = torch.cat([dh * u * (sig * (1 + g * (1 - sig))), dh * g * sig], 1)
    assert_bf16_close(d_gu[:n], ref, "d_gu", max_rel=2e-2, mean_rel=1e-3)


@pytest.mark.parametrize("T,k,E,H,I", SHAPES)
def test_gate_up_dgrad(ops, T, k, E, H, I):
    d, x, xs, wgu, wd = _setup(ops, T, k, E, H, I, 3)
    n = int(d.pad_offsets[-1])
    d_gu = torch.randn(d.rows_cap, 2 * I, device=DEV).to(torch.bfloat16)
    dxs = ops.gate_up_dgrad(d_gu, wgu, d)
    ref = torch.zeros(n, H, device=DEV)
    for e, s, t in _segments(d):
        if t > s:
            ref[s:t] = d_gu[s:t].float() @ wgu[e].float()
    assert_bf16_close(dxs[:n], ref, "dxs", max_rel=1e-2, mean_rel=5e-4)


@pytest.mark.parametrize("T,k,E,H,I", SHAPES)
def test_wgrads(ops, T, k, E, H, I):
    d, x, xs, wgu, wd = _setup(ops, T, k, E, H, I, 4)
    n = int(d.pad_offsets[-1])
    d_gu = torch.randn(d.rows_cap, 2 * I, device=DEV).to(torch.bfloat16)
    d_gu[n:] = 0
    rows = d.row_flat[: d.rows_cap].clone()
    rows[n:] = -1
    d_gu[rows < 0] = 0  # padding rows carry zero gradients in the layer
    dw = ops.wgrad(d_gu, xs, d)
    ref = torch.zeros(E, 2 * I, H, device=DEV)
    for e, s, t in _segments(d):
        if t > s:
            ref[e] = d_gu[s:t].float().t() @ xs[s:t].float()
    torch.testing.assert_close(dw, ref, rtol=1e-3, atol=1e-3 * ref.abs().max().item())
    # accumulate into an existing gradient
    dw2 = ops.wgrad(d_gu, xs, d, out=dw.clone(), accumulate=True)
    torch.testing.assert_close(dw2, 2 * ref, rtol=1e-3, atol=2e-3 * ref.abs().max().item())
    # empty experts get exact zeros
    counts = d.counts.cpu()
    for e in range(E):
        if counts[e] == 0:
            assert torch.all(dw[e] == 0)
    dy = torch.randn(d.rows_cap, H, device=DEV).to(torch.bfloat16)
    dy[rows < 0] = 0
    h = torch.randn(d.rows_cap, I, device=DEV).to(torch.bfloat16)
    dwd = ops.wgrad(dy, h, d)
    ref = torch.zeros(E, H, I, device=DEV)
    for e, s, t in _segments(d):
        if t > s:
            ref[e] = dy[s:t].float().t() @ h[s:t].float()
    torch.testing.assert_close(dwd, ref, rtol=1e-3, atol=1e-3 * ref.abs().max().item())


@pytest.mark.parametrize("T,H,E", [(1000, 256, 8), (65536 // 16, 1024, 64), (3000, 2048, 128),
                                   (777, 768, 256)])
def test_router_gemms(ops, T, H, E):
    torch.manual_seed(5)
    W = ops.router_width(E)
    x = torch.randn(T, H, device=DEV).to(torch.bfloat16)
    w = torch.randn(E, H, device=DEV) * 0.02
    wb = ops.cast_bf16(w, W)
    assert torch.all(wb[E:] == 0)
    assert torch.equal(wb[:E], w.to(torch.bfloat16))
    logits = ops.router_logits(x, wb)
    ref = x.float() @ wb.float().t()
    assert_bf16_close(logits, ref, "logits", max_rel=1e-2, mean_rel=5e-4)
    dl = torch.randn(T, W, device=DEV).to(torch.bfloat16)
    dl[:, E:] = 0
    dx = ops.router_dgrad(dl, wb)
    assert_bf16_close(dx, dl.float() @ wb.float(), "router dx", max_rel=1e-2, mean_rel=5e-4)
    dw = ops.router_wgrad(x, dl, E)
    ref = dl[:, :E].float().t() @ x.float()
    torch.testing.assert_close(dw, ref, rtol=1e-3, atol=1e-3 * ref.abs().max().item())


# --------------------------------------------------------------------------- #
# gathered-operand variants: identical operands to the materialised path, so
# results must match it bit for bit
# --------------------------------------------------------------------------- #
@pytest.mark.parametrize("T,k,E,H,I", SHAPES)
def test_gate_up_forward_gather_equals_materialised(ops, T, k, E, H, I):
    d, x, xs, wgu, wd = _setup(ops, T, k, E, H, I, 6)
    n = int(d.pad_offsets[-1])
    gu0, h0 = ops.gate_up_fwd(xs, wgu, d)
    gu1, h1 = ops.gate_up_fwd_gather(x, wgu, d)
    assert torch.equal(gu0[:n], gu1[:n])
    assert torch.equal(h0[:n], h1[:n])


@pytest.mark.parametrize("T,k,E,H,I", SHAPES)
def test_wgrad_gathers_equal_materialised(ops, T, k, E, H, I):
    d, x, xs, wgu, wd = _setup(ops, T, k, E, H, I, 7)
    n = int(d.pad_offsets[-1])
    rows = d.row_flat.clone()
    rows[n:] = -1
    d_gu = torch.randn(d.rows_cap, 2 * I, device=DEV).to(torch.bfloat16)
    d_gu[rows < 0] = 0
    assert torch.equal(ops.wgrad(d_gu, xs, d), ops.wgrad_gather_b(d_gu, x, d))
    d_out = torch.randn(T, H, device=DEV).to(torch.bfloat16)
    douts = ops.gather_rows(d_out, d)
    hw = torch.randn(d.rows_cap, I, device=DEV).to(torch.bfloat16)
    hw[rows < 0] = 0
    assert torch.equal(ops.wgrad(douts, hw, d), ops.wgrad_gather_a(d_out, hw, d))


@pytest.mark.parametrize("T,k,E,H,I", SHAPES)
def test_down_dgrad_with_combine_backward(ops, T, k, E, H, I):
    d, x, xs, wgu, wd = _setup(ops, T, k, E, H, I, 8)
    n = int(d.pad_offsets[-1])
    gu, h = ops.gate_up_fwd(xs, wgu, d)
    w = torch.rand(T, k, device=DEV).to(torch.bfloat16)
    d_out = torch.randn(T, H, device=DEV).to(torch.bfloat16)
    d_gu, hw, d_w = ops.down_dgrad_combine(d_out, w, wd, gu, h, d)
    rows = d.row_flat[:n].long()
    valid = rows >= 0
    tok = torch.where(valid, rows // k, torch.zeros_like(rows))
    wr = torch.where(valid, w.view(-1)[rows.clamp_min(0)].float(), torch.zeros_like(rows, dtype=torch.float32))
    acc = torch.zeros(n, I, device=DEV)
    for e, s, t in _segments(d):
        if t > s:
            acc[s:t] = d_out[tok[s:t]].float() @ wd[e].float()
    acc[~valid] = 0
    dh = bf16_round(wr[:, None] * acc)
    g, u = gu[:n, :I].float(), gu[:n, I:].float()
    sig = torch.sigmoid(g)
    ref = torch.cat([dh * u * (sig * (1 + g * (1 - sig))), dh * g * sig], 1)
    assert_bf16_close(d_gu[:n], ref, "d_gu", max_rel=2e-2, mean_rel=1e-3)
    assert torch.equal(hw[:n], (wr[:, None] * h[:n].float()).to(torch.bfloat16))
    ref_dw = (acc * h[:n].float()).sum(1)
    got = d_w.view(-1)[rows[valid]]
    torch.testing.assert_close(got, ref_dw[valid], rtol=1e-3, atol=1e-3 * ref_dw.abs().max().item())


@pytest.mark.parametrize("T,k,E,H,I", SHAPES)
def test_token_major_outputs_equal_padded(ops, T, k, E, H, I):
    """down fwd / gate_up dgrad writing rows in token order (row t*k+s) give the
    padded-order rows, permuted."""
    d, x, xs, wgu, wd = _setup(ops, T, k, E, H, I, 9)
    n = int(d.pad_offsets[-1])
    rf = d.row_flat[:n].long()
    gu, h = ops.gate_up_fwd(xs, wgu, d)
    y0 = ops.down_fwd(h, wd, d)
    y1 = ops.down_fwd(h, wd, d, token_major=True)
    assert torch.equal(y1[rf[rf >= 0]], y0[:n][rf >= 0])
    d_gu = torch.randn(d.rows_cap, 2 * I, device=DEV).to(torch.bfloat16)
    x0 = ops.gate_up_dgrad(d_gu, wgu, d)
    x1 = ops.gate_up_dgrad(d_gu, wgu, d, token_major=True)
    assert torch.equal(x1[rf[rf >= 0]], x0[:n][rf >= 0])


@pytest.mark.parametrize("T,k,E,H,I", SHAPES + [(3000, 8, 64, 1024, 256)])
def test_pair_tiles_equal_single_cta_tiles(ops, T, k, E, H, I):
    """The two-CTA (cta_group::2) 256-row pair kernel gives exactly the
    single-CTA kernel's results on every expert GEMM, including experts with an
    odd number of 128-row tiles (half-valid last pair) and empty experts."""
    from spark_gpt_b200 import _lib
    d, x, xs, wgu, wd = _setup(ops, T, k, E, H, I, 10)
    n = int(d.pad_offsets[-1])
    rows = d.row_flat.clone()
    rows[n:] = -1
    dy = torch.randn(d.rows_cap, H, device=DEV).to(torch.bfloat16)
    dy[rows < 0] = 0
    d_gu = torch.randn(d.rows_cap, 2 * I, device=DEV).to(torch.bfloat16)
    d_gu[rows < 0] = 0

    def run():
        gu, h = ops.gate_up_fwd(xs, wgu, d)
        y = ops.down_fwd(h, wd, d)
        dg = ops.down_dgrad_swiglu(dy, wd, gu, d)
        dxs = ops.gate_up_dgrad(d_gu, wgu, d)
        w1 = ops.wgrad(d_gu, xs, d)
        w2 = ops.wgrad(dy, h, d)
        torch.cuda.synchronize()
        return [t[:n] for t in (gu, h, y, dg, dxs)] + [w1, w2]

    prev = _lib.load().b200moe_set_pair_gemm(0)
    try:
        single = run()
        _lib.load().b200moe_set_pair_gemm(1)
        pair = run()
    finally:
        _lib.load().b200moe_set_pair_gemm(prev)
    assert _lib.read_fault() == 0
    names = ["gu", "h", "y", "d_gu", "dxs", "dW_gate_up", "dW_down"]
    for name, a, b in zip(names, single, pair):
        assert torch.equal(a, b), name


@pytest.mark.parametrize("E,M,N,chunks", [(16, 1536, 2048, 4), (8, 512, 192, 3), (8, 384, 256, 2),
                                          (32, 512, 1024, 8), (4, 256, 128, 1)])
def test_wgrad_over_row_segments(ops, E, M, N, chunks):
    """One weight gradient over several chunks' padded rows in one allocation
    (the pipelined expert-parallel layer's arena) equals the fp32 product over
    every chunk's rows of each expert: two-CTA tiles with segmented K (and a
    partial last N tile at N = 192), per-segment launches where the pair tiles
    do not apply (M = 384); an empty chunk and an expert without rows in any
    chunk included; accumulation into an existing gradient."""
    from spark_gpt_b200.ep import RowArena
    g = torch.Generator().manual_seed(E + M + N + chunks)
    sels, slots = [], []
    for c in range(chunks):
        T = 0 if (c == 1 and chunks > 2) else int(torch.randint(200, 1500, (1,), generator=g))
        p = torch.ones(E)
        p[0] = 0.0          # expert 0 gets no rows in any chunk
        p[-1] = 6.0
        sel = (torch.stack([torch.multinomial(p, 2, generator=g) for _ in range(T)])
               if T else torch.zeros(0, 2, dtype=torch.int64))
        sels.append(sel)
        slots.append(sel.numel())
    arena = RowArena.for_chunks([s.shape[0] for s in sels], slots, E, DEV)
    arena.alloc("a", M)
    arena.alloc("b", N)
    ds = []
    ref = torch.zeros(E, M, N, device=DEV)
    for c, sel in enumerate(sels):
        if sel.shape[0] == 0:
            ds.append(None)
            continue
        d = ops.dispatch(sel.to(DEV), E, routed_slots=sel.numel())
        a = arena.rows("a", c)
        b = arena.rows("b", c)
        a.copy_(torch.randn(a.shape, generator=g).to(torch.bfloat16))
        b.copy_(torch.randn(b.shape, generator=g).to(torch.bfloat16))
        rows = d.row_flat[: d.rows_cap].clone()
        rows[int(d.pad_offsets[-1]):] = -1
        a[rows < 0] = 0     # padding rows carry zeros in the layer
        b[rows < 0] = 0
        for e, s, t in _segments(d):
            if t > s:
                ref[e] += a[s:t].float().t() @ b[s:t].float()
        ds.append(d)
    segs = arena.segments(ds, E)
    dw = ops.wgrad_segments(arena.bufs["a"], arena.bufs["b"], segs, E)
    torch.testing.assert_close(dw, ref, rtol=1e-3, atol=1e-3 * ref.abs().max().item())
    assert torch.all(dw[0] == 0)
    dw2 = ops.wgrad_segments(arena.bufs["a"], arena.bufs["b"], segs, E, out=dw.clone(),
                             accumulate=True)
    torch.testing.assert_close(dw2, 2 * ref, rtol=1e-3, atol=2e-3 * ref.abs().max().item())
    torch.cuda.synchronize()
    from spark_gpt_b200 import _lib
    assert _lib.read_fault() == 0
