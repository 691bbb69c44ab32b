"""Expert-parallel kernels on one GPU.

1. Slots without an expert (negative ids): dispatch gives them no row and
   inv_pad -1; gather, combine, gather backward and combine backward skip
   them (d_weights 0).  Checked against torch references.
2. The send-plan kernels (ep_route, ep_pack, ep_unpack, ep_weight_grad)
   against a torch restatement of the plan: bit-exact.
3. The whole expert-parallel data path with P ranks emulated on one GPU (the
   all-to-all exchanges become slices of the ranks' send buffers): every
   rank's output and input gradient match the single-GPU layer on its tokens,
   and every expert shard's weight gradients match the single-GPU layer's
   summed over all ranks' tokens, within the layer's bf16 tolerance.
4. The same for the peer-memory transport (send / return kernels storing into
   the other ranks' buffers), and its barrier: passing, and giving up after
   its bounded wait with a fault bit instead of hanging.
"""

import dataclasses
from types import SimpleNamespace

import pytest
import torch

from tests.helpers import assert_bf16_close

pytestmark = pytest.mark.gpu

DEV = "cuda"


@pytest.fixture(scope="module")
def ops():
    from spark_gpt_b200 import ops as _ops
    return _ops


def _partial_routing(T, k, E, seed, keep=0.4):
    """top-k ids with a random subset of slots replaced by -1 (no expert)."""
    g = torch.Generator().manual_seed(seed)
    sel = torch.stack([torch.randperm(E, generator=g)[:k] for _ in range(T)])
    drop = torch.rand(T, k, generator=g) > keep
    drop[: T // 10] = True           # some rows with no slot at all
    drop[T // 10: T // 5] = False    # some rows with every slot
    return torch.where(drop, torch.full_like(sel, -1), sel)


@pytest.mark.parametrize("T,k,E,H", [(3000, 8, 16, 2048), (2500, 4, 8, 1024),
                                     (1700, 8, 8, 256), (900, 3, 5, 384)])
def test_slots_without_expert_are_skipped(ops, T, k, E, H):
    from spark_gpt_b200 import _lib
    sel = _partial_routing(T, k, E, T + k)
    valid = sel >= 0
    S = int(valid.sum())
    d = ops.dispatch(sel.to(DEV), E, routed_slots=S)
    assert d.rows_cap == ops.padded_rows(S, E)
    counts = torch.bincount(sel[valid], minlength=E)
    assert torch.equal(d.counts.cpu().long(), counts)
    inv = d.inv_pad.cpu().long().view(T, k)
    assert torch.all(inv[~valid] == -1) and torch.all(inv[valid] >= 0)
    rf = d.row_flat.cpu().long()
    assert torch.equal(rf[inv[valid]], torch.arange(T * k).view(T, k)[valid])
    # gather (token order) writes each valid slot's row, zero padding rows
    x = torch.randn(T, H).to(torch.bfloat16)
    xs = ops.gather_rows(x.to(DEV), d).cpu()
    t_idx = torch.arange(T).unsqueeze(1).expand(T, k)
    assert torch.equal(xs[inv[valid]], x[t_idx[valid]])
    n = int(d.pad_offsets[-1])
    assert torch.all(xs[:n][rf[:n] < 0] == 0)
    # combine: skipped slots contribute nothing
    y = torch.randn(d.rows_cap, H).to(torch.bfloat16)
    w = torch.rand(T, k).to(torch.bfloat16)
    out = ops.combine(y.to(DEV), d, w.to(DEV)).cpu().float()
    inv0 = inv.clamp_min(0)
    prod = (y.float()[inv0] * w.float().unsqueeze(-1)).to(torch.bfloat16).float()
    ref = (prod * valid.unsqueeze(-1)).sum(1)
    assert (out - ref).abs().max() <= 2 ** -7 * ref.abs().max()
    # gather backward with addend
    add = torch.randn(T, H).to(torch.bfloat16)
    dx = ops.gather_rows_bwd(y.to(DEV), d, addend=add.to(DEV)).cpu().float()
    ref = (y.float()[inv0] * valid.unsqueeze(-1)).sum(1) + add.float()
    assert (dx - ref).abs().max() <= 2 ** -7 * ref.abs().max()
    # combine backward: d_weights of skipped slots are 0
    d_out = torch.randn(T, H).to(torch.bfloat16)
    dy, dw = ops.combine_bwd(d_out.to(DEV), y.to(DEV), d, w.to(DEV))
    dy, dw = dy.cpu().float(), dw.cpu()
    assert torch.all(dw[~valid] == 0)
    ref_dw = (d_out.float().unsqueeze(1) * y.float()[inv0]).sum(-1)
    assert (dw[valid] - ref_dw[valid]).abs().max() <= 1e-4 * ref_dw.abs().max()
    ref_dy = (d_out.float()[t_idx[valid]] * w.float()[valid].unsqueeze(-1)).to(torch.bfloat16)
    assert torch.equal(dy[inv[valid]], ref_dy.float())
    assert torch.all(dy[:n][rf[:n] < 0] == 0)
    assert _lib.read_fault() == 0


def _plan_ref(sel, rw, E_loc, P):
    T, k = sel.shape
    dest = sel // E_loc
    mask = torch.zeros(T, P, dtype=torch.bool)
    mask[torch.arange(T).unsqueeze(1).expand(T, k), dest] = True
    dest_ids = torch.where(mask, torch.arange(P).expand(T, P), torch.full((T, P), -1))
    return dest, mask, dest_ids


@pytest.mark.parametrize("T,k,E,P", [(4096, 8, 128, 8), (3000, 8, 64, 2), (777, 4, 32, 4),
                                     (500, 2, 16, 16)])
def test_send_plan_kernels_bit_exact(ops, T, k, E, P):
    E_loc = E // P
    g = torch.Generator().manual_seed(T)
    sel = torch.stack([torch.randperm(E, generator=g)[:k] for _ in range(T)])
    rw = torch.rand(T, k, generator=g).to(torch.bfloat16)
    dest, mask, dest_ids = _plan_ref(sel, rw, E_loc, P)
    d_dest, d_slots = ops.ep_route(sel.to(DEV), E_loc, P)
    assert torch.equal(d_dest.cpu(), dest_ids)
    assert torch.equal(d_slots.cpu().long(), torch.bincount(dest.view(-1), minlength=P))
    send = ops.dispatch(d_dest, P, partial=True)
    assert torch.equal(send.counts.cpu().long(), mask.sum(0))
    meta = ops.ep_pack(sel.to(DEV), rw.to(DEV), send, E_loc).cpu()
    rf = send.row_flat.cpu().long()
    n = int(send.pad_offsets[-1])
    rows = rf[:n]
    real = rows >= 0
    t, r = rows[real] // P, rows[real] % P
    # rank-major, token order within a rank
    assert torch.equal(r, torch.sort(r, stable=True).values)
    mine = dest[t] == r.unsqueeze(1)
    bits = rw.view(torch.int16).long()[t] & 0xFFFF
    ref_words = torch.where(mine, (bits << 16) | (sel[t] - r.unsqueeze(1) * E_loc),
                            torch.full_like(sel[t], 0xFFFF))
    got = meta[:n][real].long() & 0xFFFFFFFF
    assert torch.equal(got, ref_words)
    assert torch.all(meta[:n][~real].long() & 0xFFFF == 0xFFFF)
    sel_loc, w_loc = ops.ep_unpack(meta[:n].to(DEV))
    sel_loc, w_loc = sel_loc.cpu()[real], w_loc.cpu()[real]
    assert torch.equal(sel_loc, torch.where(mine, sel[t] - r.unsqueeze(1) * E_loc,
                                            torch.full_like(sel[t], -1)))
    assert torch.equal(w_loc.view(torch.int16), torch.where(
        mine, rw[t].view(torch.int16), torch.zeros_like(rw[t].view(torch.int16))))
    # routing-weight gradient gathered back from the send rows
    dw_rows = torch.randn(n, k)
    d_w = ops.ep_weight_grad(dw_rows.to(DEV), send, sel.to(DEV), E_loc).cpu()
    inv = send.inv_pad.cpu().long().view(T, P)
    ref = dw_rows[inv[torch.arange(T).unsqueeze(1), dest], torch.arange(k).unsqueeze(0)]
    assert torch.equal(d_w, ref)


def _emulated_ep(ops, x_list, d_out_list, w_r, w_gu, w_d, k, P):
    """Run ExpertParallelMoE's forward and backward for P ranks on one GPU."""
    from spark_gpt_b200.ep import CudaExpertOps as B
    E = w_gu.shape[0]
    E_loc = E // P
    I, H = w_d.shape[2], w_d.shape[1]
    st = []
    for r in range(P):
        xb = x_list[r]
        logits_buf, wr, sel, rw = B.router(xb, w_r, E, k, True)
        plan, sizes = B.send_plan(sel, rw, E_loc, P)
        st.append(SimpleNamespace(xb=xb, logits_buf=logits_buf, wr=wr, sel=sel, rw=rw, plan=plan,
                                  sizes=sizes.cpu(), x_send=B.pack_rows(xb, plan)))
    starts = [torch.cat([torch.zeros(1, dtype=torch.int64), s.sizes[:, 0].cumsum(0)]) for s in st]

    def to_owner(bufs, o):  # rows every source sends to owner o, in source order
        return torch.cat([bufs[r][starts[r][o]: starts[r][o + 1]] for r in range(P)])

    def to_sources(rows_o_list):  # owner outputs back to each source's send layout
        out = []
        for r in range(P):
            parts = []
            for o in range(P):
                off = sum(int(st[q].sizes[o, 0]) for q in range(r))
                parts.append(rows_o_list[o][off: off + int(st[r].sizes[o, 0])])
            out.append(torch.cat(parts))
        return out

    own = []
    for o in range(P):
        wgu_b = ops.cast_bf16(w_gu[o * E_loc:(o + 1) * E_loc].contiguous())
        wd_b = ops.cast_bf16(w_d[o * E_loc:(o + 1) * E_loc].contiguous())
        x_recv = to_owner([s.x_send for s in st], o)
        meta = to_owner([s.plan.meta for s in st], o)
        sel_loc, w_loc = B.unpack(meta)
        slots = sum(int(s.sizes[o, 1]) for s in st)
        part, ectx = B.experts_fwd(x_recv, sel_loc, w_loc, wgu_b, wd_b, slots)
        own.append(SimpleNamespace(part=part, ectx=ectx))
    back = to_sources([o.part for o in own])
    outs = [B.reduce_rows(back[r], st[r].plan) for r in range(P)]
    d_send = [B.pack_rows(d_out_list[r], st[r].plan) for r in range(P)]
    dxr, dwr, ggu, gd = [], [], [], []
    for o in range(P):
        d_recv = to_owner(d_send, o)
        a, b, state = B.experts_dgrad(own[o].ectx, d_recv, k, d_recv.device)
        c, e = B.experts_wgrad(state, None, None, E_loc, H, I, d_recv.device)
        dxr.append(a)
        dwr.append(b)
        ggu.append(c)
        gd.append(e)
    dx_back = to_sources(dxr)
    dw_back = to_sources(dwr)
    dxs, g_routers = [], []
    for r in range(P):
        s = st[r]
        d_rw = B.weight_grad(dw_back[r], s.plan, s.sel)
        dx_router, g_router = B.router_bwd(s.xb, s.wr, s.logits_buf, s.sel, d_rw, None, E, k, True)
        dxs.append(B.reduce_rows(dx_back[r], s.plan, addend=dx_router))
        g_routers.append(g_router)
    return outs, [s.sel for s in st], dxs, g_routers, torch.cat(ggu), torch.cat(gd)


@pytest.mark.parametrize("T,H,E,k,I,P", [(2048, 1024, 32, 8, 256, 4), (1500, 2048, 16, 4, 128, 2),
                                         (1024, 512, 64, 8, 192, 8)])
def test_emulated_expert_parallel_matches_single_gpu_layer(ops, T, H, E, k, I, P):
    from spark_gpt_b200 import SparseMoE, _lib
    g = torch.Generator().manual_seed(E + P)
    w_r = (torch.randn(E, H, generator=g) * 0.05).to(DEV)
    w_gu = (torch.randn(E, 2 * I, H, generator=g) * 0.02).to(DEV)
    w_d = (torch.randn(E, H, I, generator=g) * 0.02).to(DEV)
    xs = [torch.randn(T, H, generator=g).to(torch.bfloat16).to(DEV) for _ in range(P)]
    ds = [(torch.randn(T, H, generator=g) * 1e-2).to(torch.bfloat16).to(DEV) for _ in range(P)]
    outs, sels, dxs, g_routers, g_gu, g_d = _emulated_ep(ops, xs, ds, w_r, w_gu, w_d, k, P)
    cfg = SimpleNamespace(hidden_size=H, num_experts=E, num_experts_per_tok=k,
                          moe_intermediate_size=I, norm_topk_prob=True)
    ref = SparseMoE(cfg).to(DEV)
    with torch.no_grad():
        ref.gate.weight.copy_(w_r)
        ref.experts.gate_up_proj.copy_(w_gu)
        ref.experts.down_proj.copy_(w_d)
    for r in range(P):
        xin = xs[r].clone().requires_grad_(True)
        ref.gate.weight.grad = None
        out, _, sel = ref(xin)
        out.backward(ds[r])
        assert torch.equal(sels[r], sel)
        assert_bf16_close(outs[r], out, f"out rank {r}")
        assert_bf16_close(dxs[r], xin.grad, f"dx rank {r}")
        assert_bf16_close(g_routers[r], ref.gate.weight.grad, f"dW_router rank {r}")
    # ref's expert grads accumulated over the P ranks' tokens
    assert_bf16_close(g_gu, ref.experts.gate_up_proj.grad, "dW_gate_up")
    assert_bf16_close(g_d, ref.experts.down_proj.grad, "dW_down")
    torch.cuda.synchronize()
    assert _lib.read_fault() == 0


def _emulated_p2p(ops, x_list, d_out_list, w_r, w_gu, w_d, k, P, fused=True):
    """The peer-memory transport with P ranks on one GPU: each rank's receive
    and back buffers are ordinary device tensors and the 'peer' pointer tables
    point at the other ranks' tensors, so the send / return kernels store
    across ranks exactly as over NVLink (no barrier needed: one stream)."""
    from spark_gpt_b200.ep import CudaExpertOps as B
    E = w_gu.shape[0]
    E_loc = E // P
    I, H = w_d.shape[2], w_d.shape[1]
    T = x_list[0].shape[0]
    cap = P * T
    bufs = [SimpleNamespace(recv_rows=torch.zeros(cap, H, device=DEV, dtype=torch.bfloat16),
                            recv_meta=torch.zeros(cap, k, device=DEV, dtype=torch.int32),
                            back_rows=torch.zeros(cap, H, device=DEV, dtype=torch.bfloat16),
                            back_dw=torch.zeros(cap, k, device=DEV, dtype=torch.float32))
            for _ in range(P)]
    table = lambda name: torch.tensor([getattr(b, name).data_ptr() for b in bufs],
                                      dtype=torch.int64, device=DEV)
    peers = {n: table(n) for n in ("recv_rows", "recv_meta", "back_rows", "back_dw")}
    st = []
    for r in range(P):
        logits_buf, wr, sel, rw = B.router(x_list[r], w_r, E, k, True)
        dest, slots = ops.ep_route(sel, E_loc, P)
        send = ops.dispatch(dest, P, partial=True)
        st.append(SimpleNamespace(logits_buf=logits_buf, wr=wr, sel=sel, rw=rw, send=send,
                                  counts=torch.cat([send.counts, slots])))
    gathered = torch.stack([s.counts for s in st])            # (P, 2P)
    host = gathered.cpu()
    for r in range(P):
        st[r].plan = ops.ep_p2p_plan(gathered, r, P)
        ops.ep_p2p_send(x_list[r], st[r].send, st[r].plan, peers["recv_rows"], st[r].sel,
                        st[r].rw, E_loc, peers["recv_meta"])
    own = []
    for o in range(P):
        n_recv, slots_o = int(host[:, o].sum()), int(host[:, P + o].sum())
        wgu_b = ops.cast_bf16(w_gu[o * E_loc:(o + 1) * E_loc].contiguous())
        wd_b = ops.cast_bf16(w_d[o * E_loc:(o + 1) * E_loc].contiguous())
        sel_loc, w_loc = B.unpack(bufs[o].recv_meta[:n_recv])
        if fused:   # the layer's path: combine fused with the return
            y, ectx = B.experts_fwd(bufs[o].recv_rows[:n_recv], sel_loc, w_loc, wgu_b, wd_b,
                                    slots_o, combine=False)
            ops.ep_p2p_reduce_return(y, ectx[0], st[o].plan, peers["back_rows"], P,
                                     weights=w_loc)
        else:       # combine into a local buffer, then the plain return kernel
            part, ectx = B.experts_fwd(bufs[o].recv_rows[:n_recv], sel_loc, w_loc, wgu_b, wd_b,
                                       slots_o)
            ops.ep_p2p_return(part, st[o].plan, peers["back_rows"], P)
        own.append(SimpleNamespace(ectx=ectx, n_recv=n_recv))
    outs = []
    for r in range(P):
        n_back = int(host[r, :P].sum())
        st[r].back = dataclasses.replace(st[r].send, inv_pad=ops.ep_p2p_back_inv(st[r].send,
                                                                                 st[r].plan))
        st[r].n_back = n_back
        outs.append(ops.gather_rows_bwd(bufs[r].back_rows[:n_back], st[r].back))
    for r in range(P):
        ops.ep_p2p_send(d_out_list[r], st[r].send, st[r].plan, peers["recv_rows"])
    ggu, gd = [], []
    for o in range(P):
        d_recv = bufs[o].recv_rows[:own[o].n_recv]
        if fused:
            dxs, dw_rows, state = B.experts_dgrad(own[o].ectx, d_recv, k, d_recv.device,
                                                  reduce=False)
            ops.ep_p2p_reduce_return(dxs, own[o].ectx[0], st[o].plan, peers["back_rows"], P,
                                     dw_rows=dw_rows, peer_dw=peers["back_dw"])
        else:
            dx_rows, dw_rows, state = B.experts_dgrad(own[o].ectx, d_recv, k, d_recv.device)
            ops.ep_p2p_return(dx_rows, st[o].plan, peers["back_rows"], P, dw_rows,
                              peers["back_dw"])
        c, e = B.experts_wgrad(state, None, None, E_loc, H, I, d_recv.device)
        ggu.append(c)
        gd.append(e)
    dxs, g_routers = [], []
    for r in range(P):
        s = st[r]
        d_rw = ops.ep_weight_grad(bufs[r].back_dw[:s.n_back], s.back, s.sel, E_loc)
        dx_router, g_router = B.router_bwd(x_list[r], s.wr, s.logits_buf, s.sel, d_rw, None, E,
                                           k, True)
        dxs.append(ops.gather_rows_bwd(bufs[r].back_rows[:s.n_back], s.back, addend=dx_router))
        g_routers.append(g_router)
    return outs, [s.sel for s in st], dxs, g_routers, torch.cat(ggu), torch.cat(gd)


@pytest.mark.parametrize("T,H,E,k,I,P,fused", [(2048, 1024, 32, 8, 256, 4, True),
                                               (1500, 2048, 16, 4, 128, 2, True),
                                               (1024, 512, 64, 8, 192, 8, True),
                                               (1024, 1024, 32, 8, 128, 4, False)])
def test_emulated_peer_memory_transport_matches_single_gpu_layer(ops, T, H, E, k, I, P, fused):
    from spark_gpt_b200 import SparseMoE, _lib
    g = torch.Generator().manual_seed(E * 3 + P)
    w_r = (torch.randn(E, H, generator=g) * 0.05).to(DEV)
    w_gu = (torch.randn(E, 2 * I, H, generator=g) * 0.02).to(DEV)
    w_d = (torch.randn(E, H, I, generator=g) * 0.02).to(DEV)
    xs = [torch.randn(T, H, generator=g).to(torch.bfloat16).to(DEV) for _ in range(P)]
    ds = [(torch.randn(T, H, generator=g) * 1e-2).to(torch.bfloat16).to(DEV) for _ in range(P)]
    outs, sels, dxs, g_routers, g_gu, g_d = _emulated_p2p(ops, xs, ds, w_r, w_gu, w_d, k, P,
                                                          fused)
    cfg = SimpleNamespace(hidden_size=H, num_experts=E, num_experts_per_tok=k,
                          moe_intermediate_size=I, norm_topk_prob=True)
    ref = SparseMoE(cfg).to(DEV)
    with torch.no_grad():
        ref.gate.weight.copy_(w_r)
        ref.experts.gate_up_proj.copy_(w_gu)
        ref.experts.down_proj.copy_(w_d)
    for r in range(P):
        xin = xs[r].clone().requires_grad_(True)
        ref.gate.weight.grad = None
        out, _, sel = ref(xin)
        out.backward(ds[r])
        assert torch.equal(sels[r], sel)
        assert_bf16_close(outs[r], out, f"p2p out rank {r}")
        assert_bf16_close(dxs[r], xin.grad, f"p2p dx rank {r}")
        assert_bf16_close(g_routers[r], ref.gate.weight.grad, f"p2p dW_router rank {r}")
    assert_bf16_close(g_gu, ref.experts.gate_up_proj.grad, "p2p dW_gate_up")
    assert_bf16_close(g_d, ref.experts.down_proj.grad, "p2p dW_down")
    torch.cuda.synchronize()
    assert _lib.read_fault() == 0


def _emulated_pipe(ops, x_list, d_out_list, w_r, w_gu, w_d, k, P):
    """The per-source pipelined peer-memory exchange (_EPMoEPipeFn's kernels)
    with P ranks on one GPU, run phase by phase in one stream: every rank's
    sends and send flags first, then each owner's source chunks (own rows
    first, then me-1, me-2, ...), each returned with its own flag, then each
    source's wait for all owners' flags and its sum over them; the same for
    the backward.  The point-to-point flags live in per-rank device tensors
    reached through a peer table, as over NVLink."""
    from spark_gpt_b200.ep import (CudaExpertOps as B, FLAG_WORDS, PH_BWD_RETURN,
                                   PH_BWD_SEND, PH_FWD_RETURN, PH_FWD_SEND, RowArena)
    E = w_gu.shape[0]
    E_loc = E // P
    I, H = w_d.shape[2], w_d.shape[1]
    T = x_list[0].shape[0]
    cap = P * T
    bufs = [SimpleNamespace(recv_rows=torch.zeros(cap, H, device=DEV, dtype=torch.bfloat16),
                            recv_meta=torch.zeros(cap, k, device=DEV, dtype=torch.int32),
                            back_rows=torch.zeros(cap, H, device=DEV, dtype=torch.bfloat16),
                            back_dw=torch.zeros(cap, k, device=DEV, dtype=torch.float32),
                            flags=torch.zeros(FLAG_WORDS, device=DEV, dtype=torch.int64))
            for _ in range(P)]
    table = lambda name: torch.tensor([getattr(b, name).data_ptr() for b in bufs],
                                      dtype=torch.int64, device=DEV)
    peers = {n: table(n) for n in ("recv_rows", "recv_meta", "back_rows", "back_dw", "flags")}
    step = 1
    st = []
    for r in range(P):
        logits_buf, wr, sel, rw = B.router(x_list[r], w_r, E, k, True)
        dest, slots = ops.ep_route(sel, E_loc, P)
        send = ops.dispatch(dest, P, partial=True)
        st.append(SimpleNamespace(logits_buf=logits_buf, wr=wr, sel=sel, rw=rw, send=send,
                                  counts=torch.cat([send.counts, slots])))
    gathered = torch.stack([s.counts for s in st])            # (P, 2P)
    host = gathered.cpu()
    for r in range(P):
        st[r].plan = ops.ep_p2p_plan(gathered, r, P)
        for mode in (1, 2):
            ops.ep_p2p_send_part(x_list[r], st[r].send, st[r].plan, peers["recv_rows"], r, mode,
                                 st[r].sel, st[r].rw, E_loc, peers["recv_meta"])
        ops.ep_signal(peers["flags"], PH_FWD_SEND, r, P, step)
    own = []
    for o in range(P):
        rows_from = [int(v) for v in host[:, o]]
        slots_from = [int(v) for v in host[:, P + o]]
        base = [sum(rows_from[:s]) for s in range(P)]
        wgu_b = ops.cast_bf16(w_gu[o * E_loc:(o + 1) * E_loc].contiguous())
        wd_b = ops.cast_bf16(w_d[o * E_loc:(o + 1) * E_loc].contiguous())
        ectxs = [None] * P
        arena = RowArena.for_chunks(rows_from, slots_from, E_loc, DEV)
        arena.alloc("xs", H)
        arena.alloc("h", I)
        for s in [(o - j) % P for j in range(P)]:
            if s != o:
                ops.ep_wait(bufs[o].flags, PH_FWD_SEND, P, step, src=s)
            n = rows_from[s]
            sel_loc, w_loc = B.unpack(bufs[o].recv_meta[base[s]:base[s] + n])
            y, ectxs[s] = B.experts_fwd(bufs[o].recv_rows[base[s]:base[s] + n], sel_loc, w_loc,
                                        wgu_b, wd_b, slots_from[s], combine=False,
                                        arena=arena, src=s)
            if ectxs[s] is not None:
                ops.ep_p2p_reduce_return_src(y, ectxs[s][0], st[o].plan, peers["back_rows"], P,
                                             s, weights=w_loc)
            ops.ep_signal(peers["flags"], PH_FWD_RETURN, o, P, step, dest=s)
        own.append(SimpleNamespace(ectxs=ectxs, rows_from=rows_from, base=base, arena=arena))
    outs = []
    for r in range(P):
        ops.ep_wait(bufs[r].flags, PH_FWD_RETURN, P, step)
        n_back = int(host[r, :P].sum())
        st[r].back = dataclasses.replace(st[r].send, inv_pad=ops.ep_p2p_back_inv(st[r].send,
                                                                                 st[r].plan))
        st[r].n_back = n_back
        outs.append(ops.gather_rows_bwd(bufs[r].back_rows[:n_back], st[r].back))
    for r in range(P):
        for mode in (1, 2):
            ops.ep_p2p_send_part(d_out_list[r], st[r].send, st[r].plan, peers["recv_rows"], r,
                                 mode)
        ops.ep_signal(peers["flags"], PH_BWD_SEND, r, P, step)
    ggu, gd = [], []
    for o in range(P):
        arena = own[o].arena
        arena.alloc("dy", H)
        arena.alloc("d_gu", 2 * I)
        states = [None] * P
        for s in [(o - j) % P for j in range(P)]:
            if s != o:
                ops.ep_wait(bufs[o].flags, PH_BWD_SEND, P, step, src=s)
            e = own[o].ectxs[s]
            d_rows = bufs[o].recv_rows[own[o].base[s]:own[o].base[s] + own[o].rows_from[s]]
            dxs, dw_rows, states[s] = B.experts_dgrad(e, d_rows, k, DEV, reduce=False,
                                                      arena=arena, src=s)
            if e is not None:
                ops.ep_p2p_reduce_return_src(dxs, e[0], st[o].plan, peers["back_rows"], P, s,
                                             dw_rows=dw_rows, peer_dw=peers["back_dw"])
            ops.ep_signal(peers["flags"], PH_BWD_RETURN, o, P, step, dest=s)
        g_gu, g_d = B.experts_wgrad_segments(states, arena, E_loc, H, I, DEV)
        ggu.append(g_gu)
        gd.append(g_d)
    dxs, g_routers = [], []
    for r in range(P):
        ops.ep_wait(bufs[r].flags, PH_BWD_RETURN, P, step)
        s = st[r]
        d_rw = ops.ep_weight_grad(bufs[r].back_dw[:s.n_back], s.back, s.sel, E_loc)
        dx_router, g_router = B.router_bwd(x_list[r], s.wr, s.logits_buf, s.sel, d_rw, None, E,
                                           k, True)
        dxs.append(ops.gather_rows_bwd(bufs[r].back_rows[:s.n_back], s.back, addend=dx_router))
        g_routers.append(g_router)
    return outs, [s.sel for s in st], dxs, g_routers, torch.cat(ggu), torch.cat(gd)


@pytest.mark.parametrize("T,H,E,k,I,P", [(2048, 1024, 32, 8, 256, 4),
                                         (1500, 2048, 16, 4, 128, 2),
                                         (1024, 512, 64, 8, 192, 8)])
def test_emulated_pipelined_exchange_matches_single_gpu_layer(ops, T, H, E, k, I, P):
    """Per-source chunks, the one-source return kernel and the point-to-point
    flags give the single-GPU layer's routing and, within the bf16 contract,
    its outputs and gradients (one extra rounding of an owner's partial sum)."""
    from spark_gpt_b200 import SparseMoE, _lib
    g = torch.Generator().manual_seed(E * 7 + P)
    w_r = (torch.randn(E, H, generator=g) * 0.05).to(DEV)
    w_gu = (torch.randn(E, 2 * I, H, generator=g) * 0.02).to(DEV)
    w_d = (torch.randn(E, H, I, generator=g) * 0.02).to(DEV)
    xs = [torch.randn(T, H, generator=g).to(torch.bfloat16).to(DEV) for _ in range(P)]
    ds = [(torch.randn(T, H, generator=g) * 1e-2).to(torch.bfloat16).to(DEV) for _ in range(P)]
    outs, sels, dxs, g_routers, g_gu, g_d = _emulated_pipe(ops, xs, ds, w_r, w_gu, w_d, k, P)
    cfg = SimpleNamespace(hidden_size=H, num_experts=E, num_experts_per_tok=k,
                          moe_intermediate_size=I, norm_topk_prob=True)
    ref = SparseMoE(cfg).to(DEV)
    with torch.no_grad():
        ref.gate.weight.copy_(w_r)
        ref.experts.gate_up_proj.copy_(w_gu)
        ref.experts.down_proj.copy_(w_d)
    for r in range(P):
        xin = xs[r].clone().requires_grad_(True)
        ref.gate.weight.grad = None
        out, _, sel = ref(xin)
        out.backward(ds[r])
        assert torch.equal(sels[r], sel)
        assert_bf16_close(outs[r], out, f"pipe out rank {r}")
        assert_bf16_close(dxs[r], xin.grad, f"pipe dx rank {r}")
        assert_bf16_close(g_routers[r], ref.gate.weight.grad, f"pipe dW_router rank {r}")
    assert_bf16_close(g_gu, ref.experts.gate_up_proj.grad, "pipe dW_gate_up")
    assert_bf16_close(g_d, ref.experts.down_proj.grad, "pipe dW_down")
    torch.cuda.synchronize()
    assert _lib.read_fault() == 0


def test_point_to_point_flags_pass_and_time_out_without_a_fault(ops):
    """A signalled flag passes at once; a wait on a flag nothing sets gives up
    after its limit with fault bit 1, and the context stays usable."""
    from spark_gpt_b200 import _lib
    from spark_gpt_b200.ep import FLAG_WORDS, PH_FWD_SEND
    flags = [torch.zeros(FLAG_WORDS, device=DEV, dtype=torch.int64) for _ in range(2)]
    table = torch.tensor([f.data_ptr() for f in flags], dtype=torch.int64, device=DEV)
    ops.ep_signal(table, PH_FWD_SEND, 0, 2, 3, dest=1)       # rank 0 -> rank 1
    ops.ep_wait(flags[1], PH_FWD_SEND, 2, 3, src=0)
    torch.cuda.synchronize()
    assert _lib.read_fault() == 0
    assert int(flags[1][PH_FWD_SEND * 64 + 0]) == 3 and int(flags[0].abs().sum()) == 0
    ops.ep_wait(flags[1], PH_FWD_SEND, 2, 3, src=1)          # rank 1 never signalled
    torch.cuda.synchronize()
    assert _lib.read_fault() == 1
    assert torch.equal(torch.ones(4, device=DEV).cumsum(0).cpu(), torch.arange(1, 5).float())


def test_peer_barrier_passes_and_times_out_without_a_fault(ops):
    """One rank: the barrier passes at once.  Two ranks emulated on one GPU
    with only rank 0 arriving (a flag nothing sets): the bounded wait gives up
    after its limit, records fault bit 1 and returns; the context stays usable."""
    from spark_gpt_b200 import _lib
    flags = [torch.zeros(32, device=DEV, dtype=torch.int64) for _ in range(2)]
    table = torch.tensor([f.data_ptr() for f in flags], dtype=torch.int64, device=DEV)
    ops.ep_barrier(table[:1], flags[0], 0, 1, 1)
    torch.cuda.synchronize()
    assert _lib.read_fault() == 0 and int(flags[0][0]) == 1
    ops.ep_barrier(table, flags[0], 0, 2, 2)   # rank 1 never arrives
    torch.cuda.synchronize()
    assert _lib.read_fault() == 1
    assert int(flags[1][0]) == 2               # rank 0 still signalled its peer
    assert torch.equal(torch.ones(4, device=DEV).cumsum(0).cpu(), torch.arange(1, 5).float())
