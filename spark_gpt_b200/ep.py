"""Expert-parallel MoE layer: experts sharded over a process group.

With P ranks, rank r owns experts [r*E/P, (r+1)*E/P) and keeps its own T
tokens.  Per forward:

  1. router on the local tokens (replicated router weight), top-k;
  2. send plan: each token goes ONCE to every rank that owns at least one of
     its k experts (one row per (token, destination rank), not one per slot),
     with k packed slot words (local expert id + bf16 routing weight, or "no
     expert here") beside the row; rank-major, token order within a rank;
  3. the rows and slot words cross the NVLink/NVSwitch fabric (one host read
     of the per-rank counts sizes every buffer);
  4. the owner runs its local experts on the received rows as a k-slot layer
     whose foreign slots are skipped (dispatch, gate_up GEMM + SwiGLU, down
     GEMM) and combines each row's local slots with their routing weights
     into one partial output row (fp32 sum, rounded to bf16);
  5. the partial rows travel back and the source sums each token's partial
     rows over the ranks it went to (fp32 sum, rounded once).

The backward mirrors it: d_out rows go to the owners along the same plan; the
owner computes the combine backward (slot gradients and routing-weight
gradients), its experts' dgrads, and sums each row's slot input-gradients
into one row; rows and routing-weight gradients travel back (while the owner
computes its expert weight gradients, which stay local) and the source adds
them to the router's input gradient.  The load-balancing counts are
all-reduced by global_load_balancing_loss as in the data-parallel layout
(train.py:3162).

Two transports carry steps 3 and 5:
  * "nccl": all_to_all_single of packed send buffers (_EPMoEFn); the tokens
    may be split into chunks so one chunk's exchange runs while another's
    experts compute, the persistent kernels leaving SMs to the collective;
  * "p2p": this library's kernels store the rows straight into buffers every
    rank has mapped (torch symmetric memory over NVLink/NVSwitch), the gather
    of the send plan and the owner's combine fused with the transfers, and
    bounded barriers over flag words separate the phases (_EPMoEP2PFn).

Each (token, rank) row crosses the fabric once per pass instead of once per
slot: with top-8 of 128 experts a token reaches about 5.3 of 8 ranks (2 of
2), so each of the four exchanges moves a third (three quarters) less than a
per-slot exchange.  Results agree with the single-GPU layer within bf16
rounding: the owner's partial sums are rounded to bf16 before the source adds
them (one extra rounding when a token's experts span ranks); both transports
give the same bits.

The reference trains data-parallel only (experts replicated, DDP); this module
is the expert-parallel layout of the same layer.  Expert parameters here are
this rank's shard: gate_up_proj (E/P, 2I, H), down_proj (E/P, H, I).
"""

from __future__ import annotations

import dataclasses
from contextlib import nullcontext
from types import SimpleNamespace

import torch
import torch.distributed as dist
import torch.nn as nn

from . import faults, ops
from .moe import TopKRouter, _as_bf16, _extra_logit_grad, _require_cuda

MAX_RANKS = 16  # the source-side sum over ranks reduces at most 16 rows per token
# flag words of a peer-memory transport: the group barrier's (phase 0) and the
# pipelined exchange's point-to-point completion flags, 64 words per phase
# (include/b200moe.h, b200moe_ep_signal)
FLAG_WORDS = 5 * 64
PH_FWD_SEND, PH_FWD_RETURN, PH_BWD_SEND, PH_BWD_RETURN = 1, 2, 3, 4
P2P_HIDDEN_SIZES = (256, 512, 1024, 2048)  # b200moe_ep_p2p_reduce_return


class CudaExpertOps:
    """The device kernels the expert-parallel path runs (libb200moe.so)."""

    @staticmethod
    def router(x, w_router, num_experts, top_k, norm):
        W = ops.router_width(num_experts)
        wr = ops.cast_bf16(w_router, W)
        logits_buf = ops.router_logits(x, wr)
        sel, rw = ops.router_topk(logits_buf, num_experts, top_k, norm)
        return logits_buf, wr, sel, rw

    @staticmethod
    def router_bwd(x, wr, logits_buf, sel, d_rw, d_logits, num_experts, top_k, norm):
        T, W = logits_buf.shape
        extra = _extra_logit_grad(d_logits, T, W)
        dl = ops.router_topk_bwd(logits_buf, sel, d_rw, extra, num_experts, top_k, norm)
        return ops.router_dgrad(dl, wr), ops.router_wgrad(x, dl, num_experts)

    @staticmethod
    def send_plan(sel, rw, experts_per_rank, ranks):
        """Send layout + slot words; sizes (P, 2) int64 = [rows, slots] per rank."""
        dest, slots = ops.ep_route(sel, experts_per_rank, ranks)
        send = ops.dispatch(dest, ranks, partial=True)
        meta = ops.ep_pack(sel, rw, send, experts_per_rank)
        rows = send.pad_offsets[1:] - send.pad_offsets[:-1]
        sizes = torch.stack([rows.to(torch.int64), slots.to(torch.int64)], 1)
        return SimpleNamespace(send=send, meta=meta, experts_per_rank=experts_per_rank), sizes

    @staticmethod
    def pack_rows(src, plan):
        return ops.gather_rows(_as_bf16(src), plan.send)

    @staticmethod
    def unpack(meta):
        return ops.ep_unpack(meta)

    @staticmethod
    def experts_fwd(rows, sel_loc, w_loc, w_gu, w_d, slots, combine=True, arena=None, src=0):
        """partial[i] = sum over row i's local slots of bf16(expert(rows[i]) * w);
        combine=False returns the expert outputs y (padded rows) instead.
        arena: a RowArena whose chunk `src` receives the gathered rows xs and h."""
        E = w_gu.shape[0]
        if rows.shape[0] == 0 or slots == 0:
            return rows.new_zeros(rows.shape), None
        d = ops.dispatch(sel_loc, E, routed_slots=slots)
        xs = ops.gather_rows(rows, d, out=arena.rows("xs", src) if arena else None)
        gu, h = ops.gate_up_fwd(xs, w_gu, d, out_h=arena.rows("h", src) if arena else None)
        y = ops.down_fwd(h, w_d, d)
        ctx = (d, w_loc, xs, gu, h, y, w_gu, w_d)
        return (ops.combine(y, d, w_loc) if combine else y), ctx

    @staticmethod
    def experts_dgrad(ctx, d_rows, k, device, reduce=True, arena=None, src=0):
        """-> (dx rows, d_weights (rows, k) fp32, state for experts_wgrad);
        reduce=False returns the slot input-gradients dxs (padded rows) instead
        of their per-row sums.  arena: a RowArena whose chunk `src` receives
        the rows' gradient dy and d_gu."""
        n, H = d_rows.shape
        if ctx is None:
            return d_rows.new_zeros(n, H), torch.zeros(n, k, device=device), None
        d, w_loc, xs, gu, h, y, w_gu, w_d = ctx
        dy, dw = ops.combine_bwd(_as_bf16(d_rows), y, d, w_loc,
                                 out=arena.rows("dy", src) if arena else None)
        d_gu = ops.down_dgrad_swiglu(dy, w_d, gu, d,
                                     out=arena.rows("d_gu", src) if arena else None)
        dxs = ops.gate_up_dgrad(d_gu, w_gu, d)
        return (ops.gather_rows_bwd(dxs, d) if reduce else dxs), dw, (d, dy, h, d_gu, xs)

    @staticmethod
    def experts_wgrad(state, g_gu, g_d, E, H, I, device):
        """Adds this chunk's expert weight gradients to (g_gu, g_d) (None: start)."""
        if state is None:
            if g_gu is None:
                g_gu = torch.zeros(E, 2 * I, H, device=device)
                g_d = torch.zeros(E, H, I, device=device)
            return g_gu, g_d
        d, dy, h, d_gu, xs = state
        acc = g_gu is not None
        g_d = ops.wgrad(dy, h, d, name="down_wgrad", out=g_d, accumulate=acc)
        g_gu = ops.wgrad(d_gu, xs, d, name="gate_up_wgrad", out=g_gu, accumulate=acc)
        return g_gu, g_d

    @staticmethod
    def experts_wgrad_segments(states, arena, E, H, I, device):
        """Both expert weight gradients over every chunk of `arena` at once
        (one launch each, no accumulation pass per chunk); states[s] is chunk
        s's experts_dgrad state or None."""
        ds = [None if st is None else st[0] for st in states]
        if all(d is None for d in ds):
            return (torch.zeros(E, 2 * I, H, device=device),
                    torch.zeros(E, H, I, device=device))
        segs = arena.segments(ds, E)
        g_d = ops.wgrad_segments(arena.bufs["dy"], arena.bufs["h"], segs, E, name="down_wgrad")
        g_gu = ops.wgrad_segments(arena.bufs["d_gu"], arena.bufs["xs"], segs, E,
                                  name="gate_up_wgrad")
        return g_gu, g_d

    @staticmethod
    def reduce_rows(rows_back, plan, addend=None, out=None):
        """out[t] = sum over the ranks token t went to of its returned row (+ addend)."""
        return ops.gather_rows_bwd(rows_back, plan.send, addend=addend, out=out)

    @staticmethod
    def weight_grad(dw_back, plan, sel, out=None):
        return ops.ep_weight_grad(dw_back, plan.send, sel, plan.experts_per_rank, out=out)

    @staticmethod
    def cast(w):
        return ops.cast_bf16(w)

    @staticmethod
    def raise_pending(device):
        """Raise the fault a kernel of an earlier call recorded (faults.py)."""
        faults.raise_pending(device)

    @staticmethod
    def snapshot(device):
        """Queue the copy of the device fault word that the next call checks."""
        faults.snapshot(device)

    @staticmethod
    def overlap(comm_sms):
        """Persistent kernels leave `comm_sms` SMs to the all-to-all beside them."""
        return ops.persistent_sm_limit(max(2, torch.cuda.get_device_properties(
            torch.cuda.current_device()).multi_processor_count - comm_sms))


class RowArena:
    """Row buffers shared by the per-source chunks of the pipelined layer: one
    allocation per activation the expert weight gradients read (xs and h in
    the forward, dy and d_gu in the backward), chunk s owning rows
    [base[s], base[s] + caps[s]) of each in source order, so that one
    weight-gradient launch per weight covers every chunk
    (b200moe_expert_wgrad_segments)."""

    def __init__(self, caps, device):
        self.caps = [int(c) for c in caps]
        self.base = [sum(self.caps[:s]) for s in range(len(self.caps))]
        self.total = max(sum(self.caps), 128)
        self.device = device
        self.bufs = {}

    @classmethod
    def for_chunks(cls, rows_from, slots_from, num_experts, device):
        """Capacities of the chunks' dispatches (routed_slots = the chunk's
        slots): none for a chunk without rows or slots (no experts run)."""
        return cls([ops.padded_rows(sl, num_experts) if (n and sl) else 0
                    for n, sl in zip(rows_from, slots_from)], device)

    def alloc(self, name, cols):
        self.bufs[name] = torch.empty(self.total, cols, device=self.device,
                                      dtype=torch.bfloat16)

    def rows(self, name, s):
        return self.bufs[name][self.base[s]:self.base[s] + self.caps[s]]

    def segments(self, dispatches, num_experts):
        """(chunks, E+1) int32 absolute row offsets: each chunk's padded
        expert offsets moved to its base (a chunk without experts: empty)."""
        i32 = dict(device=self.device, dtype=torch.int32)
        return torch.stack([torch.full((num_experts + 1,), self.base[s], **i32) if d is None
                            else d.pad_offsets + self.base[s] for s, d in enumerate(dispatches)])


def _backend_call(backend, name, device):
    """A backend's fault hook (raise_pending / snapshot), if it has one."""
    fn = getattr(backend, name, None)
    if fn is not None:
        fn(device)


def _layer_signature(num_experts, top_k, H, I, chunks):
    """What every rank of the group must agree on: a rank configured
    differently would route rows to experts that another rank does not hold."""
    return [num_experts, top_k, H, I, chunks]


def _check_signatures(received, mine):
    """received: one signature per rank (host ints); raise on every rank alike."""
    bad = [r for r, sig in enumerate(received) if list(sig) != list(mine)]
    if bad:
        raise ValueError(f"expert-parallel ranks disagree on the layer configuration "
                         f"(experts, top_k, hidden, intermediate, chunks): this rank has {mine}, "
                         f"rank(s) {bad} have {[list(received[r]) for r in bad]}")


def _start(buf, send_counts, recv_counts, group):
    """Asynchronous all_to_all_single of row blocks -> (receive buffer, work)."""
    out = buf.new_empty((sum(recv_counts), *buf.shape[1:]))
    work = dist.all_to_all_single(out, buf[: sum(send_counts)].contiguous(), recv_counts,
                                  send_counts, group=group, async_op=True)
    return out, work


class _EPMoEFn(torch.autograd.Function):
    """Forward and backward of the expert-parallel layer.

    The tokens are split into `chunks` contiguous ranges, each with its own send
    plan.  Chunk c+1's rows cross the fabric while chunk c's experts compute,
    and chunk c's results travel back while chunk c+1 computes; in the backward,
    each chunk's input-gradient rows travel back while the next chunk's dgrads
    and then all chunks' weight gradients compute.  With comm_sms > 0 the
    persistent kernels of those windows leave that many SMs to the collective.
    Collectives are issued in the same order on every rank."""

    @staticmethod
    def forward(ctx, x, w_router, w_gu, w_d, top_k, norm, num_experts, group, backend, chunks,
                comm_sms):
        _backend_call(backend, "raise_pending", x.device)
        P = dist.get_world_size(group)
        E_loc = w_gu.shape[0]
        T, H = x.shape
        xb = _as_bf16(x) if x.is_cuda else x
        logits_buf, wr, sel, rw = backend.router(xb, w_router, num_experts, top_k, norm)
        C = max(1, min(int(chunks), T))
        bounds = [T * c // C for c in range(C + 1)]
        span = [(bounds[c], bounds[c + 1]) for c in range(C)]
        plans, sizes = [], []
        for a, b in span:
            plan, sz = backend.send_plan(sel[a:b], rw[a:b], E_loc, P)
            plans.append(plan)
            sizes.append(sz)
        x_sends = [backend.pack_rows(xb[a:b], plans[c]) for c, (a, b) in enumerate(span)]
        sizes_t = torch.stack(sizes).transpose(0, 1)                  # (P, C, 2)
        sig = _layer_signature(num_experts, top_k, H, w_gu.shape[1] // 2, C)
        sig_t = torch.tensor(sig, dtype=sizes_t.dtype, device=sizes_t.device)
        sizes_t = torch.cat([sizes_t, sig_t.expand(P, C, len(sig))], 2).contiguous()
        recv_t = torch.empty_like(sizes_t)
        dist.all_to_all_single(recv_t, sizes_t, group=group)
        host = torch.stack([sizes_t, recv_t]).cpu()  # the one host read of the step
        _check_signatures(host[1, :, 0, 2:].tolist(), sig)
        send_rows = [host[0, :, c, 0].tolist() for c in range(C)]
        recv_rows = [host[1, :, c, 0].tolist() for c in range(C)]
        recv_slots = [int(host[1, :, c, 1].sum()) for c in range(C)]
        wgu_b, wd_b = backend.cast(w_gu), backend.cast(w_d)

        def start_rows(c):
            return (_start(x_sends[c], send_rows[c], recv_rows[c], group),
                    _start(plans[c].meta, send_rows[c], recv_rows[c], group))

        ectxs, backs = [None] * C, [None] * C
        overlap = backend.overlap(comm_sms) if (C > 1 and comm_sms) else nullcontext()
        with overlap:
            pend = start_rows(0)
            for c in range(C):
                (x_recv, wx), (meta_recv, wm) = pend
                if c + 1 < C:
                    pend = start_rows(c + 1)
                wx.wait()
                wm.wait()
                sel_loc, w_loc = backend.unpack(meta_recv)
                part, ectxs[c] = backend.experts_fwd(x_recv, sel_loc, w_loc, wgu_b, wd_b,
                                                     recv_slots[c])
                backs[c] = _start(part, recv_rows[c], send_rows[c], group)
        out = xb.new_empty(T, H)
        for c, (a, b) in enumerate(span):
            rows, w = backs[c]
            w.wait()
            backend.reduce_rows(rows, plans[c], out=out[a:b])
        _backend_call(backend, "snapshot", x.device)
        ctx.save_for_backward(xb, logits_buf, wr, sel)
        ctx.meta = (plans, ectxs, span, send_rows, recv_rows, group, backend, top_k, norm,
                    num_experts, E_loc, H, w_gu.shape[1] // 2, x.dtype, comm_sms)
        ctx.mark_non_differentiable(sel)
        E = num_experts
        logits = logits_buf if logits_buf.shape[1] == E else logits_buf[:, :E]
        return out.to(x.dtype), logits, sel

    @staticmethod
    def backward(ctx, d_out, d_logits, _d_sel):
        xb, logits_buf, wr, sel = ctx.saved_tensors
        (plans, ectxs, span, send_rows, recv_rows, group, backend, top_k, norm, num_experts,
         E_loc, H, I, xdtype, comm_sms) = ctx.meta
        _backend_call(backend, "raise_pending", xb.device)
        C = len(span)
        T = xb.shape[0]
        if d_out is None:
            d_out = torch.zeros(xb.shape, device=xb.device, dtype=xb.dtype)
        d_sends = [backend.pack_rows(d_out[a:b], plans[c]) for c, (a, b) in enumerate(span)]
        rets, states = [None] * C, [None] * C
        g_gu = g_d = None
        overlap = backend.overlap(comm_sms) if comm_sms else nullcontext()
        with overlap:
            pend = _start(d_sends[0], send_rows[0], recv_rows[0], group)
            for c in range(C):
                d_recv, wd = pend
                if c + 1 < C:
                    pend = _start(d_sends[c + 1], send_rows[c + 1], recv_rows[c + 1], group)
                wd.wait()
                dx_rows, dw_rows, states[c] = backend.experts_dgrad(ectxs[c], d_recv, top_k,
                                                                    xb.device)
                rets[c] = (_start(dx_rows, recv_rows[c], send_rows[c], group),
                           _start(dw_rows, recv_rows[c], send_rows[c], group))
            # the weight gradients run while the last input-gradient rows travel back
            for c in range(C):
                g_gu, g_d = backend.experts_wgrad(states[c], g_gu, g_d, E_loc, H, I, xb.device)
        d_rw = torch.empty(T, top_k, device=xb.device, dtype=torch.float32)
        for c, (a, b) in enumerate(span):
            (_, w1), (dw_back, w2) = rets[c]
            w1.wait()
            w2.wait()
            backend.weight_grad(dw_back, plans[c], sel[a:b], out=d_rw[a:b])
        dx_router, g_router = backend.router_bwd(xb, wr, logits_buf, sel, d_rw, d_logits,
                                                 num_experts, top_k, norm)
        dx = xb.new_empty(T, H)
        for c, (a, b) in enumerate(span):
            backend.reduce_rows(rets[c][0][0], plans[c], addend=dx_router[a:b], out=dx[a:b])
        _backend_call(backend, "snapshot", xb.device)
        return (dx.to(xdtype), g_router, g_gu, g_d, None, None, None, None, None, None, None)


class PeerTransport:
    """Peer-memory buffers of one process group for rows of width H with k slot
    words, mapped by every rank (torch symmetric memory over NVLink/NVSwitch):
    recv rows/meta (rows sent to this rank's experts), back rows/dw (results
    returned to this rank) and the barrier flags.  Capacity T_cap tokens per
    rank; grown collectively (every rank sees the same gathered token counts).
    One transport serves every layer of the same (group, H, k): the phases of
    a step are separated by barriers and each phase's data is consumed before
    the next phase writes."""

    _cache: dict = {}

    @classmethod
    def get(cls, group, H, k, device, slot=0):
        """The transport of (group, H, k) on `device`; `slot` tells apart the
        transports of a step's token chunks."""
        # Keyed by the group's name, and checked against the group object
        # itself: torch restarts its group-name counter when the process group
        # is destroyed, so a group created after destroy_process_group and a
        # new init can carry the name of a destroyed one.  A transport bound to
        # another group object is dropped (with its peer mappings) and rebuilt.
        pg = group if group is not None else dist.group.WORLD
        key = (pg.group_name, H, k, str(device), slot)
        cached = cls._cache.get(key)
        if cached is not None and cached.pg is not pg:
            cached.release()
            cached = None
        if cached is None:
            cached = cls._cache[key] = cls(group, H, k, device)
        return cached

    def __init__(self, group, H, k, device):
        self.group, self.H, self.k, self.device = group, H, k, torch.device(device)
        self.pg = group if group is not None else dist.group.WORLD
        self.P = dist.get_world_size(group)
        self.me = dist.get_rank(group)
        self.cap = 0
        self.epoch = 0
        self.step = 0
        self._buf = None

    def ensure(self, tokens: int):
        if tokens <= self.cap:
            return
        import torch.distributed._symmetric_memory as symm_mem
        cap = max(1024, -(-tokens // 1024) * 1024)
        rows = self.P * cap
        H, k = self.H, self.k
        sizes = [("recv_rows", rows * H * 2), ("recv_meta", rows * k * 4),
                 ("back_rows", rows * H * 2), ("back_dw", rows * k * 4),
                 ("flags", 8 * FLAG_WORDS)]
        offs, total = {}, 0
        for name, nbytes in sizes:
            offs[name] = total
            total += -(-nbytes // 256) * 256
        if self._buf is not None:
            torch.cuda.synchronize(self.device)  # nothing in flight uses the old buffers
        self._buf = None
        buf = symm_mem.empty(total, dtype=torch.uint8, device=self.device)
        buf.zero_()
        handle = symm_mem.rendezvous(buf, self.group if self.group is not None
                                     else dist.group.WORLD)
        ptrs = list(handle.buffer_ptrs)

        def view(name, dtype, shape):
            nbytes = sizes_d[name]
            return buf[offs[name]: offs[name] + nbytes].view(dtype).view(*shape)

        sizes_d = dict(sizes)
        self.recv_rows = view("recv_rows", torch.bfloat16, (rows, H))
        self.recv_meta = view("recv_meta", torch.int32, (rows, k))
        self.back_rows = view("back_rows", torch.bfloat16, (rows, H))
        self.back_dw = view("back_dw", torch.float32, (rows, k))
        self.flags = view("flags", torch.int64, (FLAG_WORDS,))
        table = lambda name: torch.tensor([q + offs[name] for q in ptrs], dtype=torch.int64,
                                          device=self.device)
        self.peer_recv_rows = table("recv_rows")
        self.peer_recv_meta = table("recv_meta")
        self.peer_back_rows = table("back_rows")
        self.peer_back_dw = table("back_dw")
        self.peer_flags = table("flags")
        self._buf, self._handle = buf, handle
        self.cap = cap
        self.epoch = 0
        self.step = 0  # epoch of the pipelined exchange's point-to-point flags
        torch.cuda.current_stream(self.device).synchronize()
        dist.barrier(group=self.group)  # every rank's flags are zero before the first barrier

    def release(self):
        """Drop the mapped buffers (the group they were mapped over is gone)."""
        self._buf = self._handle = None
        self.cap = 0

    def barrier(self):
        """The bounded rank barrier of a phase, then the fault-word snapshot
        that the next call checks (a peer that never arrives sets bit 1)."""
        self.epoch += 1
        ops.ep_barrier(self.peer_flags, self.flags, self.me, self.P, self.epoch)
        faults.snapshot(self.device)


_COPY_STREAMS: dict = {}


def _copy_stream(device):
    key = str(device)
    if key not in _COPY_STREAMS:
        _COPY_STREAMS[key] = torch.cuda.Stream(device)
    return _COPY_STREAMS[key]


class _EPMoEP2PFn(torch.autograd.Function):
    """The expert-parallel layer with its exchanges as peer-memory stores:
    one kernel gathers each token's row and stores it into the owners' receive
    buffers (with its slot words), one kernel reduces each received row's slots
    and stores the result into the source's buffers, and bounded barriers over
    flag words separate the phases.  One all-gather of the per-rank counts and
    one host read per step.

    Overlap (comm_sms > 0): the transfers run on a copy stream.  The tokens are
    split into `chunks` ranges, each with its own send plan and its own
    transport (buffers and barrier flags): chunk c+1's rows travel while chunk
    c's experts compute, and chunk c's results travel back while chunk c+1
    computes; in the backward the last results travel while the weight
    gradients compute.  While transfers may run beside them the persistent
    kernels leave comm_sms SMs free.  Every rank issues the same barriers in
    the same order."""

    @staticmethod
    def forward(ctx, x, w_router, w_gu, w_d, top_k, norm, num_experts, group, transports,
                comm_sms):
        faults.raise_pending(x.device)
        tr0 = transports[0]
        P, me = tr0.P, tr0.me
        C = len(transports)
        E_loc = w_gu.shape[0]
        T, H = x.shape
        B = CudaExpertOps
        xb = _as_bf16(x)
        dev = xb.device
        s0 = torch.cuda.current_stream(dev)
        s1 = _copy_stream(dev) if comm_sms else s0
        logits_buf, wr, sel, rw = B.router(xb, w_router, num_experts, top_k, norm)
        span = [(T * c // C, T * (c + 1) // C) for c in range(C)]
        sends, counts = [], []
        for a, b in span:
            dest, slots = ops.ep_route(sel[a:b], E_loc, P)
            send = ops.dispatch(dest, P, partial=True)
            sends.append(send)
            counts.append(torch.cat([send.counts, slots,
                                     torch.full((1,), b - a, device=dev, dtype=torch.int32)]))
        W = 2 * P + 1
        sig = _layer_signature(num_experts, top_k, H, w_gu.shape[1] // 2, C)
        counts.append(torch.tensor(sig, device=dev, dtype=torch.int32))
        gathered = torch.empty(P, C * W + len(sig), device=dev, dtype=torch.int32)
        dist.all_gather_into_tensor(gathered, torch.cat(counts), group=group)
        host = gathered.cpu()  # the one host read of the step
        _check_signatures(host[:, C * W:].tolist(), sig)
        n_recv, slots_in, n_back, plans = [], [], [], []
        for c in range(C):
            hc = host[:, c * W:(c + 1) * W]
            transports[c].ensure(int(hc[:, 2 * P].max()))
            n_recv.append(int(hc[:, me].sum()))
            slots_in.append(int(hc[:, P + me].sum()))
            n_back.append(int(hc[me, :P].sum()))
            plans.append(ops.ep_p2p_plan(gathered[:, c * W:], me, P))
        wgu_b, wd_b = B.cast(w_gu), B.cast(w_d)

        def send_rows(c):
            a, b = span[c]
            ops.ep_p2p_send(xb[a:b], sends[c], plans[c], transports[c].peer_recv_rows, sel[a:b],
                            rw[a:b], E_loc, transports[c].peer_recv_meta)

        ready = s0.record_event()
        send_rows(0)
        sent = [None] * C
        if C > 1:
            with torch.cuda.stream(s1):
                s1.wait_event(ready)
                for c in range(1, C):
                    send_rows(c)
                    sent[c] = s1.record_event()
        ectxs, ret, keep = [None] * C, [None] * C, []
        overlap = backend_overlap(comm_sms) if (comm_sms and C > 1) else nullcontext()
        with overlap:
            for c in range(C):
                if sent[c] is not None:
                    s0.wait_event(sent[c])
                tr = transports[c]
                tr.barrier()
                sel_loc, w_loc = B.unpack(tr.recv_meta[:n_recv[c]])
                y, ectxs[c] = B.experts_fwd(tr.recv_rows[:n_recv[c]], sel_loc, w_loc, wgu_b,
                                            wd_b, slots_in[c], combine=False)
                if ectxs[c] is None:
                    continue
                if C > 1:  # the combine + return of chunk c beside chunk c+1's experts
                    done = s0.record_event()
                    with torch.cuda.stream(s1):
                        s1.wait_event(done)
                        ops.ep_p2p_reduce_return(y, ectxs[c][0], plans[c], tr.peer_back_rows, P,
                                                 weights=w_loc)
                        ret[c] = s1.record_event()
                    keep.append(w_loc)
                else:
                    ops.ep_p2p_reduce_return(y, ectxs[c][0], plans[c], tr.peer_back_rows, P,
                                             weights=w_loc)
        out = xb.new_empty(T, H)
        backs = []
        for c, (a, b) in enumerate(span):
            if ret[c] is not None:
                s0.wait_event(ret[c])
            transports[c].barrier()
            back = dataclasses.replace(sends[c], inv_pad=ops.ep_p2p_back_inv(sends[c], plans[c]))
            backs.append(back)
            ops.gather_rows_bwd(transports[c].back_rows[:n_back[c]], back, out=out[a:b])
        ctx.save_for_backward(xb, logits_buf, wr, sel)
        ctx.meta = (span, sends, backs, plans, ectxs, n_recv, n_back, transports, top_k, norm,
                    num_experts, E_loc, H, w_gu.shape[1] // 2, x.dtype, comm_sms)
        ctx.mark_non_differentiable(sel)
        E = num_experts
        logits = logits_buf if logits_buf.shape[1] == E else logits_buf[:, :E]
        return out.to(x.dtype), logits, sel

    @staticmethod
    def backward(ctx, d_out, d_logits, _d_sel):
        xb, logits_buf, wr, sel = ctx.saved_tensors
        (span, sends, backs, plans, ectxs, n_recv, n_back, transports, top_k, norm, num_experts,
         E_loc, H, I, xdtype, comm_sms) = ctx.meta
        faults.raise_pending(xb.device)
        B = CudaExpertOps
        C = len(span)
        P = transports[0].P
        dev = xb.device
        s0 = torch.cuda.current_stream(dev)
        s1 = _copy_stream(dev) if comm_sms else s0
        if d_out is None:
            d_out = torch.zeros(xb.shape, device=dev, dtype=xb.dtype)
        d_out = _as_bf16(d_out)

        def send_rows(c):
            a, b = span[c]
            ops.ep_p2p_send(d_out[a:b], sends[c], plans[c], transports[c].peer_recv_rows)

        ready = s0.record_event()
        send_rows(0)
        sent = [None] * C
        if C > 1:
            with torch.cuda.stream(s1):
                s1.wait_event(ready)
                for c in range(1, C):
                    send_rows(c)
                    sent[c] = s1.record_event()
        ret, states, keep = [None] * C, [None] * C, []
        g_gu = g_d = None

        def beside_transfers(busy):
            """The SM limit while a transfer may run on the copy stream."""
            return backend_overlap(comm_sms) if (comm_sms and busy) else nullcontext()

        for c in range(C):
            if sent[c] is not None:
                s0.wait_event(sent[c])
            tr = transports[c]
            tr.barrier()
            # beside chunk c's dgrads: later chunks' sends and earlier chunks' returns
            with beside_transfers(C > 1):
                dxs, dw_rows, states[c] = B.experts_dgrad(
                    ectxs[c], tr.recv_rows[:n_recv[c]], top_k, dev, reduce=False)
            if ectxs[c] is None:
                continue
            if comm_sms:  # the return of chunk c beside the next GEMMs
                done = s0.record_event()
                with torch.cuda.stream(s1):
                    s1.wait_event(done)
                    ops.ep_p2p_reduce_return(dxs, ectxs[c][0], plans[c], tr.peer_back_rows,
                                             P, dw_rows=dw_rows, peer_dw=tr.peer_back_dw)
                    ret[c] = s1.record_event()
                keep.append((dxs, dw_rows))
            else:
                ops.ep_p2p_reduce_return(dxs, ectxs[c][0], plans[c], tr.peer_back_rows, P,
                                         dw_rows=dw_rows, peer_dw=tr.peer_back_dw)
        with beside_transfers(True):  # the returns run beside the weight gradients
            for c in range(C):
                g_gu, g_d = B.experts_wgrad(states[c], g_gu, g_d, E_loc, H, I, dev)
        d_rw = torch.empty(xb.shape[0], top_k, device=dev, dtype=torch.float32)
        for c, (a, b) in enumerate(span):
            if ret[c] is not None:
                s0.wait_event(ret[c])
            transports[c].barrier()
            ops.ep_weight_grad(transports[c].back_dw[:n_back[c]], backs[c], sel[a:b], E_loc,
                               out=d_rw[a:b])
        del keep
        dx_router, g_router = B.router_bwd(xb, wr, logits_buf, sel, d_rw, d_logits, num_experts,
                                           top_k, norm)
        dx = xb.new_empty(xb.shape)
        for c, (a, b) in enumerate(span):
            ops.gather_rows_bwd(transports[c].back_rows[:n_back[c]], backs[c],
                                addend=dx_router[a:b], out=dx[a:b])
        faults.snapshot(dev)
        return (dx.to(xdtype), g_router, g_gu, g_d, None, None, None, None, None, None)


class _EPMoEPipeFn(torch.autograd.Function):
    """The expert-parallel layer over peer memory, pipelined per source rank.

    Each owner works through the rows it receives one source rank at a time,
    its own rows first (a local copy, available at once) and then the others
    in the order they arrive (rank me-1, me-2, ...: each source stores to the
    ranks after it first), while the rest of the rows still cross NVLink on a
    copy stream; each source chunk's results go back to that source on the
    copy stream while the next chunk computes.  Completion is signalled point
    to point instead of by group barriers: a source sets a flag word at every
    owner when all its rows are stored, an owner sets one at a source when
    that source's results are stored (b200moe_ep_signal / _wait, bounded
    waits).  The backward mirrors it with the upstream gradient rows; the
    chunks' activations sit in shared row buffers (RowArena), so each expert
    weight gradient is one launch over every source's rows, beside the last
    returns.  Every buffer is reused only after the flag that orders it:
    a source stores the backward's rows only after its forward has received
    every owner's results, which each owner signals after it consumed that
    source's forward rows (and likewise from one step to the next)."""

    @staticmethod
    def forward(ctx, x, w_router, w_gu, w_d, top_k, norm, num_experts, group, tr, comm_sms):
        faults.raise_pending(x.device)
        P, me = tr.P, tr.me
        E_loc = w_gu.shape[0]
        T, H = x.shape
        B = CudaExpertOps
        xb = _as_bf16(x)
        dev = xb.device
        s0 = torch.cuda.current_stream(dev)
        s1 = _copy_stream(dev)
        logits_buf, wr, sel, rw = B.router(xb, w_router, num_experts, top_k, norm)
        dest, slots = ops.ep_route(sel, E_loc, P)
        send = ops.dispatch(dest, P, partial=True)
        sig = _layer_signature(num_experts, top_k, H, w_gu.shape[1] // 2, 1)
        counts = torch.cat([send.counts, slots, torch.full((1,), T, device=dev, dtype=torch.int32),
                            torch.tensor(sig, device=dev, dtype=torch.int32)])
        W = 2 * P + 1
        gathered = torch.empty(P, W + len(sig), device=dev, dtype=torch.int32)
        dist.all_gather_into_tensor(gathered, counts, group=group)
        host = gathered.cpu()  # the one host read of the step
        _check_signatures(host[:, W:].tolist(), sig)
        tr.ensure(int(host[:, 2 * P].max()))
        rows_from = [int(v) for v in host[:, me]]
        slots_from = [int(v) for v in host[:, P + me]]
        base = [sum(rows_from[:s]) for s in range(P)]
        n_back = int(host[me, :P].sum())
        plan = ops.ep_p2p_plan(gathered, me, P)
        tr.step += 1
        step = tr.step
        wgu_b, wd_b = B.cast(w_gu), B.cast(w_d)
        # this rank's own rows: a local copy, ready for the first chunk
        ops.ep_p2p_send_part(xb, send, plan, tr.peer_recv_rows, me, 1, sel, rw, E_loc,
                             tr.peer_recv_meta)
        ready = s0.record_event()
        with torch.cuda.stream(s1), _transfer_limit(comm_sms, P):
            s1.wait_event(ready)
            ops.ep_p2p_send_part(xb, send, plan, tr.peer_recv_rows, me, 2, sel, rw, E_loc,
                                 tr.peer_recv_meta)
            ops.ep_signal(tr.peer_flags, PH_FWD_SEND, me, P, step)
        order = [(me - j) % P for j in range(P)]
        ectxs, keep = [None] * P, []
        arena = RowArena.for_chunks(rows_from, slots_from, E_loc, dev)
        arena.alloc("xs", H)
        arena.alloc("h", w_gu.shape[1] // 2)
        with backend_overlap(comm_sms) if (comm_sms and P > 1) else nullcontext():
            for s in order:
                if s != me:
                    ops.ep_wait(tr.flags, PH_FWD_SEND, P, step, src=s)
                n = rows_from[s]
                rows = tr.recv_rows[base[s]:base[s] + n]
                sel_loc, w_loc = B.unpack(tr.recv_meta[base[s]:base[s] + n])
                y, ectxs[s] = B.experts_fwd(rows, sel_loc, w_loc, wgu_b, wd_b, slots_from[s],
                                            combine=False, arena=arena, src=s)
                done = s0.record_event()
                with torch.cuda.stream(s1), _transfer_limit(comm_sms, P):
                    s1.wait_event(done)
                    if ectxs[s] is not None:
                        ops.ep_p2p_reduce_return_src(y, ectxs[s][0], plan, tr.peer_back_rows, P,
                                                     s, weights=w_loc)
                    ops.ep_signal(tr.peer_flags, PH_FWD_RETURN, me, P, step, dest=s)
                keep.append((y, w_loc))
        s0.wait_stream(s1)
        del keep
        ops.ep_wait(tr.flags, PH_FWD_RETURN, P, step)
        back = dataclasses.replace(send, inv_pad=ops.ep_p2p_back_inv(send, plan))
        out = ops.gather_rows_bwd(tr.back_rows[:n_back], back)
        faults.snapshot(dev)
        ctx.save_for_backward(xb, logits_buf, wr, sel)
        ctx.meta = (send, back, plan, ectxs, rows_from, base, n_back, tr, step, top_k, norm,
                    num_experts, E_loc, H, w_gu.shape[1] // 2, x.dtype, comm_sms, arena)
        ctx.mark_non_differentiable(sel)
        E = num_experts
        logits = logits_buf if logits_buf.shape[1] == E else logits_buf[:, :E]
        return out.to(x.dtype), logits, sel

    @staticmethod
    def backward(ctx, d_out, d_logits, _d_sel):
        xb, logits_buf, wr, sel = ctx.saved_tensors
        (send, back, plan, ectxs, rows_from, base, n_back, tr, step, top_k, norm, num_experts,
         E_loc, H, I, xdtype, comm_sms, arena) = ctx.meta
        faults.raise_pending(xb.device)
        B = CudaExpertOps
        P, me = tr.P, tr.me
        dev = xb.device
        s0 = torch.cuda.current_stream(dev)
        s1 = _copy_stream(dev)
        if d_out is None:
            d_out = torch.zeros(xb.shape, device=dev, dtype=xb.dtype)
        d_out = _as_bf16(d_out)
        ops.ep_p2p_send_part(d_out, send, plan, tr.peer_recv_rows, me, 1)
        ready = s0.record_event()
        with torch.cuda.stream(s1), _transfer_limit(comm_sms, P):
            s1.wait_event(ready)
            ops.ep_p2p_send_part(d_out, send, plan, tr.peer_recv_rows, me, 2)
            ops.ep_signal(tr.peer_flags, PH_BWD_SEND, me, P, step)
        order = [(me - j) % P for j in range(P)]
        states, keep = [None] * P, []
        arena.alloc("dy", H)
        arena.alloc("d_gu", 2 * I)
        with backend_overlap(comm_sms) if (comm_sms and P > 1) else nullcontext():
            for s in order:
                if s != me:
                    ops.ep_wait(tr.flags, PH_BWD_SEND, P, step, src=s)
                d_rows = tr.recv_rows[base[s]:base[s] + rows_from[s]]
                dxs, dw_rows, states[s] = B.experts_dgrad(ectxs[s], d_rows, top_k, dev,
                                                          reduce=False, arena=arena, src=s)
                done = s0.record_event()
                with torch.cuda.stream(s1), _transfer_limit(comm_sms, P):
                    s1.wait_event(done)
                    if ectxs[s] is not None:
                        ops.ep_p2p_reduce_return_src(dxs, ectxs[s][0], plan, tr.peer_back_rows,
                                                     P, s, dw_rows=dw_rows,
                                                     peer_dw=tr.peer_back_dw)
                    ops.ep_signal(tr.peer_flags, PH_BWD_RETURN, me, P, step, dest=s)
                keep.append((dxs, dw_rows))
            # the expert weight gradients, one launch each over every source's
            # rows, run beside the last returns
            g_gu, g_d = B.experts_wgrad_segments(states, arena, E_loc, H, I, dev)
        s0.wait_stream(s1)
        del keep
        ops.ep_wait(tr.flags, PH_BWD_RETURN, P, step)
        d_rw = ops.ep_weight_grad(tr.back_dw[:n_back], back, sel, E_loc)
        dx_router, g_router = B.router_bwd(xb, wr, logits_buf, sel, d_rw, d_logits, num_experts,
                                           top_k, norm)
        dx = ops.gather_rows_bwd(tr.back_rows[:n_back], back, addend=dx_router)
        faults.snapshot(dev)
        return (dx.to(xdtype), g_router, g_gu, g_d, None, None, None, None, None, None)


def _transfer_limit(comm_sms, P):
    """The pipelined layer's copy-stream transfers keep to `comm_sms` SMs'
    worth of blocks, so the compute stream's kernels do not wait for SMs the
    transfers hold (at 8 ranks the transfers run for most of the step)."""
    return ops.transfer_sm_limit(comm_sms) if (comm_sms and P > 1) else nullcontext()


def backend_overlap(comm_sms):
    return CudaExpertOps.overlap(comm_sms)


class ExpertParallelMoE(nn.Module):
    """SparseMoE with experts sharded over `group`.

    Same call and outputs as SparseMoE: (out, router_logits, selected_experts).
    ``gate.weight`` is replicated (all-reduce its gradient like any other
    data-parallel parameter); ``experts.gate_up_proj`` / ``down_proj`` hold
    this rank's E/P experts."""

    def __init__(self, config, group=None, backend=CudaExpertOps, chunks=1, comm_sms=0,
                 transport="nccl"):
        super().__init__()
        if transport not in ("nccl", "p2p", "p2p_pipe"):
            raise ValueError(f"transport must be 'nccl', 'p2p' or 'p2p_pipe', got {transport!r}")
        if transport.startswith("p2p") and backend is not CudaExpertOps:
            raise ValueError("the peer-memory transport runs the device kernels only")
        if transport.startswith("p2p") and config.hidden_size not in P2P_HIDDEN_SIZES:
            raise ValueError(f"the peer-memory transport takes hidden sizes {P2P_HIDDEN_SIZES} "
                             f"(its combine-and-return kernel); hidden {config.hidden_size} "
                             f"runs with transport='nccl'")
        self.transport = transport
        self.chunks = chunks
        self.comm_sms = comm_sms
        self.group = group
        P = dist.get_world_size(group)
        r = dist.get_rank(group)
        E = config.num_experts
        if E % P:
            raise ValueError(f"{E} experts do not split over {P} ranks")
        if P > MAX_RANKS:
            raise ValueError(f"expert parallelism supports at most {MAX_RANKS} ranks, got {P}")
        self.num_experts = E
        self.local_experts = E // P
        self.expert_offset = r * self.local_experts
        self.backend = backend
        self.gate = TopKRouter(config)
        self.experts = nn.Module()
        I, H = config.moe_intermediate_size, config.hidden_size
        self.experts.gate_up_proj = nn.Parameter(torch.empty(self.local_experts, 2 * I, H))
        self.experts.down_proj = nn.Parameter(torch.empty(self.local_experts, H, I))

    # ------------------------------------------------------------------ #
    # checkpoints and export: shards <-> the reference's full layout
    # ------------------------------------------------------------------ #
    def get_extra_state(self):
        """Layout tag saved with this rank's shard in state_dict()."""
        return {"expert_parallel_ranks": dist.get_world_size(self.group),
                "rank": dist.get_rank(self.group), "num_experts": self.num_experts}

    def set_extra_state(self, state):
        want = self.get_extra_state()
        if state != want:
            raise ValueError(f"expert shard saved as {state} cannot load into {want}; "
                             "load the full state dict with load_full_state_dict instead")

    @torch.no_grad()
    def full_state_dict(self):
        """gate.weight and the full (E,2I,H) / (E,H,I) expert tensors, gathered
        over the group (every rank returns them): the keys, shapes and dtypes of
        the reference SparseMoE's state dict (train.py:2244-2334), so HF export
        (export_unfused_state_dict / export_hf, train.py:2540-2691) and strict
        Qwen3MoeForCausalLM loading work unchanged."""
        P = dist.get_world_size(self.group)
        out = {"gate.weight": self.gate.weight.detach().clone()}
        for name in ("gate_up_proj", "down_proj"):
            shard = getattr(self.experts, name).detach().contiguous()
            parts = [torch.empty_like(shard) for _ in range(P)]
            dist.all_gather(parts, shard, group=self.group)
            out["experts." + name] = torch.cat(parts)
        return out

    @torch.no_grad()
    def load_full_state_dict(self, state):
        """Load a full (unsharded) SparseMoE state dict: every rank keeps its
        experts [rank*E/P, (rank+1)*E/P)."""
        lo, hi = self.expert_offset, self.expert_offset + self.local_experts
        self.gate.weight.copy_(state["gate.weight"])
        for name in ("gate_up_proj", "down_proj"):
            full = state["experts." + name]
            if full.shape[0] != self.num_experts:
                raise ValueError(f"experts.{name}: expected {self.num_experts} experts, "
                                 f"got {full.shape[0]}")
            getattr(self.experts, name).copy_(full[lo:hi])

    def forward(self, hidden_states):
        if self.backend is CudaExpertOps:
            _require_cuda(hidden_states)
        shape = hidden_states.shape
        x = hidden_states.reshape(-1, shape[-1])
        if self.transport == "p2p_pipe":
            tr = PeerTransport.get(self.group, shape[-1], self.gate.top_k, x.device)
            out, logits, sel = _EPMoEPipeFn.apply(
                x, self.gate.weight, self.experts.gate_up_proj, self.experts.down_proj,
                self.gate.top_k, self.gate.norm_topk_prob, self.num_experts, self.group, tr,
                self.comm_sms)
        elif self.transport == "p2p":
            trs = tuple(PeerTransport.get(self.group, shape[-1], self.gate.top_k, x.device, c)
                        for c in range(max(1, self.chunks)))
            out, logits, sel = _EPMoEP2PFn.apply(
                x, self.gate.weight, self.experts.gate_up_proj, self.experts.down_proj,
                self.gate.top_k, self.gate.norm_topk_prob, self.num_experts, self.group, trs,
                self.comm_sms)
        else:
            out, logits, sel = _EPMoEFn.apply(
                x, self.gate.weight, self.experts.gate_up_proj, self.experts.down_proj,
                self.gate.top_k, self.gate.norm_topk_prob, self.num_experts, self.group,
                self.backend, self.chunks, self.comm_sms)
        lead = shape[:-1]
        return out.view(shape), logits.view(*lead, logits.shape[-1]), sel.view(*lead, sel.shape[-1])
