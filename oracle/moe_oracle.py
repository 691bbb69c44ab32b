"""CPU oracle for the spark-gpt Qwen3-MoE expert layer.

TEST INFRASTRUCTURE ONLY.  This module is the parity checker: only ``tests/``,
``__graft_entry__.smoke()`` and ``bench.py``'s CPU-baseline / reference arm may
import it.  The product path (``spark_gpt_b200``) never imports it and has no CPU
fallback.

It restates, in plain fp32 torch arithmetic (dense math) and numpy (integer
dispatch), the MoE path of spark-gpt's ``train.py``.  The dense math runs on
the device its inputs live on: the CPU for the golden and small cases, a GPU
in fp32 (TF32 off) for the full-size parity cases, which would take the CPU
minutes per case; the integer dispatch and top-k always run in numpy.

* router                    train.py:2144-2158  (TopKRouter.forward)
* dispatch sort/histogram   train.py:2271-2290  (Experts.forward)
* gather + its backward     train.py:2195-2217  (_GatherTopK, _sum_topk_rows)
* SwiGLU expert products    train.py:2311-2318, 1625-1716, 1899-2063
* down projection           train.py:2161-2192, 1746-1896
* combine + its backward    train.py:2220-2241  (_CombineTopK)
* load-balancing loss       train.py:3098-3197  (global_load_balancing_loss)
* post-attention RMSNorm    train.py:162-170    (RMSNorm, applied at :2370)

Every backward is written out explicitly (no autograd) so each GPU kernel can be
checked against the matching oracle function on its own.

Parity pin: ``tests/golden/make_golden.py`` runs the reference module itself on
seeded inputs and stores its outputs under ``tests/golden/``;
``tests/test_oracle_golden.py`` checks this file against them.

Top-k tie rule: the reference trains on CUDA, where ``torch.topk``
(train.py:2147) is torch's radix-select top-k (torch 2.11.0 here; the
reference tested 2.12): the selected set is the k largest probabilities with
ties at the k-th value broken toward the LOWER expert index, and the k winners
are listed in the order that torch's sort of the k results leaves them.  That
sort is a 32-slot bitonic key/value sort (descending; unstable), run on the
winners gathered as [values above the k-th, by ascending index] + [values
equal to the k-th, by ascending index]; equal values come out in a fixed,
shape-dependent order (all-equal rows: k=2 -> [1, 0], k=4 -> [1, 0, 2, 3],
k=8 -> [7, 6, 4, 5, 1, 0, 2, 3]).  ``topk_cuda_order`` restates those three
steps (torch sources: aten/src/ATen/native/cuda/TensorTopK.cu, gatherTopK;
Sort.cu, sortKeyValueInplace -> SmallBitonicSort; SortUtils.cuh, bitonicSort
and bitonicSwap).  It is pinned against ``torch.topk`` on a B200 by
``tests/test_gpu_fullsize.py`` (tie-heavy bf16 logits at E = 8..256).  torch
CPU's partial sort breaks ties differently (``topk([.5,1,1,1,.2], 2)`` gives
indices [1, 3] on CPU); the golden vectors, made on the CPU, carry no ties,
so they pin the rule-independent part.
"""

from __future__ import annotations

import math
from dataclasses import dataclass

import numpy as np
import torch


# --------------------------------------------------------------------------- #
# router (train.py:2144-2158)
# --------------------------------------------------------------------------- #
def softmax_fp32(logits: torch.Tensor) -> torch.Tensor:
    """F.softmax(logits, dtype=float32, dim=-1) (train.py:2146)."""
    z = logits.float()
    m = z.max(dim=-1, keepdim=True).values
    e = torch.exp(z - m)
    return e / e.sum(dim=-1, keepdim=True)


def _bitonic32_desc(keys: np.ndarray, vals: np.ndarray, valid: np.ndarray):
    """torch's 32-slot bitonic key/value sort, descending, on every row at once
    (SortUtils.cuh bitonicSort with bitonicSwap and a greater-than
    comparator; 16 threads, each owning one compare-exchange per substep)."""
    K, V, ok = keys.copy(), vals.copy(), valid.copy()
    t = np.arange(16)

    def substep(stride, flags):
        pos = 2 * t - (t & (stride - 1))
        a, b = pos, pos + stride
        ka, kb, oa, ob = K[:, a], K[:, b], ok[:, a], ok[:, b]
        swap = ((ka > kb) & oa) | ~ob
        x = swap == flags[None, :]
        for arr in (K, V, ok):
            va, vb = arr[:, a].copy(), arr[:, b].copy()
            arr[:, a] = np.where(x, vb, va)
            arr[:, b] = np.where(x, va, vb)

    size = 2
    while size < 32:
        flags = (t & (size // 2)) != 0
        stride = size // 2
        while stride > 0:
            substep(stride, flags)
            stride //= 2
        size *= 2
    stride = 16
    while stride > 0:
        substep(stride, np.zeros(16, dtype=bool))
        stride //= 2
    return K, V


def topk_cuda_order(probs: torch.Tensor, k: int) -> tuple[torch.Tensor, torch.Tensor]:
    """``torch.topk(probs, k)`` as torch's CUDA kernel computes it (see the
    module doc): the k largest entries per row, ties at the k-th value toward
    the lower index, listed in the order torch's bitonic sort of the gathered
    winners leaves them.  Returns (values fp32 (T,k), indices int64 (T,k)) on
    the device of ``probs``.  k <= 32."""
    assert 1 <= k <= 32
    p = probs.detach().float().cpu().numpy()
    T = p.shape[0]
    # the set: stable sort of -p keeps the lower index first among equal values
    order = np.argsort(-p, axis=-1, kind="stable")[:, :k]
    vals = np.take_along_axis(p, order, axis=-1)
    # gathered order: winners above the k-th value by index, then those equal to it
    above = vals > vals[:, k - 1:k]
    key = np.where(above, 0, 1).astype(np.int64) * (p.shape[1] + 1) + order
    g = np.argsort(key, axis=-1, kind="stable")
    gi = np.take_along_axis(order, g, axis=-1)
    gv = np.take_along_axis(vals, g, axis=-1)
    # rows without a tie among their winners sort to the unique descending
    # order; only rows with one need the network
    tie = np.nonzero((vals[:, 1:] == vals[:, :-1]).any(axis=-1))[0]
    if tie.size:
        n = tie.size
        keys = np.zeros((n, 32), dtype=np.float32)
        ids = np.zeros((n, 32), dtype=np.int64)
        valid = np.zeros((n, 32), dtype=bool)
        keys[:, :k], ids[:, :k], valid[:, :k] = gv[tie], gi[tie], True
        K, V = _bitonic32_desc(keys, ids, valid)
        vals[tie], order[tie] = K[:, :k], V[:, :k]
    dev = probs.device
    return (torch.from_numpy(np.ascontiguousarray(vals)).to(dev),
            torch.from_numpy(np.ascontiguousarray(order.astype(np.int64))).to(dev))


def router_select(logits: torch.Tensor, top_k: int, norm_topk_prob: bool = True):
    """Softmax, top-k and renormalisation from given router logits.

    train.py:2146-2153.  Returns (probs fp32 (T,E), weights fp32 (T,k),
    selected int64 (T,k)); the reference casts the weights to the logits'
    dtype afterwards (train.py:2156).
    """
    probs = softmax_fp32(logits)
    w, sel = topk_cuda_order(probs, top_k)
    if norm_topk_prob:
        w = w / w.sum(dim=-1, keepdim=True)
    return probs, w, sel


def router_forward(x: torch.Tensor, w_router: torch.Tensor, top_k: int,
                   norm_topk_prob: bool = True):
    """TopKRouter.forward in fp32: logits = x W_r^T (bias free), then select."""
    logits = x.float() @ w_router.float().t()
    probs, w, sel = router_select(logits, top_k, norm_topk_prob)
    return logits, probs, w, sel


def router_backward(x, w_router, probs, weights, selected, d_weights,
                    norm_topk_prob=True, d_logits_extra=None):
    """Backward of router_forward w.r.t. x and W_r.

    d_weights (T,k) is the gradient reaching the routing weights (from the
    combine).  Through the renormalisation w_i = p_i / S:
    dp_i = (dw_i - sum_j dw_j w_j) / S; through the softmax:
    dlogit = p * (g - <p, g>) with g the scattered dp.  ``d_logits_extra``
    (T,E) is added (the load-balancing loss's gradient into the same logits).
    Returns (d_logits, dx, dW_r) in fp32.
    """
    p = probs.float()
    dw = d_weights.float()
    if norm_topk_prob:
        p_sel = torch.gather(p, 1, selected)
        s = p_sel.sum(dim=-1, keepdim=True)
        w = p_sel / s
        dp_sel = (dw - (dw * w).sum(dim=-1, keepdim=True)) / s
    else:
        dp_sel = dw
    g = torch.zeros_like(p).scatter_(1, selected, dp_sel)
    d_logits = p * (g - (p * g).sum(dim=-1, keepdim=True))
    if d_logits_extra is not None:
        d_logits = d_logits + d_logits_extra.float()
    dx = d_logits @ w_router.float()
    dw_r = d_logits.t() @ x.float()
    return d_logits, dx, dw_r


# --------------------------------------------------------------------------- #
# dispatch (train.py:2271-2290)
# --------------------------------------------------------------------------- #
@dataclass
class Dispatch:
    permutation: np.ndarray          # (R,) int64: sorted position -> flat index t*k+s
    token_index: np.ndarray          # (R,) int64: sorted position -> token
    inverse: np.ndarray              # (R,) int64: flat index -> sorted position
    counts: np.ndarray               # (E,) int64 rows per expert
    offsets: np.ndarray              # (E,) int32 inclusive cumulative counts
    top_k: int


def dispatch(selected: torch.Tensor | np.ndarray, num_experts: int) -> Dispatch:
    """Stable sort of the flat expert ids (train.py:2271-2290).

    Rows end up ordered by (expert, flat index t*k+s); the histogram counts
    every routed row, filler tokens included.
    """
    if isinstance(selected, torch.Tensor):
        selected = selected.detach().cpu()
    sel = np.asarray(selected, dtype=np.int64)
    top_k = sel.shape[-1]
    flat = sel.reshape(-1)
    perm = np.argsort(flat, kind="stable").astype(np.int64)
    inv = np.empty_like(perm)
    inv[perm] = np.arange(perm.size, dtype=np.int64)
    counts = np.bincount(flat, minlength=num_experts).astype(np.int64)
    offsets = np.cumsum(counts).astype(np.int32)
    return Dispatch(perm, perm // top_k, inv, counts, offsets, top_k)


def _index(a: np.ndarray, like: torch.Tensor) -> torch.Tensor:
    """An integer index array as a tensor on the device of ``like`` (the dense
    math runs on whichever device its inputs live on: CPU, or fp32 on a GPU
    for the full-size parity cases)."""
    return torch.from_numpy(a).to(like.device)


def expert_ranges(offsets):
    start = 0
    for e, end in enumerate(np.asarray(offsets).tolist()):
        yield e, start, int(end)
        start = int(end)


# --------------------------------------------------------------------------- #
# gather / combine (train.py:2195-2241)
# --------------------------------------------------------------------------- #
def gather_forward(x, d: Dispatch):
    """sorted_hidden = x[token_index] (train.py:2206)."""
    return x.float()[_index(d.token_index, x)]


def gather_backward(d_rows, d: Dispatch):
    """dx[t] = sum_s d_rows[inverse[t*k+s]] (train.py:2209-2217)."""
    rows = d_rows.float()[_index(d.inverse, d_rows)]
    return rows.view(-1, d.top_k, rows.shape[-1]).sum(dim=1)


def combine_forward(y, sorted_weights, d: Dispatch):
    """out[t] = sum_s w[j] * y[j], j = inverse[t*k+s] (train.py:2229-2233)."""
    weighted = y.float() * sorted_weights.float().unsqueeze(-1)
    rows = weighted[_index(d.inverse, weighted)]
    return rows.view(-1, d.top_k, rows.shape[-1]).sum(dim=1)


def combine_backward(y, sorted_weights, d: Dispatch, d_out):
    """(dy, d_sorted_weights) of combine_forward (train.py:2235-2241)."""
    g = d_out.float()[_index(d.token_index, d_out)]
    dy = g * sorted_weights.float().unsqueeze(-1)
    dw_sorted = (g * y.float()).sum(dim=-1)
    return dy, dw_sorted


# --------------------------------------------------------------------------- #
# expert products (train.py:2304-2318 and the Triton kernels they replace)
# --------------------------------------------------------------------------- #
def swiglu_forward(xs, w_gu, offsets):
    """gu = xs_e W_gu[e]^T per expert; h = silu(g) * u (train.py:2311-2318)."""
    xs = xs.float()
    w_gu = w_gu.float()
    two_i = w_gu.shape[1]
    inter = two_i // 2
    gu = xs.new_zeros(xs.shape[0], two_i)
    for e, s, t in expert_ranges(offsets):
        if t > s:
            gu[s:t] = xs[s:t] @ w_gu[e].t()
    g, u = gu[:, :inter], gu[:, inter:]
    h = g * torch.sigmoid(g) * u
    return gu, h


def swiglu_grad_inputs(gu, dh):
    """d_gate, d_up from gu and dh (train.py:1899-1904)."""
    inter = gu.shape[1] // 2
    g, u = gu[:, :inter].float(), gu[:, inter:].float()
    dh = dh.float()
    sig = torch.sigmoid(g)
    d_gate = dh * u * (sig * (1.0 + g * (1.0 - sig)))
    d_up = dh * g * sig
    return torch.cat([d_gate, d_up], dim=1)


def swiglu_backward(xs, w_gu, gu, dh, offsets):
    """(dxs, dW_gu) of swiglu_forward (train.py:2083-2090, 1907-2026)."""
    xs = xs.float()
    w_gu = w_gu.float()
    d_gu = swiglu_grad_inputs(gu, dh)
    dxs = xs.new_zeros(xs.shape)
    dw = torch.zeros_like(w_gu)
    for e, s, t in expert_ranges(offsets):
        if t > s:
            dxs[s:t] = d_gu[s:t] @ w_gu[e]
            dw[e] = d_gu[s:t].t() @ xs[s:t]
    return dxs, dw, d_gu


def grouped_linear_forward(h, w, offsets):
    """out[r] = h[r] W[e]^T for rows of expert e (train.py:2183-2192)."""
    h = h.float()
    w = w.float()
    out = h.new_zeros(h.shape[0], w.shape[1])
    for e, s, t in expert_ranges(offsets):
        if t > s:
            out[s:t] = h[s:t] @ w[e].t()
    return out


def grouped_linear_backward(h, w, dout, offsets):
    """(dh, dW) of grouped_linear_forward (train.py:1892-1896)."""
    h = h.float()
    w = w.float()
    dout = dout.float()
    dh = h.new_zeros(h.shape)
    dw = torch.zeros_like(w)
    for e, s, t in expert_ranges(offsets):
        if t > s:
            dh[s:t] = dout[s:t] @ w[e]
            dw[e] = dout[s:t].t() @ h[s:t]
    return dh, dw


# --------------------------------------------------------------------------- #
# load-balancing loss (train.py:3098-3197)
# --------------------------------------------------------------------------- #
def lb_partials(logits, selected, valid_mask, num_experts, top_k):
    """One layer's contribution: (soft_sums (E,), hard_counts (E,), entropy, rows).

    train.py:3141-3153: masked softmax sums, masked top-k bincount, masked
    entropy and the valid-row count.
    """
    mask = valid_mask.float()
    probs = softmax_fp32(logits)
    soft = (probs * mask.unsqueeze(-1)).sum(dim=0)
    cw = mask.unsqueeze(-1).expand(-1, top_k).reshape(-1)
    hard = torch.bincount(selected.reshape(-1), weights=cw, minlength=num_experts).float()
    tiny = torch.finfo(torch.float32).tiny
    ent = -(probs * probs.clamp_min(tiny).log() * mask.unsqueeze(-1)).sum()
    return soft, hard, ent, mask.sum()


def load_balancing_loss(logits_layers, selected_layers, valid_mask, *, num_experts,
                        top_k, world_size=1, all_reduce=None):
    """global_load_balancing_loss value, stats and the gradient into each layer's logits.

    ``all_reduce`` (packed fp32 (2E+2,) -> summed over ranks) stands in for
    the NCCL all-reduce at train.py:3162; None means a single process.
    Returns (aux_value, stats dict, [d aux / d logits per layer]).
    """
    if not logits_layers:
        z = torch.zeros(())
        return z, {}, []
    dev = logits_layers[0].device
    soft = torch.zeros(num_experts, device=dev)
    hard = torch.zeros(num_experts, device=dev)
    ent = torch.zeros((), device=dev)
    rows = torch.zeros((), device=dev)
    for lg, sel in zip(logits_layers, selected_layers):
        s, h, e_, r = lb_partials(lg, sel, valid_mask, num_experts, top_k)
        soft, hard, ent, rows = soft + s, hard + h, ent + e_, rows + r
    packed = torch.cat([hard, soft, ent.reshape(1), rows.reshape(1)])
    if all_reduce is not None:
        packed = all_reduce(packed)
    g_counts = packed[:num_experts]
    g_soft = packed[num_experts:2 * num_experts]
    g_ent = packed[2 * num_experts]
    g_rows = packed[2 * num_experts + 1]
    safe = g_rows.clamp_min(1.0)
    has = (g_rows > 0).float()
    a = g_counts / safe
    aux = has * num_experts * torch.dot(a, g_soft / safe)
    frac = g_counts / (safe * top_k)
    stats = {
        "aux_loss": aux,
        "assignment_min_frac": frac.min(),
        "assignment_max_frac": frac.max(),
        "assignment_cv": frac.std(unbiased=False) / frac.mean().clamp_min(1e-12),
        "router_entropy": g_ent / safe,
        "unused_experts": (g_counts == 0).sum().float(),
    }
    # d(local proxy)/d soft_sums = has * world * E / rows * a   (train.py:3172-3179)
    coef = has * world_size * num_experts / safe * a
    mask = valid_mask.float()
    grads = []
    for lg in logits_layers:
        p = softmax_fp32(lg)
        gp = mask.unsqueeze(-1) * coef.unsqueeze(0)
        grads.append(p * (gp - (p * gp).sum(dim=-1, keepdim=True)))
    return aux, stats, grads


# --------------------------------------------------------------------------- #
# whole layer
# --------------------------------------------------------------------------- #
def layer_forward_backward(x, w_router, w_gu, w_down, top_k, d_out, *,
                           norm_topk_prob=True, selected=None, weights=None,
                           d_logits_extra=None, logits=None):
    """SparseMoE forward (train.py:2331-2334) and backward in fp32.

    ``selected``/``weights``/``logits`` may be injected so the oracle routes
    exactly as the device did.  Returns a dict of every intermediate and
    gradient (dx, dW_r, dW_gu, dW_down, ...).
    """
    E = w_gu.shape[0]
    x = x.float()
    if logits is None:
        logits = x @ w_router.float().t()
    probs, w_sel, sel = router_select(logits, top_k, norm_topk_prob)
    if selected is not None:
        sel = selected.long()
    if weights is not None:
        w_sel = weights.float()
    d = dispatch(sel, E)
    sorted_w = w_sel.reshape(-1)[_index(d.permutation, w_sel)]
    xs = gather_forward(x, d)
    gu, h = swiglu_forward(xs, w_gu, d.offsets)
    y = grouped_linear_forward(h, w_down, d.offsets)
    out = combine_forward(y, sorted_w, d)

    dy, dw_sorted = combine_backward(y, sorted_w, d, d_out)
    dh, dw_down = grouped_linear_backward(h, w_down, dy, d.offsets)
    dxs, dw_gu, d_gu = swiglu_backward(xs, w_gu, gu, dh, d.offsets)
    dx_gather = gather_backward(dxs, d)
    d_weights = torch.empty(d.permutation.size, device=x.device)
    d_weights[_index(d.permutation, x)] = dw_sorted
    d_weights = d_weights.view(-1, top_k)
    d_logits, dx_router, dw_r = router_backward(
        x, w_router, probs, w_sel, sel, d_weights, norm_topk_prob, d_logits_extra)
    return {
        "logits": logits, "probs": probs, "weights": w_sel, "selected": sel,
        "dispatch": d, "sorted_weights": sorted_w, "xs": xs, "gu": gu, "h": h,
        "y": y, "out": out, "dy": dy, "dw_sorted": dw_sorted, "dh": dh,
        "d_gu": d_gu, "dxs": dxs, "d_weights": d_weights, "d_logits": d_logits,
        "dx": dx_gather + dx_router, "dW_router": dw_r, "dW_gate_up": dw_gu,
        "dW_down": dw_down,
    }


# --------------------------------------------------------------------------- #
# post-attention RMSNorm (train.py:162-170, applied before the layer at :2370)
# --------------------------------------------------------------------------- #
def rmsnorm_forward(x, w, eps):
    """RMSNorm.forward: r = rsqrt(mean(x^2) + eps) in fp32; for bf16 input the
    result is bf16(bf16(x * r) * bf16(w)) (the cast back to the input dtype,
    then the product with the weight cast to it).  Returns (x_n fp32 holding
    the input dtype's values, r (T,))."""
    xf = x.float()
    r = torch.rsqrt(xf.pow(2).mean(dim=-1, keepdim=True) + eps)
    if x.dtype == torch.bfloat16:
        y1 = (xf * r).to(torch.bfloat16).float()
        x_n = (y1 * w.to(torch.bfloat16).float()).to(torch.bfloat16).float()
    else:
        x_n = (xf * r) * w.float()
    return x_n, r.squeeze(-1)


def rmsnorm_backward(x, w, r, g, bf16_io=True):
    """(dx, dw) of rmsnorm_forward for the upstream gradient g, in fp32 (the
    casts' backwards are identities): dy = g * w; dx = r * dy - (r^3 / H) *
    x * <dy, x>; dw = sum_t g * (x * r), with x * r rounded to bf16 when the
    input is bf16 (the value the weight multiplies)."""
    xf = x.float()
    g = g.float()
    H = xf.shape[-1]
    rr = r.float().unsqueeze(-1)
    wv = w.to(torch.bfloat16).float() if bf16_io else w.float()
    dy = g * wv
    dot = (dy * xf).sum(dim=-1, keepdim=True)
    dx = rr * dy - (rr ** 3 / H) * xf * dot
    y1 = xf * rr
    if bf16_io:
        y1 = y1.to(torch.bfloat16).float()
    dw = (g * y1).sum(dim=0)
    return dx, dw


def mup_std(hidden, base_dim=256, hidden_std=0.02, num_layers=12):
    """Expert init stds of apply_mup_init (train.py:2727-2739)."""
    m = hidden / base_dim
    std_in = hidden_std / math.sqrt(m)
    return std_in, std_in / math.sqrt(2 * num_layers)
