"""Tensor-level wrappers over the C ABI (include/b200moe.h).

Each function allocates its outputs through torch's caching allocator, passes
raw pointers plus torch's current CUDA stream to libb200moe.so, and returns
the outputs.  Shapes follow spark-gpt's MoE path (train.py:2134-2334).
"""

from __future__ import annotations

import ctypes
from contextlib import contextmanager
from dataclasses import dataclass

import torch

from . import _lib

# --------------------------------------------------------------------------- #
# launch accounting and optional per-op CUDA-event timing (used by bench.py)
# --------------------------------------------------------------------------- #
LAUNCHES = {"count": 0}
_timing: dict[str, list] | None = None


def set_timing(names):
    """Record CUDA events around the named ops (None disables)."""
    global _timing
    _timing = None if names is None else {n: [] for n in names}
    return _timing


@contextmanager
def timed(name: str):
    """CUDA events on the current stream around a block (e.g. a collective)."""
    if _timing is not None and name in _timing:
        s = torch.cuda.Event(enable_timing=True)
        e = torch.cuda.Event(enable_timing=True)
        s.record()
        yield
        e.record()
        _timing[name].append((s, e))
    else:
        yield


@contextmanager
def persistent_sm_limit(sms: int):
    """Persistent kernels enqueued inside the block use at most `sms` SMs
    (0 = all), leaving the rest to a collective running beside them."""
    prev = int(_lib.value("b200moe_set_persistent_sm_limit", int(sms)))
    try:
        yield
    finally:
        _lib.value("b200moe_set_persistent_sm_limit", prev)


@contextmanager
def transfer_sm_limit(sms: int):
    """Peer-memory transfer kernels enqueued inside the block launch at most 8
    blocks per SM of `sms` SMs (0 = all), leaving the other SMs to the
    kernels of the stream they run beside."""
    prev = int(_lib.value("b200moe_set_transfer_sm_limit", int(sms)))
    try:
        yield
    finally:
        _lib.value("b200moe_set_transfer_sm_limit", prev)


def _launch(name: str, kernels: int, fn, *args):
    LAUNCHES["count"] += kernels
    if _timing is not None and name in _timing:
        s = torch.cuda.Event(enable_timing=True)
        e = torch.cuda.Event(enable_timing=True)
        s.record()
        _lib.call(fn, *args)
        e.record()
        _timing[name].append((s, e))
    else:
        _lib.call(fn, *args)


def _p(t):
    return None if t is None else ctypes.c_void_p(t.data_ptr())


def _s(t: torch.Tensor):
    return ctypes.c_void_p(torch.cuda.current_stream(t.device).cuda_stream)


def _check(t: torch.Tensor, dtype, name):
    if not t.is_cuda:
        raise RuntimeError(f"{name}: the B200 MoE kernels need CUDA tensors (no CPU path)")
    if t.dtype != dtype:
        raise RuntimeError(f"{name}: expected {dtype}, got {t.dtype}")
    if not t.is_contiguous():
        raise RuntimeError(f"{name}: expected a contiguous tensor")


BF16 = torch.bfloat16


def padded_rows(routed_rows: int, num_experts: int) -> int:
    return int(_lib.value("b200moe_padded_rows", routed_rows, num_experts))


def router_width(num_experts: int) -> int:
    return int(_lib.value("b200moe_router_width", num_experts))


# --------------------------------------------------------------------------- #
# weights
# --------------------------------------------------------------------------- #
def cast_bf16(w: torch.Tensor, rows_out: int | None = None) -> torch.Tensor:
    """bf16 compute copy of an fp32 master (rows beyond w.shape[0] zero)."""
    if w.dtype == BF16 and rows_out in (None, w.shape[0]):
        return w.contiguous()
    w = w.detach().float().contiguous()
    rows = w.shape[0]
    cols = w[0].numel() if rows else 0
    rows_out = rows if rows_out is None else rows_out
    out = torch.empty((rows_out, *w.shape[1:]), device=w.device, dtype=BF16)
    _launch("cast", 1, "b200moe_cast_f32_to_bf16", _p(w), rows, cols, rows_out, _p(out), _s(w))
    return out


# --------------------------------------------------------------------------- #
# router (train.py:2144-2158)
# --------------------------------------------------------------------------- #
def router_logits(x: torch.Tensor, w_router: torch.Tensor) -> torch.Tensor:
    _check(x, BF16, "router_logits x")
    _check(w_router, BF16, "router_logits w")
    T, H = x.shape
    W = w_router.shape[0]
    out = torch.empty(T, W, device=x.device, dtype=BF16)
    if T:
        _launch("router_logits", 1, "b200moe_router_logits", _p(x), _p(w_router), T, H, W,
                _p(out), _s(x))
    return out


def router_topk(logits: torch.Tensor, num_experts: int, top_k: int, norm: bool):
    """logits (T, ld) bf16 or fp32 (first num_experts columns used)."""
    if logits.dtype not in (BF16, torch.float32):
        raise RuntimeError("router_topk: logits must be bf16 or fp32")
    if logits.stride(1) != 1:
        raise RuntimeError("router_topk: logits rows must be contiguous")
    T = logits.shape[0]
    sel = torch.empty(T, top_k, device=logits.device, dtype=torch.int64)
    w = torch.empty(T, top_k, device=logits.device, dtype=BF16)
    if T:
        _launch("router_topk", 1, "b200moe_router_topk_fwd", _p(logits),
                int(logits.dtype == torch.float32), logits.stride(0), T, num_experts, top_k,
                int(norm), _p(sel), _p(w), _s(logits))
    return sel, w


def router_topk_bwd(logits, selected, d_weights, d_extra, num_experts, top_k, norm):
    T, ld = logits.shape[0], logits.stride(0)
    out = torch.empty(T, ld, device=logits.device, dtype=BF16)
    if T:
        _launch("router_topk_bwd", 1, "b200moe_router_topk_bwd", _p(logits), ld, _p(selected),
                _p(d_weights), _p(d_extra), T, num_experts, top_k, int(norm), _p(out),
                _s(logits))
    return out


def router_dgrad(d_logits: torch.Tensor, w_router: torch.Tensor) -> torch.Tensor:
    T, W = d_logits.shape
    H = w_router.shape[1]
    out = torch.empty(T, H, device=d_logits.device, dtype=BF16)
    if T:
        _launch("router_dgrad", 1, "b200moe_router_dgrad", _p(d_logits), _p(w_router), T, H, W,
                _p(out), _s(d_logits))
    return out


def router_wgrad(x, d_logits, num_experts, out=None, accumulate=False):
    T, H = x.shape
    W = d_logits.shape[1]
    if out is None:
        out = torch.empty(num_experts, H, device=x.device, dtype=torch.float32)
        accumulate = False
    if T:
        nbytes = int(_lib.value("b200moe_router_wgrad_scratch_bytes", T, H, num_experts))
        scratch = torch.empty(max(nbytes, 16), device=x.device, dtype=torch.uint8)
        _launch("router_wgrad", 2, "b200moe_router_wgrad", _p(x), _p(d_logits), T, H,
                num_experts, W, _p(out), int(accumulate), _p(scratch), nbytes, _s(x))
    elif not accumulate:
        out.zero_()
    return out


# --------------------------------------------------------------------------- #
# dispatch (train.py:2271-2290)
# --------------------------------------------------------------------------- #
@dataclass
class Dispatch:
    counts: torch.Tensor       # (E,) int32
    offsets: torch.Tensor      # (E,) int32 inclusive cumsum
    pad_offsets: torch.Tensor  # (E+1,) int32 padded starts; [E] = padded total
    row_flat: torch.Tensor     # (Rcap,) int32 padded row -> flat slot, -1 padding
    inv_pad: torch.Tensor      # (R,) int32 flat slot -> padded row
    tile_expert: torch.Tensor  # (Rcap/128,) int32
    rows_cap: int
    num_tokens: int
    top_k: int
    num_experts: int
    partial: bool = False      # some slots carry no expert (id -1: no row, inv_pad -1)


def dispatch(selected: torch.Tensor, num_experts: int, routed_slots: int | None = None,
             partial: bool = False) -> Dispatch:
    """partial: negative ids may occur and mark slots without an expert (no row,
    inv_pad -1; the row reductions then skip them).  routed_slots, when given,
    is the number of non-negative ids and sizes the padded-row buffers."""
    _check(selected, torch.int64, "dispatch selected")
    T, k = selected.shape
    R = T * k
    dev = selected.device
    cap = padded_rows(R if routed_slots is None else routed_slots, num_experts)
    i32 = dict(device=dev, dtype=torch.int32)
    if R == 0:  # no slots: every expert empty, every row padding (nothing to launch)
        z = lambda n: torch.zeros(n, **i32)  # noqa: E731
        return Dispatch(z(num_experts), z(num_experts), z(num_experts + 1),
                        torch.full((cap,), -1, **i32), z(0), z(cap // 128), cap, T, k,
                        num_experts, partial or routed_slots is not None)
    counts = torch.empty(num_experts, **i32)
    offsets = torch.empty(num_experts, **i32)
    pad = torch.empty(num_experts + 1, **i32)
    row_flat = torch.empty(cap, **i32)
    inv = torch.empty(max(R, 1), **i32)
    tiles = torch.empty(cap // 128, **i32)
    nbytes = int(_lib.value("b200moe_dispatch_scratch_bytes", T, k, num_experts))
    scratch = torch.empty(nbytes, device=dev, dtype=torch.uint8)
    _launch("dispatch", 3, "b200moe_dispatch", _p(selected), T, k, num_experts, _p(counts),
            _p(offsets), _p(pad), _p(row_flat), _p(inv), _p(tiles), _p(scratch), nbytes,
            _s(selected))
    return Dispatch(counts, offsets, pad, row_flat, inv[:R], tiles, cap, T, k, num_experts,
                    partial or routed_slots is not None)


# --------------------------------------------------------------------------- #
# gather / combine (train.py:2195-2241)
# --------------------------------------------------------------------------- #
def _rows_out(out, rows: int, cols: int, like: torch.Tensor, name: str) -> torch.Tensor:
    """A caller's (rows, cols) bf16 destination (checked), or a new one."""
    if out is None:
        return torch.empty(rows, cols, device=like.device, dtype=BF16)
    _check(out, BF16, name)
    if tuple(out.shape) != (rows, cols):
        raise RuntimeError(f"{name}: expected shape {(rows, cols)}, got {tuple(out.shape)}")
    return out


def gather_rows(x: torch.Tensor, d: Dispatch, out=None) -> torch.Tensor:
    """out: an optional contiguous (rows_cap, H) bf16 destination."""
    _check(x, BF16, "gather_rows x")
    H = x.shape[1]
    xs = _rows_out(out, d.rows_cap, H, x, "gather_rows out")
    if d.num_tokens == 0:  # only padding rows
        return xs.zero_()
    _launch("gather", 1, "b200moe_gather_rows", _p(x), _p(d.row_flat),
            _p(d.inv_pad) if d.inv_pad.numel() else None, _p(d.pad_offsets), d.num_tokens,
            d.num_experts, d.top_k, H, d.rows_cap, _p(xs), _s(x))
    return xs


def gather_rows_bwd(dxs, d: Dispatch, addend=None, token_major=False, out=None) -> torch.Tensor:
    """dx[t] = sum_s dxs[row of slot t*k+s] (+ addend); token_major: row t*k+s.
    out: an optional contiguous (T, H) bf16 destination."""
    H = dxs.shape[1]
    if out is None:
        dx = torch.empty(d.num_tokens, H, device=dxs.device, dtype=BF16)
    else:
        _check(out, BF16, "gather_rows_bwd out")
        dx = out
    if d.num_tokens:
        _launch("gather_bwd", 1, "b200moe_gather_rows_bwd", _p(dxs),
                None if token_major else _p(d.inv_pad), _p(addend), d.num_tokens, d.top_k, H,
                int(d.partial), _p(dx), _s(dxs))
    return dx


def rmsnorm(x: torch.Tensor, w: torch.Tensor, eps: float):
    """The reference's RMSNorm (train.py:162-170) on bf16 rows: (x_n bf16, r fp32 per row)."""
    _check(x, BF16, "rmsnorm x")
    T, H = x.shape
    wf = w.detach().float().contiguous()
    x_n = torch.empty_like(x)
    rstd = torch.empty(T, device=x.device, dtype=torch.float32)
    if T:
        _launch("rmsnorm", 1, "b200moe_rmsnorm_fwd", _p(x), _p(wf), T, H, ctypes.c_float(eps),
                _p(x_n), _p(rstd), _s(x))
    return x_n, rstd


def gather_rows_bwd_rmsnorm(dxs, d: Dispatch, addend, x, w, rstd, token_major=False):
    """The gather backward (dxs rows summed per token + addend) with the
    RMSNorm backward folded in: (d x (T, H) bf16, d w (H,) fp32)."""
    H = dxs.shape[1]
    dev = dxs.device
    dx = torch.empty(d.num_tokens, H, device=dev, dtype=BF16)
    dw = torch.empty(H, device=dev, dtype=torch.float32)
    nbytes = int(_lib.value("b200moe_gather_rows_bwd_rmsnorm_scratch_bytes", d.num_tokens, H))
    scratch = torch.empty(max(nbytes, 16), device=dev, dtype=torch.uint8)
    _launch("gather_bwd", 2, "b200moe_gather_rows_bwd_rmsnorm", _p(dxs),
            None if token_major else _p(d.inv_pad), _p(addend), _p(x), _p(w), _p(rstd),
            d.num_tokens, d.top_k, H, int(d.partial), _p(dx), _p(dw), _p(scratch), nbytes,
            _s(dxs))
    return dx, dw


def combine(y, d: Dispatch, weights, token_major=False) -> torch.Tensor:
    _check(weights, BF16, "combine weights")
    H = y.shape[1]
    out = torch.empty(d.num_tokens, H, device=y.device, dtype=BF16)
    if d.num_tokens:
        _launch("combine", 1, "b200moe_combine_fwd", _p(y),
                None if token_major else _p(d.inv_pad), _p(weights), d.num_tokens, d.top_k, H,
                int(d.partial), _p(out), _s(y))
    return out


def combine_bwd(d_out, y, d: Dispatch, weights, token_major=False, out=None):
    """-> (dy (rows_cap, H) bf16, d_weights (T, k) fp32); out: an optional
    contiguous destination for dy."""
    _check(d_out, BF16, "combine_bwd d_out")
    H = y.shape[1]
    dy = _rows_out(out, d.rows_cap, H, y, "combine_bwd out")
    if d.num_tokens == 0:  # only padding rows, no routing weights
        return dy.zero_(), torch.zeros(0, d.top_k, device=y.device, dtype=torch.float32)
    dw = torch.empty(d.num_tokens, d.top_k, device=y.device, dtype=torch.float32)
    _launch("combine_bwd", 2 if token_major else 1, "b200moe_combine_bwd", _p(d_out), _p(y),
            _p(d.row_flat), _p(d.inv_pad), _p(d.pad_offsets), _p(weights), d.num_experts,
            d.num_tokens, d.top_k, H, d.rows_cap, int(token_major), _p(dy), _p(dw), _s(y))
    return dy, dw


# --------------------------------------------------------------------------- #
# expert products (train.py:1625-2090)
# --------------------------------------------------------------------------- #
def gate_up_fwd(xs, w_gu, d: Dispatch, out_h=None):
    """-> (gu, h); out_h: an optional contiguous (rows_cap, I) bf16 destination."""
    E, two_i, H = w_gu.shape
    I = two_i // 2
    gu = torch.empty(d.rows_cap, two_i, device=xs.device, dtype=BF16)
    h = _rows_out(out_h, d.rows_cap, I, xs, "gate_up_fwd out_h")
    _launch("gate_up_fwd", 1, "b200moe_expert_gate_up_fwd", _p(xs), _p(w_gu), _p(d.tile_expert),
            _p(d.pad_offsets), d.rows_cap, E, H, I, _p(gu), _p(h), _s(xs))
    return gu, h


def down_fwd(h, w_d, d: Dispatch, token_major=False):
    """y = h W_d[e]^T; token_major: (T*k, H) with slot t*k+s in row t*k+s."""
    E, H, I = w_d.shape
    rows = d.num_tokens * d.top_k if token_major else d.rows_cap
    y = torch.empty(max(rows, 1), H, device=h.device, dtype=BF16)
    _launch("down_fwd", 1, "b200moe_expert_down_fwd", _p(h), _p(w_d), _p(d.tile_expert),
            _p(d.pad_offsets), _p(d.row_flat) if token_major else None, d.rows_cap, E, H, I,
            _p(y), _s(h))
    return y


def down_dgrad_swiglu(dy, w_d, gu, d: Dispatch, out=None):
    """d_gu (rows_cap, 2I) bf16; out: an optional contiguous destination."""
    E, H, I = w_d.shape
    d_gu = _rows_out(out, d.rows_cap, 2 * I, dy, "down_dgrad_swiglu out")
    _launch("down_dgrad", 1, "b200moe_expert_down_dgrad_swiglu", _p(dy), _p(w_d), _p(gu),
            _p(d.tile_expert), _p(d.pad_offsets), d.rows_cap, E, H, I, _p(d_gu), _s(dy))
    return d_gu


def gate_up_dgrad(d_gu, w_gu, d: Dispatch, token_major=False):
    """dxs = d_gu W_gu[e]; token_major: (T*k, H) with slot t*k+s in row t*k+s."""
    E, two_i, H = w_gu.shape
    rows = d.num_tokens * d.top_k if token_major else d.rows_cap
    dxs = torch.empty(max(rows, 1), H, device=d_gu.device, dtype=BF16)
    _launch("gate_up_dgrad", 1, "b200moe_expert_gate_up_dgrad", _p(d_gu), _p(w_gu),
            _p(d.tile_expert), _p(d.pad_offsets), _p(d.row_flat) if token_major else None,
            d.rows_cap, E, H, two_i // 2, _p(dxs), _s(d_gu))
    return dxs


def wgrad(a, b, d: Dispatch, name="wgrad", out=None, accumulate=False):
    """(E, M, N) fp32: a_e^T b_e over the padded rows of each expert."""
    M, N = a.shape[1], b.shape[1]
    if out is None:
        out = torch.empty(d.num_experts, M, N, device=a.device, dtype=torch.float32)
        accumulate = False
    _launch(name, 1, "b200moe_expert_wgrad", _p(a), M, _p(b), N, _p(d.pad_offsets),
            d.num_experts, d.rows_cap, _p(out), int(accumulate), _s(a))
    return out


def wgrad_segments(a, b, seg_offsets, num_experts, name="wgrad", out=None, accumulate=False):
    """(E, M, N) fp32: a_e^T b_e where expert e's rows are the union over
    segments s of [seg_offsets[s, e], seg_offsets[s, e+1]) of a and b
    (rows_total, M) / (rows_total, N) bf16; seg_offsets (S, E+1) int32."""
    M, N = a.shape[1], b.shape[1]
    _check(a, BF16, f"{name} a")
    _check(b, BF16, f"{name} b")
    if a.shape[0] != b.shape[0]:
        raise RuntimeError(f"{name}: a and b must have the same rows")
    _check(seg_offsets, torch.int32, f"{name} seg_offsets")
    if seg_offsets.dim() != 2 or seg_offsets.shape[1] != num_experts + 1:
        raise RuntimeError(f"{name}: seg_offsets must be (segments, E+1)")
    if out is None:
        out = torch.empty(num_experts, M, N, device=a.device, dtype=torch.float32)
        accumulate = False
    _launch(name, 1, "b200moe_expert_wgrad_segments", _p(a), M, _p(b), N, _p(seg_offsets),
            seg_offsets.shape[0], num_experts, a.shape[0], _p(out), int(accumulate), _s(a))
    return out


# --------------------------------------------------------------------------- #
# fp8 expert path (spark-gpt --fp8-mlp, train.py:1301-1604)
# --------------------------------------------------------------------------- #
E4M3 = torch.float8_e4m3fn
E5M2 = torch.float8_e5m2
_FP8_FMT = {E4M3: 0, E5M2: 1}


def _check_fp8(t: torch.Tensor, name, dtypes=(E4M3, E5M2)):
    if not t.is_cuda:
        raise RuntimeError(f"{name}: the B200 MoE kernels need CUDA tensors (no CPU path)")
    if t.dtype not in dtypes:
        raise RuntimeError(f"{name}: expected one of {dtypes}, got {t.dtype}")
    if not t.is_contiguous():
        raise RuntimeError(f"{name}: expected a contiguous tensor")


def _check_scales(scale, amax=None):
    _check(scale, torch.float32, "fp8 scale")
    if scale.numel() < 5:
        raise RuntimeError("fp8 scale: expected the five per-site scales")
    if amax is not None:
        _check(amax, torch.float32, "fp8 amax")
        if amax.numel() < 5:
            raise RuntimeError("fp8 amax: expected the five amax slots")


def fp8_quantize_experts(w: torch.Tensor):
    """(e4m3 copy of w * q_e, q (E,) fp32) of fp32 (E, rows, cols) master
    weights, q_e = 2^floor(log2(448 / max|w_e|)) (train.py:1536-1540)."""
    w = w.detach().float().contiguous()
    E = w.shape[0]
    per = w[0].numel() if E else 0
    w8 = torch.empty(w.shape, device=w.device, dtype=E4M3)
    q = torch.empty(E, device=w.device, dtype=torch.float32)
    if E and per:
        nbytes = int(_lib.value("b200moe_fp8_quantize_experts_scratch_bytes", E))
        scratch = torch.empty(nbytes, device=w.device, dtype=torch.uint8)
        _launch("fp8_quantize", 3, "b200moe_fp8_quantize_experts", _p(w), E, per, _p(w8), _p(q),
                _p(scratch), nbytes, _s(w))
    return w8, q


def fp8_gather_quant(x: torch.Tensor, d: Dispatch, scale, amax) -> torch.Tensor:
    """x8 (Rcap, H) e4m3 = e4m3(x[token] * scale[0]), padding rows zero; amax[0] raised."""
    _check(x, BF16, "fp8_gather_quant x")
    _check_scales(scale, amax)
    H = x.shape[1]
    x8 = torch.empty(d.rows_cap, H, device=x.device, dtype=E4M3)
    if d.num_tokens == 0:
        return x8.zero_()
    _launch("gather", 1, "b200moe_fp8_gather_quant", _p(x), _p(d.row_flat), _p(d.inv_pad),
            _p(d.pad_offsets), d.num_tokens, d.num_experts, d.top_k, H, d.rows_cap, _p(scale),
            _p(amax), _p(x8), _s(x))
    return x8


def fp8_quantize_rows(src: torch.Tensor, scale_slot: torch.Tensor, amax_slot: torch.Tensor,
                      dtype=E5M2, d: Dispatch | None = None) -> torch.Tensor:
    """fp8(src * scale_slot[0]) of a bf16 matrix, amax_slot[0] raised; with a
    Dispatch, only the rows below its padded total (the rest of a padded-row
    buffer holds no data and is left unwritten)."""
    _check(src, BF16, "fp8_quantize_rows src")
    dst = torch.empty(src.shape, device=src.device, dtype=dtype)
    rows, cols = src.shape
    total = None if d is None else d.pad_offsets[d.num_experts:]
    _launch("fp8_quantize_rows", 1, "b200moe_fp8_quantize_rows", _p(src), rows, cols, _p(total),
            _p(scale_slot), _p(amax_slot), _FP8_FMT[dtype], _p(dst), _s(src))
    return dst


def fp8_combine_bwd(d_out, y, d: Dispatch, weights, scale_slot, amax_slot):
    """combine_bwd that also returns dy8 = e5m2(dy * scale_slot[0]) (padding
    rows zero) and raises amax_slot[0] with max|dy| (one pass over dy)."""
    _check(d_out, BF16, "fp8_combine_bwd d_out")
    _check(weights, BF16, "fp8_combine_bwd weights")
    H = y.shape[1]
    if d.num_tokens == 0:
        return (torch.zeros(d.rows_cap, H, device=y.device, dtype=BF16),
                torch.zeros(0, d.top_k, device=y.device, dtype=torch.float32),
                torch.zeros(d.rows_cap, H, device=y.device, dtype=E5M2))
    dy = torch.empty(d.rows_cap, H, device=y.device, dtype=BF16)
    dy8 = torch.empty(d.rows_cap, H, device=y.device, dtype=E5M2)
    dw = torch.empty(d.num_tokens, d.top_k, device=y.device, dtype=torch.float32)
    _launch("combine_bwd", 1, "b200moe_fp8_combine_bwd", _p(d_out), _p(y), _p(d.row_flat),
            _p(d.inv_pad), _p(d.pad_offsets), _p(weights), d.num_experts, d.num_tokens,
            d.top_k, H, d.rows_cap, _p(scale_slot), _p(amax_slot), _p(dy), _p(dw), _p(dy8),
            _s(y))
    return dy, dw, dy8


def fp8_gate_up_fwd(x8, w8_gu, q_gu, d: Dispatch, scale, amax):
    """gu8 (Rcap, 2I), h8 (Rcap, I) e4m3 (train.py:1317-1354)."""
    _check_fp8(x8, "fp8_gate_up_fwd x8", (E4M3,))
    _check_fp8(w8_gu, "fp8_gate_up_fwd w8", (E4M3,))
    _check_scales(scale, amax)
    E, two_i, H = w8_gu.shape
    I = two_i // 2
    gu8 = torch.empty(d.rows_cap, two_i, device=x8.device, dtype=E4M3)
    h8 = torch.empty(d.rows_cap, I, device=x8.device, dtype=E4M3)
    _launch("gate_up_fwd", 1, "b200moe_fp8_expert_gate_up_fwd", _p(x8), _p(w8_gu), _p(q_gu),
            _p(d.tile_expert), _p(d.pad_offsets), d.rows_cap, E, H, I, _p(scale), _p(amax),
            _p(gu8), _p(h8), _s(x8))
    return gu8, h8


def fp8_down_fwd(h8, wd8, q_d, d: Dispatch, scale):
    """y (Rcap, H) bf16 = h8 . W8_d[e]^T / (scale[2] q_d[e]) (train.py:1357-1379)."""
    _check_fp8(h8, "fp8_down_fwd h8", (E4M3,))
    _check_fp8(wd8, "fp8_down_fwd w8", (E4M3,))
    _check_scales(scale)
    E, H, I = wd8.shape
    y = torch.empty(d.rows_cap, H, device=h8.device, dtype=BF16)
    _launch("down_fwd", 1, "b200moe_fp8_expert_down_fwd", _p(h8), _p(wd8), _p(q_d),
            _p(d.tile_expert), _p(d.pad_offsets), d.rows_cap, E, H, I, _p(scale), _p(y), _s(h8))
    return y


def fp8_down_dgrad_swiglu(dy, w_d, gu8, d: Dispatch, scale, amax):
    """d_gu8 (Rcap, 2I) e5m2 from bf16 dy and W_d (train.py:1382-1423)."""
    _check(dy, BF16, "fp8_down_dgrad dy")
    _check(w_d, BF16, "fp8_down_dgrad w")
    _check_fp8(gu8, "fp8_down_dgrad gu8", (E4M3,))
    _check_scales(scale, amax)
    E, H, I = w_d.shape
    d_gu8 = torch.empty(d.rows_cap, 2 * I, device=dy.device, dtype=E5M2)
    _launch("down_dgrad", 1, "b200moe_fp8_expert_down_dgrad_swiglu", _p(dy), _p(w_d), _p(gu8),
            _p(d.tile_expert), _p(d.pad_offsets), d.rows_cap, E, H, I, _p(scale), _p(amax),
            _p(d_gu8), _s(dy))
    return d_gu8


def fp8_gate_up_dgrad(d_gu8, w8_gu, q_gu, d: Dispatch, scale):
    """dxs (Rcap, H) bf16 = d_gu8 . W8_gu[e] / (scale[3] q_gu[e]) (train.py:1426-1448)."""
    _check_fp8(d_gu8, "fp8_gate_up_dgrad d_gu8", (E5M2,))
    _check_fp8(w8_gu, "fp8_gate_up_dgrad w8", (E4M3,))
    _check_scales(scale)
    E, two_i, H = w8_gu.shape
    dxs = torch.empty(d.rows_cap, H, device=d_gu8.device, dtype=BF16)
    _launch("gate_up_dgrad", 1, "b200moe_fp8_expert_gate_up_dgrad", _p(d_gu8), _p(w8_gu),
            _p(q_gu), _p(d.tile_expert), _p(d.pad_offsets), d.rows_cap, E, H, two_i // 2,
            _p(scale), _p(dxs), _s(d_gu8))
    return dxs


def fp8_wgrad(a8, b8, d: Dispatch, scale_a, scale_b, name="wgrad", out=None, accumulate=False):
    """(E, M, N) fp32 (+)= a8_e^T b8_e / (scale_a[0] scale_b[0]) over the padded
    rows of each expert (train.py:1451-1478, :1504-1530)."""
    _check_fp8(a8, f"{name} a8")
    _check_fp8(b8, f"{name} b8", (E4M3,))
    M, N = a8.shape[1], b8.shape[1]
    if out is None:
        out = torch.empty(d.num_experts, M, N, device=a8.device, dtype=torch.float32)
        accumulate = False
    _launch(name, 1, "b200moe_fp8_expert_wgrad", _p(a8), _FP8_FMT[a8.dtype], M, _p(b8), N,
            _p(d.pad_offsets), d.num_experts, d.rows_cap, _p(scale_a), _p(scale_b), _p(out),
            int(accumulate), _s(a8))
    return out


# --------------------------------------------------------------------------- #
# expert products with the row gather / combine backward fused in
# --------------------------------------------------------------------------- #
def gate_up_fwd_gather(x, w_gu, d: Dispatch):
    """gate_up fwd reading xs[p] = x[row_flat[p]/k] in the GEMM's loads."""
    _check(x, BF16, "gate_up_fwd_gather x")
    E, two_i, H = w_gu.shape
    I = two_i // 2
    gu = torch.empty(d.rows_cap, two_i, device=x.device, dtype=BF16)
    h = torch.empty(d.rows_cap, I, device=x.device, dtype=BF16)
    _launch("gate_up_fwd", 1, "b200moe_expert_gate_up_fwd_gather", _p(x), _p(d.row_flat),
            d.num_tokens, d.top_k, _p(w_gu), _p(d.tile_expert), _p(d.pad_offsets), d.rows_cap,
            E, H, I, _p(gu), _p(h), _s(x))
    return gu, h


def down_dgrad_combine(d_out, weights, w_d, gu, h, d: Dispatch):
    """Combine backward + down dgrad + SwiGLU backward -> (d_gu, w*h, d_weights (T,k))."""
    _check(d_out, BF16, "down_dgrad_combine d_out")
    _check(weights, BF16, "down_dgrad_combine weights")
    E, H, I = w_d.shape
    dev = d_out.device
    d_gu = torch.empty(d.rows_cap, 2 * I, device=dev, dtype=BF16)
    hw = torch.empty(d.rows_cap, I, device=dev, dtype=BF16)
    d_w = torch.empty(d.num_tokens, d.top_k, device=dev, dtype=torch.float32)
    nbytes = int(_lib.value("b200moe_down_dgrad_combine_scratch_bytes", d.rows_cap, I))
    scratch = torch.empty(nbytes, device=dev, dtype=torch.uint8)
    _launch("down_dgrad", 2, "b200moe_expert_down_dgrad_combine", _p(d_out), _p(d.row_flat),
            _p(weights), d.num_tokens, d.top_k, _p(w_d), _p(gu), _p(h), _p(d.tile_expert),
            _p(d.pad_offsets), d.rows_cap, E, H, I, _p(d_gu), _p(hw), _p(d_w), _p(scratch),
            nbytes, _s(d_out))
    return d_gu, hw, d_w


def wgrad_gather_b(a, x, d: Dispatch, name="wgrad", out=None, accumulate=False):
    """(E, M, N) fp32: a_e^T x[tokens of expert e]."""
    M, N = a.shape[1], x.shape[1]
    if out is None:
        out = torch.empty(d.num_experts, M, N, device=a.device, dtype=torch.float32)
        accumulate = False
    _launch(name, 1, "b200moe_expert_wgrad_gather_b", _p(a), M, _p(x), N, _p(d.row_flat),
            d.num_tokens, d.top_k, _p(d.pad_offsets), d.num_experts, d.rows_cap, _p(out),
            int(accumulate), _s(a))
    return out


def wgrad_gather_a(src, b, d: Dispatch, name="wgrad", out=None, accumulate=False):
    """(E, M, N) fp32: src[tokens of expert e]^T b_e."""
    M, N = src.shape[1], b.shape[1]
    if out is None:
        out = torch.empty(d.num_experts, M, N, device=b.device, dtype=torch.float32)
        accumulate = False
    _launch(name, 1, "b200moe_expert_wgrad_gather_a", _p(src), M, _p(d.row_flat), d.num_tokens,
            d.top_k, _p(b), N, _p(d.pad_offsets), d.num_experts, d.rows_cap, _p(out),
            int(accumulate), _s(b))
    return out


# --------------------------------------------------------------------------- #
# expert parallel: send plan, slot words, routing-weight gradient
# --------------------------------------------------------------------------- #
def ep_route(selected: torch.Tensor, experts_per_rank: int, ranks: int):
    """dest (T, P) int64 (r or -1 per destination rank) and the routed slots
    per destination rank (P,) int32."""
    _check(selected, torch.int64, "ep_route selected")
    T, k = selected.shape
    dest = torch.empty(T, ranks, device=selected.device, dtype=torch.int64)
    slots = torch.empty(ranks, device=selected.device, dtype=torch.int32)
    if T == 0:
        return dest, slots.zero_()
    _launch("ep_route", 1, "b200moe_ep_route", _p(selected), T, k, experts_per_rank, ranks,
            _p(dest), _p(slots), _s(selected))
    return dest, slots


def ep_pack(selected, weights, send: Dispatch, experts_per_rank: int) -> torch.Tensor:
    """(send.rows_cap, k) int32 slot words of the send rows."""
    _check(weights, BF16, "ep_pack weights")
    k = selected.shape[1]
    if selected.shape[0] == 0:  # no rows to send: every slot word says "no expert"
        return torch.full((send.rows_cap, k), 0xFFFF, device=selected.device, dtype=torch.int32)
    meta = torch.empty(send.rows_cap, k, device=selected.device, dtype=torch.int32)
    _launch("ep_pack", 1, "b200moe_ep_pack", _p(selected), _p(weights), _p(send.row_flat),
            _p(send.pad_offsets), send.rows_cap, k, experts_per_rank, send.num_experts,
            _p(meta), _s(selected))
    return meta


def ep_unpack(meta: torch.Tensor):
    """slot words (n, k) -> local expert ids (n, k) int64 (-1: foreign) and bf16 weights."""
    _check(meta, torch.int32, "ep_unpack meta")
    n, k = meta.shape
    sel = torch.empty(n, k, device=meta.device, dtype=torch.int64)
    w = torch.empty(n, k, device=meta.device, dtype=BF16)
    if n:
        _launch("ep_unpack", 1, "b200moe_ep_unpack", _p(meta), n, k, _p(sel), _p(w), _s(meta))
    return sel, w


def ep_p2p_plan(counts: torch.Tensor, me: int, ranks: int) -> torch.Tensor:
    """counts (P, ld) int32 gathered on every rank -> this rank's plan (2 + 4P ints)."""
    plan = torch.empty(2 + 4 * ranks, device=counts.device, dtype=torch.int32)
    _launch("ep_p2p_plan", 1, "b200moe_ep_p2p_plan", _p(counts), counts.stride(0), me, ranks,
            _p(plan), _s(counts))
    return plan


def ep_p2p_send(src, send: Dispatch, plan, peer_rows, selected=None, weights=None,
                experts_per_rank: int = 1, peer_meta=None):
    """Store each token's row (and slot words) into the owners' receive buffers."""
    _check(src, BF16, "ep_p2p_send src")
    T, H = src.shape
    if T == 0:
        return
    k = selected.shape[1] if selected is not None else 0
    _launch("ep_p2p_send", 1, "b200moe_ep_p2p_send", _p(src), _p(send.inv_pad),
            _p(send.pad_offsets), _p(plan), _p(peer_rows), T, H, send.num_experts,
            _p(selected), _p(weights), k, experts_per_rank, _p(peer_meta), _s(src))


def ep_p2p_send_part(src, send: Dispatch, plan, peer_rows, me: int, dest_mode: int,
                     selected=None, weights=None, experts_per_rank: int = 1, peer_meta=None):
    """ep_p2p_send restricted to this rank's own rows (dest_mode 1) or to the
    other ranks' rows (dest_mode 2)."""
    _check(src, BF16, "ep_p2p_send_part src")
    T, H = src.shape
    if T == 0:
        return
    k = selected.shape[1] if selected is not None else 0
    _launch("ep_p2p_send", 1, "b200moe_ep_p2p_send_part", _p(src), _p(send.inv_pad),
            _p(send.pad_offsets), _p(plan), _p(peer_rows), T, H, send.num_experts,
            _p(selected), _p(weights), k, experts_per_rank, _p(peer_meta), me, dest_mode,
            _s(src))


def ep_p2p_reduce_return_src(rows, d: Dispatch, plan, peer_rows, ranks: int, src: int,
                             weights=None, dw_rows=None, peer_dw=None):
    """Owner side, one source's chunk: each of its rows' local-slot sum stored
    into the source's back rows (and the routing-weight gradients into its back dw)."""
    H = rows.shape[1]
    _launch("ep_p2p_reduce_return", 1, "b200moe_ep_p2p_reduce_return_src", _p(rows),
            _p(d.inv_pad), _p(weights), d.top_k, _p(dw_rows), _p(plan), _p(peer_rows),
            _p(peer_dw), d.num_tokens, src, H, ranks, _s(rows))


def ep_signal(peer_flags, phase: int, me: int, ranks: int, epoch: int, dest: int = -1):
    _launch("ep_signal", 1, "b200moe_ep_signal", _p(peer_flags), phase, me, ranks, dest,
            ctypes.c_ulonglong(epoch), _s(peer_flags))


def ep_wait(my_flags, phase: int, ranks: int, epoch: int, src: int = -1):
    _launch("ep_wait", 1, "b200moe_ep_wait", _p(my_flags), phase, src, ranks,
            ctypes.c_ulonglong(epoch), _s(my_flags))


def ep_p2p_return(rows, plan, peer_rows, ranks: int, dw_rows=None, peer_dw=None):
    """Store the owner's result rows (and routing-weight gradients) into the sources' back buffers."""
    _check(rows, BF16, "ep_p2p_return rows")
    n, H = rows.shape
    k = dw_rows.shape[1] if dw_rows is not None else 0
    if n == 0:
        return
    _launch("ep_p2p_return", 1, "b200moe_ep_p2p_return", _p(rows), _p(dw_rows), _p(plan),
            _p(peer_rows), _p(peer_dw), n, H, k, ranks, _s(rows))


def ep_p2p_reduce_return(rows, d: Dispatch, plan, peer_rows, ranks: int, weights=None,
                         dw_rows=None, peer_dw=None):
    """Owner side: each received row's sum over its local slots (weighted: the
    combine; unweighted: the gather backward) stored into the source's back rows."""
    H = rows.shape[1]
    _launch("ep_p2p_reduce_return", 1, "b200moe_ep_p2p_reduce_return", _p(rows), _p(d.inv_pad),
            _p(weights), d.top_k, _p(dw_rows), _p(plan), _p(peer_rows), _p(peer_dw),
            d.num_tokens, H, ranks, _s(rows))


def ep_p2p_back_inv(send: Dispatch, plan) -> torch.Tensor:
    T, P = send.num_tokens, send.num_experts
    inv = torch.empty(max(T * P, 1), device=plan.device, dtype=torch.int32)
    if T == 0:
        return inv[:0]
    _launch("ep_p2p_back_inv", 1, "b200moe_ep_p2p_back_inv", _p(send.inv_pad),
            _p(send.pad_offsets), _p(plan), T, P, _p(inv), _s(plan))
    return inv[: T * P]


def ep_barrier(peer_flags, my_flags, me: int, ranks: int, epoch: int):
    _launch("ep_barrier", 1, "b200moe_ep_barrier", _p(peer_flags), _p(my_flags), me, ranks,
            ctypes.c_ulonglong(epoch), _s(my_flags))


def ep_weight_grad(dw_rows, send: Dispatch, selected, experts_per_rank: int,
                   out=None) -> torch.Tensor:
    T, k = selected.shape
    d_w = torch.empty(T, k, device=selected.device, dtype=torch.float32) if out is None else out
    if T:
        _launch("ep_weight_grad", 1, "b200moe_ep_weight_grad", _p(dw_rows), _p(send.inv_pad),
                _p(selected), T, k, experts_per_rank, send.num_experts, _p(d_w), _s(selected))
    return d_w


# --------------------------------------------------------------------------- #
# load-balancing loss (train.py:3098-3197)
# --------------------------------------------------------------------------- #
def lb_stats(logits, selected, valid_u8, num_experts, top_k, packed):
    T = logits.shape[0]
    nbytes = int(_lib.value("b200moe_lb_scratch_bytes", T, num_experts))
    scratch = torch.empty(nbytes, device=logits.device, dtype=torch.uint8)
    if T:
        _launch("lb_stats", 3, "b200moe_lb_stats", _p(logits), logits.stride(0), _p(selected),
                _p(valid_u8), T, num_experts, top_k, _p(packed), _p(scratch), nbytes,
                _s(logits))
    return packed


def lb_finalize(packed, num_experts, top_k, world):
    dev = packed.device
    aux = torch.empty((), device=dev, dtype=torch.float32)
    stats = torch.empty(5, device=dev, dtype=torch.float32)
    coef = torch.empty(num_experts, device=dev, dtype=torch.float32)
    _launch("lb_finalize", 1, "b200moe_lb_finalize", _p(packed), num_experts, top_k, world,
            _p(aux), _p(stats), _p(coef), _s(packed))
    return aux, stats, coef


def lb_grad(logits, valid_u8, coef, grad, num_experts):
    T, ld = logits.shape[0], logits.stride(0)
    out = torch.empty(T, ld, device=logits.device, dtype=BF16)
    if T:
        _launch("lb_grad", 1, "b200moe_lb_grad", _p(logits), ld, _p(valid_u8), T, num_experts,
                _p(coef), _p(grad), _p(out), _s(logits))
    return out
