"""ctypes binding of libb200moe.so (the C ABI in include/b200moe.h).

This is the binding a Python caller (such as spark-gpt's train.py) uses: every
entry point takes raw device pointers, sizes and a cudaStream_t and returns an
int status.  A non-zero status raises RuntimeError carrying
``b200moe_last_error()``.  There is no CPU fallback: if the library is missing
the first call raises.
"""

from __future__ import annotations

import ctypes
from ctypes import c_double, c_float, c_int, c_longlong, c_uint, c_ulonglong, c_void_p, c_char_p, POINTER
from pathlib import Path

LIB_PATH = Path(__file__).resolve().parent / "libb200moe.so"

P = c_void_p
I = c_int
L = c_longlong

# name -> (restype, argtypes); mirrors include/b200moe.h
PROTOTYPES = {
    "b200moe_version": (I, []),
    "b200moe_last_error": (c_char_p, []),
    "b200moe_set_pair_gemm": (I, [I]),
    "b200moe_set_persistent_sm_limit": (I, [I]),
    "b200moe_set_transfer_sm_limit": (I, [I]),
    "b200moe_fault_read_and_clear": (I, [POINTER(c_uint)]),
    "b200moe_fault_snapshot": (I, [P, P]),
    "b200moe_padded_rows": (L, [L, I]),
    "b200moe_router_width": (I, [I]),
    "b200moe_cast_f32_to_bf16": (I, [P, L, L, L, P, P]),
    "b200moe_router_logits": (I, [P, P, L, I, I, P, P]),
    "b200moe_router_topk_fwd": (I, [P, I, L, L, I, I, I, P, P, P]),
    "b200moe_router_topk_bwd": (I, [P, L, P, P, P, L, I, I, I, P, P]),
    "b200moe_router_dgrad": (I, [P, P, L, I, I, P, P]),
    "b200moe_router_wgrad_scratch_bytes": (L, [L, I, I]),
    "b200moe_router_wgrad": (I, [P, P, L, I, I, I, P, I, P, L, P]),
    "b200moe_dispatch_scratch_bytes": (L, [L, I, I]),
    "b200moe_dispatch": (I, [P, L, I, I, P, P, P, P, P, P, P, L, P]),
    "b200moe_dispatch_noalloc": (I, [P, L, I, I, P, P, P, P, P, P, P]),
    "b200moe_gather_rows": (I, [P, P, P, P, L, I, I, I, L, P, P]),
    "b200moe_gather_rows_bwd": (I, [P, P, P, L, I, I, I, P, P]),
    "b200moe_combine_fwd": (I, [P, P, P, L, I, I, I, P, P]),
    "b200moe_rmsnorm_fwd": (I, [P, P, L, I, c_float, P, P, P]),
    "b200moe_gather_rows_bwd_rmsnorm_scratch_bytes": (L, [L, I]),
    "b200moe_gather_rows_bwd_rmsnorm": (I, [P, P, P, P, P, P, L, I, I, I, P, P, P, L, P]),
    "b200moe_combine_bwd": (I, [P, P, P, P, P, P, I, L, I, I, L, I, P, P, P]),
    "b200moe_expert_gate_up_fwd": (I, [P, P, P, P, L, I, I, I, P, P, P]),
    "b200moe_expert_down_fwd": (I, [P, P, P, P, P, L, I, I, I, P, P]),
    "b200moe_expert_down_dgrad_swiglu": (I, [P, P, P, P, P, L, I, I, I, P, P]),
    "b200moe_expert_gate_up_dgrad": (I, [P, P, P, P, P, L, I, I, I, P, P]),
    "b200moe_expert_wgrad": (I, [P, I, P, I, P, I, L, P, I, P]),
    "b200moe_expert_wgrad_segments": (I, [P, I, P, I, P, I, I, L, P, I, P]),
    "b200moe_fp8_quantize_experts_scratch_bytes": (L, [I]),
    "b200moe_fp8_quantize_experts": (I, [P, I, L, P, P, P, L, P]),
    "b200moe_fp8_gather_quant": (I, [P, P, P, P, L, I, I, I, L, P, P, P, P]),
    "b200moe_fp8_quantize_rows": (I, [P, L, I, P, P, P, I, P, P]),
    "b200moe_fp8_combine_bwd": (I, [P, P, P, P, P, P, I, L, I, I, L, P, P, P, P, P, P]),
    "b200moe_fp8_expert_gate_up_fwd": (I, [P, P, P, P, P, L, I, I, I, P, P, P, P, P]),
    "b200moe_fp8_expert_down_fwd": (I, [P, P, P, P, P, L, I, I, I, P, P, P]),
    "b200moe_fp8_expert_down_dgrad_swiglu": (I, [P, P, P, P, P, L, I, I, I, P, P, P, P]),
    "b200moe_fp8_expert_gate_up_dgrad": (I, [P, P, P, P, P, L, I, I, I, P, P, P]),
    "b200moe_fp8_expert_wgrad": (I, [P, I, I, P, I, P, I, L, P, P, P, I, P]),
    "b200moe_expert_gate_up_fwd_gather": (I, [P, P, L, I, P, P, P, L, I, I, I, P, P, P]),
    "b200moe_down_dgrad_combine_scratch_bytes": (L, [L, I]),
    "b200moe_expert_down_dgrad_combine": (I, [P, P, P, L, I, P, P, P, P, P, L, I, I, I, P, P, P,
                                              P, L, P]),
    "b200moe_expert_wgrad_gather_b": (I, [P, I, P, I, P, L, I, P, I, L, P, I, P]),
    "b200moe_expert_wgrad_gather_a": (I, [P, I, P, L, I, P, I, P, I, L, P, I, P]),
    "b200moe_ep_route": (I, [P, L, I, I, I, P, P, P]),
    "b200moe_ep_pack": (I, [P, P, P, P, L, I, I, I, P, P]),
    "b200moe_ep_unpack": (I, [P, L, I, P, P, P]),
    "b200moe_ep_weight_grad": (I, [P, P, P, L, I, I, I, P, P]),
    "b200moe_ep_p2p_plan": (I, [P, I, I, I, P, P]),
    "b200moe_ep_p2p_send": (I, [P, P, P, P, P, L, I, I, P, P, I, I, P, P]),
    "b200moe_ep_p2p_return": (I, [P, P, P, P, P, L, I, I, I, P]),
    "b200moe_ep_p2p_reduce_return": (I, [P, P, P, I, P, P, P, P, L, I, I, P]),
    "b200moe_ep_p2p_back_inv": (I, [P, P, P, L, I, P, P]),
    "b200moe_ep_barrier": (I, [P, P, I, I, c_ulonglong, P]),
    "b200moe_ep_p2p_send_part": (I, [P, P, P, P, P, L, I, I, P, P, I, I, P, I, I, P]),
    "b200moe_ep_p2p_reduce_return_src": (I, [P, P, P, I, P, P, P, P, L, I, I, I, P]),
    "b200moe_ep_signal": (I, [P, I, I, I, I, c_ulonglong, P]),
    "b200moe_ep_wait": (I, [P, I, I, I, c_ulonglong, P]),
    "b200moe_muon_momentum": (I, [P, P, P, L, c_double, I, P]),
    "b200moe_newton_schulz_scratch_bytes": (L, [I, I, I]),
    "b200moe_newton_schulz": (I, [P, I, I, I, I, c_float, c_float, c_float, P, P, c_float, P, L,
                                  P]),
    "b200moe_lb_scratch_bytes": (L, [L, I]),
    "b200moe_lb_stats": (I, [P, L, P, P, L, I, I, P, P, L, P]),
    "b200moe_lb_finalize": (I, [P, I, I, I, P, P, P, P]),
    "b200moe_lb_grad": (I, [P, L, P, L, I, P, P, P, P]),
}

_lib = None


def load(path: Path | str | None = None) -> ctypes.CDLL:
    """Load the library once and attach the prototypes."""
    global _lib
    if _lib is not None and path is None:
        return _lib
    p = Path(path) if path is not None else LIB_PATH
    if not p.exists():
        raise RuntimeError(
            f"{p} is missing: build it with `python -m spark_gpt_b200.build` "
            "(the B200 MoE layer has no CPU fallback)")
    lib = ctypes.CDLL(str(p))
    for name, (res, args) in PROTOTYPES.items():
        fn = getattr(lib, name)
        fn.restype = res
        fn.argtypes = args
    if path is None:
        _lib = lib
    return lib


def call(name: str, *args) -> int:
    """Call an int-status entry point; raise RuntimeError on failure."""
    lib = load()
    rc = getattr(lib, name)(*args)
    if rc != 0:
        msg = lib.b200moe_last_error().decode(errors="replace")
        raise RuntimeError(f"{name} failed ({rc}): {msg}")
    return rc


def value(name: str, *args):
    """Call a value-returning helper (sizes, widths)."""
    return getattr(load(), name)(*args)


def read_fault() -> int:
    """Read and clear the device fault word (bounded waits that gave up,
    out-of-range expert ids)."""
    v = c_uint(0)
    call("b200moe_fault_read_and_clear", ctypes.byref(v))
    return int(v.value)
