"""Shared helpers for the parity tests.

Error measures (used with the bf16 tolerance of the layer contract):
  max_rel  = max|a - b| / max|b|
  mean_rel = mean|a - b| / max|b|
Both are normalised by the reference tensor's scale (its largest magnitude),
as spark-gpt's own fused-SwiGLU test does (tests/test_moe.py:418-421), so that
near-zero entries do not dominate.  ``elem_rel`` (mean|a-b| / mean|b|) is
reported for information.
"""

from __future__ import annotations

import numpy as np
import torch

MAX_REL = 2e-2
MEAN_REL = 2e-3


def rel_errors(a: torch.Tensor, b: torch.Tensor):
    """In float64, on b's device (full-size cases compare on the GPU)."""
    b = b.detach().double()
    a = a.detach().double().to(b.device)
    diff = (a - b).abs()
    scale = b.abs().max().clamp_min(1e-30)
    return {
        "max_rel": float(diff.max() / scale) if diff.numel() else 0.0,
        "mean_rel": float(diff.mean() / scale) if diff.numel() else 0.0,
        "elem_rel": float(diff.mean() / b.abs().mean().clamp_min(1e-30)) if diff.numel() else 0.0,
    }


def assert_bf16_close(a, b, name="", max_rel=MAX_REL, mean_rel=MEAN_REL):
    e = rel_errors(a, b)
    assert e["max_rel"] <= max_rel and e["mean_rel"] <= mean_rel, f"{name}: {e}"
    return e


def unpadded_permutation(row_flat: torch.Tensor, pad_offsets: torch.Tensor):
    """Sorted-row -> flat-slot permutation with the padding rows removed."""
    rf = row_flat[: int(pad_offsets[-1])].cpu().numpy()
    return rf[rf >= 0].astype(np.int64)


def bf16_round(t: torch.Tensor) -> torch.Tensor:
    return t.to(torch.bfloat16).float()
