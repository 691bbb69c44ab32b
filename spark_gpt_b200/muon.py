"""Muon step for the packed 3-D expert weights on B200.

spark-gpt's optimizer (MuonAdamWHybrid, train.py:2930-3024) puts every
``experts.gate_up_proj`` (E,2I,H) and ``experts.down_proj`` (E,H,I) into its
Muon group (build_optimizer, train.py:3066-3070).  For each such tensor one
step is

    v <- lerp(v, g, 1 - m);  u = lerp(g, v, m) (nesterov) or v, as bf16
    X  = Newton-Schulz_5(u) per expert matrix (transposed when rows > cols)
    p <- p - lr * max(1, rows/cols)^0.5 * X

Here the momentum stage is one fused HBM pass, and the five Newton-Schulz
iterations run as grouped tcgen05 GEMMs over the E matrices of the tensor
(libb200moe.so: b200moe_muon_momentum, b200moe_newton_schulz), with the last
product applied straight to the fp32 parameter.

``muon_step_packed`` is the drop-in for the 3-D shapes of ``_muon_group``;
``PackedExpertMuon`` wraps it as a torch optimizer for parameter groups that
hold only packed expert tensors.  Shapes: rows and cols multiples of 128.
"""

from __future__ import annotations

import ctypes

import torch

from . import _lib, faults
from .ops import _launch, _p, _s

NS_COEFFS = (3.4445, -4.7750, 2.0315)  # train.py:2899


def momentum_stage(grad: torch.Tensor, buf: torch.Tensor, momentum: float,
                   nesterov: bool = True, out: torch.Tensor | None = None) -> torch.Tensor:
    """Update the fp32 momentum buffer in place; return the bf16 staged update."""
    for t, name in ((grad, "grad"), (buf, "momentum buffer")):
        if not t.is_cuda or t.dtype != torch.float32 or not t.is_contiguous():
            raise RuntimeError(f"momentum_stage: {name} must be a contiguous fp32 CUDA tensor")
    if out is None:
        out = torch.empty(grad.shape, device=grad.device, dtype=torch.bfloat16)
    _launch("muon_momentum", 1, "b200moe_muon_momentum", _p(grad), _p(buf), _p(out),
            grad.numel(), ctypes.c_double(momentum), int(nesterov), _s(grad))
    return out


def newton_schulz(x: torch.Tensor, steps: int = 5, update: torch.Tensor | None = None,
                  neg_lr: float = 0.0) -> torch.Tensor | None:
    """Orthogonalise each matrix of x (B, rows, cols) bf16 (x is consumed).

    Returns the bf16 result, or, with `update` (B, rows, cols) fp32, applies
    update += neg_lr * result in the last product and returns None."""
    if not x.is_cuda or x.dtype != torch.bfloat16 or not x.is_contiguous() or x.dim() != 3:
        raise RuntimeError("newton_schulz: x must be a contiguous (B, rows, cols) bf16 CUDA tensor")
    B, rows, cols = x.shape
    if update is not None and (update.shape != x.shape or update.dtype != torch.float32
                               or not update.is_contiguous()):
        raise RuntimeError("newton_schulz: update must be a contiguous fp32 tensor shaped like x")
    nbytes = int(_lib.value("b200moe_newton_schulz_scratch_bytes", B, rows, cols))
    scratch = torch.empty(max(nbytes, 16), device=x.device, dtype=torch.uint8)
    out = None if update is not None else torch.empty_like(x)
    a, b, c = NS_COEFFS
    _launch("newton_schulz", 4 + 3 * steps, "b200moe_newton_schulz", _p(x), B, rows, cols, steps,
            ctypes.c_float(a), ctypes.c_float(b), ctypes.c_float(c), _p(out), _p(update),
            ctypes.c_float(neg_lr), _p(scratch), nbytes, _s(x))
    return out


_SIDE_STREAMS: dict = {}


def _side_stream(dev: torch.device, i: int) -> torch.cuda.Stream:
    key = (dev.index, i)
    if key not in _SIDE_STREAMS:
        _SIDE_STREAMS[key] = torch.cuda.Stream(dev)
    return _SIDE_STREAMS[key]


@torch.no_grad()
def muon_step_packed(params, momentum_buffers, lr: float, momentum: float = 0.95,
                     nesterov: bool = True, ns_steps: int = 5, streams: int = 2) -> None:
    """One Muon step of packed 3-D fp32 parameters with .grad set
    (MuonAdamWHybrid._muon_group, train.py:2972-3024, for 3-D tensors).

    momentum_buffers: one fp32 tensor per parameter (zeros at the first step),
    updated in place.  The parameters' updates are independent, so they run on
    `streams` CUDA streams in turn (the caller's and side streams that start
    after the caller's pending work and that the caller's stream waits for on
    return): one tensor's short Newton-Schulz products fill the SMs that
    another's leave idle at the end of each launch."""
    todo = [(p, v) for p, v in zip(params, momentum_buffers) if p.grad is not None]
    if not todo:
        return
    for p, _ in todo:
        if (not p.is_cuda or p.dim() != 3 or p.dtype != torch.float32
                or not p.is_contiguous()):
            raise RuntimeError("muon_step_packed: parameters must be contiguous fp32 "
                               "(E, rows, cols) CUDA tensors")
    dev = todo[0][0].device
    faults.raise_pending(dev)
    main = torch.cuda.current_stream(dev)
    lanes = [main] + [_side_stream(dev, i) for i in range(max(1, min(streams, len(todo))) - 1)]
    for s in lanes[1:]:
        s.wait_stream(main)  # the gradients and parameters are ready
    for i, (p, v) in enumerate(todo):
        with torch.cuda.stream(lanes[i % len(lanes)]):
            g = p.grad.float().contiguous()
            staged = momentum_stage(g, v, momentum, nesterov)
            rows, cols = p.shape[-2], p.shape[-1]
            lr_eff = lr * max(1, rows / cols) ** 0.5
            newton_schulz(staged, ns_steps, update=p.data, neg_lr=-lr_eff)
    for s in lanes[1:]:
        main.wait_stream(s)
    faults.snapshot(dev)


class PackedExpertMuon(torch.optim.Optimizer):
    """Muon over packed expert tensors only (a Muon param group of
    build_optimizer, train.py:3066-3070, whose members are all 3-D)."""

    def __init__(self, params, lr=0.02, momentum=0.95, nesterov=True, ns_steps=5, streams=2):
        super().__init__(params, dict(lr=lr, momentum=momentum, nesterov=nesterov,
                                      ns_steps=ns_steps))
        self.streams = streams

    @torch.no_grad()
    def step(self, closure=None):
        loss = None
        if closure is not None:
            with torch.enable_grad():
                loss = closure()
        for group in self.param_groups:
            params = [p for p in group["params"] if p.grad is not None]
            bufs = []
            for p in params:
                st = self.state[p]
                if "v" not in st:
                    st["v"] = torch.zeros_like(p, dtype=torch.float32)
                bufs.append(st["v"])
            muon_step_packed(params, bufs, group["lr"], group["momentum"], group["nesterov"],
                             group["ns_steps"], self.streams)
        return loss
