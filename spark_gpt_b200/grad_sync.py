"""Data-parallel gradient all-reduce of a SparseMoE layer, overlapped with the
layer's own backward, and in-place gradient accumulation.

In the reference, DDP (train.py:3781) all-reduces every gradient, the expert
tensors included, bucket by bucket as autograd produces them.  This layer's
backward is one fused op, so DDP would only see its three weight gradients
once the whole op has finished.  GradSync takes them from inside the
backward instead:

* the three fp32 weight gradients are written straight into one flat buffer
  owned by GradSync (gate_up | down | router: the two expert gradients form
  one contiguous bucket), which becomes the parameters' ``.grad`` (as DDP's
  ``gradient_as_bucket_view``).  When ``.grad`` already is that buffer
  (micro-batches without ``zero_grad``), the weight-gradient GEMMs add into it
  in their epilogue instead of autograd adding a fresh tensor: no extra fp32
  pass over the expert gradients;
* as soon as both expert gradients are final -- the backward computes them
  before the gate_up dgrad -- their all-reduce (the average over the group,
  as DDP) starts on a side stream and runs beside the gate_up dgrad, the
  router backward and the row-gather backward; the persistent GEMM beside it
  leaves ``comm_sms`` SMs to the collective;
* the router gradient's all-reduce follows at the end of the backward;
* :meth:`GradSync.wait` (call it before ``optimizer.step()``) orders the
  current stream after both.

Inside :meth:`GradSync.no_sync` the backward accumulates locally and reduces
nothing; the first backward after it reduces the accumulated buffer (DDP's
``no_sync`` semantics).  With a world of one nothing is reduced: in-place
accumulation only.  When the rest of the model is wrapped in DDP, leave these
three parameters out of it (``model._ddp_params_and_buffers_to_ignore``).
Eager only: under ``torch.compile`` the layer keeps its custom-op path, whose
gradients DDP reduces after the op.
"""

from __future__ import annotations

from contextlib import contextmanager
from types import SimpleNamespace

import torch
import torch.distributed as dist

from . import ops


class GradSync:
    def __init__(self, layer, group=None, comm_sms: int = 16):
        self.layer = layer
        self.group = group
        self.world = dist.get_world_size(group) if dist.is_initialized() else 1
        self.comm_sms = int(comm_sms)
        self.params = [layer.experts.gate_up_proj, layer.experts.down_proj, layer.gate.weight]
        dev = self.params[0].device
        sizes = [p.numel() for p in self.params]
        self.flat = torch.zeros(sum(sizes), dtype=torch.float32, device=dev)
        self.views, off = [], 0
        for p, n in zip(self.params, sizes):
            self.views.append(self.flat[off:off + n].view(p.shape))
            off += n
        self.expert_bucket = self.flat[: sizes[0] + sizes[1]]
        self.router_bucket = self.views[2].view(-1)
        self._reduce = True
        self._works = []
        self._divide = []
        self._stream = torch.cuda.Stream(dev) if dev.type == "cuda" else None
        backend = dist.get_backend(group) if dist.is_initialized() else None
        self._avg_in_collective = backend == "nccl"
        layer._grad_sync = self

    # ------------------------------------------------------------------ #
    # user API
    # ------------------------------------------------------------------ #
    @contextmanager
    def no_sync(self):
        """Backward passes inside accumulate locally and reduce nothing."""
        prev, self._reduce = self._reduce, False
        try:
            yield
        finally:
            self._reduce = prev

    def wait(self) -> None:
        """Make the current stream wait for the started all-reduces (and scale
        the sums on backends without an averaging collective)."""
        for w in self._works:
            w.wait()
        self._works.clear()
        for t in self._divide:
            t.div_(self.world)
        self._divide.clear()

    def detach(self) -> None:
        """Return the layer to its plain path (gradients from autograd)."""
        self.wait()
        if getattr(self.layer, "_grad_sync", None) is self:
            self.layer._grad_sync = None

    # ------------------------------------------------------------------ #
    # called by the layer's backward
    # ------------------------------------------------------------------ #
    def begin(self) -> SimpleNamespace:
        """Destinations of this backward's weight gradients: write when .grad
        is None (it becomes the buffer view), add when .grad is the view."""
        self.wait()  # a reduction still in flight from an earlier backward
        acc = []
        for p, v in zip(self.params, self.views):
            if p.grad is None:
                p.grad = v
                acc.append(False)
            elif p.grad.data_ptr() == v.data_ptr() and p.grad.shape == v.shape:
                acc.append(True)
            else:
                raise RuntimeError("GradSync: a parameter's .grad was replaced by another tensor; "
                                   "call optimizer.zero_grad(set_to_none=True) or detach() first")
        return SimpleNamespace(gate_up=self.views[0], down=self.views[1], router=self.views[2],
                               accumulate=(acc[2], acc[0], acc[1]),
                               experts_ready=self._experts_ready,
                               router_ready=self._router_ready)

    def _start(self, bucket) -> None:
        if not self._reduce or self.world == 1:
            return
        op = dist.ReduceOp.AVG if self._avg_in_collective else dist.ReduceOp.SUM
        if self._stream is not None:
            self._stream.wait_stream(torch.cuda.current_stream(bucket.device))
            with torch.cuda.stream(self._stream):
                self._works.append(dist.all_reduce(bucket, op=op, group=self.group,
                                                   async_op=True))
        else:
            self._works.append(dist.all_reduce(bucket, op=op, group=self.group, async_op=True))
        if not self._avg_in_collective:
            self._divide.append(bucket)

    def _experts_ready(self):
        self._start(self.expert_bucket)
        if self._works and self.comm_sms and self._stream is not None:
            sms = torch.cuda.get_device_properties(self.flat.device).multi_processor_count
            return ops.persistent_sm_limit(max(2, sms - self.comm_sms))
        return None

    def _router_ready(self) -> None:
        self._start(self.router_bucket)
