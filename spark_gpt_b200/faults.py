"""Device faults surfaced on the layer's own path.

The library's kernels never trap.  A bounded wait that gives up (a GEMM
pipeline barrier, the expert-parallel rank barrier), an expert id outside
[0, E) or inconsistent sizes set a bit in a per-device fault word, and the
kernel returns early, leaving its outputs incomplete.  So that training does
not continue on such outputs:

* every layer call (forward and backward of SparseMoE, TopKRouter, Experts,
  ExpertParallelMoE, and each barrier phase of the latter; the Muon step)
  ends by queueing an asynchronous copy of that word into pinned host memory
  (``b200moe_fault_snapshot``: no host synchronisation);
* every layer call starts by reading the last copy that landed; a non-zero
  word raises :class:`DeviceFault` (a ``RuntimeError``) there, after clearing
  it, so a fault stops the step at most one layer call after it happened;
* :func:`check_faults` reads the word synchronously, for trainers that poll
  at log steps.

The reference's only failure signal on this path is a collective that times
out (``--ddp-timeout-seconds``, train.py:3561-3562, :3653-3656).
"""

from __future__ import annotations

import ctypes

import torch

from . import _lib

FAULT_BITS = {
    1: "a bounded device wait gave up (a GEMM pipeline barrier or the expert-parallel rank "
       "barrier: a peer rank that never arrived, or a stalled kernel)",
    2: "an expert id outside [0, num_experts)",
    4: "a kernel saw inconsistent sizes",
}


class DeviceFault(RuntimeError):
    """A kernel of the MoE library recorded a fault; its outputs are incomplete."""

    def __init__(self, word: int, device):
        self.word = word
        self.device = device
        why = "; ".join(msg for bit, msg in FAULT_BITS.items() if word & bit) or "unknown"
        super().__init__(f"spark_gpt_b200: device fault word 0x{word:x} on {device}: {why}")


class _Watch:
    """Pinned landing slot of one device's fault-word snapshots."""

    def __init__(self, device: torch.device):
        self.device = device
        self.host = torch.zeros(1, dtype=torch.int32).pin_memory()
        self.ptr = ctypes.c_void_p(self.host.data_ptr())


_WATCH: dict[int, _Watch] = {}


def _watch(device) -> _Watch:
    device = torch.device(device)
    idx = device.index if device.index is not None else torch.cuda.current_device()
    w = _WATCH.get(idx)
    if w is None:
        w = _WATCH[idx] = _Watch(torch.device("cuda", idx))
    return w


def _clear(w: _Watch) -> int:
    """Wait for the device, read and clear its fault word and the host slot."""
    torch.cuda.synchronize(w.device)
    with torch.cuda.device(w.device):
        word = _lib.read_fault()
    w.host.zero_()
    return word


def raise_pending(device) -> None:
    """Raise DeviceFault if the last snapshot that landed holds a fault.

    Reads pinned host memory only: no device synchronisation unless a fault
    is found (then the device is synchronised and its word cleared)."""
    w = _watch(device)
    seen = int(w.host[0])
    if seen:
        word = _clear(w) | seen
        raise DeviceFault(word, w.device)


def snapshot(device, stream=None) -> None:
    """Queue a copy of the device fault word into the host slot on `stream`
    (default: torch's current stream of `device`)."""
    w = _watch(device)
    if stream is None:
        stream = torch.cuda.current_stream(w.device)
    _lib.call("b200moe_fault_snapshot", w.ptr, ctypes.c_void_p(stream.cuda_stream))


def check_faults(device=None) -> None:
    """Synchronously read and clear the fault word of `device` (default: the
    current device); raise DeviceFault if it was set."""
    if device is None:
        device = torch.device("cuda", torch.cuda.current_device())
    w = _watch(device)
    word = _clear(w)
    if word:
        raise DeviceFault(word, w.device)
