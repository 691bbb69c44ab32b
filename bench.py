#!/usr/bin/env python
"""MoE-layer forward+backward throughput on B200 (BASELINE.json metric).

    python bench.py [--gpus N] [--steps K] [--warmup W] [--config cfg2|cfg3|cfg4|cfg5]
                    [--impl b200|reference]

One step = forward of spark_gpt_b200.SparseMoE on T tokens, the global
load-balancing loss (its 2E+2 all-reduce when N > 1), and the backward of
(out . d_out + 1e-3 * aux) into x and all three fp32 master parameters, with
the fp32 -> bf16 weight casts inside the step as in the reference
(train.py:2306-2309).  N > 1 runs the reference's data-parallel layout, one
rank per GPU under torchrun, T tokens per GPU (weak scaling): experts
replicated, the load-balance counts all-reduced, and the layer's fp32 weight
gradients averaged over the ranks as DDP does (train.py:3781), the expert
gradients' all-reduce started inside the backward (grad_sync.py).

Default workload: BASELINE config 2 (hidden 1024, 64 experts, top-8,
moe_intermediate 256, 65,536 tokens per GPU, near-uniform routing).  The
line also carries, measured in the same run:
  * roofline: the dominant GEMM's algorithmic TFLOP/s over the measured burst
    bf16 peak; gemms / hbm_kernels: every GEMM's and every HBM-bound kernel's
    achieved rate against the tensor peak and the measured copy bandwidth;
  * e2e: the reference arm's training step with x copied from pinned host
    memory every step and the loss read back, with a per-phase breakdown;
  * muon_step: the Muon optimizer step of the packed expert tensors;
  * configs (N = 1): BASELINE configs[2] (cfg3: H2048/E128/I768, Zipf-skewed
    routing) and the MoE layer of configs[3] (cfg4: H768/E32/k4/I384), each
    with its GEMM roofline and its rows per expert;
  * ep: BASELINE configs[4] (cfg5) at this N -- the single-GPU layer at its
    per-GPU shape, and at N > 1 the expert-parallel layer with the
    peer-memory and the NCCL transports, with per-phase times and the
    efficiency against the single-GPU layer;
  * torch_gpu_path (N = 1): the reference's own GPU path with FUSED_SWIGLU
    off (F.grouped_mm) restated in stock torch ops, timed on the same GPU
    with its agreement against this layer, plus cuBLAS on dense GEMMs of the
    expert GEMMs' shapes (the library's rate for those M/N/K);
  * fp8 (N = 1): the same step with the experts on the fp8 path
    (spark-gpt --fp8-mlp), after a prewarm step and a scale update.

--impl reference times the reference's CPU path (the oracle port of
train.py's torch MoE path, fp32) on the host cores on a bounded token sample
of the same shapes; rank 0 alone runs it.  Its step is the forward, the
load-balancing loss and the backward of out . g + 1e-3 * aux for a fixed
upstream gradient g (the MoE work of one training step).
"""

from __future__ import annotations

import argparse
import contextlib
import json
import math
import os
import statistics
import subprocess
import sys
import threading
import time
from datetime import timedelta
from pathlib import Path
from types import SimpleNamespace

import torch

ROOT = Path(__file__).resolve().parent
sys.path.insert(0, str(ROOT))

METRIC = "MoE-layer fwd+bwd tokens/s/GPU and % BF16 tensor peak at 1/2/4/8 B200"
CONFIGS = {
    "cfg2": dict(T=65536, H=1024, E=64, k=8, I=256, routing="near-uniform"),
    "cfg3": dict(T=16384, H=2048, E=128, k=8, I=768, routing="zipf1.1"),
    # the MoE layer of BASELINE config 4's 12-layer model at its 65,536-token batch
    "cfg4": dict(T=65536, H=768, E=32, k=4, I=384, routing="near-uniform"),
    # experts sharded over the GPUs (expert parallel)
    "cfg5": dict(T=32768, H=2048, E=128, k=8, I=768, routing="near-uniform", ep=True),
    "cfg5z": dict(T=32768, H=2048, E=128, k=8, I=768, routing="zipf1.1", ep=True),
}
CONFIG_INDEX = {"cfg2": 1, "cfg3": 2, "cfg4": 3, "cfg5": 4, "cfg5z": 4}
# Zipf(s=1.1) router bias scale for cfg3: max expert count ~8x the mean
# (calibrated once on seeded inputs with bf16 logits: max/mean = 8.02, min 247 rows).
ZIPF_ALPHA = 0.35
AUX_COEF = 1e-3


def parse_args():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=50)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--config", default="cfg2", choices=sorted(CONFIGS))
    ap.add_argument("--impl", default="b200", choices=["b200", "reference"])
    ap.add_argument("--cpu-sample-tokens", type=int, default=8192)
    ap.add_argument("--tokens", type=int, default=None,
                    help="override tokens per GPU (small cases for profiling only)")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--no-e2e", action="store_true")
    ap.add_argument("--no-muon", action="store_true",
                    help="skip the Muon optimizer-step measurement of the expert tensors")
    ap.add_argument("--ep-chunks", type=int, default=1,
                    help="expert parallel: token chunks pipelined against the exchanges")
    ap.add_argument("--transport", default="p2p", choices=["nccl", "p2p", "p2p_pipe"],
                    help="expert parallel: NCCL all-to-all, peer-memory stores with group "
                         "barriers, or peer-memory stores pipelined per source rank")
    ap.add_argument("--comm-sms", type=int, default=16,
                    help="SMs the persistent kernels leave to a transfer or collective "
                         "running beside them (expert-parallel exchanges, the data-parallel "
                         "gradient all-reduce; 0: none)")
    ap.add_argument("--no-grad-sync", action="store_true",
                    help="data parallel (N > 1): skip the gradient all-reduce of the layer's "
                         "weights (replicas only)")
    ap.add_argument("--no-extra", action="store_true",
                    help="N = 1: skip the cfg3 / cfg4 sub-blocks")
    ap.add_argument("--sub-steps", type=int, default=20,
                    help="timed steps of each cfg3 / cfg4 sub-block")
    ap.add_argument("--no-ep", action="store_true",
                    help="skip the expert-parallel (config 5) block")
    ap.add_argument("--ep-config", default="cfg5", choices=["cfg5", "cfg5z"],
                    help="expert-parallel block: uniform or Zipf-skewed routing")
    ap.add_argument("--ep-steps", type=int, default=20,
                    help="timed steps of each expert-parallel block measurement")
    ap.add_argument("--fp8", action="store_true",
                    help="N = 1: time the step with the experts on the fp8 path (spark-gpt "
                         "--fp8-mlp), after a prewarm step and a scale update (profiling runs "
                         "of the fp8 kernels; the default line is bf16)")
    return ap.parse_args()


def peaks():
    p = ROOT / "MEASURED_PEAKS.json"
    if p.exists():
        d = json.loads(p.read_text())
        return {"hbm_gbs": d["hbm_gbs"], "bf16": d["bf16_tflops"],
                "bf16_sustained": d["bf16_tflops_sustained"], "source": "measured"}
    return {"hbm_gbs": 6650.0, "bf16": 1590.0, "bf16_sustained": 1400.0, "source": "fallback"}


def gemm_flops(c, T):
    R = T * c["k"]
    H, I, E = c["H"], c["I"], c["E"]
    return {
        "gate_up_fwd": 4 * R * H * I, "down_fwd": 2 * R * H * I, "down_dgrad": 2 * R * H * I,
        "down_wgrad": 2 * R * H * I, "gate_up_dgrad": 4 * R * H * I,
        "gate_up_wgrad": 4 * R * H * I, "router_logits": 2 * T * H * E,
        "router_dgrad": 2 * T * H * E, "router_wgrad": 2 * T * H * E,
    }


def layer_flops(c, T):
    return 18 * c["H"] * c["I"] * c["k"] * T


# --------------------------------------------------------------------------- #
# inputs
# --------------------------------------------------------------------------- #
def zipf_bias(E, seed):
    g = torch.Generator().manual_seed(seed + 7)
    perm = torch.randperm(E, generator=g).float()
    return ZIPF_ALPHA * torch.log((perm + 1.0) ** -1.1)


def make_weights(c, seed):
    """muP init at base width 256 (train.py:2727-2739), 12-layer writer scale."""
    g = torch.Generator().manual_seed(seed)
    std_in = 0.02 / math.sqrt(c["H"] / 256)
    std_w = std_in / math.sqrt(2 * 12)
    w_r = torch.randn(c["E"], c["H"], generator=g) * 0.02
    w_gu = torch.randn(c["E"], 2 * c["I"], c["H"], generator=g) * std_in
    w_d = torch.randn(c["E"], c["H"], c["I"], generator=g) * std_w
    if c["routing"].startswith("zipf"):
        w_r[:, 0] = zipf_bias(c["E"], seed)
    return w_r, w_gu, w_d


def make_tokens(c, T, seed):
    g = torch.Generator().manual_seed(seed + 1)
    x = torch.randn(T, c["H"], generator=g)
    if c["routing"].startswith("zipf"):
        x[:, 0] = 1.0
    d_out = torch.randn(T, c["H"], generator=g) * 1e-2
    return x, d_out


# --------------------------------------------------------------------------- #
# clocks
# --------------------------------------------------------------------------- #
class ClockSampler:
    """SM clock and clock-event reasons sampled during the timed region: NVML
    every 20 ms (read-only queries), nvidia-smi at 200 ms if NVML is missing."""

    REASONS = {"hw_slowdown": 0x8, "hw_thermal_slowdown": 0x40,
               "sw_thermal_slowdown": 0x20, "sw_power_cap": 0x4}

    def __init__(self, device):
        self.device = device
        self.samples = []  # (sm_mhz, reasons bitmask)
        self.max_mhz = None
        self._stop = threading.Event()
        self._thread = None
        self._proc = None

    def _nvml_loop(self, nvml, h):
        while not self._stop.is_set():
            try:
                sm = nvml.nvmlDeviceGetClockInfo(h, nvml.NVML_CLOCK_SM)
                rs = nvml.nvmlDeviceGetCurrentClocksEventReasons(h)
                self.samples.append((float(sm), int(rs)))
            except Exception:  # noqa: BLE001 - sampling is best effort
                pass
            self._stop.wait(0.02)

    def _smi_loop(self):
        for line in self._proc.stdout:
            parts = [x.strip() for x in line.split(",")]
            try:
                mask = 0
                for name, bit in zip(["hw_slowdown", "hw_thermal_slowdown",
                                      "sw_thermal_slowdown", "sw_power_cap"], parts[2:6]):
                    if bit.lower() == "active":
                        mask |= self.REASONS[name]
                self.samples.append((float(parts[0]), mask))
                self.max_mhz = float(parts[1])
            except (ValueError, IndexError):
                continue

    def __enter__(self):
        try:
            import pynvml as nvml
            nvml.nvmlInit()
            pr = torch.cuda.get_device_properties(self.device)
            bus = f"{pr.pci_domain_id:08x}:{pr.pci_bus_id:02x}:{pr.pci_device_id:02x}.0"
            h = nvml.nvmlDeviceGetHandleByPciBusId(bus)
            self.max_mhz = float(nvml.nvmlDeviceGetMaxClockInfo(h, nvml.NVML_CLOCK_SM))
            self._thread = threading.Thread(target=self._nvml_loop, args=(nvml, h), daemon=True)
        except Exception:  # noqa: BLE001 - fall back to nvidia-smi
            try:
                self._proc = subprocess.Popen(
                    ["nvidia-smi", "-i", str(torch.cuda.current_device()),
                     "--query-gpu=clocks.sm,clocks.max.sm,clocks_event_reasons.hw_slowdown,"
                     "clocks_event_reasons.hw_thermal_slowdown,"
                     "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap",
                     "--format=csv,noheader,nounits", "-lms", "200"],
                    stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
                self._thread = threading.Thread(target=self._smi_loop, daemon=True)
            except (OSError, ValueError):
                self._thread = None
        if self._thread is not None:
            self._thread.start()
        return self

    def __exit__(self, *exc):
        self._stop.set()
        if self._proc is not None:
            self._proc.terminate()
            try:
                self._proc.wait(timeout=5)
            except subprocess.TimeoutExpired:
                self._proc.kill()
        if self._thread is not None:
            self._thread.join(timeout=5)

    def summary(self):
        if not self.samples:
            return {"sm_mhz": None, "sm_max_mhz": self.max_mhz, "reasons": [], "samples": 0}
        mask = 0
        for _, m in self.samples:
            mask |= m
        return {"sm_mhz": statistics.median(s for s, _ in self.samples),
                "sm_max_mhz": self.max_mhz,
                "reasons": sorted(n for n, bit in self.REASONS.items() if mask & bit),
                "samples": len(self.samples)}


# --------------------------------------------------------------------------- #
# CPU arm: the reference's torch MoE path restated in oracle/ (fp32, host cores)
# --------------------------------------------------------------------------- #
def cpu_layer_step(c, T, w, x, d_out):
    from oracle import moe_oracle as O
    w_r, w_gu, w_d = w
    logits = x @ w_r.t()
    _, sel = O.topk_cuda_order(O.softmax_fp32(logits), c["k"])
    valid = torch.ones(T, dtype=torch.bool)
    aux, _, g_aux = O.load_balancing_loss((logits,), (sel,), valid, num_experts=c["E"],
                                          top_k=c["k"])
    res = O.layer_forward_backward(x, w_r, w_gu, w_d, c["k"], d_out, logits=logits,
                                   d_logits_extra=AUX_COEF * g_aux[0])
    return float(aux) + float(res["out"][0, 0])


def cpu_throughput(c, T, steps, warmup):
    cores = os.cpu_count() or 1
    torch.set_num_threads(cores)
    w = make_weights(c, 0)
    x, d_out = make_tokens(c, T, 0)
    for _ in range(warmup):
        cpu_layer_step(c, T, w, x, d_out)
    t0 = time.perf_counter()
    for _ in range(steps):
        cpu_layer_step(c, T, w, x, d_out)
    dt = time.perf_counter() - t0
    return T * steps / dt, cores


def run_reference(args, c):
    rank = int(os.environ.get("RANK", "0"))
    if rank != 0:
        return
    T = args.cpu_sample_tokens
    steps = max(1, args.steps)
    warm = min(args.warmup, 1)
    v, cores = cpu_throughput(c, T, steps, warm)
    sample = (f"{T} tokens of {args.config} shapes per step (fp32 torch-CPU port of "
              f"train.py's torch MoE path, forward+aux+backward)")
    line = {
        "impl": "reference", "metric": METRIC, "value": v, "unit": "tokens/s",
        "n_gpus": args.gpus, "steps": steps, "warmup": warm, "ms_per_step": 1e3 * T / v,
        "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "f32",
        "data": "synthetic", "config": {**config_block(args, dict(c, T=T), args.gpus),
                                        "full_config_tokens_per_gpu": c["T"]},
        "cpu_baseline": {"value": v, "unit": "tokens/s", "cores": cores, "kind": "port",
                         "sample": sample},
        "e2e": {"value": v, "unit": "tokens/s", "h2d_bytes_per_step": 0,
                "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)


def config_block(args, c, n, grad_sync=False):
    if c.get("ep"):
        if n == 1:
            par = "ep1 = the single-GPU layer, all experts local (the scaling baseline)"
        elif args.transport == "p2p":
            par = (f"ep{n} (experts sharded, one row per (token, rank) stored into the owners' "
                   f"peer memory by the gather / combine kernels, bounded barriers)")
        elif args.transport == "p2p_pipe":
            par = (f"ep{n} (experts sharded, peer-memory stores pipelined per source rank: own "
                   f"rows first, transfers beside the experts, point-to-point flags)")
        else:
            par = (f"ep{n} (experts sharded, NCCL all_to_all, one row per (token, rank), "
                   f"{args.ep_chunks} token chunks overlapped, {args.comm_sms} SMs left to NCCL)")
    elif n > 1 and grad_sync:
        par = (f"dp{n} (replicated experts; the layer's fp32 weight gradients averaged over "
               f"the ranks with NCCL, started inside the backward as soon as the expert "
               f"gradients are final, as DDP does in the reference's step)")
    else:
        par = f"dp{n} (replicated experts)"
    return {"workload": f"{args.config}: single Qwen3-MoE layer fwd+bwd (BASELINE configs"
                        f"[{CONFIG_INDEX[args.config]}])",
            "tokens_per_gpu": c["T"], "global_batch": c["T"] * n, "hidden": c["H"],
            "experts": c["E"], "top_k": c["k"], "moe_intermediate": c["I"],
            "routing": c["routing"], "parallelism": par,
            "l2": "inputs larger than L2: each step streams ~10 GiB of activations"}


# --------------------------------------------------------------------------- #
# GPU arm
# --------------------------------------------------------------------------- #
ROW_KERNELS = ["gather", "combine", "combine_bwd", "gather_bwd", "dispatch", "router_topk",
               "router_topk_bwd", "cast", "lb_stats", "lb_grad", "lb_finalize"]
EP_KERNELS = ["ep_route", "ep_pack", "ep_unpack", "ep_weight_grad", "ep_p2p_send",
              "ep_p2p_reduce_return", "ep_barrier", "ep_p2p_plan", "ep_p2p_back_inv"]


def hbm_bytes(c, T):
    """Algorithmic bytes per launch of the HBM-bound kernels (each tensor read
    or written once; bf16 activations, int64 expert ids, fp32 routing-weight
    gradients).  W = router width (E padded to 64/128/256)."""
    R = T * c["k"]
    H, E, k = c["H"], c["E"], c["k"]
    W = 64 if E <= 64 else 128 if E <= 128 else 256
    return {
        "gather": T * H * 2 + R * H * 2,                      # x read, xs written
        "combine": R * H * 2 + R * 2 + T * H * 2,             # y, w read; out written
        "combine_bwd": T * H * 2 + R * H * 2 + R * H * 2 + R * 4,  # d_out, y; dy, d_w
        "gather_bwd": R * H * 2 + T * H * 2 + T * H * 2,      # dxs, addend; dx
        "router_logits": T * H * 2 + T * W * 2,               # x; logits
        "router_topk": T * W * 2 + T * k * 10,                # logits; ids, weights
        "router_topk_bwd": 2 * T * W * 2 + T * k * 12 + T * W * 2,  # logits, d_extra; d_logits
        "router_dgrad": T * W * 2 + T * H * 2,                # d_logits; dx_router
        "router_wgrad": T * H * 2 + T * W * 2,                # x, d_logits
        "lb_stats": T * W * 2 + T * k * 8 + T,                # logits, ids, mask
        "lb_grad": T * W * 2 + T * W * 2 + T,                 # logits; d_logits
        "dispatch": 2 * T * k * 8 + 3 * R * 4,                # ids (two passes); maps
    }


def layer_cfg(c):
    return SimpleNamespace(hidden_size=c["H"], num_experts=c["E"], num_experts_per_tok=c["k"],
                           moe_intermediate_size=c["I"], norm_topk_prob=True)


class Run:
    """One rank's view of the job: device, world, collectives over ranks."""

    def __init__(self):
        import torch.distributed as dist
        self.dist = dist
        self.world = int(os.environ.get("WORLD_SIZE", "1"))
        self.rank = int(os.environ.get("RANK", "0"))
        local = int(os.environ.get("LOCAL_RANK", "0"))
        torch.cuda.set_device(local)
        self.dev = torch.device("cuda", local)
        if self.world > 1:
            dist.init_process_group("nccl", timeout=timedelta(seconds=300), device_id=self.dev)

    def barrier(self):
        if self.world > 1:
            self.dist.barrier()

    def max(self, v):
        if self.world == 1:
            return v
        t = torch.tensor([v], device=self.dev, dtype=torch.float64)
        self.dist.all_reduce(t, op=self.dist.ReduceOp.MAX)
        return float(t)


def time_steps(run, step, steps, warmup, names, clocks=None):
    """W warm-up steps, then K timed steps between barriers and device syncs;
    CUDA events on the current stream (max over ranks) and per-op events."""
    from spark_gpt_b200 import ops
    for _ in range(warmup):
        step()
    torch.cuda.synchronize()
    timing = ops.set_timing(names)
    launches0 = ops.LAUNCHES["count"]
    run.barrier()
    torch.cuda.synchronize()
    ev0 = torch.cuda.Event(enable_timing=True)
    ev1 = torch.cuda.Event(enable_timing=True)
    ctx = ClockSampler(run.dev) if clocks is not None else contextlib.nullcontext()
    with ctx as sampler:
        ev0.record()
        for _ in range(steps):
            step()
        ev1.record()
        torch.cuda.synchronize()
    run.barrier()
    launches = ops.LAUNCHES["count"] - launches0
    ops.set_timing(None)
    if clocks is not None:
        clocks.update(sampler.summary())
    ms = run.max(ev0.elapsed_time(ev1)) / steps
    per_op, per_step = {}, {}
    for n, evs in timing.items():
        if evs:
            t = [s.elapsed_time(e) for s, e in evs]
            per_op[n] = sum(t) / len(t)          # ms per launch
            per_step[n] = sum(t) / steps          # ms per step
    return ms, per_op, per_step, launches


def gemm_roofline(c, T, per_op, per_step, pk):
    flops = gemm_flops(c, T)
    dominant = max((n for n in per_op if n in flops), key=lambda n: per_step[n])
    ach = flops[dominant] / (per_op[dominant] / 1e3) / 1e12
    return dominant, ach, {
        n: {"ms": round(per_op[n], 5), "tflops": round(flops[n] / (per_op[n] / 1e3) / 1e12, 1),
            "frac_of_burst": round(flops[n] / (per_op[n] / 1e3) / 1e12 / pk["bf16"], 3)}
        for n in flops if n in per_op}


def hbm_rooflines(c, T, per_op, pk):
    out = {}
    for n, b in hbm_bytes(c, T).items():
        if n in per_op and per_op[n] > 0:
            gbs = b / (per_op[n] / 1e3) / 1e9
            out[n] = {"ms": round(per_op[n], 5), "bytes": b, "gb_s": round(gbs, 1),
                      "frac_of_hbm": round(gbs / pk["hbm_gbs"], 3)}
    return out


def make_layer(c, run, w=None):
    from spark_gpt_b200 import SparseMoE
    layer = SparseMoE(layer_cfg(c)).to(run.dev)
    w_r, w_gu, w_d = w if w is not None else make_weights(c, 0)
    with torch.no_grad():
        layer.gate.weight.copy_(w_r)
        layer.experts.gate_up_proj.copy_(w_gu)
        layer.experts.down_proj.copy_(w_d)
    return layer


def make_inputs(c, T, run):
    x_h, d_h = make_tokens(c, T, run.rank)
    x_pin = x_h.to(torch.bfloat16).pin_memory()
    d_pin = d_h.to(torch.bfloat16).pin_memory()
    return x_pin, d_pin, x_pin.to(run.dev), d_pin.to(run.dev)


def layer_step(layer, c, valid, coef, sync=None):
    from spark_gpt_b200 import global_load_balancing_loss

    def step(xb, db):
        for p in layer.parameters():
            p.grad = None
        xin = xb.detach().requires_grad_(True)
        out, logits, sel = layer(xin)
        aux, _ = global_load_balancing_loss((logits,), (sel,), valid, num_experts=c["E"],
                                            top_k=c["k"])
        torch.autograd.backward([out, aux], [db, coef])
        if sync is not None:
            sync.wait()
        return aux
    return step


def sub_block(name, run, args, pk):
    """A compact line for another single-GPU config (N = 1 only)."""
    c = dict(CONFIGS[name])
    T = c["T"]
    layer = make_layer(c, run)
    _, _, x, d_out = make_inputs(c, T, run)
    valid = torch.ones(T, dtype=torch.bool, device=run.dev)
    coef = torch.tensor(AUX_COEF, device=run.dev)
    step = layer_step(layer, c, valid, coef)
    names = list(gemm_flops(c, T)) + ROW_KERNELS
    ms, per_op, per_step, launches = time_steps(run, lambda: step(x, d_out), args.sub_steps,
                                                max(3, args.warmup), names)
    with torch.no_grad():
        _, _, sel = layer(x)
    counts = torch.bincount(sel.reshape(-1), minlength=c["E"]).float()
    dominant, ach, gemms = gemm_roofline(c, T, per_op, per_step, pk)
    lt = layer_flops(c, T) / (ms / 1e3) / 1e12
    del layer, x, d_out
    return {
        "workload": f"{name}: BASELINE configs[{CONFIG_INDEX[name]}] "
                    + ("(its 12-layer model's MoE layer at the config's 65,536-token batch)"
                       if name == "cfg4" else "single layer"),
        "tokens": T, "hidden": c["H"], "experts": c["E"], "top_k": c["k"],
        "moe_intermediate": c["I"], "routing": c["routing"], "steps": args.sub_steps,
        "ms_per_step": ms, "tokens_per_s": T / (ms / 1e3), "layer_gemm_tflops": lt,
        "layer_frac_of_burst": lt / pk["bf16"],
        "gemm_kernels_ms_per_step": sum(per_step.get(n, 0.0) for n in gemm_flops(c, T)),
        "roofline": {"bound": "tensor", "kernel": dominant, "achieved": ach, "peak": pk["bf16"],
                     "unit": "TFLOP/s", "frac": ach / pk["bf16"],
                     "peak_source": f"{pk['source']} bf16 burst (MEASURED_PEAKS.json)"},
        "gemms": gemms, "hbm_kernels": hbm_rooflines(c, T, per_op, pk),
        "rows_per_expert": {"max": int(counts.max()), "mean": float(counts.mean()),
                            "min": int(counts.min()),
                            "max_over_mean": float(counts.max() / counts.mean())},
        "gpu_launches_per_step": launches / args.sub_steps,
    }


# --------------------------------------------------------------------------- #
# On-box GPU comparator: the reference's stock-torch GPU path, not the product
# --------------------------------------------------------------------------- #
class _TorchGatherRows(torch.autograd.Function):
    """rows = x[token] with the backward as a gather of each token's k rows
    and a sum (the reference's _GatherTopK, train.py:2195-2217)."""

    @staticmethod
    def forward(ctx, x, token, inv, k):
        ctx.save_for_backward(inv)
        ctx.k = k
        return x[token]

    @staticmethod
    def backward(ctx, g):
        (inv,) = ctx.saved_tensors
        return g[inv].view(-1, ctx.k, g.shape[-1]).sum(dim=1), None, None, None


class _TorchCombineRows(torch.autograd.Function):
    """out[t] = sum of w * y over token t's k rows, gathers both ways (the
    reference's _CombineTopK, train.py:2220-2241)."""

    @staticmethod
    def forward(ctx, y, w, inv, token, k):
        ctx.save_for_backward(y, w, token)
        weighted = y * w.unsqueeze(-1)
        return weighted[inv].view(-1, k, y.shape[-1]).sum(dim=1)

    @staticmethod
    def backward(ctx, g):
        y, w, token = ctx.saved_tensors
        g_rows = g[token]
        return g_rows * w.unsqueeze(-1), (g_rows * y).sum(dim=-1), None, None, None


def torch_path_step(layer, c, valid, coef):
    """One step of the reference's GPU path with FUSED_SWIGLU off, in stock
    torch ops on the same fp32 master weights: router F.linear + fp32 softmax
    + torch.topk + renorm (train.py:2144-2158), sort / inverse / histc /
    cumsum (:2271-2290), F.grouped_mm on the bf16 view of each expert tensor
    (:2160-2181) with SiLU(gate) * up between (:2312-2318), the gather-based
    combine, and the load-balancing loss (:3098-3197) as autograd over the
    softmax.  cuBLAS / CUTLASS library kernels throughout: this is the GPU bar
    the hand-written layer is compared against, under autocast(bf16) as the
    reference's training step runs it."""
    import torch.nn.functional as F
    E, k = c["E"], c["k"]
    w_r = layer.gate.weight
    w_gu, w_d = layer.experts.gate_up_proj, layer.experts.down_proj

    def step(xb, db):
        for p in layer.parameters():
            p.grad = None
        xin = xb.detach().requires_grad_(True)
        with torch.autocast("cuda", dtype=torch.bfloat16):
            logits = F.linear(xin, w_r)
        probs = F.softmax(logits, dtype=torch.float32, dim=-1)
        rw, sel = torch.topk(probs, k, dim=-1)
        rw = (rw / rw.sum(dim=-1, keepdim=True)).to(logits.dtype)
        flat = sel.reshape(-1)
        sorted_e, perm = torch.sort(flat)
        token = perm // k
        inv = torch.empty_like(perm)
        inv[perm] = torch.arange(perm.numel(), device=perm.device)
        counts = torch.histc(sorted_e.int() if sorted_e.is_cuda else sorted_e.float(),
                             bins=E, min=0, max=E - 1)
        offs = torch.cumsum(counts, dim=0, dtype=torch.int32)
        xs = _TorchGatherRows.apply(xin, token, inv, k)
        gu = F.grouped_mm(xs, w_gu.to(xs.dtype).transpose(-2, -1), offs=offs)
        gate, up = gu.chunk(2, dim=-1)
        y = F.grouped_mm(F.silu(gate) * up, w_d.to(xs.dtype).transpose(-2, -1), offs=offs)
        out = _TorchCombineRows.apply(y, rw.reshape(-1)[perm], inv, token, k).to(xin.dtype)
        rows = valid.sum().clamp_min(1).float()
        frac = torch.bincount(flat, minlength=E).float() / rows
        soft = (probs * valid.unsqueeze(-1)).sum(dim=0) / rows
        aux = E * torch.dot(frac, soft)
        torch.autograd.backward([out, aux], [db, coef])
        return out, xin
    return step


def torch_path_block(run, args, pk):
    """cfg2 through the stock-torch comparator on this GPU, timed like the
    product (same weights and inputs), with its agreement against the
    product layer on one step (bf16 contract: relative to the product's
    max magnitude)."""
    c = dict(CONFIGS[args.config])
    T = c["T"]
    layer = make_layer(c, run)
    _, _, x, d_out = make_inputs(c, T, run)
    valid = torch.ones(T, dtype=torch.bool, device=run.dev)
    coef = torch.tensor(AUX_COEF, device=run.dev)
    step = torch_path_step(layer, c, valid, coef)
    try:
        out_t, x_t = step(x, d_out)
    except (RuntimeError, NotImplementedError) as e:  # grouped_mm unsupported here
        return {"unavailable": f"{type(e).__name__}: {str(e).splitlines()[0][:200]}"}
    ref = (out_t.detach().float(), x_t.grad.float(), layer.experts.gate_up_proj.grad.clone())
    mine = layer_step(layer, c, valid, coef)
    xin = x.detach().requires_grad_(True)
    from spark_gpt_b200 import global_load_balancing_loss
    for p in layer.parameters():
        p.grad = None
    out, logits, sel = layer(xin)
    aux, _ = global_load_balancing_loss((logits,), (sel,), valid, num_experts=c["E"],
                                        top_k=c["k"])
    torch.autograd.backward([out, aux], [d_out, coef])

    def rel(a, b):
        return float((a.float() - b).abs().max() / b.abs().max().clamp_min(1e-30))
    agree = {"out": rel(out.detach(), ref[0]), "dx": rel(xin.grad, ref[1]),
             "dW_gate_up": rel(layer.experts.gate_up_proj.grad, ref[2])}
    del out, logits, sel, aux, xin, out_t, x_t, ref
    ms_t, _, _, _ = time_steps(run, lambda: step(x, d_out), args.sub_steps,
                               max(3, args.warmup), [])
    ms_m, _, _, _ = time_steps(run, lambda: mine(x, d_out), args.sub_steps,
                               max(3, args.warmup), [])
    lf = layer_flops(c, T)
    del layer, x, d_out, step, mine
    dense = dense_gemm_block(c, T, pk)
    return {
        "workload": f"{args.config}, {T} tokens: the reference's GPU path with "
                    f"FUSED_SWIGLU off (F.grouped_mm, train.py:2160-2181) in stock torch ops",
        "steps": args.sub_steps,
        "torch_ms_per_step": ms_t, "torch_tokens_per_s": T / (ms_t / 1e3),
        "torch_layer_frac_of_burst": lf / (ms_t / 1e3) / 1e12 / pk["bf16"],
        "b200_ms_per_step": ms_m, "b200_tokens_per_s": T / (ms_m / 1e3),
        "speedup": ms_t / ms_m,
        "max_rel_diff_vs_b200": agree,
        "cublas_dense_same_shapes": dense,
        "note": "the reference's Triton fused path (train.py:2304-2310) cannot run here: the "
                "reference checkout is not on the GPU box and its kernels are not copied",
    }


def dense_gemm_block(c, T, pk, reps=10):
    """cuBLAS (torch.mm, bf16) on one dense GEMM of each expert GEMM's total
    shape -- all R routed rows against one expert's weight -- the library's
    rate on this M/N/K without the grouping: what the grouped kernels' frac
    of the square-GEMM burst peak should be read against."""
    R, H, I = T * c["k"], c["H"], c["I"]
    shapes = {  # name: (M, N, K) of the output M x N with reduction K
        "gate_up_fwd": (R, 2 * I, H), "down_fwd": (R, H, I), "down_dgrad": (R, I, H),
        "gate_up_dgrad": (R, H, 2 * I), "gate_up_wgrad": (2 * I, H, R), "down_wgrad": (H, I, R),
    }
    out = {}
    for n, (M, N, K) in shapes.items():
        if n.endswith("wgrad"):   # dW = A^T B with the rows as the reduction (column-major A)
            a = torch.randn(K, M, device="cuda", dtype=torch.bfloat16).t()
        else:
            a = torch.randn(M, K, device="cuda", dtype=torch.bfloat16)
        b = torch.randn(K, N, device="cuda", dtype=torch.bfloat16)
        o = torch.empty(M, N, device="cuda", dtype=torch.bfloat16)
        for _ in range(3):
            torch.mm(a, b, out=o)
        e0 = torch.cuda.Event(enable_timing=True)
        e1 = torch.cuda.Event(enable_timing=True)
        torch.cuda.synchronize()
        e0.record()
        for _ in range(reps):
            torch.mm(a, b, out=o)
        e1.record()
        torch.cuda.synchronize()
        ms = e0.elapsed_time(e1) / reps
        tf = 2 * M * N * K / (ms / 1e3) / 1e12
        out[n] = {"mnk": [M, N, K], "ms": round(ms, 5), "tflops": round(tf, 1),
                  "frac_of_burst": round(tf / pk["bf16"], 3)}
        del a, b, o
    return out


def fp8_block(run, args, pk):
    """The layer step on the fp8 expert path (spark-gpt --fp8-mlp on MoE
    layers, train.py:1258-1604) at this config, N = 1: the same step as the
    headline with spark_gpt_b200.fp8.FP8_MLP on, after a prewarm step and a
    scale update as the reference's trainer does (train.py:4001-4002).  The
    fp8 GEMMs' rates are against twice the measured bf16 burst peak (the dense
    fp8 rate is twice the bf16 one on this part; no fp8 peak is measured
    here), and the bf16 step is timed in the same run for the speed-up."""
    from spark_gpt_b200 import fp8, fp8_update_scales
    c = dict(CONFIGS[args.config])
    T = c["T"]
    layer = make_layer(c, run)
    layer.train()
    _, _, x, d_out = make_inputs(c, T, run)
    valid = torch.ones(T, dtype=torch.bool, device=run.dev)
    coef = torch.tensor(AUX_COEF, device=run.dev)
    step = layer_step(layer, c, valid, coef)
    names = list(gemm_flops(c, T)) + ROW_KERNELS + ["fp8_quantize", "fp8_quantize_rows"]
    ms_bf16, _, _, _ = time_steps(run, lambda: step(x, d_out), args.sub_steps,
                                  max(3, args.warmup), names)
    saved = fp8.FP8_MLP
    fp8.FP8_MLP = True
    try:
        if not fp8.use_fp8(layer.experts, x):
            return {"unavailable": "shape outside the fp8 kernels' range"}
        step(x, d_out)                    # prewarm: records the amax
        fp8_update_scales(layer)
        ms, per_op, _, launches = time_steps(run, lambda: step(x, d_out), args.sub_steps,
                                             max(3, args.warmup), names)
        scale = [float(v) for v in layer.experts.fp8_scale]
    finally:
        fp8.FP8_MLP = saved
    flops = gemm_flops(c, T)
    peak8 = 2 * pk["bf16"]
    gemms = {}
    for n in ("gate_up_fwd", "down_fwd", "gate_up_dgrad", "gate_up_wgrad", "down_wgrad"):
        if n in per_op:
            tf = flops[n] / (per_op[n] / 1e3) / 1e12
            gemms[n] = {"ms": round(per_op[n], 5), "tflops": round(tf, 1),
                        "frac_of_2x_bf16_burst": round(tf / peak8, 3)}
    if "down_dgrad" in per_op:  # bf16 operands on this path too (train.py:1382-1423)
        tf = flops["down_dgrad"] / (per_op["down_dgrad"] / 1e3) / 1e12
        gemms["down_dgrad"] = {"ms": round(per_op["down_dgrad"], 5), "tflops": round(tf, 1),
                               "frac_of_bf16_burst": round(tf / pk["bf16"], 3),
                               "operands": "bf16"}
    del layer, x, d_out, step
    return {
        "workload": f"{args.config}, {T} tokens: the layer step with the experts on the fp8 path "
                    f"(e4m3 x/gu/h/weights, e5m2 d_gu/dy, delayed scales)",
        "steps": args.sub_steps, "ms_per_step": ms, "tokens_per_s": T / (ms / 1e3),
        "bf16_ms_per_step": ms_bf16, "speedup_vs_bf16": ms_bf16 / ms,
        "scales_after_prewarm": scale,
        "gemms": gemms,
        "kernels_ms": {n: round(v, 5) for n, v in sorted(per_op.items())},
        "gpu_launches_per_step": launches / args.sub_steps,
        "peak_note": "fp8 GEMM fractions are of 2x the measured bf16 burst peak "
                     f"({peak8:.0f} TFLOP/s; the nominal dense fp8 rate is 2x bf16)",
    }


def ep_block(run, args, pk):
    """BASELINE config 5 at this N: the single-GPU layer at cfg5's per-GPU
    shape on every rank (the baseline), then the expert-parallel layer over
    all ranks with each transport; efficiency = single-GPU ms / EP ms (the
    same tokens per GPU)."""
    from spark_gpt_b200 import global_load_balancing_loss
    name = args.ep_config
    c = dict(CONFIGS[name])
    T = c["T"]
    w = make_weights(c, 0)
    valid = torch.ones(T, dtype=torch.bool, device=run.dev)
    coef = torch.tensor(AUX_COEF, device=run.dev)
    _, _, x, d_out = make_inputs(c, T, run)
    res = {"workload": f"{name}: BASELINE configs[4] (H {c['H']}, E {c['E']}, top-{c['k']}, "
                       f"I {c['I']}, {T} tokens per GPU, {c['routing']} routing)",
           "n_gpus": run.world, "steps": args.ep_steps}
    layer = make_layer(c, run, w)
    step = layer_step(layer, c, valid, coef)
    ms1, per_op, per_step, _ = time_steps(run, lambda: step(x, d_out), args.ep_steps,
                                          max(3, args.warmup), list(gemm_flops(c, T)))
    res["single_gpu"] = {"ms_per_step": ms1, "tokens_per_s_per_gpu": T / (ms1 / 1e3),
                         "gemm_kernels_ms_per_step": sum(per_step.values())}
    del layer, step
    if run.world == 1:
        return res
    from spark_gpt_b200.ep import ExpertParallelMoE
    for transport in ("p2p_pipe", "p2p", "nccl"):
        layer = ExpertParallelMoE(layer_cfg(c), chunks=1, comm_sms=args.comm_sms,
                                  transport=transport).to(run.dev)
        lo, hi = layer.expert_offset, layer.expert_offset + layer.local_experts
        with torch.no_grad():
            layer.gate.weight.copy_(w[0])
            layer.experts.gate_up_proj.copy_(w[1][lo:hi])
            layer.experts.down_proj.copy_(w[2][lo:hi])

        def step():
            for p in layer.parameters():
                p.grad = None
            xin = x.detach().requires_grad_(True)
            out, logits, sel = layer(xin)
            aux, _ = global_load_balancing_loss((logits,), (sel,), valid, num_experts=c["E"],
                                                top_k=c["k"])
            torch.autograd.backward([out, aux], [d_out, coef])
            # the replicated router weight's gradient: averaged as DDP does
            run.dist.all_reduce(layer.gate.weight.grad, op=run.dist.ReduceOp.AVG)

        names = list(gemm_flops(c, T)) + ROW_KERNELS + EP_KERNELS
        ms, per_op, per_step, _ = time_steps(run, step, args.ep_steps, max(3, args.warmup), names)
        gemm_ms = sum(per_step.get(n, 0.0) for n in gemm_flops(c, T))
        res[transport] = {
            "ms_per_step": ms, "tokens_per_s_per_gpu": T / (ms / 1e3),
            "tokens_per_s": run.world * T / (ms / 1e3), "efficiency": ms1 / ms,
            "gemm_kernels_ms_per_step": gemm_ms,
            "phases_ms_per_step": {n: round(per_step[n], 4) for n in
                                   EP_KERNELS + ["dispatch", "gather", "combine", "gather_bwd",
                                                 "combine_bwd"] if n in per_step},
            "comm_sms": args.comm_sms,
        }
        del layer
        torch.cuda.synchronize()
    return res


def main():
    args = parse_args()
    c = dict(CONFIGS[args.config])
    if args.tokens:
        c["T"] = args.tokens
    if args.impl == "reference":
        run_reference(args, c)
        return

    run = Run()
    world, rank, dev = run.world, run.rank, run.dev
    from spark_gpt_b200 import ops

    T = c["T"]
    pk = peaks()
    w_r, w_gu, w_d = make_weights(c, 0)
    if c.get("ep") and world > 1:
        from spark_gpt_b200.ep import ExpertParallelMoE
        layer = ExpertParallelMoE(layer_cfg(c), chunks=args.ep_chunks, comm_sms=args.comm_sms,
                                  transport=args.transport).to(dev)
        lo, hi = layer.expert_offset, layer.expert_offset + layer.local_experts
        w_gu, w_d = w_gu[lo:hi], w_d[lo:hi]
        with torch.no_grad():
            layer.gate.weight.copy_(w_r)
            layer.experts.gate_up_proj.copy_(w_gu)
            layer.experts.down_proj.copy_(w_d)
    else:
        layer = make_layer(c, run, (w_r, w_gu, w_d))
    # data parallel: the gradient all-reduce DDP does in the reference's step
    # (train.py:3781), started inside the backward as soon as the expert
    # gradients are final (grad_sync.py)
    sync = None
    if world > 1 and not c.get("ep") and not args.no_grad_sync:
        from spark_gpt_b200.grad_sync import GradSync
        sync = GradSync(layer, comm_sms=args.comm_sms)
    x_pin, d_pin, x, d_out = make_inputs(c, T, run)
    valid = torch.ones(T, dtype=torch.bool, device=dev)
    coef = torch.tensor(AUX_COEF, device=dev)
    step = layer_step(layer, c, valid, coef, sync)
    if args.fp8:
        if world > 1 or c.get("ep"):
            raise SystemExit("bench.py --fp8: single-GPU, non-expert-parallel configs only")
        from spark_gpt_b200 import fp8, fp8_update_scales
        fp8.FP8_MLP = True
        layer.train()
        step(x, d_out)  # prewarm: the first amax
        fp8_update_scales(layer)

    # ---------------- timed region: inputs resident in HBM
    names = list(gemm_flops(c, T)) + ROW_KERNELS + (EP_KERNELS if c.get("ep") else [])
    clocks = {}
    ms, per_op, per_step, launches = time_steps(run, lambda: step(x, d_out), args.steps,
                                                args.warmup, names, clocks=clocks)
    value = world * T / (ms / 1e3)
    dominant, ach, gemms = gemm_roofline(c, T, per_op, per_step, pk)
    traffic = None
    tfile = ROOT / "profiles" / "traffic.json"
    if tfile.exists():
        traffic = json.loads(tfile.read_text()).get(args.config, {}).get(dominant)
    layer_tflops = layer_flops(c, T) / (ms / 1e3) / 1e12
    gemm_ms = sum(per_step.get(n, 0.0) for n in gemm_flops(c, T))

    # ---------------- end to end: host buffers, copies inside the timed region.
    e2e = None if args.no_e2e else e2e_block(run, layer, c, T, x, x_pin, valid, args, sync)

    # ---------------- Muon step of the packed expert tensors (the optimizer that
    # consumes the fp32 weight gradients written above, train.py:2930-3024)
    muon_line = None
    if not args.no_muon and not (c.get("ep") and world > 1):
        muon_line = muon_block(layer, c, step, x, d_out, args, pk)
    if sync is not None:
        sync.detach()

    cpu = None
    if rank == 0 and world == 1 and not args.no_cpu_baseline and not c.get("ep"):
        Ts = args.cpu_sample_tokens
        v, cores = cpu_throughput(c, Ts, 3, 1)
        cpu = {"value": v, "unit": "tokens/s", "cores": cores, "kind": "port",
               "sample": f"{Ts} tokens of {args.config} shapes, fp32 torch-CPU port of the "
                         f"reference's torch MoE path, 3 timed steps after 1 warm-up"}
    del layer, step

    subs = {}
    torch_path = None
    fp8_line = None
    if world == 1 and args.config == "cfg2" and not args.no_extra:
        for name in ("cfg3", "cfg4"):
            subs[name] = sub_block(name, run, args, pk)
        try:
            torch_path = torch_path_block(run, args, pk)
        except Exception as e:  # a comparator failure must not cost the product's line
            torch_path = {"unavailable": f"{type(e).__name__}: {str(e).splitlines()[0][:200]}"}
        fp8_line = fp8_block(run, args, pk)
    ep = None
    if not args.no_ep and not c.get("ep"):
        ep = ep_block(run, args, pk)

    if run.dist.is_initialized():
        run.dist.barrier()
        run.dist.destroy_process_group()
    if rank != 0:
        return
    line = {
        "metric": METRIC, "value": value, "unit": "tokens/s", "n_gpus": world,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": ms,
        "higher_is_better": True, "scaling": "weak", "vs_baseline": None,
        "dtype": "fp8 experts (e4m3/e5m2), bf16 elsewhere" if args.fp8 else "bf16",
        "data": "synthetic (seeded N(0,1) tokens, muP-init weights)",
        "config": config_block(args, c, world, sync is not None),
        "per_gpu_tokens_per_s": value / world,
        "layer_gemm_tflops": layer_tflops,
        "tensor_peak_frac": layer_tflops / pk["bf16"],
        "gemm_kernels_ms_per_step": gemm_ms,
        "roofline": {"bound": "tensor", "kernel": dominant, "achieved": ach,
                     "peak": pk["bf16"], "unit": "TFLOP/s", "frac": ach / pk["bf16"],
                     "frac_of_sustained": ach / pk["bf16_sustained"], "traffic": traffic,
                     "peak_source": f"{pk['source']} bf16 burst (MEASURED_PEAKS.json): the "
                                    f"timed region is well under a second"},
        "gemms": gemms,
        "hbm_kernels": hbm_rooflines(c, T, per_op, pk),
        "kernels_ms": {n: round(v, 5) for n, v in sorted(per_op.items())},
        "cpu_baseline": cpu,
        "e2e": e2e,
        "muon_step": muon_line,
        "configs": subs or None,
        "torch_gpu_path": torch_path,
        "fp8": fp8_line,
        "ep": ep,
        "gpu_launches": launches,
        "gpu_launches_per_step": launches / max(args.steps, 1),
        "clocks": clocks,
    }
    # the dominant kernel against cuBLAS on a dense GEMM of its own shape, measured
    # in this run (the square-GEMM burst peak is out of reach for short-K shapes)
    dense = (torch_path or {}).get("cublas_dense_same_shapes") or {}
    if dominant in dense:
        line["roofline"]["cublas_same_shape_tflops"] = dense[dominant]["tflops"]
        line["roofline"]["frac_of_cublas_same_shape"] = ach / dense[dominant]["tflops"]
    print(json.dumps(line), flush=True)


class _MeanSquare(torch.autograd.Function):
    """mean(out^2) in fp32 with one read of out forward and one read + one
    bf16 write backward (the same value and gradient as
    out.float().square().mean(), without its fp32 copies of out)."""

    @staticmethod
    def forward(ctx, out):
        ctx.save_for_backward(out)
        n = torch.linalg.vector_norm(out.reshape(-1), dtype=torch.float32)
        return n * n / out.numel()

    @staticmethod
    def backward(ctx, g):
        (out,) = ctx.saved_tensors
        return out * (g * (2.0 / out.numel())).to(out.dtype)


def e2e_block(run, layer, c, T, x, x_pin, valid, args, sync):
    """The training step of the reference arm -- forward, loss = mean(out^2) +
    1e-3 * aux, backward -- with its one input, x, copied from pinned host
    memory every step and the loss read back to pinned host memory.  As a
    training input pipeline does, the copy of step i+1's x runs on a copy
    stream while step i computes (two device buffers, ordered by events).
    Every copy lies inside the timed region.  Per phase (CUDA events on the
    compute stream): waiting for the input copy, forward, loss, backward
    (with the gradient all-reduce when data parallel), loss read-back."""
    from spark_gpt_b200 import global_load_balancing_loss
    dev = run.dev
    loss_h = torch.empty((), dtype=torch.float32).pin_memory()
    comp = torch.cuda.current_stream(dev)
    copy = torch.cuda.Stream(dev)
    bufs = [torch.empty_like(x) for _ in range(2)]
    copied = [torch.cuda.Event() for _ in range(2)]
    freed = [torch.cuda.Event() for _ in range(2)]
    phases = ["h2d_wait", "forward", "loss", "backward", "d2h"]
    marks = []

    def ev():
        e = torch.cuda.Event(enable_timing=True)
        e.record(comp)
        return e

    def loss_step(xb, mark=None):
        for p in layer.parameters():
            p.grad = None
        xin = xb.detach().requires_grad_(True)
        t1 = ev() if mark is not None else None
        out, logits, sel = layer(xin)
        t2 = ev() if mark is not None else None
        aux, _ = global_load_balancing_loss((logits,), (sel,), valid, num_experts=c["E"],
                                            top_k=c["k"])
        loss = _MeanSquare.apply(out) + AUX_COEF * aux
        t3 = ev() if mark is not None else None
        loss.backward()
        if sync is not None:
            sync.wait()
        t4 = ev() if mark is not None else None
        if mark is not None:
            mark.extend([t1, t2, t3, t4])
        return loss

    def prefetch(i):
        xb = bufs[i % 2]
        with torch.cuda.stream(copy):
            if i >= 2:
                copy.wait_event(freed[i % 2])  # step i-2 is done with this buffer
            xb.copy_(x_pin, non_blocking=True)
            copied[i % 2].record(copy)

    for _ in range(2):
        loss_step(x)  # warm the loss's own kernels
    torch.cuda.synchronize()
    run.barrier()
    e0 = torch.cuda.Event(enable_timing=True)
    e1 = torch.cuda.Event(enable_timing=True)
    e0.record(comp)
    prefetch(0)
    for i in range(args.steps):
        if i + 1 < args.steps:
            prefetch(i + 1)
        m = [ev()]
        comp.wait_event(copied[i % 2])
        loss = loss_step(bufs[i % 2], m)
        freed[i % 2].record(comp)
        loss_h.copy_(loss.detach(), non_blocking=True)
        m.append(ev())
        marks.append(m)
    e1.record(comp)
    torch.cuda.synchronize()
    run.barrier()
    e2e_ms = run.max(e0.elapsed_time(e1)) / args.steps
    ph = {p: 0.0 for p in phases}
    for m in marks:
        for j, p in enumerate(phases):
            ph[p] += m[j].elapsed_time(m[j + 1]) / len(marks)
    return {"value": run.world * T / (e2e_ms / 1e3), "unit": "tokens/s",
            "h2d_bytes_per_step": x_pin.numel() * 2, "d2h_bytes_per_step": 4,
            "ms_per_step": e2e_ms, "phases_ms": {p: round(v, 4) for p, v in ph.items()},
            "step": "forward, loss = mean(out^2) + 1e-3*aux, backward (the reference arm's "
                    "step); x from pinned host memory, the loss read back",
            "pipeline": "next step's H2D overlapped with this step's compute (copy stream, "
                        "double-buffered inputs)"}


def muon_block(layer, c, step, x, d_out, args, pk):
    from spark_gpt_b200.muon import PackedExpertMuon
    step(x, d_out)
    eparams = [layer.experts.gate_up_proj, layer.experts.down_proj]
    saved = [p.detach().clone() for p in eparams]
    opt = PackedExpertMuon(eparams, lr=0.02)
    for _ in range(3):
        opt.step()
    torch.cuda.synchronize()
    m0 = torch.cuda.Event(enable_timing=True)
    m1 = torch.cuda.Event(enable_timing=True)
    n_muon = max(5, args.steps // 2)
    m0.record()
    for _ in range(n_muon):
        opt.step()
    m1.record()
    torch.cuda.synchronize()
    muon_ms = m0.elapsed_time(m1) / n_muon
    with torch.no_grad():
        for p, s0 in zip(eparams, saved):
            p.copy_(s0)

    def ns_flops(Eq, r, cc, steps=5):
        g, G = min(r, cc), max(r, cc)
        return Eq * steps * (4 * g * g * G + 2 * g ** 3)

    mflops = (ns_flops(layer.experts.gate_up_proj.shape[0], 2 * c["I"], c["H"]) +
              ns_flops(layer.experts.down_proj.shape[0], c["H"], c["I"]))
    mt = mflops / (muon_ms / 1e3) / 1e12
    return {"ms_per_step": muon_ms, "ns_tflop": mflops / 1e12, "tflops": mt,
            "frac_of_bf16_burst": mt / pk["bf16"],
            "what": "PackedExpertMuon.step on gate_up_proj + down_proj: momentum, "
                    "5 Newton-Schulz iterations as grouped tcgen05 GEMMs, fused "
                    "parameter update"}


if __name__ == "__main__":
    main()
