"""Generate golden vectors by running the spark-gpt reference itself.

Run in a container that has the reference checkout (never on the GPU box):

    python tests/golden/make_golden.py --reference PATH
    (or SPARK_GPT_REFERENCE=PATH python tests/golden/make_golden.py)

It imports ``train.py`` from the reference checkout (not copied), runs its
``SparseMoE`` (train.py:2325-2334) and ``global_load_balancing_loss``
(train.py:3098-3197) on seeded CPU fp32 inputs, back-propagates
``(out * probe).sum() + 1e-3 * aux``, and stores inputs and outputs in
``tests/golden/moe_golden.pt``; it also runs two ``MuonAdamWHybrid`` steps
(train.py:2930-3024) on seeded packed expert tensors and the batched
Newton-Schulz iteration (train.py:2877-2927) on its own, stored in
``tests/golden/muon_golden.pt`` (``--only muon`` writes just that file); and it runs
the reference's ``RMSNorm`` (train.py:162-170) forward and backward into
``tests/golden/norm_golden.pt`` (``--only norm``), and the pure-torch pieces of
its fp8 expert path (train.py:938-946, :1536-1540) into
``tests/golden/fp8_golden.pt`` (``--only fp8``).  The large config-1 case stores its inputs as a
seed plus checksums and keeps only slices and norms of the float outputs, so
the fixture stays small.
"""

from __future__ import annotations

import argparse
import os
import sys
from pathlib import Path

import torch

HERE = Path(__file__).resolve().parent


def seeded_inputs(T, H, E, I, seed, std_router=0.02, std_gu=0.02, std_down=0.02):
    g = torch.Generator().manual_seed(seed)
    x = torch.randn(T, H, generator=g)
    w_r = torch.randn(E, H, generator=g) * std_router
    w_gu = torch.randn(E, 2 * I, H, generator=g) * std_gu
    w_d = torch.randn(E, H, I, generator=g) * std_down
    probe = torch.randn(T, H, generator=g)
    return x, w_r, w_gu, w_d, probe


def run_layer(train, x, w_r, w_gu, w_d, probe, top_k, norm, valid):
    T, H = x.shape
    E, twoI, _ = w_gu.shape
    cfg = train.ModelConfig(hidden_size=H, num_experts=E, num_experts_per_tok=top_k,
                            moe_intermediate_size=twoI // 2, norm_topk_prob=norm,
                            num_hidden_layers=1, mlp_only_layers=())
    moe = train.SparseMoE(cfg)
    with torch.no_grad():
        moe.gate.weight.copy_(w_r)
        moe.experts.gate_up_proj.copy_(w_gu)
        moe.experts.down_proj.copy_(w_d)
    xin = x.clone().requires_grad_(True)
    out, logits, selected = moe(xin)
    aux, stats = train.global_load_balancing_loss(
        (logits,), (selected,), valid, num_experts=E, top_k=top_k)
    loss = (out * probe).sum() + 1e-3 * aux
    loss.backward()
    # dispatch exactly as Experts.forward does (train.py:2271-2290)
    flat = selected.reshape(-1)
    _, perm = torch.sort(flat)
    inv = torch.empty_like(perm)
    inv[perm] = torch.arange(perm.numel())
    counts = torch.bincount(flat, minlength=E)
    rw = moe.gate(xin.detach())[1]
    return {
        "out": out.detach(), "logits": logits.detach(), "selected": selected,
        "routing_weights": rw.detach(), "permutation": perm, "inverse": inv,
        "offsets": torch.cumsum(counts, 0).to(torch.int32), "aux": aux.detach(),
        **{f"stat_{k}": v.detach() for k, v in stats.items()},
        "dx": xin.grad, "dW_router": moe.gate.weight.grad,
        "dW_gate_up": moe.experts.gate_up_proj.grad, "dW_down": moe.experts.down_proj.grad,
    }


MUON_CASES = {
    # name: (E, rows, cols, lr, momentum, nesterov, seed): gate_up-like wide and
    # down-like tall packed expert tensors
    "muon_wide": (2, 128, 256, 0.02, 0.95, True, 11),
    "muon_tall": (2, 256, 128, 0.02, 0.95, True, 12),
    "muon_square_plain": (1, 128, 128, 0.05, 0.9, False, 13),
}
NS_CASES = {"ns_wide": ((2, 128, 256), 21), "ns_tall": ((2, 256, 128), 22)}


def muon_case_inputs(E, rows, cols, seed):
    """Initial packed parameter and the two steps' gradients of a Muon case."""
    g = torch.Generator().manual_seed(seed)
    p0 = torch.randn(E, rows, cols, generator=g) * 0.02
    grads = [torch.randn(E, rows, cols, generator=g) * 1e-3 for _ in range(2)]
    return p0, grads


def ns_case_input(shape, seed):
    g = torch.Generator().manual_seed(seed)
    return (torch.randn(*shape, generator=g) * 0.3).to(torch.bfloat16)


def make_muon_golden(train, out_path):
    """Two MuonAdamWHybrid steps (train.py:2930-3024) on seeded packed expert
    tensors, run by the reference itself on CPU (its lerp + bmm/baddbmm path).
    Inputs are regenerated from the seeds (muon_case_inputs); stored: the
    parameter change after two steps and the momentum buffer."""
    cases = {}
    for name, (E, rows, cols, lr, mom, nest, seed) in MUON_CASES.items():
        p0, grads = muon_case_inputs(E, rows, cols, seed)
        p = torch.nn.Parameter(p0.clone())
        opt = train.MuonAdamWHybrid([{"params": [p], "use_muon": True, "lr": lr,
                                      "momentum": mom, "nesterov": nest, "ns_steps": 5}])
        for gr in grads:
            p.grad = gr.clone()
            opt.step()
        cases[name] = {"delta2": p.detach() - p0, "v2": opt.state[p]["v"].clone(),
                       "input_sum": p0.double().sum() + sum(gr.double().sum() for gr in grads)}
    # the orthogonalisation on its own (train.py:2877-2927)
    for name, (shape, seed) in NS_CASES.items():
        x = ns_case_input(shape, seed)
        cases[name] = {"out": train._newtonschulz5_batched(x.clone(), steps=5)}
    torch.save(cases, out_path)
    print(f"wrote {out_path}: {', '.join(cases)}")


def make_norm_golden(train, out_path):
    """The reference's RMSNorm (train.py:162-170) forward and backward on
    seeded inputs: bf16 rows (as under autocast) and an fp32 weight, in fp32
    (autograd), plus the fp32-input case."""
    cases = {}
    for name, (T, H, seed, dtype) in {
        "norm_bf16": (64, 256, 11, torch.bfloat16),
        "norm_f32": (48, 768, 12, torch.float32),
    }.items():
        g = torch.Generator().manual_seed(seed)
        x = (torch.randn(T, H, generator=g) * 2.0).to(dtype)
        w = 1.0 + 0.1 * torch.randn(H, generator=g)
        probe = torch.randn(T, H, generator=g).to(dtype)
        norm = train.RMSNorm(H, eps=1e-6)
        with torch.no_grad():
            norm.weight.copy_(w)
        xin = x.clone().requires_grad_(True)
        out = norm(xin)
        (out.float() * probe.float()).sum().backward()
        cases[name] = {"x": x, "w": w, "eps": torch.tensor(1e-6), "probe": probe,
                       "out": out.detach(), "dx": xin.grad, "dw": norm.weight.grad.clone()}
    torch.save(cases, out_path)
    print(f"wrote {out_path}: {', '.join(cases)}")


def make_fp8_golden(train, out_path):
    """The reference's pure-torch pieces of the fp8 expert path: the per-expert
    e4m3 weight copies (train.py:1536-1540) and the delayed-scale update
    (train.py:938-946) on seeded and edge-case inputs (an all-zero expert,
    exact powers of two, amax slots that recorded nothing)."""
    cases = {}
    g = torch.Generator().manual_seed(21)
    w = torch.randn(6, 64, 96, generator=g) * torch.tensor([0.02, 0.5, 3.0, 1e-4, 0.0, 7.0])[:, None, None]
    w[5, 0, 0] = 448.0 / 8.0  # amax exactly 56: 448 / amax = 8 = 2^3
    w8, q = train._fp8_quantize_experts(w)
    cases["quantize_experts"] = {"w": w, "w8": w8.view(torch.uint8), "q": q}
    amaxes = torch.tensor([
        [4.5625, 3.4688, 5.1289, 0.0, 0.0],
        [1.0, 448.0, 0.5, 57344.0, 3.0e-3],
        [0.0, 0.0, 0.0, 0.0, 0.0],
        [1e-35, 2.0 ** -20, 7.0, 1e10, 0.7],
    ])
    upd = []
    for a in amaxes:
        m = torch.nn.Module()
        m.__class__ = type("M", (train.Experts,), {})  # fp8_update_scales matches Experts
        torch.nn.Module.__init__(m)
        m.register_buffer("fp8_scale", torch.tensor([2.0, 0.5, 1.0, 4.0, 1.0]))
        m.register_buffer("fp8_amax", a.clone())
        train.fp8_update_scales(m)
        upd.append((a, m.fp8_scale.clone(), m.fp8_amax.clone()))
    cases["update_scales"] = {"scale_in": torch.tensor([2.0, 0.5, 1.0, 4.0, 1.0]),
                              "amax": torch.stack([u[0] for u in upd]),
                              "scale_out": torch.stack([u[1] for u in upd]),
                              "amax_out": torch.stack([u[2] for u in upd])}
    torch.save(cases, out_path)
    print(f"wrote {out_path}: {', '.join(cases)}")


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--reference", default=os.environ.get("SPARK_GPT_REFERENCE"),
                    help="reference checkout holding train.py (default: $SPARK_GPT_REFERENCE)")
    ap.add_argument("--out", default=str(HERE / "moe_golden.pt"))
    ap.add_argument("--muon-out", default=str(HERE / "muon_golden.pt"))
    ap.add_argument("--norm-out", default=str(HERE / "norm_golden.pt"))
    ap.add_argument("--fp8-out", default=str(HERE / "fp8_golden.pt"))
    ap.add_argument("--only", choices=["moe", "muon", "norm", "fp8"], default=None)
    args = ap.parse_args()
    if not args.reference:
        ap.error("name the reference checkout with --reference or SPARK_GPT_REFERENCE")
    sys.dont_write_bytecode = True
    sys.path.insert(0, args.reference)
    import train  # the reference module, imported in place
    import torch.nn.functional as F

    if args.only in (None, "fp8"):
        make_fp8_golden(train, args.fp8_out)
    if args.only == "fp8":
        return
    if args.only in (None, "norm"):
        make_norm_golden(train, args.norm_out)
    if args.only == "norm":
        return
    if args.only != "moe":
        make_muon_golden(train, args.muon_out)
    if args.only == "muon":
        return

    torch.set_num_threads(max(1, os.cpu_count() or 1))
    cases = {}

    # 1. hand-built router case (tests/test_moe.py:34-55 shape)
    w = torch.tensor([[1.0, 0, 0], [0, 1.0, 0], [0, 0, 1.0], [-1.0, -1.0, -1.0]])
    hid = torch.tensor([[2.0, 1.0, 0.0], [0.0, 1.0, 3.0]])
    cfg = train.ModelConfig(hidden_size=3, num_experts=4, num_experts_per_tok=2)
    router = train.TopKRouter(cfg)
    with torch.no_grad():
        router.weight.copy_(w)
    lg, rw, sel = router(hid)
    cases["router_known"] = {"x": hid, "w_router": w, "top_k": 2, "norm": True,
                             "logits": lg.detach(), "weights": rw.detach(), "selected": sel}

    # 2. hand-routed experts case (tests/test_moe.py:57-98 shape), given routing
    torch.manual_seed(0)
    cfg = train.ModelConfig(hidden_size=4, num_experts=3, num_experts_per_tok=2,
                            moe_intermediate_size=3)
    ex = train.Experts(cfg)
    with torch.no_grad():
        ex.gate_up_proj.normal_(0.0, 0.2)
        ex.down_proj.normal_(0.0, 0.2)
    hidden = torch.randn(5, 4, requires_grad=True)
    selected = torch.tensor([[0, 1], [2, 0], [1, 2], [0, 2], [1, 0]])
    weights = torch.tensor([[0.7, 0.3], [0.6, 0.4], [0.8, 0.2], [0.55, 0.45], [0.9, 0.1]])
    probe = torch.randn(5, 4)
    out = ex(hidden, selected, weights)
    (out * probe).sum().backward()
    cases["experts_given_routing"] = {
        "x": hidden.detach(), "w_gate_up": ex.gate_up_proj.detach().clone(),
        "w_down": ex.down_proj.detach().clone(), "selected": selected, "weights": weights,
        "probe": probe, "out": out.detach(), "dx": hidden.grad,
        "dW_gate_up": ex.gate_up_proj.grad, "dW_down": ex.down_proj.grad}

    # 3. masked aux loss (tests/test_moe.py:146-184 shape)
    logits = torch.tensor([[3.0, 1.0, 0.0, -1.0], [0.0, 2.0, 1.0, -2.0],
                           [1.0, 0.0, 3.0, -1.0], [99.0, -99.0, -99.0, -99.0]], requires_grad=True)
    sel = logits.detach().softmax(-1).topk(2, dim=-1).indices
    valid = torch.tensor([True, True, True, False])
    loss, stats = train.global_load_balancing_loss((logits,), (sel,), valid, num_experts=4, top_k=2)
    loss.backward()
    cases["aux_masked"] = {"logits": logits.detach(), "selected": sel, "valid": valid,
                           "aux": loss.detach(), "d_logits": logits.grad,
                           **{f"stat_{k}": v.detach() for k, v in stats.items()}}
    logits = torch.randn(5, 4, generator=torch.Generator().manual_seed(3), requires_grad=True)
    sel = logits.detach().topk(2, dim=-1).indices
    loss, stats = train.global_load_balancing_loss(
        (logits,), (sel,), torch.zeros(5, dtype=torch.bool), num_experts=4, top_k=2)
    loss.backward()
    cases["aux_all_filler"] = {"logits": logits.detach(), "selected": sel,
                               "valid": torch.zeros(5, dtype=torch.bool),
                               "aux": loss.detach(), "d_logits": logits.grad}

    # 4. small full layers, stored whole
    for name, (T, H, E, k, I, norm, seed, filler) in {
        "layer_small": (256, 64, 8, 2, 32, True, 1, 0),
        "layer_nonorm_filler": (200, 48, 6, 3, 40, False, 2, 37),
        "layer_wide_k8": (128, 64, 64, 8, 16, True, 4, 5),
    }.items():
        x, w_r, w_gu, w_d, probe = seeded_inputs(T, H, E, I, seed, std_router=0.5)
        valid = torch.ones(T, dtype=torch.bool)
        if filler:
            valid[-filler:] = False
        res = run_layer(train, x, w_r, w_gu, w_d, probe, k, norm, valid)
        cases[name] = {"x": x, "w_router": w_r, "w_gate_up": w_gu, "w_down": w_d,
                       "probe": probe, "valid": valid, "top_k": k, "norm": norm, **res}

    # 5. config 1: inputs from a seed, outputs as slices + norms
    T, H, E, k, I = 4096, 256, 8, 2, 128
    x, w_r, w_gu, w_d, probe = seeded_inputs(T, H, E, I, 0)
    valid = torch.ones(T, dtype=torch.bool)
    res = run_layer(train, x, w_r, w_gu, w_d, probe, k, True, valid)
    c1 = {"shape": torch.tensor([T, H, E, k, I]), "seed": 0,
          "input_sums": torch.stack([t.double().sum() for t in (x, w_r, w_gu, w_d, probe)]),
          "selected": res["selected"].to(torch.int8), "permutation": res["permutation"].to(torch.int32),
          "offsets": res["offsets"], "aux": res["aux"]}
    for key in ("out", "logits", "routing_weights", "dx"):
        c1[key + "_head"] = res[key][:64].clone()
        c1[key + "_norm"] = res[key].double().norm()
    for key in ("dW_router", "dW_gate_up", "dW_down"):
        c1[key + "_norm"] = res[key].double().norm()
        c1[key + "_head"] = res[key].reshape(-1)[:4096].clone()
    for key, v in res.items():
        if key.startswith("stat_"):
            c1[key] = v
    cases["config1"] = c1

    torch.save(cases, args.out)
    print(f"wrote {args.out}: {', '.join(cases)}")


if __name__ == "__main__":
    main()
