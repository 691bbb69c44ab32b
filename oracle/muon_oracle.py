"""CPU oracle for Muon on the packed 3-D expert weights (spark-gpt train.py).

TEST INFRASTRUCTURE ONLY: imported by ``tests/`` as the parity checker; the
product path (``spark_gpt_b200.muon``) never imports it.

It restates in plain torch-CPU arithmetic the Muon step that spark-gpt's
``MuonAdamWHybrid`` applies to each 3-D expert tensor (``experts.gate_up_proj``
(E,2I,H) and ``experts.down_proj`` (E,H,I), the Muon group of
``build_optimizer``, train.py:3066-3070):

* momentum        train.py:3001-3005   v <- lerp(v, g, 1-m); u <- lerp(g, v, m)
                                        (nesterov) as bf16, one rounding
* Newton-Schulz   train.py:2898-2927   per matrix (transposed when rows > cols):
                                        X /= ||X||_F + 1e-7 (bf16), then 5 x
                                        A = X X^T; B = c A A + b A; X = B X + a X
* update          train.py:3008-3024   p -= lr * max(1, rows/cols)^0.5 * X

The products follow the reference's CUDA path (_bmm_epilogue, train.py:2754-2800:
fp32 accumulation, alpha*acc + beta*C in fp32, one rounding to bf16); here the
fp32 products are torch-CPU matmuls of the bf16 operands.

Parity pin: ``tests/golden/make_golden.py`` runs the reference's
``MuonAdamWHybrid`` itself (its CPU bmm/baddbmm path) on seeded packed expert
tensors and stores the results in ``tests/golden/muon_golden.pt``;
``tests/test_oracle_golden.py`` checks this file against them.
"""

from __future__ import annotations

import torch

NS_COEFFS = (3.4445, -4.7750, 2.0315)  # train.py:2899


def _lerp(start, end, w):
    """torch.lerp's two branches (train.py:2806-2820 states the same formulas)."""
    if abs(w) < 0.5:
        return start + w * (end - start)
    return end - (end - start) * (1.0 - w)


def momentum_stage(g, v, momentum, nesterov=True):
    """-> (new momentum buffer fp32, staged bf16)."""
    g = g.float()
    v_new = _lerp(v.float(), g, 1.0 - momentum)
    staged = _lerp(g, v_new, momentum) if nesterov else v_new
    return v_new, staged.to(torch.bfloat16)


def _bf16_product(a, b, alpha=1.0, beta=0.0, c=None):
    acc = torch.bmm(a.float(), b.float()) * alpha
    if c is not None:
        acc = acc + beta * c.float()
    return acc.to(torch.bfloat16)


def newton_schulz(x, steps=5):
    """x (B, r, c) bf16 -> bf16 orthogonalised stack (train.py:2877-2927)."""
    a, b, c = NS_COEFFS
    X = x.to(torch.bfloat16)
    tall = X.shape[-2] > X.shape[-1]
    if tall:
        X = X.mT
    nrm = X.float().norm(dim=(-2, -1), keepdim=True).to(torch.bfloat16)
    d = (nrm.float() + 1e-7).to(torch.bfloat16)
    X = (X.float() / d.float()).to(torch.bfloat16)
    for _ in range(steps):
        A = _bf16_product(X, X.mT)
        B = _bf16_product(A, A, alpha=c, beta=b, c=A)
        X = _bf16_product(B, X, alpha=1.0, beta=a, c=X)
    return X.mT if tall else X


def muon_step(p, g, v, lr, momentum=0.95, nesterov=True, ns_steps=5):
    """One Muon step of a packed (E, rows, cols) fp32 parameter -> (p, v)."""
    v_new, staged = momentum_stage(g, v, momentum, nesterov)
    rows, cols = p.shape[-2], p.shape[-1]
    lr_eff = lr * max(1, rows / cols) ** 0.5
    ortho = newton_schulz(staged, ns_steps)
    return p.float() - lr_eff * ortho.float(), v_new
