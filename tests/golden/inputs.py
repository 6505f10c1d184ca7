"""Seeded synthetic inputs for the MoCE parity cases.

Shared by ``make_golden.py`` (which runs the reference ``MoCE.py`` on them, in
the development container only) and by the tests, which regenerate the same
tensors from the same seeds with torch's CPU generator.  Order of draws per
case: ``torch.manual_seed(seed)``, then X, then the routing logits L, then the
gate parameters, then dY -- the order the workload description fixes.

Each case is a dict with the layer hyper-parameters; ``make_inputs`` returns
float32 CPU tensors.
"""
from __future__ import annotations

import math

import torch

# name -> parameters.  E counts the residual expert (E_r = E - 1 routed).
CASES = {
    # non-trivial residual: 15*4 = 60 picks over 64 channels
    "small_resid": dict(B=2, C=64, H=5, W=5, E=16, k=4, tmin=0.1, tmax=10.0, tau=1.0, seed=1),
    # every channel covered, odd spatial size
    "covered_odd": dict(B=2, C=32, H=3, W=5, E=33, k=8, tmin=0.1, tmax=10.0, tau=1.0, seed=2),
    # 1x1 spatial extent
    "hw1": dict(B=3, C=16, H=1, W=1, E=5, k=3, tmin=0.2, tmax=5.0, tau=1.0, seed=3),
    # temperature clamp (1e-3) active for most (b, e)
    "tclamp": dict(B=2, C=24, H=4, W=4, E=9, k=4, tmin=0.1, tmax=10.0, tau=2e-4, seed=4),
    # selected-logit std below 1 -> scale clamped to 1
    "std_small": dict(B=2, C=40, H=3, W=3, E=11, k=6, tmin=0.2, tmax=5.0, tau=1.0, seed=5, lscale=0.1),
    # large logit spread -> std > 1 branch
    "std_large": dict(B=2, C=40, H=3, W=3, E=11, k=6, tmin=0.2, tmax=5.0, tau=1.0, seed=6, lscale=4.0),
    # k == C: every expert selects every channel
    "k_eq_c": dict(B=2, C=8, H=2, W=3, E=4, k=8, tmin=0.1, tmax=10.0, tau=1.0, seed=7),
    # a single routed expert
    "e2": dict(B=2, C=12, H=3, W=3, E=2, k=5, tmin=0.1, tmax=10.0, tau=1.0, seed=8),
    # wide k (> 32 and not a multiple of 32)
    "k40": dict(B=2, C=96, H=2, W=5, E=7, k=40, tmin=0.1, tmax=10.0, tau=1.0, seed=9),
    # the single-layer workload (N=8, C=256, 14x14, E=1024, k=16), stored as summaries
    "cfg1": dict(B=8, C=256, H=14, W=14, E=1024, k=16, tmin=0.1, tmax=10.0, tau=1.0, seed=0,
                 summary=True),
}


def make_inputs(case: dict, with_grad: bool = True):
    """Return dict of float32 CPU tensors X, L, gate_w [1,k], gate_b [1], dY."""
    B, C, H, W, E, k = (case[n] for n in ("B", "C", "H", "W", "E", "k"))
    g = torch.Generator().manual_seed(case["seed"])
    # post-ReLU activations: |N(0,1)| (half-normal)
    X = torch.randn(B, C, H, W, generator=g).abs()
    L = torch.randn(E - 1, C, generator=g) * float(case.get("lscale", 1.0))
    # nn.Linear(k, 1) with xavier_uniform weight and zero bias (MoCE.py:66-68)
    bound = math.sqrt(6.0 / (k + 1))
    gate_w = (torch.rand(1, k, generator=g) * 2.0 - 1.0) * bound
    gate_b = torch.zeros(1)
    if case.get("gate_bias"):
        gate_b = torch.randn(1, generator=g) * float(case["gate_bias"])
    out = dict(X=X, L=L, gate_w=gate_w, gate_b=gate_b)
    if with_grad:
        out["dY"] = torch.randn(B, E, H, W, generator=g)
    return out


def tie_logits(E_r: int, C: int, seed: int) -> torch.Tensor:
    """Integer-valued logits in [-2, 2]: rows full of ties."""
    g = torch.Generator().manual_seed(seed)
    return torch.randint(-2, 3, (E_r, C), generator=g).float()
