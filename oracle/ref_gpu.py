"""The reference's own GPU eval path -- TEST INFRASTRUCTURE ONLY.

``forward_eval`` restates the ATen half of the reference
``MoCE.forward_eval`` (``MoCE.py:204-230``: fp32 upcast, adaptive average
pool, the gathered gate logit, the clamped temperature, the materialised
softmax weights) in torch, then calls the reference's compiled kernel
``fused_moce_forward_dynamic_temp`` (``moce_kernel.cu:1079-1153``: K2/K4, or
K3/K5 when H*W <= 16) from the extension that ``oracle/build_ref.py`` builds
from the reference sources.  It is the "GPU kernel to beat": the tests use it
as a second fp32 oracle and ``bench.py --impl reference`` times it.  Nothing
in the product package imports this module.
"""
from __future__ import annotations

import torch
import torch.nn.functional as F


def cache(L: torch.Tensor, k: int):
    """The reference eval cache (``MoCE.py:85-109``): int64 top-k indices,
    normalised selected logits, and the uncovered-channel mask (int32)."""
    _, idx = torch.topk(L, k, dim=1)
    sel = torch.gather(L, 1, idx)
    mean = sel.mean(dim=1, keepdim=True)
    std = sel.std(dim=1, keepdim=True).clamp(min=1.0)
    ln = (sel - mean) / std
    mask = torch.ones(L.shape[1], dtype=torch.int32, device=L.device)
    mask[idx.reshape(-1)] = 0
    return idx.contiguous(), ln.contiguous(), mask


def forward_eval(mod, x, idx, ln, gate_w, gate_b, mask, tmin, tmax, tau):
    """MoCE.forward_eval on the GPU: ATen pool / gate / softmax, then the
    reference kernel (stream: the legacy default stream, as the reference
    launches it).  `mod` is the loaded reference extension."""
    x32 = x.float() if x.dtype != torch.float32 else x
    pooled = F.adaptive_avg_pool2d(x32, 1).flatten(1)
    sel = pooled[:, idx]
    g = (sel * gate_w.reshape(-1)).sum(-1) + gate_b.reshape(-1)[0]
    temp = (tmin * tau + (tmax - tmin) * tau * torch.sigmoid(g)).clamp(min=1e-3)
    w = torch.softmax(ln.unsqueeze(0) / temp.unsqueeze(-1), dim=-1).contiguous()
    out, = mod.fused_moce_forward_dynamic_temp(x32.contiguous(), idx, w, mask)
    return out.to(x.dtype)
