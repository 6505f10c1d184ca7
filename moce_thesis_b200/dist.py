"""Data-parallel gradient exchange for MoCE layers.

The reference trains with DDP over NCCL (``test.py:855``), which all-reduces
every parameter gradient in 25 MB buckets.  For the MoCE layers the exchange
is small and fixed: the routing-logit gradient [E_r, C] and the shared
Linear(k,1) gate gradient [1, k] + [1] of each layer.  ``allreduce_moce_grads``
packs those of all layers into one flat fp32 buffer, runs ONE all-reduce
(sum) on the current stream and scatters the mean back -- one launch-latency
bound collective per step instead of one per bucket.

Works with any torch.distributed backend (NCCL on the GPUs, gloo in tests).
"""
from __future__ import annotations

from typing import Iterable, List

import torch
import torch.distributed as dist

from .moce import MoCE


def moce_layers(model: torch.nn.Module) -> List[MoCE]:
    return [m for m in model.modules() if isinstance(m, MoCE)]


def moce_grad_params(layers: Iterable[MoCE]) -> List[torch.nn.Parameter]:
    """The parameters whose gradients are exchanged, in a fixed order."""
    out = []
    for m in layers:
        out += [m.routing_logits, m.gate.weight, m.gate.bias]
    return out


def allreduce_moce_grads(model_or_layers, group=None, average: bool = True) -> int:
    """Average the MoCE gradients over the process group with one all-reduce.

    Parameters without a gradient contribute zeros (so every rank takes the
    same collective with the same size).  Returns the number of elements
    exchanged.  A no-op when torch.distributed is not initialised or the
    group has one rank.
    """
    layers = moce_layers(model_or_layers) if isinstance(model_or_layers, torch.nn.Module) else list(model_or_layers)
    params = moce_grad_params(layers)
    if not params or not dist.is_available() or not dist.is_initialized():
        return 0
    world = dist.get_world_size(group)
    if world == 1:
        return 0
    dev = params[0].device
    sizes = [p.numel() for p in params]
    flat = torch.empty(sum(sizes), dtype=torch.float32, device=dev)
    off = 0
    for p, n in zip(params, sizes):
        if p.grad is None:
            flat[off:off + n].zero_()
        else:
            flat[off:off + n].copy_(p.grad.reshape(-1))
        off += n
    dist.all_reduce(flat, op=dist.ReduceOp.SUM, group=group)
    if average:
        flat.div_(world)
    off = 0
    for p, n in zip(params, sizes):
        g = flat[off:off + n].view_as(p).to(p.dtype)
        if p.grad is None:
            p.grad = g.clone()
        else:
            p.grad.copy_(g)
        off += n
    return flat.numel()
