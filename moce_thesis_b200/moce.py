"""The MoCE layer on the sm_100a kernels.

``MoCE`` keeps the public surface of the reference module
(Elianiluk/MoCE_thesis ``MoCE.py:11-230``): constructor arguments,
``routing_logits`` and ``gate`` parameters, the ``aux_loss`` attribute,
``build_eval_cache`` / ``clear_eval_cache``, ``forward_train`` /
``forward_eval``, the ``cached_*`` attributes and the state_dict keys.  What
changes is where the work runs:

* eval (``MoCE.py:204-230``): pass 1 (pool + gate + temperature) and pass 2
  (softmax + gather-mix + residual) are two native kernels; bf16/fp16 inputs
  are read and written natively (the reference upcasts to fp32, then casts
  back).
* train (``MoCE.py:153-201``): the same two passes under
  ``MoCEFunction``, whose backward is a native kernel chain (the reference
  trains through autograd over multi-GB gathered tensors).  Supports are
  re-selected every step, as the reference does (``MoCE.py:160``).

The auxiliary/coverage loss (``MoCE.py:118-151``) depends on the routing
logits only; its forward and gradient are native kernels too
(``AuxLossFunction``).
"""
from __future__ import annotations

import math
import os

import torch
import torch.nn as nn
import torch.nn.functional as F


def native():
    """The compiled binding ``moce_fixed.moce_cuda`` (raises if unbuilt)."""
    import moce_fixed.moce_cuda as m
    return m


# MOCE_CHECK_FAULTS=1: synchronise after every tensor-core forward and raise
# if one of its bounded waits ran out (the launch then left part of y
# unwritten).  Off by default, because the check synchronises the device.
_CHECK_FAULTS = os.environ.get("MOCE_CHECK_FAULTS", "0") not in ("", "0")


def check_faults(clear: bool = True) -> None:
    """Raise if a bounded wait inside a tensor-core kernel ran out since the
    last check (the device flag moce_tc_fault reads).  Synchronises the
    current device; call it after a batch of forwards."""
    m = native()
    if m.tc_fault(bool(clear)):
        info = m.tc_fault_info(bool(clear))
        names = ("set", "site", "parity", "unit", "block", "thread", "C", "HW", "E_r", "k", "B", "tiles", "N",
                 "waited_ns")
        raise RuntimeError("MoCE tensor-core kernel: a bounded wait ran out; the outputs of the launches since "
                           "the last check are incomplete (" + ", ".join(f"{n}={v}" for n, v in zip(names, info)) +
                           ")")


class _Route:
    """Native route cache of one logits tensor: int32 supports, normalised
    logits, coverage, optional transposed lists (backward) and, when k fits
    the scheduled mix kernel, the warp groups and support schedule.  The
    schedule is built on the first call that runs the scheduled mix, so
    inputs that take the tensor-core mix never pay for it."""

    __slots__ = ("idx", "ln", "mask", "meta", "toff", "tslot", "group_expert", "sched", "channels", "balance")

    def __init__(self, logits: torch.Tensor, k: int, transposed: bool, balance: bool = True):
        m = native()
        L = logits.detach().float().contiguous()
        self.idx, self.ln, self.mask, self.meta, self.toff, self.tslot = m.route_build(L, int(k), bool(transposed))
        self.group_expert = self.sched = None
        self.channels = int(L.shape[1])
        self.balance = bool(balance)

    def schedule(self):
        """(group_expert, sched) for the scheduled mix, or None if k does not fit it."""
        m = native()
        if self.sched is None and m.schedule_supported(int(self.idx.shape[1])):
            self.group_expert, self.sched = m.schedule_build(self.idx, self.channels, self.balance)
        return None if self.sched is None else (self.group_expert, self.sched)

    def forward(self, x, gate_w, gate_b, tmin_tau, trange_tau, want_T=False, out=None):
        """Both forward passes; returns (y, z, T).  T is None unless wanted.

        bf16/fp16 inputs with C <= 512 and k <= 64 whose tiles fit shared
        memory run the tensor-core mix; shapes with H*W <= 512 and k <= 64
        whose sample fits shared memory the lanes-over-pixels CUDA-core mix;
        shapes with H*W <= 1024 and k <= 128 the same mix reading X from
        global memory; other shapes the scheduled CUDA-core mix (k <= 44) or
        the general two passes.
        """
        m = native()
        k = int(self.idx.shape[1])
        if m.tc_supported(x, k):
            y, z, T = m.forward_tc(x, self.idx, self.ln, self.mask, self.meta, gate_w, gate_b, float(tmin_tau),
                                   float(trange_tau), bool(want_T), out)
            if _CHECK_FAULTS:
                check_faults()
            return y, z, (T if want_T else None)
        if m.px_supported(x, k):
            y, z, T = m.forward_px(x, self.idx, self.ln, self.mask, self.meta, gate_w, gate_b, float(tmin_tau),
                                   float(trange_tau), bool(want_T), out)
            return y, z, (T if want_T else None)
        if m.gx_supported(x, k):
            y, z, T = m.forward_gx(x, self.idx, self.ln, self.mask, self.meta, gate_w, gate_b, float(tmin_tau),
                                   float(trange_tau), bool(want_T), out)
            return y, z, (T if want_T else None)
        if self.schedule() is not None:
            y, z, T = m.forward_scheduled(x, self.ln, self.mask, self.meta, self.group_expert, self.sched, gate_w,
                                          gate_b, float(tmin_tau), float(trange_tau), bool(want_T), out)
            return y, z, (T if want_T else None)
        z, T = m.gate_temperature(x, self.idx, gate_w, gate_b, float(tmin_tau), float(trange_tau))
        return m.mix(x, self.idx, self.ln, T, self.mask, out), z, T


class MoCEFunction(torch.autograd.Function):
    """Y = MoCE(X; L, gate) with the native forward and backward.

    Inputs: x [B, C, H, W]; logits [E_r, C]; gate_w [1, k]; gate_b [1]; the
    temperature constants tmin_tau = temp_min * tau and
    trange_tau = (temp_max - temp_min) * tau; and a route cache built from
    the same logits (with transposed lists when gradients are needed).
    """

    @staticmethod
    def forward(ctx, x, logits, gate_w, gate_b, tmin_tau, trange_tau, route):
        m = native()
        x = x.contiguous()
        gw = gate_w.detach().reshape(-1).float().contiguous()
        gb = gate_b.detach().reshape(-1).float().contiguous()
        y, z, T = route.forward(x, gw, gb, tmin_tau, trange_tau, want_T=True)
        ctx.save_for_backward(x, logits.detach(), gw, gb, z, T)
        ctx.route = route
        ctx.consts = (float(tmin_tau), float(trange_tau))
        ctx.gate_shapes = (gate_w.shape, gate_b.shape)
        return y

    @staticmethod
    def backward(ctx, dy):
        x, logits, gw, gb, z, T = ctx.saved_tensors
        r = ctx.route
        if r.toff.numel() == 0:
            raise RuntimeError("MoCEFunction: route cache was built without transposed lists")
        dx, dL, dgw, dgb = native().backward(
            x, dy.to(x.dtype).contiguous(), logits.float().contiguous(), r.idx, r.ln, r.mask, r.meta, r.toff,
            r.tslot, gw, gb, ctx.consts[0], ctx.consts[1], z, T)
        wshape, bshape = ctx.gate_shapes
        return (dx, dL.to(logits.dtype), dgw.reshape(wshape), dgb.reshape(bshape), None, None, None)


class AuxLossFunction(torch.autograd.Function):
    """The auxiliary (coverage) loss of the routing logits on the native
    kernels: balance + specialisation + diversity of ``MoCE.py:118-151``
    (softmax over channels, usage variance, per-channel entropy, mean
    off-diagonal overlap), forward and gradient, with deterministic
    reductions.  Returns a 0-d float32 tensor."""

    @staticmethod
    def forward(ctx, logits, tau, balance_w, spec_w, div_w, log_target):
        L = logits.detach().float().contiguous()
        consts = (float(tau), float(balance_w), float(spec_w), float(div_w), float(log_target))
        out = native().aux_loss(L, *consts)
        ctx.save_for_backward(L)
        ctx.consts = consts
        ctx.ldtype = logits.dtype
        return out

    @staticmethod
    def backward(ctx, go):
        (L,) = ctx.saved_tensors
        dL = native().aux_loss_backward(L, *ctx.consts, go.detach().float().reshape(1).contiguous())
        return dL.to(ctx.ldtype), None, None, None, None, None


class MoCEFunctionT(torch.autograd.Function):
    """Y = MoCE(X; L, T) with the temperatures T [B, E_r] given.

    For a gate the caller differentiates itself (the two-layer gate): the
    native forward from given temperatures and the native backward, which
    returns dX (mix and residual terms), dL and dT; autograd carries dT back
    through the caller's gate (and its dz / H*W term into dX).
    """

    @staticmethod
    def forward(ctx, x, logits, T, route):
        x = x.contiguous()
        Tc = T.detach().float().contiguous()
        y = native().forward_given_t(x, route.idx, route.ln, route.mask, route.meta, Tc)
        if _CHECK_FAULTS:
            check_faults()
        ctx.save_for_backward(x, logits.detach(), Tc)
        ctx.route = route
        return y

    @staticmethod
    def backward(ctx, dy):
        x, logits, T = ctx.saved_tensors
        r = ctx.route
        if r.toff.numel() == 0:
            raise RuntimeError("MoCEFunctionT: route cache was built without transposed lists")
        dx, dL, dT = native().backward_t(x, dy.to(x.dtype).contiguous(), logits.float().contiguous(), r.idx, r.ln,
                                         r.mask, r.meta, r.toff, r.tslot, T)
        return dx, dL.to(logits.dtype), dT, None


class MoCE(nn.Module):
    """Mixture of Channel Experts: E-1 routed experts + 1 residual expert.

    Same constructor and attributes as the reference (``MoCE.py:26-79``).
    ``gate_type="mlp"`` (an addition, off by default) replaces the reference's
    shared Linear(k,1) temperature gate with a two-layer gate
    C -> C/16 -> E-1 with ReLU and Kaiming-normal weights, ``gate_mlp``.
    """

    def __init__(self, in_channels=256, sampling_factor=4, k=8, tau=1.0, balance_weight=0.05,
                 specialization_weight=0.1, diversity_weight=0.01, temp_min=0.2, temp_max=5.0,
                 gate_type="linear"):
        super().__init__()
        if gate_type not in ("linear", "mlp"):
            raise ValueError("gate_type must be 'linear' or 'mlp'")
        self.gate_type = gate_type
        self.in_channels = in_channels
        self.num_experts = in_channels // sampling_factor
        self.k = k
        self.tau = tau
        self.balance_weight = balance_weight
        self.specialization_weight = specialization_weight
        self.diversity_weight = diversity_weight
        self.temp_min = temp_min
        self.temp_max = temp_max
        self._last_temperature = None
        self.aux_loss = 0.0
        routed = max(self.num_experts - 1, 1)
        self.target_experts_per_channel = routed * self.k / max(float(self.in_channels), 1.0)
        self.routing_logits = nn.Parameter(torch.randn(self.num_experts - 1, in_channels))
        self.gate = nn.Linear(k, 1)
        nn.init.xavier_uniform_(self.gate.weight)
        nn.init.zeros_(self.gate.bias)
        self.register_buffer("cached_indices", None)
        self.register_buffer("cached_selected_logits_norm", None)
        self.register_buffer("cached_mask_int", None, persistent=False)
        self.cached_temp_min_tau = None
        self.cached_temp_range_tau = None
        self.cached_gate_weight = None
        self.cached_gate_bias = None
        self._route = None        # native eval cache (int32 supports etc.)
        self._f32_cache = {}      # fp32 gate parameters / folded BatchNorm, keyed by tensor versions
        if gate_type == "mlp":
            self.reset_gate_mlp()

    def reset_gate_mlp(self):
        """(Re)create the two-layer gate for the current ``in_channels`` and
        ``num_experts`` (call it after changing ``num_experts``): Linear(C,
        C/16) -> ReLU -> Linear(C/16, E-1), weights Kaiming-normal (ReLU
        gain), biases zero, on the device of ``routing_logits``."""
        hd = max(1, self.in_channels // 16)
        mlp = nn.Sequential(nn.Linear(self.in_channels, hd), nn.ReLU(), nn.Linear(hd, self.num_experts - 1))
        for lin in (mlp[0], mlp[2]):
            nn.init.kaiming_normal_(lin.weight, nonlinearity="relu")
            nn.init.zeros_(lin.bias)
        self.gate_mlp = mlp.to(self.routing_logits.device)

    def _mlp_params(self):
        lin1, lin2 = self.gate_mlp[0], self.gate_mlp[2]
        return tuple(t.detach().float().contiguous() for t in (lin1.weight, lin1.bias, lin2.weight, lin2.bias))

    # ------------------------------------------------------------------
    def forward(self, x):
        return self.forward_train(x) if self.training else self.forward_eval(x)

    # ------------------------------------------------------------------
    def build_eval_cache(self):
        """Select supports, normalise their logits and mark uncovered channels.

        Runs the native route-build kernel; fills the reference's cached_*
        attributes (``MoCE.py:85-109``) plus the int32 native cache.
        """
        with torch.no_grad():
            route = _Route(self.routing_logits, self.k, transposed=False)
            self._route = route
            self.cached_indices = route.idx.long()
            self.cached_selected_logits_norm = route.ln.to(self.routing_logits.dtype)
            self.cached_mask_int = route.mask
        self.cached_temp_min_tau = float(self.temp_min) * float(self.tau)
        self.cached_temp_range_tau = float(self.temp_max - self.temp_min) * float(self.tau)
        self.cached_gate_weight = self.gate.weight.squeeze(0).contiguous()
        # as in the reference, .contiguous() of the (contiguous) bias returns
        # the Parameter itself, which nn.Module registers under this name
        self.cached_gate_bias = self.gate.bias.contiguous()

    def clear_eval_cache(self):
        self.cached_indices = None
        self.cached_selected_logits_norm = None
        self.cached_mask_int = None
        self._route = None
        self._f32_cache = {}

    # ------------------------------------------------------------------
    def _compute_aux_losses(self, x, E_routed, tau):
        """Balance + specialisation + diversity losses (``MoCE.py:118-151``),
        on the native kernels (AuxLossFunction): the mean off-diagonal of
        P P^T is (sum of squared column sums - sum of squares) / (E (E - 1)),
        so the E x C x E product is never formed."""
        target = math.log(max(float(self.target_experts_per_channel), 1.0))
        self.aux_loss = AuxLossFunction.apply(self.routing_logits, tau, self.balance_weight,
                                              self.specialization_weight, self.diversity_weight, target)

    def forward_train(self, x):
        B, C, H, W = x.shape
        E_routed = self.num_experts - 1
        tau = max(float(self.tau), 1e-4)
        with torch.no_grad():
            # supports are re-selected every step; the warp grouping is the
            # identity here (balancing is a sequential pass worth doing once)
            route = _Route(self.routing_logits, self.k, transposed=True, balance=False)
        self._compute_aux_losses(x, E_routed, tau)
        if self.gate_type == "mlp":
            # the two-layer gate in torch (3 small ops), differentiated by
            # autograd; the mix and its backward native, from the given T
            z = x.float().mean(dim=(2, 3))
            g = self.gate_mlp(z)
            T = (self.temp_min * tau + (self.temp_max - self.temp_min) * tau * torch.sigmoid(g)).clamp(min=1e-3)
            return MoCEFunctionT.apply(x, self.routing_logits, T, route)
        y = MoCEFunction.apply(x, self.routing_logits, self.gate.weight, self.gate.bias,
                               self.temp_min * tau, (self.temp_max - self.temp_min) * tau, route)
        return y

    # ------------------------------------------------------------------
    def forward_eval(self, x):
        if self.cached_indices is None:
            raise RuntimeError("MoCE eval cache not built. Call build_moce_cache(model) before eval.")
        route = self._route
        if route is None or route.idx.device != x.device:
            # cache restored from a state_dict, or moved: rebuild the native part
            route = _Route(self.routing_logits, self.k, transposed=False)
            self._route = route
        return self._eval_native(route, x.contiguous())

    def _eval_native(self, route, x, out=None):
        """The eval forward of either gate on the native kernels, into `out`
        when given: the fused tensor-core chain (pass 1 -> temperatures ->
        mix) where it takes the input, else pass 1, the gate and the
        CUDA-core mix."""
        if self.gate_type == "mlp":
            m = native()
            w1, b1, w2, b2 = self._mlp_params()
            tmin_tau, trange_tau = float(self.cached_temp_min_tau), float(self.cached_temp_range_tau)
            if m.tc_supported(x, self.k):
                y = m.forward_tc_mlp(x, route.idx, route.ln, route.mask, route.meta, w1, b1, w2, b2, tmin_tau,
                                     trange_tau, out)[0]
            else:
                y, z = m.pool_residual(x, route.mask, route.meta, int(route.idx.shape[0]), out)
                T, _ = m.temperature_mlp(z, w1, b1, w2, b2, tmin_tau, trange_tau)
                m.mix_given_t(x, route.idx, route.ln, route.mask, T, y)
            if _CHECK_FAULTS:
                check_faults()
            return y
        gw, gb = self._gate_f32()
        y, _, _ = route.forward(x, gw, gb, self.cached_temp_min_tau, self.cached_temp_range_tau, False, out)
        return y

    def _cached_f32(self, name, tensors, make, extra=()):
        """make() once per version of `tensors` (and value of `extra`): an
        eval forward otherwise launches a conversion kernel per parameter per
        call."""
        key = tuple((t.data_ptr(), t._version, t.dtype, t.device) if t is not None else None
                    for t in tensors) + tuple(extra)
        hit = self._f32_cache.get(name)
        if hit is not None and hit[0] == key:
            return hit[1]
        with torch.no_grad():
            val = make()
        self._f32_cache[name] = (key, val)
        return val

    def _gate_f32(self):
        """The shared gate's weight [k] and bias [1] in fp32, contiguous."""
        w, b = self.cached_gate_weight, self.cached_gate_bias
        return self._cached_f32("gate", (w, b), lambda: (w.detach().reshape(-1).float().contiguous(),
                                                          b.detach().reshape(-1).float().contiguous()))

    # ------------------------------------------------------------------
    def forward_eval_bn_relu(self, x, bn, relu=True):
        """``relu(bn(forward_eval(x)))`` for an eval-mode ``BatchNorm2d`` over
        the layer's E outputs: the sequence MoCE -> bn1 -> relu1 of
        ``BottleneckWithMoCEProjection.forward`` (models_unified.py:155-165).

        On the tensor-core path the BatchNorm, folded to a per-channel
        scale / shift, and the ReLU are applied to each output in the mix's
        store (one pass over Y instead of three).  The CUDA-core paths run
        forward_eval and then the folded BatchNorm and ReLU as one native
        pass over Y (``moce_bn_act``); a BatchNorm in training mode, or a CPU
        tensor, runs the torch ops.
        """
        if self.cached_indices is None:
            raise RuntimeError("MoCE eval cache not built. Call build_moce_cache(model) before eval.")
        m = native()
        use_bn_stats = (not bn.training) and bn.running_mean is not None and bn.running_var is not None
        if not use_bn_stats or not x.is_cuda:
            y = bn(self.forward_eval(x))
            return F.relu(y) if relu else y

        def fold():
            inv = torch.rsqrt(bn.running_var.float() + float(bn.eps))
            scale = inv if bn.weight is None else bn.weight.float() * inv
            shift = -bn.running_mean.float() * scale
            if bn.bias is not None:
                shift = shift + bn.bias.float()
            return scale.contiguous(), shift.contiguous()
        scale, shift = self._cached_f32("bn", (bn.running_mean, bn.running_var, bn.weight, bn.bias), fold,
                                        (float(bn.eps),))
        if not m.tc_supported(x, self.k) or self.gate_type == "mlp":
            # the CUDA-core paths: the layer, then the folded BatchNorm and the
            # ReLU as one native pass in place
            y = self.forward_eval(x)
            return m.bn_act(y, scale, shift, relu=bool(relu), out=y)
        route = self._route
        if route is None or route.idx.device != x.device:
            route = _Route(self.routing_logits, self.k, transposed=False)
            self._route = route
        gw, gb = self._gate_f32()
        y = m.forward_tc_ep(x.contiguous(), route.idx, route.ln, route.mask, route.meta, gw, gb,
                            float(self.cached_temp_min_tau), float(self.cached_temp_range_tau),
                            scale, shift, bool(relu))
        if _CHECK_FAULTS:
            check_faults()
        return y

    # ------------------------------------------------------------------
    def forward_host(self, x, out=None, slices=8):
        """Eval forward of a batch in host memory, with the result in host memory.

        The batch is cut into ``slices`` runs of samples that flow through
        three CUDA streams of this layer's device: the host-to-device copy of
        run i+1, the two passes of run i and the device-to-host copy of run
        i-1 overlap, so both PCIe directions and the GPU are busy at once
        (the routed output is four times the input at the stage-4 shape, so
        the device-to-host copy sets the pace).  Two device buffers per
        direction are reused across runs and calls.

        ``x``: CPU tensor [B, C, H, W], pinned for the copies to be
        asynchronous.  ``out``: CPU tensor [B, E, H, W] of x's dtype
        (allocated pinned when not given).  The call returns once the work
        is queued; the current CUDA stream waits on the last copy, so
        synchronizing that stream (or the device) completes the result, and
        ``x`` must not change before then.
        """
        if self.cached_indices is None:
            raise RuntimeError("MoCE eval cache not built. Call build_moce_cache(model) before eval.")
        if x.is_cuda:
            raise ValueError("forward_host: x must be a host tensor")
        dev = self.routing_logits.device
        if dev.type != "cuda":
            raise RuntimeError("forward_host: the layer must be on a CUDA device")
        B, C, H, W = x.shape
        E = self.num_experts
        if out is None:
            out = torch.empty(B, E, H, W, dtype=x.dtype, pin_memory=True)
        if B == 0:
            return out
        route = self._route
        if route is None or route.idx.device != dev:
            route = _Route(self.routing_logits, self.k, transposed=False)
            self._route = route
        n = max(1, min(int(slices), B))
        run = (B + n - 1) // n
        st = self.__dict__.get("_host_pipe")
        key = (dev, run, C, H, W, E, x.dtype)
        if st is None or st["key"] != key:
            if st is not None:
                # the old buffers return to the allocator on the current
                # stream: order them after the side streams' last use
                cur0 = torch.cuda.current_stream(dev)
                cur0.wait_stream(st["h2d"])
                cur0.wait_stream(st["d2h"])
            with torch.cuda.device(dev):
                st = {"key": key,
                      "h2d": torch.cuda.Stream(dev), "d2h": torch.cuda.Stream(dev),
                      "xb": [torch.empty(run, C, H, W, dtype=x.dtype, device=dev) for _ in range(2)],
                      "yb": [torch.empty(run, E, H, W, dtype=x.dtype, device=dev) for _ in range(2)],
                      "in": [torch.cuda.Event() for _ in range(2)],
                      "done": [torch.cuda.Event() for _ in range(2)],
                      "out": [torch.cuda.Event() for _ in range(2)],
                      "used": [False, False]}
            self.__dict__["_host_pipe"] = st
        cur = torch.cuda.current_stream(dev)
        h2d, d2h = st["h2d"], st["d2h"]
        last = None
        for i, b0 in enumerate(range(0, B, run)):
            b1 = min(B, b0 + run)
            j = i % 2
            xb, yb = st["xb"][j][:b1 - b0], st["yb"][j][:b1 - b0]
            if st["used"][j]:
                h2d.wait_event(st["done"][j])              # the passes that read xb are done
            with torch.cuda.stream(h2d):
                xb.copy_(x[b0:b1], non_blocking=True)
                st["in"][j].record(h2d)
            cur.wait_event(st["in"][j])
            if st["used"][j]:
                cur.wait_event(st["out"][j])               # the copy that read yb is done
            self._eval_native(route, xb, yb)
            st["done"][j].record(cur)
            d2h.wait_event(st["done"][j])
            with torch.cuda.stream(d2h):
                out[b0:b1].copy_(yb, non_blocking=True)
                st["out"][j].record(d2h)
            st["used"][j] = True
            last = st["out"][j]
        cur.wait_event(last)
        return out
