"""Torch-tensor conveniences over the C ABI (ctypes), used by the GPU tests.

Every helper calls exactly one or two entry points of ``include/moce_b200.h``
with device pointers of torch tensors and the current stream; outputs are
allocated here (the entry points never allocate).
"""
from __future__ import annotations

import torch

from moce_thesis_b200 import capi
from moce_thesis_b200.capi import call, dtype_code, ptr, stream_handle


def route_build(L: torch.Tensor, k: int, transposed: bool = True):
    E_r, C = L.shape
    dev = L.device
    i32 = dict(dtype=torch.int32, device=dev)
    idx = torch.empty(E_r, k, **i32)
    ln = torch.empty(E_r, k, dtype=torch.float32, device=dev)
    mask = torch.empty(C, **i32)
    meta = torch.empty(2, **i32)
    toff = torch.empty(C + 1, **i32) if transposed else None
    tslot = torch.empty(E_r * k, **i32) if transposed else None
    call("moce_route_build", ptr(L), E_r, C, k, ptr(idx), ptr(ln), ptr(mask), ptr(meta), ptr(toff), ptr(tslot),
         stream_handle())
    return dict(idx=idx, ln=ln, mask=mask, meta=meta, toff=toff, tslot=tslot)


def gate_temperature(x, idx, gate_w, gate_b, tmin_tau, trange_tau, pooled=None):
    B, C = x.shape[:2]
    HW = x.shape[2] * x.shape[3]
    E_r, k = idx.shape
    z = torch.empty(B, C, dtype=torch.float32, device=x.device)
    T = torch.empty(B, E_r, dtype=torch.float32, device=x.device)
    call("moce_gate_temperature", ptr(x), dtype_code(x), ptr(pooled), B, C, HW, ptr(idx), E_r, k, ptr(gate_w),
         ptr(gate_b), tmin_tau, trange_tau, ptr(z), ptr(T), stream_handle())
    return z, T


def mix(x, idx, ln, T, mask):
    B, C, H, W = x.shape
    E_r, k = idx.shape
    y = torch.empty(B, E_r + 1, H, W, dtype=x.dtype, device=x.device)
    call("moce_mix", ptr(x), dtype_code(x), B, C, H * W, ptr(idx), ptr(ln), ptr(T), E_r, k, ptr(mask), ptr(y),
         stream_handle())
    return y


def schedule_build(idx, C, balance=True):
    E_r, k = idx.shape
    G = (E_r + 31) // 32
    S = capi.lib().moce_schedule_steps(k)
    ge = torch.empty(G * 32, dtype=torch.int32, device=idx.device)
    sched = torch.empty(G * S * 32, dtype=torch.int32, device=idx.device)
    call("moce_schedule_build", ptr(idx), E_r, C, k, 1 if balance else 0, ptr(ge), ptr(sched), stream_handle())
    return ge, sched


def schedule_supported(k):
    return capi.lib().moce_schedule_steps(k) <= 52


def forward_fast(x, r, gate_w, gate_b, tmin_tau, trange_tau, want_T=True):
    """Fast path through the C ABI: pass 1 (pool + residual), pass 2 (scheduled mix)."""
    B, C, H, W = x.shape
    E_r, k = r["idx"].shape
    y = torch.empty(B, E_r + 1, H, W, dtype=x.dtype, device=x.device)
    z = torch.empty(B, C, dtype=torch.float32, device=x.device)
    T = torch.empty(B, E_r, dtype=torch.float32, device=x.device) if want_T else None
    call("moce_pool_residual", ptr(x), dtype_code(x), B, C, H * W, ptr(r["mask"]), ptr(r["meta"]), ptr(z), ptr(y),
         E_r, stream_handle())
    call("moce_mix_scheduled", ptr(x), dtype_code(x), B, C, H * W, ptr(z), ptr(r["ln"]), E_r, k,
         ptr(r["group_expert"]), ptr(r["sched"]), ptr(gate_w), ptr(gate_b), tmin_tau, trange_tau, ptr(y), ptr(T),
         stream_handle())
    return y, z, T


def tc_supported(x, k):
    C, HW = x.shape[1], x.shape[2] * x.shape[3]
    return bool(capi.lib().moce_tc_supported(dtype_code(x), C, HW, k))


def forward_tc(x, r, gate_w, gate_b, tmin_tau, trange_tau, want_T=True):
    """Tensor-core path through the C ABI: pass 1 (pool + residual + operand
    staging), then the tcgen05 mix with the gate computed from z."""
    B, C, H, W = x.shape
    E_r, k = r["idx"].shape
    y = torch.empty(B, E_r + 1, H, W, dtype=x.dtype, device=x.device)
    z = torch.empty(B, C, dtype=torch.float32, device=x.device)
    T = torch.empty(B, E_r, dtype=torch.float32, device=x.device) if want_T else None
    xs = torch.empty(capi.lib().moce_tc_stage_bytes(B, C, H * W), dtype=torch.uint8, device=x.device)
    call("moce_pool_stage", ptr(x), dtype_code(x), B, C, H * W, ptr(r["mask"]), ptr(r["meta"]), ptr(z), ptr(y),
         E_r, ptr(xs), stream_handle())
    call("moce_mix_tc", ptr(xs), dtype_code(x), B, C, H * W, ptr(z), ptr(r["idx"]), ptr(r["ln"]), E_r, k,
         ptr(gate_w), ptr(gate_b), tmin_tau, trange_tau, ptr(y), ptr(T), stream_handle())
    return y, z, T


def forward_tc_t(x, r, T):
    """Tensor-core path with given temperatures: pass 1, then moce_mix_tc_t."""
    B, C, H, W = x.shape
    E_r, k = r["idx"].shape
    y = torch.empty(B, E_r + 1, H, W, dtype=x.dtype, device=x.device)
    z = torch.empty(B, C, dtype=torch.float32, device=x.device)
    xs = torch.empty(capi.lib().moce_tc_stage_bytes(B, C, H * W), dtype=torch.uint8, device=x.device)
    call("moce_pool_stage", ptr(x), dtype_code(x), B, C, H * W, ptr(r["mask"]), ptr(r["meta"]), ptr(z), ptr(y),
         E_r, ptr(xs), stream_handle())
    call("moce_mix_tc_t", ptr(xs), dtype_code(x), B, C, H * W, ptr(T), ptr(r["idx"]), ptr(r["ln"]), E_r, k, ptr(y),
         stream_handle())
    return y


def temperature(z, idx, gate_w, gate_b, tmin_tau, trange_tau):
    B, C = z.shape
    E_r, k = idx.shape
    T = torch.empty(B, E_r, dtype=torch.float32, device=z.device)
    call("moce_temperature", ptr(z), B, C, ptr(idx), E_r, k, ptr(gate_w), ptr(gate_b), tmin_tau, trange_tau, ptr(T),
         stream_handle())
    return T


def temperature_mlp(z, w1, b1, w2, b2, tmin_tau, trange_tau):
    B, C = z.shape
    Hd, E_r = w1.shape[0], w2.shape[0]
    T = torch.empty(B, E_r, dtype=torch.float32, device=z.device)
    h = torch.empty(B, Hd, dtype=torch.float32, device=z.device)
    call("moce_temperature_mlp", ptr(z), B, C, Hd, E_r, ptr(w1), ptr(b1), ptr(w2), ptr(b2), tmin_tau, trange_tau,
         ptr(h), ptr(T), stream_handle())
    return T, h


def forward_tc_mlp(x, r, w1, b1, w2, b2, tmin_tau, trange_tau):
    """Tensor-core forward with the two-layer gate, one call (three launches)."""
    B, C, H, W = x.shape
    E_r, k = r["idx"].shape
    Hd = w1.shape[0]
    y = torch.empty(B, E_r + 1, H, W, dtype=x.dtype, device=x.device)
    z = torch.empty(B, C, dtype=torch.float32, device=x.device)
    T = torch.empty(B, E_r, dtype=torch.float32, device=x.device)
    h = torch.empty(B, Hd, dtype=torch.float32, device=x.device)
    xs = torch.empty(capi.lib().moce_tc_stage_bytes(B, C, H * W), dtype=torch.uint8, device=x.device)
    call("moce_forward_tc_mlp", ptr(x), dtype_code(x), B, C, H * W, ptr(r["mask"]), ptr(r["meta"]), ptr(r["idx"]),
         ptr(r["ln"]), E_r, k, Hd, ptr(w1), ptr(b1), ptr(w2), ptr(b2), tmin_tau, trange_tau, ptr(z), ptr(h), ptr(xs),
         ptr(y), ptr(T), stream_handle())
    return y, z, T, h


def px_supported(x, k):
    C, HW = x.shape[1], x.shape[2] * x.shape[3]
    return bool(capi.lib().moce_px_supported(dtype_code(x), C, HW, k))


def forward_px(x, r, gate_w, gate_b, tmin_tau, trange_tau, want_T=True):
    """Lanes-over-pixels CUDA-core path through the C ABI: pass 1 (pool + residual), then the mix."""
    B, C, H, W = x.shape
    E_r, k = r["idx"].shape
    y = torch.empty(B, E_r + 1, H, W, dtype=x.dtype, device=x.device)
    z = torch.empty(B, C, dtype=torch.float32, device=x.device)
    T = torch.empty(B, E_r, dtype=torch.float32, device=x.device) if want_T else None
    call("moce_pool_residual", ptr(x), dtype_code(x), B, C, H * W, ptr(r["mask"]), ptr(r["meta"]), ptr(z), ptr(y),
         E_r, stream_handle())
    call("moce_mix_px", ptr(x), dtype_code(x), B, C, H * W, ptr(z), ptr(r["idx"]), ptr(r["ln"]), E_r, k,
         ptr(gate_w), ptr(gate_b), tmin_tau, trange_tau, ptr(y), ptr(T), stream_handle())
    return y, z, T


def gx_supported(x, k):
    C, HW = x.shape[1], x.shape[2] * x.shape[3]
    return bool(capi.lib().moce_gx_supported(dtype_code(x), C, HW, k))


def forward_gx(x, r, gate_w, gate_b, tmin_tau, trange_tau, want_T=True):
    """CUDA-core path reading X from global memory: pass 1 (pool + residual), then the mix."""
    B, C, H, W = x.shape
    E_r, k = r["idx"].shape
    y = torch.empty(B, E_r + 1, H, W, dtype=x.dtype, device=x.device)
    z = torch.empty(B, C, dtype=torch.float32, device=x.device)
    T = torch.empty(B, E_r, dtype=torch.float32, device=x.device) if want_T else None
    call("moce_pool_residual", ptr(x), dtype_code(x), B, C, H * W, ptr(r["mask"]), ptr(r["meta"]), ptr(z), ptr(y),
         E_r, stream_handle())
    call("moce_mix_gx", ptr(x), dtype_code(x), B, C, H * W, ptr(z), ptr(r["idx"]), ptr(r["ln"]), E_r, k,
         ptr(gate_w), ptr(gate_b), tmin_tau, trange_tau, ptr(y), ptr(T), stream_handle())
    return y, z, T


def tc_fault(clear=True):
    import ctypes
    flag = ctypes.c_int(0)
    call("moce_tc_fault", ctypes.addressof(flag), 1 if clear else 0)
    return flag.value


def forward(x, L, gate_w, gate_b, k, tmin, tmax, tau, route=None, path="general", balance=True):
    """Eval-form forward through the C ABI: route build, then either the
    general two passes (pool + gate -> T, softmax + mix) or the fast path."""
    r = route or route_build(L, k, transposed=False)
    if path == "tc":
        y, z, T = forward_tc(x, r, gate_w, gate_b, tmin * tau, (tmax - tmin) * tau)
        return y, dict(r, z=z, T=T)
    if path == "gx":
        y, z, T = forward_gx(x, r, gate_w, gate_b, tmin * tau, (tmax - tmin) * tau)
        return y, dict(r, z=z, T=T)
    if path == "px":
        y, z, T = forward_px(x, r, gate_w, gate_b, tmin * tau, (tmax - tmin) * tau)
        return y, dict(r, z=z, T=T)
    if path == "fast":
        r["group_expert"], r["sched"] = schedule_build(r["idx"], L.shape[1], balance)
        y, z, T = forward_fast(x, r, gate_w, gate_b, tmin * tau, (tmax - tmin) * tau)
        return y, dict(r, z=z, T=T)
    z, T = gate_temperature(x, r["idx"], gate_w, gate_b, tmin * tau, (tmax - tmin) * tau)
    return mix(x, r["idx"], r["ln"], T, r["mask"]), dict(r, z=z, T=T)


def forward_dynamic_temp(x, indices, weights, mask):
    B, C, H, W = x.shape
    E_r, K = indices.shape
    y = torch.empty(B, E_r + 1, H, W, dtype=x.dtype, device=x.device)
    bits = 64 if indices.dtype == torch.int64 else 32
    call("moce_forward_dynamic_temp", ptr(x), dtype_code(x), ptr(indices), bits, ptr(weights), ptr(mask), ptr(y),
         B, C, H * W, E_r, K, stream_handle())
    return y


def gate_route(x, pooled, indices, ln, gate_w, gate_b, mask, tmin, tmax, tau):
    B, C, H, W = x.shape
    E_r, K = indices.shape
    y = torch.empty(B, E_r + 1, H, W, dtype=x.dtype, device=x.device)
    nb = capi.lib().moce_gate_route_workspace_bytes(B, C, E_r)
    ws = torch.empty(nb + 256, dtype=torch.uint8, device=x.device)
    wp = (ws.data_ptr() + 255) & ~255
    bits = 64 if indices.dtype == torch.int64 else 32
    call("moce_gate_route", ptr(x), dtype_code(x), ptr(pooled), ptr(indices), bits, ptr(ln), ptr(gate_w),
         ptr(gate_b), ptr(mask), tmin, tmax, tau, ptr(y), B, C, H * W, E_r, K, wp, nb, stream_handle())
    return y


def backward(x, dy, L, r, gate_w, gate_b, tmin_tau, trange_tau):
    B, C, H, W = x.shape
    E_r, k = r["idx"].shape
    dx = torch.empty_like(x)
    dL = torch.empty(E_r, C, dtype=torch.float32, device=x.device)
    dgw = torch.empty(k, dtype=torch.float32, device=x.device)
    dgb = torch.empty(1, dtype=torch.float32, device=x.device)
    nb = capi.lib().moce_backward_workspace_bytes(B, C, H * W, E_r, k)
    ws = torch.empty(nb + 256, dtype=torch.uint8, device=x.device)
    wp = (ws.data_ptr() + 255) & ~255
    call("moce_backward", ptr(x), ptr(dy), dtype_code(x), B, C, H * W, ptr(L), ptr(r["idx"]), ptr(r["ln"]),
         ptr(r["mask"]), ptr(r["meta"]), ptr(r["toff"]), ptr(r["tslot"]), E_r, k, ptr(gate_w), ptr(gate_b),
         tmin_tau, trange_tau, ptr(r["z"]), ptr(r["T"]), ptr(dx), ptr(dL), ptr(dgw), ptr(dgb), wp, nb,
         stream_handle())
    return dict(dX=dx, dL=dL, dgate_w=dgw, dgate_b=dgb)
