"""CPU oracle for the MoCE layer hot path -- TEST INFRASTRUCTURE ONLY.

This module restates, in numpy, the algorithm of the reference MoCE layer
(Elianiluk/MoCE_thesis, ``MoCE.py`` and ``moce_fixed/moce_kernel.cu``).  It is
the checker the parity tests, ``__graft_entry__.smoke()`` and the CPU baseline
leg of ``bench.py`` compare the CUDA kernels against.  Nothing in the product
package imports it; the product path has no CPU fallback.

Pinning: the functions here are checked against golden vectors produced by
the unmodified reference ``MoCE.py`` (train forward, autograd backward and the
auxiliary loss), see ``tests/golden/make_golden.py`` and
``tests/test_oracle_golden.py``.  The reference ships no tests or golden
vectors of its own, so these fixtures are the only pins.

Arithmetic is float64 by default so the oracle is a cleaner truth than the
fp32 reference; ``dtype=np.float32`` reproduces fp32 rounding behaviour where a
test wants it.

Support ties: ``torch.topk`` leaves the order of equal logits unspecified.  The
oracle (and the CUDA route-build kernel) order supports by descending logit and
then ascending channel index; for tie-free rows (all fixtures with random
N(0,1) logits) this is exactly ``torch.topk``'s order.
"""
from __future__ import annotations

import numpy as np

__all__ = [
    "select_supports", "normalize_selected", "uncovered_mask", "transposed_lists",
    "gap", "gate_temperature", "softmax_weights", "routed_mix", "residual",
    "forward", "forward_with_weights", "backward", "aux_loss", "gate_temperature_mlp",
]


def _rowwise_desc_order(L: np.ndarray) -> np.ndarray:
    """Stable descending order of each row (ties -> lower index first).

    NaN is treated as larger than every number, as ``torch.topk`` does.
    """
    L = np.asarray(L, dtype=np.float32)
    # sort key: (is_not_nan, -value) ascending; lexsort uses the last key first.
    neg = -L.astype(np.float64)
    neg[np.isnan(L)] = -np.inf
    return np.argsort(neg, axis=1, kind="stable")


def select_supports(L: np.ndarray, k: int) -> np.ndarray:
    """S_e = TopK(L_e, k) in descending logit order.

    Reference: ``MoCE.py:91`` (eval cache) and ``MoCE.py:160`` (train).
    Returns int64 [E_r, k].
    """
    L = np.asarray(L, dtype=np.float32)
    if k > L.shape[1] or k < 1:
        raise ValueError("k must be in [1, C]")
    return _rowwise_desc_order(L)[:, :k].astype(np.int64)


def normalize_selected(L: np.ndarray, idx: np.ndarray, dtype=np.float64) -> np.ndarray:
    """ln = (sel - mean) / clamp(std_unbiased, min=1).

    Reference: ``MoCE.py:92-97`` and ``MoCE.py:182-187``.  For k == 1 the
    unbiased std is 0/0 = NaN, the clamp keeps NaN, so ln is NaN (as torch).
    """
    sel = np.take_along_axis(np.asarray(L, dtype=np.float32), idx, axis=1).astype(dtype)
    k = sel.shape[1]
    cen = sel - sel.mean(axis=1, keepdims=True)
    with np.errstate(invalid="ignore", divide="ignore"):
        var = (cen * cen).sum(axis=1, keepdims=True) / dtype(k - 1) if k > 1 else \
            np.full((sel.shape[0], 1), np.nan, dtype=dtype)
        sd = np.sqrt(var)
        scale = np.where(np.isnan(sd), np.nan, np.maximum(sd, 1.0))
        return cen / scale


def uncovered_mask(C: int, idx: np.ndarray) -> np.ndarray:
    """mask[c] = 1 iff no routed expert selects channel c (int32 [C]).

    Reference: ``MoCE.py:102-105`` (eval) and ``MoCE.py:192-195`` (train).
    """
    mask = np.ones(C, dtype=np.int32)
    mask[np.asarray(idx).reshape(-1)] = 0
    return mask


def transposed_lists(C: int, idx: np.ndarray):
    """Per channel c the flat slots e*k+i with idx[e,i] == c, ascending (CSR).

    No reference counterpart (the reference has no backward kernel); this is
    the layout the dX scatter uses.  Returns (offsets int32 [C+1], slots int32).
    """
    flat = np.asarray(idx).reshape(-1)
    order = np.argsort(flat, kind="stable")
    counts = np.bincount(flat, minlength=C)
    offs = np.zeros(C + 1, dtype=np.int32)
    offs[1:] = np.cumsum(counts)
    return offs, order.astype(np.int32)


def gap(X: np.ndarray, dtype=np.float64) -> np.ndarray:
    """z[b,c] = mean over H*W of X[b,c].

    Reference: ``MoCE.py:174`` (train) / ``MoCE.py:212`` (eval); unused
    kernel ``moce_kernel.cu:30-46``.
    """
    B, C = X.shape[:2]
    return np.asarray(X, dtype=dtype).reshape(B, C, -1).mean(axis=2)


def gate_temperature(z, idx, gate_w, gate_b, temp_min, temp_max, tau, dtype=np.float64):
    """Effective temperature T[b,e] from the shared Linear(k,1) gate.

    Reference: ``MoCE.py:175-178`` (train) / ``MoCE.py:216-218`` (eval):
    g = w . z[b, S_e] + b0;  T = clamp((tmin + (tmax-tmin) sigmoid(g)) * tau, 1e-3).
    Returns (T_eff, g) as [B, E_r] arrays.
    """
    z = np.asarray(z, dtype=dtype)
    zs = z[:, np.asarray(idx)]                       # [B, E_r, k]
    g = (zs * np.asarray(gate_w, dtype=dtype).reshape(1, 1, -1)).sum(-1) + dtype(np.asarray(gate_b).reshape(-1)[0])
    sig = 1.0 / (1.0 + np.exp(-g))
    T = (dtype(temp_min) + dtype(temp_max - temp_min) * sig) * dtype(tau)
    return np.maximum(T, dtype(1e-3)), g


def gate_temperature_mlp(z, w1, b1, w2, b2, temp_min, temp_max, tau, dtype=np.float64):
    """Temperatures from the opt-in two-layer gate C -> Hd -> E_r with ReLU:
    h = relu(z w1^T + b1), g = h w2^T + b2, T = clamp((tmin + (tmax-tmin)
    sigmoid(g)) * tau, 1e-3).

    No reference counterpart (the reference's gate is the Linear(k,1) of
    ``MoCE.py:66-68``); this restates the two-layer gate of the benchmark
    configurations with the reference's temperature map (``MoCE.py:177-178``).
    Parity for it is against this restatement only (unpinned by the
    reference).  Returns (T, g, h) as [B, E_r], [B, E_r], [B, Hd].
    """
    z = np.asarray(z, dtype=dtype)
    a1 = z @ np.asarray(w1, dtype=dtype).T + np.asarray(b1, dtype=dtype).reshape(1, -1)
    h = np.maximum(a1, 0.0)
    g = h @ np.asarray(w2, dtype=dtype).T + np.asarray(b2, dtype=dtype).reshape(1, -1)
    sig = 1.0 / (1.0 + np.exp(-g))
    T = (dtype(temp_min) + dtype(temp_max - temp_min) * sig) * dtype(tau)
    return np.maximum(T, dtype(1e-3)), g, h


def softmax_weights(ln, T):
    """a[b,e,:] = softmax(ln[e,:] / T[b,e]).

    Reference: ``MoCE.py:188`` (train) / ``MoCE.py:219-221`` (eval).
    """
    u = np.asarray(ln)[None, :, :] / np.asarray(T)[:, :, None]
    m = u.max(axis=2, keepdims=True)
    ex = np.exp(u - m)
    return ex / ex.sum(axis=2, keepdims=True)


def routed_mix(X, idx, a, dtype=np.float64):
    """Y[b,e,p] = sum_i a[b,e,i] * X[b, idx[e,i], p] for e < E_r.

    Reference: ``MoCE.py:167-171`` + ``MoCE.py:189`` (train) and the eval
    kernels ``moce_kernel.cu:57-89`` / ``moce_kernel.cu:97-141``.
    Returns [B, E_r, HW].
    """
    B, C = X.shape[:2]
    Xf = np.asarray(X, dtype=dtype).reshape(B, C, -1)
    idx = np.asarray(idx)
    E_r, k = idx.shape
    out = np.zeros((B, E_r, Xf.shape[2]), dtype=dtype)
    for i in range(k):                      # k gathers of [B, E_r, HW]
        out += np.asarray(a, dtype=dtype)[:, :, i:i + 1] * Xf[:, idx[:, i], :]
    return out


def residual(X, mask, dtype=np.float64):
    """Residual expert: mean of X over uncovered channels, 0 if there are none.

    Reference: ``MoCE.py:191-196`` (train) and ``moce_kernel.cu:148-180`` /
    ``moce_kernel.cu:187-231`` (eval, "count > 0 ? sum / count : 0").
    Returns [B, 1, HW].
    """
    B, C = X.shape[:2]
    Xf = np.asarray(X, dtype=dtype).reshape(B, C, -1)
    m = np.asarray(mask).astype(bool)
    n = int(m.sum())
    if n == 0:
        return np.zeros((B, 1, Xf.shape[2]), dtype=dtype)
    return Xf[:, m, :].sum(axis=1, keepdims=True) / dtype(n)


def forward(X, L, gate_w, gate_b, k, temp_min=0.2, temp_max=5.0, tau=1.0,
            mode="eval", dtype=np.float64, return_aux=False, mlp=None):
    """Full MoCE forward: Y [B, E_r+1, H, W].

    mode="train" follows ``MoCE.forward_train`` (``MoCE.py:153-201``, where
    tau is floored at 1e-4, ``MoCE.py:157``); mode="eval" follows
    ``MoCE.forward_eval`` (``MoCE.py:204-230``).  ``mlp=(w1, b1, w2, b2)``
    replaces the Linear(k,1) gate by the two-layer gate
    (``gate_temperature_mlp``; gate_w / gate_b are then unused).
    """
    X = np.asarray(X)
    B, C, H, W = X.shape
    tau_eff = max(float(tau), 1e-4) if mode == "train" else float(tau)
    idx = select_supports(L, k)
    ln = normalize_selected(L, idx, dtype=dtype)
    mask = uncovered_mask(C, idx)
    z = gap(X, dtype=dtype)
    h = None
    if mlp is None:
        T, g = gate_temperature(z, idx, gate_w, gate_b, temp_min, temp_max, tau_eff, dtype=dtype)
    else:
        T, g, h = gate_temperature_mlp(z, *mlp, temp_min, temp_max, tau_eff, dtype=dtype)
    a = softmax_weights(ln, T)
    Y = np.concatenate([routed_mix(X, idx, a, dtype=dtype), residual(X, mask, dtype=dtype)], axis=1)
    Y = Y.reshape(B, idx.shape[0] + 1, H, W)
    if return_aux:
        return Y, dict(idx=idx, ln=ln, mask=mask, z=z, T=T, g=g, a=a, h=h)
    return Y


def forward_with_weights(X, idx, weights, mask, dtype=np.float64):
    """The reference's CUDA entry point ``fused_moce_forward_dynamic_temp``.

    Given per-sample weights [B, E_r, K] (computed by the caller), returns the
    routed mix plus the residual channel.  Reference:
    ``moce_kernel.cu:1079-1153`` (K2/K4 or K3/K5).
    """
    X = np.asarray(X)
    B, C, H, W = X.shape
    Y = np.concatenate([routed_mix(X, idx, weights, dtype=dtype), residual(X, mask, dtype=dtype)], axis=1)
    return Y.reshape(B, -1, H, W)


def backward(X, L, gate_w, gate_b, k, dY, temp_min=0.2, temp_max=5.0, tau=1.0,
             mode="train", dtype=np.float64, mlp=None):
    """Gradients of sum(Y * dY) w.r.t. X, L (main path only) and the gate.

    Derived by hand from ``MoCE.forward_train`` (``MoCE.py:153-201``); the
    reference has no backward kernel and trains through autograd.  The
    auxiliary-loss gradient of L is not included (see ``aux_loss``).
    Returns dict(dX, dL, dgate_w, dgate_b, dT), and with ``mlp`` (the
    two-layer gate) dict(dX, dL, dw1, db1, dw2, db2, dT) instead of the
    Linear(k,1) gate's gradients.  dT is the gradient with respect to the
    temperatures after the 1e-3 clamp.
    """
    X = np.asarray(X, dtype=dtype)
    B, C, H, W = X.shape
    HW = H * W
    tau_eff = max(float(tau), 1e-4) if mode == "train" else float(tau)
    _, aux = forward(X, L, gate_w, gate_b, k, temp_min, temp_max, tau, mode=mode,
                     dtype=dtype, return_aux=True, mlp=mlp)
    idx, ln, mask, z, T, g, a = (aux[n] for n in ("idx", "ln", "mask", "z", "T", "g", "a"))
    E_r = idx.shape[0]
    Xf = X.reshape(B, C, HW)
    dYf = np.asarray(dY, dtype=dtype).reshape(B, E_r + 1, HW)
    dYr, dYres = dYf[:, :E_r, :], dYf[:, E_r, :]

    # da[b,e,i] = sum_p dY[b,e,p] * X[b, S_ei, p]
    da = np.zeros((B, E_r, k), dtype=dtype)
    for i in range(k):
        da[:, :, i] = (dYr * Xf[:, idx[:, i], :]).sum(-1)
    du = a * (da - (a * da).sum(-1, keepdims=True))
    dln_b = du / T[:, :, None]
    u = ln[None] / T[:, :, None]
    dT = -(du * u).sum(-1) / T
    dT_out = dT.copy()
    T_raw = (temp_min + (temp_max - temp_min) / (1.0 + np.exp(-g))) * tau_eff
    dT = np.where(T_raw >= 1e-3, dT, 0.0) * tau_eff
    sig = 1.0 / (1.0 + np.exp(-g))
    dg = dT * (temp_max - temp_min) * sig * (1.0 - sig)

    gate_grads = {}
    if mlp is None:
        zs = z[:, idx]
        w = np.asarray(gate_w, dtype=dtype).reshape(-1)
        gate_grads["dgate_w"] = (dg[:, :, None] * zs).sum((0, 1)).reshape(1, -1)
        gate_grads["dgate_b"] = np.array([dg.sum()], dtype=dtype)
        dz = np.zeros((B, C), dtype=dtype)
        for i in range(k):
            np.add.at(dz, (slice(None), idx[:, i]), dg * w[i])
    else:
        # g = h w2^T + b2, h = relu(a1), a1 = z w1^T + b1
        w1, b1, w2, b2 = (np.asarray(t, dtype=dtype) for t in mlp)
        h = aux["h"]
        gate_grads["dw2"] = dg.T @ h
        gate_grads["db2"] = dg.sum(0)
        da1 = (dg @ w2) * (h > 0)
        gate_grads["dw1"] = da1.T @ z
        gate_grads["db1"] = da1.sum(0)
        dz = da1 @ w1

    dX = np.zeros((B, C, HW), dtype=dtype)
    for i in range(k):
        contrib = a[:, :, i:i + 1] * dYr            # [B, E_r, HW]
        np.add.at(dX, (slice(None), idx[:, i], slice(None)), contrib)
    n_u = int(mask.sum())
    if n_u > 0:
        dX[:, mask.astype(bool), :] += dYres[:, None, :] / dtype(n_u)
    dX += dz[:, :, None] / dtype(HW)

    # ln = cen / scale, scale = max(std_unbiased(sel), 1)
    dln = dln_b.sum(0)
    sel = np.take_along_axis(np.asarray(L, dtype=np.float32), idx, axis=1).astype(dtype)
    cen = sel - sel.mean(1, keepdims=True)
    sd = np.sqrt((cen * cen).sum(1, keepdims=True) / max(k - 1, 1))
    scale = np.maximum(sd, 1.0)
    dcen = dln / scale
    dscale = -(dln * cen).sum(1, keepdims=True) / (scale * scale)
    dcen = dcen + np.where(sd >= 1.0, dscale, 0.0) * cen / (max(k - 1, 1) * np.where(sd > 0, sd, 1.0))
    dsel = dcen - dcen.mean(1, keepdims=True)
    dL = np.zeros(np.asarray(L).shape, dtype=dtype)
    np.put_along_axis(dL, idx, dsel, axis=1)
    return dict(dX=dX.reshape(B, C, H, W), dL=dL, dT=dT_out, **gate_grads)


def aux_loss(L, k, tau=1.0, balance_weight=0.05, specialization_weight=0.1,
             diversity_weight=0.01, dtype=np.float64):
    """Coverage/auxiliary loss of ``MoCE._compute_aux_losses`` (``MoCE.py:118-151``)."""
    L = np.asarray(L, dtype=dtype)
    E_r, C = L.shape
    tau = max(float(tau), 1e-4)
    s = L / tau
    P = np.exp(s - s.max(1, keepdims=True))
    P = P / P.sum(1, keepdims=True)
    usage = P.mean(0)
    balance = ((usage - usage.mean()) ** 2).mean()
    egc = P / np.maximum(P.sum(0, keepdims=True), 1e-8)
    ent = -(egc * np.log(np.maximum(egc, 1e-8))).sum(0)
    target = np.log(max(E_r * k / max(float(C), 1.0), 1.0))
    spec = np.maximum(ent - target, 0.0).mean()
    if E_r > 1:
        ov = P @ P.T
        div = ov[~np.eye(E_r, dtype=bool)].mean()
    else:
        div = 0.0
    return balance_weight * balance + specialization_weight * spec + diversity_weight * div
