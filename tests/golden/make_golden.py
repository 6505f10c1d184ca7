"""Generate golden vectors from the unmodified reference ``MoCE.py``.

Run in the development container, where the reference checkout exists:

    python tests/golden/make_golden.py <path of the reference checkout>

The reference module does ``import moce_fixed.moce_cuda`` at import time; a
stub module is installed in ``sys.modules`` first.  The stub restates the one
CUDA entry point ``MoCE.forward_eval`` calls (``fused_moce_forward_dynamic_temp``,
``moce_kernel.cu:1079-1153``) on the CPU and records its arguments, so eval
goldens carry the exact per-sample weights the reference computed in ATen.

Train-mode goldens (forward, autograd backward, auxiliary loss) run only
reference code.  Output: one ``<case>.npz`` per case next to this script.
"""
from __future__ import annotations

import os
import sys
import types

import numpy as np
import torch

HERE = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, HERE)
from inputs import CASES, make_inputs, tie_logits  # noqa: E402

_calls = []


def _stub_forward_dynamic_temp(inp, indices, weights, mask_int):
    _calls.append(dict(indices=indices.clone(), weights=weights.clone(), mask=mask_int.clone()))
    B, C, H, W = inp.shape
    E_r, K = indices.shape
    xf = inp.reshape(B, C, H * W)
    g = xf[:, indices.reshape(-1), :].reshape(B, E_r, K, H * W)
    routed = (g * weights.unsqueeze(-1)).sum(2)
    m = mask_int.bool()
    n = int(m.sum())
    res = xf[:, m, :].sum(1, keepdim=True) / n if n > 0 else torch.zeros(B, 1, H * W)
    return [torch.cat([routed, res], 1).reshape(B, E_r + 1, H, W)]


def _import_reference(ref_root):
    pkg = types.ModuleType("moce_fixed")
    mod = types.ModuleType("moce_fixed.moce_cuda")
    mod.fused_moce_forward_dynamic_temp = _stub_forward_dynamic_temp
    pkg.moce_cuda = mod
    sys.modules["moce_fixed"] = pkg
    sys.modules["moce_fixed.moce_cuda"] = mod
    sys.path.insert(0, ref_root)
    import MoCE  # noqa: F401  (the reference module, unmodified)
    return MoCE.MoCE


def build_layer(MoCE, case, t):
    """Reference layer with E, k and the logits forced to the case's values.

    ``MoCE.__init__`` derives E from in_channels // sampling_factor; build with
    sampling_factor=1, then overwrite E, the logits and the derived target.
    """
    C, E, k = case["C"], case["E"], case["k"]
    m = MoCE(in_channels=C, sampling_factor=1, k=k, tau=case["tau"],
             temp_min=case["tmin"], temp_max=case["tmax"])
    m.num_experts = E
    m.routing_logits = torch.nn.Parameter(t["L"].clone())
    m.target_experts_per_channel = (max(E - 1, 1) * k) / max(float(C), 1.0)
    with torch.no_grad():
        m.gate.weight.copy_(t["gate_w"])
        m.gate.bias.copy_(t["gate_b"])
    return m


def run_case(MoCE, name, case, L_override=None):
    t = make_inputs(case)
    if L_override is not None:
        t["L"] = L_override
    m = build_layer(MoCE, case, t)
    # --- train forward + backward (pure reference code) ---
    m.train()
    X = t["X"].clone().requires_grad_(True)
    Y = m(X)
    aux = m.aux_loss
    (Y * t["dY"]).sum().backward()
    dX, dL, dgw, dgb = X.grad.clone(), m.routing_logits.grad.clone(), m.gate.weight.grad.clone(), m.gate.bias.grad.clone()
    m.zero_grad()
    m._compute_aux_losses(X, case["E"] - 1, max(float(case["tau"]), 1e-4))
    m.aux_loss.backward()
    dL_aux = m.routing_logits.grad.clone()
    # --- eval forward (reference ATen + restated CUDA mix) ---
    m.eval()
    m.build_eval_cache()
    _calls.clear()
    with torch.no_grad():
        Ye = m(t["X"])
    call = _calls[-1]
    out = dict(
        X=t["X"].numpy(), L=t["L"].numpy(), gate_w=t["gate_w"].numpy(), gate_b=t["gate_b"].numpy(),
        dY=t["dY"].numpy(),
        Y_train=Y.detach().numpy(), aux=np.array(float(aux)), dX=dX.numpy(), dL=dL.numpy(),
        dgate_w=dgw.numpy(), dgate_b=dgb.numpy(), dL_aux=dL_aux.numpy(),
        Y_eval=Ye.numpy(), idx=m.cached_indices.numpy(), ln=m.cached_selected_logits_norm.numpy(),
        mask=m.cached_mask_int.numpy(), weights=call["weights"].numpy(),
    )
    return out


def summarize(d, seed=1234):
    """Reduce full-size tensors to pins: checksums, samples, exact small parts."""
    rng = np.random.default_rng(seed)
    s = {}
    for key in ("X", "L", "dY"):
        s[key + "_sum"] = np.array(d[key].astype(np.float64).sum())
        s[key + "_head"] = d[key].reshape(-1)[:64]
    s["gate_w"], s["gate_b"] = d["gate_w"], d["gate_b"]
    for key in ("Y_train", "Y_eval", "dX"):
        a = d[key]
        s[key + "_chsum"] = a.astype(np.float64).sum(axis=(2, 3))          # [B, E or C]
        flat = a.reshape(-1)
        pos = rng.choice(flat.size, size=min(4096, flat.size), replace=False)
        s[key + "_pos"] = pos.astype(np.int64)
        s[key + "_val"] = flat[pos]
    E_r, k = d["idx"].shape
    s["dL_at_idx"] = np.take_along_axis(d["dL"], d["idx"], axis=1)
    s["dL_sum"] = np.array(d["dL"].astype(np.float64).sum())
    s["dL_aux_sum"] = np.array(d["dL_aux"].astype(np.float64).sum())
    for key in ("aux", "dgate_w", "dgate_b", "idx", "ln", "mask"):
        s[key] = d[key]
    s["idx"] = s["idx"].astype(np.int16 if d["L"].shape[1] < 32768 else np.int32)
    return s


def main():
    if len(sys.argv) != 2:
        sys.exit("usage: python tests/golden/make_golden.py <path of the reference checkout>")
    ref_root = sys.argv[1]
    torch.set_num_threads(os.cpu_count() or 1)
    MoCE = _import_reference(ref_root)
    for name, case in CASES.items():
        d = run_case(MoCE, name, case)
        if case.get("summary"):
            d = summarize(d)
        np.savez_compressed(os.path.join(HERE, f"{name}.npz"), **d)
        print("wrote", name)
    # rows full of ties: only the selected VALUES are pinned (torch.topk leaves
    # the order of equal logits unspecified)
    case = dict(CASES["small_resid"])
    Lt = tie_logits(case["E"] - 1, case["C"], seed=11)
    vals, _ = torch.topk(Lt, case["k"], dim=1)
    np.savez_compressed(os.path.join(HERE, "ties.npz"), L=Lt.numpy(), k=np.array(case["k"]),
                        topk_values=vals.numpy())
    print("wrote ties")


if __name__ == "__main__":
    main()
