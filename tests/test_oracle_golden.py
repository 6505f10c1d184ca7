"""Pin the numpy oracle against golden vectors from the reference ``MoCE.py``.

Tolerances: supports bit-exact (values and order); fp32 reference outputs vs
the float64 oracle within 1e-5 relative (elementwise, with an absolute floor
of 1e-6 times the tensor's scale); gradients within 1e-5 relative to the
tensor's max magnitude floored at 1e-3 (they contain cancellations, and a
gradient that is zero in exact arithmetic is fp32 rounding noise in the
reference).
"""
import os

import numpy as np
import pytest
import torch

from oracle import moce_oracle as O
from inputs import CASES, make_inputs

GOLD = os.path.join(os.path.dirname(__file__), "golden")
FULL = [n for n, c in CASES.items() if not c.get("summary")]


def load(name):
    return dict(np.load(os.path.join(GOLD, f"{name}.npz")))


def close(a, b, rtol=1e-5, floor=1e-6):
    a = np.asarray(a, dtype=np.float64)
    b = np.asarray(b, dtype=np.float64)
    scale = max(np.abs(b).max(), 1e-30)
    return np.all(np.abs(a - b) <= rtol * np.abs(b) + floor * scale)


def maxrel(a, b):
    a = np.asarray(a, dtype=np.float64)
    b = np.asarray(b, dtype=np.float64)
    return float(np.abs(a - b).max() / max(np.abs(b).max(), 1e-3))


@pytest.mark.parametrize("name", FULL)
def test_inputs_regenerate(name):
    g = load(name)
    t = make_inputs(CASES[name])
    for key in ("X", "L", "gate_w", "gate_b", "dY"):
        np.testing.assert_array_equal(t[key].numpy(), g[key])


@pytest.mark.parametrize("name", FULL)
def test_supports_bit_exact(name):
    g, c = load(name), CASES[name]
    idx = O.select_supports(g["L"], c["k"])
    np.testing.assert_array_equal(idx, g["idx"])
    np.testing.assert_array_equal(O.uncovered_mask(c["C"], idx), g["mask"])


@pytest.mark.parametrize("name", FULL)
def test_forward_train_and_eval(name):
    g, c = load(name), CASES[name]
    args = (g["X"], g["L"], g["gate_w"], g["gate_b"], c["k"], c["tmin"], c["tmax"], c["tau"])
    Yt = O.forward(*args, mode="train")
    Ye, aux = O.forward(*args, mode="eval", return_aux=True)
    assert close(Yt, g["Y_train"]), maxrel(Yt, g["Y_train"])
    assert close(Ye, g["Y_eval"]), maxrel(Ye, g["Y_eval"])
    assert close(aux["ln"], g["ln"]), maxrel(aux["ln"], g["ln"])
    assert close(aux["a"], g["weights"]), maxrel(aux["a"], g["weights"])
    Yw = O.forward_with_weights(g["X"], g["idx"], g["weights"], g["mask"])
    assert close(Yw, g["Y_eval"])


@pytest.mark.parametrize("name", FULL)
def test_backward(name):
    g, c = load(name), CASES[name]
    d = O.backward(g["X"], g["L"], g["gate_w"], g["gate_b"], c["k"], g["dY"],
                   c["tmin"], c["tmax"], c["tau"], mode="train")
    for key in ("dX", "dL", "dgate_w", "dgate_b"):
        assert maxrel(d[key], g[key]) < 1e-5, (key, maxrel(d[key], g[key]))


@pytest.mark.parametrize("name", FULL)
def test_aux_loss(name):
    g, c = load(name), CASES[name]
    v = O.aux_loss(g["L"], c["k"], c["tau"])
    assert abs(v - float(g["aux"])) <= 1e-5 * max(abs(float(g["aux"])), 1e-6)


def test_cfg1_summary():
    """Single-layer workload (N=8, C=256, 14x14, E=1024, k=16) against pins."""
    c = CASES["cfg1"]
    g = load("cfg1")
    t = make_inputs(c)
    assert abs(t["X"].double().sum().item() - float(g["X_sum"])) < 1e-6 * abs(float(g["X_sum"]))
    np.testing.assert_array_equal(t["X"].numpy().reshape(-1)[:64], g["X_head"])
    X, L, gw, gb, dY = (t[n].numpy() for n in ("X", "L", "gate_w", "gate_b", "dY"))
    idx = O.select_supports(L, c["k"])
    np.testing.assert_array_equal(idx, g["idx"].astype(np.int64))
    np.testing.assert_array_equal(O.uncovered_mask(c["C"], idx), g["mask"])
    args = (X, L, gw, gb, c["k"], c["tmin"], c["tmax"], c["tau"])
    for mode, key in (("train", "Y_train"), ("eval", "Y_eval")):
        Y = O.forward(*args, mode=mode)
        assert close(Y.reshape(-1)[g[key + "_pos"]], g[key + "_val"])
        assert close(Y.sum(axis=(2, 3)), g[key + "_chsum"], rtol=1e-5, floor=1e-5)
    d = O.backward(*args[:5], dY, c["tmin"], c["tmax"], c["tau"])
    assert maxrel(np.take_along_axis(d["dL"], idx, 1), g["dL_at_idx"]) < 1e-5
    assert maxrel(d["dX"].reshape(-1)[g["dX_pos"]], g["dX_val"]) < 1e-5
    assert maxrel(d["dgate_w"], g["dgate_w"]) < 1e-5
    assert maxrel(d["dgate_b"], g["dgate_b"]) < 1e-5


def test_tie_rows_select_topk_values():
    g = load("ties")
    k = int(g["k"])
    idx = O.select_supports(g["L"], k)
    vals = np.take_along_axis(g["L"], idx, 1)
    np.testing.assert_array_equal(vals, g["topk_values"])
    # deterministic rule: equal values appear in ascending channel order
    for e in range(idx.shape[0]):
        for i in range(k - 1):
            if vals[e, i] == vals[e, i + 1]:
                assert idx[e, i] < idx[e, i + 1]


def test_transposed_lists_roundtrip():
    rng = np.random.default_rng(0)
    L = rng.standard_normal((37, 50)).astype(np.float32)
    idx = O.select_supports(L, 7)
    offs, slots = O.transposed_lists(50, idx)
    assert offs[-1] == idx.size
    for c in range(50):
        s = slots[offs[c]:offs[c + 1]]
        assert np.all(np.diff(s) > 0)
        assert np.all(idx.reshape(-1)[s] == c)
