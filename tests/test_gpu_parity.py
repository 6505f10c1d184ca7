"""GPU parity: the sm_100a kernels, called through the C ABI, against the
numpy oracle and the reference golden vectors.

Tolerances (stated by the workload): supports and masks bit-exact; fp32
outputs within 1e-5 relative (elementwise, absolute floor 1e-6 x the tensor
scale); bf16 outputs within 1e-2 relative against the fp32 oracle evaluated on
the bf16-rounded input; gradients within 1e-5 relative to the tensor's max
magnitude (floor 1e-3).
"""
import os

import numpy as np
import pytest
import torch

from oracle import moce_oracle as O
from inputs import CASES, make_inputs, tie_logits
import capi_helpers as H

pytestmark = pytest.mark.gpu
GOLD = os.path.join(os.path.dirname(__file__), "golden")
FULL = [n for n, c in CASES.items() if not c.get("summary")]
DEV = "cuda:0"


def load(name):
    return dict(np.load(os.path.join(GOLD, f"{name}.npz")))


def cu(a, dtype=None):
    t = torch.as_tensor(np.ascontiguousarray(a)).to(DEV)
    return t.to(dtype) if dtype is not None else t


def host(t):
    torch.cuda.synchronize()
    return t.detach().float().cpu().numpy().astype(np.float64)


def close(a, b, rtol=1e-5, floor=1e-6):
    a = np.asarray(a, dtype=np.float64)
    b = np.asarray(b, dtype=np.float64)
    scale = max(np.abs(b).max(), 1e-30)
    return bool(np.all(np.abs(a - b) <= rtol * np.abs(b) + floor * scale))


def maxrel(a, b, floor=1e-3):
    a = np.asarray(a, dtype=np.float64)
    b = np.asarray(b, dtype=np.float64)
    return float(np.abs(a - b).max() / max(np.abs(b).max(), floor))


def relerr(a, b):
    a = np.asarray(a, dtype=np.float64)
    b = np.asarray(b, dtype=np.float64)
    return float((np.abs(a - b) / np.maximum(np.abs(b), 1e-6 * max(np.abs(b).max(), 1e-30))).max())


# ---------------------------------------------------------------- route build

@pytest.mark.parametrize("name", FULL)
def test_route_build_matches_golden(name):
    g, c = load(name), CASES[name]
    r = H.route_build(cu(g["L"]), c["k"])
    torch.cuda.synchronize()
    np.testing.assert_array_equal(r["idx"].cpu().numpy(), g["idx"])
    np.testing.assert_array_equal(r["mask"].cpu().numpy(), g["mask"])
    assert int(r["meta"][0]) == int(g["mask"].sum())
    assert close(host(r["ln"]), g["ln"]), relerr(host(r["ln"]), g["ln"])
    offs, slots = O.transposed_lists(c["C"], g["idx"])
    np.testing.assert_array_equal(r["toff"].cpu().numpy(), offs)
    np.testing.assert_array_equal(r["tslot"].cpu().numpy(), slots)


def test_route_build_ties_deterministic():
    g = load("ties")
    k = int(g["k"])
    r = H.route_build(cu(g["L"]), k)
    torch.cuda.synchronize()
    np.testing.assert_array_equal(r["idx"].cpu().numpy(), O.select_supports(g["L"], k))


@pytest.mark.parametrize("E_r,C,k", [(2047, 512, 32), (1023, 256, 16), (511, 2048, 128), (7, 5, 5)])
def test_route_build_large_rows(E_r, C, k):
    gen = torch.Generator().manual_seed(E_r + C)
    L = torch.randn(E_r, C, generator=gen)
    r = H.route_build(L.to(DEV), k)
    torch.cuda.synchronize()
    np.testing.assert_array_equal(r["idx"].cpu().numpy(), O.select_supports(L.numpy(), k))
    tv, ti = torch.topk(L, k, dim=1)
    got = r["idx"].cpu().numpy()
    # same selected values everywhere; same order on rows without ties
    np.testing.assert_array_equal(np.take_along_axis(L.numpy(), got, 1), tv.numpy())
    ties = np.array([len(np.unique(row)) < C for row in L.numpy()])
    np.testing.assert_array_equal(got[~ties], ti.numpy()[~ties])


# ---------------------------------------------------------------- forward

PATHS = ["general", "fast", "px"]


def path_ok(path, k):
    if path == "px":
        return k <= 64
    return path == "general" or H.schedule_supported(k)


@pytest.mark.parametrize("name", FULL)
@pytest.mark.parametrize("path", PATHS)
def test_forward_fp32_matches_golden(name, path):
    g, c = load(name), CASES[name]
    if not path_ok(path, c["k"]):
        pytest.skip("k beyond the scheduled kernel")
    y, st = H.forward(cu(g["X"]), cu(g["L"]), cu(g["gate_w"]), cu(g["gate_b"]), c["k"], c["tmin"], c["tmax"],
                      c["tau"], path=path)
    Y = host(y)
    assert close(Y, g["Y_eval"]), relerr(Y, g["Y_eval"])
    ref = O.forward(g["X"], g["L"], g["gate_w"], g["gate_b"], c["k"], c["tmin"], c["tmax"], c["tau"], mode="eval")
    assert close(Y, ref), relerr(Y, ref)
    # pass-1 outputs
    _, aux = O.forward(g["X"], g["L"], g["gate_w"], g["gate_b"], c["k"], c["tmin"], c["tmax"], c["tau"],
                       mode="eval", return_aux=True)
    assert close(host(st["z"]), aux["z"])
    assert close(host(st["T"]), aux["T"])


@pytest.mark.parametrize("name", FULL)
@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float16])
@pytest.mark.parametrize("path", PATHS)
def test_forward_half_matches_oracle(name, dtype, path):
    g, c = load(name), CASES[name]
    if not path_ok(path, c["k"]):
        pytest.skip("k beyond the scheduled kernel")
    x = cu(g["X"], dtype)
    y, _ = H.forward(x, cu(g["L"]), cu(g["gate_w"]), cu(g["gate_b"]), c["k"], c["tmin"], c["tmax"], c["tau"],
                     path=path)
    assert y.dtype == dtype
    xr = x.float().cpu().numpy()
    ref = O.forward(xr, g["L"], g["gate_w"], g["gate_b"], c["k"], c["tmin"], c["tmax"], c["tau"], mode="eval")
    assert close(host(y), ref, rtol=1e-2, floor=1e-3), relerr(host(y), ref)


@pytest.mark.parametrize("name", FULL)
@pytest.mark.parametrize("bits", [64, 32])
def test_forward_dynamic_temp_reference_entry(name, bits):
    g = load(name)
    idx = cu(g["idx"].astype(np.int64 if bits == 64 else np.int32))
    y = H.forward_dynamic_temp(cu(g["X"]), idx, cu(g["weights"]), cu(g["mask"]))
    assert close(host(y), g["Y_eval"]), relerr(host(y), g["Y_eval"])


@pytest.mark.parametrize("name", FULL)
@pytest.mark.parametrize("pooled_given", [True, False])
def test_gate_route_reference_entries(name, pooled_given):
    g, c = load(name), CASES[name]
    x = cu(g["X"])
    pooled = cu(O.gap(g["X"]).astype(np.float32)) if pooled_given else None
    y = H.gate_route(x, pooled, cu(g["idx"]), cu(g["ln"]), cu(g["gate_w"].reshape(-1)), cu(g["gate_b"]),
                     cu(g["mask"]), c["tmin"], c["tmax"], c["tau"])
    assert close(host(y), g["Y_eval"]), relerr(host(y), g["Y_eval"])


# ---------------------------------------------------------------- backward

@pytest.mark.parametrize("name", FULL)
def test_backward_matches_golden(name):
    g, c = load(name), CASES[name]
    x, L, gw, gb = cu(g["X"]), cu(g["L"]), cu(g["gate_w"]), cu(g["gate_b"])
    tau = max(float(c["tau"]), 1e-4)
    r = H.route_build(L, c["k"])
    z, T = H.gate_temperature(x, r["idx"], gw, gb, c["tmin"] * tau, (c["tmax"] - c["tmin"]) * tau)
    r.update(z=z, T=T)
    d = H.backward(x, cu(g["dY"]), L, r, gw, gb, c["tmin"] * tau, (c["tmax"] - c["tmin"]) * tau)
    for key in ("dX", "dL", "dgate_w", "dgate_b"):
        got, want = host(d[key]), g[key].reshape(host(d[key]).shape)
        assert maxrel(got, want) < 1e-5, (key, maxrel(got, want))


def test_backward_deterministic():
    c = CASES["small_resid"]
    t = make_inputs(c)
    x, L, gw, gb, dy = (t[n].to(DEV) for n in ("X", "L", "gate_w", "gate_b", "dY"))
    r = H.route_build(L, c["k"])
    z, T = H.gate_temperature(x, r["idx"], gw, gb, c["tmin"], c["tmax"] - c["tmin"])
    r.update(z=z, T=T)
    a = H.backward(x, dy, L, r, gw, gb, c["tmin"], c["tmax"] - c["tmin"])
    b = H.backward(x, dy, L, r, gw, gb, c["tmin"], c["tmax"] - c["tmin"])
    for key in a:
        assert torch.equal(a[key], b[key]), key


# ---------------------------------------------------------------- the single-layer workload

@pytest.mark.parametrize("path", PATHS)
def test_cfg1_against_pins(path):
    c, g = CASES["cfg1"], load("cfg1")
    t = make_inputs(c)
    x, L, gw, gb, dy = (t[n].to(DEV) for n in ("X", "L", "gate_w", "gate_b", "dY"))
    y, st = H.forward(x, L, gw, gb, c["k"], c["tmin"], c["tmax"], c["tau"], path=path)
    Y = host(y)
    np.testing.assert_array_equal(st["idx"].cpu().numpy(), g["idx"].astype(np.int32))
    assert close(Y.reshape(-1)[g["Y_eval_pos"]], g["Y_eval_val"])
    assert close(Y.sum(axis=(2, 3)), g["Y_eval_chsum"], rtol=1e-5, floor=1e-5)
    r = H.route_build(L, c["k"])
    r.update(z=st["z"], T=st["T"])
    d = H.backward(x, dy, L, r, gw, gb, c["tmin"], c["tmax"] - c["tmin"])
    assert maxrel(host(d["dX"]).reshape(-1)[g["dX_pos"]], g["dX_val"]) < 1e-5
    idx = g["idx"].astype(np.int64)
    assert maxrel(np.take_along_axis(host(d["dL"]), idx, 1), g["dL_at_idx"]) < 1e-5
    assert maxrel(host(d["dgate_w"]), g["dgate_w"].reshape(-1)) < 1e-5


# ---------------------------------------------------------------- shapes the fixtures do not cover

@pytest.mark.parametrize("B,C,H_,W_,E,k,dtype", [
    (3, 64, 56, 56, 16, 8, torch.float32),     # many pixel tiles (HW = 3136)
    (2, 2048, 7, 7, 64, 128, torch.float32),   # wide C: one-column tiles, k > 64
    (2, 2048, 7, 7, 64, 128, torch.bfloat16),
    (5, 130, 3, 7, 40, 33, torch.float32),     # ragged everything
    (1, 16, 1, 1, 2, 16, torch.float32),       # k == C, HW == 1, one routed expert
    (1, 64, 2, 2, 2048, 8, torch.float32),     # E > 1800: the dX kernel without a staged dY tile
    (2, 96, 13, 11, 50, 20, torch.float32),    # HW = 143: two pixel slabs, rows padded to 144
])
@pytest.mark.parametrize("path", PATHS)
def test_forward_backward_odd_shapes(B, C, H_, W_, E, k, dtype, path):
    if not path_ok(path, k):
        pytest.skip("k beyond the scheduled kernel")
    if path == "px" and not H.px_supported(torch.empty(1, C, H_, W_, dtype=dtype), k):
        pytest.skip("shape beyond the lanes-over-pixels kernel")
    gen = torch.Generator().manual_seed(B * 1000 + C)
    X = torch.randn(B, C, H_, W_, generator=gen).abs()
    L = torch.randn(E - 1, C, generator=gen)
    gw = torch.rand(1, k, generator=gen) - 0.5
    gb = torch.randn(1, generator=gen) * 0.1
    dY = torch.randn(B, E, H_, W_, generator=gen)
    x = X.to(DEV, dtype)
    Xr = x.float().cpu().numpy()
    y, st = H.forward(x, L.to(DEV), gw.to(DEV), gb.to(DEV), k, 0.1, 10.0, 1.0, path=path)
    ref = O.forward(Xr, L.numpy(), gw.numpy(), gb.numpy(), k, 0.1, 10.0, 1.0, mode="eval")
    rt = 1e-5 if dtype == torch.float32 else 1e-2
    assert close(host(y), ref, rtol=rt, floor=rt / 10), relerr(host(y), ref)
    if dtype != torch.float32:
        return
    r = H.route_build(L.to(DEV), k)
    r.update(z=st["z"], T=st["T"])
    d = H.backward(x, dY.to(DEV), L.to(DEV), r, gw.to(DEV), gb.to(DEV), 0.1, 9.9)
    want = O.backward(Xr, L.numpy(), gw.numpy(), gb.numpy(), k, dY.numpy(), 0.1, 10.0, 1.0, mode="eval")
    for key in ("dX", "dL", "dgate_w", "dgate_b"):
        got = host(d[key]).reshape(np.shape(want[key]))
        assert maxrel(got, want[key]) < 1e-5, (key, maxrel(got, want[key]))


@pytest.mark.parametrize("path", PATHS)
def test_empty_batch_is_a_noop(path):
    c = CASES["small_resid"]
    t = make_inputs(c)
    x = t["X"][:0].to(DEV)
    y, _ = H.forward(x, t["L"].to(DEV), t["gate_w"].to(DEV), t["gate_b"].to(DEV), c["k"], 0.1, 10.0, 1.0, path=path)
    assert y.shape[0] == 0


def test_invalid_arguments_raise():
    c = CASES["small_resid"]
    t = make_inputs(c)
    x = t["X"].to(DEV)
    r = H.route_build(t["L"].to(DEV), c["k"], transposed=False)
    with pytest.raises(RuntimeError, match="status 1"):
        # k larger than C
        H.route_build(t["L"].to(DEV), c["C"] + 1)
    z, T = H.gate_temperature(x, r["idx"], t["gate_w"].to(DEV), t["gate_b"].to(DEV), 0.1, 9.9)
    with pytest.raises(RuntimeError, match="null pointer"):
        H.mix(x, r["idx"], r["ln"], T, None)


# ---------------------------------------------------------------- schedule

@pytest.mark.parametrize("E_r,C,k,balance", [(2047, 512, 32, True), (1023, 256, 16, False), (63, 40, 7, True),
                                              (5, 3, 3, True)])
def test_schedule_is_a_permutation_of_the_supports(E_r, C, k, balance):
    gen = torch.Generator().manual_seed(k)
    L = torch.randn(E_r, C, generator=gen).to(DEV)
    r = H.route_build(L, k, transposed=False)
    ge, sched = H.schedule_build(r["idx"], C, balance)
    torch.cuda.synchronize()
    ge, sched, idx = ge.cpu().numpy(), sched.cpu().numpy(), r["idx"].cpu().numpy()
    S = H.capi.lib().moce_schedule_steps(k)
    G = (E_r + 31) // 32
    assert sorted(ge[ge >= 0].tolist()) == list(range(E_r))
    sched = sched.reshape(G, S, 32).view(np.uint32)
    conflicts = 0
    for g in range(G):
        for lane in range(32):
            e = ge[g * 32 + lane]
            ent = sched[g, :, lane]
            slots = ent >> 16
            chans = ent & 0xFFFF
            valid = slots != 0xFFFF
            if e < 0:
                assert not valid.any()
                continue
            assert sorted(slots[valid].tolist()) == list(range(k))
            assert np.all(idx[e, slots[valid]] == chans[valid])
        for s in range(S):
            banks = (sched[g, s, :] & 0xFFFF) % 32
            conflicts += 32 - len(set(banks.tolist()))
    # balanced groups of wide layers schedule with (almost) no bank conflicts
    if balance and E_r >= 32 and C >= 256:
        assert conflicts <= G * S * 32 // 50, conflicts
