"""GPU parity of the tensor-core mix (tcgen05) against the oracle.

The tensor-core path rounds the softmax weights to the input's 16-bit type
before the product; the bf16/fp16 tolerance (1e-2 relative against the fp32
oracle on the rounded input) covers it.  Every case also checks that no
bounded wait inside the kernel ran out.
"""
import numpy as np
import pytest
import torch

from oracle import moce_oracle as O
import capi_helpers as H

pytestmark = pytest.mark.gpu
DEV = "cuda:0"


def close(a, b, rtol, floor):
    a = np.asarray(a, dtype=np.float64)
    b = np.asarray(b, dtype=np.float64)
    return bool(np.all(np.abs(a - b) <= rtol * np.abs(b) + floor * max(np.abs(b).max(), 1e-30)))


def relerr(a, b):
    a = np.asarray(a, dtype=np.float64)
    b = np.asarray(b, dtype=np.float64)
    return float((np.abs(a - b) / np.maximum(np.abs(b), 1e-3 * max(np.abs(b).max(), 1e-30))).max())


@pytest.mark.parametrize("B,C,H_,W_,E,k,dtype", [
    (2, 64, 5, 5, 16, 4, torch.bfloat16),       # smallest: one K block, uncovered channels
    (3, 32, 3, 5, 33, 8, torch.float16),        # C < 64 (K padding), odd pixels
    (4, 512, 7, 7, 300, 32, torch.bfloat16),    # stage-4 widths, partial last expert tile
    (2, 130, 3, 7, 140, 33, torch.bfloat16),    # ragged C (not a multiple of 8), k > 32
    (2, 16, 1, 1, 2, 16, torch.float16),        # k == C, HW == 1
    (2, 96, 8, 8, 129, 40, torch.bfloat16),     # HW == 64 exactly
    (3, 64, 3, 11, 40, 8, torch.bfloat16),      # HW == 33: odd rows carry column 31 to the last column
    (2, 192, 6, 6, 70, 12, torch.float16),      # HW == 36, even rows
    (2, 256, 14, 14, 300, 16, torch.bfloat16),  # 14x14: N = 208 over four pixel atoms, one accumulator
    (2, 128, 10, 10, 140, 8, torch.float16),    # HW == 100: N = 112 over two atoms, two partial accumulators
    (2, 64, 16, 16, 40, 12, torch.bfloat16),    # HW == 256: N = 256, the largest tile
    (2, 96, 12, 12, 4, 8, torch.bfloat16),      # HW == 144 with uncovered channels (residual sums over 144 pixels)
    (2, 128, 28, 28, 90, 16, torch.bfloat16),   # 28x28: four pixel tiles of 208 / 160, weights reused per tile
    (1, 64, 56, 56, 40, 8, torch.float16),      # 56x56: thirteen pixel tiles of 256 / 64
    (2, 32, 20, 21, 3, 4, torch.bfloat16),      # HW == 420: two tiles of 224 / 196, uncovered channels
    (1, 256, 56, 56, 140, 8, torch.bfloat16),   # 56x56 at C=256: 128-pixel tiles (three ring slots)
    (2, 512, 28, 28, 130, 32, torch.bfloat16),  # 28x28 at C=512: 64-pixel tiles (a 208-pixel ring slot would not fit)
    (2, 64, 24, 24, 20, 8, torch.bfloat16),     # HW == 576 in 8-pixel rows with uncovered channels (residual block)
    (3, 72, 4, 4, 100, 8, torch.float16),       # HW == 16, 16-byte staging stores of one tile
    (59, 512, 7, 7, 601, 32, torch.bfloat16),   # 5 expert tiles (the last of 88 rows), samples split 29 ways
    (59, 192, 6, 6, 601, 16, torch.float16),    # the same through the general one-tile kernel (N = 48)
    (11, 64, 56, 56, 64, 4, torch.bfloat16),    # 143 (sample, tile) units over 143 CTAs: ranges inside samples
    (13, 128, 28, 28, 300, 16, torch.bfloat16), # 3 expert tiles x 49 CTAs over 52 units: ranges cross samples
    (7, 256, 14, 14, 130, 16, torch.float16),   # two expert tiles (the second of one row), one-tile samples
])
def test_tc_mix_matches_oracle(B, C, H_, W_, E, k, dtype):
    gen = torch.Generator().manual_seed(B * 100 + C + k)
    X = torch.randn(B, C, H_, W_, generator=gen).abs()
    L = torch.randn(E - 1, C, generator=gen)
    gw = torch.rand(1, k, generator=gen) - 0.5
    gb = torch.randn(1, generator=gen) * 0.1
    x = X.to(DEV, dtype)
    assert H.tc_supported(x, k)
    H.tc_fault(clear=True)
    y, st = H.forward(x, L.to(DEV), gw.to(DEV), gb.to(DEV), k, 0.1, 10.0, 1.0, path="tc")
    torch.cuda.synchronize()
    assert H.tc_fault() == 0
    ref = O.forward(x.float().cpu().numpy(), L.numpy(), gw.numpy(), gb.numpy(), k, 0.1, 10.0, 1.0, mode="eval")
    got = y.float().cpu().numpy()
    assert close(got, ref, 1e-2, 1e-3), relerr(got, ref)
    _, aux = O.forward(x.float().cpu().numpy(), L.numpy(), gw.numpy(), gb.numpy(), k, 0.1, 10.0, 1.0, mode="eval",
                       return_aux=True)
    assert close(st["T"].cpu().numpy(), aux["T"], 1e-5, 1e-6)


def test_tc_mix_stage4_workload_against_scheduled_path():
    """N=256, C=512, 7x7, E=2048, k=32 (bf16): the tensor-core and the
    scheduled CUDA-core paths agree, and a subset matches the oracle."""
    gen = torch.Generator().manual_seed(7)
    B, C, E, k = 256, 512, 2048, 32
    X = torch.randn(B, C, 7, 7, generator=gen).abs()
    L = torch.randn(E - 1, C, generator=gen)
    gw = torch.rand(1, k, generator=gen) - 0.5
    gb = torch.zeros(1)
    x = X.to(DEV, torch.bfloat16)
    H.tc_fault(clear=True)
    y_tc, _ = H.forward(x, L.to(DEV), gw.to(DEV), gb.to(DEV), k, 0.1, 10.0, 1.0, path="tc")
    y_f, _ = H.forward(x, L.to(DEV), gw.to(DEV), gb.to(DEV), k, 0.1, 10.0, 1.0, path="fast")
    torch.cuda.synchronize()
    assert H.tc_fault() == 0
    a, b = y_tc.float().cpu().numpy(), y_f.float().cpu().numpy()
    assert close(a, b, 1e-2, 1e-3), relerr(a, b)
    ref = O.forward(x[:4].float().cpu().numpy(), L.numpy(), gw.numpy(), gb.numpy(), k, 0.1, 10.0, 1.0, mode="eval")
    assert close(a[:4], ref, 1e-2, 1e-3), relerr(a[:4], ref)


def test_forward_tc_single_call_matches_two_calls():
    """moce_forward_tc (pass 2 as a programmatic dependent of pass 1) gives
    the same bits as moce_pool_stage followed by moce_mix_tc."""
    from moce_thesis_b200 import capi
    gen = torch.Generator().manual_seed(11)
    B, C, Hh, E, k = 6, 256, 14, 300, 16
    x = torch.randn(B, C, Hh, Hh, generator=gen).abs().to(DEV, torch.bfloat16)
    L = torch.randn(E - 1, C, generator=gen).to(DEV)
    gw = (torch.rand(1, k, generator=gen) - 0.5).to(DEV)
    gb = torch.zeros(1, device=DEV)
    r = H.route_build(L, k, transposed=False)
    y2, z2, T2 = H.forward_tc(x, r, gw, gb, 0.1, 9.9)
    y1 = torch.empty_like(y2)
    z1 = torch.empty_like(z2)
    T1 = torch.empty_like(T2)
    xs = torch.empty(capi.lib().moce_tc_stage_bytes(B, C, Hh * Hh), dtype=torch.uint8, device=DEV)
    capi.call("moce_forward_tc", capi.ptr(x), capi.dtype_code(x), B, C, Hh * Hh, capi.ptr(r["mask"]),
              capi.ptr(r["meta"]), capi.ptr(r["idx"]), capi.ptr(r["ln"]), E - 1, k, capi.ptr(gw), capi.ptr(gb),
              0.1, 9.9, capi.ptr(z1), capi.ptr(xs), capi.ptr(y1), capi.ptr(T1), capi.stream_handle())
    torch.cuda.synchronize()
    assert torch.equal(y1, y2) and torch.equal(z1, z2) and torch.equal(T1, T2)


@pytest.mark.parametrize("C,Hh,E,k", [(128, 28, 90, 16), (64, 7, 70, 8), (96, 14, 50, 8), (32, 56, 40, 4)])
def test_tc_unaligned_buffers(C, Hh, E, k):
    """X and Y that start 2 bytes past a 16-byte boundary (views one element
    into larger buffers): pass 1 takes the per-sample cluster kernel and the
    mix stages rows with 16-bit stores and element copies; results match the
    oracle."""
    from moce_thesis_b200 import capi
    gen = torch.Generator().manual_seed(C + Hh)
    B = 2
    HW = Hh * Hh
    X = torch.randn(B, C, Hh, Hh, generator=gen).abs()
    L = torch.randn(E - 1, C, generator=gen)
    gw = (torch.rand(1, k, generator=gen) - 0.5).to(DEV)
    gb = torch.zeros(1, device=DEV)
    xbuf = torch.empty(B * C * HW + 8, dtype=torch.bfloat16, device=DEV)
    x = xbuf[1:1 + B * C * HW].view(B, C, Hh, Hh)
    x.copy_(X.to(DEV, torch.bfloat16))
    ybuf = torch.zeros(B * E * HW + 8, dtype=torch.bfloat16, device=DEV)
    y = ybuf[1:1 + B * E * HW].view(B, E, Hh, Hh)
    assert x.data_ptr() % 16 == 2 and y.data_ptr() % 16 == 2
    r = H.route_build(L.to(DEV), k, transposed=False)
    z = torch.empty(B, C, device=DEV)
    T = torch.empty(B, E - 1, device=DEV)
    xs = torch.empty(capi.lib().moce_tc_stage_bytes(B, C, HW), dtype=torch.uint8, device=DEV)
    H.tc_fault(clear=True)
    capi.call("moce_forward_tc", capi.ptr(x), capi.dtype_code(x), B, C, HW, capi.ptr(r["mask"]),
              capi.ptr(r["meta"]), capi.ptr(r["idx"]), capi.ptr(r["ln"]), E - 1, k, capi.ptr(gw), capi.ptr(gb),
              0.1, 9.9, capi.ptr(z), capi.ptr(xs), capi.ptr(y), capi.ptr(T), capi.stream_handle())
    torch.cuda.synchronize()
    assert H.tc_fault() == 0
    assert ybuf[0].item() == 0 and float(ybuf[1 + B * E * HW:].abs().sum()) == 0   # nothing outside Y
    ref = O.forward(x.float().cpu().numpy(), L.numpy(), gw.cpu().numpy(), gb.cpu().numpy(), k, 0.1, 10.0, 1.0,
                    mode="eval")
    got = y.float().cpu().numpy()
    assert close(got, ref, 1e-2, 1e-3), relerr(got, ref)


@pytest.mark.parametrize("C,Hh,E,k,relu,B", [
    (512, 7, 300, 32, True, 3),     # 7x7 one tile, two partial accumulators
    (256, 14, 140, 16, True, 3),    # 14x14 one tile, one accumulator
    (128, 28, 90, 16, False, 3),    # 28x28 pixel tiles through padded staging rows, no ReLU
    (96, 12, 4, 8, True, 3),        # uncovered channels: the residual row goes through the epilogue too
    (512, 7, 601, 32, True, 59),    # 5 expert tiles, the last of 88 rows, 2-3 samples per block
])
def test_forward_tc_ep_matches_bn_relu(C, Hh, E, k, relu, B):
    """moce_forward_tc_ep (BatchNorm folded to scale / shift and ReLU applied
    in the output store) against forward_tc followed by torch's eval
    BatchNorm and ReLU on the same inputs (bf16 tolerance)."""
    from moce_thesis_b200 import capi
    gen = torch.Generator().manual_seed(C + k)
    x = torch.randn(B, C, Hh, Hh, generator=gen).abs().to(DEV, torch.bfloat16)
    L = torch.randn(E - 1, C, generator=gen).to(DEV)
    gw = (torch.rand(1, k, generator=gen) - 0.5).to(DEV)
    gb = torch.zeros(1, device=DEV)
    bn = torch.nn.BatchNorm2d(E).to(DEV).eval()
    with torch.no_grad():
        bn.weight.copy_(torch.rand(E, generator=gen) * 2 - 0.5)
        bn.bias.copy_(torch.randn(E, generator=gen) * 0.2)
        bn.running_mean.copy_(torch.randn(E, generator=gen) * 0.1)
        bn.running_var.copy_(torch.rand(E, generator=gen) + 0.5)
    r = H.route_build(L, k, transposed=False)
    y0, z0, _ = H.forward_tc(x, r, gw, gb, 0.1, 9.9)
    with torch.no_grad():
        ref = bn(y0.float())
        ref = torch.relu(ref) if relu else ref
        inv = torch.rsqrt(bn.running_var + bn.eps)
        scale = (bn.weight * inv).contiguous()
        shift = (bn.bias - bn.running_mean * bn.weight * inv).contiguous()
    y = torch.empty_like(y0)
    z = torch.empty_like(z0)
    xs = torch.empty(capi.lib().moce_tc_stage_bytes(B, C, Hh * Hh), dtype=torch.uint8, device=DEV)
    H.tc_fault(clear=True)
    capi.call("moce_forward_tc_ep", capi.ptr(x), capi.dtype_code(x), B, C, Hh * Hh, capi.ptr(r["mask"]),
              capi.ptr(r["meta"]), capi.ptr(r["idx"]), capi.ptr(r["ln"]), E - 1, k, capi.ptr(gw), capi.ptr(gb),
              0.1, 9.9, capi.ptr(scale), capi.ptr(shift), 1 if relu else 0, capi.ptr(z), capi.ptr(xs), capi.ptr(y),
              None, capi.stream_handle())
    torch.cuda.synchronize()
    assert H.tc_fault() == 0
    assert torch.equal(z, z0)
    got, want = y.float().cpu().numpy(), ref.cpu().numpy()
    assert close(got, want, 1e-2, 1e-3), relerr(got, want)
    if relu:
        assert float(y.float().min()) >= 0.0
