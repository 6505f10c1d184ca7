"""GPU parity of the fused block epilogue (moce_bn_act) and of the ResNet-50 +
MoCE eval forward that uses it.

* moce_bn_act against the same fp32 arithmetic in torch (a folded BatchNorm,
  an optional residual with an optional affine of its own, an optional
  ReLU, one rounding), for fp32 / bf16 / fp16, with 16-, 8-, 4-byte or
  element access and vectors inside channel rows or across them (7x7 maps,
  rows shorter than a vector): fp32 within 1e-6, 16-bit outputs within one
  unit in the last place;
* against torch's eval BatchNorm2d, add and ReLU modules;
* NaN stays NaN through the ReLU;
* the ResNet-50 + MoCE eval forward with the fused epilogues against the
  same model running the reference's torch ops, bf16 within 2e-2 of the
  largest logit.
"""
import pytest
import torch
import torch.nn.functional as F

pytestmark = pytest.mark.gpu
DEV = "cuda:0"


def _native():
    from moce_thesis_b200 import native
    return native()


def _bn(C, gen):
    bn = torch.nn.BatchNorm2d(C).eval()
    with torch.no_grad():
        bn.running_mean.copy_(torch.randn(C, generator=gen) * 0.5)
        bn.running_var.copy_(torch.rand(C, generator=gen) + 0.5)
        bn.weight.copy_(torch.randn(C, generator=gen))
        bn.bias.copy_(torch.randn(C, generator=gen) * 0.1)
    return bn.to(DEV)


def _affine(bn):
    from moce_thesis_b200.resnet import bn_affine
    return bn_affine(bn)


@pytest.mark.parametrize("dtype", [torch.float32, torch.bfloat16, torch.float16])
@pytest.mark.parametrize("shape", [
    (4, 64, 56, 56),     # 16-byte vectors inside channel rows
    (3, 256, 7, 7),      # 49-pixel rows: vectors span rows
    (2, 96, 14, 14),     # 196-pixel rows
    (5, 3, 1, 1),        # 15 elements: element access
    (2, 6, 3, 5),        # 15-pixel rows, vectors across rows and samples
    (4, 6, 1, 2),        # rows shorter than a vector
])
@pytest.mark.parametrize("mode", ["bn_relu", "bn_res_relu", "bn_bnres_relu", "bn_only"])
def test_bn_act_matches_fp32_arithmetic(dtype, shape, mode):
    N, C, H, W = shape
    gen = torch.Generator().manual_seed(N * 1000 + C + H)
    x = torch.randn(shape, generator=gen).to(DEV, dtype)
    r = torch.randn(shape, generator=gen).to(DEV, dtype)
    bn, bnr = _bn(C, gen), _bn(C, gen)
    s, t = _affine(bn)
    rs, rt = _affine(bnr)
    m = _native()
    relu = mode != "bn_only"
    if mode in ("bn_relu", "bn_only"):
        y = m.bn_act(x, s, t, relu=relu)
        want = x.float() * s.view(1, -1, 1, 1) + t.view(1, -1, 1, 1)
    elif mode == "bn_res_relu":
        y = m.bn_act(x, s, t, r, relu=True)
        want = (x.float() * s.view(1, -1, 1, 1) + t.view(1, -1, 1, 1)) + r.float()
    else:
        y = m.bn_act(x, s, t, r, rs, rt, relu=True)
        want = (x.float() * s.view(1, -1, 1, 1) + t.view(1, -1, 1, 1)) + \
               (r.float() * rs.view(1, -1, 1, 1) + rt.view(1, -1, 1, 1))
    if relu:
        want = torch.relu(want)
    torch.cuda.synchronize()
    if dtype == torch.float32:
        torch.testing.assert_close(y, want, rtol=1e-6, atol=1e-6)
    else:
        # one rounding of the fp32 result: equal to want rounded, up to the
        # fused multiply-adds' last bit landing on a rounding boundary
        eps = torch.finfo(dtype).eps
        torch.testing.assert_close(y.float(), want.to(dtype).float(), rtol=eps, atol=1e-6)


@pytest.mark.parametrize("dtype", [torch.float32, torch.bfloat16])
def test_bn_act_matches_torch_modules(dtype):
    gen = torch.Generator().manual_seed(7)
    N, C, H, W = 3, 128, 28, 28
    x = torch.randn(N, C, H, W, generator=gen).to(DEV, dtype)
    sc = torch.randn(N, C, H, W, generator=gen).to(DEV, dtype)
    bn3, bnsc = _bn(C, gen).to(dtype), _bn(C, gen).to(dtype)
    with torch.no_grad():
        want = F.relu(bn3(x) + bnsc(sc))
        y = _native().bn_act(x, *_affine(bn3), sc, *_affine(bnsc), relu=True)
    torch.cuda.synchronize()
    tol = 1e-5 if dtype == torch.float32 else 2e-2
    torch.testing.assert_close(y.float(), want.float(), rtol=tol, atol=tol)


def test_bn_act_in_place_and_nan():
    gen = torch.Generator().manual_seed(3)
    x = torch.randn(2, 8, 7, 7, generator=gen).to(DEV, torch.bfloat16)
    x[0, 1, 2, 3] = float("nan")
    s = torch.ones(8, device=DEV)
    t = torch.zeros(8, device=DEV)
    want = torch.relu(x.float()).to(torch.bfloat16)
    want[0, 1, 2, 3] = float("nan")
    y = _native().bn_act(x, s, t, relu=True, out=x)
    torch.cuda.synchronize()
    assert y.data_ptr() == x.data_ptr()
    assert torch.isnan(y[0, 1, 2, 3])
    torch.testing.assert_close(y, want, equal_nan=True)


def test_resnet50_fused_epilogues_match_torch_ops():
    from moce_thesis_b200 import resnet
    torch.manual_seed(0)
    kcfg = [[4, 16, 16], [16, 32, 32, 32], [32, 64, 64, 64, 64, 64], [64, 128, 128]]
    model = resnet.resnet50_moce_projection(dataset="imagenet", num_classes=1000, k=kcfg)
    gen = torch.Generator().manual_seed(1)
    with torch.no_grad():
        for mod in model.modules():
            if isinstance(mod, torch.nn.BatchNorm2d):       # non-trivial folded affines
                mod.running_mean.copy_(torch.randn(mod.num_features, generator=gen) * 0.1)
                mod.running_var.copy_(torch.rand(mod.num_features, generator=gen) + 0.5)
                mod.weight.copy_(torch.rand(mod.num_features, generator=gen) + 0.5)
                mod.bias.copy_(torch.randn(mod.num_features, generator=gen) * 0.1)
    model = model.to(DEV, torch.bfloat16).eval()
    resnet.build_moce_cache(model)
    x = torch.randn(4, 3, 224, 224, generator=gen).to(DEV, torch.bfloat16)
    with torch.no_grad():
        resnet.set_fused_epilogue(model, True)
        y = model(x).float()
        resnet.set_fused_epilogue(model, False)
        want = model(x).float()
    torch.cuda.synchronize()
    assert torch.isfinite(y).all()
    err = (y - want).abs().max().item()
    assert err <= 2e-2 * want.abs().max().item() + 1e-3, (err, want.abs().max().item())
