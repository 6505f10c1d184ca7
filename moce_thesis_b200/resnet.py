"""ResNet-50 with MoCE bottleneck entrances, on the native MoCE layer.

The caller of the hot path in the reference (Elianiluk/MoCE_thesis
``models_unified.py:110-290``), kept with the same constructor arguments,
module names and state_dict keys so that its checkpoints load: each
bottleneck's first 1x1 convolution is a ``MoCE`` layer with
E = C_in / sampling_factor outputs (sampling factor 1 for the first block of
layer1, 2 for the other first blocks, 4 elsewhere, ``models_unified.py:
227-258``), followed by BatchNorm and ReLU (or a 1x1 projection when E differs
from the block width).  The convolutions, BatchNorms and the classifier are
torch / cuDNN.

What differs: in eval mode a block without projection runs MoCE -> bn1 ->
relu1 as one native call (``MoCE.forward_eval_bn_relu``: on the tensor-core
path the BatchNorm, folded to a per-channel scale and shift, and the ReLU are
applied in the mix's output store), and the block's other BatchNorms run as
one native pass each with what follows them (``moce_bn_act``: relu2(bn2(.)),
and relu3(bn3(.) + shortcut) with the shortcut's own BatchNorm folded in),
as does the stem's BatchNorm and ReLU.  ``fuse_epilogue=False`` on a block,
or ``set_fused_epilogue(model, False)``, restores the separate torch ops.
"""
from __future__ import annotations

import torch
import torch.nn as nn

from .moce import MoCE, native

# per-block k (one list per stage), models_unified.py:25-30
DEFAULT_MOCE_K_50 = [[8, 8, 8], [12, 12, 12, 12], [24] * 6, [48, 48, 48]]


def _bn_eval(bn) -> bool:
    """An eval-mode BatchNorm2d with running statistics (foldable)."""
    return (isinstance(bn, nn.BatchNorm2d) and not bn.training and bn.running_mean is not None
            and bn.running_var is not None)


def bn_affine(bn):
    """The eval BatchNorm as fp32 (scale, shift) per channel: scale = weight /
    sqrt(running_var + eps), shift = bias - running_mean * scale.  Cached on
    the module per version of its buffers and parameters."""
    ts = (bn.running_mean, bn.running_var, bn.weight, bn.bias)
    key = tuple((t.data_ptr(), t._version, t.device) if t is not None else None for t in ts) + (float(bn.eps),)
    hit = bn.__dict__.get("_moce_affine")
    if hit is not None and hit[0] == key:
        return hit[1]
    with torch.no_grad():
        inv = torch.rsqrt(bn.running_var.float() + float(bn.eps))
        scale = inv if bn.weight is None else bn.weight.float() * inv
        shift = -bn.running_mean.float() * scale
        if bn.bias is not None:
            shift = shift + bn.bias.float()
    val = (scale.contiguous(), shift.contiguous())
    bn.__dict__["_moce_affine"] = (key, val)
    return val


def normalize_k_config(k, layers_config):
    """An int (same k everywhere) or one list of k per stage, one value per
    block (models_unified.py:47-69)."""
    if isinstance(k, int):
        return [[k] * n for n in layers_config]
    if not isinstance(k, (list, tuple)) or len(k) != len(layers_config):
        raise ValueError(f"k must be an int or a list with {len(layers_config)} stage lists.")
    out = []
    for i, (ks, n) in enumerate(zip(k, layers_config)):
        if not isinstance(ks, (list, tuple)) or len(ks) != n:
            raise ValueError(f"k[{i}] must contain exactly {n} values.")
        out.append(list(ks))
    return out


class BottleneckWithMoCEProjection(nn.Module):
    """Bottleneck whose entrance 1x1 convolution is a MoCE layer
    (models_unified.py:110-169)."""

    expansion = 4

    def __init__(self, in_channels, mid_channels, stride=1, sampling_factor=4, k=8):
        super().__init__()
        self.moce = MoCE(in_channels, sampling_factor=sampling_factor, k=k)
        squeezed = in_channels // sampling_factor
        if squeezed != mid_channels:
            self.projection = nn.Conv2d(squeezed, mid_channels, 1, bias=False)
            self.bn_proj = nn.BatchNorm2d(mid_channels)
        else:
            self.projection = None
            self.bn1 = nn.BatchNorm2d(squeezed)
        self.relu1 = nn.ReLU(inplace=True)
        self.conv2 = nn.Conv2d(mid_channels, mid_channels, 3, stride, 1, bias=False)
        self.bn2 = nn.BatchNorm2d(mid_channels)
        self.relu2 = nn.ReLU(inplace=True)
        self.conv3 = nn.Conv2d(mid_channels, mid_channels * self.expansion, 1, bias=False)
        self.bn3 = nn.BatchNorm2d(mid_channels * self.expansion)
        self.shortcut = nn.Sequential()
        if stride != 1 or in_channels != mid_channels * self.expansion:
            self.shortcut = nn.Sequential(
                nn.Conv2d(in_channels, mid_channels * self.expansion, 1, stride, bias=False),
                nn.BatchNorm2d(mid_channels * self.expansion))
        self.relu3 = nn.ReLU(inplace=True)
        self.fuse_epilogue = True

    def forward(self, x):
        if self.projection is None and not self.training and self.fuse_epilogue:
            out = self.moce.forward_eval_bn_relu(x, self.bn1, relu=True)
        elif (self.projection is not None and not self.training and self.fuse_epilogue and x.is_cuda
              and _bn_eval(self.bn_proj)):
            # MoCE, the projection, then relu1(bn_proj(.)) as one native pass
            out = self.projection(self.moce(x)).contiguous()
            out = native().bn_act(out, *bn_affine(self.bn_proj), relu=True, out=out)
        else:
            out = self.moce(x)
            out = self.bn_proj(self.projection(out)) if self.projection is not None else self.bn1(out)
            out = self.relu1(out)
        sc_bn = self.shortcut[1] if len(self.shortcut) == 2 else None
        if (not self.training and self.fuse_epilogue and out.is_cuda and _bn_eval(self.bn2) and _bn_eval(self.bn3)
                and (sc_bn is None or _bn_eval(sc_bn))):
            # relu2(bn2(conv2)) and relu3(bn3(conv3) + shortcut) as one
            # native pass each, in place on the convolution outputs
            m = native()
            out = self.conv2(out).contiguous()
            out = m.bn_act(out, *bn_affine(self.bn2), relu=True, out=out)
            out = self.conv3(out).contiguous()
            if sc_bn is None:
                return m.bn_act(out, *bn_affine(self.bn3), x.contiguous(), relu=True, out=out)
            r = self.shortcut[0](x).contiguous()
            return m.bn_act(out, *bn_affine(self.bn3), r, *bn_affine(sc_bn), relu=True, out=out)
        out = self.relu2(self.bn2(self.conv2(out)))
        out = self.bn3(self.conv3(out))
        out = out + self.shortcut(x)
        return self.relu3(out)


class ResNet50(nn.Module):
    """ResNet-50 layout with a dataset-specific stem (models_unified.py:172-290)."""

    def __init__(self, block=BottleneckWithMoCEProjection, num_classes=100, reduction_ratios=None,
                 sampling_factor=None, dataset="cifar100", k=8, layers_config=None):
        super().__init__()
        if block is not BottleneckWithMoCEProjection:
            raise ValueError("only the MoCE bottleneck is provided here")
        self.in_channels = 64
        self.block = block
        self.dataset = dataset.lower()
        self.k = k
        self.layers_config = layers_config or [3, 4, 6, 3]
        if self.dataset not in {"cifar100", "imagenet"}:
            raise ValueError(f"Unsupported dataset '{dataset}'. Use 'cifar100' or 'imagenet'.")
        self.sampling_factor = 4 if sampling_factor is None else sampling_factor
        self.reduction_ratios = None
        self.k_per_block = normalize_k_config(k, self.layers_config)
        if self.dataset == "imagenet":
            self.conv1 = nn.Conv2d(3, 64, kernel_size=7, stride=2, padding=3, bias=False)
            self.maxpool = nn.MaxPool2d(kernel_size=3, stride=2, padding=1)
        else:
            self.conv1 = nn.Conv2d(3, 64, kernel_size=3, stride=1, padding=1, bias=False)
            self.maxpool = nn.Identity()
        self.bn1 = nn.BatchNorm2d(64)
        self.relu = nn.ReLU(inplace=True)
        self.fuse_epilogue = True
        widths, strides = (64, 128, 256, 512), (1, 2, 2, 2)
        for i in range(4):
            setattr(self, f"layer{i + 1}", self._make_layer(widths[i], self.layers_config[i], strides[i], i))
        self.avgpool = nn.AdaptiveAvgPool2d((1, 1))
        self.fc = nn.Linear(512 * BottleneckWithMoCEProjection.expansion, num_classes)
        self._initialize_weights()

    def _make_layer(self, mid_channels, blocks, stride, layer_idx):
        # first block: sampling factor 1 in layer1, 2 elsewhere; then 4
        ks = self.k_per_block[layer_idx]
        layers = [BottleneckWithMoCEProjection(self.in_channels, mid_channels, stride,
                                               sampling_factor=1 if layer_idx == 0 else 2, k=ks[0])]
        self.in_channels = mid_channels * BottleneckWithMoCEProjection.expansion
        for j in range(1, blocks):
            layers.append(BottleneckWithMoCEProjection(self.in_channels, mid_channels, 1, sampling_factor=4, k=ks[j]))
        return nn.Sequential(*layers)

    def _initialize_weights(self):
        # Kaiming-normal convolutions, unit BatchNorm, N(0, 0.01) classifier;
        # MoCE layers keep their own initialisation
        for m in self.modules():
            if isinstance(m, MoCE):
                continue
            if isinstance(m, nn.Conv2d):
                nn.init.kaiming_normal_(m.weight, mode="fan_out", nonlinearity="relu")
            elif isinstance(m, nn.BatchNorm2d):
                nn.init.constant_(m.weight, 1)
                nn.init.constant_(m.bias, 0)
            elif isinstance(m, nn.Linear):
                nn.init.normal_(m.weight, 0, 0.01)
                if m.bias is not None:
                    nn.init.constant_(m.bias, 0)

    def forward(self, x):
        if not self.training and self.fuse_epilogue and x.is_cuda and _bn_eval(self.bn1):
            y = self.conv1(x).contiguous()
            x = self.maxpool(native().bn_act(y, *bn_affine(self.bn1), relu=True, out=y))
        else:
            x = self.maxpool(self.relu(self.bn1(self.conv1(x))))
        x = self.layer4(self.layer3(self.layer2(self.layer1(x))))
        return self.fc(torch.flatten(self.avgpool(x), 1))


def resnet50_moce_projection(sampling_factor=4, k=DEFAULT_MOCE_K_50, **kwargs):
    """ResNet-50 + MoCE (models_unified.py:305-316)."""
    return ResNet50(BottleneckWithMoCEProjection, sampling_factor=sampling_factor, k=k,
                    layers_config=[3, 4, 6, 3], **kwargs)


def build_moce_cache(model):
    """Build every MoCE layer's eval cache (the reference test.py:356-360)."""
    m = model.module if hasattr(model, "module") else model
    for module in m.modules():
        if hasattr(module, "build_eval_cache"):
            module.build_eval_cache()


def set_fused_epilogue(model, on=True):
    """Switch the eval-mode MoCE -> bn1 -> relu1 fusion of every block."""
    for module in model.modules():
        if isinstance(module, (BottleneckWithMoCEProjection, ResNet50)):
            module.fuse_epilogue = bool(on)

