"""Record the state_dict layout of the reference ResNet-50 + MoCE model.

Run in the development container, where the reference checkout exists:

    python tests/golden/make_resnet_keys.py <path of the reference checkout>

Imports the unmodified ``models_unified.py`` (its ``import moce_fixed.moce_cuda``
is satisfied by an empty stub module: building the model calls no kernel) and
writes ``resnet50_moce_keys.json``: {key: shape} of
``resnet50_moce_projection(dataset, num_classes)`` for the ImageNet and CIFAR
stems, so that a test can check that reference checkpoints load into
``moce_thesis_b200.resnet``.
"""
from __future__ import annotations

import json
import os
import sys
import types

import torch

HERE = os.path.dirname(os.path.abspath(__file__))


def main(ref):
    pkg = types.ModuleType("moce_fixed")
    mod = types.ModuleType("moce_fixed.moce_cuda")
    pkg.moce_cuda = mod
    sys.modules["moce_fixed"] = pkg
    sys.modules["moce_fixed.moce_cuda"] = mod
    sys.path.insert(0, ref)
    import models_unified as M  # the reference module, unmodified
    out = {}
    for name, kw in (("imagenet_1000", dict(dataset="imagenet", num_classes=1000)),
                     ("cifar100_100", dict(dataset="cifar100", num_classes=100))):
        torch.manual_seed(0)
        m = M.resnet50_moce_projection(**kw)
        out[name] = {k: list(v.shape) for k, v in m.state_dict().items()}
    with open(os.path.join(HERE, "resnet50_moce_keys.json"), "w") as f:
        json.dump(out, f, indent=0, sort_keys=True)


if __name__ == "__main__":
    if len(sys.argv) != 2:
        sys.exit("usage: python tests/golden/make_resnet_keys.py <path of the reference checkout>")
    main(sys.argv[1])
