"""The ResNet-50 + MoCE caller (moce_thesis_b200.resnet) has the reference
model's state_dict layout, so reference checkpoints load into it.

The fixture ``golden/resnet50_moce_keys.json`` is written by
``golden/make_resnet_keys.py`` from the unmodified reference
``models_unified.py``.  Building the model runs no kernel (CPU only).
"""
import json
import os

import pytest
import torch

from moce_thesis_b200 import resnet

HERE = os.path.dirname(os.path.abspath(__file__))


@pytest.mark.parametrize("name,kw", [("imagenet_1000", dict(dataset="imagenet", num_classes=1000)),
                                     ("cifar100_100", dict(dataset="cifar100", num_classes=100))])
def test_state_dict_layout_matches_reference(name, kw):
    want = json.load(open(os.path.join(HERE, "golden", "resnet50_moce_keys.json")))[name]
    torch.manual_seed(0)
    m = resnet.resnet50_moce_projection(**kw)
    got = {k: list(v.shape) for k, v in m.state_dict().items()}
    assert got == want
    # a checkpoint with the reference's keys and shapes loads strictly
    sd = {k: torch.zeros(s) for k, s in want.items()}
    m.load_state_dict(sd, strict=True)


def test_moce_layers_and_k_config():
    m = resnet.resnet50_moce_projection(dataset="imagenet", num_classes=1000,
                                        k=[[4, 16, 16], [16, 32, 32, 32], [32] + [64] * 5, [64, 128, 128]])
    layers = [b.moce for b in m.modules() if isinstance(b, resnet.BottleneckWithMoCEProjection)]
    assert len(layers) == 16
    # E = C_in / sampling factor: 1 for layer1's first block, 2 for the other first blocks, 4 elsewhere
    assert [(l.in_channels, l.num_experts, l.k) for l in layers[:5]] == [
        (64, 64, 4), (256, 64, 16), (256, 64, 16), (256, 128, 16), (512, 128, 32)]
    assert (layers[-1].in_channels, layers[-1].num_experts, layers[-1].k) == (2048, 512, 128)
    with pytest.raises(ValueError):
        resnet.normalize_k_config([[8]], [3, 4, 6, 3])

