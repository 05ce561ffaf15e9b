"""GroupedInt8RotLinear on the CPU: the torch path of each layer, and the constructor's checks."""

from __future__ import annotations

import pytest
import torch

from hyperflow_h3_flash_b200 import int8 as I
from hyperflow_h3_flash_b200 import synthetic
from hyperflow_h3_flash_b200.grouped import GroupedInt8RotLinear


def _layer(K, N, r, bias, seed):
    w = synthetic.linear_weights(K, N, rank=r, bias=bias, group=256, seed_offset=seed)
    ly = I.Int8RotLinear(K, N, 256, bias=bias, rank=r)
    synthetic.load_into(ly, w)
    return ly


def test_cpu_forward_is_each_layer_on_its_own():
    layers = [_layer(512, 256, 16, True, s) for s in range(3)]
    x = synthetic.activations(20, 512, seed=5)
    outs = GroupedInt8RotLinear(*layers)(x)
    assert len(outs) == 3
    for ly, o in zip(layers, outs, strict=True):
        assert torch.equal(o, ly(x))


def test_the_group_adds_no_state():
    layers = [_layer(512, 256, 0, False, s) for s in range(2)]
    group = GroupedInt8RotLinear(*layers)
    assert not group.state_dict() and group.layers == tuple(layers)


def test_constructor_checks():
    a = _layer(512, 256, 16, True, 1)
    with pytest.raises(ValueError):
        GroupedInt8RotLinear(a)  # one layer
    with pytest.raises(ValueError):
        GroupedInt8RotLinear(a, _layer(512, 512, 16, True, 2))  # different widths
    with pytest.raises(ValueError):
        GroupedInt8RotLinear(a, _layer(512, 256, 16, False, 3))  # bias on one only
    with pytest.raises(ValueError):
        GroupedInt8RotLinear(_layer(512, 256, 12, True, 4), _layer(512, 256, 12, True, 5))  # rank % 8
    with pytest.raises(ValueError):
        GroupedInt8RotLinear(_layer(512, 160, 16, True, 6), _layer(512, 160, 16, True, 7))  # width % 256 with rank


def test_groups_built_under_inference_mode_work():
    with torch.inference_mode():
        layers = [_layer(512, 256, 16, True, s) for s in range(2)]
        group = GroupedInt8RotLinear(*layers)
        group._stacked()  # inference tensors have no version counter; the cache keys them by address
        x = synthetic.activations(9, 512, seed=6)
        outs = group(x)
        assert all(torch.equal(o, ly(x)) for ly, o in zip(layers, outs, strict=True))
