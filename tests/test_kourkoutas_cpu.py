"""Kourkoutas-beta host logic without a GPU: the layer map
(Kourkoutas.py:25-57) and its one-prepare-launch-per-group ranges."""
from collections import defaultdict

import pytest
import torch

from advanced_optimizers_b200.optim._kourkoutas import KourkoutasBeta, default_layer_key


class _Opt:
    def __init__(self, groups, layer_key_fn=None):
        self.param_groups = groups
        self.defaults = dict(kourkoutas_beta=True, betas=(0.9, 0.999), beta2_min=0.9, ema_alpha=0.95,
                             tiny_spike=1e-9, k_warmup_steps=0)
        self.state = defaultdict(dict)
        self.layer_key_fn = layer_key_fn


def _p(*shape):
    return torch.nn.Parameter(torch.zeros(shape))


def test_default_key_buckets_by_shape_and_isolates_adapters():
    a, b, c = _p(8, 4), _p(8, 4), _p(4)
    d = _p(4)
    d._is_dora_scale = True
    opt = _Opt([{"params": [a, b, c, d], "kourkoutas_beta": True}])
    kk = KourkoutasBeta(opt)
    assert opt.layer_key_fn is default_layer_key
    assert kk.n == 3
    assert kk.layer_index(a) == kk.layer_index(b) == 0
    assert kk.layer_index(c) == 1
    assert kk.layer_index(d) == 2          # a DoRA scale is its own layer, keyed by id
    assert kk.layer_table([c, a, d]) == [1, 0, 2]


def test_groups_without_kourkoutas_are_left_out_and_ranges_are_per_group():
    a, b, c, e = _p(8, 4), _p(16), _p(8, 4), _p(3, 3)
    g0 = {"params": [a, b], "kourkoutas_beta": True}
    g1 = {"params": [e], "kourkoutas_beta": False}
    g2 = {"params": [c, e], "kourkoutas_beta": True, "beta2_min": 0.8}
    opt = _Opt([g0, g1, g2])
    kk = KourkoutasBeta(opt)
    # c shares a's shape: same layer, whose hyperparameters come from g0 (the first group holding it)
    assert kk.layer_index(c) == kk.layer_index(a) == 0
    assert kk.layer_index(e) == 2
    assert [(r[0] is g0, r[1], r[2]) for r in kk.ranges] == [(True, 0, 2), (False, 2, 3)]
    assert kk.ranges[1][0] is g2


def test_custom_layer_key_fn():
    a, b, c = _p(8, 4), _p(8, 4), _p(4)
    names = {id(a): "block0", id(b): "block1", id(c): "block0"}
    opt = _Opt([{"params": [a, b, c], "kourkoutas_beta": True}], layer_key_fn=lambda p: names[id(p)])
    kk = KourkoutasBeta(opt)
    assert kk.layer_index(a) == kk.layer_index(c) == 0
    assert kk.layer_index(b) == 1


def test_lora_params_are_rejected():
    a = _p(8, 4)
    a._is_lora_A = True
    with pytest.raises(NotImplementedError):
        KourkoutasBeta(_Opt([{"params": [a], "kourkoutas_beta": True}]))


def test_prepare_once_per_step():
    a = _p(8, 4)
    kk = KourkoutasBeta(_Opt([{"params": [a], "kourkoutas_beta": True}]))
    calls = []
    kk.prepare = lambda step, device, d_dev=0: calls.append((step, d_dev))
    kk.maybe_prepare(0, None)
    kk.maybe_prepare(0, None)
    kk.maybe_prepare(1, None, d_dev=4096)
    assert calls == [(0, 0), (1, 4096)]
