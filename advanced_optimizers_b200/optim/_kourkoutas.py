"""Kourkoutas-beta on the device: a layer-wise dynamic beta2 for the Adam
family (Kourkoutas.py:6-257, KourkoutasHelper).

Each layer (params sharing a layer key; the param's shape by default,
Kourkoutas.py:34-47) keeps a float32 EMA of its pooled grad norm.  At the
start of a step, for the norm pooled over the PREVIOUS step's grads,

    ema    = ema * alpha + (1 - alpha) * pooled          (Kourkoutas.py:165)
    raw    = pooled / (ema + tiny_spike)
    beta2  = (1 - w) * beta2_max + w * (beta2_max - (beta2_max - beta2_min) * raw / (1 + raw))

with w = min(1, step / k_warmup_steps) (Kourkoutas.py:169-179).  The step's
v update then uses beta2 and 1 - beta2 of the tensor's layer; bias
correction keeps betas[1] (AdamW_adv.py:289-302).

The reference keeps one 0-dim tensor per layer and reads each beta2 back to
the host (`.item()`, Kourkoutas.py:182-185); here every layer lives in three
device arrays and nothing is read back:

    advopt_kourkoutas_prepare     ema, layer_beta2 from acc; acc = 0 (one launch per group of layers)
    advopt_adam_step              v update with layer_beta2; per-piece sum(g*g) (ADVOPT_F_GRAD_SQ)
    advopt_kourkoutas_accumulate  acc[layer] += each tensor's sum (one launch per step launch)

state[p]['kourkoutas_r_ema'] of every param of a layer is a 0-dim view of
that layer's EMA entry, so state_dict() saves it under the reference's key;
a loaded value is adopted at the next prepare (Kourkoutas.py:84-101).
"""
from __future__ import annotations

import ctypes

import numpy as np
import torch

from .. import _lib as L
from .._device import stream_handle


def default_layer_key(p):
    """Kourkoutas.py:38-46: adapters get a layer of their own, every other
    param is bucketed by shape."""
    if (getattr(p, "_is_oft", False) or getattr(p, "_is_lora_A", False) or getattr(p, "_is_lora_B", False)
            or getattr(p, "_is_dora_scale", False)):
        return (id(p),)
    return tuple(p.shape)


class KourkoutasBeta:
    """Device-resident KourkoutasHelper for one optimizer.  `prefix` is
    'adam_' for the hybrid optimizers' auxiliary Adam (Kourkoutas.py:152-158)."""

    def __init__(self, optimizer, prefix: str = ""):
        self.optimizer = optimizer
        self.prefix = prefix
        if getattr(optimizer, "layer_key_fn", None) is None:
            optimizer.layer_key_fn = default_layer_key
        self.key_fn = optimizer.layer_key_fn
        self.enable_key = f"{prefix}kourkoutas_beta"
        self.layer_of = {}     # layer key -> index
        self.layer_params = []  # index -> params (in group order)
        self.layer_group = []   # index -> the group whose hyperparameters the layer uses
        for group in optimizer.param_groups:
            if not group.get("kourkoutas_beta", False) and not group.get("adam_kourkoutas_beta", False):
                continue
            for p in group["params"]:
                if getattr(p, "_is_oft", False) or getattr(p, "_is_lora_A", False) or getattr(p, "_is_lora_B", False):
                    raise NotImplementedError(
                        "Kourkoutas-beta on LoRA / OFT adapter params (a per-row beta2) is not supported by the "
                        "B200 kernels")
                k = self.key_fn(p)
                li = self.layer_of.get(k)
                if li is None:
                    li = len(self.layer_params)
                    self.layer_of[k] = li
                    self.layer_params.append([])
                    self.layer_group.append(group)
                self.layer_params[li].append(p)
        self.n = len(self.layer_params)
        # layers are numbered group by group, so the layers of one group form
        # one contiguous range: one prepare launch per group
        self.ranges = []
        for li, g in enumerate(self.layer_group):
            if self.ranges and self.ranges[-1][0] is g:
                self.ranges[-1][2] = li + 1
            else:
                self.ranges.append([g, li, li + 1])
        self.device = None
        self.acc = self.ema = self.beta2 = None
        self.views = [None] * self.n
        self.adopted = False
        self.prepared_step = -1
        self.launches = 0

    def _alloc(self, device):
        if self.acc is not None:
            if self.device != device:
                raise NotImplementedError("Kourkoutas-beta needs all of an optimizer's params on one device")
            return
        self.device = device
        n = max(1, self.n)
        self.acc = torch.zeros(n, dtype=torch.float32, device=device)
        self.ema = torch.zeros(n, dtype=torch.float32, device=device)
        self.beta2 = torch.zeros(2 * n, dtype=torch.float32, device=device)

    def layer_index(self, p) -> int:
        """The param's layer, or -1 for a param outside every Kourkoutas group."""
        return self.layer_of.get(self.key_fn(p), -1) if self.n else -1

    def _hp(self, group, name):
        key = f"{self.prefix}{name}"
        return group.get(key, self.optimizer.defaults[key])

    def _adopt_states(self):
        """Kourkoutas.py:60-131: every param of a layer holds the layer's EMA
        as state['kourkoutas_r_ema']; a tensor found there that is not ours
        (a loaded checkpoint) supplies the EMA's value."""
        state = self.optimizer.state
        for li, ps in enumerate(self.layer_params):
            view = self.views[li]
            ext = state[ps[0]].get("kourkoutas_r_ema")
            if view is None:
                view = self.ema[li]
                self.views[li] = view
            if ext is not None and ext is not view:
                view.copy_(ext.reshape(()).to(device=view.device, dtype=torch.float32))
            for p in ps:
                if state[p].get("kourkoutas_r_ema") is not view:
                    state[p]["kourkoutas_r_ema"] = view

    def loaded(self):
        """A state dict was loaded: adopt its EMAs at the next prepare."""
        self.adopted = False

    def maybe_prepare(self, current_step: int, device, d_dev: int = 0):
        """Kourkoutas.py:202-208: prepare once per step, from the step count
        of the first param stepped.  d_dev: address of Prodigy's device d,
        whose square multiplies 1 - beta2 in the v update's weight."""
        if self.prepared_step < current_step:
            self.prepare(current_step, device, d_dev)
        self.prepared_step = current_step

    @torch.no_grad()
    def prepare(self, current_step: int, device, d_dev: int = 0):
        """Kourkoutas.py:131-200 for every layer, on the device."""
        if not self.n:
            return
        self._alloc(device)
        if not self.adopted:
            self._adopt_states()
            self.adopted = True
        lib = L.lib()
        stream = stream_handle(self.device)
        f32 = lambda x: float(np.float32(x))
        for group, lo, hi in self.ranges:
            b2max = self._hp(group, "betas")[1]
            b2min = self._hp(group, "beta2_min")
            alpha = self._hp(group, "ema_alpha")
            tiny = self._hp(group, "tiny_spike")
            kw = self._hp(group, "k_warmup_steps")
            w = min(1.0, current_step / kw) if kw > 0 else 1.0
            a = L.KourkoutasArgs()
            a.acc = int(self.acc.data_ptr()) + 4 * lo
            a.ema = int(self.ema.data_ptr()) + 4 * lo
            a.layer_beta2 = int(self.beta2.data_ptr()) + 8 * lo
            a.n_layers = hi - lo
            a.beta2_max = f32(b2max)
            a.beta2_min_gap = f32(b2max - b2min)
            a.ema_alpha = f32(alpha)
            a.one_minus_alpha = f32(1.0 - alpha)
            a.tiny_spike = f32(tiny)
            a.w = f32(w)
            a.one_minus_w_bmax = f32((1.0 - w) * b2max)
            a.cv_scale = 1.0
            a.d_dev = int(d_dev)
            L.check(lib.advopt_kourkoutas_prepare(ctypes.byref(a), stream), "advopt_kourkoutas_prepare")
            self.launches += 1

    def layer_table(self, params):
        """int32 [n_tensors]: each param's layer (-1: fixed beta2)."""
        return [self.layer_index(p) for p in params]

    def accumulate(self, plan, stream):
        """Fold one step launch's per-piece sums into the layers' pooled
        squared norms (Kourkoutas.py:231-247)."""
        a = L.KourkoutasArgs()
        a.acc = int(self.acc.data_ptr())
        a.layer_of_tensor = int(plan.layer_dev.data_ptr())
        a.piece_gsq = int(plan.gsq.data_ptr())
        a.pieces = int(plan.pieces_dev.data_ptr())
        a.n_layers = self.n
        a.n_tensors = plan.n
        a.n_pieces = plan.n_pieces
        a.gsq_bf16 = 1 if plan.math_bf16 else 0
        L.check(L.lib().advopt_kourkoutas_accumulate(ctypes.byref(a), stream), "advopt_kourkoutas_accumulate")
        self.launches += 1

    @property
    def last_beta2_stats(self) -> dict:
        """Kourkoutas.py:194-200: the mean of the layers' beta2 of the last
        prepared step (read back on request only)."""
        if self.beta2 is None or not self.n:
            return {}
        return {"mean": float(self.beta2.view(-1, 2)[:, 0].double().mean().item())}

    def dynamic_beta2(self, p) -> float:
        """The beta2 the last prepared step used for p (read back on request)."""
        li = self.layer_index(p)
        if li < 0 or self.beta2 is None:
            return None
        return float(self.beta2[2 * li].item())
