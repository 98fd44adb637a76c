"""Prodigy_adv on B200: drop-in for adv_optm.Prodigy_adv (Prodigy_adv.py:19-576).

The elementwise step and the slice statistics of every parameter run in the
Adam-family kernel (algo PRODIGY); the per-tensor statistics are folded into
the group's d_numerator / d_denom on the device in parameter order.  d itself
lives on the device (advopt_prodigy_dev): the step's scalars are derived from
it there and `calculate_d` runs there in double precision with the
reference's arithmetic, so a step never waits for the GPU.  The param groups'
'd', 'd_max' and 'd_numerator' are filled in when read (that read waits for
the step that produced them, like the reference's `.item()`), and values
written to them are uploaded before the next step.  With `fsdp_in_use` (or a
flattened FSDP parameter) and an initialised process group, the two sums are
all-reduced over torch.distributed (NCCL on GPUs) before `calculate_d`
(Prodigy_adv.py:550-554).
"""
from __future__ import annotations

import ctypes
import math
from typing import Callable, Optional

import numpy as np
import torch
import torch.distributed as dist

from .. import _lib as L
from .._device import stream_handle
from ._adam_family import AdamCfg, AdamFamilyRunner, SUPPORTED_PRECISIONS, SpectralInit, init_adam_state
from ._common import load_state_dict_exact, reject
from ._kourkoutas import KourkoutasBeta


class _DeviceDGroup(dict):
    """A Prodigy param group whose d, d_max and d_numerator are kept on the
    device.  Reading one waits for the step that produced it; writing one
    (or d0) is uploaded before the next step.  Copies and pickles are plain
    dicts with the current values."""

    LAZY = ("d", "d_max", "d_numerator")
    WATCH = ("d", "d0", "d_max", "d_numerator")

    def __init__(self, group, owner):
        super().__init__(group)
        self._owner = owner

    def _pull(self):
        o = getattr(self, "_owner", None)
        if o is not None:
            o._pull_d()

    def __getitem__(self, key):
        if key in self.LAZY:
            self._pull()
        return dict.__getitem__(self, key)

    def get(self, key, default=None):
        if key in self.LAZY:
            self._pull()
        return dict.get(self, key, default)

    def items(self):
        self._pull()
        return dict.items(self)

    def values(self):
        self._pull()
        return dict.values(self)

    def copy(self):
        self._pull()
        return dict(dict.items(self))

    def __repr__(self):
        self._pull()
        return dict.__repr__(self)

    def __setitem__(self, key, value):
        if key in self.WATCH:
            self._pull()
            o = getattr(self, "_owner", None)
            if o is not None:
                o._d_dirty = True
        dict.__setitem__(self, key, value)

    def raw(self, key):
        """The host copy without waiting (internal)."""
        return dict.__getitem__(self, key)

    def __reduce__(self):
        return (dict, (self.copy(),))


class Prodigy_adv(torch.optim.Optimizer):
    """Prodigy (learning-rate-free Adam) with the adv_optm options."""

    def __init__(
        self,
        params,
        lr: float = 1,
        betas: tuple[float, float] = (0.9, 0.999),
        eps: float | None = 1e-8,
        weight_decay: float = 0.0,
        fisher_wd: bool = False,
        cautious_wd: bool = False,
        stochastic_rounding: bool = True,
        use_atan2: bool = False,
        orthogonal_gradient: str = "disabled",
        nesterov: bool = False,
        nesterov_coef: float | None = None,
        state_precision: str = "auto",
        factored_2nd: bool = False,
        nnmf_factor: bool = False,
        vector_reshape: bool = False,
        compiled_optimizer: bool = False,
        beta3: float = None,
        d0: float = 1e-6,
        d_coef: float = 1,
        growth_rate: float = float("inf"),
        safeguard_warmup: bool = False,
        fsdp_in_use: bool = False,
        slice_p: int = 11,
        prodigy_steps: int = 0,
        d_limiter: bool = False,
        kourkoutas_beta: bool = False,
        beta2_min: float = 0.9,
        ema_alpha: float = 0.95,
        tiny_spike: float = 1e-9,
        k_warmup_steps: int = 0,
        k_logging: int = 0,
        layer_key_fn: Optional[Callable] = None,
        centered_wd: float = 0.0,
        centered_wd_mode: str = "float8",
    ):
        # Prodigy_adv.py:158-178
        if not (lr >= 0.0):
            raise ValueError(f"Learning-rate should be >= 0.0. Got {lr}")
        if not (0.0 <= betas[0] < 1.0 and 0.0 <= betas[1] < 1.0):
            raise ValueError(f"Betas should be in [0.0, 1.0). Got {betas}")
        if not (eps >= 0.0):
            raise ValueError(f"Epsilon should be >= 0.0. Got {eps}")
        if not (weight_decay >= 0.0):
            raise ValueError(f"Weight-decay should be >= 0.0. Got {weight_decay}")
        if not (prodigy_steps >= 0):
            raise ValueError(f"prodigy_steps should be >= 0. Got {prodigy_steps}")
        if kourkoutas_beta and not (betas[1] > beta2_min):
            raise ValueError(f"For Kourkoutas-β, betas[1] (as beta2_max) must be > beta2_min. Got {betas[1]} and {beta2_min}")
        state_precision = state_precision.lower()
        valid_precisions = {"auto", "fp32", "factored", "bf16_sr", "fp16", "int8_sr"}
        if state_precision not in valid_precisions:
            raise ValueError(f"state_precision must be one of {valid_precisions}. Got {state_precision}")
        if nnmf_factor:
            state_precision = "factored"
        reject(orthogonal_gradient != "disabled", "orthogonal_gradient")
        reject(state_precision not in SUPPORTED_PRECISIONS, f"state_precision='{state_precision}'")
        defaults = {
            "lr": lr, "betas": betas, "eps": eps, "weight_decay": weight_decay,
            "fisher_wd": fisher_wd, "cautious_wd": cautious_wd,
            "use_atan2": use_atan2,
            "orthogonal_gradient": orthogonal_gradient,
            "compiled_optimizer": compiled_optimizer,
            "beta3": beta3, "d": d0, "d0": d0, "d_max": d0, "d_numerator": 0.0, "d_coef": d_coef,
            "growth_rate": growth_rate, "safeguard_warmup": safeguard_warmup, "k": 0, "slice_p": slice_p,
            "fsdp_in_use": fsdp_in_use, "prodigy_steps": prodigy_steps, "d_limiter": d_limiter,
            "nesterov": nesterov, "nesterov_coef": nesterov_coef, "state_precision": state_precision,
            "kourkoutas_beta": kourkoutas_beta, "beta2_min": beta2_min, "ema_alpha": ema_alpha,
            "tiny_spike": tiny_spike, "k_warmup_steps": k_warmup_steps, "k_logging": k_logging,
            "centered_wd": centered_wd, "centered_wd_mode": centered_wd_mode,
            "nnmf_factor": nnmf_factor, "vector_reshape": vector_reshape, "factored_2nd": factored_2nd,
        }
        self.stochastic_rounding = stochastic_rounding
        self.fsdp_in_use = fsdp_in_use
        self.kourkoutas_beta = kourkoutas_beta
        self.layer_key_fn = layer_key_fn
        super().__init__(params, defaults)
        self.device = self.param_groups[0]["params"][0].device
        self._runner = AdamFamilyRunner(seed=42)
        self._ids = {}
        self._carry_scale = 1.0      # 0 on the ranks of a sharded run that do not carry the numerator
        self._process_group = None   # group of the d all-reduce (default group when None)
        # d on the device: advopt_prodigy_dev (4 doubles, 2 sums, 5 launch scalars)
        self._dblock = torch.zeros(L.PRODIGY_DEV_BYTES // 8, dtype=torch.float64, device=self.device)
        self._dsums = self._dblock.view(torch.float32)[L.PRODIGY_DEV_SUMS // 4:L.PRODIGY_DEV_SUMS // 4 + 2]
        self._dhost = torch.zeros(4, dtype=torch.float64, pin_memory=True)
        self._d_pending = None       # event of the last d read-back not yet folded into the groups
        self._d_dirty = True         # host group values to upload before the next step
        self._sums_ready = False
        self._wrap_groups()
        self.kourkoutas_helper = KourkoutasBeta(self) if kourkoutas_beta else None
        self.init_step()

    def _wrap_groups(self):
        self.param_groups = [g if isinstance(g, _DeviceDGroup) else _DeviceDGroup(g, self)
                             for g in self.param_groups]
        self._d_dirty = True

    def add_param_group(self, param_group: dict) -> None:
        super().add_param_group(param_group)
        if hasattr(self, "_dblock"):
            self._wrap_groups()

    def load_state_dict(self, state_dict: dict) -> None:
        self._pull_d()
        load_state_dict_exact(self, state_dict)
        self._wrap_groups()
        self._runner.invalidate()
        if self.kourkoutas_helper is not None:
            self.kourkoutas_helper.loaded()

    @property
    def supports_fused_back_pass(self):
        return True

    @property
    def supports_memory_efficient_fp16(self):
        return True

    @property
    def supports_flat_params(self):
        return False

    def compile(self, *args, **kwargs):
        return None

    def init_step(self):
        """Prodigy_adv.py:246-257: beta1, beta2 and beta3 of the next step.
        The accumulators' reset (d_numerator * beta3, 0) is made on the
        device by calculate_d."""
        g = self.param_groups[0]
        self.beta1, self.beta2_default = g["betas"]
        self.beta3 = g["beta3"]
        if self.beta3 is None:
            self.beta3 = math.sqrt(self.beta2_default)

    # ---- d on the device ----
    def _pull_d(self):
        """Fold the last read-back of d, d_max and d_numerator into the
        groups (waits for the step that produced them)."""
        ev = self._d_pending
        if ev is None:
            return
        ev.synchronize()
        self._d_pending = None
        d, _, d_max, d_num = self._dhost.tolist()
        for g in self.param_groups:
            for key, v in (("d", d), ("d_max", d_max), ("d_numerator", d_num)):
                dict.__setitem__(g, key, v)

    def _push_d(self):
        """Upload the groups' d, d0, d_max and d_numerator (first step, and
        after they were written); the first upload also starts the sums, from
        d_numerator without beta3 as the reference's first step does
        (Prodigy_adv.py:333-335)."""
        if not self._d_dirty:
            return
        g0 = self.param_groups[0]
        vals = [g0.raw("d"), g0.raw("d0"), g0.raw("d_max"), g0.raw("d_numerator")]
        for g in self.param_groups[1:]:
            if g.raw("d") != vals[0] or g.raw("d0") != vals[1]:
                raise NotImplementedError("Prodigy_adv on B200 keeps one d for all param groups; "
                                          "the groups hold different d or d0")
        self._dblock[:4].copy_(torch.tensor(vals, dtype=torch.float64))
        if not self._sums_ready:
            self._dsums[0] = float(np.float32(vals[3])) * self._carry_scale
            self._dsums[1] = 0.0
            self._sums_ready = True
        self._d_dirty = False

    def _set_carry(self, value: float):
        """Set the next step's carried d_numerator (its first sum) directly."""
        self._push_d()
        self._dsums[0] = float(value)

    def _tid(self, p):
        t = self._ids.get(id(p))
        if t is None:
            t = len(self._ids)
            self._ids[id(p)] = t
        return t

    @torch.no_grad()
    def _init_state(self, p, group):
        """Prodigy_adv.py:271-331."""
        state = self.state[p]
        if "step" in state:
            return
        req = group["state_precision"]
        group["actual_state_precision"] = "auto" if req == "factored" else req
        init_adam_state(p, state, precision=req, factored_2nd=group.get("factored_2nd", False),
                        beta1=group["betas"][0], vector_reshape=group["vector_reshape"],
                        centered_wd=group.get("centered_wd", 0.0),
                        centered_wd_mode=group.get("centered_wd_mode", "float8"),
                        fisher_wd=group.get("fisher_wd", False))
        if group.get("spectral_normalization", False):
            # a param-group key only: the constructor takes no such argument
            # (Prodigy_adv.py:319-320, 490-493)
            if not hasattr(self, "_spectral_init"):
                self._spectral_init = SpectralInit()
            self._spectral_init(state, p)
        sp = group["slice_p"]
        state["s"] = torch.zeros_like(p.flatten()[::sp]).detach().contiguous()
        if p.any():
            state["p0"] = p.flatten()[::sp].detach().clone().contiguous()
        else:
            state["p0"] = torch.tensor(0, device=p.device, dtype=p.dtype)

    def _cfg(self, group, stats):
        pd = dict(d=group.raw("d"), d0=group.raw("d0"), beta3=self.beta3, safeguard_warmup=group["safeguard_warmup"],
                  slice_p=group["slice_p"], stats=stats, dev=self._dblock)
        return AdamCfg(algo=L.ALGO_PRODIGY, lr=group["lr"], betas=group["betas"], eps=group["eps"],
                       weight_decay=group["weight_decay"], precision="factored" if group["state_precision"] == "factored" else group["actual_state_precision"],
                       nesterov=group.get("nesterov", False), nesterov_coef=group.get("nesterov_coef"),
                       use_atan2=group["use_atan2"], cautious_wd=group.get("cautious_wd", False),
                       fisher_wd=group.get("fisher_wd", False), centered_wd=group.get("centered_wd", 0.0),
                       centered_wd_mode=group.get("centered_wd_mode", "float8"),
                       stochastic_rounding=self.stochastic_rounding, prodigy=pd,
                       kourkoutas=self.kourkoutas_helper if group.get("kourkoutas_beta", False) else None,
                       spectral=group.get("spectral_normalization", False))

    def _step_params(self, gi, group, params):
        for p in params:
            if hasattr(p, "_fsdp_flattened"):
                self.fsdp_in_use = True
            self._init_state(p, group)
        stats = group["prodigy_steps"] <= 0 or group["k"] < group["prodigy_steps"]
        if not stats:
            for p in params:
                self.state[p].pop("s", None)
                self.state[p].pop("p0", None)
        if group.get("kourkoutas_beta", False):
            # once per step, before the first param of a Kourkoutas group
            # (Prodigy_adv.py:337-342); v's weight is d * d * (1 - beta2)
            self.kourkoutas_helper.maybe_prepare(self.state[params[0]]["step"], params[0].device,
                                                 d_dev=int(self._dblock.data_ptr()))
        by_dtype = {}
        for p in params:
            by_dtype.setdefault((p.dtype, p.device), []).append(p)
        cfg = self._cfg(group, stats)
        for (dt, dev), ps in by_dtype.items():
            key = (gi, dt, dev, tuple(id(p) for p in ps), stats)
            self._runner.run(key, ps, [self.state[p] for p in ps], [self._tid(p) for p in ps], cfg,
                             prodigy_sums=self._dsums)

    @torch.no_grad()
    def step_parameter(self, p: torch.Tensor, group: dict, i: int | None = None):
        if p.grad is None:
            return
        self._push_d()
        gi = next(k for k, g in enumerate(self.param_groups) if g is group)
        self._step_params(gi, group, [p])

    @torch.no_grad()
    def step(self, closure=None):
        loss = None
        if closure is not None:
            with torch.enable_grad():
                loss = closure()
        self._push_d()
        for gi, group in enumerate(self.param_groups):
            params = [p for p in group["params"] if p.grad is not None]
            if params:
                self._step_params(gi, group, params)
        self._runner.test_noise = None
        self.calculate_d()
        self.init_step()
        return loss

    def calculate_d(self):
        """Prodigy_adv.py:540-576 on the device (advopt_prodigy_update_d),
        followed by the reset of the sums that init_step makes in the
        reference (d_numerator * beta3 carried, d_denom 0).  Nothing is read
        back here: the groups' d, d_max and d_numerator are filled in when
        read."""
        self._push_d()
        g_group = self.param_groups[0]
        active = not (g_group.get("prodigy_steps", 0) > 0 and g_group["k"] >= g_group["prodigy_steps"])
        if active and self.fsdp_in_use and dist.is_available() and dist.is_initialized():
            dist.all_reduce(self._dsums, op=dist.ReduceOp.SUM, group=self._process_group)
        # init_step's beta3 for the carry (Prodigy_adv.py:249-256)
        beta3 = g_group["beta3"]
        if beta3 is None:
            beta3 = math.sqrt(g_group["betas"][1])
        a = L.ProdigyDArgs()
        a.dev = int(self._dblock.data_ptr())
        a.active = 1 if active else 0
        a.d_limiter = 1 if g_group.get("d_limiter", False) else 0
        a.d_coef = float(g_group["d_coef"])
        a.growth_rate = float(g_group["growth_rate"])
        a.limiter_factor = 2 ** 0.25
        a.beta3 = float(beta3)
        a.carry_scale = float(self._carry_scale)
        L.check(L.lib().advopt_prodigy_update_d(ctypes.byref(a), stream_handle(self.device)),
                "advopt_prodigy_update_d")
        self._runner.launch_count += 1
        # read-back for the groups, folded in when one of them is read
        self._dhost.copy_(self._dblock[:4], non_blocking=True)
        ev = torch.cuda.Event()
        ev.record(torch.cuda.current_stream(self.device))
        self._d_pending = ev
        for group in self.param_groups:
            dict.__setitem__(group, "k", group["k"] + 1)

    def check_errors(self):
        self._runner.check_errors()

    def set_test_noise(self, noise):
        """Use the reference's random integers for the next step (see AdamW_adv.set_test_noise)."""
        self._runner.test_noise = None if noise is None else {id(p): v for p, v in noise.items()}
