"""Prodigy_adv on B200: drop-in for adv_optm.Prodigy_adv (Prodigy_adv.py:19-576).

The elementwise step and the slice statistics of every parameter run in the
Adam-family kernel (algo PRODIGY); the per-tensor statistics are folded into
the group's d_numerator / d_denom on the device in parameter order, then
`calculate_d` runs on the host in double precision exactly as the reference
does.  With `fsdp_in_use` (or a flattened FSDP parameter) and an initialised
process group, the two sums are all-reduced over torch.distributed (NCCL on
GPUs) before `calculate_d` (Prodigy_adv.py:550-554).
"""
from __future__ import annotations

import math
from typing import Callable, Optional

import numpy as np
import torch
import torch.distributed as dist

from .. import _lib as L
from ._adam_family import AdamCfg, AdamFamilyRunner, SUPPORTED_PRECISIONS, init_adam_state
from ._common import load_state_dict_exact, reject


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
        reject(kourkoutas_beta, "kourkoutas_beta")
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
        self._first = True
        self._carry_scale = 1.0      # 0 on the ranks of a sharded run that do not carry the numerator
        self._process_group = None   # group of the d all-reduce (default group when None)
        self.init_step()

    def load_state_dict(self, state_dict: dict) -> None:
        load_state_dict_exact(self, state_dict)
        self._runner.invalidate()

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
        """Prodigy_adv.py:246-257: beta3 and the accumulators of the next step."""
        g = self.param_groups[0]
        self.beta1, self.beta2_default = g["betas"]
        self.beta3 = g["beta3"]
        if self.beta3 is None:
            self.beta3 = math.sqrt(self.beta2_default)
        if not self._first:
            self._d_num_carry = float(np.float32(g.get("d_numerator", 0.0) * self.beta3)) * self._carry_scale

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
        group["actual_state_precision"] = req
        init_adam_state(p, state, precision=req, factored_2nd=group.get("factored_2nd", False),
                        beta1=group["betas"][0], vector_reshape=group["vector_reshape"],
                        centered_wd=group.get("centered_wd", 0.0),
                        centered_wd_mode=group.get("centered_wd_mode", "float8"),
                        fisher_wd=group.get("fisher_wd", False))
        sp = group["slice_p"]
        state["s"] = torch.zeros_like(p.flatten()[::sp]).detach().contiguous()
        if p.any():
            state["p0"] = p.flatten()[::sp].detach().clone().contiguous()
        else:
            state["p0"] = torch.tensor(0, device=p.device, dtype=p.dtype)

    def _cfg(self, group, stats):
        pd = dict(d=group["d"], d0=group["d0"], beta3=self.beta3, safeguard_warmup=group["safeguard_warmup"],
                  slice_p=group["slice_p"], stats=stats)
        return AdamCfg(algo=L.ALGO_PRODIGY, lr=group["lr"], betas=group["betas"], eps=group["eps"],
                       weight_decay=group["weight_decay"], precision=group["actual_state_precision"],
                       nesterov=group.get("nesterov", False), nesterov_coef=group.get("nesterov_coef"),
                       use_atan2=group["use_atan2"], cautious_wd=group.get("cautious_wd", False),
                       fisher_wd=group.get("fisher_wd", False), centered_wd=group.get("centered_wd", 0.0),
                       centered_wd_mode=group.get("centered_wd_mode", "float8"),
                       stochastic_rounding=self.stochastic_rounding, prodigy=pd)

    def _ensure_sums(self):
        if not hasattr(self, "_sums"):
            self._sums = torch.zeros(2, dtype=torch.float32, device=self.device)
            self._d_num_carry = float(np.float32(self.param_groups[0].get("d_numerator", 0.0))) * self._carry_scale
            self._first = False

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
        by_dtype = {}
        for p in params:
            by_dtype.setdefault((p.dtype, p.device), []).append(p)
        cfg = self._cfg(group, stats)
        for (dt, dev), ps in by_dtype.items():
            key = (gi, dt, dev, tuple(id(p) for p in ps), stats)
            self._runner.run(key, ps, [self.state[p] for p in ps], [self._tid(p) for p in ps], cfg,
                             prodigy_sums=self._sums)

    @torch.no_grad()
    def step_parameter(self, p: torch.Tensor, group: dict, i: int | None = None):
        if p.grad is None:
            return
        self._ensure_sums()
        gi = next(k for k, g in enumerate(self.param_groups) if g is group)
        self._step_params(gi, group, [p])

    @torch.no_grad()
    def step(self, closure=None):
        loss = None
        if closure is not None:
            with torch.enable_grad():
                loss = closure()
        self._ensure_sums()
        self._sums[0] = self._d_num_carry
        self._sums[1] = 0.0
        for gi, group in enumerate(self.param_groups):
            params = [p for p in group["params"] if p.grad is not None]
            if params:
                self._step_params(gi, group, params)
        self._runner.test_noise = None
        self.calculate_d()
        self.init_step()
        return loss

    def calculate_d(self):
        """Prodigy_adv.py:540-576 on the host, from the device sums."""
        g_group = self.param_groups[0]
        active = not (g_group.get("prodigy_steps", 0) > 0 and g_group["k"] >= g_group["prodigy_steps"])
        if active:
            d_max, d_coef, growth_rate = g_group["d_max"], g_group["d_coef"], g_group["growth_rate"]
            if self.fsdp_in_use and dist.is_available() and dist.is_initialized():
                dist.all_reduce(self._sums, op=dist.ReduceOp.SUM, group=self._process_group)
            gn, gd = self._sums.tolist()
            d_hat = g_group["d"]
            if gd > 0:
                d_hat = d_coef * gn / gd
                if g_group.get("d_limiter", False):
                    d_hat = min(g_group["d"] * (2 ** 0.25), d_hat)
                if g_group["d"] == g_group["d0"]:
                    g_group["d"] = max(g_group["d"], d_hat)
                d_max = max(d_max, d_hat)
                g_group["d"] = min(d_max, g_group["d"] * growth_rate)
            for group in self.param_groups:
                group["d_numerator"] = gn
                group["d"] = g_group["d"]
                group["d_max"] = d_max
        for group in self.param_groups:
            group["k"] += 1

    def check_errors(self):
        self._runner.check_errors()

    def set_test_noise(self, noise):
        """Use the reference's random integers for the next step (see AdamW_adv.set_test_noise)."""
        self._runner.test_noise = None if noise is None else {id(p): v for p, v in noise.items()}
