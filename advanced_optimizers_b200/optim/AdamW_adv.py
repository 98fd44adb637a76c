"""AdamW_adv on B200: drop-in for adv_optm.AdamW_adv (AdamW_adv.py:18-482).

Same constructor arguments, defaults, validation, param-group keys, state
keys and dtypes.  `step()` runs one multi-tensor sm_100a launch per group
(plus the factored_2nd finish) instead of ~30 eager ATen passes per tensor.
Options the kernels do not implement raise NotImplementedError at
construction; nothing falls back to a CPU or eager path.
"""
from __future__ import annotations

from typing import Callable, Optional

import torch

from .. import _lib as L
from ._adam_family import AdamCfg, AdamFamilyRunner, SUPPORTED_PRECISIONS, SpectralInit, init_adam_state
from ._common import load_state_dict_exact, reject
from ._kourkoutas import KourkoutasBeta


class AdamW_adv(torch.optim.Optimizer):
    """AdamW with the adv_optm options: int8/bf16 stochastic-rounded states,
    factored second moment, Nesterov, atan2, normed momentum, cautious /
    centered / Fisher weight decay, bf16 stochastic rounding of params."""

    def __init__(
        self,
        params,
        lr: float = 1e-3,
        betas: tuple[float, float] = (0.9, 0.999),
        eps: float | None = 1e-8,
        weight_decay: float = 0.0,
        fisher_wd: bool = False,
        cautious_wd: bool = False,
        use_bias_correction: bool = True,
        stochastic_rounding: bool = True,
        use_atan2: bool = False,
        orthogonal_gradient: str = "disabled",
        nesterov: bool = False,
        nesterov_coef: float | None = None,
        normed_momentum: bool = False,
        kourkoutas_beta: bool = False,
        beta2_min: float = 0.9,
        ema_alpha: float = 0.95,
        tiny_spike: float = 1e-9,
        k_warmup_steps: int = 0,
        k_logging: int = 0,
        layer_key_fn: Optional[Callable] = None,
        spectral_normalization: bool = False,
        centered_wd: float = 0.0,
        centered_wd_mode: str = "float8",
        state_precision: str = "auto",
        factored_2nd: bool = False,
        nnmf_factor: bool = False,
        vector_reshape: bool = False,
        compiled_optimizer: bool = False,
    ):
        # validation order and messages follow AdamW_adv.py:137-151
        if not (lr >= 0.0):
            raise ValueError(f"Learning-rate should be >= 0.0. Got {lr}")
        if not (0.0 <= betas[0] < 1.0 and 0.0 <= betas[1] < 1.0):
            raise ValueError(f"Betas should be in [0.0, 1.0). Got {betas}")
        if not (eps >= 0.0):
            raise ValueError(f"Epsilon should be >= 0.0. Got {eps}")
        if not (weight_decay >= 0.0):
            raise ValueError(f"Weight-decay should be >= 0.0. Got {weight_decay}")
        if kourkoutas_beta and not (betas[1] > beta2_min):
            raise ValueError(f"For Kourkoutas-β, betas[1] (as beta2_max) must be > beta2_min. Got {betas[1]} and {beta2_min}")
        state_precision = state_precision.lower()
        valid_precisions = {"auto", "fp32", "factored", "bf16_sr", "fp16", "int8_sr"}
        if state_precision not in valid_precisions:
            raise ValueError(f"state_precision must be one of {valid_precisions}. Got {state_precision}")
        if nnmf_factor:
            state_precision = "factored"
        reject(orthogonal_gradient != "disabled", "orthogonal_gradient")
        reject(spectral_normalization and fisher_wd, "spectral_normalization with fisher_wd")
        reject(state_precision not in SUPPORTED_PRECISIONS, f"state_precision='{state_precision}'")
        reject(centered_wd and centered_wd_mode not in ("full", "float8", "int8", "int4"),
               f"centered_wd_mode='{centered_wd_mode}'")
        defaults = {
            "lr": lr, "betas": betas, "eps": eps, "weight_decay": weight_decay,
            "fisher_wd": fisher_wd, "cautious_wd": cautious_wd,
            "use_atan2": use_atan2, "nesterov": nesterov, "nesterov_coef": nesterov_coef,
            "normed_momentum": normed_momentum,
            "orthogonal_gradient": orthogonal_gradient, "use_bias_correction": use_bias_correction,
            "compiled_optimizer": compiled_optimizer,
            "kourkoutas_beta": kourkoutas_beta, "beta2_min": beta2_min, "ema_alpha": ema_alpha,
            "tiny_spike": tiny_spike, "k_warmup_steps": k_warmup_steps, "k_logging": k_logging,
            "spectral_normalization": spectral_normalization,
            "centered_wd": centered_wd, "centered_wd_mode": centered_wd_mode,
            "state_precision": state_precision,
            "nnmf_factor": nnmf_factor, "vector_reshape": vector_reshape, "factored_2nd": factored_2nd,
        }
        self.stochastic_rounding = stochastic_rounding
        self.kourkoutas_beta = kourkoutas_beta
        self.layer_key_fn = layer_key_fn
        self._init_lr = lr if lr > 0 else 1
        super().__init__(params, defaults)
        self._runner = AdamFamilyRunner(seed=42)
        self._spectral_init = SpectralInit()
        self._ids = {}
        # Kourkoutas-beta's layer map is built once, before the first step
        # (Kourkoutas.py:25-57)
        self.kourkoutas_helper = KourkoutasBeta(self) if kourkoutas_beta else None
        self.init_step()

    # ---- reference API surface ----
    def load_state_dict(self, state_dict: dict) -> None:
        load_state_dict_exact(self, state_dict)
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
        """The step is already one fused launch per group; kept for API parity."""
        return None

    def init_step(self):
        for group in self.param_groups:
            for p in group["params"]:
                self._init_state(p, group)

    def _tid(self, p):
        t = self._ids.get(id(p))
        if t is None:
            t = len(self._ids)
            self._ids[id(p)] = t
        return t

    @torch.no_grad()
    def _init_state(self, p, group):
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
            self._spectral_init(state, p)       # AdamW_adv.py:272-273

    def _cfg(self, group):
        return AdamCfg(algo=L.ALGO_ADAMW, lr=group["lr"], betas=group["betas"], eps=group["eps"],
                       weight_decay=group["weight_decay"], precision="factored" if group["state_precision"] == "factored" else group["actual_state_precision"],
                       nesterov=group.get("nesterov", False), nesterov_coef=group.get("nesterov_coef"),
                       use_bias_correction=group["use_bias_correction"], use_atan2=group["use_atan2"],
                       normed_momentum=group.get("normed_momentum", False), cautious_wd=group.get("cautious_wd", False),
                       fisher_wd=group.get("fisher_wd", False), centered_wd=group.get("centered_wd", 0.0),
                       centered_wd_mode=group.get("centered_wd_mode", "float8"),
                       stochastic_rounding=self.stochastic_rounding,
                       kourkoutas=self.kourkoutas_helper if group.get("kourkoutas_beta", False) else None,
                       spectral=group.get("spectral_normalization", False))

    def _step_params(self, gi, group, params):
        for p in params:
            self._init_state(p, group)
        if group.get("kourkoutas_beta", False):
            # prepare once per step, before the first param of a Kourkoutas
            # group (AdamW_adv.py:291-295)
            self.kourkoutas_helper.maybe_prepare(self.state[params[0]]["step"], params[0].device)
        by_dtype = {}
        for p in params:
            by_dtype.setdefault((p.dtype, p.device), []).append(p)
        cfg = self._cfg(group)
        for (dt, dev), ps in by_dtype.items():
            key = (gi, dt, dev, tuple(id(p) for p in ps))
            self._runner.run(key, ps, [self.state[p] for p in ps], [self._tid(p) for p in ps], cfg)

    @torch.no_grad()
    def step_parameter(self, p: torch.Tensor, group: dict, i: int | None = None):
        if p.grad is None:
            return
        gi = next(k for k, g in enumerate(self.param_groups) if g is group)
        self._step_params(gi, group, [p])

    @torch.no_grad()
    def step(self, closure=None):
        loss = None
        if closure is not None:
            with torch.enable_grad():
                loss = closure()
        for gi, group in enumerate(self.param_groups):
            params = [p for p in group["params"] if p.grad is not None]
            if params:
                self._step_params(gi, group, params)
        self._runner.test_noise = None
        return loss

    def check_errors(self):
        """Synchronise and raise if a kernel of this optimizer reported a
        bounded wait that gave up (never expected; a guard against hangs)."""
        self._runner.check_errors()

    # ---- test hook: the reference's own random integers ----
    def set_test_noise(self, noise):
        """Use the given int32 noise for the next step only:
        {param: {'exp_avg': t, 'exp_avg_sq': t, 'param': t}} (the reference's
        randint draws, param_update.py:181-264).  None restores Philox."""
        self._runner.test_noise = None if noise is None else {id(p): v for p, v in noise.items()}
