"""Lion_adv on B200: drop-in for adv_optm.Lion_adv (Lion_adv.py:17-296).

One elementwise launch per group (csrc/lion.cu): update = sign(lerp(g, m,
beta1)) * lr, m = lerp(m, g, 1 - beta2), then the reference's weight decay
and bf16 stochastic rounding.  Under nnmf_factor the 2-D params keep m as
signed rank-1 factors (Lion_adv.py:161-176, 232-254) and step in the
Adam-family general kernel (ADVOPT_ALGO_LION, float32).  kappa_p = 1 (sign)
only; the other Lion-K geometries need a global norm and are rejected, as are
the options listed in reject() calls below.
"""
from __future__ import annotations

import ctypes
from typing import Optional, Tuple

import numpy as np
import torch

from .. import _lib as L
from .._device import DeviceTable, aligned16, dtype_code, ptr, require_cuda_tensor, stream_handle, upload_static
from .._plan import plan as plan_pieces
from .._plan import effective_shape
from ._adam_family import SHIFTER, AdamCfg, AdamFamilyRunner, SpectralInit, adjust_wds, f32, sign_storage
from ._common import load_state_dict_exact, reject


class _LionPlan:
    def __init__(self, params, states, ids):
        self.params = list(params)
        self.device = params[0].device
        self.pdt = dtype_code(params[0].dtype)
        n = len(params)
        self.descs = np.zeros(n, L.LION_TENSOR_DT)
        d = self.descs
        self.vec_ok = []
        for i, (p, st) in enumerate(zip(params, states)):
            d["param"][i] = ptr(p)
            d["exp_avg"][i] = ptr(st["exp_avg"])
            d["numel"][i] = p.numel()
            d["tensor_id"][i] = ids[i]
            self.vec_ok.append(aligned16(p, st["exp_avg"]))
        numels = [p.numel() for p in params]
        dev = self.device.index if self.device.index is not None else torch.cuda.current_device()
        sms = torch.cuda.get_device_properties(dev).multi_processor_count
        pieces, offsets, _ = plan_pieces(numels, [0] * n, sms * 8)
        self.n_pieces = len(pieces)
        self.pieces_dev = upload_static(pieces, self.device)
        self.table = DeviceTable(self.descs.nbytes, self.device)


class Lion_adv(torch.optim.Optimizer):
    """Lion with the adv_optm options (cautious weight decay, bf16 stochastic rounding)."""

    def __init__(
        self,
        params,
        lr: float = 1e-4,
        betas: Tuple[float, float] = (0.9, 0.99),
        weight_decay: float = 0.0,
        cautious_wd: bool = False,
        stochastic_rounding: bool = True,
        orthogonal_gradient: str = "disabled",
        kappa_p: float = 1.0,
        auto_kappa_p: bool = False,
        stochastic_sign: bool = False,
        centered_wd: float = 0.0,
        centered_wd_mode: str = "float8",
        spectral_normalization: bool = False,
        nnmf_factor: bool = False,
        vector_reshape: bool = False,
        compiled_optimizer: bool = False,
    ):
        # Lion_adv.py:88-93
        if not lr > 0.0:
            raise ValueError(f"Learning rate must be > 0.0, but got {lr}")
        if not all(0.0 <= beta <= 1.0 for beta in betas):
            raise ValueError(f"Betas should be in [0.0, 1.0], but got {betas}")
        if not weight_decay >= 0.0:
            raise ValueError(f"Weight decay must be >= 0.0, but got {weight_decay}")
        reject(orthogonal_gradient != "disabled", "orthogonal_gradient")
        reject(stochastic_sign, "stochastic_sign")
        reject(centered_wd, "centered_wd for Lion_adv")
        reject(kappa_p != 1.0 and not auto_kappa_p, f"kappa_p={kappa_p}")
        defaults = dict(lr=lr, betas=betas, weight_decay=weight_decay, cautious_wd=cautious_wd,
                        vector_reshape=vector_reshape, orthogonal_gradient=orthogonal_gradient, kappa_p=kappa_p,
                        auto_kappa_p=auto_kappa_p, stochastic_sign=stochastic_sign,
                        spectral_normalization=spectral_normalization, nnmf_factor=nnmf_factor,
                        centered_wd=centered_wd, centered_wd_mode=centered_wd_mode)
        self.stochastic_rounding = stochastic_rounding
        self._init_lr = lr if lr > 0 else 1
        super().__init__(params, defaults)
        self._plans = {}
        self._ids = {}
        self._test_noise = None
        self.seed = 42
        self._fruner = AdamFamilyRunner(seed=42)     # factored / spectral-normalised tensors
        self._spectral_init = SpectralInit()
        self.init_step()

    def load_state_dict(self, state_dict: dict) -> None:
        load_state_dict_exact(self, state_dict)
        self._plans.clear()
        self._fruner.invalidate()

    @property
    def supports_fused_back_pass(self) -> bool:
        return True

    @property
    def supports_memory_efficient_fp16(self) -> bool:
        return True

    @property
    def supports_flat_params(self) -> bool:
        return False

    def compile(self, *args, **kwargs):
        return None

    def init_step(self):
        for group in self.param_groups:
            for p in group["params"]:
                self._init_state(p, group)

    @torch.no_grad()
    def _init_state(self, p, group):
        """Lion_adv.py:156-181: signed rank-1 m (float32 factors, 1-bit signs)
        for params of two or more dims under nnmf_factor, else m in the
        param dtype."""
        state = self.state[p]
        if "step" not in state:
            state["step"] = 0
            state["factored"] = bool(group["nnmf_factor"] and
                                     not (p.dim() == 1 and not group["vector_reshape"]))
            if state["factored"]:
                d1, d2 = effective_shape(p.numel())
                state["effective_shape"] = (d1, d2)
                state["mu_m_nmf"] = torch.zeros(d1, device=p.device, dtype=torch.float32)
                state["mv_m_nmf"] = torch.zeros(d2, device=p.device, dtype=torch.float32)
                state["sign"] = sign_storage(d1, (d2 + 7) // 8, p.device)
                state["shifter"] = torch.tensor(SHIFTER, device=p.device, dtype=torch.uint8)
            else:
                state["exp_avg"] = torch.zeros_like(p, device=p.device, dtype=p.dtype)
            if group.get("spectral_normalization", False):
                self._spectral_init(state, p)             # Lion_adv.py:179-180

    def _tid(self, p):
        t = self._ids.get(id(p))
        if t is None:
            t = len(self._ids)
            self._ids[id(p)] = t
        return t

    def _run(self, gi, group, params):
        for p in params:
            self._init_state(p, group)
            require_cuda_tensor(p, "param")
            require_cuda_tensor(p.grad, "grad")
        # factored tensors, and every tensor of a spectral-normalised group,
        # step in the Adam-family general kernel (ADVOPT_ALGO_LION)
        spectral = group.get("spectral_normalization", False)
        fac = [p for p in params if self.state[p]["factored"] or spectral]
        if fac:
            self._run_general(gi, group, fac)
        params = [p for p in params if not (self.state[p]["factored"] or spectral)]
        by_dtype = {}
        for p in params:
            if group.get("auto_kappa_p", False) and p.ndim >= 4:
                raise NotImplementedError("Lion-K with kappa_p=2 (4-D params under auto_kappa_p) is not supported")
            by_dtype.setdefault((p.dtype, p.device), []).append(p)
        beta1, beta2 = group["betas"]
        for (dt, dev), ps in by_dtype.items():
            key = (gi, dt, dev, tuple(id(p) for p in ps))
            pl = self._plans.get(key)
            if pl is None or any(pl.descs["param"][i] != ptr(p) for i, p in enumerate(ps)):
                pl = _LionPlan(ps, [self.state[p] for p in ps], [self._tid(p) for p in ps])
                self._plans[key] = pl
            d = pl.descs
            keep = []
            for i, p in enumerate(ps):
                st = self.state[p]
                st["step"] += 1                       # Lion increments before its math (Lion_adv.py:192)
                gp = p.grad.data_ptr()
                d["grad"][i] = gp
                d["flags"][i] = L.T_VEC if (pl.vec_ok[i] and gp % 16 == 0) else 0
                wd, _ = adjust_wds(group["weight_decay"], 0.0, p)
                d["lr"][i] = group["lr"]
                d["wd"][i] = wd * group["lr"] if wd != 0 else 0.0
                d["step"][i] = st["step"] & 0xFFFFFFFF
                nz = None if self._test_noise is None else self._test_noise.get(id(p), {}).get("param")
                if nz is not None:
                    nz = nz.to(device=p.device, dtype=torch.int32).contiguous()
                    if nz.numel() < p.numel():
                        raise ValueError("injected noise 'param' is shorter than the parameter")
                    keep.append(nz)
                d["noise_p"][i] = ptr(nz)
            flags = 0
            if self.stochastic_rounding and pl.pdt == L.DT_BF16:
                flags |= L.F_SR
            if group.get("cautious_wd", False):
                flags |= L.F_CAUTIOUS
            if self._test_noise is not None:
                flags |= L.F_NOISE_IN
                if flags & L.F_SR and any(d["noise_p"][i] == 0 for i in range(len(ps))):
                    raise ValueError("injected noise 'param' missing")
            pl.table.upload(d)
            L.check(L.lib().advopt_lion_step(pl.table.ptr, len(ps), int(pl.pieces_dev.data_ptr()), pl.n_pieces,
                                             pl.pdt, f32(beta1), f32(1 - beta2), flags, self.seed,
                                             stream_handle(pl.device)), "advopt_lion_step")
            if keep:
                torch.cuda.current_stream(pl.device).synchronize()

    def _run_general(self, gi, group, params):
        """Params stepped by the general kernel: one launch per (dtype,
        factored) — float32 for factored m, the param dtype otherwise
        (Lion_adv.py:214-278) — with the spectral scaling when the group
        asks for it."""
        by_kind = {}
        for p in params:
            if group.get("auto_kappa_p", False) and p.ndim >= 4:
                raise NotImplementedError("Lion-K with kappa_p=2 (4-D params under auto_kappa_p) is not supported")
            by_kind.setdefault((p.dtype, p.device, bool(self.state[p]["factored"])), []).append(p)
        if self._test_noise is not None:
            self._fruner.test_noise = {id(p): {"param": self._test_noise[id(p)]["param"]}
                                       for p in params if "param" in self._test_noise.get(id(p), {})}
        for (dt, dev, fac), ps in by_kind.items():
            cfg = AdamCfg(algo=L.ALGO_LION, lr=group["lr"], betas=group["betas"], eps=1.0,
                          weight_decay=group["weight_decay"], precision="factored" if fac else "auto",
                          use_bias_correction=False, cautious_wd=group.get("cautious_wd", False),
                          stochastic_rounding=self.stochastic_rounding,
                          spectral=group.get("spectral_normalization", False))
            key = (gi, dt, dev, fac, tuple(id(p) for p in ps))
            self._fruner.run(key, ps, [self.state[p] for p in ps], [self._tid(p) for p in ps], cfg)
        self._fruner.test_noise = None

    def check_errors(self):
        """Synchronise and raise if a factored step's kernel reported a bounded wait that gave up."""
        self._fruner.check_errors()

    @torch.no_grad()
    def step_parameter(self, p: torch.Tensor, group: dict, i: Optional[int] = None):
        if p.grad is None:
            return
        gi = next(k for k, g in enumerate(self.param_groups) if g is group)
        self._run(gi, group, [p])

    @torch.no_grad()
    def step(self, closure: Optional[callable] = None):
        loss = None
        if closure is not None:
            with torch.enable_grad():
                loss = closure()
        for gi, group in enumerate(self.param_groups):
            params = [p for p in group["params"] if p.grad is not None]
            if params:
                self._run(gi, group, params)
        self._test_noise = None
        return loss

    def set_test_noise(self, noise):
        """Use the reference's random integers for the next step: {param: {'param': t}}."""
        self._test_noise = None if noise is None else {id(p): v for p, v in noise.items()}
