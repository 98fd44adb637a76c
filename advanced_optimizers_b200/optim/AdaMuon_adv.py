"""AdaMuon_adv on B200: drop-in for adv_optm.AdaMuon_adv (AdaMuon_adv.py:17-673).

'muon' parameters: momentum, the Lion-K projection (sign for kappa_p = 1;
identity for kappa_p = 2, which the normalisation inside Newton–Schulz
absorbs), Newton–Schulz / CANS on the tcgen05 GEMM chain, then the second
moment v = beta2 v + (1-beta2) u^2 (f32 / bf16 / uint8 blocks), u / (sqrt(v)
+ eps) (or atan2), RMS rescale and the parameter update, all in
csrc/muon.cu.  'adam' parameters take the auxiliary AdamW step.
"""
from __future__ import annotations

from ._common import reject
from ._muon_base import MuonFamilyBase
from .Muon_adv import VALID_PRECISIONS


class AdaMuon_adv(MuonFamilyBase):
    """AdaMuon: Muon with a per-element second moment on the orthogonalised update."""

    _adamuon = True

    def __init__(
        self,
        params,
        lr: float = 1e-3,
        betas: tuple[float, float] = (0.95, 0.95),
        eps: float = 1e-8,
        weight_decay: float = 0,
        cautious_wd: bool = False,
        nesterov: bool = True,
        nesterov_coef: float | None = None,
        rms_rescaling: bool = True,
        ns_steps: int = 5,
        ns_eps: float | None = 1e-7,
        ns_coeffs: tuple[float, float, float] = (3.4445, -4.7750, 2.0315),
        stochastic_rounding: bool = True,
        orthogonal_gradient: str = "disabled",
        use_atan2: bool = False,
        normuon_variant: bool = False,
        use_muon: bool | None = None,
        state_precision: str = "auto",
        factored_2nd: bool = False,
        kappa_p: float = 1.0,
        auto_projection: bool = True,
        low_rank_ortho: bool = False,
        ortho_rank: int = 128,
        vector_reshape: bool = False,
        nnmf_factor: bool = False,
        accelerated_ns: bool = False,
        cns_a_bound: float | None = None,
        approx_mars: bool = False,
        mars_gamma: float = 0.025,
        n_layers: int = 1,
        spectral_normalization: bool = False,
        centered_wd: float = 0.0,
        centered_wd_mode: str = "float8",
        compiled_optimizer: bool = False,
        adam_betas: tuple[float, float] = (0.9, 0.99),
        adam_eps: float | None = 1e-8,
        adam_weight_decay: float = 0.0,
        adam_fisher_wd: bool = False,
        adam_use_bias_correction: bool = True,
        adam_use_atan2: bool = False,
        adam_orthogonal_gradient: str = "disabled",
        adam_nesterov: bool = False,
        adam_nesterov_coef: float | None = None,
        adam_kourkoutas_beta: bool = False,
        adam_beta2_min: float = 0.9,
        adam_ema_alpha: float = 0.95,
        adam_tiny_spike: float = 1e-9,
        adam_k_warmup_steps: int = 0,
        adam_spectral_normalization: bool = False,
        adam_state_precision: str = "auto",
        adam_nnmf_factor: bool = False,
        adam_factored_2nd: bool = False,
    ):
        # AdaMuon_adv.py:207-229
        if not (lr >= 0.0):
            raise ValueError(f"Learning-rate should be >= 0.0. Got {lr}")
        if not (weight_decay >= 0.0):
            raise ValueError(f"Weight-decay should be >= 0.0. Got {weight_decay}")
        if not (ns_steps > 0):
            raise ValueError(f"Newton-Schulz steps should be > 0. Got {ns_steps}")
        if spectral_normalization and rms_rescaling:
            print("Warning: spectral_normalization is incompatible with rms_rescaling, Disabling rms_rescaling.")
            rms_rescaling = False
        if spectral_normalization and accelerated_ns:
            raise ValueError("spectral_normalization violates accelerated Newton-Schulz assumptions. Pick one of them.")
        if nnmf_factor:
            state_precision = "factored"
        state_precision = state_precision.lower()
        if state_precision not in VALID_PRECISIONS:
            raise ValueError(f"state_precision must be one of {VALID_PRECISIONS}. Got {state_precision}")
        adam_state_precision = adam_state_precision.lower()
        if adam_state_precision not in VALID_PRECISIONS:
            raise ValueError(f"adam_state_precision must be one of {VALID_PRECISIONS}. Got {adam_state_precision}")
        reject(orthogonal_gradient != "disabled" or adam_orthogonal_gradient != "disabled", "orthogonal_gradient")
        # 'factored' on the orthogonalised path: the reference's factored AdaMuon path fails (original_shape unset, AdaMuon_adv.py:578,657)
        reject(state_precision in ("factored", "fp16"), f"state_precision='{state_precision}'")
        reject(adam_state_precision == "fp16", "adam_state_precision='fp16'")
        # spectral normalisation of the orthogonalised update: the reference
        # calls it without its target_scale argument and fails
        reject(spectral_normalization, "spectral_normalization")
        reject(adam_spectral_normalization and adam_fisher_wd, "adam_spectral_normalization with adam_fisher_wd")
        reject(centered_wd, "centered_wd for AdaMuon_adv")
        reject(not auto_projection and kappa_p not in (1.0, 2.0), f"kappa_p={kappa_p}")
        defaults = {
            "lr": lr, "betas": betas, "weight_decay": weight_decay, "cautious_wd": cautious_wd,
            "eps": eps, "rms_rescaling": rms_rescaling, "ns_steps": ns_steps,
            "ns_eps": ns_eps, "ns_coeffs": ns_coeffs, "nnmf_factor": nnmf_factor,
            "vector_reshape": vector_reshape, "nesterov": nesterov, "nesterov_coef": nesterov_coef,
            "use_atan2": use_atan2, "normuon_variant": normuon_variant, "orthogonal_gradient": orthogonal_gradient,
            "compiled_optimizer": compiled_optimizer, "use_muon": use_muon, "state_precision": state_precision,
            "factored_2nd": factored_2nd, "kappa_p": kappa_p, "auto_projection": auto_projection,
            "low_rank_ortho": low_rank_ortho, "ortho_rank": ortho_rank, "accelerated_ns": accelerated_ns,
            "cns_a_bound": cns_a_bound, "approx_mars": approx_mars, "mars_gamma": mars_gamma,
            "n_layers": n_layers, "spectral_normalization": spectral_normalization, "centered_wd": centered_wd,
            "centered_wd_mode": centered_wd_mode,
            "adam_betas": adam_betas, "adam_eps": adam_eps, "adam_weight_decay": adam_weight_decay,
            "adam_fisher_wd": adam_fisher_wd, "adam_use_bias_correction": adam_use_bias_correction,
            "adam_use_atan2": adam_use_atan2, "adam_orthogonal_gradient": adam_orthogonal_gradient,
            "adam_nesterov": adam_nesterov, "adam_nesterov_coef": adam_nesterov_coef,
            "adam_kourkoutas_beta": adam_kourkoutas_beta, "adam_beta2_min": adam_beta2_min,
            "adam_ema_alpha": adam_ema_alpha, "adam_tiny_spike": adam_tiny_spike,
            "adam_k_warmup_steps": adam_k_warmup_steps, "adam_spectral_normalization": adam_spectral_normalization,
            "adam_state_precision": adam_state_precision, "adam_nnmf_factor": adam_nnmf_factor,
            "adam_factored_2nd": adam_factored_2nd,
        }
        self.stochastic_rounding = stochastic_rounding
        self._init_lr = lr if lr > 0 else 1
        super().__init__(params, defaults)
        self._setup()

    def _normuon_hp(self, group):
        """AdaMuon_adv.py:558-559, 614-615: normuon_update(update, v, beta2, eps)."""
        return (1 - group["betas"][1], group["eps"])

    def _muon_hp(self, group, p):
        """AdaMuon_adv._muon_step_parameter's hyperparameters (AdaMuon_adv.py:492-659)."""
        kappa = group.get("kappa_p", 1.0)
        if group.get("auto_projection", False):
            kappa = 2.0 if p.ndim >= 4 else 1.0
        if kappa not in (1.0, 2.0):
            raise NotImplementedError(f"kappa_p={kappa} is not supported by the B200 optimizer kernels")
        beta1, beta2 = group["betas"]
        return dict(lr=group["lr"], beta1=beta1, beta2=beta2, eps=group["eps"], nesterov=group["nesterov"],
                    nesterov_coef=group.get("nesterov_coef"), ns_steps=group["ns_steps"], ns_eps=group["ns_eps"],
                    ns_coeffs=tuple(group["ns_coeffs"]), cns=group["accelerated_ns"],
                    cns_a_bound=group["cns_a_bound"], rms_rescaling=group["rms_rescaling"],
                    use_atan2=group["use_atan2"], sign_projection=kappa == 1.0,
                    weight_decay=group["weight_decay"], cautious_wd=group.get("cautious_wd", False))
