"""Muon_adv on B200: drop-in for adv_optm.Muon_adv (Muon_adv.py:13-569).

'muon' parameters (2-D and higher, flattened to [shape[0], -1]) take the
momentum / Newton–Schulz / RMS-rescale path on the device: csrc/muon.cu for
the elementwise stages and csrc/ns_gemm.cu (tcgen05 + TMEM + TMA) for every
GEMM of the quintic or CANS iteration.  'adam' parameters take the
auxiliary AdamW step (Muon_AuxAdam.py) in the Adam-family kernel.  Options
the kernels do not implement raise NotImplementedError at construction.
"""
from __future__ import annotations

from ._common import reject
from ._muon_base import MuonFamilyBase

VALID_PRECISIONS = {"auto", "fp32", "factored", "bf16_sr", "fp16", "int8_sr"}


class Muon_adv(MuonFamilyBase):
    """Muon (momentum orthogonalised by Newton–Schulz) with an auxiliary AdamW."""

    _adamuon = False

    def __init__(
        self,
        params,
        lr: float = 1e-3,
        beta1: float = 0.95,
        weight_decay: float = 0.0,
        cautious_wd: bool = False,
        nesterov: bool = True,
        nesterov_coef: float | None = None,
        ns_steps: int = 5,
        ns_eps: float | None = 1e-7,
        ns_coeffs: tuple[float, float, float] = (3.4445, -4.7750, 2.0315),
        stochastic_rounding: bool = True,
        orthogonal_gradient: str = "disabled",
        rms_rescaling: bool = True,
        nnmf_factor: bool = False,
        vector_reshape: bool = False,
        use_muon: bool | None = None,
        state_precision: str = "auto",
        low_rank_ortho: bool = False,
        ortho_rank: int = 128,
        normuon_variant: bool = False,
        beta2_normuon: float = 0.95,
        normuon_eps: float = 1e-8,
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
        # Muon_adv.py:176-200
        if not (lr >= 0.0):
            raise ValueError(f"Learning-rate should be >= 0.0. Got {lr}")
        if not (0.0 <= beta1 < 1.0):
            raise ValueError(f"beta1 should be in [0.0, 1.0). Got {beta1}")
        if normuon_variant and not (0.0 <= beta2_normuon < 1.0):
            raise ValueError(f"beta2_normuon should be in [0.0, 1.0) for NorMuon. Got {beta2_normuon}")
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
        # 'factored' on the orthogonalised path: the reference's factored Muon path never applies lr to the update (Muon_adv.py:463-503)
        reject(state_precision in ("factored", "fp16"), f"state_precision='{state_precision}'")
        reject(adam_state_precision == "fp16", "adam_state_precision='fp16'")
        # spectral normalisation of the orthogonalised update: the reference
        # calls it without its target_scale argument and fails
        reject(spectral_normalization, "spectral_normalization")
        reject(adam_spectral_normalization and adam_fisher_wd, "adam_spectral_normalization with adam_fisher_wd")
        reject(centered_wd, "centered_wd for Muon_adv")
        defaults = {
            "lr": lr, "beta1": beta1, "weight_decay": weight_decay, "cautious_wd": cautious_wd,
            "nesterov": nesterov, "nesterov_coef": nesterov_coef, "ns_steps": ns_steps, "ns_eps": ns_eps,
            "ns_coeffs": ns_coeffs, "nnmf_factor": nnmf_factor, "vector_reshape": vector_reshape,
            "rms_rescaling": rms_rescaling, "orthogonal_gradient": orthogonal_gradient,
            "compiled_optimizer": compiled_optimizer, "use_muon": use_muon, "state_precision": state_precision,
            "low_rank_ortho": low_rank_ortho, "ortho_rank": ortho_rank, "normuon_variant": normuon_variant,
            "beta2_normuon": beta2_normuon, "normuon_eps": normuon_eps, "accelerated_ns": accelerated_ns,
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
        self.compiled_optimizer = compiled_optimizer
        self._init_lr = lr if lr > 0 else 1
        super().__init__(params, defaults)
        self._setup()

    def _normuon_hp(self, group):
        """Muon_adv.py:505: normuon_update(update, v, beta2_normuon, normuon_eps)."""
        return (1 - group["beta2_normuon"], group["normuon_eps"])

    def _muon_hp(self, group, p):
        """Muon_adv._muon_step_parameter's hyperparameters (Muon_adv.py:443-555)."""
        return dict(lr=group["lr"], beta1=group["beta1"], beta2=0.0, eps=None, nesterov=group["nesterov"],
                    nesterov_coef=group.get("nesterov_coef"), ns_steps=group["ns_steps"], ns_eps=group["ns_eps"],
                    ns_coeffs=tuple(group["ns_coeffs"]), cns=group["accelerated_ns"],
                    cns_a_bound=group["cns_a_bound"], rms_rescaling=group["rms_rescaling"], use_atan2=False,
                    sign_projection=False, weight_decay=group["weight_decay"],
                    cautious_wd=group.get("cautious_wd", False))
