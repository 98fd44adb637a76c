"""Generate the golden fixtures in tests/golden/*.npz from the reference.

Runs adv_optm 2.5.4 (imported from the reference checkout given by
--reference or the ADV_OPTM_REFERENCE environment variable) on CPU over small seeded parameter
sets, and records for every case:

  * the constructor kwargs, param-group layout, shapes and dtypes,
  * the initial parameters and the gradients of every step,
  * every random integer tensor the reference drew, in draw order, labelled
    with the state key (or 'param') it was drawn for, found by walking the
    call stack at draw time (param_update.py:181-204,240-264),
  * the parameters and every optimizer state tensor after every step,
  * Prodigy's group scalars (d, d_max, d_numerator, k) after every step.

The fixtures pin oracle/oracle.py: tests/test_oracle_golden.py replays the
recorded draws through the oracle and compares.  Re-run with
    python tests/golden/make_golden.py
in a container that holds the reference; the GPU tests never need it.
"""
from __future__ import annotations

import argparse
import inspect
import json
import os
import sys

import numpy as np
import torch

HERE = os.path.dirname(os.path.abspath(__file__))


def bits(t: torch.Tensor) -> np.ndarray:
    t = t.detach().cpu()
    if t.dtype == torch.bfloat16:
        return t.view(torch.int16).numpy().view(np.uint16).copy()
    if t.dtype == torch.float8_e4m3fn:
        return t.view(torch.uint8).numpy().copy()
    return t.numpy().copy()


class DrawRecorder:
    """Wraps the reference's two random-integer sources and records each draw
    with the label of the state it feeds."""

    def __init__(self, pu):
        self.pu = pu
        self.draws = []
        self._orig_sr = pu._get_random_int_for_sr
        self._orig_8 = pu._get_random_int_for_8bit_sr
        self._orig_sk = pu._get_random_noise_for_low_rank_ortho

        self.param_index = {}

        def label():
            lab, idx = "unknown", -1
            for fr in inspect.stack()[2:]:
                if lab == "unknown" and fr.function == "set_state":
                    lab = fr.frame.f_locals["key"]
                if lab == "unknown" and fr.function == "apply_parameter_update":
                    lab = "param"
                if fr.function == "step_parameter":
                    idx = self.param_index.get(id(fr.frame.f_locals["p"]), -1)
                    break
            return lab, idx

        def sr(source):
            r = self._orig_sr(source)
            self.draws.append((*label(), r.clone()))
            return r

        def b8(source, numel=None):
            r = self._orig_8(source, numel)
            self.draws.append((*label(), r.clone()))
            return r

        def sketch(source, ortho_rank):
            r = self._orig_sk(source, ortho_rank)
            self.draws.append(("sketch", label()[1], r.clone()))
            return r

        pu._get_random_int_for_sr = sr
        pu._get_random_int_for_8bit_sr = b8
        pu._get_random_noise_for_low_rank_ortho = sketch

    def take(self):
        d, self.draws = self.draws, []
        return d

    def restore(self):
        self.pu._get_random_int_for_sr = self._orig_sr
        self.pu._get_random_int_for_8bit_sr = self._orig_8
        self.pu._get_random_noise_for_low_rank_ortho = self._orig_sk


def make_params(shapes, dtype, seed, ln_ones=False):
    g = torch.Generator().manual_seed(seed)
    ps = []
    for sh in shapes:
        t = torch.randn(*sh, generator=g) * 0.02
        if ln_ones and len(sh) == 1:
            t = torch.ones(*sh)
        ps.append(torch.nn.Parameter(t.to(dtype)))
    return ps


def make_grad(p, gen, scale=1e-3, outliers=False):
    t = torch.randn(p.shape, generator=gen) * scale
    if outliers:
        mask = torch.rand(p.shape, generator=gen) < 0.01
        t = torch.where(mask, t * 100, t)
    return t.to(p.dtype)


CASES = {
    # config 1 semantics (fp32 AdamW, weight decay)
    "adamw_fp32": dict(cls="AdamW_adv", dtype="f32",
                       shapes=[(96, 48), (48,), (50, 7), (2304,)],
                       kw=dict(lr=1e-3, betas=(0.9, 0.999), eps=1e-8, weight_decay=0.01,
                               state_precision="fp32", factored_2nd=False), steps=3),
    # config 2 semantics (int8_sr + factored_2nd + nesterov, bf16, outlier grads)
    "adamw_int8_f2nd": dict(cls="AdamW_adv", dtype="bf16",
                            shapes=[(300, 70), (64, 64), (96,), (37,), (6, 5)],
                            kw=dict(state_precision="int8_sr", factored_2nd=True, nesterov=True),
                            steps=3, outliers=True),
    "adamw_int8_plain_cautious": dict(cls="AdamW_adv", dtype="bf16",
                                      shapes=[(300, 70), (40,)],
                                      kw=dict(state_precision="int8_sr", weight_decay=0.1, cautious_wd=True,
                                              lr=3e-3), steps=3),
    "adamw_bf16sr": dict(cls="AdamW_adv", dtype="bf16", shapes=[(64, 32), (50,)],
                         kw=dict(state_precision="bf16_sr", weight_decay=0.01), steps=3),
    "adamw_auto_bf16": dict(cls="AdamW_adv", dtype="bf16", shapes=[(64, 32), (50,)],
                            kw=dict(state_precision="auto", weight_decay=0.01, nesterov=True), steps=3),
    "adamw_auto_bf16_f2nd": dict(cls="AdamW_adv", dtype="bf16", shapes=[(64, 32), (50,)],
                                 kw=dict(state_precision="auto", factored_2nd=True), steps=3),
    "adamw_atan2_nesterov_coef": dict(cls="AdamW_adv", dtype="f32", shapes=[(64, 32), (50,)],
                                      kw=dict(state_precision="fp32", use_atan2=True, nesterov=True,
                                              nesterov_coef=0.8), steps=3),
    "adamw_normed_cautious": dict(cls="AdamW_adv", dtype="f32", shapes=[(64, 32), (50,)],
                                  kw=dict(state_precision="fp32", normed_momentum=True, weight_decay=0.05,
                                          cautious_wd=True), steps=3),
    "adamw_nobeta1_nobc": dict(cls="AdamW_adv", dtype="bf16", shapes=[(64, 32), (50,)],
                               kw=dict(state_precision="fp32", betas=(0.0, 0.99), use_bias_correction=False),
                               steps=3),
    "adamw_fisher": dict(cls="AdamW_adv", dtype="bf16", shapes=[(64, 32), (50,)],
                         kw=dict(state_precision="fp32", fisher_wd=True, weight_decay=0.1), steps=3),
    "adamw_centered_int8": dict(cls="AdamW_adv", dtype="bf16", shapes=[(64, 33), (50,)],
                                kw=dict(state_precision="fp32", centered_wd=0.1, centered_wd_mode="int8",
                                        weight_decay=0.01), steps=3),
    "adamw_centered_int4": dict(cls="AdamW_adv", dtype="bf16", shapes=[(64, 33), (50,)],
                                kw=dict(state_precision="fp32", centered_wd=0.1, centered_wd_mode="int4"),
                                steps=3),
    # Kourkoutas-beta: layer-wise dynamic beta2 from the pooled grad norms of the
    # previous step (layers = params of one shape), with and without warm-up
    "adamw_kourkoutas_fp32": dict(cls="AdamW_adv", dtype="f32",
                                  shapes=[(64, 32), (64, 32), (50,), (50,), (96, 48)],
                                  kw=dict(state_precision="fp32", kourkoutas_beta=True, beta2_min=0.9,
                                          ema_alpha=0.9, k_warmup_steps=2, weight_decay=0.01), steps=4),
    "adamw_kourkoutas_int8_f2nd": dict(cls="AdamW_adv", dtype="bf16",
                                       shapes=[(300, 70), (300, 70), (96,), (37,)],
                                       kw=dict(state_precision="int8_sr", factored_2nd=True, nesterov=True,
                                               kourkoutas_beta=True, beta2_min=0.88), steps=4, outliers=True),
    # centered weight decay with the reference's default anchor storage (float8_e4m3fn)
    "adamw_centered_float8": dict(cls="AdamW_adv", dtype="bf16", shapes=[(64, 33), (50,)],
                                  kw=dict(state_precision="fp32", centered_wd=0.1, weight_decay=0.01), steps=3),
    "adamw_centered_float8_f32": dict(cls="AdamW_adv", dtype="f32", shapes=[(64, 33), (50,)],
                                      kw=dict(state_precision="int8_sr", centered_wd=0.05, cautious_wd=True),
                                      steps=3),
    "adamw_centered_full_f32": dict(cls="AdamW_adv", dtype="f32", shapes=[(64, 33), (50,)],
                                    kw=dict(state_precision="fp32", centered_wd=0.1, centered_wd_mode="full",
                                            cautious_wd=True), steps=3),
    # config 3 semantics (Muon quintic, bf16 'auto' momentum; aux Adam fp32)
    "muon_auto_bf16": dict(cls="Muon_adv", dtype="bf16",
                           groups=[dict(shapes=[(64, 48), (48, 96)], optim_type="muon"),
                                   dict(shapes=[(100, 32), (48,)], optim_type="adam")],
                           kw=dict(lr=1e-3, beta1=0.95, adam_state_precision="fp32"), steps=2),
    "muon_int8_wd": dict(cls="Muon_adv", dtype="bf16",
                         groups=[dict(shapes=[(64, 48), (96, 40)], optim_type="muon"),
                                 dict(shapes=[(48,)], optim_type="adam")],
                         kw=dict(lr=2e-3, state_precision="int8_sr", weight_decay=0.01,
                                 adam_state_precision="int8_sr", adam_weight_decay=0.01), steps=2),
    # no optim_type / use_muon: every param is routed by _is_suitable_for_muon
    # (2-D, 3-D flattened, 1-D, degenerate and extreme-aspect shapes)
    "muon_auto_route": dict(cls="Muon_adv", dtype="bf16",
                            groups=[dict(shapes=[(64, 48), (48,), (2, 64), (600, 4), (8, 4, 3), (1, 64), (40, 96)],
                                         optim_type=None)],
                            kw=dict(lr=1e-3, adam_state_precision="fp32"), steps=2),
    # Kourkoutas-beta on the auxiliary Adam: the mixed third group loses the
    # flag at state creation; its 1-D param still pools into the (48,) layer.
    # With bias correction the v update keeps adam_betas[1].
    "muon_kourkoutas_bc": dict(cls="Muon_adv", dtype="bf16",
                               groups=[dict(shapes=[(64, 48), (48, 96)], optim_type="muon"),
                                       dict(shapes=[(100, 32), (100, 32), (48,)], optim_type="adam"),
                                       dict(shapes=[(48,), (40, 96)], optim_type=None)],
                               kw=dict(lr=1e-3, adam_state_precision="fp32", adam_kourkoutas_beta=True,
                                       adam_beta2_min=0.88, adam_ema_alpha=0.9, adam_k_warmup_steps=1), steps=4),
    # without bias correction the dynamic beta2 reaches v; an auxiliary param
    # outside every layer takes AdaMuon's betas[1]
    "adamuon_kourkoutas_nobc": dict(cls="AdaMuon_adv", dtype="bf16",
                                    groups=[dict(shapes=[(64, 48)], optim_type="muon"),
                                            dict(shapes=[(100, 32), (48,)], optim_type="adam"),
                                            dict(shapes=[(48,), (33,), (64, 48)], optim_type=None)],
                                    kw=dict(lr=1e-3, adam_state_precision="fp32", adam_kourkoutas_beta=True,
                                            adam_use_bias_correction=False, adam_beta2_min=0.88,
                                            adam_ema_alpha=0.9), steps=4),
    # NorMuon (row-wise second moment after Newton-Schulz) and approximated
    # MARS-M (grad correction from the previous grad)
    "muon_normuon_mars": dict(cls="Muon_adv", dtype="bf16",
                              groups=[dict(shapes=[(64, 48), (48, 96), (8, 4, 3)], optim_type="muon"),
                                      dict(shapes=[(48,)], optim_type="adam")],
                              kw=dict(lr=1e-3, normuon_variant=True, approx_mars=True, mars_gamma=0.05), steps=3),
    "muon_normuon_fp32_states": dict(cls="Muon_adv", dtype="bf16",
                                     groups=[dict(shapes=[(64, 48), (48, 96)], optim_type="muon")],
                                     kw=dict(lr=1e-3, normuon_variant=True, state_precision="fp32",
                                             beta2_normuon=0.9), steps=3),
    "adamuon_normuon_mars": dict(cls="AdaMuon_adv", dtype="bf16",
                                 groups=[dict(shapes=[(64, 48), (40, 96)], optim_type="muon"),
                                         dict(shapes=[(48,)], optim_type="adam")],
                                 kw=dict(lr=1e-3, normuon_variant=True, approx_mars=True), steps=3),
    # low-rank Newton-Schulz: Gaussian sketch, QR, projected chain
    "muon_low_rank": dict(cls="Muon_adv", dtype="bf16",
                          groups=[dict(shapes=[(96, 64), (64, 160), (40, 96)], optim_type="muon")],
                          kw=dict(lr=1e-3, low_rank_ortho=True, ortho_rank=16), steps=2),
    "adamuon_low_rank_cans": dict(cls="AdaMuon_adv", dtype="bf16",
                                  groups=[dict(shapes=[(96, 64), (64, 160)], optim_type="muon")],
                                  kw=dict(lr=1e-3, low_rank_ortho=True, ortho_rank=24, accelerated_ns=True),
                                  steps=2),
    # AdaMuon's factored second moment (mu_vbuf_nmf / mv_vbuf_nmf)
    "adamuon_factored_2nd": dict(cls="AdaMuon_adv", dtype="bf16",
                                 groups=[dict(shapes=[(64, 48), (48, 96), (40, 30)], optim_type="muon")],
                                 kw=dict(lr=1e-3, factored_2nd=True), steps=3),
    # config 4 semantics (Prodigy bf16_sr)
    "prodigy_bf16sr": dict(cls="Prodigy_adv", dtype="bf16", shapes=[(120, 40), (40,), (64, 64)],
                           kw=dict(state_precision="bf16_sr", d0=1e-6, slice_p=11), steps=3,
                           log_scale=True),
    "prodigy_fp32_wd": dict(cls="Prodigy_adv", dtype="f32", shapes=[(120, 40), (40,)],
                            kw=dict(state_precision="fp32", d0=1e-4, weight_decay=0.01, slice_p=5,
                                    nesterov=True), steps=3, log_scale=True),
    # the d estimate stops after prodigy_steps: s and p0 are freed, d is frozen
    "prodigy_steps_bf16": dict(cls="Prodigy_adv", dtype="bf16", shapes=[(120, 40), (40,)],
                               kw=dict(state_precision="bf16_sr", d0=1e-4, slice_p=7, prodigy_steps=2),
                               steps=4, log_scale=True),
    # Kourkoutas-beta under Prodigy: v's weight is d * d * (1 - beta2_dyn)
    "prodigy_kourkoutas_fp32": dict(cls="Prodigy_adv", dtype="f32", shapes=[(120, 40), (120, 40), (40,), (64, 64)],
                                    kw=dict(state_precision="fp32", d0=1e-4, slice_p=5, kourkoutas_beta=True,
                                            beta2_min=0.88, ema_alpha=0.9, k_warmup_steps=2),
                                    steps=4, log_scale=True),
    # config 5 semantics (AdaMuon CANS, int8_sr)
    "adamuon_cans_int8": dict(cls="AdaMuon_adv", dtype="bf16",
                              groups=[dict(shapes=[(64, 48), (48, 96)], optim_type="muon"),
                                      dict(shapes=[(48,)], optim_type="adam")],
                              kw=dict(accelerated_ns=True, state_precision="int8_sr"), steps=2),
    "lion_bf16": dict(cls="Lion_adv", dtype="bf16", shapes=[(64, 32), (32,)],
                      kw=dict(lr=1e-4, weight_decay=0.01), steps=3),
    "lion_fp32_cautious": dict(cls="Lion_adv", dtype="f32", shapes=[(64, 32), (32,)],
                               kw=dict(lr=1e-4, weight_decay=0.1, cautious_wd=True), steps=3),
    # state_precision='factored': m as signed rank-1 factors (1-bit sign), v as
    # rank-1 factors; 1-D params keep fp32 states.  Effective shapes (150, 140),
    # (64, 64), (40, 33) (a ragged last sign byte) and a 3-D param.
    "adamw_factored_bf16": dict(cls="AdamW_adv", dtype="bf16",
                                shapes=[(300, 70), (64, 64), (96,), (40, 33), (8, 4, 3)],
                                kw=dict(state_precision="factored", nesterov=True, weight_decay=0.01),
                                steps=3, outliers=True),
    "adamw_factored_f32_atan2": dict(cls="AdamW_adv", dtype="f32", shapes=[(64, 48), (50,), (40, 33)],
                                     kw=dict(nnmf_factor=True, use_atan2=True, cautious_wd=True,
                                             weight_decay=0.05), steps=3),
    "adamw_factored_normed": dict(cls="AdamW_adv", dtype="bf16", shapes=[(64, 48), (50,)],
                                  kw=dict(state_precision="factored", betas=(0.9, 0.99), normed_momentum=True),
                                  steps=3),
    "prodigy_factored_bf16": dict(cls="Prodigy_adv", dtype="bf16", shapes=[(120, 40), (40,), (40, 33)],
                                  kw=dict(state_precision="factored", d0=1e-6, slice_p=11, nesterov=True),
                                  steps=3, log_scale=True),
    "lion_factored_bf16": dict(cls="Lion_adv", dtype="bf16", shapes=[(64, 32), (32,), (40, 33)],
                               kw=dict(lr=1e-4, weight_decay=0.01, nnmf_factor=True), steps=3),
    "lion_factored_f32_cautious": dict(cls="Lion_adv", dtype="f32", shapes=[(64, 48), (40, 33)],
                                       kw=dict(lr=1e-4, weight_decay=0.1, cautious_wd=True, nnmf_factor=True),
                                       steps=3),
    "muon_aux_factored": dict(cls="Muon_adv", dtype="bf16",
                              groups=[dict(shapes=[(64, 48)], optim_type="muon"),
                                      dict(shapes=[(100, 32), (48,), (40, 33)], optim_type="adam")],
                              kw=dict(lr=1e-3, adam_state_precision="factored", adam_nesterov=True), steps=3),
    # spectral normalisation (one power-iteration step per 2-D update, max-abs
    # scaling for 1-D updates); the initial singular vectors are recorded in st0
    "adamw_spectral_bf16": dict(cls="AdamW_adv", dtype="bf16", shapes=[(64, 48), (48,), (40, 96), (8, 4, 3)],
                                kw=dict(state_precision="auto", spectral_normalization=True, weight_decay=0.01),
                                steps=3),
    "adamw_spectral_factored_f32": dict(cls="AdamW_adv", dtype="f32", shapes=[(64, 48), (50,)],
                                        kw=dict(state_precision="factored", spectral_normalization=True,
                                                cautious_wd=True, weight_decay=0.05), steps=3),
    # bf16 params without stochastic rounding: decoupled and centered decay run
    # as add_(target, alpha=-wd*lr) on the bf16 param, which rounds alpha to bf16
    "adamw_bf16_nosr_wd": dict(cls="AdamW_adv", dtype="bf16", shapes=[(64, 33), (50,)],
                               kw=dict(state_precision="auto", weight_decay=0.37, centered_wd=0.21,
                                       centered_wd_mode="full", stochastic_rounding=False, lr=3e-3), steps=3),
    "lion_bf16_nosr_wd": dict(cls="Lion_adv", dtype="bf16", shapes=[(64, 32), (32,)],
                              kw=dict(lr=3e-4, weight_decay=0.37, stochastic_rounding=False), steps=3),
    "muon_nosr_wd": dict(cls="Muon_adv", dtype="bf16",
                         groups=[dict(shapes=[(64, 48)], optim_type="muon"),
                                 dict(shapes=[(100, 32), (48,)], optim_type="adam")],
                         kw=dict(lr=3e-3, weight_decay=0.37, adam_weight_decay=0.29, stochastic_rounding=False,
                                 adam_state_precision="auto"), steps=2),
    # Prodigy_adv has no spectral_normalization argument; its step reads the
    # param-group key (Prodigy_adv.py:319-320, 490-493)
    "prodigy_spectral_group_key": dict(cls="Prodigy_adv", dtype="bf16", shapes=[(120, 40), (40,), (24, 5, 6)],
                                       kw=dict(state_precision="auto", d0=1e-4, slice_p=7, weight_decay=0.01),
                                       group_kw=dict(spectral_normalization=True), steps=3, log_scale=True),
    "lion_spectral_bf16": dict(cls="Lion_adv", dtype="bf16", shapes=[(64, 32), (32,)],
                               kw=dict(lr=1e-4, weight_decay=0.01, spectral_normalization=True), steps=3),
    "muon_aux_spectral": dict(cls="Muon_adv", dtype="bf16",
                              groups=[dict(shapes=[(64, 48)], optim_type="muon"),
                                      dict(shapes=[(100, 32), (48,)], optim_type="adam")],
                              kw=dict(lr=1e-3, adam_state_precision="fp32", adam_spectral_normalization=True),
                              steps=3),
}


def run_case(name, spec, adv_optm, pu):
    dtype = torch.bfloat16 if spec["dtype"] == "bf16" else torch.float32
    if "groups" in spec:
        shapes = [sh for gspec in spec["groups"] for sh in gspec["shapes"]]
    else:
        shapes = spec["shapes"]
    params = make_params(shapes, dtype, seed=1234, ln_ones=spec.get("ln_ones", False))
    if "groups" in spec:
        groups, k = [], 0
        for gspec in spec["groups"]:
            n = len(gspec["shapes"])
            grp = {"params": params[k:k + n]}
            if gspec["optim_type"] is not None:
                grp["optim_type"] = gspec["optim_type"]
            groups.append(grp)
            k += n
    elif "group_kw" in spec:
        # keys the constructor does not take but a param group may carry
        groups = [dict(params=params, **spec["group_kw"])]
    else:
        groups = params
    cls = getattr(adv_optm, spec["cls"])
    torch.manual_seed(0)
    rec = DrawRecorder(pu)
    rec.param_index = {id(p): i for i, p in enumerate(params)}
    out = {}
    # the initial spectral singular vectors, recorded where they are drawn
    # (Prodigy_adv creates its states at the first step)
    mod = sys.modules[cls.__module__]
    orig_init_sn = getattr(mod, "init_spectral_norm", None)
    init_sn = {}
    if orig_init_sn is not None:
        def rec_init_sn(state, p):
            orig_init_sn(state, p)
            i = rec.param_index.get(id(p), -1)
            init_sn[i] = {k: bits(state[k]) for k in ("spectral_u", "spectral_v") if k in state}
        mod.init_spectral_norm = rec_init_sn
    try:
        # the optimizer's constructor reseeds the per-device generator to 42
        opt = cls(groups, **spec["kw"])
        out["meta"] = np.array(json.dumps(dict(name=name, cls=spec["cls"], dtype=spec["dtype"],
                                                shapes=[list(s) for s in shapes],
                                                groups=[dict(n=len(g["shapes"]), optim_type=g["optim_type"])
                                                        for g in spec["groups"]] if "groups" in spec else None,
                                                kw=spec["kw"], steps=spec["steps"],
                                                group_kw=spec.get("group_kw"))))
        for i, p in enumerate(params):
            out[f"p0_{i}"] = bits(p)
            st = opt.state.get(p, {})
            if "is_muon" in st:
                out[f"route_{i}"] = np.array(int(bool(st["is_muon"])))
            for key, val in st.items():
                if torch.is_tensor(val):
                    out[f"st0_{i}_{key}"] = bits(val)
        gen = torch.Generator().manual_seed(99)
        for s in range(spec["steps"]):
            scale = 1e-3
            if spec.get("log_scale"):
                scale = float(10 ** (-4 + 2 * torch.rand(1, generator=gen).item()))
            for i, p in enumerate(params):
                p.grad = make_grad(p, gen, scale, spec.get("outliers", False))
                out[f"g_{s}_{i}"] = bits(p.grad)
            rec.take()
            opt.step()
            draws = rec.take()
            # draws are keyed by step, param index and label; values < 2**16
            # are stored as uint16.  `order_{s}` keeps the draw order.
            order = []
            for lab, idx, r in draws:
                if lab == "sketch":
                    # low-rank Newton-Schulz: the Gaussian sketch, in the update's dtype
                    out[f"sk_{s}_{idx}"] = bits(r)
                    order.append(f"{idx}:{lab}")
                    continue
                out[f"r_{s}_{idx}_{lab}"] = r.numpy().astype(np.uint16).reshape(-1)
                order.append(f"{idx}:{lab}")
            out[f"order_{s}"] = np.array(json.dumps(order))
            for i, p in enumerate(params):
                out[f"p_{s}_{i}"] = bits(p)
                for key, val in opt.state[p].items():
                    if torch.is_tensor(val):
                        out[f"st_{s}_{i}_{key}"] = bits(val)
                    elif key == "step":
                        out[f"st_{s}_{i}_step"] = np.array(val)
            if spec["cls"] == "Prodigy_adv":
                g0 = opt.param_groups[0]
                out[f"d_{s}"] = np.array([g0["d"], g0["d_max"], g0["d_numerator"], g0["k"]], np.float64)
    finally:
        rec.restore()
        if orig_init_sn is not None:
            mod.init_spectral_norm = orig_init_sn
    for i, d in init_sn.items():
        for k, v in d.items():
            out.setdefault(f"st0_{i}_{k}", v)
    return out


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--reference", default=os.environ.get("ADV_OPTM_REFERENCE"),
                    help="checkout of Koratahiu/Advanced_Optimizers (the directory holding adv_optm/)")
    ap.add_argument("--only", default=None)
    args = ap.parse_args()
    if not args.reference:
        ap.error("give --reference or set ADV_OPTM_REFERENCE")
    sys.path.insert(0, args.reference)
    import adv_optm  # noqa: E402
    from adv_optm.util import param_update as pu  # noqa: E402
    torch.set_num_threads(max(1, os.cpu_count() or 1))
    for name, spec in CASES.items():
        if args.only and name != args.only:
            continue
        out = run_case(name, spec, adv_optm, pu)
        path = os.path.join(HERE, f"{name}.npz")
        np.savez_compressed(path, **out)
        print(f"{name}: {os.path.getsize(path) / 1024:.1f} KiB")


if __name__ == "__main__":
    main()
