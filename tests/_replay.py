"""Shared helpers for tests: load golden fixtures and replay them through
the oracle (test infrastructure; imports oracle/)."""
from __future__ import annotations

import json
import math
import os
import sys

import numpy as np

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
GOLDEN = os.path.join(ROOT, "tests", "golden")
if ROOT not in sys.path:
    sys.path.insert(0, ROOT)

from oracle import oracle as O  # noqa: E402

ADAMW_DEFAULTS = dict(lr=1e-3, betas=(0.9, 0.999), eps=1e-8, weight_decay=0.0, fisher_wd=False,
                      cautious_wd=False, use_bias_correction=True, stochastic_rounding=True,
                      use_atan2=False, nesterov=False, nesterov_coef=None, normed_momentum=False,
                      centered_wd=0.0, centered_wd_mode="float8", state_precision="auto",
                      factored_2nd=False, kourkoutas_beta=False, beta2_min=0.9, ema_alpha=0.95,
                      tiny_spike=1e-9, k_warmup_steps=0, nnmf_factor=False, spectral_normalization=False)
MUON_DEFAULTS = dict(lr=1e-3, beta1=0.95, weight_decay=0.0, cautious_wd=False, nesterov=True,
                     nesterov_coef=None, ns_steps=5, ns_eps=1e-7, ns_coeffs=(3.4445, -4.7750, 2.0315),
                     stochastic_rounding=True, rms_rescaling=True, state_precision="auto",
                     accelerated_ns=False, cns_a_bound=None, centered_wd=0.0, centered_wd_mode="float8",
                     adam_betas=(0.9, 0.99), adam_eps=1e-8, adam_weight_decay=0.0, adam_fisher_wd=False,
                     adam_use_bias_correction=True, adam_use_atan2=False, adam_nesterov=False,
                     adam_nesterov_coef=None, adam_state_precision="auto", adam_factored_2nd=False,
                     adam_kourkoutas_beta=False, adam_beta2_min=0.9, adam_ema_alpha=0.95, adam_tiny_spike=1e-9,
                     adam_k_warmup_steps=0, normuon_variant=False, beta2_normuon=0.95, normuon_eps=1e-8,
                     approx_mars=False, mars_gamma=0.025, low_rank_ortho=False, ortho_rank=128,
                     adam_nnmf_factor=False, adam_spectral_normalization=False)
ADAMUON_DEFAULTS = dict(MUON_DEFAULTS, betas=(0.95, 0.95), eps=1e-8, use_atan2=False, factored_2nd=False,
                        kappa_p=1.0, auto_projection=True)
PRODIGY_DEFAULTS = dict(lr=1.0, betas=(0.9, 0.999), eps=1e-8, weight_decay=0.0, fisher_wd=False,
                        cautious_wd=False, stochastic_rounding=True, use_atan2=False, nesterov=False,
                        nesterov_coef=None, state_precision="auto", factored_2nd=False, beta3=None,
                        d0=1e-6, d_coef=1.0, growth_rate=float("inf"), safeguard_warmup=False,
                        slice_p=11, prodigy_steps=0, d_limiter=False, centered_wd=0.0,
                        centered_wd_mode="float8", kourkoutas_beta=False, beta2_min=0.9, ema_alpha=0.95,
                        tiny_spike=1e-9, k_warmup_steps=0)
LION_DEFAULTS = dict(lr=1e-4, betas=(0.9, 0.99), weight_decay=0.0, cautious_wd=False, stochastic_rounding=True,
                     nnmf_factor=False, spectral_normalization=False)


def list_cases():
    return sorted(f[:-4] for f in os.listdir(GOLDEN) if f.endswith(".npz"))


def load(name):
    z = np.load(os.path.join(GOLDEN, name + ".npz"))
    meta = json.loads(str(z["meta"]))
    return meta, z


def values(arr, dt):
    """fixture array -> float32 values."""
    return O.from_bf16_bits(arr) if dt == "bf16" else np.asarray(arr, np.float32)


def route_kinds(meta):
    """'muon' / 'adam' per param of a Muon-family case: the group's optim_type,
    or the oracle's _is_suitable_for_muon where the group names none; 'main'
    for the other optimizers."""
    shapes = [tuple(s) for s in meta["shapes"]]
    if not meta["groups"]:
        return ["main"] * len(shapes)
    kinds, k = [], 0
    for g in meta["groups"]:
        for sh in shapes[k:k + g["n"]]:
            t = g["optim_type"]
            kinds.append(t if t is not None else ("muon" if O.is_suitable_for_muon(sh) else "adam"))
        k += g["n"]
    return kinds


def draws(z, step, i):
    out = {}
    pre = f"r_{step}_{i}_"
    for k in z.files:
        if k.startswith(pre):
            out[k[len(pre):]] = z[k].astype(np.int32)
    if f"sk_{step}_{i}" in z.files:
        out["sketch"] = z[f"sk_{step}_{i}"]      # low-rank Newton-Schulz sketch (the update's dtype)
    return out


def _adam_hp(kw, aux=False, precision=None):
    if aux:
        d = {k: v for k, v in MUON_DEFAULTS.items()}
        d.update(kw)
        return dict(lr=d["lr"], betas=tuple(d["adam_betas"]), eps=d["adam_eps"],
                    weight_decay=d["adam_weight_decay"], fisher_wd=d["adam_fisher_wd"],
                    cautious_wd=d["cautious_wd"], use_bias_correction=d["adam_use_bias_correction"],
                    stochastic_rounding=d["stochastic_rounding"], use_atan2=d["adam_use_atan2"],
                    nesterov=d["adam_nesterov"], nesterov_coef=d["adam_nesterov_coef"],
                    centered_wd=d["centered_wd"], centered_wd_mode=d["centered_wd_mode"],
                    precision="factored" if d["adam_nnmf_factor"] else d["adam_state_precision"],
                    factored_2nd=d["adam_factored_2nd"], spectral=d["adam_spectral_normalization"])
    d = dict(ADAMW_DEFAULTS)
    d.update(kw)
    d["betas"] = tuple(d["betas"])
    d["precision"] = "factored" if d["nnmf_factor"] else d["state_precision"]
    d["spectral"] = d["spectral_normalization"]
    return d


def inject_initial(z, states):
    """States the reference draws at construction (the spectral singular
    vectors, from its torch generator) are taken from the fixture."""
    for i, st in enumerate(states):
        for key in ("spectral_u", "spectral_v"):
            if f"st0_{i}_{key}" in z.files:
                st[key] = np.array(z[f"st0_{i}_{key}"])


def replay(name, steps=None, pin_d=False, teacher=False):
    """Run the oracle over a golden case.  Yields (step, i, p_values, state)
    after every param update, in the reference's loop order."""
    meta, z = load(name)
    dt = meta["dtype"]
    shapes = [tuple(s) for s in meta["shapes"]]
    kw = meta["kw"]
    cls = meta["cls"]
    nsteps = meta["steps"] if steps is None else steps
    ps = [values(z[f"p0_{i}"], dt).reshape(shapes[i]) for i in range(len(shapes))]
    kinds = route_kinds(meta)
    states = []
    group = None
    kk = None
    if cls == "AdamW_adv":
        hp = _adam_hp(kw)
        if hp.get("kourkoutas_beta"):
            kk = O.Kourkoutas(shapes, hp["betas"][1], hp["beta2_min"], hp["ema_alpha"], hp["tiny_spike"],
                              hp["k_warmup_steps"])
        for i, sh in enumerate(shapes):
            st = O.adamw_init_state(sh, dt, hp["precision"], hp["factored_2nd"], hp["betas"][0])
            if hp["centered_wd"]:
                st.update(O.init_anchor(ps[i], dt, hp["centered_wd_mode"]))
            states.append(st)
    elif cls in ("Muon_adv", "AdaMuon_adv"):
        base = dict(MUON_DEFAULTS if cls == "Muon_adv" else ADAMUON_DEFAULTS)
        base.update(kw)
        base["precision"] = base["state_precision"]
        base["betas"] = tuple(base.get("betas", (0.95, 0.95)))
        aux = _adam_hp(kw, aux=True)
        for i, sh in enumerate(shapes):
            if kinds[i] == "muon":
                st = {}
                O.init_state_tensor(st, "momentum_buffer", sh, base["precision"], dt)
                if cls == "AdaMuon_adv" and base.get("factored_2nd") and not base["normuon_variant"]:
                    d1, d2 = O.effective_shape(int(np.prod(sh)))
                    st["effective_shape"] = (d1, d2)
                    st["factored_2nd"] = True
                    st["mu_vbuf_nmf"] = np.zeros(d1, np.float32)
                    st["mv_vbuf_nmf"] = np.zeros(d2, np.float32)
                elif cls == "AdaMuon_adv" and not base["normuon_variant"]:
                    O.init_state_tensor(st, "second_momentum_buffer", sh, base["precision"], dt, non_neg=True)
                if base["normuon_variant"]:
                    st["normuon_v"] = np.zeros(sh[0], np.float32)
                if base["approx_mars"]:
                    st["last_grad"] = np.zeros(sh, np.uint16 if dt == "bf16" else np.float32)
                states.append(st)
            else:
                states.append(O.adamw_init_state(sh, dt, aux["precision"], aux["factored_2nd"], aux["betas"][0]))
        kk_members = set()
        if base.get("adam_kourkoutas_beta"):
            # the helper is built after the states: groups holding a Muon param
            # have lost the flag by then (Muon_adv.py:248-252, 353)
            layer_shapes, k = [], 0
            for gm in meta["groups"]:
                idx = list(range(k, k + gm["n"]))
                if all(kinds[j] != "muon" for j in idx):
                    layer_shapes += [shapes[j] for j in idx]
                    kk_members.update(idx)
                k += gm["n"]
            if layer_shapes:
                kk = O.Kourkoutas(layer_shapes, aux["betas"][1], base["adam_beta2_min"], base["adam_ema_alpha"],
                                  base["adam_tiny_spike"], base["adam_k_warmup_steps"])
    elif cls == "Prodigy_adv":
        hp = dict(PRODIGY_DEFAULTS)
        hp.update(kw)
        if hp.get("kourkoutas_beta"):
            kk = O.Kourkoutas(shapes, hp["betas"][1], hp["beta2_min"], hp["ema_alpha"], hp["tiny_spike"],
                              hp["k_warmup_steps"])
        hp["betas"] = tuple(hp["betas"])
        hp["precision"] = "factored" if hp.get("nnmf_factor") else hp["state_precision"]
        hp["spectral"] = hp.get("spectral_normalization", False) or \
            bool((meta.get("group_kw") or {}).get("spectral_normalization", False))
        group = dict(d=hp["d0"], d0=hp["d0"], d_max=hp["d0"], d_numerator=0.0, d_coef=hp["d_coef"],
                     growth_rate=hp["growth_rate"], d_limiter=hp["d_limiter"], k=0,
                     prodigy_steps=hp["prodigy_steps"],
                     beta3=hp["beta3"] if hp["beta3"] is not None else math.sqrt(hp["betas"][1]))
        for i, sh in enumerate(shapes):
            st = O.adamw_init_state(sh, dt, hp["precision"], hp["factored_2nd"], hp["betas"][0])
            sl = ps[i].reshape(-1)[::hp["slice_p"]]
            st["s"] = np.zeros(sl.shape, np.uint16) if dt == "bf16" else np.zeros(sl.shape, np.float32)
            if np.any(ps[i] != 0):
                st["p0"] = O.bf16_bits(sl) if dt == "bf16" else sl.astype(np.float32).copy()
            else:
                st["p0"] = np.zeros((), np.uint16 if dt == "bf16" else np.float32)
            states.append(st)
    elif cls == "Lion_adv":
        hp = dict(LION_DEFAULTS)
        hp.update(kw)
        hp["betas"] = tuple(hp["betas"])
        hp["spectral"] = hp["spectral_normalization"]
        for i, sh in enumerate(shapes):
            states.append(O.lion_init_state(sh, dt, hp["nnmf_factor"]))
    else:
        raise KeyError(cls)
    inject_initial(z, states)

    d_num_carry = np.float32(0.0)
    for s in range(nsteps):
        if cls == "Prodigy_adv":
            d_num = np.float32(d_num_carry)
            d_den = np.float32(0.0)
        if teacher and s > 0:
            # start every step from the reference's own params and states so
            # that each step's comparison measures that step alone
            for i, sh in enumerate(shapes):
                ps[i] = values(z[f"p_{s - 1}_{i}"], dt).reshape(sh)
                for key in list(states[i].keys()):
                    fk = f"st_{s - 1}_{i}_{key}"
                    if fk in z.files and isinstance(states[i][key], np.ndarray):
                        states[i][key] = np.array(z[fk]).astype(states[i][key].dtype).reshape(states[i][key].shape)
        if kk is not None:
            if teacher and s > 0:
                for i, sh in enumerate(shapes):
                    fk = f"st_{s - 1}_{i}_kourkoutas_r_ema"
                    if fk in z.files:
                        kk.ema[tuple(sh)] = np.float32(z[fk])
            kk.prepare(s)
        for i, sh in enumerate(shapes):
            g = values(z[f"g_{s}_{i}"], dt).reshape(sh)
            r = draws(z, s, i)
            if cls == "AdamW_adv":
                hp_i = hp if kk is None else dict(hp, beta2_dyn=kk.beta2[tuple(sh)], kourkoutas=kk)
                ps[i] = O.adam_family_step(ps[i], dt, g, states[i], hp_i, r, algo="adamw")
                if kk is not None:
                    states[i]["kourkoutas_r_ema"] = np.array(kk.ema[tuple(sh)], np.float32)
            elif cls in ("Muon_adv", "AdaMuon_adv"):
                if kinds[i] == "muon":
                    fn = O.muon_step if cls == "Muon_adv" else O.adamuon_step
                    ps[i] = fn(ps[i], dt, g, states[i], base, r)
                else:
                    aux_i = aux
                    if kk is not None:
                        # pooled by layer key whatever the group; the dynamic
                        # beta2 only without bias correction, else beta2 of
                        # 'betas' (AdaMuon) or adam_betas (Muon_adv.py:377-391,
                        # Muon_AuxAdam.py:76-78, Kourkoutas.py:250-257)
                        if tuple(sh) in kk.keys:
                            aux_i = dict(aux, kourkoutas=kk)
                            if not aux["use_bias_correction"]:
                                aux_i["beta2_dyn"] = kk.beta2[tuple(sh)]
                        elif not aux["use_bias_correction"] and cls == "AdaMuon_adv":
                            aux_i = dict(aux, beta2_dyn=base["betas"][1])
                    ps[i] = O.adam_family_step(ps[i], dt, g, states[i], aux_i, r, algo="auxadam")
                    if i in kk_members:
                        states[i]["kourkoutas_r_ema"] = np.array(kk.ema[tuple(sh)], np.float32)
            elif cls == "Prodigy_adv":
                hp_s = dict(hp, d=group["d"], k=group["k"], beta3=group["beta3"])
                if kk is not None:
                    hp_s.update(beta2_dyn=kk.beta2[tuple(sh)], kourkoutas=kk)
                ps[i], stats = O.adam_family_step(ps[i], dt, g, states[i], hp_s, r, algo="prodigy")
                if kk is not None:
                    states[i]["kourkoutas_r_ema"] = np.array(kk.ema[tuple(sh)], np.float32)
                if stats is not None:
                    d_num = np.float32(d_num + np.float32(stats[0]))
                    d_den = np.float32(d_den + np.float32(stats[1]))
            elif cls == "Lion_adv":
                ps[i] = O.lion_step(ps[i], dt, g, states[i], hp, r)
            yield s, i, ps[i], states[i], group
        if cls == "Prodigy_adv":
            d_num_carry = O.prodigy_calculate_d(group, d_num, d_den)
            yield s, -1, None, None, dict(group)
            if pin_d:
                # continue from the reference's own d so that per-step
                # comparisons do not accumulate d's summation-order error
                ref = z[f"d_{s}"]
                group["d"], group["d_max"], group["d_numerator"] = float(ref[0]), float(ref[1]), float(ref[2])
                d_num_carry = float(np.float32(group["d_numerator"] * group["beta3"]))
