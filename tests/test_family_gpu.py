"""Prodigy_adv and Lion_adv on the GPU against the reference's own outputs
(golden fixtures, the reference's random integers injected).  Every step
starts from the reference's params, states and (Prodigy) group scalars.

Tolerances: bf16 params within 1 bf16 ulp; fp32 params 1e-6 relative to the
larger of the old and new value; bf16-SR'd states within 1 ulp; fp32 states
2e-6; Prodigy's d within 1e-4 relative (it is d_coef * sum<g, p0 - p> /
sum|s|, a cancelling float32 reduction whose order differs)."""
import math

import numpy as np
import pytest
import torch

from _compare import check_bf16_param, check_fp32, check_state
from _gpu import load_state, to_numpy, to_torch
from _replay import list_cases, load

pytestmark = pytest.mark.gpu

CASES = [c for c in list_cases() if c.startswith(("prodigy_", "lion_"))]


def _draws(z, s, i):
    pre = f"r_{s}_{i}_"
    return {k[len(pre):]: torch.from_numpy(z[k].astype(np.int32)).cuda() for k in z.files if k.startswith(pre)}


@pytest.mark.parametrize("name", CASES)
def test_matches_reference_golden(name):
    import advanced_optimizers_b200 as A
    meta, z = load(name)
    dt = meta["dtype"]
    shapes = [tuple(s) for s in meta["shapes"]]
    params = [torch.nn.Parameter(to_torch(z[f"p0_{i}"], dt).reshape(sh)) for i, sh in enumerate(shapes)]
    cls = getattr(A, meta["cls"])
    # keys only a param group carries (Prodigy_adv's spectral_normalization)
    opt = cls([dict(params=params, **meta["group_kw"])] if meta.get("group_kw") else params, **meta["kw"])
    prodigy = meta["cls"] == "Prodigy_adv"
    if prodigy and any(f"st0_{i}_spectral_u" in z.files for i in range(len(shapes))):
        # Prodigy creates its states at the first step; create them now so
        # that the reference's initial singular vectors can be loaded
        for g in opt.param_groups:
            for p in g["params"]:
                opt._init_state(p, g)
    for s in range(meta["steps"]):
        for i, p in enumerate(params):
            if s > 0:
                p.data.copy_(to_torch(z[f"p_{s - 1}_{i}"], dt).reshape(p.shape))
            if s == 0 and prodigy:
                # Prodigy creates its states at the first step: step once the
                # init path only when states exist
                pass
            if opt.state.get(p):
                load_state(opt, p, z, s - 1 if s > 0 else -1, i)
            p.grad = to_torch(z[f"g_{s}_{i}"], dt).reshape(p.shape)
        if prodigy and s > 0:
            ref = z[f"d_{s - 1}"]
            for g in opt.param_groups:
                g["d"], g["d_max"], g["d_numerator"] = float(ref[0]), float(ref[1]), float(ref[2])
            opt._set_carry(float(np.float32(float(ref[2]) * opt.beta3)))
        opt.set_test_noise({p: _draws(z, s, i) for i, p in enumerate(params)})
        opt.step()
        torch.cuda.synchronize()
        for i, p in enumerate(params):
            what = f"{name} step {s} param {i}"
            ref_p = z[f"p_{s}_{i}"]
            if dt == "bf16":
                check_bf16_param(to_numpy(p), ref_p, what)
            else:
                prev = z[f"p_{s - 1}_{i}"] if s > 0 else z[f"p0_{i}"]
                check_fp32(to_numpy(p), ref_p, 1e-6, what, prev)
            for key, val in opt.state[p].items():
                rk = f"st_{s}_{i}_{key}"
                if torch.is_tensor(val) and rk in z.files:
                    pk = f"st_{s - 1}_{i}_{key}" if s > 0 else f"st0_{i}_{key}"
                    prev = z[pk] if pk in z.files and z[pk].shape == z[rk].shape else None
                    check_state(key, to_numpy(val), z[rk], f"{what} {key}", prev)
        if prodigy:
            ref = z[f"d_{s}"]
            g0 = opt.param_groups[0]
            assert g0["k"] == int(ref[3])
            for j, key in enumerate(("d", "d_max", "d_numerator")):
                np.testing.assert_allclose(g0[key], ref[j], rtol=1e-4, err_msg=f"{name} step {s} {key}")


@pytest.mark.parametrize("dt", ["bf16", "f32"])
def test_lion_factored_matches_oracle_large(dt):
    """Lion_adv(nnmf_factor=True) at sizes that take the one-sign-byte-per-thread
    path (effective d2 = 2048, 4096) beside ragged rows ((777, 3) -> (63, 37))
    and a 1-D param, against the oracle; each step starts from the device's
    factors.  Tolerances as above (factors 2e-6, signs exact)."""
    import advanced_optimizers_b200 as A
    from _replay import O
    shapes = [(4096, 1024), (2048, 2048), (96,), (777, 3)]
    g = torch.Generator().manual_seed(3)
    tdt = torch.bfloat16 if dt == "bf16" else torch.float32
    p_host = [(torch.randn(sh, generator=g) * 0.02).to(tdt) for sh in shapes]
    params = [torch.nn.Parameter(t.cuda()) for t in p_host]
    kw = dict(lr=1e-4, weight_decay=0.01, nnmf_factor=True, cautious_wd=(dt == "f32"))
    opt = A.Lion_adv(params, **kw)
    hp = dict(lr=1e-4, betas=(0.9, 0.99), weight_decay=0.01, cautious_wd=kw["cautious_wd"], stochastic_rounding=True)
    ostate = [{k: (to_numpy(v) if torch.is_tensor(v) else v) for k, v in opt.state[p].items()} for p in params]
    p_o = [O.from_bf16_bits(to_numpy(t)) if dt == "bf16" else to_numpy(t) for t in p_host]
    for s in range(2):
        grads = [(torch.randn(sh, generator=g) * 1e-3).to(tdt) for sh in shapes]
        noise = {p: {"param": torch.randint(0, 65536, (math.prod(sh),), generator=g, dtype=torch.int32)}
                 for p, sh in zip(params, shapes)}
        for p, gr in zip(params, grads):
            p.grad = gr.cuda()
        opt.set_test_noise({p: {k: v.cuda() for k, v in nz.items()} for p, nz in noise.items()})
        opt.step()
        torch.cuda.synchronize()
        for i, (p, sh) in enumerate(zip(params, shapes)):
            gnp = to_numpy(grads[i])
            gv = O.from_bf16_bits(gnp).reshape(sh) if dt == "bf16" else gnp
            prev = p_o[i].copy()
            p_o[i] = O.lion_step(p_o[i], dt, gv, ostate[i], hp, {"param": noise[p]["param"].numpy()})
            what = f"{sh} step {s}"
            if dt == "bf16":
                check_bf16_param(to_numpy(p), O.bf16_bits(p_o[i]), what)
            else:
                check_fp32(to_numpy(p), p_o[i], 1e-6, what, prev)
            for key, val in opt.state[p].items():
                if torch.is_tensor(val) and isinstance(ostate[i].get(key), np.ndarray):
                    check_state(key, to_numpy(val), ostate[i][key], f"{what} {key}")
            for key in ("mu_m_nmf", "mv_m_nmf", "sign", "exp_avg"):
                if key in ostate[i]:
                    ostate[i][key] = to_numpy(opt.state[p][key])
            p_o[i] = O.from_bf16_bits(to_numpy(p)).reshape(sh) if dt == "bf16" else to_numpy(p).reshape(sh)


@pytest.mark.parametrize("which", ["prodigy", "auxadam"])
def test_factored_fast_layout_matches_oracle(which):
    """state_precision='factored' at sizes whose effective rows take the fast
    kernel's factored-momentum variant (d2 = 1024 / 2048 -> fast layout for
    (4096, 1024) as (2048, 2048), (2048, 2048)), beside a 1-D param, for
    Prodigy_adv (slice statistics and the d estimate on top) and Muon_adv's
    auxiliary Adam, one step against the oracle.  Tolerances: params within 1
    bf16 ulp; sign bits exact; rank-1 factors 2e-6 relative; Prodigy's s bf16
    within 1 ulp and d within 1e-4 relative."""
    import advanced_optimizers_b200 as A
    from _replay import O, PRODIGY_DEFAULTS
    shapes = [(4096, 1024), (2048, 2048), (96,)]
    g = torch.Generator().manual_seed(11)
    p_host = [(torch.randn(sh, generator=g) * 0.02).bfloat16() for sh in shapes]
    params = [torch.nn.Parameter(t.cuda()) for t in p_host]
    if which == "prodigy":
        kw = dict(state_precision="factored", d0=1e-4, slice_p=11, nesterov=True, weight_decay=0.01)
        opt = A.Prodigy_adv(params, **kw)
        for p in params:
            opt._init_state(p, opt.param_groups[0])
        hp = dict(PRODIGY_DEFAULTS)
        hp.update(kw)
        hp["betas"] = tuple(hp["betas"])
        hp["precision"] = "factored"
        beta3 = math.sqrt(hp["betas"][1])
        group = dict(d=1e-4, d0=1e-4, d_max=1e-4, d_numerator=0.0, d_coef=1.0, growth_rate=float("inf"),
                     d_limiter=False, k=0, prodigy_steps=0, beta3=beta3)
        hp = dict(hp, d=group["d"], k=0, beta3=beta3)
        algo = "prodigy"
    else:
        kw = dict(lr=1e-3, adam_state_precision="factored", adam_nesterov=True, adam_weight_decay=0.01)
        opt = A.Muon_adv([dict(params=params, optim_type="adam")], **kw)
        hp = dict(lr=1e-3, betas=(0.9, 0.99), eps=1e-8, weight_decay=0.01, use_bias_correction=True,
                  stochastic_rounding=True, nesterov=True, precision="factored")
        algo = "auxadam"
    ostate = [{k: (to_numpy(v) if torch.is_tensor(v) else v) for k, v in opt.state[p].items()} for p in params]
    grads = [(torch.randn(sh, generator=g) * 1e-3).bfloat16() for sh in shapes]
    noise = {p: {"param": torch.randint(0, 65536, (math.prod(sh),), generator=g, dtype=torch.int32)}
             for p, sh in zip(params, shapes)}
    for p, gr in zip(params, grads):
        p.grad = gr.cuda()
    opt.set_test_noise({p: {k: v.cuda() for k, v in nz.items()} for p, nz in noise.items()})
    opt.step()
    torch.cuda.synchronize()
    d_num, d_den = np.float32(0.0), np.float32(0.0)
    from _replay import O as _O
    for i, (p, sh) in enumerate(zip(params, shapes)):
        gv = _O.from_bf16_bits(to_numpy(grads[i])).reshape(sh)
        pv = _O.from_bf16_bits(to_numpy(p_host[i])).reshape(sh)
        out = _O.adam_family_step(pv, "bf16", gv, ostate[i], hp, {"param": noise[p]["param"].numpy()}, algo=algo)
        if algo == "prodigy":
            out, stats = out
            d_num = np.float32(d_num + np.float32(stats[0]))
            d_den = np.float32(d_den + np.float32(stats[1]))
        what = f"{which} {sh}"
        check_bf16_param(to_numpy(p), _O.bf16_bits(out), what)
        for key, val in opt.state[p].items():
            if torch.is_tensor(val) and isinstance(ostate[i].get(key), np.ndarray):
                check_state(key, to_numpy(val), ostate[i][key], f"{what} {key}")
    if algo == "prodigy":
        _O.prodigy_calculate_d(group, d_num, d_den)
        np.testing.assert_allclose(opt.param_groups[0]["d"], group["d"], rtol=1e-4, err_msg="prodigy d")
