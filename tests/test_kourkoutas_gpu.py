"""Kourkoutas-beta (Kourkoutas.py) on the GPU against the oracle at sizes
that take the fast kernel: layer-wise dynamic beta2 from the previous step's
pooled grad norm, computed and applied on the device.

The per-layer sum of g*g is summed in another order than torch.sum (per
piece in float64 here), so the pooled norm, the EMA and beta2 agree with the
oracle to a few float32 ulps rather than bit for bit; params are compared at
the tolerances of the other AdamW parity tests (bf16: at most one ulp on a
few elements; fp32 within 1e-6 relative), EMA and beta2 within 2e-6 relative.
"""
import math

import numpy as np
import pytest
import torch

import oracle.oracle as O
from _compare import check_bf16_param, check_fp32, check_state
from _gpu import to_numpy

pytestmark = pytest.mark.gpu

CASES = [
    # bf16 'auto': v in bf16, the squares summed from bf16-rounded g*g
    ([(2048, 2048), (2048, 2048), (96,)], "bf16",
     dict(state_precision="auto", nesterov=True, weight_decay=0.01)),
    # the Llama configuration's storage: int8_sr codes, factored v
    ([(4096, 1024), (4096, 1024), (1024,), (1024,)], "bf16",
     dict(state_precision="int8_sr", factored_2nd=True, nesterov=True)),
    ([(768, 2304), (2304,), (768, 2304)], "f32", dict(state_precision="fp32", weight_decay=0.01)),
]


@pytest.mark.parametrize("case", CASES)
def test_kourkoutas_matches_oracle(case):
    import advanced_optimizers_b200 as A
    shapes, dt, kw = case
    kw = dict(kw, kourkoutas_beta=True, beta2_min=0.88, ema_alpha=0.9, k_warmup_steps=2)
    g = torch.Generator().manual_seed(5)
    tdt = torch.bfloat16 if dt == "bf16" else torch.float32
    p_host = [(torch.randn(sh, generator=g) * 0.02).to(tdt) for sh in shapes]
    params = [torch.nn.Parameter(t.cuda()) for t in p_host]
    opt = A.AdamW_adv(params, **kw)
    ostate = [{k: (to_numpy(v) if torch.is_tensor(v) else v) for k, v in opt.state[p].items()} for p in params]
    hp = dict(lr=1e-3, betas=(0.9, 0.999), eps=1e-8, weight_decay=0.0, nesterov=False, use_bias_correction=True,
              stochastic_rounding=True, precision=kw["state_precision"])
    hp.update({k: v for k, v in kw.items() if k not in ("state_precision", "kourkoutas_beta", "beta2_min",
                                                      "ema_alpha", "k_warmup_steps")})
    kk = O.Kourkoutas(shapes, 0.999, 0.88, 0.9, 1e-9, 2)
    p_o = [to_numpy(t) for t in p_host]
    p_o = [O.from_bf16_bits(x) if dt == "bf16" else x for x in p_o]
    for s in range(4):
        # the grad scale changes between steps so that beta2 moves
        scale = [1e-3, 3e-3, 5e-4, 2e-3][s]
        grads = [(torch.randn(sh, generator=g) * scale).to(tdt) for sh in shapes]
        noise = {}
        for p, sh in zip(params, shapes):
            n = math.prod(sh)
            pad = ((n + 2047) // 2048) * 2048
            noise[p] = {"exp_avg": torch.randint(0, 65536, (pad,), generator=g, dtype=torch.int32),
                        "exp_avg_sq": torch.randint(0, 65536, (pad,), generator=g, dtype=torch.int32),
                        "param": torch.randint(0, 65536, (n,), generator=g, dtype=torch.int32)}
        for p, gr in zip(params, grads):
            p.grad = gr.cuda()
        opt.set_test_noise({p: {k: v.cuda() for k, v in nz.items()} for p, nz in noise.items()})
        opt.step()
        torch.cuda.synchronize()
        opt.check_errors()
        kk.prepare(s)
        for i, (p, sh) in enumerate(zip(params, shapes)):
            gnp = to_numpy(grads[i])
            gv = O.from_bf16_bits(gnp).reshape(sh) if dt == "bf16" else gnp
            n = math.prod(sh)
            nz = {k: (v.numpy() if (k != "param" and hp["precision"] == "int8_sr") else v.numpy()[:n])
                  for k, v in noise[p].items()}
            prev = p_o[i].copy()
            hp_i = dict(hp, beta2_dyn=kk.beta2[tuple(sh)], kourkoutas=kk)
            p_o[i] = O.adam_family_step(p_o[i], dt, gv, ostate[i], hp_i, nz, algo="adamw")
            what = f"{shapes[i]} step {s}"
            b2 = opt.kourkoutas_helper.dynamic_beta2(p)
            assert abs(b2 - kk.beta2[tuple(sh)]) <= 2e-6 * kk.beta2[tuple(sh)], (what, b2, kk.beta2[tuple(sh)])
            ema = float(opt.state[p]["kourkoutas_r_ema"])
            assert abs(ema - float(kk.ema[tuple(sh)])) <= 2e-6 * abs(float(kk.ema[tuple(sh)])) + 1e-30, (what, ema)
            if dt == "bf16":
                check_bf16_param(to_numpy(p), O.bf16_bits(p_o[i]), what)
            else:
                check_fp32(to_numpy(p), p_o[i], 1e-6, what, prev)
            for key, val in opt.state[p].items():
                if torch.is_tensor(val) and key in ostate[i] and isinstance(ostate[i][key], np.ndarray) \
                        and key != "kourkoutas_r_ema":
                    check_state(key, to_numpy(val), ostate[i][key], f"{what} {key}")
            # keep the oracle on the device's params and factors: each step compares one step
            for key in ("mu_v_nmf", "mv_v_nmf"):
                if key in ostate[i]:
                    ostate[i][key] = to_numpy(opt.state[p][key])
            p_o[i] = O.from_bf16_bits(to_numpy(p)).reshape(sh) if dt == "bf16" else to_numpy(p).reshape(sh)
        # the device EMA drives the next step: keep the oracle on it as well
        for p, sh in zip(params, shapes):
            kk.ema[tuple(sh)] = np.float32(float(opt.state[p]["kourkoutas_r_ema"]))
    stats = opt.kourkoutas_helper.last_beta2_stats
    assert 0.88 <= stats["mean"] <= 0.999


def test_kourkoutas_state_dict_round_trip():
    """kourkoutas_r_ema is saved under the reference's key, shared by every
    param of a layer, and a loaded value drives the next step."""
    import advanced_optimizers_b200 as A
    torch.manual_seed(0)
    shapes = [(256, 64), (256, 64), (64,)]
    mk = lambda: [torch.nn.Parameter(torch.randn(sh, device="cuda") * 0.02) for sh in shapes]
    pa, pb = mk(), mk()
    for x, y in zip(pa, pb):
        y.data.copy_(x.data)
    kw = dict(state_precision="fp32", kourkoutas_beta=True, beta2_min=0.9)
    oa = A.AdamW_adv(pa, **kw)
    for s in range(3):
        for p in pa:
            p.grad = torch.randn_like(p) * (1e-3 * (s + 1))
        oa.step()
    sd = oa.state_dict()
    assert all("kourkoutas_r_ema" in sd["state"][i] for i in range(3))
    assert oa.state[pa[0]]["kourkoutas_r_ema"].data_ptr() == oa.state[pa[1]]["kourkoutas_r_ema"].data_ptr()
    ob = A.AdamW_adv(pb, **kw)
    for x, y in zip(pa, pb):
        y.data.copy_(x.data)
    ob.load_state_dict(sd)
    # the accumulator of the last step is not part of the state: run both
    # from one more step whose pooled norm starts from zero on both sides
    grads = [torch.randn_like(p) * 2e-3 for p in pa]
    for opt, ps in ((oa, pa), (ob, pb)):
        if opt.kourkoutas_helper.acc is not None:
            opt.kourkoutas_helper.acc.zero_()
        for p, gr in zip(ps, grads):
            p.grad = gr.clone()
        opt.step()
    torch.cuda.synchronize()
    for x, y in zip(pa, pb):
        assert torch.equal(x, y)
    for i in range(3):
        assert torch.equal(oa.state[pa[i]]["kourkoutas_r_ema"], ob.state[pb[i]]["kourkoutas_r_ema"])
