"""AdamW_adv on the GPU against (1) the reference's own outputs recorded in
the golden fixtures, with the reference's random integers injected, and (2)
the oracle at sizes that exercise the fast factored path (d2 >= 2048).

Tolerances (stated per check): int8/uint8 codes and block scales bit-exact;
bf16 params within 1 bf16 ulp; fp32 values within 1e-6 relative (params) /
2e-6 (states; factored row/column factors are sums whose float32 order
differs from the reference's)."""
import math

import numpy as np
import pytest
import torch

from _compare import check_bf16_param, check_fp32, check_state
from _gpu import load_state, to_numpy, to_torch
from _replay import O, list_cases, load, values

pytestmark = pytest.mark.gpu

ADAMW_CASES = [c for c in list_cases() if c.startswith("adamw_")]


def _draws(z, s, i):
    pre = f"r_{s}_{i}_"
    return {k[len(pre):]: torch.from_numpy(z[k].astype(np.int32)).cuda() for k in z.files if k.startswith(pre)}


@pytest.mark.parametrize("name", ADAMW_CASES)
def test_adamw_matches_reference_golden(name):
    import advanced_optimizers_b200 as A
    meta, z = load(name)
    dt = meta["dtype"]
    shapes = [tuple(s) for s in meta["shapes"]]
    params = [torch.nn.Parameter(to_torch(z[f"p0_{i}"], dt).reshape(sh)) for i, sh in enumerate(shapes)]
    opt = A.AdamW_adv(params, **meta["kw"])
    for s in range(meta["steps"]):
        # teacher forcing: start each step from the reference's params and states
        for i, p in enumerate(params):
            if s > 0:
                p.data.copy_(to_torch(z[f"p_{s - 1}_{i}"], dt).reshape(p.shape))
            load_state(opt, p, z, s - 1 if s > 0 else -1, i)
            p.grad = to_torch(z[f"g_{s}_{i}"], dt).reshape(p.shape)
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
            assert opt.state[p]["step"] == int(z[f"st_{s}_{i}_step"])


def _oracle_state_from_torch(st):
    out = {}
    for k, v in st.items():
        out[k] = to_numpy(v) if torch.is_tensor(v) else v
    return out


@pytest.mark.parametrize("case", [
    # (shapes, dtype, kwargs) — effective shapes hit d2 = 2048, 4096, 7168 (fast path) and small d2
    ([(4096, 1024), (2048, 2048), (4096,), (1024, 4096)], "bf16",
     dict(state_precision="int8_sr", factored_2nd=True, nesterov=True)),
    # a factored tensor with d2 < 2048 sends the launch through the general kernel
    ([(4096, 1024), (777, 3), (300, 70)], "bf16", dict(state_precision="int8_sr", factored_2nd=True, nesterov=True)),
    ([(2048, 2048), (96,)], "bf16", dict(state_precision="bf16_sr", factored_2nd=True, weight_decay=0.1,
                                         cautious_wd=True)),
    ([(2048, 2048), (96,)], "bf16", dict(state_precision="auto", nesterov=True, weight_decay=0.01)),
    ([(14336, 4096)], "bf16", dict(state_precision="int8_sr", factored_2nd=True, nesterov=True)),
    ([(1024, 4096), (4096,), (33, 65)], "bf16", dict(state_precision="int8_sr", weight_decay=0.1, lr=1e-2)),
    ([(768, 2304), (2304,), (50257, 64)], "f32",
     dict(state_precision="fp32", weight_decay=0.01)),
    # state_precision='factored': signed rank-1 m on the fast factored layout
    # (d2 = 1024 / 2048 / 4096 -> 2048 and 4096 take the one-byte-per-thread
    # sign path) and on ragged rows (777 x 3 -> (777, 3), 1000 x 7)
    pytest.param(([(4096, 1024), (2048, 2048), (96,), (1024, 4096), (777, 3), (1000, 7)], "bf16",
                  dict(state_precision="factored", nesterov=True, weight_decay=0.01)), id="factored_bf16"),
    pytest.param(([(4096, 4096), (4096,), (333, 12)], "f32",
                  dict(state_precision="factored", cautious_wd=True, weight_decay=0.05)), id="factored_f32"),
    # 'factored' without momentum (betas[0] = 0): rank-1 v only; the
    # reference fails here (its v reconstruction reads a shifter it never made)
    pytest.param(([(2048, 2048), (96,), (333, 12)], "bf16",
                  dict(state_precision="factored", betas=(0.0, 0.99), weight_decay=0.01)), id="factored_no_momentum"),
    # spectral normalisation: one power-iteration step per 2-D update (bf16
    # singular vectors), max-abs scaling of the 1-D update
    pytest.param(([(2048, 1024), (1024,), (512, 1536), (96, 40, 3)], "bf16",
                  dict(state_precision="auto", spectral_normalization=True, weight_decay=0.01, nesterov=True)),
                 id="spectral_bf16"),
    pytest.param(([(4096, 1024), (1024,)], "bf16",
                  dict(state_precision="factored", spectral_normalization=True, cautious_wd=True,
                       weight_decay=0.05)), id="spectral_factored_bf16"),
])
def test_adamw_matches_oracle_large(case):
    import advanced_optimizers_b200 as A
    shapes, dt, kw = case
    g = torch.Generator().manual_seed(0)
    tdt = torch.bfloat16 if dt == "bf16" else torch.float32
    p_host = [(torch.randn(sh, generator=g) * 0.02).to(tdt) for sh in shapes]
    params = [torch.nn.Parameter(t.cuda()) for t in p_host]
    opt = A.AdamW_adv(params, **kw)
    ostate = [_oracle_state_from_torch(opt.state[p]) for p in params]
    hp = dict(lr=1e-3, betas=(0.9, 0.999), eps=1e-8, weight_decay=0.0, nesterov=False, use_bias_correction=True,
              stochastic_rounding=True, precision=kw.get("state_precision", "auto"))
    hp.update({k: v for k, v in kw.items() if k != "state_precision"})
    hp["spectral"] = kw.get("spectral_normalization", False)
    p_o = [to_numpy(t) for t in p_host]
    p_o = [O.from_bf16_bits(x) if dt == "bf16" else x for x in p_o]
    for s in range(2):
        grads = []
        for sh in shapes:
            t = torch.randn(sh, generator=g) * 1e-3
            mask = torch.rand(sh, generator=g) < 0.01
            grads.append(torch.where(mask, t * 100, t).to(tdt))
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
        for i, (p, sh) in enumerate(zip(params, shapes)):
            gnp = to_numpy(grads[i])
            gv = O.from_bf16_bits(gnp).reshape(sh) if dt == "bf16" else gnp
            n = math.prod(sh)
            # int8_sr draws over the padded numel, bf16_sr over the numel (param_update.py:181-264)
            nz = {k: (v.numpy() if (k != "param" and hp["precision"] == "int8_sr") else v.numpy()[:n])
                  for k, v in noise[p].items()}
            prev = p_o[i].copy()
            p_o[i] = O.adam_family_step(p_o[i], dt, gv, ostate[i], hp, nz, algo="adamw")
            what = f"{shapes[i]} step {s}"
            if dt == "bf16":
                check_bf16_param(to_numpy(p), O.bf16_bits(p_o[i]), what)
            else:
                check_fp32(to_numpy(p), p_o[i], 1e-6, what, prev)
            for key, val in opt.state[p].items():
                if torch.is_tensor(val) and key in ostate[i] and isinstance(ostate[i][key], np.ndarray):
                    check_state(key, to_numpy(val), ostate[i][key], f"{what} {key}")
            # keep the oracle on the device's factors so later steps compare one step each
            for key in ("mu_v_nmf", "mv_v_nmf", "mu_m_nmf", "mv_m_nmf", "sign", "spectral_u", "spectral_v"):
                if key in ostate[i]:
                    ostate[i][key] = to_numpy(opt.state[p][key])
            p_o[i] = O.from_bf16_bits(to_numpy(p)).reshape(sh) if dt == "bf16" else to_numpy(p).reshape(sh)


def test_bit_exact_against_oracle_llama_shapes():
    """The Llama-3-8B configuration (int8_sr + factored_2nd + Nesterov, bf16,
    outlier grads) on a q/k/gate-shaped subset plus a norm, two steps,
    injected random integers shared with the oracle: int8 codes, block scales
    and every parameter bit-identical to the oracle (the update's square root
    and divisions are correctly rounded), factors within 2e-6."""
    import advanced_optimizers_b200 as A
    rng = np.random.default_rng(21)
    shapes = [(4096, 4096), (1024, 4096), (14336, 512), (4096,)]
    hp = dict(lr=1e-3, betas=(0.9, 0.999), eps=1e-8, nesterov=True, precision="int8_sr")
    p_np = [O.round_bf16((rng.standard_normal(sh, dtype=np.float32) * 0.02)) for sh in shapes]
    params = [torch.nn.Parameter(torch.from_numpy(v.copy()).cuda().to(torch.bfloat16)) for v in p_np]
    opt = A.AdamW_adv(params, state_precision="int8_sr", factored_2nd=True, nesterov=True)
    states = [O.adamw_init_state(sh, "bf16", "int8_sr", True, 0.9) for sh in shapes]
    for step in range(2):
        noise = []
        for i, sh in enumerate(shapes):
            g = (rng.standard_normal(sh, dtype=np.float32) * 1e-3)
            g = np.where(rng.random(sh) < 0.01, g * 100, g).astype(np.float32)
            g = O.round_bf16(g)
            params[i].grad = torch.from_numpy(g).cuda().to(torch.bfloat16)
            n = int(np.prod(sh))
            pad = ((n + 2047) // 2048) * 2048
            nz = {"exp_avg": rng.integers(0, 65536, pad, dtype=np.int32),
                  "exp_avg_sq": rng.integers(0, 65536, pad, dtype=np.int32),
                  "param": rng.integers(0, 65536, n, dtype=np.int32)}
            noise.append(nz)
            p_np[i] = O.adam_family_step(p_np[i], "bf16", g, states[i], hp, nz, algo="adamw")
        opt.set_test_noise({p: {k: torch.from_numpy(v).cuda() for k, v in nz.items()} for p, nz in zip(params, noise)})
        opt.step()
        torch.cuda.synchronize()
        opt.check_errors()
        for i, sh in enumerate(shapes):
            what = f"step {step} {sh}"
            st = opt.state[params[i]]
            np.testing.assert_array_equal(to_numpy(st["exp_avg"]), states[i]["exp_avg"], err_msg=f"{what}: m codes")
            np.testing.assert_array_equal(to_numpy(st["exp_avg_scale"]), states[i]["exp_avg_scale"],
                                          err_msg=f"{what}: m scales")
            if "mu_v_nmf" in states[i]:
                check_fp32(to_numpy(st["mu_v_nmf"]), states[i]["mu_v_nmf"], 2e-6, f"{what}: mu_v_nmf")
                check_fp32(to_numpy(st["mv_v_nmf"]), states[i]["mv_v_nmf"], 2e-6, f"{what}: mv_v_nmf")
                # the next step starts from the oracle's factors on both sides
                st["mu_v_nmf"].copy_(torch.from_numpy(states[i]["mu_v_nmf"]))
                st["mv_v_nmf"].copy_(torch.from_numpy(states[i]["mv_v_nmf"]))
            else:
                np.testing.assert_array_equal(to_numpy(st["exp_avg_sq"]), states[i]["exp_avg_sq"],
                                              err_msg=f"{what}: v codes")
            mine = to_numpy(params[i]).reshape(-1)
            ref = O.bf16_bits(p_np[i]).reshape(-1)
            nd = int(np.count_nonzero(mine != ref))
            assert nd == 0, f"{what}: {nd} params differ"
            # both sides continue from the oracle's params
            params[i].data.copy_(torch.from_numpy(O.bf16_bits(p_np[i]).view(np.int16)).cuda().view(torch.bfloat16))
