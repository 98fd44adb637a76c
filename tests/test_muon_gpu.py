"""Muon_adv / AdaMuon_adv and the Newton–Schulz chain on the GPU.

Against the reference's own outputs (golden fixtures, its random integers
injected, teacher forcing: every step starts from the reference's params
and states) and against the oracle at larger, ragged and transposed shapes.

Tolerances:
  * momentum_buffer (codes, block scales, bf16 values): bit-exact — it is
    computed before the Newton–Schulz chain;
  * params on the Muon path: within 2 bf16 ulps (fp32: 1e-6) of the larger
    of the old and new value plus 10% of the update's RMS, and the update
    within 3% (AdaMuon 5%) in the Frobenius norm — the bf16 GEMM chain rounds
    in a different accumulation order than the reference's CPU addmm and
    rounding flips propagate through the iterations; AdaMuon may have up to
    5e-4 of its elements outside the band (see check_ns_param);
  * AdaMuon second_momentum_buffer (after the chain): uint8 codes within 16
    and on average within 0.5, scales 5e-2 relative;
  * auxiliary Adam params: 1 bf16 ulp; their states as in the AdamW tests;
  * newton_schulz output: within 2 bf16 ulps + 10% of its RMS elementwise,
    and 2% relative in the Frobenius norm (five quintic iterations amplify
    a rounding difference in the smallest singular directions up to
    3.4445^5 ~ 480 times, so single elements move more than the whole).
"""
import math

import numpy as np
import pytest
import torch

from _compare import check_bf16_param, check_fp32, check_state
from _gpu import load_state, to_numpy, to_torch
from _replay import O, list_cases, load, route_kinds

pytestmark = pytest.mark.gpu

CASES = [c for c in list_cases() if c.startswith(("muon_", "adamuon_"))]
QUINTIC = (3.4445, -4.7750, 2.0315)


def _draws(z, s, i):
    pre = f"r_{s}_{i}_"
    out = {k[len(pre):]: torch.from_numpy(z[k].astype(np.int32)).cuda() for k in z.files if k.startswith(pre)}
    if f"sk_{s}_{i}" in z.files:
        # the low-rank chain's Gaussian sketch (bf16 bits)
        out["sketch"] = torch.from_numpy(z[f"sk_{s}_{i}"].view(np.int16).copy()).view(torch.bfloat16).cuda()
    return out


def check_ns_param(mine, ref, old, dt, what, adamuon=False, allowed_frac=None):
    """Params after a Newton–Schulz step (values as float arrays): within 2
    bf16 ulps (bf16) or 1e-6 (fp32) of the larger of the old and new value
    plus 10% of the update's RMS.  AdaMuon divides by sqrt(v), which at small
    v turns the update into a sign: where the chain's output is near zero a
    rounding difference flips an element by twice the update, so up to 5e-4
    of its elements may sit outside the band (Muon: 1e-5)."""
    a = np.asarray(mine, np.float64).reshape(-1)
    b = np.asarray(ref, np.float64).reshape(-1)
    o = np.asarray(old, np.float64).reshape(-1)
    scale = np.maximum(np.abs(b), np.abs(o))
    upd = b - o
    u_rms = np.sqrt(np.mean(upd ** 2))
    ulp = 2.0 ** -6 if dt == "bf16" else 1e-6
    bad = np.count_nonzero(np.abs(a - b) > ulp * scale + 0.1 * u_rms)
    if allowed_frac is None:
        allowed_frac = 5e-4 if adamuon else 1e-5
    allowed = math.ceil(allowed_frac * a.size)
    # one ulp of the param is rounding slack (an update smaller than the
    # param's ulp moves it by whole ulps under stochastic rounding)
    excess = np.maximum(np.abs(a - b) - 0.5 * ulp * scale, 0.0)
    frob = np.linalg.norm(excess) / max(np.linalg.norm(upd), 1e-30)
    stats = f"{bad}/{a.size} outside 2 ulps + 10% of the update RMS, update Frobenius relative {frob:.3g}"
    assert bad <= allowed, f"{what}: {stats}"
    assert frob < (0.05 if adamuon else 0.03), f"{what}: {stats}"


def check_second_moment(key, val, ref, what):
    """AdaMuon's v after the chain: uint8 codes within 16 and on average
    within 0.5; block scales 5e-2 relative; float states compared through
    sqrt(v) (proportional to |U|) like the chain's output: 2 bf16 ulps + 10%
    of its RMS, at most 5e-4 of the elements outside, 3% in the Frobenius norm."""
    if val.dtype == np.uint8:
        dq = np.abs(val.astype(np.int32) - ref.astype(np.int32))
        assert dq.max() <= 16 and dq.mean() < 0.5, f"{what}: codes max {dq.max()} mean {dq.mean():.3f}"
        return
    if key.endswith("_scale"):
        check_fp32(val, ref, 5e-2, what)
        return
    if val.dtype == np.uint16:
        val, ref = O.from_bf16_bits(val), O.from_bf16_bits(ref)
    sa = np.sqrt(np.asarray(val, np.float64).reshape(-1))
    sb = np.sqrt(np.asarray(ref, np.float64).reshape(-1))
    rms = np.sqrt(np.mean(sb ** 2))
    d = np.abs(sa - sb)
    bad = np.count_nonzero(d > 2.0 ** -6 * sb + 0.1 * rms)
    frob = np.linalg.norm(sa - sb) / max(np.linalg.norm(sb), 1e-30)
    assert bad <= math.ceil(5e-4 * sa.size) and frob < 0.03, f"{what}: {bad}/{sa.size} outside, Frobenius {frob:.3g}"


@pytest.mark.parametrize("name", CASES)
def test_matches_reference_golden(name):
    import advanced_optimizers_b200 as A
    meta, z = load(name)
    dt = meta["dtype"]
    shapes = [tuple(s) for s in meta["shapes"]]
    params = [torch.nn.Parameter(to_torch(z[f"p0_{i}"], dt).reshape(sh)) for i, sh in enumerate(shapes)]
    groups, k = [], 0
    for g in meta["groups"]:
        grp = dict(params=params[k:k + g["n"]])
        if g["optim_type"] is not None:
            grp["optim_type"] = g["optim_type"]
        groups.append(grp)
        k += g["n"]
    kinds = route_kinds(meta)
    opt = getattr(A, meta["cls"])(groups, **meta["kw"])
    for i, p in enumerate(params):
        if f"route_{i}" in z.files:
            # routing by _is_suitable_for_muon where the group names no optim_type
            assert bool(opt.state[p]["is_muon"]) == bool(z[f"route_{i}"]), f"{name} param {i}: routing"
    for s in range(meta["steps"]):
        for i, p in enumerate(params):
            if s > 0:
                p.data.copy_(to_torch(z[f"p_{s - 1}_{i}"], dt).reshape(p.shape))
            load_state(opt, p, z, s - 1 if s > 0 else -1, i)
            p.grad = to_torch(z[f"g_{s}_{i}"], dt).reshape(p.shape)
        opt.set_test_noise({p: _draws(z, s, i) for i, p in enumerate(params)})
        opt.step()
        torch.cuda.synchronize()
        opt.check_errors()
        for i, p in enumerate(params):
            what = f"{name} step {s} param {i}"
            ref_p = z[f"p_{s}_{i}"]
            old = z[f"p_{s - 1}_{i}"] if s > 0 else z[f"p0_{i}"]
            muon = kinds[i] == "muon"
            if muon:
                vals = (lambda x: O.from_bf16_bits(x)) if dt == "bf16" else (lambda x: x)
                check_ns_param(vals(to_numpy(p)), vals(ref_p), vals(old), dt, what, meta["cls"] == "AdaMuon_adv")
            elif dt == "bf16":
                check_bf16_param(to_numpy(p), ref_p, what)
            else:
                check_fp32(to_numpy(p), ref_p, 1e-6, what, old)
            for key, val in opt.state[p].items():
                rk = f"st_{s}_{i}_{key}"
                if not (torch.is_tensor(val) and rk in z.files):
                    continue
                if muon and key.startswith(("second_momentum_buffer", "normuon_v", "mu_vbuf_nmf", "mv_vbuf_nmf")):
                    # statistics of the chain's output
                    check_second_moment(key, to_numpy(val), z[rk], f"{what} {key}")
                else:
                    pk = f"st_{s - 1}_{i}_{key}" if s > 0 else f"st0_{i}_{key}"
                    prev = z[pk] if pk in z.files and z[pk].shape == z[rk].shape else None
                    check_state(key, to_numpy(val), z[rk], f"{what} {key}", prev)


def _check_ns_output(mine, ref, what):
    a = mine.astype(np.float64).reshape(-1)
    b = ref.astype(np.float64).reshape(-1)
    rms = np.sqrt(np.mean(b ** 2))
    d = np.abs(a - b)
    rel = np.linalg.norm(a - b) / np.linalg.norm(b)
    stats = f"max |d|/rms {d.max() / rms:.3g}, Frobenius relative {rel:.3g}"
    bad = np.count_nonzero(d > 2.0 ** -6 * np.abs(b) + 0.1 * rms)
    assert bad == 0, f"{what}: {bad}/{a.size} beyond 2 bf16 ulps + 10% of the RMS ({stats})"
    assert rel < 2e-2, f"{what}: {stats}"


@pytest.mark.parametrize("shape,cns,dtype", [
    ((256, 512), False, "f32"), ((1024, 384), False, "bf16"), ((300, 700), True, "f32"),
    ((640, 128), True, "bf16"), ((48, 64), False, "bf16"), ((512, 512), False, "f32"),
])
def test_newton_schulz_matches_oracle(shape, cns, dtype):
    import advanced_optimizers_b200 as A
    rng = np.random.default_rng(7)
    g = (rng.standard_normal(shape) * 0.01).astype(np.float32)
    if dtype == "bf16":
        g = O.round_bf16(g)
    G = torch.from_numpy(g).cuda()
    if dtype == "bf16":
        G = G.to(torch.bfloat16)
    mine = A.newton_schulz(G, steps=5, eps=1e-7, coeffs=QUINTIC, cns=cns)
    torch.cuda.synchronize()
    assert mine.dtype == G.dtype and mine.shape == G.shape
    ref = O.newton_schulz(O.T(g, dtype), 5, 1e-7, QUINTIC, cns, None).v
    _check_ns_output(mine.float().cpu().numpy(), ref, f"NS {shape} cns={cns}")


@pytest.mark.parametrize("shape,cns", [
    ((1024, 4096), False), ((1024, 4096), True),      # k/v projections: m = 1024, 4 x 4 blocks of 256
    ((4096, 4096), False), ((4096, 4096), True),      # q/o projections: m = 4096, 16 x 16 blocks
    ((14336, 4096), False),                           # gate/up: transposed into the workspace
    ((4096, 14336), False),                           # down
])
def test_newton_schulz_matches_oracle_at_llama_shapes(shape, cns):
    """The whole chain at the Llama-3-8B matrix shapes, where the symmetric
    products run on the production tilings (upper blocks computed, lower
    blocks mirrored), against the oracle's chain (each GEMM in float32,
    rounded to bf16), with the tolerance of the smaller shapes above."""
    import advanced_optimizers_b200 as A
    rng = np.random.default_rng(shape[0] + 3 * shape[1] + int(cns))
    g = O.round_bf16((rng.standard_normal(shape, dtype=np.float32) * 1e-3).astype(np.float32))
    G = torch.from_numpy(g).cuda().to(torch.bfloat16)
    mine = A.newton_schulz(G, steps=5, eps=1e-7, coeffs=QUINTIC, cns=cns)
    torch.cuda.synchronize()
    assert mine.dtype == G.dtype and mine.shape == G.shape
    ref = O.newton_schulz(O.T(g, "bf16"), 5, 1e-7, QUINTIC, cns, None).v
    _check_ns_output(mine.float().cpu().numpy(), ref, f"NS {shape} cns={cns}")


def test_newton_schulz_orthogonalises_llama_shape():
    """Size-independent property at a Llama-3-8B k/v projection shape
    (1024 x 4096): the quintic iteration drives every singular value into
    roughly [0.6, 1.25] (the polynomial's fixed band), whatever the input."""
    import advanced_optimizers_b200 as A
    gen = torch.Generator(device="cuda").manual_seed(3)
    G = (torch.randn(4096, 1024, device="cuda", generator=gen) * 1e-3).to(torch.bfloat16)
    U = A.newton_schulz(G)
    sv = torch.linalg.svdvals(U.float())
    assert sv.min().item() > 0.5 and sv.max().item() < 1.3, (sv.min().item(), sv.max().item())
    # CANS with the default bound: the same band property
    U2 = A.newton_schulz(G, cns=True)
    sv2 = torch.linalg.svdvals(U2.float())
    assert sv2.min().item() > 0.5 and sv2.max().item() < 1.5, (sv2.min().item(), sv2.max().item())


def _oracle_hp(adamuon, **kw):
    hp = dict(lr=2e-3, beta1=0.95, betas=(0.95, 0.95), eps=1e-8, weight_decay=0.0, cautious_wd=False,
              nesterov=True, nesterov_coef=None, ns_steps=5, ns_eps=1e-7, ns_coeffs=QUINTIC,
              stochastic_rounding=True, rms_rescaling=True, precision="auto", accelerated_ns=False,
              cns_a_bound=None, centered_wd=0.0, kappa_p=1.0, auto_projection=True, use_atan2=False)
    hp.update(kw)
    return hp


@pytest.mark.parametrize("adamuon,dt,prec,extra", [
    (False, "bf16", "int8_sr", dict(weight_decay=0.01, cautious_wd=True)),
    (False, "bf16", "auto", dict(nesterov=False, rms_rescaling=False)),
    (False, "f32", "bf16_sr", dict(weight_decay=0.1)),
    (False, "bf16", "bf16_sr", dict(weight_decay=0.01)),
    (False, "bf16", "fp32", dict(nesterov=False)),
    (True, "bf16", "int8_sr", dict(accelerated_ns=True)),
    (True, "bf16", "auto", dict(use_atan2=True)),
    (True, "f32", "fp32", dict(weight_decay=0.01, rms_rescaling=False)),
])
def test_matches_oracle_larger_shapes(adamuon, dt, prec, extra):
    """Ragged (300 x 700), transposed (1536 x 512) and wide (512 x 1536)
    matrices, two steps, injected noise shared with the oracle."""
    import advanced_optimizers_b200 as A
    rng = np.random.default_rng(11)
    shapes = [(300, 700), (1536, 512), (512, 1536)]
    hp = _oracle_hp(adamuon, precision=prec, **extra)
    ps0 = []
    for sh in shapes:
        v = (rng.standard_normal(sh) * 0.02).astype(np.float32)
        ps0.append(O.round_bf16(v) if dt == "bf16" else v)
    params = [torch.nn.Parameter(torch.from_numpy(v.copy()).cuda().to(torch.bfloat16 if dt == "bf16" else torch.float32))
              for v in ps0]
    kw = dict(lr=hp["lr"], weight_decay=hp["weight_decay"], cautious_wd=hp["cautious_wd"], nesterov=hp["nesterov"],
              rms_rescaling=hp["rms_rescaling"], state_precision=prec, accelerated_ns=hp["accelerated_ns"])
    if adamuon:
        opt = A.AdaMuon_adv([dict(params=params, optim_type="muon")], betas=hp["betas"], use_atan2=hp["use_atan2"],
                            **kw)
    else:
        opt = A.Muon_adv([dict(params=params, optim_type="muon")], beta1=hp["beta1"], **kw)
    states = []
    for sh in shapes:
        st = {}
        O.init_state_tensor(st, "momentum_buffer", sh, prec, dt)
        if adamuon:
            O.init_state_tensor(st, "second_momentum_buffer", sh, prec, dt, non_neg=True)
        states.append(st)
    cur = [v.copy() for v in ps0]
    for s in range(2):
        noise = []
        for i, (p, sh) in enumerate(zip(params, shapes)):
            n = int(np.prod(sh))
            pad = (n + 2047) // 2048 * 2048 if prec == "int8_sr" else n
            nz = {"momentum_buffer": rng.integers(0, 1 << 16, pad, dtype=np.int32),
                  "param": rng.integers(0, 1 << 16, n, dtype=np.int32)}
            if adamuon:
                nz["second_momentum_buffer"] = rng.integers(0, 1 << 16, pad, dtype=np.int32)
            noise.append(nz)
            g = (rng.standard_normal(sh) * 1e-3).astype(np.float32)
            g = O.round_bf16(g) if dt == "bf16" else g
            p.grad = torch.from_numpy(g.copy()).cuda().to(p.dtype)
            step_fn = O.adamuon_step if adamuon else O.muon_step
            # teacher forcing: the oracle steps from the GPU's params and states
            p_before = p.detach().float().cpu().numpy()
            st_np = {k: to_numpy(v) for k, v in opt.state[p].items() if torch.is_tensor(v)} if s > 0 else states[i]
            cur[i] = step_fn(p_before, dt, g, st_np, hp, nz)
            states[i] = st_np
        opt.set_test_noise({p: {k: torch.from_numpy(v).cuda() for k, v in noise[i].items()}
                            for i, p in enumerate(params)})
        old = [p.detach().float().cpu().numpy() for p in params]
        opt.step()
        torch.cuda.synchronize()
        opt.check_errors()
        for i, p in enumerate(params):
            what = f"step {s} {shapes[i]}"
            mine = p.detach().float().cpu().numpy()
            check_ns_param(mine, cur[i], old[i], dt, what, adamuon)
            for key, val in opt.state[p].items():
                if not torch.is_tensor(val) or key not in states[i]:
                    continue
                if key.startswith("second_momentum_buffer"):
                    check_second_moment(key, to_numpy(val), np.asarray(states[i][key]), f"{what} {key}")
                else:
                    check_state(key, to_numpy(val), np.asarray(states[i][key]), f"{what} {key}")


def test_philox_mode_runs_and_is_deterministic():
    """Without injected noise the step draws Philox bits: two optimizers
    from identical inputs produce identical results, and the int8 momentum
    dequantises to within one block step of the fp32 momentum."""
    import advanced_optimizers_b200 as A
    torch.manual_seed(0)
    p0 = (torch.randn(768, 2304) * 0.02).to(torch.bfloat16).cuda()
    g = (torch.randn(768, 2304) * 1e-3).to(torch.bfloat16).cuda()
    outs = []
    for _ in range(2):
        p = torch.nn.Parameter(p0.clone())
        opt = A.Muon_adv([dict(params=[p], optim_type="muon")], state_precision="int8_sr")
        p.grad = g.clone()
        opt.step()
        torch.cuda.synchronize()
        outs.append((p.detach().clone(), opt.state[p]["momentum_buffer"].clone(),
                     opt.state[p]["momentum_buffer_scale"].clone()))
    assert torch.equal(outs[0][0], outs[1][0]) and torch.equal(outs[0][1], outs[1][1])
    m_true = 0.05 * g.float().reshape(-1)
    sc = outs[0][2].repeat_interleave(2048)[: m_true.numel()]
    deq = outs[0][1].float().reshape(-1) * sc
    assert torch.all((deq - m_true).abs() <= sc * 1.0001 + 1e-12)
    assert not torch.equal(outs[0][0], p0)


@pytest.mark.parametrize("adamuon", [False, True])
def test_low_rank_with_device_sketch_matches_oracle(adamuon):
    """Low-rank Newton-Schulz (ortho_rank 64) without injected noise: the
    device draws its Gaussian sketch from Philox (advopt_lr_sketch, read back
    here for the oracle), takes the QR by shifted CholeskyQR3 and runs the
    chain on the [64][cols] projection; params within the chain's tolerance
    of the oracle (which takes numpy's Householder QR) on a tall, a wide and
    a ragged matrix.  The sketch itself is N(0, 1) to within sampling error."""
    import ctypes
    import advanced_optimizers_b200 as A
    from advanced_optimizers_b200 import _lib as L
    rng = np.random.default_rng(12)
    shapes = [(1536, 512), (512, 1536), (300, 700)]
    r = 64
    ps0 = [O.round_bf16((rng.standard_normal(sh) * 0.02).astype(np.float32)) for sh in shapes]
    params = [torch.nn.Parameter(torch.from_numpy(v.copy()).cuda().to(torch.bfloat16)) for v in ps0]
    hp = _oracle_hp(adamuon, precision="auto", low_rank_ortho=True, ortho_rank=r, stochastic_rounding=False)
    kw = dict(lr=hp["lr"], nesterov=hp["nesterov"], state_precision="auto", low_rank_ortho=True, ortho_rank=r,
              stochastic_rounding=False)
    if adamuon:
        opt = A.AdaMuon_adv([dict(params=params, optim_type="muon")], betas=hp["betas"], **kw)
    else:
        opt = A.Muon_adv([dict(params=params, optim_type="muon")], beta1=hp["beta1"], **kw)
    stream = torch.cuda.current_stream().cuda_stream
    for i, (p, sh) in enumerate(zip(params, shapes)):
        g = O.round_bf16((rng.standard_normal(sh) * 1e-3).astype(np.float32))
        p.grad = torch.from_numpy(g.copy()).cuda().to(torch.bfloat16)
        # the sketch the device draws for this tensor at step 0
        sk = torch.empty((sh[1], min(r, *sh)), dtype=torch.bfloat16, device="cuda")
        L.check(L.lib().advopt_lr_sketch(sk.data_ptr(), sk.shape[0], sk.shape[1], 42, opt._tid(p), 0, stream),
                "advopt_lr_sketch")
        skf = sk.float().cpu().numpy()
        assert abs(skf.mean()) < 0.05 and abs(skf.std() - 1.0) < 0.05
        st = {}
        O.init_state_tensor(st, "momentum_buffer", sh, "auto", "bf16")
        if adamuon:
            O.init_state_tensor(st, "second_momentum_buffer", sh, "auto", "bf16", non_neg=True)
        step_fn = O.adamuon_step if adamuon else O.muon_step
        p._oracle = step_fn(ps0[i].copy(), "bf16", g, st, hp, {"sketch": O.bf16_bits(skf)})
    opt.step()
    torch.cuda.synchronize()
    opt.check_errors()
    for i, p in enumerate(params):
        mine = p.detach().float().cpu().numpy()
        # the QR differs in arithmetic (float64 CholeskyQR3 here, float32
        # Householder in the oracle), which moves Q by bf16 ulps; AdaMuon's
        # first step makes the update a sign pattern, so near-zero chain
        # outputs flip: up to 1e-3 of its elements outside the band
        check_ns_param(mine, p._oracle, ps0[i], "bf16", f"low rank {shapes[i]}", adamuon,
                       allowed_frac=1e-3 if adamuon else None)


@pytest.mark.parametrize("shape,r,cns", [((512, 1536), 64, False), ((1536, 512), 96, True), ((300, 700), 40, False)])
def test_newton_schulz_low_rank_matches_oracle(shape, r, cns):
    """newton_schulz(low_rank_ortho=True) with a given sketch against the
    oracle's low-rank chain (float32 Householder QR there, float64 shifted
    CholeskyQR3 here), at the tolerance of the full chain."""
    import advanced_optimizers_b200 as A
    rng = np.random.default_rng(shape[0] + r)
    g = O.round_bf16((rng.standard_normal(shape) * 0.01).astype(np.float32))
    sk = O.round_bf16(rng.standard_normal((shape[1], r)).astype(np.float32))
    G = torch.from_numpy(g).cuda().to(torch.bfloat16)
    S = torch.from_numpy(sk).cuda().to(torch.bfloat16)
    mine = A.newton_schulz(G, steps=5, eps=1e-7, coeffs=QUINTIC, cns=cns, low_rank_ortho=True, ortho_rank=r,
                           G_sketch=S)
    torch.cuda.synchronize()
    assert mine.dtype == torch.bfloat16 and mine.shape == G.shape
    ref = O.newton_schulz(O.T(g, "bf16"), 5, 1e-7, QUINTIC, cns, None, sketch=O.bf16_bits(sk)).v
    _check_ns_output(mine.float().cpu().numpy(), ref, f"low-rank NS {shape} r={r} cns={cns}")
