"""Edge cases on the GPU: empty tensors, all-zero / tiny / huge gradients (the
IEEE fallback of the fast kernel), parameters without gradients, mixed
dtypes in one group, step_parameter() against step(), state_dict round
trips, and AdaMuon on a 4-D (convolution-shaped) parameter.

Where the oracle is the reference, tolerances are those of the other parity
tests (int8 codes and scales exact, bf16 params within 1 ulp, fp32 1e-6);
the structural tests (round trips, step_parameter, mixed dtypes, empty
tensors) compare two runs of this library and require identical bits."""
import math

import numpy as np
import pytest
import torch

from _compare import check_bf16_param, check_fp32, check_state
from _gpu import to_numpy
from _replay import O

pytestmark = pytest.mark.gpu


def _noise(shapes, g, int8=True):
    out = []
    for sh in shapes:
        n = max(1, math.prod(sh))
        pad = ((n + 2047) // 2048) * 2048 if int8 else n
        out.append({"exp_avg": torch.randint(0, 65536, (pad,), generator=g, dtype=torch.int32),
                    "exp_avg_sq": torch.randint(0, 65536, (pad,), generator=g, dtype=torch.int32),
                    "param": torch.randint(0, 65536, (n,), generator=g, dtype=torch.int32)})
    return out


def _adamw_vs_oracle(shapes, grads_fn, kw, steps=2):
    """Steps on the GPU and in the oracle from the same params, states and
    injected noise; every step starts from the GPU's params and factors."""
    import advanced_optimizers_b200 as A
    g = torch.Generator().manual_seed(11)
    p_host = [(torch.randn(sh, generator=g) * 0.02).bfloat16() for sh in shapes]
    params = [torch.nn.Parameter(t.cuda()) for t in p_host]
    opt = A.AdamW_adv(params, **kw)
    ostate = [{k: (to_numpy(v) if torch.is_tensor(v) else v) for k, v in opt.state[p].items()} for p in params]
    hp = dict(lr=1e-3, betas=(0.9, 0.999), eps=1e-8, precision=kw.get("state_precision", "auto"))
    hp.update({k: v for k, v in kw.items() if k != "state_precision"})
    prev = [O.from_bf16_bits(to_numpy(t)).reshape(sh) for t, sh in zip(p_host, shapes)]
    for s in range(steps):
        grads = [grads_fn(sh, g).bfloat16() for sh in shapes]
        noise = _noise(shapes, g, hp["precision"] == "int8_sr")
        for p, gr in zip(params, grads):
            p.grad = gr.cuda()
        opt.set_test_noise({p: {k: v.cuda() for k, v in nz.items()} for p, nz in zip(params, noise)})
        opt.step()
        torch.cuda.synchronize()
        for i, (p, sh) in enumerate(zip(params, shapes)):
            n = math.prod(sh)
            nz = {k: (v.numpy() if (k != "param" and hp["precision"] == "int8_sr") else v.numpy()[:n])
                  for k, v in noise[i].items()}
            gv = O.from_bf16_bits(to_numpy(grads[i])).reshape(sh)
            new = O.adam_family_step(prev[i], "bf16", gv, ostate[i], hp, nz)
            check_bf16_param(to_numpy(p), O.bf16_bits(new), f"{sh} step {s}")
            for key, val in opt.state[p].items():
                if torch.is_tensor(val) and key in ostate[i] and isinstance(ostate[i][key], np.ndarray):
                    check_state(key, to_numpy(val), ostate[i][key], f"{sh} step {s} {key}")
            for key in ("mu_v_nmf", "mv_v_nmf"):
                if key in ostate[i]:
                    ostate[i][key] = to_numpy(opt.state[p][key])
        prev = [O.from_bf16_bits(to_numpy(p)).reshape(sh) for p, sh in zip(params, shapes)]


@pytest.mark.parametrize("kind", ["zero", "tiny", "huge", "mixed"])
def test_extreme_gradients_match_oracle(kind):
    """v = 0, subnormal-range v and |v| near overflow take the IEEE path of
    the fast kernel; results still match the reference's arithmetic."""
    def grads(sh, g):
        t = torch.randn(sh, generator=g)
        if kind == "zero":
            return torch.zeros(sh)
        if kind == "tiny":
            return t * 1e-30
        if kind == "huge":
            return t * 1e18
        mask = torch.rand(sh, generator=g)
        return torch.where(mask < 0.2, torch.zeros(sh), torch.where(mask < 0.4, t * 1e-25, t * 1e-3))
    _adamw_vs_oracle([(2048, 2048), (4096,), (1024, 4096)], grads,
                     dict(state_precision="int8_sr", factored_2nd=True, nesterov=True))


def test_empty_tensors_and_missing_grads():
    """Empty parameters and parameters without a gradient are left alone;
    the others step exactly as without them (round to nearest, so the noise
    streams do not matter)."""
    import advanced_optimizers_b200 as A
    g = torch.Generator().manual_seed(2)
    def make():
        ps = [torch.nn.Parameter(torch.zeros(0, 16, dtype=torch.bfloat16, device="cuda")),
              torch.nn.Parameter((torch.randn(64, 48, generator=g) * 0.02).bfloat16().cuda()),
              torch.nn.Parameter(torch.zeros(0, dtype=torch.bfloat16, device="cuda")),
              torch.nn.Parameter((torch.randn(300, generator=g) * 0.02).bfloat16().cuda())]
        return ps
    for cls, kw in ((A.AdamW_adv, dict(state_precision="fp32")), (A.Lion_adv, {}), (A.Prodigy_adv, {})):
        g.manual_seed(2)
        ps = make()
        g.manual_seed(2)
        ref = make()
        grads = [torch.randn(p.shape, generator=g).bfloat16().cuda() * 1e-3 for p in ps]
        o1 = cls(ps, stochastic_rounding=False, **kw)
        o2 = cls([ref[1]], stochastic_rounding=False, **kw)
        for p, gr in zip(ps, grads):
            p.grad = gr.clone()
        ps[3].grad = None
        ref[1].grad = grads[1].clone()
        o1.step()
        o2.step()
        torch.cuda.synchronize()
        assert ps[0].numel() == 0 and ps[2].numel() == 0
        assert torch.equal(ps[1], ref[1]), cls.__name__
        assert torch.equal(ps[3], ref[3]), cls.__name__   # no grad: untouched


def test_mixed_dtypes_in_one_group():
    import advanced_optimizers_b200 as A
    g = torch.Generator().manual_seed(4)
    a32 = (torch.randn(512, 384, generator=g) * 0.02).cuda()
    a16 = (torch.randn(384, 512, generator=g) * 0.02).bfloat16().cuda()
    g32 = (torch.randn(512, 384, generator=g) * 1e-3).cuda()
    g16 = (torch.randn(384, 512, generator=g) * 1e-3).bfloat16().cuda()
    kw = dict(state_precision="int8_sr", factored_2nd=True, stochastic_rounding=False)
    p = [torch.nn.Parameter(a32.clone()), torch.nn.Parameter(a16.clone())]
    q = [torch.nn.Parameter(a32.clone()), torch.nn.Parameter(a16.clone())]
    o = A.AdamW_adv(p, **kw)
    o32, o16 = A.AdamW_adv([q[0]], **kw), A.AdamW_adv([q[1]], **kw)
    for _ in range(2):
        p[0].grad, p[1].grad = g32.clone(), g16.clone()
        q[0].grad, q[1].grad = g32.clone(), g16.clone()
        o.step()
        o32.step()
        o16.step()
    torch.cuda.synchronize()
    # int8 momentum draws noise per tensor id: compare the deterministic parts
    assert torch.equal(o.state[p[0]]["mu_v_nmf"], o32.state[q[0]]["mu_v_nmf"])
    assert torch.equal(o.state[p[1]]["mv_v_nmf"], o16.state[q[1]]["mv_v_nmf"])


def test_step_parameter_matches_step():
    import advanced_optimizers_b200 as A
    g = torch.Generator().manual_seed(5)
    shapes = [(1024, 512), (512,), (256, 2048)]
    init = [(torch.randn(s, generator=g) * 0.02).bfloat16().cuda() for s in shapes]
    grads = [[(torch.randn(s, generator=g) * 1e-3).bfloat16().cuda() for s in shapes] for _ in range(2)]
    # no factored second moment here: its column sums follow the launch's
    # piece plan, which differs between one launch per tensor and per group
    for cls, kw in ((A.AdamW_adv, dict(state_precision="int8_sr", nesterov=True)), (A.Lion_adv, {})):
        p1 = [torch.nn.Parameter(t.clone()) for t in init]
        p2 = [torch.nn.Parameter(t.clone()) for t in init]
        o1, o2 = cls(p1, **kw), cls(p2, **kw)
        for s in range(2):
            for a, b, gr in zip(p1, p2, grads[s]):
                a.grad, b.grad = gr.clone(), gr.clone()
            o1.step()
            for b in p2:
                o2.step_parameter(b, o2.param_groups[0], None)
        torch.cuda.synchronize()
        for a, b in zip(p1, p2):
            assert torch.equal(a, b), cls.__name__


@pytest.mark.parametrize("cls_name", ["AdamW_adv", "Muon_adv", "AdaMuon_adv", "Lion_adv"])
def test_state_dict_round_trip(cls_name):
    """Two steps in one optimizer equal one step, state_dict(), a fresh
    optimizer, load_state_dict(), one more step.  (Prodigy is left out: like
    the reference, a fresh optimizer restarts its numerator carry from
    d_numerator without the beta3 factor, Prodigy_adv.py:333-335.)"""
    import advanced_optimizers_b200 as A
    cls = getattr(A, cls_name)
    g = torch.Generator().manual_seed(6)
    shapes = [(512, 384), (384,)]
    init = [(torch.randn(s, generator=g) * 0.02).bfloat16().cuda() for s in shapes]
    grads = [[(torch.randn(s, generator=g) * 1e-3).bfloat16().cuda() for s in shapes] for _ in range(2)]
    kw = dict(stochastic_rounding=False)
    if cls_name == "AdamW_adv":
        kw["state_precision"] = "int8_sr"
    if cls_name in ("Muon_adv", "AdaMuon_adv"):
        kw["state_precision"] = "int8_sr"

    def groups(ps):
        if cls_name in ("Muon_adv", "AdaMuon_adv"):
            return [dict(params=[ps[0]], optim_type="muon"), dict(params=[ps[1]], optim_type="adam")]
        return ps

    a = [torch.nn.Parameter(t.clone()) for t in init]
    oa = cls(groups(a), **kw)
    b = [torch.nn.Parameter(t.clone()) for t in init]
    ob = cls(groups(b), **kw)
    for s in range(2):
        for p, gr in zip(a, grads[s]):
            p.grad = gr.clone()
        oa.step()
    for p, gr in zip(b, grads[0]):
        p.grad = gr.clone()
    ob.step()
    sd = ob.state_dict()
    c = [torch.nn.Parameter(p.detach().clone()) for p in b]
    oc = cls(groups(c), **kw)
    oc.load_state_dict(sd)
    for p, gr in zip(c, grads[1]):
        p.grad = gr.clone()
    oc.step()
    torch.cuda.synchronize()
    for x, y in zip(a, c):
        if cls_name in ("Muon_adv", "AdaMuon_adv"):
            # int8 momentum noise is keyed by an internal step count that a
            # fresh optimizer restarts; the deterministic update must agree closely
            assert float((x.float() - y.float()).abs().max()) <= 2e-3, cls_name
        else:
            assert torch.equal(x, y), cls_name
    for key, val in oa.state[a[0]].items():
        if torch.is_tensor(val):
            assert val.dtype == oc.state[c[0]][key].dtype, key


def test_adamuon_conv_parameter_matches_oracle():
    """A 4-D parameter under auto_projection: kappa_p = 2 (no sign), the
    update is orthogonalised as the flattened [out, in*kh*kw] matrix and
    rescaled in the parameter's own last two dimensions."""
    import advanced_optimizers_b200 as A
    g = torch.Generator().manual_seed(8)
    shape = (64, 16, 3, 3)
    p0 = (torch.randn(shape, generator=g) * 0.02).bfloat16()
    p = torch.nn.Parameter(p0.cuda())
    opt = A.AdaMuon_adv([dict(params=[p], optim_type="muon")], state_precision="fp32", rms_rescaling=False)
    st = {}
    O.init_state_tensor(st, "momentum_buffer", shape, "fp32", "bf16")
    O.init_state_tensor(st, "second_momentum_buffer", shape, "fp32", "bf16", non_neg=True)
    gr = (torch.randn(shape, generator=g) * 1e-3).bfloat16()
    nz = torch.randint(0, 65536, (math.prod(shape),), generator=g, dtype=torch.int32)
    p.grad = gr.cuda()
    opt.set_test_noise({p: {"param": nz.cuda()}})
    opt.step()
    torch.cuda.synchronize()
    hp = dict(lr=1e-3, betas=(0.95, 0.95), eps=1e-8, nesterov=True, nesterov_coef=None, ns_steps=5, ns_eps=1e-7,
              ns_coeffs=(3.4445, -4.7750, 2.0315), precision="fp32", rms_rescaling=False, kappa_p=1.0,
              auto_projection=True)
    new = O.adamuon_step(p0.float().numpy(), "bf16", gr.float().numpy(), st, hp, {"param": nz.numpy()})
    mine = p.detach().float().cpu().numpy().reshape(-1).astype(np.float64)
    ref = new.reshape(-1).astype(np.float64)
    old = p0.float().numpy().reshape(-1).astype(np.float64)
    excess = np.maximum(np.abs(mine - ref) - 2.0 ** -7 * np.maximum(np.abs(ref), np.abs(old)), 0.0)
    assert np.linalg.norm(excess) <= 0.05 * np.linalg.norm(ref - old)
    check_fp32(to_numpy(opt.state[p]["momentum_buffer"]), st["momentum_buffer"], 1e-6, "momentum")
