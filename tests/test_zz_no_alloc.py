"""advopt_adam_step_noalloc against the ordinary entry point, two calls in a row.

Some callers cannot allocate device memory during an optimizer step: a
runtime that owns a fixed, pre-sized device arena with no allocator hook, or
code that must not call cudaMalloc (or a framework's caching allocator) in the
middle of a training step.  advopt_adam_step_noalloc serves them: it takes
only the caller's own tensors and keeps the scratch that advopt_adam_step
expects from the caller (descriptor table, CTA plan, factored column
partials) in a static device array of ADVOPT_NOALLOC_SCRATCH_BYTES.

Checked through the C ABI against AdamW_adv / Muon_adv's auxiliary Adam (which
call advopt_adam_step), on identical inputs and injected random integers,
with the tolerances of the other parity tests: int8 codes, block scales and
params bit-exact (the same arithmetic on the same values); the factored
row/column factors within 2e-6 relative (the two entry points cut the tensor
into different pieces, so the float32 column partials are summed in a
different order).  The cases cover the fast kernel (factored and not), the
general kernel (atan2), the auxiliary-Adam order of the moments, a factored
tensor wide enough (d2 = 14336) that its column partials live in the array
and the array caps the grid, and the rejection of a tensor whose partials
cannot fit at all.
"""
import ctypes
import math

import numpy as np
import pytest
import torch

from _compare import check_fp32
from _gpu import to_numpy

pytestmark = pytest.mark.gpu

A_ATAN2 = 4 / math.pi

CASES = {
    "int8_factored_bf16": ((4096, 1024), torch.bfloat16, "adamw",
                           dict(lr=1e-3, betas=(0.9, 0.999), eps=1e-8, weight_decay=0.0,
                                state_precision="int8_sr", factored_2nd=True, nesterov=True)),
    "int8_plain_f32_cautious": ((3000, 7), torch.float32, "adamw",
                                dict(lr=1e-3, betas=(0.9, 0.99), eps=1e-8, weight_decay=0.05, cautious_wd=True,
                                     state_precision="int8_sr", factored_2nd=False, nesterov=False)),
    "atan2_general_kernel": ((640, 96), torch.bfloat16, "adamw",
                             dict(lr=2e-3, betas=(0.9, 0.999), eps=1e-8, weight_decay=0.01, use_atan2=True,
                                  state_precision="fp32", factored_2nd=False, nesterov=False)),
    "auxadam_fp32": ((1000, 33), torch.float32, "auxadam",
                     dict(lr=1e-3, adam_betas=(0.9, 0.99), adam_eps=1e-8, adam_weight_decay=0.01,
                          adam_state_precision="fp32")),
    "int8_factored_wide_grid_capped": ((14336, 14336), torch.bfloat16, "adamw",
                                       dict(lr=1e-3, betas=(0.9, 0.999), eps=1e-8, weight_decay=0.0,
                                            state_precision="int8_sr", factored_2nd=True, nesterov=True)),
}


def _ordinary(kind, p, kw):
    import advanced_optimizers_b200 as A
    if kind == "adamw":
        return A.AdamW_adv([p], **kw)
    return A.Muon_adv([{"params": [p], "optim_type": "adam"}], **kw)


@pytest.mark.parametrize("name", list(CASES))
def test_noalloc_matches_ordinary_entry_point(name):
    from advanced_optimizers_b200 import _lib as L

    shape, dtype, kind, kw = CASES[name]
    lib = L.lib()
    dev = torch.device("cuda", 0)
    g = torch.Generator(device=dev).manual_seed(7)
    n = math.prod(shape)
    pad = ((n + 2047) // 2048) * 2048
    p0 = (torch.randn(shape, generator=g, device=dev) * 0.02).to(dtype)
    grads = [(torch.randn(shape, generator=g, device=dev) * 1e-3).to(dtype) for _ in range(2)]
    noise = [{"exp_avg": torch.randint(0, 65536, (pad,), generator=g, device=dev, dtype=torch.int32),
              "exp_avg_sq": torch.randint(0, 65536, (pad,), generator=g, device=dev, dtype=torch.int32),
              "param": torch.randint(0, 65536, (n,), generator=g, device=dev, dtype=torch.int32)}
             for _ in range(2)]

    # ordinary entry point, through the optimizer class
    pa = torch.nn.Parameter(p0.clone())
    opt_a = _ordinary(kind, pa, kw)
    # the caller's own tensors for the no-allocation entry point (allocated
    # here by the test, as a caller with its own arena would hold them)
    pb = torch.nn.Parameter(p0.clone())
    st_b = _ordinary(kind, pb, kw).state[pb]
    gb = torch.empty_like(pb)

    if kind == "adamw":
        b1, b2 = kw["betas"]
        lr, wd, eps = kw["lr"], kw["weight_decay"], kw["eps"]
        precision = kw["state_precision"]
        algo = L.ALGO_ADAMW
        nesterov, atan2 = kw.get("nesterov", False), kw.get("use_atan2", False)
    else:
        b1, b2 = kw["adam_betas"]
        lr, wd, eps = kw["lr"], kw["adam_weight_decay"], kw["adam_eps"]
        precision = kw["adam_state_precision"]
        algo = L.ALGO_AUXADAM
        nesterov, atan2 = False, False
    fact = bool(st_b.get("factored_2nd", False))
    for step in range(2):
        pa.grad = grads[step].clone()
        opt_a.set_test_noise({pa: noise[step]})
        opt_a.step()

        gb.copy_(grads[step])
        t = st_b["step"]
        bc1 = 1.0 - b1 ** (t + 1)
        sbc2 = (1.0 - b2 ** (t + 1)) ** 0.5
        d = np.zeros(1, L.ADAM_TENSOR_DT)
        d["param"] = pb.data_ptr()
        d["grad"] = gb.data_ptr()
        d["exp_avg"] = st_b["exp_avg"].data_ptr()
        d["exp_avg_scale"] = st_b["exp_avg_scale"].data_ptr() if "exp_avg_scale" in st_b else 0
        if fact:
            d["row_factor"] = st_b["mu_v_nmf"].data_ptr()
            d["col_factor"] = st_b["mv_v_nmf"].data_ptr()
            d["d1"], d["d2"] = st_b["effective_shape"]
        else:
            d["exp_avg_sq"] = st_b["exp_avg_sq"].data_ptr()
            d["exp_avg_sq_scale"] = st_b["exp_avg_sq_scale"].data_ptr() if "exp_avg_sq_scale" in st_b else 0
        d["noise_m"] = noise[step]["exp_avg"].data_ptr()
        d["noise_v"] = noise[step]["exp_avg_sq"].data_ptr()
        d["noise_p"] = noise[step]["param"].data_ptr()
        d["numel"] = n
        d["step_size"] = (lr / bc1) * (A_ATAN2 if atan2 else 1.0)
        d["sqrt_bc2"] = sbc2
        d["eps"] = eps
        d["wd"] = wd * lr
        d["fisher_clip"] = 1.0
        d["step"] = t
        d["flags"] = (L.T_FACTORED if fact else 0) | L.T_VEC
        launch = L.AdamLaunch()
        launch.algo = algo
        launch.precision = L.PREC[precision]
        launch.param_dtype = L.DT_BF16 if dtype == torch.bfloat16 else L.DT_F32
        launch.flags = (L.F_HAS_M | L.F_NOISE_IN | (L.F_SR if dtype == torch.bfloat16 else 0)
                        | (L.F_NESTEROV if nesterov else 0) | (L.F_CAUTIOUS if kw.get("cautious_wd") else 0)
                        | (L.F_ATAN2 if atan2 else 0) | (0 if wd else L.F_NO_WD))
        launch.beta1 = float(np.float32(b1))
        launch.beta2 = float(np.float32(b2))
        launch.w_m = float(np.float32(1.0 - b1))
        launch.w_nest = float(np.float32(1 - b1))
        launch.c_v = float(np.float32(1.0 - b2))
        launch.seed = 42
        stream = torch.cuda.current_stream(dev).cuda_stream
        rc = lib.advopt_adam_step_noalloc(d.ctypes.data_as(ctypes.c_void_p), ctypes.byref(launch), stream)
        L.check(rc, "advopt_adam_step_noalloc")
        st_b["step"] += 1
        torch.cuda.synchronize()

        st_a = opt_a.state[pa]
        what = f"{name} call {step + 1}"
        assert torch.equal(pb.view(-1).view(torch.int16 if dtype == torch.bfloat16 else torch.int32),
                           pa.view(-1).view(torch.int16 if dtype == torch.bfloat16 else torch.int32)), \
            f"{what}: params differ"
        for key in ("exp_avg", "exp_avg_scale") + (() if fact else ("exp_avg_sq", "exp_avg_sq_scale")):
            if key in st_a:
                assert torch.equal(st_b[key], st_a[key]), f"{what}: {key} differs"
        if fact:
            check_fp32(to_numpy(st_b["mu_v_nmf"]), to_numpy(st_a["mu_v_nmf"]), 2e-6, f"{what}: mu_v_nmf")
            check_fp32(to_numpy(st_b["mv_v_nmf"]), to_numpy(st_a["mv_v_nmf"]), 2e-6, f"{what}: mv_v_nmf")
            # keep both sides on the same factors so the second call compares one step
            st_b["mu_v_nmf"].copy_(st_a["mu_v_nmf"])
            st_b["mv_v_nmf"].copy_(st_a["mv_v_nmf"])


def test_noalloc_rejects_partials_too_wide_for_the_array():
    """A factored tensor whose one row of column partials exceeds the static
    array is refused with ADVOPT_E_INVALID before any kernel runs (the
    descriptor's device pointers are never touched)."""
    from advanced_optimizers_b200 import _lib as L

    lib = L.lib()
    d2 = 5_000_000                      # 20 MB of float32 partials per row
    d = np.zeros(1, L.ADAM_TENSOR_DT)
    for f in ("param", "grad", "exp_avg", "exp_avg_scale", "row_factor", "col_factor"):
        d[f] = 1 << 20                  # never dereferenced: the call is refused first
    d["numel"], d["d1"], d["d2"] = d2, 1, d2
    d["sqrt_bc2"], d["eps"], d["step_size"] = 1.0, 1e-8, 1e-3
    d["flags"] = L.T_FACTORED | L.T_VEC
    launch = L.AdamLaunch()
    launch.algo = L.ALGO_ADAMW
    launch.precision = L.PREC["int8_sr"]
    launch.param_dtype = L.DT_BF16
    launch.flags = L.F_HAS_M | L.F_SR
    rc = lib.advopt_adam_step_noalloc(d.ctypes.data_as(ctypes.c_void_p), ctypes.byref(launch),
                                      torch.cuda.current_stream().cuda_stream)
    assert rc == -1, rc
    assert b"scratch array" in lib.advopt_last_error()
