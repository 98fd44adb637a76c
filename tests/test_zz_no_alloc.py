"""advopt_adam_step_noalloc against the ordinary entry point, two calls in a row.

Some callers cannot allocate device memory during an optimizer step: a
runtime that owns a fixed, pre-sized device arena with no allocator hook, or
code that must not call cudaMalloc (or a framework's caching allocator) in the
middle of a training step.  advopt_adam_step_noalloc serves them: it takes
only the caller's own tensors and keeps the scratch that advopt_adam_step
expects from the caller (descriptor table, CTA plan, factored column
partials) in a static device array of ADVOPT_NOALLOC_SCRATCH_BYTES.

Checked through the C ABI against AdamW_adv (which calls advopt_adam_step),
on identical inputs and injected random integers, with the tolerances of the
other parity tests: int8 codes, block scales and params bit-exact (the same
arithmetic on the same values); the factored row/column factors within 2e-6
relative (the two entry points cut the tensor into different pieces, so the
float32 column partials are summed in a different order).
"""
import ctypes
import math

import numpy as np
import pytest
import torch

from _compare import check_fp32
from _gpu import to_numpy

pytestmark = pytest.mark.gpu

CASES = [
    ((4096, 1024), torch.bfloat16, dict(lr=1e-3, betas=(0.9, 0.999), eps=1e-8, weight_decay=0.0,
                                        state_precision="int8_sr", factored_2nd=True, nesterov=True)),
    ((3000, 7), torch.float32, dict(lr=1e-3, betas=(0.9, 0.99), eps=1e-8, weight_decay=0.05, cautious_wd=True,
                                    state_precision="int8_sr", factored_2nd=False, nesterov=False)),
]


@pytest.mark.parametrize("shape,dtype,kw", CASES)
def test_noalloc_matches_ordinary_entry_point(shape, dtype, kw):
    import advanced_optimizers_b200 as A
    from advanced_optimizers_b200 import _lib as L

    lib = L.lib()
    dev = torch.device("cuda", 0)
    g = torch.Generator().manual_seed(7)
    n = math.prod(shape)
    pad = ((n + 2047) // 2048) * 2048
    p_host = (torch.randn(shape, generator=g) * 0.02).to(dtype)
    grads = [(torch.randn(shape, generator=g) * 1e-3).to(dtype) for _ in range(2)]
    noise = [{"exp_avg": torch.randint(0, 65536, (pad,), generator=g, dtype=torch.int32).to(dev),
              "exp_avg_sq": torch.randint(0, 65536, (pad,), generator=g, dtype=torch.int32).to(dev),
              "param": torch.randint(0, 65536, (n,), generator=g, dtype=torch.int32).to(dev)} for _ in range(2)]

    # ordinary entry point, through the optimizer class
    pa = torch.nn.Parameter(p_host.to(dev))
    opt_a = A.AdamW_adv([pa], **kw)
    # the caller's own tensors for the no-allocation entry point (allocated
    # here by the test, as a caller with its own arena would hold them)
    pb = torch.nn.Parameter(p_host.to(dev))
    st_b = A.AdamW_adv([pb], **kw).state[pb]
    gb = torch.empty_like(pb)

    b1, b2 = kw["betas"]
    lr, wd = kw["lr"], kw["weight_decay"]
    fact = st_b["factored_2nd"]
    for step in range(2):
        pa.grad = grads[step].to(dev)
        opt_a.set_test_noise({pa: noise[step]})
        opt_a.step()

        gb.copy_(grads[step].to(dev))
        t = st_b["step"]
        bc1 = 1.0 - b1 ** (t + 1)
        sbc2 = (1.0 - b2 ** (t + 1)) ** 0.5
        d = np.zeros(1, L.ADAM_TENSOR_DT)
        d["param"] = pb.data_ptr()
        d["grad"] = gb.data_ptr()
        d["exp_avg"] = st_b["exp_avg"].data_ptr()
        d["exp_avg_scale"] = st_b["exp_avg_scale"].data_ptr()
        if fact:
            d["row_factor"] = st_b["mu_v_nmf"].data_ptr()
            d["col_factor"] = st_b["mv_v_nmf"].data_ptr()
            d["d1"], d["d2"] = st_b["effective_shape"]
        else:
            d["exp_avg_sq"] = st_b["exp_avg_sq"].data_ptr()
            d["exp_avg_sq_scale"] = st_b["exp_avg_sq_scale"].data_ptr()
        d["noise_m"] = noise[step]["exp_avg"].data_ptr()
        d["noise_v"] = noise[step]["exp_avg_sq"].data_ptr()
        d["noise_p"] = noise[step]["param"].data_ptr()
        d["numel"] = n
        d["step_size"] = lr / bc1
        d["sqrt_bc2"] = sbc2
        d["eps"] = kw["eps"]
        d["wd"] = wd * lr
        d["fisher_clip"] = 1.0
        d["step"] = t
        d["flags"] = (L.T_FACTORED if fact else 0) | L.T_VEC
        launch = L.AdamLaunch()
        launch.algo = L.ALGO_ADAMW
        launch.precision = L.PREC["int8_sr"]
        launch.param_dtype = L.DT_BF16 if dtype == torch.bfloat16 else L.DT_F32
        launch.flags = (L.F_HAS_M | L.F_NOISE_IN | (L.F_SR if dtype == torch.bfloat16 else 0)
                        | (L.F_NESTEROV if kw["nesterov"] else 0) | (L.F_CAUTIOUS if kw.get("cautious_wd") else 0))
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
        what = f"{shape} {dtype} call {step + 1}"
        np.testing.assert_array_equal(to_numpy(pb), to_numpy(pa), err_msg=f"{what}: params")
        np.testing.assert_array_equal(to_numpy(st_b["exp_avg"]), to_numpy(st_a["exp_avg"]), err_msg=f"{what}: m codes")
        np.testing.assert_array_equal(to_numpy(st_b["exp_avg_scale"]), to_numpy(st_a["exp_avg_scale"]),
                                      err_msg=f"{what}: m scales")
        if fact:
            check_fp32(to_numpy(st_b["mu_v_nmf"]), to_numpy(st_a["mu_v_nmf"]), 2e-6, f"{what}: mu_v_nmf")
            check_fp32(to_numpy(st_b["mv_v_nmf"]), to_numpy(st_a["mv_v_nmf"]), 2e-6, f"{what}: mv_v_nmf")
            # keep both sides on the same factors so the second call compares one step
            st_b["mu_v_nmf"].copy_(st_a["mu_v_nmf"])
            st_b["mv_v_nmf"].copy_(st_a["mv_v_nmf"])
        else:
            np.testing.assert_array_equal(to_numpy(st_b["exp_avg_sq"]), to_numpy(st_a["exp_avg_sq"]),
                                          err_msg=f"{what}: v codes")
            np.testing.assert_array_equal(to_numpy(st_b["exp_avg_sq_scale"]), to_numpy(st_a["exp_avg_sq_scale"]),
                                          err_msg=f"{what}: v scales")
