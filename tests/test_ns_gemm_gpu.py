"""The tcgen05 Newton–Schulz GEMM against an fp32 reference of the same op:
D = bf16(alpha * A @ B + beta * C) with bf16 inputs.  The tensor cores
accumulate in fp32 in their own order, so D may land on the other side of a
bf16 rounding boundary: per element |D - ref| <= 2^-8 |ref| + 1e-3 rms(ref)
(one bf16 ulp, plus the fp32 accumulation-order error that dominates for
outputs near zero), and the relative Frobenius error stays below 4e-3."""
import ctypes

import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu


def _ulps(a, b):
    a = a.view(torch.int16).to(torch.int32)
    b = b.view(torch.int16).to(torch.int32)
    a = torch.where(a < 0, -(a & 0x7FFF), a)
    b = torch.where(b < 0, -(b & 0x7FFF), b)
    return (a - b).abs()


@pytest.mark.parametrize("M,N,K,bmn,alpha,beta", [
    (128, 256, 64, False, 1.0, 0.0),
    (256, 512, 1024, False, 1.0, 0.0),
    (256, 512, 1024, True, 1.0, 0.0),
    (512, 256, 512, False, 2.0315, -4.775),
    (384, 768, 384, True, 1.0, 3.4445),
    (1024, 1024, 4096, False, -0.5, 0.25),
])
def test_ns_gemm_matches_fp32_reference(M, N, K, bmn, alpha, beta):
    from advanced_optimizers_b200 import _lib as L
    g = torch.Generator(device="cuda").manual_seed(M * 7 + N + K)
    A = (torch.randn(M, K, generator=g, device="cuda") * 0.05).bfloat16()
    Bt = (torch.randn(K, N, generator=g, device="cuda") * 0.05).bfloat16()   # logical [K][N]
    B = Bt.contiguous() if bmn else Bt.t().contiguous()                       # stored [K][N] or [N][K]
    C = (torch.randn(M, N, generator=g, device="cuda") * 0.05).bfloat16()
    D = torch.empty(M, N, device="cuda", dtype=torch.bfloat16)
    err = torch.zeros(1, dtype=torch.int32, device="cuda")
    ldb = N if bmn else K
    rc = L.lib().advopt_ns_gemm(D.data_ptr(), N, A.data_ptr(), K, B.data_ptr(), ldb, 1 if bmn else 0,
                                C.data_ptr() if beta != 0 else None, N, M, N, K, alpha, beta, err.data_ptr(),
                                torch.cuda.current_stream().cuda_stream)
    L.check(rc, "advopt_ns_gemm")
    torch.cuda.synchronize()
    assert int(err.item()) == 0
    ref32 = alpha * (A.float() @ Bt.float()) + (beta * C.float() if beta != 0 else 0.0)
    diff = (D.float() - ref32).abs()
    rms = float(ref32.pow(2).mean().sqrt())
    bad = int((diff > 2.0 ** -8 * ref32.abs() + 1e-3 * rms).sum())
    assert bad == 0, f"{bad} elements beyond 1 bf16 ulp + 1e-3 rms; max diff {float(diff.max()):.3g}, rms {rms:.3g}"
    rel = float((D.float() - ref32).norm() / ref32.norm())
    assert rel < 4e-3, rel
