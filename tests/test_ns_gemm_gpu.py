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


@pytest.mark.parametrize("m,k", [(1024, 4096), (4096, 4096), (4096, 14336)])
def test_symmetric_products_at_llama_shapes(m, k):
    """The symmetric-output path at the production tilings (4 x 4 and
    16 x 16 blocks of 256): A = X X^T from X [m][k] (the k/v, q and gate
    Newton-Schulz shapes), then B = b A + c A A with the quintic
    coefficients.  Every element — the computed blocks on or above the
    diagonal and the mirrored stores below it — is checked against the fp32
    product, and D must be exactly symmetric.  Per element the tolerance is
    one bf16 ulp of the result plus the fp32 accumulation-order error, which
    scales with the magnitudes summed rather than with the result: on the
    diagonal of b A + c A A the two terms cancel (c (A A)_ii ~ 9, b A_ii ~ -9,
    result ~ 0.2 at 4096 x 14336), so the accumulation term is
    2^-12 (|c| |A| |A| + |b| |A|): K u, the worst-case bound of a K = 4096-term
    float32 sum (the tensor cores measured about 2^-13.5 there)."""
    from advanced_optimizers_b200 import _lib as L
    g = torch.Generator(device="cuda").manual_seed(m + k)
    X = (torch.randn(m, k, generator=g, device="cuda") / (m * k) ** 0.25).bfloat16()
    A = torch.empty(m, m, device="cuda", dtype=torch.bfloat16)
    B = torch.empty_like(A)
    err = torch.zeros(1, dtype=torch.int32, device="cuda")
    s = torch.cuda.current_stream().cuda_stream
    lib = L.lib()
    # A = X X^T: both operands X, stored [m][k] (K-major)
    L.check(lib.advopt_ns_gemm_sym(A.data_ptr(), m, X.data_ptr(), k, X.data_ptr(), k, 0, None, m, m, k,
                                   1.0, 0.0, err.data_ptr(), s), "advopt_ns_gemm_sym")
    # B = c A A + b A: A is symmetric, so A stored [m][m] serves as [K][N]
    b, c = -4.7750, 2.0315
    L.check(lib.advopt_ns_gemm_sym(B.data_ptr(), m, A.data_ptr(), m, A.data_ptr(), m, 1, A.data_ptr(), m, m, m,
                                   c, b, err.data_ptr(), s), "advopt_ns_gemm_sym")
    torch.cuda.synchronize()
    assert int(err.item()) == 0
    Xa, Aa = X.float().abs(), A.float().abs()
    for D, ref32, mag, what in ((A, X.float() @ X.float().t(), Xa @ Xa.t(), "X X^T"),
                                (B, c * (A.float() @ A.float()) + b * A.float(), abs(c) * (Aa @ Aa) + abs(b) * Aa,
                                 "b A + c A A")):
        assert torch.equal(D.view(torch.int16), D.t().contiguous().view(torch.int16)), f"{what}: not symmetric"
        diff = (D.float() - ref32).abs()
        rms = float(ref32.pow(2).mean().sqrt())
        bad = diff > 2.0 ** -8 * ref32.abs() + 2.0 ** -12 * mag + 1e-3 * rms
        nb = int(bad.sum())
        if nb:
            r, cidx = torch.nonzero(bad)[0].tolist()
            raise AssertionError(f"{what} m={m}: {nb} elements beyond 1 bf16 ulp + 1e-3 rms, first at ({r}, {cidx}) "
                                 f"block ({r // 256}, {cidx // 256}); max diff {float(diff.max()):.3g}, rms {rms:.3g}")
        rel = float((D.float() - ref32).norm() / ref32.norm())
        assert rel < 4e-3, (what, rel)
