"""Comparison helpers with the tolerances the parity tests state."""
import numpy as np

from _replay import O


def ulp_diff_bf16(a_bits, b_bits):
    a = np.asarray(a_bits).astype(np.int32)
    b = np.asarray(b_bits).astype(np.int32)
    a = np.where(a & 0x8000, 0x8000 - (a & 0x7FFF), a + 0x8000)
    b = np.where(b & 0x8000, 0x8000 - (b & 0x7FFF), b + 0x8000)
    return np.abs(a - b)


def check_fp32(a, b, rtol=1e-6, what="", ref_scale=None):
    """|a-b| <= rtol * max(|b|, |ref_scale|)."""
    a = np.asarray(a, np.float32).reshape(-1)
    b = np.asarray(b, np.float32).reshape(-1)
    err = np.abs(a.astype(np.float64) - b.astype(np.float64))
    scale = np.abs(b.astype(np.float64))
    if ref_scale is not None:
        scale = np.maximum(scale, np.abs(np.asarray(ref_scale, np.float64).reshape(-1)))
    tol = rtol * scale + 1e-30
    bad = np.count_nonzero(err > tol)
    assert bad == 0, f"{what}: {bad}/{a.size} beyond rtol {rtol}; max rel {np.max(err / (np.abs(b) + 1e-30)):.3g}"


def check_bf16_param(a_bits, b_bits, what, max_ulp=1):
    d = ulp_diff_bf16(np.asarray(a_bits).reshape(-1), np.asarray(b_bits).reshape(-1))
    assert d.max() <= max_ulp, f"{what}: max {d.max()} bf16 ulps ({np.count_nonzero(d)} differ)"
    return d


def check_state(key, val, ref, what, prev=None):
    """State tensors: codes, scales and SR'd bf16 exact; fp32 within 2e-6."""
    val = np.asarray(val)
    ref = np.asarray(ref)
    if key in ("shifter", "anchor_data", "anchor_scale", "anchor_min"):
        np.testing.assert_array_equal(val.reshape(-1), ref.reshape(-1), err_msg=what)
    elif key in ("spectral_u", "spectral_v"):
        # unit vectors from matrix-vector products summed in another order:
        # within 1e-5 (fp32) or 1 bf16 ulp of the largest element
        vv = O.from_bf16_bits(val) if val.dtype == np.uint16 else val
        rr = O.from_bf16_bits(ref) if ref.dtype == np.uint16 else ref
        mx = float(np.max(np.abs(rr)))
        tol = 2.0 ** (np.floor(np.log2(mx)) - 7) if val.dtype == np.uint16 and mx > 0 else 1e-5 * mx
        err = np.max(np.abs(np.asarray(vv, np.float64) - np.asarray(rr, np.float64)))
        assert err <= tol, f"{what}: max error {err:.3g} above {tol:.3g}"
    elif val.dtype in (np.int8, np.uint8):
        np.testing.assert_array_equal(val.reshape(-1), ref.reshape(-1), err_msg=what)
    elif val.dtype == np.uint16:
        # 1 bf16 ulp, of the larger of the new and the pre-step value (`prev`)
        # where an update cancels the state towards zero
        d = ulp_diff_bf16(val.reshape(-1), ref.reshape(-1))
        if d.max() > 1 and prev is not None and np.asarray(prev).shape == ref.shape:
            vv = O.from_bf16_bits(val).reshape(-1).astype(np.float64)
            rr = O.from_bf16_bits(ref).reshape(-1).astype(np.float64)
            sc = np.maximum(np.abs(rr), np.abs(O.from_bf16_bits(np.asarray(prev)).reshape(-1).astype(np.float64)))
            ulp = 2.0 ** (np.floor(np.log2(np.maximum(sc, 1e-38))) - 7)
            bad = np.count_nonzero(np.abs(vv - rr) > ulp)
            assert bad == 0, f"{what}: {bad} beyond 1 ulp of the larger of the old and new value"
        else:
            assert d.max() <= 1, f"{what}: max {d.max()} ulps"
    elif key.endswith("_scale"):
        np.testing.assert_array_equal(val.reshape(-1), ref.reshape(-1), err_msg=what)
    else:
        check_fp32(val, ref, 2e-6, what, prev)
