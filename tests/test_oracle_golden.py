"""The oracle against the reference's own outputs (golden fixtures made by
tests/golden/make_golden.py).  CPU only.

Tolerances (the oracle restates the reference op for op; what remains are
the reference's non-exact CPU primitives):
  * int8/uint8 state codes, block scales, bf16-SR'd states that do not depend
    on a square root or a reduction: bit-exact;
  * fp32 values: |a-b| <= 1e-6*|b| + 1e-30 (torch's CPU sqrt is faithful,
    not correctly rounded: ~0.6% of elements are 1 ulp low; its float32
    cascade sums differ from the float64 sums here in the last bits);
  * bf16 params: within 1 bf16 ulp;
  * Newton-Schulz paths: bf16 GEMM chains differ by accumulation order, so
    momentum states are compared bit-exactly (they precede the NS) and the
    updated params to within 2 bf16 ulps plus 5% of the update's RMS.
Every step starts from the reference's own params and states (teacher
forcing), so each comparison measures one step.
"""
import numpy as np
import pytest

from _replay import O, list_cases, load, replay, route_kinds

CASES = list_cases()


def ulp_diff_bf16(a_bits, b_bits):
    a = a_bits.astype(np.int32)
    b = b_bits.astype(np.int32)
    # monotone integer mapping of bf16 bit patterns
    a = np.where(a & 0x8000, 0x8000 - (a & 0x7FFF), a + 0x8000)
    b = np.where(b & 0x8000, 0x8000 - (b & 0x7FFF), b + 0x8000)
    return np.abs(a - b)


def check_fp32(a, b, rtol=1e-6, what="", ref_scale=None):
    """|a-b| <= rtol * max(|b|, |ref_scale|): relative to the value, or to the
    pre-update value where an update cancels the parameter towards zero."""
    a = np.asarray(a, np.float32).reshape(-1)
    b = np.asarray(b, np.float32).reshape(-1)
    err = np.abs(a.astype(np.float64) - b.astype(np.float64))
    scale = np.abs(b.astype(np.float64))
    if ref_scale is not None:
        scale = np.maximum(scale, np.abs(np.asarray(ref_scale, np.float64).reshape(-1)))
    tol = rtol * scale + 1e-30
    bad = np.count_nonzero(err > tol)
    assert bad == 0, f"{what}: {bad}/{a.size} beyond rtol {rtol}; max rel {np.max(err / (np.abs(b) + 1e-30)):.3g}"


@pytest.mark.parametrize("name", CASES)
def test_oracle_matches_reference(name):
    meta, z = load(name)
    dt = meta["dtype"]
    ns = meta["cls"] in ("Muon_adv", "AdaMuon_adv")
    kinds = route_kinds(meta)
    for i in range(len(meta["shapes"])):
        if f"route_{i}" in z.files:
            # the reference's own routing decision (state['is_muon'])
            assert (kinds[i] == "muon") == bool(z[f"route_{i}"]), f"{name} param {i}: routing"
    prev = {i: z[f"p0_{i}"] for i in range(len(meta["shapes"]))}
    for s, i, p, st, group in replay(name, pin_d=True, teacher=True):
        if i < 0:
            ref = z[f"d_{s}"]
            assert group["k"] == int(ref[3])
            # d = d_coef * sum(<g, p0 - p>) / sum|s|: a cancelling dot product,
            # so the float32 summation order shows at the 1e-5 level
            for j, key in enumerate(("d", "d_max", "d_numerator")):
                np.testing.assert_allclose(group[key], ref[j], rtol=1e-4, err_msg=f"{name} step {s} {key}")
            continue
        is_ns_param = ns and kinds[i] == "muon"
        ref_p = z[f"p_{s}_{i}"]
        if dt == "bf16" and is_ns_param:
            # bf16 GEMM chain: within 2 bf16 ulps of the larger of the old and new value
            a, b = p.reshape(-1).astype(np.float64), O.from_bf16_bits(ref_p).reshape(-1).astype(np.float64)
            old = O.from_bf16_bits(prev[i]).reshape(-1).astype(np.float64)
            scale = np.maximum(np.abs(b), np.abs(old))
            u_rms = np.sqrt(np.mean((old - b) ** 2))
            bad = np.count_nonzero(np.abs(a - b) > 2.0 ** -6 * scale + 0.05 * u_rms)
            # AdaMuon divides by sqrt(v): where the chain's output is near zero
            # the update is a sign, and a rounding difference flips it
            allowed = int(np.ceil(5e-4 * a.size)) if meta["cls"] == "AdaMuon_adv" else 0
            assert bad <= allowed, f"{name} step {s} param {i}: {bad} beyond 2 bf16 ulps + 5% of the update RMS"
        elif dt == "bf16":
            mine = O.bf16_bits(p)
            d = ulp_diff_bf16(mine.reshape(-1), ref_p.reshape(-1))
            assert d.max() <= 1, f"{name} step {s} param {i}: max {d.max()} bf16 ulps"
        else:
            check_fp32(p, ref_p, 1e-2 if is_ns_param else 1e-6, f"{name} step {s} param {i}", prev[i])
        prev[i] = ref_p
        for key, val in st.items():
            rk = f"st_{s}_{i}_{key}"
            if rk not in z.files or not isinstance(val, np.ndarray):
                continue
            ref = z[rk]
            what = f"{name} step {s} param {i} {key}"
            if key in ("shifter", "anchor_data", "anchor_scale", "anchor_min"):
                np.testing.assert_array_equal(val.reshape(-1), ref.reshape(-1), err_msg=what)
            elif key in ("spectral_u", "spectral_v"):
                # unit vectors from matrix-vector products whose summation
                # order the reference does not fix: within 1e-5 (fp32) or
                # 1 bf16 ulp of the largest element
                vv = O.from_bf16_bits(val) if val.dtype == np.uint16 else val
                rr = O.from_bf16_bits(ref) if ref.dtype == np.uint16 else ref
                mx = float(np.max(np.abs(rr)))
                tol = 2.0 ** (np.floor(np.log2(mx)) - 7) if val.dtype == np.uint16 and mx > 0 else 1e-5 * mx
                err = np.max(np.abs(np.asarray(vv, np.float64) - np.asarray(rr, np.float64)))
                assert err <= tol, f"{what}: max error {err:.3g} above {tol:.3g}"
            elif is_ns_param and key.startswith(("second_momentum_buffer", "normuon_v", "mu_vbuf_nmf", "mv_vbuf_nmf")):
                # statistics of the Newton-Schulz output (bf16 GEMM chain)
                if val.dtype in (np.int8, np.uint8):
                    dq = np.abs(val.astype(np.int32) - ref.astype(np.int32))
                    assert np.mean(dq) < 0.5 and dq.max() <= 16, what
                else:
                    # through sqrt (proportional to the chain's output), like
                    # the chain's output: 2 bf16 ulps + 10% of its RMS, up to
                    # 5e-4 of the elements outside, 3% in the Frobenius norm
                    vv = O.from_bf16_bits(val) if val.dtype == np.uint16 else val
                    rr = O.from_bf16_bits(ref) if ref.dtype == np.uint16 else ref
                    sa = np.sqrt(np.asarray(vv, np.float64).reshape(-1))
                    sb = np.sqrt(np.asarray(rr, np.float64).reshape(-1))
                    rms = np.sqrt(np.mean(sb ** 2))
                    bad = np.count_nonzero(np.abs(sa - sb) > 2.0 ** -6 * sb + 0.1 * rms)
                    frob = np.linalg.norm(sa - sb) / max(np.linalg.norm(sb), 1e-30)
                    assert bad <= int(np.ceil(5e-4 * sa.size)) and frob < 0.03, \
                        f"{what}: {bad}/{sa.size} outside, Frobenius {frob:.3g}"
            elif val.dtype in (np.int8, np.uint8):
                np.testing.assert_array_equal(val.reshape(-1), ref.reshape(-1), err_msg=what)
            elif val.dtype == np.uint16:
                # 1 bf16 ulp, of the larger of the new and the pre-step value
                # where an update cancels the state towards zero
                d = ulp_diff_bf16(val.reshape(-1), ref.reshape(-1))
                pk = f"st_{s - 1}_{i}_{key}" if s > 0 else f"st0_{i}_{key}"
                if d.max() > 1 and pk in z.files and z[pk].shape == ref.shape:
                    vv = O.from_bf16_bits(val).reshape(-1).astype(np.float64)
                    rr = O.from_bf16_bits(ref).reshape(-1).astype(np.float64)
                    sc = np.maximum(np.abs(rr), np.abs(O.from_bf16_bits(z[pk]).reshape(-1).astype(np.float64)))
                    ulp = 2.0 ** (np.floor(np.log2(np.maximum(sc, 1e-38))) - 7)
                    bad = np.count_nonzero(np.abs(vv - rr) > ulp)
                    assert bad == 0, f"{what}: {bad} beyond 1 ulp of the larger of the old and new value"
                else:
                    assert d.max() <= 1, f"{what}: max {d.max()} ulps"
            elif key.endswith("_scale"):
                np.testing.assert_array_equal(val.reshape(-1), ref.reshape(-1), err_msg=what)
            else:
                pk = f"st_{s - 1}_{i}_{key}" if s > 0 else f"st0_{i}_{key}"
                check_fp32(val, ref, 2e-6, what, z[pk] if pk in z.files and z[pk].shape == ref.shape else None)
