"""ctypes binding of libadvopt.so (the C ABI declared in include/advopt.h).

The library is built in-tree by ``python -m advanced_optimizers_b200.build``
(or ``__graft_entry__.build()``).  There is no fallback: every optimizer
step runs through these entry points, and a missing library or a missing
CUDA device raises immediately.
"""
from __future__ import annotations

import ctypes
import os
import threading

import numpy as np

_PKG = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(_PKG, "libadvopt.so")
ABI_VERSION = 5

# ---- constants mirrored from include/advopt.h ----
DT_F32, DT_BF16 = 0, 1
PREC = {"fp32": 0, "bf16_sr": 1, "int8_sr": 2, "auto": 3}
ALGO_ADAMW, ALGO_AUXADAM, ALGO_PRODIGY, ALGO_LION = 0, 1, 2, 3
F_NESTEROV = 1 << 0
F_ATAN2 = 1 << 1
F_NORMED = 1 << 2
F_CAUTIOUS = 1 << 3
F_SR = 1 << 4
F_NOISE_IN = 1 << 5
F_HAS_M = 1 << 6
F_PRODIGY_STATS = 1 << 7
F_FISHER = 1 << 8
F_FISHER_STATS = 1 << 9
F_ANCHORS = 1 << 10
F_NO_WD = 1 << 11
F_GRAD_SQ = 1 << 12
F_EMIT_UPDATE = 1 << 13
F_FACT_M = 1 << 14
T_FACTORED = 1 << 0
T_VEC = 1 << 1
T_P0_SCALAR = 1 << 2
T_FACT_M = 1 << 3
T_ANCHOR_SHIFT = 4
T_UPD_BF16 = 1 << 7
ANCHOR = {"none": 0, "full": 1, "float8": 2, "int8": 3, "int4": 4}

# advopt_adam_tensor (232 bytes)
ADAM_TENSOR_DT = np.dtype([
    ("param", "<u8"), ("grad", "<u8"), ("exp_avg", "<u8"), ("exp_avg_scale", "<u8"),
    ("exp_avg_sq", "<u8"), ("exp_avg_sq_scale", "<u8"), ("row_factor", "<u8"), ("col_factor", "<u8"),
    ("col_partial", "<u8"), ("aux0", "<u8"), ("aux1", "<u8"), ("aux2", "<u8"),
    ("noise_v", "<u8"), ("noise_m", "<u8"), ("noise_p", "<u8"),
    ("m_row_factor", "<u8"), ("m_col_factor", "<u8"), ("m_col_partial", "<u8"), ("m_sign", "<u8"),
    ("update_out", "<u8"),
    ("numel", "<i8"), ("d1", "<i8"), ("d2", "<i8"),
    ("step_size", "<f4"), ("sqrt_bc2", "<f4"), ("eps", "<f4"), ("wd", "<f4"), ("cwd", "<f4"),
    ("fisher_clip", "<f4"),
    ("tensor_id", "<u4"), ("step", "<u4"), ("flags", "<u4"), ("slice_p", "<u4"),
    ("slot_base", "<i4"), ("n_slots", "<i4"),
])
PIECE_DT = np.dtype([("begin", "<i8"), ("end", "<i8"), ("tensor", "<i4"), ("slot", "<i4")])
# advopt_spectral_tensor (80 bytes)
S_UPD_BF16, S_VEC_BF16, S_MAXABS = 1, 2, 4
SPECTRAL_TENSOR_DT = np.dtype([
    ("update", "<u8"), ("u", "<u8"), ("v", "<u8"), ("v_partial", "<u8"), ("u_raw", "<u8"), ("scalars", "<u8"),
    ("d_out", "<i8"), ("d_in", "<i8"), ("target", "<f4"), ("flags", "<u4"), ("n_slabs", "<i4"), ("pad", "<i4"),
])
LION_TENSOR_DT = np.dtype([
    ("param", "<u8"), ("grad", "<u8"), ("exp_avg", "<u8"), ("noise_p", "<u8"), ("numel", "<i8"),
    ("lr", "<f4"), ("wd", "<f4"), ("tensor_id", "<u4"), ("step", "<u4"), ("flags", "<u4"), ("pad", "<u4"),
])


class AdamLaunch(ctypes.Structure):
    _fields_ = [
        ("tensors", ctypes.c_uint64), ("pieces", ctypes.c_uint64), ("cta_offsets", ctypes.c_uint64),
        ("piece_stats", ctypes.c_uint64), ("err", ctypes.c_uint64),
        ("n_tensors", ctypes.c_int32), ("n_pieces", ctypes.c_int32), ("grid", ctypes.c_int32),
        ("smem_floats", ctypes.c_int32), ("gen_offset", ctypes.c_int32), ("algo", ctypes.c_int32),
        ("precision", ctypes.c_int32), ("param_dtype", ctypes.c_int32), ("flags", ctypes.c_uint32),
        ("beta1", ctypes.c_float), ("beta2", ctypes.c_float), ("w_m", ctypes.c_float),
        ("w_nest", ctypes.c_float), ("c_v", ctypes.c_float), ("c_m", ctypes.c_float),
        ("d_eps", ctypes.c_float), ("beta3", ctypes.c_float), ("s_alpha", ctypes.c_float),
        ("d", ctypes.c_float), ("stages", ctypes.c_int32), ("seed", ctypes.c_uint64),
        ("layer_beta2", ctypes.c_uint64), ("layer_of_tensor", ctypes.c_uint64), ("piece_gsq", ctypes.c_uint64),
        ("prodigy", ctypes.c_uint64),
    ]


# advopt_prodigy_dev: byte offsets inside the 64-byte device block
PRODIGY_DEV_BYTES = 64
PRODIGY_DEV_SUMS = 32          # float sums[2]


class ProdigyScalarArgs(ctypes.Structure):
    """advopt_prodigy_scalar_args."""
    _fields_ = [("dev", ctypes.c_uint64), ("tensors", ctypes.c_uint64), ("tensor_consts", ctypes.c_uint64),
                ("n_tensors", ctypes.c_int32), ("safeguard_warmup", ctypes.c_int32),
                ("lr", ctypes.c_double), ("beta1", ctypes.c_double), ("beta2", ctypes.c_double),
                ("step_scale", ctypes.c_double)]


class ProdigyDArgs(ctypes.Structure):
    """advopt_prodigy_d_args."""
    _fields_ = [("dev", ctypes.c_uint64), ("active", ctypes.c_int32), ("d_limiter", ctypes.c_int32),
                ("d_coef", ctypes.c_double), ("growth_rate", ctypes.c_double),
                ("limiter_factor", ctypes.c_double), ("beta3", ctypes.c_double), ("carry_scale", ctypes.c_double)]


class KourkoutasArgs(ctypes.Structure):
    """advopt_kourkoutas_args."""
    _fields_ = [(n, ctypes.c_uint64) for n in (
        "acc", "ema", "layer_beta2", "layer_of_tensor", "piece_gsq", "pieces")] + [
        ("n_layers", ctypes.c_int32), ("n_tensors", ctypes.c_int32), ("n_pieces", ctypes.c_int32),
        ("gsq_bf16", ctypes.c_int32),
        ("beta2_max", ctypes.c_float), ("beta2_min_gap", ctypes.c_float), ("ema_alpha", ctypes.c_float),
        ("one_minus_alpha", ctypes.c_float), ("tiny_spike", ctypes.c_float), ("w", ctypes.c_float),
        ("one_minus_w_bmax", ctypes.c_float), ("pad", ctypes.c_float), ("cv_scale", ctypes.c_double),
        ("d_dev", ctypes.c_uint64),
    ]


MU_NESTEROV = 1 << 0
MU_SIGN = 1 << 1
MU_SR = 1 << 2
MU_CAUTIOUS = 1 << 3
MU_NOISE_IN = 1 << 4
MU_RMS = 1 << 5
MU_TRANSPOSED = 1 << 6
MU_ATAN2 = 1 << 7
MU_MARS = 1 << 8
MU_NORMUON = 1 << 9
MU_VFACT = 1 << 10
MU_LOWRANK = 1 << 11
VCOL_SPLIT = 16
ST_F32, ST_BF16, ST_BF16_SR, ST_Q8 = 0, 1, 2, 3


class MuonArgs(ctypes.Structure):
    """advopt_muon_args."""
    _fields_ = [(n, ctypes.c_uint64) for n in (
        "param", "grad", "m", "m_scale", "v", "v_scale", "x0", "ns", "ns_result", "u", "partial", "scalars",
        "noise_m", "noise_v", "noise_p")] + [
        ("numel", ctypes.c_int64), ("rows", ctypes.c_int64), ("cols", ctypes.c_int64), ("ld_ns", ctypes.c_int64),
        ("m_pad", ctypes.c_int64), ("n_pad", ctypes.c_int64), ("seed", ctypes.c_uint64),
        ("w_m", ctypes.c_float), ("w_nest", ctypes.c_float), ("beta2", ctypes.c_float), ("c_v", ctypes.c_float),
        ("eps", ctypes.c_float), ("ns_eps", ctypes.c_float), ("wd", ctypes.c_float), ("scale_const", ctypes.c_float),
        ("tensor_id", ctypes.c_uint32), ("step", ctypes.c_uint32), ("flags", ctypes.c_uint32),
        ("m_storage", ctypes.c_int32), ("v_storage", ctypes.c_int32), ("param_bf16", ctypes.c_int32),
        ("math_bf16", ctypes.c_int32), ("update_bf16", ctypes.c_int32),
        ("last_grad", ctypes.c_uint64), ("mars_factor", ctypes.c_float), ("nm_w", ctypes.c_float),
        ("nm_eps", ctypes.c_float), ("pad0", ctypes.c_int32),
        ("row_v", ctypes.c_uint64), ("row_den", ctypes.c_uint64),
        ("v_row", ctypes.c_uint64), ("v_col", ctypes.c_uint64), ("v_full", ctypes.c_uint64),
        ("v_sums", ctypes.c_uint64), ("d1", ctypes.c_int64), ("d2", ctypes.c_int64),
    ]


_LIB = None
_LOCK = threading.Lock()


class AdvOptError(RuntimeError):
    pass


def lib():
    """Load libadvopt.so once; raise if it is missing or its layout differs."""
    global _LIB
    if _LIB is not None:
        return _LIB
    with _LOCK:
        if _LIB is not None:
            return _LIB
        if not os.path.exists(LIB_PATH):
            raise AdvOptError(f"{LIB_PATH} is missing: build it with `python -m advanced_optimizers_b200.build` "
                              "(there is no CPU fallback)")
        L = ctypes.CDLL(LIB_PATH)
        P, I32, U32, F, U64 = ctypes.c_void_p, ctypes.c_int32, ctypes.c_uint32, ctypes.c_float, ctypes.c_uint64
        sig = {
            "advopt_adam_step": ([ctypes.POINTER(AdamLaunch), P], ctypes.c_int),
            "advopt_factored_finish": ([ctypes.POINTER(AdamLaunch), P, I32, I32, P], ctypes.c_int),
            "advopt_prodigy_finish": ([ctypes.POINTER(AdamLaunch), P, F, I32, P], ctypes.c_int),
            "advopt_fisher_finish": ([ctypes.POINTER(AdamLaunch), P, P], ctypes.c_int),
            "advopt_lion_step": ([P, I32, P, I32, I32, F, F, U32, U64, P], ctypes.c_int),
            "advopt_sizeof": ([ctypes.c_int], ctypes.c_size_t),
            "advopt_abi_version": ([], ctypes.c_int),
            "advopt_last_error": ([], ctypes.c_char_p),
            "advopt_adam_occupancy": ([I32, I32, I32, I32, I32, ctypes.POINTER(I32), ctypes.POINTER(I32)],
                                      ctypes.c_int),
            "advopt_adam_step_noalloc": ([P, ctypes.POINTER(AdamLaunch), P], ctypes.c_int),
            "advopt_ns_gemm": ([P, I32, P, I32, P, I32, I32, P, I32, I32, I32, I32, F, F, P, P], ctypes.c_int),
            "advopt_ns_gemm_sym": ([P, I32, P, I32, P, I32, I32, P, I32, I32, I32, F, F, P, P], ctypes.c_int),
            "advopt_muon_stage": ([ctypes.POINTER(MuonArgs), I32, P], ctypes.c_int),
            "advopt_philox4x32_10": ([P, P, ctypes.c_int64, P], ctypes.c_int),
            "advopt_ns_chain": ([P, P, P, P, I32, I32, I32, I32, ctypes.c_double, ctypes.c_double, ctypes.c_double,
                                 ctypes.c_double, ctypes.POINTER(ctypes.c_void_p), P, P], ctypes.c_int),
            "advopt_noise_fill": ([P, ctypes.c_int64, U64, U32, U32, U32, P], ctypes.c_int),
            "advopt_kourkoutas_prepare": ([ctypes.POINTER(KourkoutasArgs), P], ctypes.c_int),
            "advopt_kourkoutas_accumulate": ([ctypes.POINTER(KourkoutasArgs), P], ctypes.c_int),
            "advopt_prodigy_scalars": ([ctypes.POINTER(ProdigyScalarArgs), P], ctypes.c_int),
            "advopt_prodigy_update_d": ([ctypes.POINTER(ProdigyDArgs), P], ctypes.c_int),
            "advopt_lr_sketch": ([P, ctypes.c_int64, ctypes.c_int64, U64, U32, U32, P], ctypes.c_int),
            "advopt_lr_gemm": ([P, P, P, ctypes.c_int64, ctypes.c_int64, ctypes.c_int64, I32, P], ctypes.c_int),
            "advopt_lr_qr_work": ([ctypes.c_int64, ctypes.c_int64], ctypes.c_int64),
            "advopt_lr_qr": ([P, P, ctypes.c_int64, ctypes.c_int64, P, P], ctypes.c_int),
            "advopt_ipc_get_handle": ([P, P, ctypes.POINTER(U64)], ctypes.c_int),
            "advopt_ipc_open": ([P, ctypes.POINTER(ctypes.c_void_p)], ctypes.c_int),
            "advopt_ipc_close": ([P], ctypes.c_int),
            "advopt_enable_peer": ([I32], ctypes.c_int),
            "advopt_copy_async": ([P, P, U64, P], ctypes.c_int),
            "advopt_spectral_step": ([ctypes.POINTER(AdamLaunch), P, P, I32, P, I32, P], ctypes.c_int),
        }
        for name, (args, res) in sig.items():
            fn = getattr(L, name)
            fn.argtypes = args
            fn.restype = res
        if L.advopt_abi_version() != ABI_VERSION:
            raise AdvOptError("libadvopt.so ABI version mismatch; rebuild the library")
        for which, size in ((0, ADAM_TENSOR_DT.itemsize), (1, PIECE_DT.itemsize),
                            (2, ctypes.sizeof(AdamLaunch)), (3, LION_TENSOR_DT.itemsize),
                            (4, ctypes.sizeof(MuonArgs)), (5, ctypes.sizeof(KourkoutasArgs)),
                            (6, PRODIGY_DEV_BYTES), (7, ctypes.sizeof(ProdigyScalarArgs)),
                            (8, ctypes.sizeof(ProdigyDArgs)), (9, SPECTRAL_TENSOR_DT.itemsize)):
            got = L.advopt_sizeof(which)
            if got != size:
                raise AdvOptError(f"struct layout mismatch (#{which}: C {got} bytes, Python {size})")
        _LIB = L
        return L


def check(rc: int, what: str):
    if rc != 0:
        msg = lib().advopt_last_error().decode(errors="replace")
        raise AdvOptError(f"{what} failed ({rc}): {msg}")


def exported_symbols():
    """Names the header declares (used by the load test)."""
    return ["advopt_adam_step", "advopt_factored_finish", "advopt_prodigy_finish", "advopt_fisher_finish",
            "advopt_lion_step", "advopt_sizeof", "advopt_abi_version", "advopt_last_error",
            "advopt_adam_occupancy", "advopt_adam_step_noalloc", "advopt_ns_gemm", "advopt_ns_gemm_sym", "advopt_muon_stage", "advopt_philox4x32_10",
            "advopt_noise_fill", "advopt_ns_chain", "advopt_kourkoutas_prepare", "advopt_kourkoutas_accumulate",
            "advopt_prodigy_scalars", "advopt_prodigy_update_d", "advopt_lr_sketch", "advopt_lr_gemm",
            "advopt_lr_qr_work", "advopt_lr_qr", "advopt_ipc_get_handle", "advopt_ipc_open", "advopt_ipc_close",
            "advopt_enable_peer", "advopt_copy_async", "advopt_spectral_step"]


_OCC_CACHE = {}


def adam_occupancy(precision: int, param_dtype: int, algo: int, smem_floats: int, fast: bool = False):
    key = (precision, param_dtype, algo, smem_floats, bool(fast))
    if key not in _OCC_CACHE:
        sms, ctas = ctypes.c_int32(0), ctypes.c_int32(0)
        check(lib().advopt_adam_occupancy(precision, param_dtype, algo, smem_floats, 1 if fast else 0,
                                          ctypes.byref(sms), ctypes.byref(ctas)), "advopt_adam_occupancy")
        _OCC_CACHE[key] = (sms.value, max(1, ctas.value))
    return _OCC_CACHE[key]
