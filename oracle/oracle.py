"""ORACLE — test infrastructure only.

CPU restatement (numpy + the C primitives in ``orc_kernels.c``) of the
optimizer-step arithmetic of adv_optm 2.5.4 (``AdamW_adv``, ``Muon_adv``'s
auxiliary Adam, ``Prodigy_adv``, ``Lion_adv``, ``Muon_adv``, ``AdaMuon_adv``),
written op for op against the reference so that every rounding happens where
PyTorch's CPU kernels round.  Only ``tests/``, ``__graft_entry__.smoke()`` and
``bench.py``'s CPU-baseline leg import this module, and only as the checker or
the CPU baseline; the product (``advanced_optimizers_b200``) never does.

Pinned against the reference itself: ``tests/golden/make_golden.py`` runs the
reference on seeded inputs in a container that has it and records inputs, the
exact random integers it drew, and its outputs; ``tests/test_oracle_golden.py``
replays them through this module.

Values are numpy arrays.  bfloat16 tensors are held as float32 arrays whose
values are exactly representable in bf16 (``T.dt == 'bf16'``); conversion to
and from raw bf16 bits is explicit (``bf16_bits`` / ``from_bf16_bits``).
Optimizer states use the reference's state-dict keys and storage dtypes
(int8 / uint8 codes, float32 scales, bf16 as uint16 bits, fp32).

Random integers: the reference draws ``torch.randint(0, 2**16)`` int32 tensors
from one generator per device (param_update.py:181-204,240-264); every step
function here takes them as arguments (``noise[...]``), in the reference's
draw order, so the oracle is deterministic given the reference's draws.
"""
from __future__ import annotations

import ctypes
import math
import os
import subprocess
import threading

import numpy as np

BLOCK = 2048  # state_util.py:10
_HERE = os.path.dirname(os.path.abspath(__file__))
_LIB = None
_LOCK = threading.Lock()
f32 = np.float32


def _lib():
    global _LIB
    with _LOCK:
        if _LIB is None:
            path = os.path.join(_HERE, "liborc.so")
            if not os.path.exists(path):
                subprocess.check_call(["make", "-s", "-C", _HERE])
            lib = ctypes.CDLL(path)
            P = ctypes.c_void_p
            I = ctypes.c_int64
            F = ctypes.c_float
            for name, args in {
                "orc_lerp": [P, P, P, F, I],
                "orc_addcmul": [P, P, P, P, F, I],
                "orc_add_alpha": [P, P, P, F, I],
                "orc_round_bf16": [P, P, I],
                "orc_to_bf16_bits": [P, P, I],
                "orc_sr_bf16_bits": [P, P, P, I],
                "orc_quant_block": [P, P, P, P, I, I, ctypes.c_int],
                "orc_dequant_block": [P, P, P, I, I, ctypes.c_int],
                "orc_outer": [P, P, P, I, I],
                "orc_row_col_sums": [P, P, P, I, I],
                "orc_fma": [P, P, P, P, I],
            }.items():
                fn = getattr(lib, name)
                fn.argtypes = args
                fn.restype = None
            lib.orc_num_threads.restype = ctypes.c_int
            lib.orc_set_num_threads.argtypes = [ctypes.c_int]
            lib.orc_set_num_threads.restype = None
            _LIB = lib
    return _LIB


def num_threads() -> int:
    return int(_lib().orc_num_threads())


def set_num_threads(n: int) -> None:
    """Threads of the C primitives' OpenMP loops."""
    _lib().orc_set_num_threads(int(n))


def _c(a, dtype=np.float32):
    return np.ascontiguousarray(a, dtype=dtype)


def _ptr(a):
    return a.ctypes.data_as(ctypes.c_void_p)


# ---------------------------------------------------------------------------
# bf16 helpers
# ---------------------------------------------------------------------------

def round_bf16(x):
    x = _c(x)
    out = np.empty_like(x)
    _lib().orc_round_bf16(_ptr(out), _ptr(x), x.size)
    return out


def bf16_bits(x):
    """float32 values -> uint16 bf16 bits (round to nearest even)."""
    x = _c(x)
    out = np.empty(x.shape, np.uint16)
    _lib().orc_to_bf16_bits(_ptr(out), _ptr(x), x.size)
    return out


def from_bf16_bits(b):
    b = np.ascontiguousarray(b, dtype=np.uint16)
    return (b.astype(np.uint32) << 16).view(np.float32)


def sr_bf16_bits(x, r):
    """param_update._copy_stochastic_core_ (param_update.py:206-219)."""
    x = _c(x)
    r = _c(r, np.int32).reshape(x.shape)
    out = np.empty(x.shape, np.uint16)
    _lib().orc_sr_bf16_bits(_ptr(out), _ptr(x), _ptr(r), x.size)
    return out


# ---------------------------------------------------------------------------
# dtype-tagged values: float32 storage + the torch dtype the reference holds
# ---------------------------------------------------------------------------

class T:
    """A tensor value with torch semantics: every op computes in float32
    (ATen's opmath for bf16) and rounds its result to the result dtype."""

    __slots__ = ("v", "dt")

    def __init__(self, v, dt="f32"):
        v = _c(v)
        self.v = round_bf16(v) if dt == "bf16" else v
        self.dt = dt

    @staticmethod
    def _res(a, b=None):
        if b is None or not isinstance(b, T):
            return a.dt
        return "f32" if "f32" in (a.dt, b.dt) else "bf16"

    def to(self, dt):
        return T(self.v, dt)

    def clone(self):
        return T(self.v.copy(), self.dt)

    def mul_s(self, s):       # tensor * python scalar (scalar cast to float)
        return T(self.v * f32(s), self.dt)

    def div_s(self, s):       # tensor / python scalar: true division (pinned)
        return T(self.v / f32(s), self.dt)

    def add_s(self, s):
        return T(self.v + f32(s), self.dt)

    def mul(self, o, dt=None):
        return T(self.v * o.v, dt or self._res(self, o))

    def div(self, o, dt=None):
        return T(self.v / o.v, dt or self._res(self, o))

    def add(self, o, dt=None):
        return T(self.v + o.v, dt or self._res(self, o))

    def sqrt(self):
        return T(np.sqrt(self.v), self.dt)

    def neg(self):
        return T(-self.v, self.dt)

    def sign(self):
        return T(np.sign(self.v).astype(np.float32), self.dt)

    def atan2(self, o, dt=None):
        # float64 atan2 rounded once: within 1 ulp of ATen's (Sleef u10) result
        v = np.arctan2(self.v.astype(np.float64), o.v.astype(np.float64)).astype(np.float32)
        return T(v, dt or self._res(self, o))

    def lerp(self, end, w, dt=None):
        a, b = _c(self.v), _c(end.v)
        out = np.empty_like(a)
        _lib().orc_lerp(_ptr(out), _ptr(a), _ptr(b), f32(w), a.size)
        return T(out, dt or self.dt)

    def addcmul(self, t1, t2, value, dt=None):
        a, b, c = _c(self.v), _c(t1.v), _c(t2.v)
        out = np.empty_like(a)
        _lib().orc_addcmul(_ptr(out), _ptr(a), _ptr(b), _ptr(c), f32(value), a.size)
        return T(out, dt or self.dt)

    def add_alpha(self, other, alpha, dt=None):
        """self + alpha * other (add_ with alpha): between two bf16 tensors
        ATen first rounds alpha to bf16; otherwise alpha is float32."""
        a, b = _c(self.v), _c(other.v)
        out = np.empty_like(a)
        al = f32(alpha)
        if self.dt == "bf16" and other.dt == "bf16":
            al = f32(round_bf16(np.array([al], np.float32))[0])
        _lib().orc_add_alpha(_ptr(out), _ptr(a), _ptr(b), al, a.size)
        return T(out, dt or self.dt)


# ---------------------------------------------------------------------------
# state storage (state_util.py)
# ---------------------------------------------------------------------------

def padded(n):
    return ((n + BLOCK - 1) // BLOCK) * BLOCK


def quant_block(x, r, non_neg):
    """set_state(..., 'int8_sr') body: returns (codes, scales)."""
    x = _c(x).reshape(-1)
    n = x.size
    nb = (n + BLOCK - 1) // BLOCK
    r = _c(r, np.int32).reshape(-1)
    assert r.size >= n
    q = np.empty(n, np.uint8 if non_neg else np.int8)
    s = np.empty(nb, np.float32)
    _lib().orc_quant_block(_ptr(q), _ptr(s), _ptr(x), _ptr(r), n, BLOCK, 1 if non_neg else 0)
    return q, s


def dequant_block(q, scale, non_neg):
    q = np.ascontiguousarray(q).reshape(-1)
    out = np.empty(q.size, np.float32)
    _lib().orc_dequant_block(_ptr(out), _ptr(q), _ptr(_c(scale)), q.size, BLOCK, 1 if non_neg else 0)
    return out


def init_state_tensor(state, key, shape, precision, p_dt, non_neg=False):
    """state_util.py:13-37."""
    n = int(np.prod(shape)) if len(shape) else 1
    if precision == "fp32" or (precision == "auto" and p_dt == "f32"):
        state[key] = np.zeros(shape, np.float32)
    elif precision == "bf16_sr" or (precision == "auto" and p_dt == "bf16"):
        state[key] = np.zeros(shape, np.uint16)
    elif precision == "int8_sr":
        state[key] = np.zeros(shape, np.uint8 if non_neg else np.int8)
        state[key + "_scale"] = np.ones((n + BLOCK - 1) // BLOCK, np.float32)
    else:
        raise NotImplementedError(precision)


def get_state(state, key, precision, p_dt, non_neg=False):
    """state_util.py:40-56 -> T (fp32 except 'auto' with bf16 storage)."""
    t = state[key]
    if precision == "int8_sr":
        return T(dequant_block(t, state[key + "_scale"], non_neg).reshape(t.shape), "f32")
    if t.dtype == np.uint16:
        return T(from_bf16_bits(t), "f32" if precision == "bf16_sr" else "bf16")
    return T(t, "f32")


def set_state(state, key, value: T, precision, r, non_neg=False):
    """state_util.py:109-163."""
    shape = state[key].shape
    if precision == "int8_sr":
        q, s = quant_block(value.v, r, non_neg)
        state[key] = q.reshape(shape)
        state[key + "_scale"] = s
    elif precision == "bf16_sr":
        state[key] = sr_bf16_bits(value.v, r).reshape(shape)
    elif state[key].dtype == np.uint16:        # 'auto' with bf16 storage
        state[key] = bf16_bits(value.v).reshape(shape)
    else:
        state[key] = _c(value.v).reshape(shape).copy()


def upcast(grad: T, precision):
    """state_util.py:165-179 (non-factored optimizers)."""
    if precision in ("fp32", "bf16_sr", "int8_sr", "factored"):
        return grad.to("f32")
    return grad


# ---------------------------------------------------------------------------
# rank-1 factorisation (factorization_util.py)
# ---------------------------------------------------------------------------

def effective_shape(numel):
    """factorization_util.py:43-50."""
    if numel <= 0:
        return (0, 0)
    for i in range(int(numel ** 0.5), 0, -1):
        if numel % i == 0:
            return (numel // i, i)
    return (numel, 1)


def unnmf(row, col):
    row, col = _c(row), _c(col)
    out = np.empty((row.size, col.size), np.float32)
    _lib().orc_outer(_ptr(out), _ptr(row), _ptr(col), row.size, col.size)
    return out


def nnmf(matrix):
    """factorization_util.py:60-80.  Sums are exact-ish (float64) and rounded
    to float32; the reference's float32 cascade sums differ in the last bits."""
    m = _c(matrix)
    d1, d2 = m.shape
    rows = np.empty(d1, np.float64)
    cols = np.empty(d2, np.float64)
    _lib().orc_row_col_sums(_ptr(rows), _ptr(cols), _ptr(m), d1, d2)
    mu = rows.astype(np.float32)
    mv = cols.astype(np.float32)
    if d1 < d2:
        scale = max(f32(rows.sum()), f32(1e-12))
        mu = (mu / f32(scale)).astype(np.float32)
    else:
        scale = max(f32(cols.sum()), f32(1e-12))
        mv = (mv / f32(scale)).astype(np.float32)
    return mu, mv


SHIFTER = np.array([1, 2, 4, 8, 16, 32, 64, 128], np.uint8)


def pack_signs(mask):
    """_pack_bools (factorization_util.py:87-95): bit j of byte b of row i is
    column 8*b + j; the last byte of a row is zero-padded."""
    mask = np.asarray(mask, bool)
    d1, d2 = mask.shape
    pd2 = (d2 + 7) // 8
    pad = np.zeros((d1, pd2 * 8), np.uint8)
    pad[:, :d2] = mask
    return (pad.reshape(d1, pd2, 8) * SHIFTER).sum(axis=2, dtype=np.uint8)


def unpack_signs(packed, d2):
    """_unpack_bools (factorization_util.py:98-104)."""
    packed = np.asarray(packed, np.uint8)
    return ((packed[:, :, None] & SHIFTER[None, None, :]) != 0).reshape(packed.shape[0], -1)[:, :d2]


def reconstruct_signed(mu, mv, sign, d2):
    """_reconstruct_state(signed=True) (factorization_util.py:9-19):
    outer(mu, mv), negated where the sign bit is clear."""
    full = unnmf(mu, mv)
    return np.where(unpack_signs(sign, d2), full, -full).astype(np.float32)


def factorize_signed(m):
    """_factorize_state(signed=True) (factorization_util.py:25-32):
    (mu, mv, sign) of a full momentum; the sign bit is m > 0."""
    m = np.asarray(m, np.float32)
    sign = pack_signs(m > 0)
    mu, mv = nnmf(np.abs(m))
    return mu, mv, sign


def init_factored(st, shape, has_m, m_keys=("mu_m_nmf", "mv_m_nmf", "sign")):
    """The 'factored' state of one tensor (AdamW_adv.py:242-256): signed
    rank-1 m (when betas[0] > 0) and rank-1 v over the effective shape."""
    d1, d2 = effective_shape(int(np.prod(shape)))
    st["factored"] = True
    st["effective_shape"] = (d1, d2)
    if has_m:
        st[m_keys[0]] = np.zeros(d1, np.float32)
        st[m_keys[1]] = np.zeros(d2, np.float32)
        st[m_keys[2]] = np.zeros((d1, (d2 + 7) // 8), np.uint8)
        st["shifter"] = SHIFTER.copy()


# ---------------------------------------------------------------------------
# weight decay and the final update (param_update.py:15-156)
# ---------------------------------------------------------------------------

def f32_to_e4m3fn(x):
    """float32 -> float8_e4m3fn codes (uint8), round to nearest even, as
    torch's p.to(torch.float8_e4m3fn) (centered_decay.py:55-57): 1 sign, 4
    exponent (bias 7) and 3 mantissa bits, subnormals down to 2^-9, largest
    finite 448; no infinity, so magnitudes that round above 448 become the
    NaN code 0x7F (the conversion does not saturate)."""
    x = np.asarray(x, np.float32).reshape(-1)
    sign = np.where(np.signbit(x), 0x80, 0).astype(np.uint8)
    a = np.abs(x.astype(np.float64))
    code = np.zeros(a.shape, np.int64)
    nan = np.isnan(a)
    a = np.where(nan, 0.0, a)
    sub = a < 2.0 ** -6
    q_sub = np.rint(a / 2.0 ** -9).astype(np.int64)            # 0..8 (8 = the smallest normal)
    _, e = np.frexp(np.where(sub, 1.0, a))                      # a = f * 2^e, f in [0.5, 1)
    E = e - 1                                                   # a in [2^E, 2^(E+1))
    q = np.rint(np.where(sub, 8.0, a) / np.ldexp(1.0, E - 3)).astype(np.int64)   # 8..16
    E = np.where(q == 16, E + 1, E)
    q = np.where(q == 16, 8, q)
    normal_code = ((E + 7) << 3) | (q - 8)
    code = np.where(sub, q_sub, normal_code)
    big = (~sub) & ((E > 8) | ((E == 8) & (q - 8 > 6)))         # above 448: NaN
    code = np.where(big | nan, 0x7F, code)
    return (code.astype(np.uint8) | sign)


def e4m3fn_to_f32(b):
    """float8_e4m3fn codes -> float32 values (exact)."""
    b = np.asarray(b, np.uint8).astype(np.int64)
    s = np.where(b & 0x80, -1.0, 1.0)
    e = (b >> 3) & 0xF
    m = b & 0x7
    v = np.where(e == 0, m * 2.0 ** -9, (1.0 + m / 8.0) * np.ldexp(1.0, e - 7))
    v = np.where((e == 0xF) & (m == 0x7), np.nan, v)
    return (s * v).astype(np.float32)


def dequantize_anchor(state, mode, n):
    """centered_decay.py:78-119 (float32 result)."""
    data = state["anchor_data"]
    if data.dtype == np.uint8:
        # float8_e4m3fn storage: anchor_data.to(dtype) is exact
        return e4m3fn_to_f32(data).reshape(-1)[:n]
    if mode in ("full", "float8") or data.dtype in (np.float32, np.uint16):
        if data.dtype == np.uint16:
            return from_bf16_bits(data).reshape(-1)[:n]
        return _c(data).reshape(-1)[:n]
    sc, mi = state["anchor_scale"], state["anchor_min"]
    scales = from_bf16_bits(sc) if sc.dtype == np.uint16 else _c(sc)
    mins = from_bf16_bits(mi) if mi.dtype == np.uint16 else _c(mi)
    if mode == "int4":
        d = data.reshape(-1).astype(np.int8)
        hi = (d >> 4).astype(np.int8)
        lo = ((d << 4).astype(np.int8) >> 4).astype(np.int8)
        q = np.empty(d.size * 2, np.int8)
        q[0::2], q[1::2] = hi, lo
        blk, qmin = 32, -8
    else:
        q = data.reshape(-1).astype(np.int8)
        blk, qmin = 128, -128
    qb = q.reshape(-1, blk).astype(np.float32)
    out = (qb - f32(qmin)) * scales[:, None] + mins[:, None]
    return out.reshape(-1)[:n].astype(np.float32)


def apply_parameter_update(p, p_dt, update: T, state, *, lr, wd, cautious, sr, r_param,
                           wd_scaler=None, cwd=0.0, cwd_mode="float8", init_lr=None,
                           decoupled=False):
    """param_update.py:77-156 for one tensor.  `p` is float32 values (bf16
    values when p_dt == 'bf16'); returns the new float32 values (exact bf16
    values for bf16 params)."""
    decay_factor = (lr / init_lr) if decoupled else lr
    scaled_wd = (wd * decay_factor) if wd != 0 else None
    scaled_cwd = (cwd * decay_factor) if cwd != 0 else None
    if wd_scaler is not None:
        if scaled_wd is not None:
            scaled_wd = T(wd_scaler.v * f32(scaled_wd), "f32")
        if scaled_cwd is not None:
            scaled_cwd = T(wd_scaler.v * f32(scaled_cwd), "f32")
    if p_dt == "bf16" and sr:
        pc = T(p, "f32")
        uc = update.to("f32")
        pc = _apply_weight_decay(pc, uc, state, scaled_wd, scaled_cwd, cautious, cwd_mode)
        pc = pc.add(uc.neg())
        bits = sr_bf16_bits(pc.v, r_param)
        return from_bf16_bits(bits).reshape(np.shape(p))
    pc = T(p, p_dt)
    pc = _apply_weight_decay(pc, update, state, scaled_wd, scaled_cwd, cautious, cwd_mode)
    pc = pc.add(update.neg(), dt=p_dt)
    return pc.v.reshape(np.shape(p))


def _apply_weight_decay(pc: T, uc: T, state, scaled_wd, scaled_cwd, cautious, cwd_mode):
    """param_update.py:15-75."""
    if scaled_wd is not None:
        tgt = pc
        if cautious:
            mask = T((uc.v * tgt.v >= 0).astype(np.float32), pc.dt)
            if isinstance(scaled_wd, T):
                pc = pc.addcmul(tgt, mask.mul(scaled_wd, dt=pc.dt), -1.0)
            else:
                pc = pc.addcmul(tgt, mask, -scaled_wd)
        else:
            if isinstance(scaled_wd, T):
                pc = pc.addcmul(tgt, scaled_wd, -1.0)
            else:
                pc = pc.add_alpha(tgt, -scaled_wd)
    if scaled_cwd is not None and "anchor_data" in state:
        anchor = T(dequantize_anchor(state, cwd_mode, pc.v.size).reshape(pc.v.shape), pc.dt)
        target = pc.add(anchor.neg(), dt=pc.dt)
        if cautious:
            mask = T((uc.v * target.v >= 0).astype(np.float32), pc.dt)
            if isinstance(scaled_cwd, T):
                pc = pc.addcmul(target, mask.mul(scaled_cwd, dt=pc.dt), -1.0)
            else:
                pc = pc.addcmul(target, mask, -scaled_cwd)
        else:
            if isinstance(scaled_cwd, T):
                pc = pc.addcmul(target, scaled_cwd, -1.0)
            else:
                pc = pc.add_alpha(target, -scaled_cwd)
    return pc


def _rdiv(s, t: T) -> T:
    """python scalar / tensor: torch evaluates it as reciprocal(t) * s."""
    return T(f32(1.0) / t.v, t.dt).mul_s(s)


def _state_vals(a):
    return (from_bf16_bits(a), "bf16") if a.dtype == np.uint16 else (np.asarray(a, np.float32), "f32")


def _store_like(a, v):
    return bf16_bits(v).reshape(a.shape) if a.dtype == np.uint16 else np.asarray(v, np.float32).reshape(a.shape)


def max_abs_normalization(upd: T, lr) -> T:
    """scaled_optm.py:160-168: update * (lr / max(|update|)), in the update's dtype."""
    norm = T(np.maximum(np.max(np.abs(upd.v)), f32(1e-12)).reshape(1), upd.dt)
    return T(upd.v * _rdiv(lr, norm).v[0], upd.dt)


def spectral_normalization(upd: T, state, lr, target_scale) -> T:
    """scaled_optm.py:255-295: one power-iteration step on the update viewed
    as (d_out, d_in) in the singular vectors' dtype, then
    update * lr * target_scale / max(sigma, 1/(sqrt(d_out)+sqrt(d_in))).
    The matrix-vector products and norms are summed in float64 and rounded
    once to that dtype (the reference's accumulation order is not pinned)."""
    u0, sdt = _state_vals(state["spectral_u"])
    v0, _ = _state_vals(state["spectral_v"])
    d_out = u0.size
    d_in = upd.v.size // d_out
    U = upd.to(sdt).v.reshape(d_out, d_in)
    U64 = U.astype(np.float64)

    def rnd(x):
        return T(np.asarray(x, np.float32).reshape(-1), sdt).v

    v_raw = rnd(U64.T @ u0.astype(np.float64))
    v_norm = rnd(np.sqrt(np.sum(v_raw.astype(np.float64) ** 2)))[0]
    cand_v = rnd(v_raw / np.maximum(v_norm, rnd(1e-8)[0]))
    next_v = cand_v if v_norm >= 1e-6 else v0
    state["spectral_v"] = _store_like(state["spectral_v"], next_v)
    u_raw = rnd(U64 @ next_v.astype(np.float64))
    u_norm = rnd(np.sqrt(np.sum(u_raw.astype(np.float64) ** 2)))[0]
    cand_u = rnd(u_raw / np.maximum(u_norm, rnd(1e-8)[0]))
    next_u = cand_u if u_norm >= 1e-6 else u0
    state["spectral_u"] = _store_like(state["spectral_u"], next_u)
    # linalg.vecdot is (u * u_raw).sum(): each product rounded to the dtype
    sigma = rnd(np.sum(rnd(next_u * u_raw).astype(np.float64)))[0]
    eps = 1.0 / (math.sqrt(d_out) + math.sqrt(d_in))
    sig = T(np.array([sigma if sigma >= eps else eps], np.float32), sdt)     # clamp_min_(eps)
    scale = _rdiv(target_scale, sig).mul_s(lr)
    return T(U.reshape(-1) * scale.v[0], sdt)


def scale_update(shape, upd: T, lr, state) -> T:
    """scale_update (scaled_optm.py:35-72) for params without DoRA / OFT /
    LoRA markers: max-abs scaling for 1-D, spectral scaling with target
    sqrt(d_out / d_in) otherwise."""
    if len(shape) < 2:
        return max_abs_normalization(upd, lr)
    d_out = shape[0]
    d_in = int(np.prod(shape)) // d_out
    out = spectral_normalization(upd, state, lr, math.sqrt(d_out / d_in))
    return T(out.v.reshape(upd.v.shape), out.dt)


def fisher_wd_scaler(p: T, denom: T, atan2: bool):
    """update_util.py:15-36 (AdamW/Prodigy call it with eps=None)."""
    if atan2:
        ws = T(np.arctan2(1.0, denom.v.astype(np.float64)).astype(np.float32) * f32(4 / math.pi), "f32")
        return ws
    ws = T(f32(1.0) / denom.v, denom.dt)
    pw = p.mul(ws)
    gw_rms = np.sqrt(np.mean((pw.v.astype(np.float32) ** 2).astype(np.float64)).astype(np.float32))
    clip = max(f32(gw_rms), f32(1.0))
    return T(ws.v / f32(clip), ws.dt)


def init_anchor(p_vals, p_dt, mode):
    """centered_decay.py:43-76 -> dict of anchor state entries."""
    st = {}
    flat = _c(p_vals).reshape(-1)
    if mode == "full":
        st["anchor_data"] = bf16_bits(flat).reshape(np.shape(p_vals)) if p_dt == "bf16" else flat.reshape(np.shape(p_vals)).copy()
        return st
    if mode == "float8":
        st["anchor_data"] = f32_to_e4m3fn(flat).reshape(np.shape(p_vals))
        return st
    blk, bits = (128, 8) if mode == "int8" else (32, 4)
    n = flat.size
    pad = (blk - n % blk) % blk
    vals = np.concatenate([flat, np.full(pad, flat[-1], np.float32)]) if pad else flat.copy()
    vb = vals.reshape(-1, blk)
    mn, mx = vb.min(1, keepdims=True), vb.max(1, keepdims=True)
    qmin, qmax = -(1 << (bits - 1)), (1 << (bits - 1)) - 1
    scales = ((mx - mn) / f32(qmax - qmin)).astype(np.float32)
    scales[scales == 0] = 1.0
    q = np.clip(np.round((vb - mn) / scales + f32(qmin)), qmin, qmax).astype(np.int8)
    if mode == "int4":
        qf = q.reshape(-1)
        packed = ((qf[0::2] & 0x0F) << 4) | (qf[1::2] & 0x0F)
        st["anchor_data"] = packed.astype(np.int8)
    else:
        st["anchor_data"] = q
    if p_dt == "bf16":
        st["anchor_scale"] = bf16_bits(scales.reshape(-1))
        st["anchor_min"] = bf16_bits(mn.reshape(-1))
    else:
        st["anchor_scale"] = scales.reshape(-1).astype(np.float32)
        st["anchor_min"] = mn.reshape(-1).astype(np.float32)
    return st


# ---------------------------------------------------------------------------
# AdamW_adv (and Muon's auxiliary Adam)
# ---------------------------------------------------------------------------

def adamw_init_state(shape, p_dt, precision, factored_2nd, beta1, vector_reshape=False):
    """AdamW_adv.py:221-277.  Under 'factored' a 2-D (or larger) param keeps
    signed rank-1 m and rank-1 v; a 1-D one float32 m and v."""
    st = {"step": 0}
    is_vector = len(shape) == 1 and not vector_reshape
    st["factored"] = False
    if precision == "factored":
        if not is_vector:
            init_factored(st, shape, beta1 > 0)
            st["mu_v_nmf"] = np.zeros(st["effective_shape"][0], np.float32)
            st["mv_v_nmf"] = np.zeros(st["effective_shape"][1], np.float32)
            return st
        precision = "fp32"
    st["factored_2nd"] = bool(factored_2nd and not is_vector)
    if beta1 > 0:
        init_state_tensor(st, "exp_avg", shape, precision, p_dt)
    if st["factored_2nd"]:
        d1, d2 = effective_shape(int(np.prod(shape)))
        st["effective_shape"] = (d1, d2)
        st["mu_v_nmf"] = np.zeros(d1, np.float32)
        st["mv_v_nmf"] = np.zeros(d2, np.float32)
        st["shifter"] = np.array([1, 2, 4, 8, 16, 32, 64, 128], np.uint8)
    else:
        init_state_tensor(st, "exp_avg_sq", shape, precision, p_dt, non_neg=True)
    return st


def adam_family_step(p, p_dt, g, state, hp, noise, *, algo="adamw"):
    """One tensor's step.

    algo='adamw'   : AdamW_adv.step_parameter/_step_parameter (AdamW_adv.py:279-465)
    algo='auxadam' : Muon_AuxAdam._adam_step_parameter (Muon_AuxAdam.py:70-192),
                     called from Muon_adv.py:377-415 (m before v)
    algo='prodigy' : Prodigy_adv._step_parameter (Prodigy_adv.py:372-519);
                     returns the (d_numerator, d_denom) contributions.

    `p` / `g`: float32 values (bf16 values when p_dt == 'bf16').  `noise`
    maps 'exp_avg_sq', 'exp_avg', 'param' to the int32 draws the reference
    makes for them.  Returns new p values (and prodigy stats).
    """
    prec = hp["precision"]           # group['actual_state_precision']
    grad_prec = prec
    if prec == "factored":
        # float32 states and math for every tensor of a 'factored' group
        # (state_util.py:165-179; AdamW_adv.py:236-239)
        prec = "fp32"
    beta1, beta2 = hp["betas"]
    step = state["step"]
    factored_2nd = state.get("factored_2nd", False)
    nesterov = hp.get("nesterov", False)
    nv_coef = hp.get("nesterov_coef")
    use_mt = beta1 > 0
    atan2 = hp.get("use_atan2", False)
    normed = hp.get("normed_momentum", False) and algo == "adamw"
    eps = hp["eps"] if hp["eps"] is not None else 1.0 / math.sqrt(g.size)   # scaled_optm.py:75-82
    if algo == "prodigy":
        d = hp["d"]
        dlr = d * hp["lr"]
        step_size = dlr
        sqrt_bc2 = None
    else:
        if hp.get("use_bias_correction", True):
            s1 = step + 1
            bc1 = 1.0 - beta1 ** s1
            sqrt_bc2 = (1.0 - beta2 ** s1) ** 0.5
        else:
            bc1, sqrt_bc2 = 1, 1
        step_size = hp["lr"] / bc1
    grad = upcast(T(g, p_dt), grad_prec)
    shape = np.shape(p)
    if "kourkoutas" in hp:
        # the grad's squared norm for the next step's beta2 (AdamW_adv.py:336-338)
        hp["kourkoutas"].accumulate(shape, grad)

    def v_path():
        if factored_2nd:
            d1, d2 = state["effective_shape"]
            v = T(unnmf(state["mu_v_nmf"], state["mv_v_nmf"]).reshape(shape), "f32")
            gv = grad.to("f32")
        else:
            v = get_state(state, "exp_avg_sq", prec, p_dt, non_neg=True)
            gv = grad
        # Kourkoutas-beta replaces beta2 in the v update only (the bias
        # correction keeps group['betas'][1]; AdamW_adv.py:291-304)
        b2 = hp.get("beta2_dyn", beta2)
        if algo == "prodigy":
            v = v.mul_s(b2).addcmul(gv, gv, d * d * (1.0 - b2))
        else:
            v = v.mul_s(b2).addcmul(gv, gv, 1.0 - b2)
        if factored_2nd:
            d1, d2 = state["effective_shape"]
            state["mu_v_nmf"], state["mv_v_nmf"] = nnmf(np.abs(v.v).reshape(d1, d2))
            v = T(np.abs(v.v), v.dt)
        else:
            set_state(state, "exp_avg_sq", v, prec, noise.get("exp_avg_sq"), non_neg=True)
        return v

    def m_path(grad):
        m = get_state(state, "exp_avg", prec, p_dt)
        if algo == "prodigy":
            m = m.mul_s(beta1).add_alpha(grad, d * (1.0 - beta1))
        else:
            m = m.lerp(grad, 1.0 - beta1)
        upd = m.clone()
        if nesterov:
            c = beta1 if nv_coef is None else nv_coef
            upd = upd.lerp(grad, 1 - c)
        set_state(state, "exp_avg", m, prec, noise.get("exp_avg"))
        return upd

    def make_denom(v):
        den = v.sqrt()
        if algo == "prodigy":
            if not atan2:
                den = den.add_s(d * eps)
        else:
            den = den.div_s(sqrt_bc2)
            if not atan2:
                den = den.add_s(eps)
        return den

    if state.get("factored", False):
        # state_precision='factored' (AdamW_adv.py:342-399, Muon_AuxAdam.py:86-133,
        # Prodigy_adv.py:387-434): m rebuilt from its signed rank-1 factors,
        # v from its rank-1 factors, both refactorised after their update
        d1, d2 = state["effective_shape"]
        gv = T(grad.to("f32").v.reshape(d1, d2), "f32")
        b2 = hp.get("beta2_dyn", beta2)

        def fm(gin):
            m = T(reconstruct_signed(state["mu_m_nmf"], state["mv_m_nmf"], state["sign"], d2), "f32")
            if algo == "prodigy":
                m = m.mul_s(beta1).add_alpha(gin, d * (1.0 - beta1))
            else:
                m = m.lerp(gin, 1.0 - beta1)
            state["mu_m_nmf"], state["mv_m_nmf"], state["sign"] = factorize_signed(m.v)
            if nesterov:
                c = beta1 if nv_coef is None else nv_coef
                m = m.lerp(gin, 1 - c)
            return m

        def fv():
            v = T(unnmf(state["mu_v_nmf"], state["mv_v_nmf"]), "f32")
            v = v.mul_s(b2).addcmul(gv, gv, (d * d * (1.0 - b2)) if algo == "prodigy" else (1.0 - b2))
            state["mu_v_nmf"], state["mv_v_nmf"] = nnmf(np.abs(v.v))
            return T(np.abs(v.v), "f32")

        if algo == "adamw":
            v = fv()
            den = make_denom(v)
            if normed:
                gv = gv.atan2(den) if atan2 else gv.div(den)
            upd = fm(gv) if use_mt else gv.clone()
        else:
            upd = fm(gv) if use_mt else None
            v = fv()
            den = make_denom(v)
            if upd is None:
                upd = gv.mul_s(d) if algo == "prodigy" else gv.clone()
        if not normed:
            upd = upd.atan2(den) if atan2 else upd.div(den)
        upd = T(upd.v.reshape(shape), upd.dt)
        den = T(den.v.reshape(shape), den.dt)
        normed = True    # the division is done
    elif algo == "auxadam":                   # Muon_AuxAdam.py:139-180
        upd = m_path(grad) if use_mt else grad.clone()
        v = v_path()
        den = make_denom(v)
    else:                                     # AdamW_adv.py:405-447
        if algo == "prodigy" and use_mt:
            upd = m_path(grad)
            v = v_path()
            den = make_denom(v)
        else:
            v = v_path()
            den = make_denom(v)
            if normed:
                grad = grad.atan2(den.to(grad.dt), dt=grad.dt) if atan2 else grad.div(den.to(grad.dt), dt=grad.dt)
            if use_mt:
                upd = m_path(grad)
            else:
                upd = grad.clone() if algo != "prodigy" else grad.mul_s(d)
        if algo == "prodigy" and not use_mt:
            pass
    if not normed:
        dd = den.to(upd.dt)
        upd = upd.atan2(dd, dt=upd.dt) if atan2 else upd.div(dd, dt=upd.dt)
    wd_scaler = None
    if hp.get("fisher_wd", False):
        wd_scaler = fisher_wd_scaler(T(p, p_dt), den, atan2)
    scaling = step_size * (4 / math.pi) if atan2 else step_size
    if hp.get("spectral", False):
        upd = scale_update(shape, upd, scaling, state)   # AdamW_adv.py:459-463
    else:
        upd = upd.mul_s(scaling)

    stats = None
    if algo == "prodigy":                      # Prodigy_adv.py:495-511
        if hp["prodigy_steps"] <= 0 or hp["k"] < hp["prodigy_steps"]:
            sp = hp["slice_p"]
            d0 = hp["d0"]
            gs = grad.v.reshape(-1)[::sp].astype(np.float32)
            ps = np.asarray(p, np.float32).reshape(-1)[::sp]
            p0 = from_bf16_bits(state["p0"]).reshape(-1) if state["p0"].dtype == np.uint16 else _c(state["p0"]).reshape(-1)
            dot = np.float32(np.dot((p0 - ps).astype(np.float64), gs.astype(np.float64)))
            num = f32(f32((d / d0) * dlr) * dot)
            alpha = ((d / d0) * d) if hp["safeguard_warmup"] else ((d / d0) * dlr)
            s_dt = "bf16" if state["s"].dtype == np.uint16 else "f32"
            s = T(from_bf16_bits(state["s"]) if s_dt == "bf16" else state["s"], s_dt)
            s = s.mul_s(hp["beta3"]).add_alpha(T(gs, "f32"), alpha, dt=s_dt)
            state["s"] = bf16_bits(s.v) if s_dt == "bf16" else s.v.copy()
            den_sum = np.abs(s.v).astype(np.float64).sum()
            den_sum = float(round_bf16(np.float32(den_sum).reshape(1))[0]) if s_dt == "bf16" else float(np.float32(den_sum))
            stats = (float(num), den_sum)

    lr_for_wd = dlr if algo == "prodigy" else hp["lr"]
    wd = hp.get("weight_decay", 0.0)
    newp = apply_parameter_update(p, p_dt, upd, state, lr=lr_for_wd, wd=wd,
                                  cautious=hp.get("cautious_wd", False),
                                  sr=hp.get("stochastic_rounding", True),
                                  r_param=noise.get("param"), wd_scaler=wd_scaler,
                                  cwd=hp.get("centered_wd", 0.0),
                                  cwd_mode=hp.get("centered_wd_mode", "float8"))
    state["step"] = step + 1
    return (newp, stats) if algo == "prodigy" else newp


def prodigy_calculate_d(group, d_numerator, d_denom):
    """Prodigy_adv.py:540-576 plus init_step's reset (:246-257), for one
    group dict holding d, d0, d_max, d_coef, growth_rate, d_limiter, k,
    prodigy_steps, beta3.  d_numerator/d_denom are the float32 sums."""
    active = not (group.get("prodigy_steps", 0) > 0 and group["k"] >= group["prodigy_steps"])
    if active:
        d_max, d_coef, growth = group["d_max"], group["d_coef"], group["growth_rate"]
        gn, gd = float(np.float32(d_numerator)), float(np.float32(d_denom))
        if gd > 0:
            d_hat = d_coef * gn / gd
            if group.get("d_limiter", False):
                d_hat = min(group["d"] * (2 ** 0.25), d_hat)
            if group["d"] == group["d0"]:
                group["d"] = max(group["d"], d_hat)
            d_max = max(d_max, d_hat)
            group["d"] = min(d_max, group["d"] * growth)
        group["d_numerator"] = gn
        group["d_max"] = d_max
    group["k"] += 1
    return float(np.float32(group["d_numerator"] * group["beta3"]))


# ---------------------------------------------------------------------------
# Lion_adv (Lion_adv.py:213-278, lion_k.py:5-24)
# ---------------------------------------------------------------------------

def lion_init_state(shape, p_dt, nnmf_factor, vector_reshape=False):
    """Lion_adv.py:156-181: signed rank-1 m for 2-D params under nnmf_factor,
    else m in the param dtype."""
    st = {"step": 0}
    if nnmf_factor and not (len(shape) == 1 and not vector_reshape):
        init_factored(st, shape, True)
    else:
        st["factored"] = False
        st["exp_avg"] = np.zeros(shape, np.uint16 if p_dt == "bf16" else np.float32)
    return st


def lion_step(p, p_dt, g, state, hp, noise):
    beta1, beta2 = hp["betas"]
    grad = T(g, p_dt)
    shape = np.shape(p)
    if state.get("factored", False):
        # Lion_adv.py:232-254: float32 grad, m from its signed rank-1 factors
        d1, d2 = state["effective_shape"]
        gv = T(grad.v.reshape(d1, d2), "f32")
        m = T(reconstruct_signed(state["mu_m_nmf"], state["mv_m_nmf"], state["sign"], d2), "f32")
        upd = gv.lerp(m, beta1)
        m = m.lerp(gv, 1 - beta2)
        state["mu_m_nmf"], state["mv_m_nmf"], state["sign"] = factorize_signed(m.v)
        upd = T(upd.v.reshape(shape), "f32")
    else:
        m = T(from_bf16_bits(state["exp_avg"]) if state["exp_avg"].dtype == np.uint16 else state["exp_avg"], p_dt)
        upd = grad.lerp(m, beta1)
        m = m.lerp(grad, 1 - beta2)
        state["exp_avg"] = bf16_bits(m.v) if p_dt == "bf16" else m.v.copy()
    upd = upd.sign()
    if hp.get("spectral", False):
        upd = scale_update(shape, upd, hp["lr"], state)    # Lion_adv.py:273-276
    else:
        upd = upd.mul_s(hp["lr"])
    state["step"] = state.get("step", 0) + 1
    return apply_parameter_update(p, p_dt, upd, state, lr=hp["lr"], wd=hp.get("weight_decay", 0.0),
                                  cautious=hp.get("cautious_wd", False),
                                  sr=hp.get("stochastic_rounding", True), r_param=noise.get("param"))


# ---------------------------------------------------------------------------
# Newton–Schulz (Muon_util.py:7-121,192-237)
# ---------------------------------------------------------------------------

def cans_coeffs(steps, a_bound):
    """CANS coefficient recursion, Muon_util.py:69-105."""
    lb, ub = a_bound, 1.0
    out = []
    for _ in range(steps):
        lb_ub = lb * ub
        e_sq = (lb * lb + lb_ub + ub * ub) / 3.0
        K = 2.0 * e_sq ** 1.5
        L = lb_ub * (lb + ub)
        den = K + L
        alpha = 6.0 / den
        out.append((alpha * e_sq, -alpha / 3.0))
        eps_val = (K - L) / den
        lb, ub = 1.0 - eps_val, 1.0 + eps_val
    return out


def default_cns_bound(M, N):
    """Muon_util.py:229-237."""
    return max(1.0 / math.sqrt(M * N), abs(1.0 / math.sqrt(N) - 1.0 / math.sqrt(M)))


def _mm_bf16(a, b, alpha=1.0, beta=0.0, c=None):
    """bf16 addmm: float32 accumulation, alpha/beta applied in float32, one
    rounding of the output to bf16."""
    acc = np.matmul(a.astype(np.float32), b.astype(np.float32))
    if beta != 0.0 and c is not None:
        out = f32(alpha) * acc + f32(beta) * c.astype(np.float32)
    else:
        out = f32(alpha) * acc
    return round_bf16(out)


def _mm_dt(a, b, dt):
    """torch.matmul in `dt`: bf16 operands accumulate in float32 and round the
    output once to bf16; float32 is a float32 product."""
    out = np.matmul(a.astype(np.float32), b.astype(np.float32)).astype(np.float32)
    return round_bf16(out) if dt == "bf16" else out


def low_rank_newton_schulz(G: T, sketch, steps, eps, coeffs, cns, cns_a_bound):
    """Muon_util.newton_schulz, low-rank path (Muon_util.py:239-270): MG =
    G @ sketch, Q from the QR of MG in float32 (cast back to G's dtype), the
    chain on Q^T G, then Q @ result.  eps and the CANS bound come from G's
    full shape.  QR is unique up to the signs of Q's columns, and the result
    does not depend on them (NS(D X) = D NS(X) for a diagonal D of +-1)."""
    M = G.v
    S = from_bf16_bits(sketch) if G.dt == "bf16" else np.asarray(sketch, np.float32)
    S = S.reshape(M.shape[1], -1)
    MG = _mm_dt(M, S, G.dt)
    Q, _ = np.linalg.qr(MG.astype(np.float32))
    Q = Q.astype(np.float32)
    if G.dt == "bf16":
        Q = round_bf16(Q)
    P = T(_mm_dt(Q.T, M, G.dt), G.dt)
    O = newton_schulz(P, steps, eps, coeffs, cns, cns_a_bound)
    return T(_mm_dt(Q, O.v, G.dt), G.dt)


def newton_schulz(G: T, steps=5, eps=1e-7, coeffs=(3.4445, -4.7750, 2.0315), cns=False, cns_a_bound=None,
                  sketch=None):
    """Muon_util.newton_schulz / _newton_schulz_iteration (standard path, or
    the low-rank path when a sketch is given): returns T in G's dtype."""
    M, N = G.v.shape
    if eps is None:
        eps = 1 / math.sqrt(G.v.size)
    if cns_a_bound is None:
        cns_a_bound = default_cns_bound(M, N)
    if sketch is not None:
        return low_rank_newton_schulz(G, sketch, steps, eps, coeffs, cns, cns_a_bound)
    X = round_bf16(G.v)
    transposed = X.shape[0] > X.shape[1]
    if transposed:
        X = np.ascontiguousarray(X.T)
    nrm = round_bf16(np.float32(np.sqrt((X.astype(np.float64) ** 2).sum())).reshape(1))[0]
    nrm = max(nrm, float(round_bf16(np.float32(eps).reshape(1))[0]))
    X = round_bf16(X / f32(nrm))
    a, b, c = coeffs
    if cns:
        for c1, c3 in cans_coeffs(steps, cns_a_bound):
            A = _mm_bf16(X, X.T)
            X = _mm_bf16(A, X, alpha=c3, beta=c1, c=X)
    else:
        for _ in range(steps):
            A = _mm_bf16(X, X.T)
            B = _mm_bf16(A, A, alpha=c, beta=b, c=A)
            X = _mm_bf16(B, X, alpha=1.0, beta=a, c=X)
    if transposed:
        X = np.ascontiguousarray(X.T)
    return T(X, "bf16").to(G.dt)


def rms_adjustment(u: T, rms_rescaling, lr):
    """Muon_util.py:362-372 (python float / 0-dim tensor = reciprocal * scalar)."""
    if rms_rescaling:
        norm = np.sqrt((u.v.astype(np.float64) ** 2).sum())
        nt = T(np.float32(norm).reshape(1), u.dt)
        nt = T(np.maximum(nt.v, f32(1e-8)), u.dt)
        recip = T(f32(1.0) / nt.v, u.dt)
        scale = recip.mul_s(lr * 0.2 * math.sqrt(u.v.size))
        return T(u.v * scale.v[0], u.dt)
    r, c = u.v.shape[-2], u.v.shape[-1]
    return u.mul_s(lr * math.sqrt(max(1, r / c)))


def approx_mars(grad: T, state, p_dt, mars_gamma, beta1):
    """Muon_util.approx_mars (Muon_util.py:333-347): c = (g - last).mul_(f).add_(g)
    with f = gamma * beta1 / (1 - beta1), each op rounding to the grad's dtype;
    last_grad (the param's dtype) takes the current grad."""
    f = mars_gamma * beta1 / (1.0 - beta1)
    last = T(state["last_grad"].astype(np.float32) if p_dt == "f32" else from_bf16_bits(state["last_grad"]), p_dt)
    c = grad.add(last.neg(), dt=grad.dt).mul_s(f).add(grad, dt=grad.dt)
    state["last_grad"] = grad.v.astype(np.float32) if p_dt == "f32" else bf16_bits(grad.v)
    return c


def normuon_update(u: T, state, beta2, eps):
    """Muon_util.normuon_update (Muon_util.py:349-360) on the 2-D update:
    v = lerp(v, mean(u^2 over each row) [u^2 in u's dtype, the mean in
    float32], 1 - beta2); u = u / (sqrt(v) + eps), computed in float32 and
    stored in u's dtype."""
    sq = T(u.v * u.v, u.dt)
    mean = np.float32(sq.v.astype(np.float64).sum(axis=1).astype(np.float32) / np.float32(u.v.shape[1]))
    v = T(state["normuon_v"].astype(np.float32), "f32").lerp(T(mean, "f32"), 1 - beta2)
    state["normuon_v"] = v.v.copy()
    den = (np.sqrt(v.v) + f32(eps)).astype(np.float32)
    return T(u.v / den[:, None], u.dt)


class Kourkoutas:
    """Kourkoutas.py:6-257 (KourkoutasHelper) for the default layer key (the
    param's shape): a float32 EMA of each layer's pooled grad norm and, per
    step, beta2 = beta2_max - (beta2_max - beta2_min) * sun(raw) with
    raw = pooled / (ema + tiny_spike), sun(x) = x / (1 + x), blended in over
    k_warmup_steps.  The pooled norm is that of the PREVIOUS step's grads
    (accumulated while stepping, reset by prepare)."""

    def __init__(self, shapes, beta2_max, beta2_min, ema_alpha, tiny_spike, k_warmup_steps):
        self.keys = []
        for sh in shapes:
            if tuple(sh) not in self.keys:
                self.keys.append(tuple(sh))
        self.acc = {k: f32(0.0) for k in self.keys}
        self.ema = {k: f32(0.0) for k in self.keys}
        self.beta2 = {}
        self.b2max, self.b2min, self.alpha, self.tiny, self.kw = beta2_max, beta2_min, ema_alpha, tiny_spike, k_warmup_steps

    def prepare(self, current_step):
        """Kourkoutas.py:131-197: every op on float32 0-dim tensors with the
        Python scalar rounded to float32."""
        for k in self.keys:
            pooled = np.sqrt(f32(self.acc[k]))
            e = f32(self.ema[k] * f32(self.alpha))
            # add_(pooled, alpha=1 - ema_alpha): ATen's fused add-with-alpha
            e = T(np.array([e], np.float32), "f32").add_alpha(T(np.array([pooled], np.float32), "f32"),
                                                              1.0 - self.alpha).v[0]
            self.ema[k] = f32(e)
            raw = f32(pooled / f32(self.ema[k] + f32(self.tiny)))
            sun = f32(raw / f32(f32(1.0) + raw))
            target = f32(f32(self.b2max) - f32(f32(self.b2max - self.b2min) * sun))
            weight = min(1.0, current_step / self.kw) if self.kw > 0 else 1.0
            b2 = f32(f32((1.0 - weight) * self.b2max) + f32(f32(weight) * target))
            self.beta2[k] = float(b2)
            self.acc[k] = f32(0.0)

    def accumulate(self, shape, grad):
        """Kourkoutas.py:231-247: torch.sum(grad.pow(2)).float() added to the
        layer's float32 accumulator (a bf16 grad squares and sums in bf16)."""
        if grad.dt == "bf16":
            sq = round_bf16(np.float32(np.sum(round_bf16(grad.v.astype(np.float32) ** 2).astype(np.float64))))
        else:
            sq = np.float32(np.sum((grad.v.astype(np.float32) ** 2).astype(np.float32).astype(np.float64)))
        k = tuple(shape)
        self.acc[k] = f32(self.acc[k] + f32(sq))


def is_suitable_for_muon(shape, min_dim_size=4, max_aspect_ratio=128.0):
    """Muon_util._is_suitable_for_muon (Muon_util.py:285-331) on a shape:
    at least two non-unit dims, no unit dim in the first two positions, the
    (out, prod(rest)) view no smaller than min_dim_size and no more elongated
    than max_aspect_ratio."""
    s = tuple(int(d) for d in shape)
    if len(s) < 2 or sum(1 for d in s if d > 1) < 2:
        return False
    if s[0] == 1 or s[1] == 1:
        return False
    dims = (s[0], int(np.prod(s[1:]))) if len(s) >= 3 else s
    if min(dims) < min_dim_size:
        return False
    return max(dims) / min(dims) <= max_aspect_ratio


def muon_step(p, p_dt, g, state, hp, noise):
    """Muon_adv._muon_step_parameter, non-factored 2-D path (Muon_adv.py:443-555)."""
    prec = hp["precision"]
    beta1 = hp["beta1"]
    grad = upcast(T(g, p_dt), prec)
    if hp.get("approx_mars", False):
        grad = approx_mars(grad, state, p_dt, hp.get("mars_gamma", 0.025), beta1)
    m = get_state(state, "momentum_buffer", prec, p_dt)
    m = m.lerp(grad, 1 - beta1)
    if hp.get("nesterov", True):
        c = beta1 if hp.get("nesterov_coef") is None else hp["nesterov_coef"]
        upd = grad.lerp(m, c, dt=T._res(grad, m))
    else:
        upd = m.clone()
    set_state(state, "momentum_buffer", m, prec, noise.get("momentum_buffer"))
    shape = np.shape(p)
    upd = T(upd.v.reshape(shape[0], -1), upd.dt)
    upd = newton_schulz(upd, hp["ns_steps"], hp["ns_eps"], hp["ns_coeffs"], hp.get("accelerated_ns", False), hp.get("cns_a_bound"),
                            sketch=noise.get("sketch") if hp.get("low_rank_ortho", False) else None)
    if hp.get("normuon_variant", False):
        upd = normuon_update(upd, state, hp.get("beta2_normuon", 0.95), hp.get("normuon_eps", 1e-8))
    upd = rms_adjustment(upd, hp.get("rms_rescaling", True), hp["lr"])
    upd = T(upd.v.reshape(shape), upd.dt)
    return apply_parameter_update(p, p_dt, upd, state, lr=hp["lr"], wd=hp.get("weight_decay", 0.0),
                                  cautious=hp.get("cautious_wd", False),
                                  sr=hp.get("stochastic_rounding", True), r_param=noise.get("param"),
                                  cwd=hp.get("centered_wd", 0.0), cwd_mode=hp.get("centered_wd_mode", "float8"))


def adamuon_step(p, p_dt, g, state, hp, noise):
    """AdaMuon_adv._muon_step_parameter, non-factored path (AdaMuon_adv.py:492-659)."""
    prec = hp["precision"]
    beta1, beta2 = hp["betas"]
    grad = upcast(T(g, p_dt), prec)
    shape = np.shape(p)
    eps = hp["eps"] if hp["eps"] is not None else 1.0 / math.sqrt(grad.v.size)
    if hp.get("approx_mars", False):
        grad = approx_mars(grad, state, p_dt, hp.get("mars_gamma", 0.025), beta1)
    m = get_state(state, "momentum_buffer", prec, p_dt)
    m = m.lerp(grad, 1 - beta1)
    if hp.get("nesterov", True):
        c = beta1 if hp.get("nesterov_coef") is None else hp["nesterov_coef"]
        upd = grad.lerp(m, c, dt=T._res(grad, m))
    else:
        upd = m.clone()
    set_state(state, "momentum_buffer", m, prec, noise.get("momentum_buffer"))
    kappa = hp.get("kappa_p", 1.0)
    if hp.get("auto_projection", True):
        kappa = 2.0 if len(shape) >= 4 else 1.0
    if kappa == 1.0:
        upd = upd.sign()
    upd = T(upd.v.reshape(shape[0], -1), upd.dt)
    upd = newton_schulz(upd, hp["ns_steps"], hp["ns_eps"], hp["ns_coeffs"], hp.get("accelerated_ns", False), hp.get("cns_a_bound"),
                            sketch=noise.get("sketch") if hp.get("low_rank_ortho", False) else None)
    normuon = hp.get("normuon_variant", False)
    if normuon:
        # replaces the second moment (AdaMuon_adv.py:614-616)
        upd = normuon_update(upd, state, beta2, hp["eps"])
    upd = T(upd.v.reshape(shape), upd.dt)
    atan2 = hp.get("use_atan2", False) and not normuon
    if normuon:
        pass
    elif state.get("factored_2nd", False):
        d1, d2 = state["effective_shape"]
        uf = upd.to("f32")
        v = T(unnmf(state["mu_vbuf_nmf"], state["mv_vbuf_nmf"]), "f32")
        uf2 = T(uf.v.reshape(d1, d2), "f32")
        v = v.mul_s(beta2).addcmul(uf2, uf2, 1 - beta2)
        state["mu_vbuf_nmf"], state["mv_vbuf_nmf"] = nnmf(np.abs(v.v))
        den = T(np.abs(v.v), "f32").sqrt()
        if not atan2:
            den = den.add_s(eps)
        den = T(den.v.reshape(shape), "f32").to(upd.dt)
        upd = upd.atan2(den, dt=upd.dt) if atan2 else upd.div(den, dt=upd.dt)
    else:
        v = get_state(state, "second_momentum_buffer", prec, p_dt, non_neg=True)
        v = v.mul_s(beta2).addcmul(upd, upd, 1 - beta2)
        den = v.sqrt()
        if not atan2:
            den = den.add_s(eps)
        upd = upd.atan2(den) if atan2 else upd.div(den)
        set_state(state, "second_momentum_buffer", v, prec, noise.get("second_momentum_buffer"), non_neg=True)
    step_scale = hp["lr"] * (4 / math.pi) if atan2 else hp["lr"]
    upd = T(upd.v.reshape(shape[0], -1), upd.dt)
    upd = rms_adjustment(upd, hp.get("rms_rescaling", True), step_scale)
    upd = T(upd.v.reshape(shape), upd.dt)
    return apply_parameter_update(p, p_dt, upd, state, lr=hp["lr"], wd=hp.get("weight_decay", 0.0),
                                  cautious=hp.get("cautious_wd", False),
                                  sr=hp.get("stochastic_rounding", True), r_param=noise.get("param"),
                                  cwd=hp.get("centered_wd", 0.0), cwd_mode=hp.get("centered_wd_mode", "float8"))
