"""Host side of the Adam-family step (AdamW_adv, Muon's auxiliary Adam,
Prodigy_adv): state creation with the reference's keys and dtypes, the
per-group plan (device descriptor table + pieces), and the launches.

State layout follows AdamW_adv.py:221-277, Muon_AuxAdam.py:15-67 and
Prodigy_adv.py:271-331 key for key, so checkpoints cross-load with the
reference.
"""
from __future__ import annotations

import ctypes
import math

import numpy as np
import torch

from .. import _lib as L
from .._device import DeviceTable, aligned16, dtype_code, ptr, require_cuda_tensor, stream_handle, upload_static
from .._plan import effective_shape, plan as plan_pieces
from ._common import ErrorWatch

A_ATAN2 = 4 / math.pi
SHIFTER = [1, 2, 4, 8, 16, 32, 64, 128]
BLOCK = 2048
SUPPORTED_PRECISIONS = ("auto", "fp32", "bf16_sr", "int8_sr", "factored")
FAST_COLS = 8192   # shared-memory column accumulator of the fast kernel (floats)


def f32(x) -> float:
    """The float32 value a Python scalar takes as an ATen op argument."""
    return float(np.float32(x))


# ---------------------------------------------------------------------------
# state creation (state_util.init_state_tensor, state_util.py:13-37)
# ---------------------------------------------------------------------------

def init_state_tensor(state, key, p, precision, non_neg=False):
    if precision == "fp32":
        dt = torch.float32
    elif precision == "bf16_sr":
        dt = torch.bfloat16
    elif precision == "int8_sr":
        dt = torch.uint8 if non_neg else torch.int8
    elif precision == "auto":
        dt = p.dtype
    else:
        raise NotImplementedError(f"state_precision '{precision}' is not supported by the B200 kernels")
    state[key] = torch.zeros(p.shape, dtype=dt, device=p.device)
    if dt in (torch.uint8, torch.int8):
        nb = (p.numel() + BLOCK - 1) // BLOCK
        state[f"{key}_scale"] = torch.ones(nb, dtype=torch.float32, device=p.device)


def is_wd_centered(p) -> bool:
    """centered_decay.is_wd_centered (centered_decay.py:4-12)."""
    return bool(getattr(p, "_is_lora_A", False) or getattr(p, "_is_lora_B", False) or getattr(p, "_is_oft", False))


def adjust_wds(wd, cwd, p):
    """scaled_optm.adjust_wds (scaled_optm.py:84-105)."""
    if getattr(p, "_is_dora_scale", False):
        return wd, cwd
    if getattr(p, "_is_oft", False):
        return wd, 0.0
    if p.ndim >= 2 and (getattr(p, "_is_lora_A", False) or getattr(p, "_is_lora_B", False)):
        return wd, 0.0
    return wd, cwd


@torch.no_grad()
def init_anchor(p, state, centered_wd, mode):
    """centered_decay._init_anchor (centered_decay.py:43-76)."""
    if not centered_wd or is_wd_centered(p) or "anchor_data" in state:
        return
    if mode == "float8":
        state["anchor_data"] = p.to(torch.float8_e4m3fn)
    elif mode in ("int8", "int4"):
        blk, bits = (128, 8) if mode == "int8" else (32, 4)
        flat = p.flatten()
        n = flat.numel()
        pad = (blk - n % blk) % blk
        vals = torch.nn.functional.pad(flat.unsqueeze(0), (0, pad), mode="replicate").squeeze(0) if pad else flat.clone()
        vb = vals.view(-1, blk).float()
        mn, mx = torch.aminmax(vb, dim=1, keepdim=True)
        qmin, qmax = -(1 << (bits - 1)), (1 << (bits - 1)) - 1
        scales = (mx - mn).div_(float(qmax - qmin))
        scales.masked_fill_(scales == 0, 1.0)
        q = vb.sub_(mn).div_(scales).add_(qmin).round_().clamp_(qmin, qmax).to(torch.int8)
        if mode == "int4":
            qf = q.view(-1)
            q = (((qf[0::2] & 0x0F) << 4) | (qf[1::2] & 0x0F)).to(torch.int8)
        state["anchor_data"] = q
        state["anchor_scale"] = scales.squeeze(1).to(p.dtype)
        state["anchor_min"] = mn.squeeze(1).to(p.dtype)
    elif mode == "full":
        state["anchor_data"] = p.clone()


def anchor_code(state, mode) -> int:
    """Storage of the centered-WD anchor, as dequantize_anchor reads it
    (centered_decay.py:78-119): by dtype, with the group's mode telling
    int8 from int4 codes."""
    if "anchor_data" not in state:
        return 0
    d = state["anchor_data"]
    if d.dtype == torch.float8_e4m3fn:
        return L.ANCHOR["float8"]
    if d.dtype == torch.int8:
        if mode == "int4":
            return L.ANCHOR["int4"]
        if mode == "int8":
            return L.ANCHOR["int8"]
        raise NotImplementedError(f"int8 anchor data with centered_wd_mode '{mode}'")
    return L.ANCHOR["full"]


def sign_storage(d1, packed_d2, device):
    """A zeroed (d1, ceil(d2/8)) uint8 sign array whose storage is a whole
    number of 4-byte words (the kernel sets sign bits with 32-bit atomics)."""
    n = d1 * packed_d2
    return torch.zeros(((n + 3) // 4) * 4, dtype=torch.uint8, device=device)[:n].view(d1, packed_d2)


def ensure_sign_words(state, key="sign"):
    """Re-home a sign array (e.g. one loaded from a checkpoint) into storage
    that ends on a 4-byte word, keeping its values."""
    t = state.get(key)
    if t is None:
        return
    n = t.numel()
    room = t.untyped_storage().nbytes() - t.storage_offset()
    if t.is_contiguous() and t.data_ptr() % 4 == 0 and room >= ((n + 3) // 4) * 4:
        return
    s = sign_storage(t.shape[0], t.shape[1], t.device)
    s.copy_(t)
    state[key] = s


@torch.no_grad()
def init_adam_state(p, state, *, precision, factored_2nd, beta1, vector_reshape, centered_wd, centered_wd_mode,
                    fisher_wd):
    """AdamW_adv.__init_state (AdamW_adv.py:221-277); Muon_AuxAdam._init_auxadam_state
    is the same with adam_* keys (Muon_AuxAdam.py:15-67).  Under 'factored' a
    param of two or more dims keeps m as signed rank-1 factors (mu_m_nmf,
    mv_m_nmf, 1-bit sign) and v as rank-1 factors; a 1-D one float32 m and v."""
    state["step"] = 0
    is_vector = p.dim() == 1 and not vector_reshape
    state["factored"] = False
    if precision == "factored":
        if not is_vector:
            d1, d2 = effective_shape(p.numel())
            state["factored"] = True
            state["factored_2nd"] = bool(factored_2nd)
            state["effective_shape"] = (d1, d2)
            if beta1 > 0:
                state["mu_m_nmf"] = torch.zeros(d1, device=p.device, dtype=torch.float32)
                state["mv_m_nmf"] = torch.zeros(d2, device=p.device, dtype=torch.float32)
                state["sign"] = sign_storage(d1, (d2 + 7) // 8, p.device)
                state["shifter"] = torch.tensor(SHIFTER, device=p.device, dtype=torch.uint8)
            state["mu_v_nmf"] = torch.zeros(d1, device=p.device, dtype=torch.float32)
            state["mv_v_nmf"] = torch.zeros(d2, device=p.device, dtype=torch.float32)
            init_anchor(p, state, centered_wd, centered_wd_mode)
            if fisher_wd:
                state["wd_scaler"] = torch.tensor(1.0, device=p.device)
            return
        precision = "fp32"        # float32 states for 1-D params of a 'factored' group
    state["factored_2nd"] = bool(factored_2nd and not is_vector)
    if beta1 > 0:
        init_state_tensor(state, "exp_avg", p, precision)
    if state["factored_2nd"]:
        d1, d2 = effective_shape(p.numel())
        state["effective_shape"] = (d1, d2)
        state["mu_v_nmf"] = torch.zeros(d1, device=p.device, dtype=torch.float32)
        state["mv_v_nmf"] = torch.zeros(d2, device=p.device, dtype=torch.float32)
        state["shifter"] = torch.tensor(SHIFTER, device=p.device, dtype=torch.uint8)
    else:
        init_state_tensor(state, "exp_avg_sq", p, precision, non_neg=True)
    init_anchor(p, state, centered_wd, centered_wd_mode)
    if fisher_wd:
        state["wd_scaler"] = torch.tensor(1.0, device=p.device)


# ---------------------------------------------------------------------------
# spectral normalisation state (scaled_optm.py:108-142)
# ---------------------------------------------------------------------------

def is_spectral(p) -> bool:
    """scaled_optm.is_spectral (scaled_optm.py:108-116)."""
    if getattr(p, "_is_oft", False):
        return True
    if p.ndim < 2:
        return False
    if getattr(p, "_is_dora_scale", False) or getattr(p, "is_vector", False):
        return False
    return bool(getattr(p, "is_hidden", True))


def spectral_kind(p) -> str:
    """How scale_update treats p's update (scaled_optm.py:54-72): 'maxabs'
    (1-D, DoRA magnitudes) or 'spectral' (2-D and larger)."""
    if getattr(p, "_is_oft", False):
        raise NotImplementedError("spectral normalisation of OFT blocks is not supported by the B200 kernels")
    if p.ndim < 2 or getattr(p, "_is_dora_scale", False):
        return "maxabs"
    if not is_spectral(p):
        # the reference has no singular vectors for it and fails in scale_update
        raise NotImplementedError("spectral normalisation of a 2-D param marked is_vector / not is_hidden")
    return "spectral"


@torch.no_grad()
def init_spectral_norm(state, p, generator):
    """init_spectral_norm (scaled_optm.py:118-142), non-OFT: unit Gaussian v
    (d_in) then u (d_out) in the param dtype, drawn on the param's device."""
    if not is_spectral(p) or "spectral_u" in state:
        return
    d_out = p.shape[0]
    d_in = p.numel() // d_out
    v = torch.randn(d_in, device=p.device, dtype=p.dtype, generator=generator)
    state["spectral_v"] = v.div_(v.norm().add_(1e-12))
    u = torch.randn(d_out, device=p.device, dtype=p.dtype, generator=generator)
    state["spectral_u"] = u.div_(u.norm().add_(1e-12))


class SpectralInit:
    """Creates spectral_u / spectral_v for params that get spectral
    normalisation, from one seeded torch generator per device (the
    reference draws them from its own per-device generator)."""

    def __init__(self, seed: int = 42):
        self.seed = int(seed)
        self.gens = {}

    def __call__(self, state, p):
        spectral_kind(p)            # raises for updates the kernels do not scale
        g = self.gens.get(p.device)
        if g is None:
            g = torch.Generator(device=p.device)
            g.manual_seed(self.seed)
            self.gens[p.device] = g
        init_spectral_norm(state, p, g)


class SpectralPlan:
    """Scratch, descriptor table and work lists of advopt_spectral_step for
    one group plan: per tensor the unscaled update (param dtype for 2-D
    updates, which the reference casts to the singular vectors' dtype; the
    update's own dtype for 1-D ones), the U^T u column partials per row slab,
    U v and two scalars."""

    def __init__(self, gp):
        n = gp.n
        sd = np.zeros(n, L.SPECTRAL_TENSOR_DT)
        self.bufs = []
        kinds = [spectral_kind(p) for p in gp.params]
        rows_2d = sum(p.shape[0] for p, k in zip(gp.params, kinds) if k == "spectral")
        # row slabs of the U^T u pass: about 600 work items, 8..64 rows each
        slab = int(min(64, max(8, ((-(-rows_2d // 600) + 7) // 8) * 8)))
        col_items, row_items = [], []
        for i, (p, st, kind) in enumerate(zip(gp.params, gp.states, kinds)):
            numel = p.numel()
            if kind == "spectral":
                if "spectral_u" not in st:
                    raise RuntimeError("spectral normalisation state missing (spectral_u / spectral_v)")
                vbf = st["spectral_u"].dtype == torch.bfloat16
                d_out = p.shape[0]
                d_in = numel // d_out
                n_slabs = -(-d_out // slab)
                vpart = torch.empty(n_slabs * d_in, dtype=torch.float32, device=gp.device)
                uraw = torch.empty(d_out, dtype=torch.float32, device=gp.device)
                self.bufs += [vpart, uraw]
                flags = (L.S_UPD_BF16 | L.S_VEC_BF16) if vbf else 0
                target = 1.0 if getattr(p, "_is_lora_A", False) else math.sqrt(d_out / d_in)
                sd["u"][i], sd["v"][i] = ptr(st["spectral_u"]), ptr(st["spectral_v"])
                sd["v_partial"][i], sd["u_raw"][i] = ptr(vpart), ptr(uraw)
                sd["d_out"][i], sd["d_in"][i], sd["n_slabs"][i], sd["target"][i] = d_out, d_in, n_slabs, target
                for s in range(n_slabs):
                    col_items.append((s * slab, min((s + 1) * slab, d_out), i, s))
                for r0 in range(0, d_out, 64):
                    row_items.append((r0, min(r0 + 64, d_out), i, 0))
                ubf = vbf
            else:
                # max-abs scaling in the update's own dtype: bf16 under bf16 math
                ubf = gp.math_bf16 and not st.get("factored", False)
                flags = L.S_MAXABS | (L.S_UPD_BF16 if ubf else 0)
                sd["d_out"][i], sd["d_in"][i], sd["n_slabs"][i], sd["target"][i] = 1, numel, 0, 1.0
                for k in range(0, numel, 65536):
                    row_items.append((k, min(k + 65536, numel), i, 0))
            upd = torch.empty(numel, dtype=torch.bfloat16 if ubf else torch.float32, device=gp.device)
            scal = torch.zeros(4, dtype=torch.float32, device=gp.device)
            self.bufs += [upd, scal]
            sd["update"][i], sd["scalars"][i], sd["flags"][i] = ptr(upd), ptr(scal), flags
            gp.descs["update_out"][i] = ptr(upd)
            gp.vec_ok[i] = gp.vec_ok[i] and ptr(upd) % 16 == 0
            if ubf:
                gp.descs["flags"][i] |= L.T_UPD_BF16
        self.table = upload_static(sd, gp.device)

        def pieces(items):
            a = np.zeros(max(1, len(items)), L.PIECE_DT)
            for j, (b, e, t, s) in enumerate(items):
                a[j] = (b, e, t, s)
            return upload_static(a, gp.device), len(items)

        self.col_dev, self.n_col = pieces(col_items)
        self.row_dev, self.n_row = pieces(row_items)


# ---------------------------------------------------------------------------
# launch configuration
# ---------------------------------------------------------------------------

class AdamCfg:
    """Group-level hyperparameters of one launch, already in the reference's
    scalar semantics.  `algo` is L.ALGO_*."""

    def __init__(self, *, algo, lr, betas, eps, weight_decay, precision, nesterov=False, nesterov_coef=None,
                 use_bias_correction=True, use_atan2=False, normed_momentum=False, cautious_wd=False,
                 fisher_wd=False, centered_wd=0.0, centered_wd_mode="float8", stochastic_rounding=True,
                 prodigy=None, kourkoutas=None, kourkoutas_apply=True, spectral=False):
        self.algo = algo
        self.lr = float(lr)
        self.beta1, self.beta2 = float(betas[0]), float(betas[1])
        self.eps = eps
        self.weight_decay = float(weight_decay)
        self.precision = precision
        self.nesterov = bool(nesterov)
        self.nesterov_coef = nesterov_coef
        self.use_bias_correction = bool(use_bias_correction)
        self.use_atan2 = bool(use_atan2)
        self.normed = bool(normed_momentum) and algo == L.ALGO_ADAMW
        self.cautious = bool(cautious_wd)
        self.fisher = bool(fisher_wd)
        self.centered_wd = float(centered_wd)
        self.centered_wd_mode = centered_wd_mode
        self.sr = bool(stochastic_rounding)
        # dict: d, d0, beta3, safeguard_warmup, slice_p, stats (bool), dev (the
        # advopt_prodigy_dev block: d on the device; d and d0 above are then unused)
        self.prodigy = prodigy
        self.kourkoutas = kourkoutas   # KourkoutasBeta of the optimizer, or None
        # False: the grads' squared norms are pooled but the v update keeps
        # beta2 (the hybrid optimizers' auxiliary Adam under bias correction)
        self.kourkoutas_apply = bool(kourkoutas_apply)
        # spectral_normalization: the step emits the unscaled update and
        # advopt_spectral_step scales and applies it (scaled_optm.py:35-72)
        self.spectral = bool(spectral)
        if self.spectral and self.fisher:
            raise NotImplementedError("spectral_normalization with fisher_wd is not supported by the B200 kernels")


class GroupPlan:
    """Static part of one launch: the tensors (params with grads, one dtype),
    their descriptor table, the pieces and the scratch buffers."""

    def __init__(self, params, states, tensor_ids, cfg: AdamCfg, reserve_sms: int = 0):
        self.params = list(params)
        self.states = list(states)
        p0 = self.params[0]
        self.device = p0.device
        self.pdt = dtype_code(p0.dtype)
        n = len(self.params)
        self.n = n
        prec = cfg.precision
        if prec == "auto" and self.pdt == L.DT_F32:
            prec = "fp32"
        if prec == "factored":
            prec = "fp32"          # float32 math and states throughout (state_util.py:165-179)
        self.precision = L.PREC[prec]
        self.descs = np.zeros(n, L.ADAM_TENSOR_DT)
        d = self.descs
        numels, d2s = [], []
        max_d2 = 0
        any_generic = False
        self.has_anchor = False
        self.any_fact_m = False
        vec_ok = []
        for i, (p, st) in enumerate(zip(self.params, self.states)):
            numel = p.numel()
            numels.append(numel)
            flags = 0
            smmf = bool(st.get("factored", False))
            fact = bool(st.get("factored_2nd", False)) or smmf
            m = st.get("exp_avg")
            v = st.get("exp_avg_sq")
            tensors = [p, m, v]
            if smmf and "mu_m_nmf" in st:
                # signed rank-1 momentum (state_precision='factored')
                ensure_sign_words(st)
                flags |= L.T_FACT_M
                self.any_fact_m = True
                d["m_row_factor"][i] = ptr(st["mu_m_nmf"])
                d["m_col_factor"][i] = ptr(st["mv_m_nmf"])
                d["m_sign"][i] = ptr(st["sign"])
            if fact:
                d1, d2 = st["effective_shape"]
                flags |= L.T_FACTORED
                d["d1"][i], d["d2"][i] = d1, d2
                # (factored Lion has no second moment)
                d["row_factor"][i] = ptr(st.get("mu_v_nmf"))
                d["col_factor"][i] = ptr(st.get("mv_v_nmf"))
                d2s.append(d2)
                max_d2 = max(max_d2, d2)
                # the kernel takes its generic path for these rows (and then
                # needs the staging area in shared memory)
                cols = [t for t in (st.get("mv_v_nmf"), st.get("mv_m_nmf") if smmf else None) if t is not None]
                if d2 < 2048 or d2 % 8 != 0 or not aligned16(*cols):
                    any_generic = True
                tensors += [t for t in (st.get("mu_v_nmf"), st.get("mv_v_nmf")) if t is not None]
            else:
                d2s.append(0)
            d["param"][i] = ptr(p)
            d["exp_avg"][i] = ptr(m)
            d["exp_avg_scale"][i] = ptr(st.get("exp_avg_scale"))
            d["exp_avg_sq"][i] = ptr(v)
            d["exp_avg_sq_scale"][i] = ptr(st.get("exp_avg_sq_scale"))
            d["numel"][i] = numel
            d["tensor_id"][i] = tensor_ids[i]
            d["fisher_clip"][i] = 1.0
            ac = anchor_code(st, cfg.centered_wd_mode)
            if ac:
                self.has_anchor = True
                flags |= ac << L.T_ANCHOR_SHIFT
                d["aux0"][i] = ptr(st["anchor_data"])
                d["aux1"][i] = ptr(st.get("anchor_scale"))
                d["aux2"][i] = ptr(st.get("anchor_min"))
            if cfg.prodigy is not None and cfg.prodigy["stats"]:
                # s and p0 exist while the d estimate runs (Prodigy_adv.py:
                # 494-509); after prodigy_steps they are freed
                d["aux0"][i] = ptr(st["s"])
                d["aux1"][i] = ptr(st["p0"])
                d["slice_p"][i] = cfg.prodigy["slice_p"]
                if st["p0"].dim() == 0:
                    flags |= L.T_P0_SCALAR
            vec_ok.append(aligned16(*tensors))
            if vec_ok[-1]:
                flags |= L.T_VEC
            d["flags"][i] = flags
        self.numels = numels
        self.vec_ok = vec_ok
        self.max_d2 = max_d2
        self.gen_offset = ((max_d2 + 3) // 4) * 4
        # fast path: no extended options and only wide factored tensors
        ext = cfg.use_atan2 or cfg.normed or cfg.fisher or self.has_anchor
        factors_aligned = all(aligned16(st["mu_v_nmf"], st["mv_v_nmf"]) for st in self.states
                              if "mu_v_nmf" in st)
        # the fast kernel keeps element offsets in 32 bits (tensors below 2^34
        # elements); signed rank-1 momentum runs in the general kernel
        # spectral normalisation: the fast kernel emits the update in the param
        # dtype, so it runs when every tensor's update has that dtype (the
        # singular vectors' dtype for 2-D updates; the math dtype for 1-D ones)
        spectral_fast = True
        if cfg.spectral:
            math_bf16 = cfg.precision == "auto" and self.pdt == L.DT_BF16
            for p, st in zip(self.params, self.states):
                if spectral_kind(p) == "spectral":
                    same = "spectral_u" in st and st["spectral_u"].dtype == p.dtype
                else:
                    same = self.pdt == L.DT_F32 or math_bf16
                spectral_fast = spectral_fast and same
        # signed rank-1 momentum takes the fast kernel's FM variant when every
        # row is on the fast layout (no generic rows) and nothing needs the
        # general kernel (update emission, Lion)
        fm_ok = (not self.any_fact_m) or (not cfg.spectral and all(
            aligned16(st["mv_m_nmf"]) for st in self.states if "mv_m_nmf" in st))
        self.fast = (not ext) and (not any_generic) and factors_aligned and max(numels, default=0) < (1 << 34) \
            and fm_ok and spectral_fast and cfg.algo != L.ALGO_LION
        if self.fast:
            bpp = 2 if self.pdt == L.DT_BF16 else 4
            bps = {0: 4, 1: 2, 2: 1, 3: 2 if self.pdt == L.DT_BF16 else 4}[self.precision]
            stage = 2048 * (2 * bpp + 2 * bps)
            # factored tensors wider than FAST_COLS keep their column partials
            # in global memory, so one wide tensor does not cut occupancy
            self.gen_offset = min(self.gen_offset, FAST_COLS)
            three = self.precision == L.PREC["int8_sr"] and self.pdt == L.DT_BF16 and cfg.algo != L.ALGO_PRODIGY
            per_cta = (227 * 1024) // (3 if three else 2) - 2048
            # FM: a second column-sum area for |m|
            areas = 2 if self.any_fact_m else 1
            budget = per_cta - areas * self.gen_offset * 4
            self.stages = int(max(2, min(4, budget // stage)))
            self.smem_floats = areas * self.gen_offset + self.stages * stage // 4
        elif self.any_fact_m:
            # two equal halves: the second-moment and the |m| column sums, with
            # the generic path's staging when a row is not on the fast layout
            if not all(st.get("factored", False) and "mu_m_nmf" in st for st in self.states):
                raise RuntimeError("a factored-momentum launch holds only factored-momentum tensors")
            self.stages = 0
            self.smem_floats = 2 * (self.gen_offset + (2 * 2048 + 4 if any_generic else 0))
            if self.smem_floats > 56832:
                raise NotImplementedError(
                    f"state_precision='factored' with an effective row of {max_d2} columns: the B200 kernel keeps "
                    f"both factors' column sums in shared memory (at most 24316 columns)")
        else:
            self.stages = 0
            self.smem_floats = self.gen_offset + (2 * 2048 + 4 if any_generic else 0)
        sms, ctas = L.adam_occupancy(self.precision, self.pdt, cfg.algo, self.smem_floats, self.fast)
        total_chunks = sum((x + 2047) // 2048 for x in numels)
        # SMs left free for work running beside the step (a sharded run's
        # all-gather of the previous bucket)
        sms = max(1, sms - max(0, int(reserve_sms)))
        self.grid = max(1, min(sms * ctas, total_chunks))
        pieces, offsets, n_slots = plan_pieces(numels, d2s, self.grid)
        self.n_pieces = len(pieces)
        # factored scratch: one row of column partials per piece
        self.scratch = []
        fact_idx = []
        for i in range(n):
            if d["flags"][i] & L.T_FACTORED:
                d2 = int(d["d2"][i])
                if d["row_factor"][i]:
                    buf = torch.empty(max(1, n_slots[i]) * d2, dtype=torch.float32, device=self.device)
                    self.scratch.append(buf)
                    d["col_partial"][i] = ptr(buf)
                d["n_slots"][i] = n_slots[i]
                if d["flags"][i] & L.T_FACT_M:
                    mbuf = torch.empty(max(1, n_slots[i]) * d2, dtype=torch.float32, device=self.device)
                    self.scratch.append(mbuf)
                    d["m_col_partial"][i] = ptr(mbuf)
                fact_idx.append(i)
        self.fact_idx = fact_idx
        self.fact_idx_dev = upload_static(np.asarray(fact_idx, np.int32), self.device) if fact_idx else None
        self.pieces_dev = upload_static(pieces, self.device)
        self.offsets_dev = upload_static(offsets, self.device)
        need_stats = cfg.prodigy is not None or cfg.fisher
        self.stats = torch.zeros(max(1, 2 * self.n_pieces), dtype=torch.float64, device=self.device) \
            if need_stats else None
        self.table = DeviceTable(self.descs.nbytes, self.device)
        self.err = None   # the runner's device error word (set by AdamFamilyRunner.get_plan)
        self.eps_cache = [None] * n
        # Kourkoutas-beta: each tensor's layer and the per-piece sums of g*g
        self.params = list(params)
        self.layer_dev = None
        self.gsq = None
        self.math_bf16 = cfg.precision == "auto" and self.pdt == L.DT_BF16
        # Prodigy with d on the device: per-tensor (eps_t, wd_t, cwd_t) in double
        self.pconsts_host = None
        self.pconsts_dev = None
        self.spectral = SpectralPlan(self) if cfg.spectral else None

    def kourkoutas_tables(self, kk):
        if self.layer_dev is None:
            self.layer_dev = upload_static(np.asarray(kk.layer_table(self.params), np.int32), self.device)
            self.gsq = torch.zeros(max(1, self.n_pieces), dtype=torch.float64, device=self.device)

    def launch_struct(self, cfg: AdamCfg, flags: int, seed: int) -> L.AdamLaunch:
        s = L.AdamLaunch()
        s.tensors = self.table.ptr
        s.pieces = int(self.pieces_dev.data_ptr())
        s.cta_offsets = int(self.offsets_dev.data_ptr())
        s.piece_stats = int(self.stats.data_ptr()) if self.stats is not None else 0
        s.n_tensors = self.n
        s.n_pieces = self.n_pieces
        s.grid = self.grid
        s.smem_floats = self.smem_floats
        s.gen_offset = self.gen_offset
        s.algo = cfg.algo
        s.precision = self.precision
        s.param_dtype = self.pdt
        s.flags = flags
        s.seed = seed
        s.stages = self.stages
        s.err = int(self.err.data_ptr())
        kk = cfg.kourkoutas
        if kk is not None and kk.n:
            self.kourkoutas_tables(kk)
            if cfg.kourkoutas_apply:
                s.layer_beta2 = int(kk.beta2.data_ptr())
                s.layer_of_tensor = int(self.layer_dev.data_ptr())
            s.piece_gsq = int(self.gsq.data_ptr())
        return s


def grads_of(params):
    return [p.grad for p in params]


class AdamFamilyRunner:
    """Owns the plans of one optimizer and performs group launches."""

    def __init__(self, seed: int = 42):
        self.plans = {}
        self.seed = int(seed)
        self.test_noise = None   # {id(param): {label: int32 CUDA tensor}} for the next step only
        self.kernel_events = None  # list to collect (start, end) CUDA events around the main launch
        self.launch_count = 0      # kernels launched so far (for launch accounting)
        self.reserve_sms = 0       # SMs the step's grid leaves free (see GroupPlan)
        self.errors = ErrorWatch("an Adam-family step kernel")

    def invalidate(self):
        self.plans.clear()

    def check_errors(self):
        """Raise if a kernel reported a bounded wait that gave up (synchronises)."""
        self.errors.check(sync=True)

    def get_plan(self, key, params, states, ids, cfg):
        pl = self.plans.get(key)
        if pl is None or (pl.spectral is not None) != cfg.spectral or \
                any(pl.descs["param"][i] != ptr(p) for i, p in enumerate(params)):
            pl = GroupPlan(params, states, ids, cfg, self.reserve_sms)
            pl.err = self.errors.word(pl.device)
            self.plans[key] = pl
        return pl

    @torch.no_grad()
    def run(self, key, params, states, ids, cfg: AdamCfg, prodigy_sums=None):
        """One launch over `params` (same dtype and device, all with grads);
        under 'factored' two, when the group mixes signed rank-1 momentum
        tensors with others (1-D params keep float32 m and v)."""
        if cfg.precision == "factored":
            fm = [bool(st.get("factored", False) and "mu_m_nmf" in st) for st in states]
            if any(fm) and not all(fm):
                for sel in (True, False):
                    idx = [i for i, f in enumerate(fm) if f == sel]
                    self.run(key + (sel,), [params[i] for i in idx], [states[i] for i in idx],
                             [ids[i] for i in idx], cfg, prodigy_sums)
                return
        for p in params:
            require_cuda_tensor(p, "param")
            require_cuda_tensor(p.grad, "grad")
        # an earlier step's kernels that gave up are reported here, without a sync
        self.errors.check()
        pl = self.get_plan(key, params, states, ids, cfg)
        d = pl.descs
        for i, p in enumerate(params):
            gp = p.grad.data_ptr()
            d["grad"][i] = gp
            if gp % 16:
                d["flags"][i] &= ~L.T_VEC
            elif pl.vec_ok[i]:
                d["flags"][i] |= L.T_VEC
        # per-tensor scalars in the reference's arithmetic (Python floats, cast to fp32)
        lr = cfg.lr
        step_cache = {}
        pdev = cfg.algo == L.ALGO_PRODIGY and cfg.prodigy.get("dev") is not None
        pconsts = np.zeros((len(params), 3), np.float64) if pdev else None
        for i, (p, st) in enumerate(zip(params, states)):
            t = st["step"]
            if cfg.algo == L.ALGO_PRODIGY:
                dd = cfg.prodigy["d"]
                dlr = dd * lr
                ss = dlr * A_ATAN2 if cfg.use_atan2 else dlr
                sbc2 = 1.0
                lr_wd = dlr
            elif cfg.algo == L.ALGO_LION:
                ss, sbc2, lr_wd = lr, 1.0, lr      # update.mul_(lr) (Lion_adv.py:273-276)
            else:
                sc = step_cache.get(t)
                if sc is None:
                    if cfg.use_bias_correction:
                        s1 = t + 1
                        bc1 = 1.0 - cfg.beta1 ** s1
                        sbc2 = (1.0 - cfg.beta2 ** s1) ** 0.5
                    else:
                        bc1, sbc2 = 1, 1
                    step_size = lr / bc1
                    sc = (step_size * A_ATAN2 if cfg.use_atan2 else step_size, sbc2)
                    step_cache[t] = sc
                ss, sbc2 = sc
                lr_wd = lr
            eps = cfg.eps if cfg.eps is not None else 1.0 / math.sqrt(p.numel())
            wd, cwd = adjust_wds(cfg.weight_decay, cfg.centered_wd, p)
            if pdev:
                pconsts[i] = (eps, wd, cwd)
            if cfg.algo == L.ALGO_PRODIGY:
                eps = cfg.prodigy["d"] * eps
            d["step_size"][i] = ss
            d["sqrt_bc2"][i] = sbc2
            d["eps"][i] = eps
            d["wd"][i] = wd * lr_wd if wd != 0 else 0.0
            d["cwd"][i] = cwd * lr_wd if cwd != 0 else 0.0
            d["step"][i] = t & 0xFFFFFFFF
        flags = 0
        if cfg.beta1 > 0 or cfg.algo == L.ALGO_LION:
            flags |= L.F_HAS_M
        if cfg.nesterov:
            flags |= L.F_NESTEROV
        if cfg.use_atan2:
            flags |= L.F_ATAN2
        if cfg.normed:
            flags |= L.F_NORMED
        if cfg.cautious:
            flags |= L.F_CAUTIOUS
        if cfg.sr and pl.pdt == L.DT_BF16:
            flags |= L.F_SR
        if pl.has_anchor:
            flags |= L.F_ANCHORS
        if not d["wd"].any():
            flags |= L.F_NO_WD
        if pl.any_fact_m:
            flags |= L.F_FACT_M
        if cfg.spectral:
            flags |= L.F_EMIT_UPDATE
        noise_keep = []
        if self.test_noise is not None:
            flags |= L.F_NOISE_IN
            for i, p in enumerate(params):
                nz = self.test_noise.get(id(p), {})
                n = p.numel()
                padded = ((n + BLOCK - 1) // BLOCK) * BLOCK
                for label, field in (("exp_avg_sq", "noise_v"), ("exp_avg", "noise_m"), ("param", "noise_p")):
                    t = nz.get(label)
                    if t is not None:
                        t = t.to(device=p.device, dtype=torch.int32).contiguous()
                        need = padded if (label != "param" and cfg.precision == "int8_sr") else n
                        if t.numel() < need:
                            raise ValueError(f"injected noise '{label}' has {t.numel()} entries, {need} needed")
                        noise_keep.append(t)
                        d[field][i] = t.data_ptr()
                    else:
                        d[field][i] = 0
        if self.test_noise is not None:
            need = []
            if cfg.sr and pl.pdt == L.DT_BF16:
                need.append("noise_p")
            if cfg.precision in ("int8_sr", "bf16_sr") and cfg.beta1 > 0:
                need.append("noise_m")
            for i in range(pl.n):
                for field in need + (["noise_v"] if cfg.precision in ("int8_sr", "bf16_sr")
                                     and not (d["flags"][i] & L.T_FACTORED) else []):
                    if d[field][i] == 0:
                        raise ValueError(f"injected noise missing for tensor {i} ({field})")
        pl.table.upload(d)
        stream = stream_handle(pl.device)
        lib = L.lib()
        if pdev:
            # the d-dependent scalars and table fields from the device d
            if pl.pconsts_host is None or not np.array_equal(pl.pconsts_host, pconsts):
                pl.pconsts_host = pconsts
                pl.pconsts_dev = upload_static(pconsts, pl.device)
            pa = L.ProdigyScalarArgs()
            pa.dev = int(cfg.prodigy["dev"].data_ptr())
            pa.tensors = pl.table.ptr
            pa.tensor_consts = int(pl.pconsts_dev.data_ptr())
            pa.n_tensors = pl.n
            pa.safeguard_warmup = 1 if cfg.prodigy["safeguard_warmup"] else 0
            pa.lr = float(cfg.lr)
            pa.beta1 = float(cfg.beta1)
            pa.beta2 = float(cfg.beta2)
            pa.step_scale = A_ATAN2 if cfg.use_atan2 else 1.0
            L.check(lib.advopt_prodigy_scalars(ctypes.byref(pa), stream), "advopt_prodigy_scalars")
            self.launch_count += 1
        s = pl.launch_struct(cfg, flags, self.seed)
        if pdev:
            s.prodigy = int(cfg.prodigy["dev"].data_ptr())
        nc = cfg.nesterov_coef
        nv_coef = cfg.beta1 if nc is None else nc
        s.beta1 = f32(cfg.beta1)
        s.beta2 = f32(cfg.beta2)
        # Lion: torch.lerp(grad, m, beta1) for the update, m.lerp_(grad, 1 - beta2)
        s.w_m = f32(1.0 - cfg.beta2) if cfg.algo == L.ALGO_LION else f32(1.0 - cfg.beta1)
        s.w_nest = f32(1 - nv_coef)
        if cfg.algo == L.ALGO_PRODIGY:
            pd = cfg.prodigy
            dd, d0 = pd["d"], pd["d0"]
            s.c_v = f32(dd * dd * (1.0 - cfg.beta2))
            s.c_m = f32(dd * (1.0 - cfg.beta1))
            s.d = f32(dd)
            s.beta3 = f32(pd["beta3"])
            dlr = dd * lr
            s.s_alpha = f32(((dd / d0) * dd) if pd["safeguard_warmup"] else ((dd / d0) * dlr))
            if pd["stats"]:
                s.flags |= L.F_PRODIGY_STATS
        else:
            s.c_v = f32(1.0 - cfg.beta2)
        if cfg.fisher:
            if not cfg.use_atan2:
                st_s = L.AdamLaunch.from_buffer_copy(s)
                st_s.flags = (s.flags | L.F_FISHER_STATS) & ~L.F_PRODIGY_STATS
                L.check(lib.advopt_adam_step(ctypes.byref(st_s), stream), "advopt_adam_step (Fisher statistics)")
                L.check(lib.advopt_fisher_finish(ctypes.byref(st_s), pl.table.ptr, stream), "advopt_fisher_finish")
                self.launch_count += 2
            s.flags |= L.F_FISHER
        if self.kernel_events is not None:
            ev0, ev1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            ev0.record(torch.cuda.current_stream(pl.device))
        kk = cfg.kourkoutas if (cfg.kourkoutas is not None and cfg.kourkoutas.n) else None
        if kk is not None:
            s.flags |= L.F_GRAD_SQ
        L.check(lib.advopt_adam_step(ctypes.byref(s), stream), "advopt_adam_step")
        self.launch_count += 1
        if kk is not None:
            kk.accumulate(pl, stream)
            self.launch_count += 1
        if self.kernel_events is not None:
            ev1.record(torch.cuda.current_stream(pl.device))
            self.kernel_events.append((ev0, ev1, pl))
        if pl.fact_idx:
            self.launch_count += 2
            L.check(lib.advopt_factored_finish(ctypes.byref(s), int(pl.fact_idx_dev.data_ptr()), len(pl.fact_idx),
                                               pl.max_d2, stream), "advopt_factored_finish")
        if cfg.algo == L.ALGO_PRODIGY and cfg.prodigy["stats"]:
            pd = cfg.prodigy
            coef = f32((pd["d"] / pd["d0"]) * (pd["d"] * lr))
            s_bf16 = 1 if (pl.pdt == L.DT_BF16) else 0
            L.check(lib.advopt_prodigy_finish(ctypes.byref(s), int(prodigy_sums.data_ptr()), coef, s_bf16, stream),
                    "advopt_prodigy_finish")
            self.launch_count += 1
        if cfg.spectral:
            sp = pl.spectral
            L.check(lib.advopt_spectral_step(ctypes.byref(s), int(sp.table.data_ptr()), int(sp.col_dev.data_ptr()),
                                             sp.n_col, int(sp.row_dev.data_ptr()), sp.n_row, stream),
                    "advopt_spectral_step")
            self.launch_count += 3 + (1 if sp.n_col else 0) + (1 if sp.n_row else 0)
        self.errors.after_launch(pl.device)
        for st in states:
            st["step"] += 1
        if noise_keep:
            # keep the injected arrays alive until the kernels that read them are done
            torch.cuda.current_stream(pl.device).synchronize()
