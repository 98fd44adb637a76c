"""Host side of Muon_adv / AdaMuon_adv: state creation with the reference's
keys, the Newton–Schulz GEMM chain on a per-device workspace, and the
elementwise stages of csrc/muon.cu.

Per matrix the device runs: stage 0 (momentum, X0, ||X0||, normalised and
possibly transposed X in the padded workspace), then ns_steps iterations of
bf16 tcgen05 GEMMs (quintic: A = X X^T, B = bA + cAA, X = aX + BX; CANS:
A = X X^T, X = c1 X + c3 AX; Muon_util.py:7-121), then the RMS rescale and
parameter update (Muon) or the second moment, RMS rescale and update
(AdaMuon).  The auxiliary Adam groups run through the Adam-family runner
with algo AUXADAM (Muon_AuxAdam.py:70-192).
"""
from __future__ import annotations

import ctypes
import math

import torch

from .. import _lib as L
from .._device import dtype_code, ptr, require_cuda_tensor, stream_handle
from .._plan import effective_shape
from ._adam_family import SHIFTER, adjust_wds, f32, init_state_tensor
from ._common import ErrorWatch

NS_ALIGN = 256   # the GEMM's N tile; also a multiple of its M (128) and K (64) tiles


def round_up(x: int, a: int) -> int:
    return (x + a - 1) // a * a


def cans_coeffs(steps: int, a_bound: float):
    """(c1, c3) of each CANS iteration from the singular-value bounds,
    Muon_util.py:69-105, in Python double as the reference computes them."""
    lb, ub = a_bound, 1.0
    out = []
    for _ in range(steps):
        lb_ub = lb * ub
        e_sq = (lb * lb + lb_ub + ub * ub) / 3.0
        k = 2.0 * e_sq ** 1.5
        l_ = lb_ub * (lb + ub)
        den = k + l_
        alpha = 6.0 / den
        out.append((alpha * e_sq, -alpha / 3.0))
        eps_val = (k - l_) / den
        lb, ub = 1.0 - eps_val, 1.0 + eps_val
    return out


def default_cns_bound(rows: int, cols: int) -> float:
    """Muon_util.py:229-237."""
    return max(1.0 / math.sqrt(rows * cols), abs(1.0 / math.sqrt(cols) - 1.0 / math.sqrt(rows)))


def is_suitable_for_muon(p: torch.Tensor, min_dim_size: int = 4, max_aspect_ratio: float = 128.0) -> bool:
    """_is_suitable_for_muon (Muon_util.py:285-331)."""
    s = p.shape
    if p.ndim < 2 or sum(1 for d in s if d > 1) < 2:
        return False
    if s[0] == 1 or s[1] == 1:
        return False
    if p.ndim >= 3:
        inner = 1
        for d in s[1:]:
            inner *= d
        dims = (s[0], inner)
    else:
        dims = tuple(s)
    lo = min(dims)
    if lo < min_dim_size:
        return False
    return max(dims) / lo <= max_aspect_ratio


def storage_code(precision: str, p: torch.Tensor) -> int:
    if precision == "fp32":
        return L.ST_F32
    if precision == "bf16_sr":
        return L.ST_BF16_SR
    if precision == "int8_sr":
        return L.ST_Q8
    if precision == "auto":
        return L.ST_BF16 if p.dtype == torch.bfloat16 else L.ST_F32
    raise NotImplementedError(f"state_precision '{precision}' is not supported by the B200 kernels")


class NSWorkspace:
    """Per-device scratch of the Muon path, grown on demand and then reused:
    the Newton–Schulz buffers X, C ([m_pad][n_pad]) and A, B ([m_pad][m_pad])
    in bf16, X0 and U (bf16, one matrix), partial sums, scalars and the
    bounded-wait error word."""

    def __init__(self, device):
        self.device = device
        self.ns = None
        self.ns_cap = 0
        self.vec = None
        self.vec_cap = 0
        self.partial = None
        self.part_cap = 0
        self.scalars = torch.zeros(4, dtype=torch.float32, device=device)
        self.err = torch.zeros(1, dtype=torch.int32, device=device)
        self.aux = {}

    def scratch(self, key: str, n: int, dtype) -> int:
        """Address of a scratch array of at least n elements (NorMuon row
        denominators, AdaMuon's factored v and its sums), grown on demand."""
        t = self.aux.get(key)
        if t is None or t.numel() < n or t.dtype != dtype:
            t = torch.empty(max(1, n), dtype=dtype, device=self.device)
            self.aux[key] = t
        return int(t.data_ptr())

    def ensure(self, numel: int, m_pad: int, n_pad: int):
        need_ns = 2 * m_pad * n_pad + 2 * m_pad * m_pad
        if need_ns > self.ns_cap:
            self.ns = torch.empty(need_ns, dtype=torch.bfloat16, device=self.device)
            self.ns_cap = need_ns
        need_vec = 2 * round_up(numel, 128)
        if need_vec > self.vec_cap:
            self.vec = torch.empty(need_vec, dtype=torch.bfloat16, device=self.device)
            self.vec_cap = need_vec
        need_part = max((numel + 2047) // 2048, ((m_pad + 31) // 32) * ((n_pad + 31) // 32)) + 1
        if need_part > self.part_cap:
            self.partial = torch.empty(need_part, dtype=torch.float64, device=self.device)
            self.part_cap = need_part

    def pointers(self, numel: int, m_pad: int, n_pad: int):
        base = int(self.ns.data_ptr())
        xy = m_pad * n_pad * 2
        aa = m_pad * m_pad * 2
        x, c = base, base + xy
        a, b = base + 2 * xy, base + 2 * xy + aa
        v = int(self.vec.data_ptr())
        return dict(x=x, c=c, a=a, b=b, x0=v, u=v + 2 * round_up(numel, 128))


def run_ns_chain(ws: NSWorkspace, ptrs, m_pad: int, n_pad: int, steps: int, coeffs, cns: bool, cns_bound: float,
                 stream: int) -> int:
    """The Newton–Schulz iterations on the workspace (X already loaded), in
    one native call (advopt_ns_chain: 3 GEMMs per quintic iteration, 2 per
    CANS iteration, each a tcgen05 GEMM with fp32 accumulation and one bf16
    rounding of alpha*acc + beta*C, matching torch.addmm's bf16 semantics);
    returns the device address of the final X."""
    out = ctypes.c_void_p(0)
    qa, qb, qc = (float(v) for v in coeffs)
    L.check(L.lib().advopt_ns_chain(ptrs["x"], ptrs["c"], ptrs["a"], ptrs["b"], m_pad, n_pad, int(steps),
                                    1 if cns else 0, qa, qb, qc, float(cns_bound), ctypes.byref(out),
                                    int(ws.err.data_ptr()), stream), "advopt_ns_chain")
    return int(out.value)


def ns_launches(steps: int, cns: bool) -> int:
    return steps * (2 if cns else 3)


def ns_flops(m: int, n: int, steps: int, cns: bool) -> int:
    """Algorithmic FLOPs of the chain on an m x n matrix (m <= n):
    quintic 4m^2n + 2m^3 per iteration, CANS 4m^2n."""
    return steps * (4 * m * m * n + (0 if cns else 2 * m ** 3))


def ns_flops_executed(m_pad: int, n_pad: int, steps: int, cns: bool) -> int:
    """Tensor-core FLOPs the chain issues on the padded workspace: X X^T and
    (quintic) b A + c A A computed on the 256 x 256 blocks on or above the
    diagonal only (they are symmetric), the X update in full."""
    blocks = (m_pad // 256) * (m_pad // 256 + 1) // 2          # upper 256 x 256 blocks
    sym_gemm = lambda k: 2 * k * 256 * 256 * blocks             # noqa: E731
    per_iter = sym_gemm(n_pad) + 2 * m_pad * n_pad * m_pad
    if not cns:
        per_iter += sym_gemm(m_pad)
    return steps * per_iter


# the chain's GEMM tiles (128 x 256) per second on one SM at a full wave:
# a sustained ~1.3 PFLOP/s over 148 SMs
NS_TILE_FLOPS_PER_SM_S = 1.3e15 / 148
NS_SMS = 148
# per matrix: the chain's launches and the elementwise stages around it
# (measured on B200: a 1024 x 4096 chain takes 0.42 ms in a step against
# 0.23 ms of tile waves)
NS_CHAIN_OVERHEAD_S = 0.19e-3


def ns_time_estimate(m: int, n: int, steps: int, cns: bool) -> float:
    """Seconds of the chain on an m x n matrix (m <= n), counted in waves of
    the persistent GEMM's 128 x 256 tiles over 148 SMs: a small matrix (the
    1024-row k / v projections) fills few SMs, which its FLOP count alone
    does not show.  X X^T and b A + c A A run on the upper 256 x 256 blocks."""
    m_pad, n_pad = round_up(m, NS_ALIGN), round_up(n, NS_ALIGN)
    nb = m_pad // 256
    sym_tiles = nb * (nb + 1)                   # 2 tiles of 128 x 256 per upper block

    def gemm(tiles, k):
        waves = -(-tiles // NS_SMS)
        return waves * 2.0 * 128 * 256 * k / NS_TILE_FLOPS_PER_SM_S

    per_iter = gemm(sym_tiles, n_pad) + gemm((m_pad // 128) * (n_pad // 256), m_pad)
    if not cns:
        per_iter += gemm(sym_tiles, m_pad)
    return steps * per_iter + NS_CHAIN_OVERHEAD_S


_DEVICE_WS = {}


class MuonMatrixRunner:
    """Runs the Muon / AdaMuon step of one matrix at a time on its device."""

    def __init__(self, seed: int = 42):
        self.seed = int(seed)
        self.ws = {}
        self.launch_count = 0
        self.gemm_events = None   # (start, end, algorithmic flops, executed flops) of each NS chain
        self.errors = ErrorWatch("a Newton-Schulz GEMM")

    def workspace(self, device) -> NSWorkspace:
        # one workspace per device, shared by every runner: the chains of all
        # optimizers on a device run in stream order, one matrix at a time
        ws = _DEVICE_WS.get(device)
        if ws is None:
            ws = NSWorkspace(device)
            _DEVICE_WS[device] = ws
        self.ws[device] = ws
        self.errors.word(device, ws.err)
        return ws

    def check_errors(self):
        self.errors.check(sync=True)

    def after_step(self):
        """Queue the non-blocking read-back of the error words (once per step)."""
        for dev in self.ws:
            self.errors.after_launch(dev)

    @torch.no_grad()
    def step_matrix(self, p, state, *, adamuon: bool, lr: float, beta1: float, beta2: float, eps, nesterov: bool,
                    nesterov_coef, ns_steps: int, ns_eps, ns_coeffs, cns: bool, cns_a_bound, rms_rescaling: bool,
                    use_atan2: bool, sign_projection: bool, weight_decay: float, cautious_wd: bool, sr: bool,
                    precision: str, tensor_id: int, step: int, noise=None, normuon=None, mars_factor=None,
                    vfact: bool = False, low_rank=None):
        """One matrix.  normuon: (1 - beta2, eps) of the NorMuon row-wise
        second moment (state['normuon_v']); mars_factor: approx MARS-M's
        gamma * beta1 / (1 - beta1) (state['last_grad']); vfact: AdaMuon's
        factored second moment (state['mu_vbuf_nmf'], state['mv_vbuf_nmf']);
        low_rank: ortho_rank of the low-rank chain (Muon_util.py:239-270)."""
        require_cuda_tensor(p, "param")
        require_cuda_tensor(p.grad, "grad")
        if p.ndim < 2:
            raise NotImplementedError("the Muon path needs a parameter with at least 2 dimensions")
        numel = p.numel()
        if numel == 0:
            return
        pbf = dtype_code(p.dtype) == L.DT_BF16
        rows = p.shape[0]
        cols = numel // rows
        m, n = min(rows, cols), max(rows, cols)
        m_pad, n_pad = round_up(m, NS_ALIGN), round_up(n, NS_ALIGN)
        ws = self.workspace(p.device)
        if low_rank is not None:
            # the chain runs on the [r][cols] projection only
            if not (precision == "auto" and dtype_code(p.dtype) == L.DT_BF16):
                raise NotImplementedError("low_rank_ortho needs a bf16 update (state_precision='auto' with bf16 "
                                          "params) on the B200 kernels")
            r = min(int(low_rank), rows, cols)
            m2, n2 = min(r, cols), max(r, cols)
            ws_m, ws_n = round_up(m2, NS_ALIGN), round_up(n2, NS_ALIGN)
        else:
            ws_m, ws_n = m_pad, n_pad
        ws.ensure(numel, ws_m, ws_n)
        ptrs = ws.pointers(numel, ws_m, ws_n)
        stream = stream_handle(p.device)

        a = L.MuonArgs()
        a.param, a.grad = ptr(p), ptr(p.grad)
        mb = state["momentum_buffer"]
        a.m = ptr(mb)
        a.m_scale = ptr(state.get("momentum_buffer_scale"))
        if adamuon and not vfact and normuon is None:
            vb = state["second_momentum_buffer"]
            a.v = ptr(vb)
            a.v_scale = ptr(state.get("second_momentum_buffer_scale"))
        if mars_factor is not None:
            a.last_grad = ptr(state["last_grad"])
            a.mars_factor = f32(mars_factor)
        if normuon is not None:
            a.nm_w, a.nm_eps = f32(normuon[0]), f32(normuon[1])
            a.row_v = ptr(state["normuon_v"])
            a.row_den = ws.scratch("row_den", rows, torch.float32)
        if vfact:
            d1, d2 = state["effective_shape"]
            a.d1, a.d2 = d1, d2
            a.v_row, a.v_col = ptr(state["mu_vbuf_nmf"]), ptr(state["mv_vbuf_nmf"])
            a.v_full = ws.scratch("v_full", numel, torch.float32)
            a.v_sums = ws.scratch("v_sums", d1 + L.VCOL_SPLIT * d2, torch.float64)
        a.x0, a.ns, a.u = ptrs["x0"], ptrs["x"], ptrs["u"]
        a.partial, a.scalars = ptr(ws.partial), ptr(ws.scalars)
        a.numel, a.rows, a.cols = numel, rows, cols
        a.ld_ns, a.m_pad, a.n_pad = n_pad, m_pad, n_pad
        a.seed = self.seed
        a.w_m = f32(1.0 - beta1)
        nv = beta1 if nesterov_coef is None else nesterov_coef
        a.w_nest = f32(nv)
        a.beta2 = f32(beta2)
        a.c_v = f32(1.0 - beta2)
        a.eps = f32(eps if eps is not None else 1.0 / math.sqrt(numel))
        a.ns_eps = f32(ns_eps if ns_eps is not None else 1.0 / math.sqrt(numel))
        wd, _ = adjust_wds(weight_decay, 0.0, p)
        a.wd = f32(wd * lr) if wd != 0 else 0.0
        # NorMuon replaces AdaMuon's second moment, atan2 included (AdaMuon_adv.py:635)
        step_scale = lr * (4 / math.pi) if (adamuon and use_atan2 and normuon is None) else lr
        if rms_rescaling:
            a.scale_const = f32(step_scale * 0.2 * math.sqrt(numel))
        else:
            # AdaMuon rescales in the param's shape, Muon (and AdaMuon's
            # NorMuon branch, AdaMuon_adv.py:614-616) in the flattened one
            r, c = (p.shape[-2], p.shape[-1]) if (adamuon and normuon is None) else (rows, cols)
            a.scale_const = f32(step_scale * math.sqrt(max(1, r / c)))
        a.tensor_id = tensor_id & 0xFFFFFFFF
        a.step = step & 0xFFFFFFFF
        flags = 0
        if nesterov:
            flags |= L.MU_NESTEROV
        if sign_projection:
            flags |= L.MU_SIGN
        if sr and pbf:
            flags |= L.MU_SR
        if cautious_wd:
            flags |= L.MU_CAUTIOUS
        if rms_rescaling:
            flags |= L.MU_RMS
        if rows > cols:
            flags |= L.MU_TRANSPOSED
        if adamuon and use_atan2 and normuon is None:
            flags |= L.MU_ATAN2
        if mars_factor is not None:
            flags |= L.MU_MARS
        if normuon is not None:
            flags |= L.MU_NORMUON
        if vfact:
            flags |= L.MU_VFACT
        if low_rank is not None:
            flags |= L.MU_LOWRANK
        keep = []
        if noise is not None:
            flags |= L.MU_NOISE_IN
            for label, field in (("momentum_buffer", "noise_m"), ("second_momentum_buffer", "noise_v"),
                                 ("param", "noise_p")):
                t = noise.get(label)
                if t is not None:
                    t = t.to(device=p.device, dtype=torch.int32).contiguous()
                    if t.numel() < numel:
                        raise ValueError(f"injected noise '{label}' has {t.numel()} entries, {numel} needed")
                    keep.append(t)
                    setattr(a, field, ptr(t))
        a.flags = flags
        a.m_storage = storage_code(precision, p)
        a.v_storage = storage_code(precision, p) if (adamuon and not vfact and normuon is None) else 0
        auto_bf16 = precision == "auto" and pbf
        a.param_bf16 = 1 if pbf else 0
        a.math_bf16 = 1 if auto_bf16 else 0
        a.update_bf16 = 1 if auto_bf16 else 0

        lib = L.lib()
        L.check(lib.advopt_muon_stage(ctypes.byref(a), 0, stream), "advopt_muon_stage (prep)")
        # eps and the CANS bound come from the full shape, low rank or not (Muon_util.py:225-237)
        bound = cns_a_bound if cns_a_bound is not None else default_cns_bound(rows, cols)
        if self.gemm_events is not None:
            ev0, ev1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            ev0.record(torch.cuda.current_stream(p.device))
        if low_rank is not None:
            sketch = None if noise is None else noise.get("sketch")
            self._low_rank_chain(a, ws, ptrs, r, ws_m, ws_n, ns_steps, ns_coeffs, cns, bound, stream, sketch)
            flops = (ns_flops(m2, n2, ns_steps, cns) + 6 * rows * cols * r,
                     ns_flops_executed(ws_m, ws_n, ns_steps, cns) + 6 * rows * cols * r)
        else:
            a.ns_result = run_ns_chain(ws, ptrs, m_pad, n_pad, ns_steps, ns_coeffs, cns, bound, stream)
            flops = (ns_flops(m, n, ns_steps, cns), ns_flops_executed(m_pad, n_pad, ns_steps, cns))
        if self.gemm_events is not None:
            ev1.record(torch.cuda.current_stream(p.device))
            self.gemm_events.append((ev0, ev1) + flops)
        u_ready = low_rank is not None       # the low-rank chain leaves U in `u`
        if u_ready and normuon is None and not vfact and not adamuon:
            L.check(lib.advopt_muon_stage(ctypes.byref(a), 13, stream), "advopt_muon_stage (U statistics)")
            L.check(lib.advopt_muon_stage(ctypes.byref(a), 2, stream), "advopt_muon_stage (update)")
            self.launch_count += 2 + 2
        elif normuon is not None:
            if not u_ready:
                L.check(lib.advopt_muon_stage(ctypes.byref(a), 3, stream), "advopt_muon_stage (U)")
            L.check(lib.advopt_muon_stage(ctypes.byref(a), 7, stream), "advopt_muon_stage (NorMuon rows)")
            L.check(lib.advopt_muon_stage(ctypes.byref(a), 8, stream), "advopt_muon_stage (NorMuon statistics)")
            L.check(lib.advopt_muon_stage(ctypes.byref(a), 9, stream), "advopt_muon_stage (NorMuon update)")
            self.launch_count += 3 + 1 + 1 + 2 + 1
        elif vfact:
            if not u_ready:
                L.check(lib.advopt_muon_stage(ctypes.byref(a), 3, stream), "advopt_muon_stage (U)")
            L.check(lib.advopt_muon_stage(ctypes.byref(a), 10, stream), "advopt_muon_stage (AdaMuon factored v)")
            L.check(lib.advopt_muon_stage(ctypes.byref(a), 11, stream), "advopt_muon_stage (AdaMuon update)")
            self.launch_count += 3 + 1 + 5 + 1
        elif adamuon:
            if not u_ready:
                L.check(lib.advopt_muon_stage(ctypes.byref(a), 3, stream), "advopt_muon_stage (U)")
            L.check(lib.advopt_muon_stage(ctypes.byref(a), 4, stream), "advopt_muon_stage (AdaMuon statistics)")
            L.check(lib.advopt_muon_stage(ctypes.byref(a), 5, stream), "advopt_muon_stage (AdaMuon update)")
            self.launch_count += 3 + 1 + 2 + 1
        else:
            L.check(lib.advopt_muon_stage(ctypes.byref(a), 1, stream), "advopt_muon_stage (U, scale)")
            L.check(lib.advopt_muon_stage(ctypes.byref(a), 2, stream), "advopt_muon_stage (update)")
            self.launch_count += 3 + 2 + 1
        self.launch_count += ns_launches(ns_steps, cns)
        if keep:
            torch.cuda.current_stream(p.device).synchronize()

    def _low_rank_chain(self, a, ws, ptrs, r, m_pad2, n_pad2, ns_steps, ns_coeffs, cns, bound, stream, sketch):
        """Muon_util.py:239-270 on X0 = the update in bf16 ([rows][cols], after
        stage 0): MG = X0 S, Q = qr(MG), P = Q^T X0, the chain on P, U = Q NS(P)
        into `u`."""
        lib = L.lib()
        rows, cols = a.rows, a.cols
        x0 = ptrs["x0"]
        s_ptr = ws.scratch("lr_sketch", cols * r, torch.bfloat16)
        if sketch is not None:
            t = sketch.to(device=ws.device).reshape(-1)
            if t.dtype != torch.bfloat16:
                # the reference's bf16 bit patterns, as integers
                t = t.to(torch.int32).to(torch.int16).view(torch.bfloat16)
            if t.numel() != cols * r:
                raise ValueError(f"injected sketch has {t.numel()} entries, {cols * r} needed")
            ws.aux["lr_sketch"][: cols * r].copy_(t)
        else:
            L.check(lib.advopt_lr_sketch(s_ptr, cols, r, a.seed, a.tensor_id, a.step, stream), "advopt_lr_sketch")
        mg = ws.scratch("lr_mg", rows * r, torch.bfloat16)
        q = ws.scratch("lr_q", rows * r, torch.bfloat16)
        pp = ws.scratch("lr_p", r * cols, torch.bfloat16)
        oo = ws.scratch("lr_o", r * cols, torch.bfloat16)
        work = ws.scratch("lr_work", int(lib.advopt_lr_qr_work(rows, r)), torch.float64)
        L.check(lib.advopt_lr_gemm(mg, x0, s_ptr, rows, r, cols, 0, stream), "advopt_lr_gemm (M S)")
        L.check(lib.advopt_lr_qr(q, mg, rows, r, work, stream), "advopt_lr_qr")
        L.check(lib.advopt_lr_gemm(pp, q, x0, r, cols, rows, 1, stream), "advopt_lr_gemm (Q^T M)")
        # the ordinary chain on P [r][cols]: stage 6 (P -> workspace), chain, stage 3 (-> oo)
        b = L.MuonArgs.from_buffer_copy(a)
        b.grad = pp
        b.param, b.m = 0, 0
        b.u = oo
        b.rows, b.cols, b.numel = r, cols, r * cols
        b.m_pad, b.n_pad, b.ld_ns = m_pad2, n_pad2, n_pad2
        b.ns = ptrs["x"]
        b.param_bf16 = 1
        b.flags = L.MU_TRANSPOSED if r > cols else 0
        L.check(lib.advopt_muon_stage(ctypes.byref(b), 6, stream), "advopt_muon_stage (low-rank load)")
        b.ns_result = run_ns_chain(ws, ptrs, m_pad2, n_pad2, ns_steps, ns_coeffs, cns, bound, stream)
        L.check(lib.advopt_muon_stage(ctypes.byref(b), 3, stream), "advopt_muon_stage (low-rank U)")
        L.check(lib.advopt_lr_gemm(a.u, q, oo, rows, cols, r, 0, stream), "advopt_lr_gemm (Q NS(P))")
        self.launch_count += (0 if sketch is not None else 1) + 3 + 10 + 1 + 3 + 1 + 1


_NS_RUNNER = None


@torch.no_grad()
def newton_schulz(G: torch.Tensor, steps: int = 5, eps: float | None = 1e-7,
                  coeffs: tuple[float, float, float] = (3.4445, -4.7750, 2.0315), cns: bool = False,
                  cns_a_bound: float | None = None, low_rank_ortho: bool = False, ortho_rank: int = 128,
                  G_sketch=None, compiled: bool = False) -> torch.Tensor:
    """Muon_util.newton_schulz (Muon_util.py:193-283) on the tcgen05 GEMM
    chain: X = bf16(G) (transposed if rows > cols), divided by
    max(||X||_F, eps), then `steps` quintic or CANS iterations in bf16 with
    fp32 accumulation; returns a new tensor in G's dtype.  With
    low_rank_ortho (bf16 G), the chain runs on Q^T G for the Q factor of
    G @ G_sketch (a [cols][r] sketch; drawn N(0, 1) when None) and the result
    is Q NS(Q^T G)."""
    global _NS_RUNNER
    if low_rank_ortho and G.dtype != torch.bfloat16:
        raise NotImplementedError("low_rank_ortho needs a bf16 matrix on the B200 kernels")
    if G.ndim != 2:
        raise NotImplementedError("newton_schulz takes one 2-D matrix")
    require_cuda_tensor(G, "G")
    dtype_code(G.dtype)
    rows, cols = G.shape
    numel = G.numel()
    out = torch.empty((rows, cols), dtype=torch.bfloat16, device=G.device)
    if numel == 0:
        return out.to(G.dtype)
    if _NS_RUNNER is None:
        _NS_RUNNER = MuonMatrixRunner()
    ws = _NS_RUNNER.workspace(G.device)
    m, n = min(rows, cols), max(rows, cols)
    m_pad, n_pad = round_up(m, NS_ALIGN), round_up(n, NS_ALIGN)
    r = min(int(ortho_rank), rows, cols) if low_rank_ortho else 0
    if r > 0:
        ws_m, ws_n = round_up(min(r, cols), NS_ALIGN), round_up(max(r, cols), NS_ALIGN)
    else:
        ws_m, ws_n = m_pad, n_pad
    ws.ensure(numel, ws_m, ws_n)
    ptrs = ws.pointers(numel, ws_m, ws_n)
    stream = stream_handle(G.device)
    a = L.MuonArgs()
    a.grad = ptr(G)
    a.x0, a.ns, a.u = ptrs["x0"], ptrs["x"], ptr(out)
    a.partial, a.scalars = ptr(ws.partial), ptr(ws.scalars)
    a.numel, a.rows, a.cols = numel, rows, cols
    a.ld_ns, a.m_pad, a.n_pad = n_pad, m_pad, n_pad
    a.ns_eps = f32(eps if eps is not None else 1.0 / math.sqrt(numel))
    a.flags = L.MU_TRANSPOSED if rows > cols else 0
    a.param_bf16 = 1 if G.dtype == torch.bfloat16 else 0
    lib = L.lib()
    bound = cns_a_bound if cns_a_bound is not None else default_cns_bound(rows, cols)
    if r > 0:
        a.flags |= L.MU_LOWRANK
        a.seed = _NS_RUNNER.seed
        L.check(lib.advopt_muon_stage(ctypes.byref(a), 6, stream), "advopt_muon_stage (X0)")
        _NS_RUNNER._low_rank_chain(a, ws, ptrs, r, ws_m, ws_n, steps, coeffs, cns, bound, stream, G_sketch)
        return out
    L.check(lib.advopt_muon_stage(ctypes.byref(a), 6, stream), "advopt_muon_stage (load)")
    a.ns_result = run_ns_chain(ws, ptrs, m_pad, n_pad, steps, coeffs, cns, bound, stream)
    L.check(lib.advopt_muon_stage(ctypes.byref(a), 3, stream), "advopt_muon_stage (store)")
    return out if G.dtype == torch.bfloat16 else out.to(G.dtype)


def init_muon_state(p, state, precision: str, adamuon: bool, group=None):
    """Muon_adv.__init_state / AdaMuon_adv.__init_state, non-factored
    (Muon_adv.py:304-345, AdaMuon_adv.py:361-397): the momentum; AdaMuon's
    second moment, full or factored (effective shape, mu_vbuf_nmf /
    mv_vbuf_nmf, shifter) unless NorMuon replaces it; NorMuon's row-wise
    normuon_v; MARS-M's last_grad."""
    group = group or {}
    normuon = bool(group.get("normuon_variant", False))
    state["factored"] = False
    init_state_tensor(state, "momentum_buffer", p, precision)
    if adamuon:
        use_f2 = bool(group.get("factored_2nd", False)) and not normuon and not (
            p.ndim == 1 and not group.get("vector_reshape", False))
        state["factored_2nd"] = use_f2
        if use_f2:
            d1, d2 = effective_shape(p.numel())
            state["effective_shape"] = (d1, d2)
            state["mu_vbuf_nmf"] = torch.zeros(d1, device=p.device, dtype=torch.float32)
            state["mv_vbuf_nmf"] = torch.zeros(d2, device=p.device, dtype=torch.float32)
            state["shifter"] = torch.tensor(SHIFTER, device=p.device, dtype=torch.uint8)
        elif not normuon:
            init_state_tensor(state, "second_momentum_buffer", p, precision, non_neg=True)
    if normuon and p.ndim >= 2:
        state["normuon_v"] = torch.zeros(p.shape[0], device=p.device, dtype=torch.float32)
    if group.get("approx_mars", False):
        state["last_grad"] = torch.zeros_like(p, device=p.device, dtype=p.dtype)
