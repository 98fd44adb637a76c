"""Shared host logic of Muon_adv and AdaMuon_adv: routing of each parameter
to the Muon path or the auxiliary Adam (Muon_adv.py:283-357,
AdaMuon_adv.py:293-395), state creation, and the per-step dispatch."""
from __future__ import annotations

import torch

from .. import _lib as L
from ._adam_family import AdamCfg, AdamFamilyRunner, SUPPORTED_PRECISIONS, SpectralInit, init_adam_state
from ._common import load_state_dict_exact, reject
from ._kourkoutas import KourkoutasBeta
from ._muon_family import MuonMatrixRunner, init_muon_state, is_suitable_for_muon


class MuonFamilyBase(torch.optim.Optimizer):
    _adamuon = False

    def _setup(self):
        self.device = self.param_groups[0]["params"][0].device if self.param_groups[0]["params"] else None
        self._adam_runner = AdamFamilyRunner(seed=42)
        self._spectral_init = SpectralInit()
        self._muon_runner = MuonMatrixRunner(seed=42)
        self._ids = {}
        self._mstep = {}
        self._test_noise = None
        self.init_step()
        # Kourkoutas-beta of the auxiliary Adam, built after the states as the
        # reference does (Muon_adv.py:248-252): a group holding a Muon param
        # has had adam_kourkoutas_beta switched off by then
        self.kourkoutas_helper = (KourkoutasBeta(self, prefix="adam_")
                                  if any(g.get("adam_kourkoutas_beta", False) for g in self.param_groups) else None)

    def load_state_dict(self, state_dict: dict) -> None:
        load_state_dict_exact(self, state_dict)
        self._adam_runner.invalidate()
        if self.kourkoutas_helper is not None:
            self.kourkoutas_helper.loaded()

    @property
    def supports_fused_back_pass(self):
        return True

    @property
    def supports_memory_efficient_fp16(self):
        return True

    @property
    def supports_flat_params(self):
        return False

    def compile(self, *args, **kwargs):
        """The step is already fused into native kernels: nothing to compile."""
        return None

    def init_step(self):
        for group in self.param_groups:
            for p in group["params"]:
                self._init_state(p, group)

    def _tid(self, p):
        t = self._ids.get(id(p))
        if t is None:
            t = len(self._ids)
            self._ids[id(p)] = t
        return t

    @torch.no_grad()
    def _init_state(self, p, group):
        state = self.state[p]
        if "is_muon" in state:
            return
        if group.get("use_muon") is not None:
            is_muon = bool(group["use_muon"])
        elif group.get("optim_type") is not None:
            is_muon = group["optim_type"] == "muon"
        else:
            is_muon = is_suitable_for_muon(p)
        if is_muon:
            req = group["state_precision"]
            reject(req not in SUPPORTED_PRECISIONS, f"state_precision='{req}' on the Muon path")
            group["actual_state_precision"] = req
            init_muon_state(p, state, req, self._adamuon, group)
            group["adam_kourkoutas_beta"] = False
            state["is_muon"] = True
        else:
            req = group.get("adam_state_precision", "auto")
            reject(req not in SUPPORTED_PRECISIONS, f"adam_state_precision='{req}'")
            # adam_nnmf_factor factors the 2-D params only; 1-D ones keep
            # adam_state_precision (Muon_AuxAdam.py:24-34)
            is_vec = p.dim() == 1 and not group.get("vector_reshape", False)
            smmf = req == "factored" or (group.get("adam_nnmf_factor", False) and not is_vec)
            group["adam_actual_state_precision"] = "auto" if req == "factored" else req
            init_adam_state(p, state, precision="factored" if smmf else req,
                            factored_2nd=group.get("adam_factored_2nd", False),
                            beta1=group["adam_betas"][0], vector_reshape=group.get("vector_reshape", False),
                            centered_wd=group.get("centered_wd", 0.0),
                            centered_wd_mode=group.get("centered_wd_mode", "float8"),
                            fisher_wd=group.get("adam_fisher_wd", False))
            if group.get("adam_spectral_normalization", False):
                self._spectral_init(state, p)            # Muon_AuxAdam.py:63-64
            state["is_muon"] = False

    def _adam_cfg(self, group, factored=False):
        """Muon_AuxAdam._adam_step_parameter's hyperparameters (Muon_AuxAdam.py:70-192).

        Kourkoutas-beta (Muon_adv.py:377-391, AdaMuon_adv.py:425-441): with a
        helper, every auxiliary-Adam param pools its grad norm into its layer
        (by layer key, whatever its group).  The dynamic beta2 reaches the v
        update only without bias correction (with it, adam_betas is read
        again after the lookup); then params outside every layer take
        group['betas'][1] where the group has 'betas' (AdaMuon), else
        adam_betas[1] (Kourkoutas.py:250-257)."""
        kk = self.kourkoutas_helper
        bc = group.get("adam_use_bias_correction", True)
        betas = group["adam_betas"]
        if kk is not None and not bc and group.get("betas") is not None:
            betas = (betas[0], group["betas"][1])
        req = group.get("adam_state_precision", "auto")
        return AdamCfg(algo=L.ALGO_AUXADAM, lr=group["lr"], betas=betas, eps=group["adam_eps"],
                       weight_decay=group["adam_weight_decay"],
                       precision="factored" if (factored or req == "factored") else
                       group.get("adam_actual_state_precision", req),
                       nesterov=group.get("adam_nesterov", False), nesterov_coef=group.get("adam_nesterov_coef"),
                       use_bias_correction=group.get("adam_use_bias_correction", True),
                       use_atan2=group.get("adam_use_atan2", False), cautious_wd=group.get("cautious_wd", False),
                       fisher_wd=group.get("adam_fisher_wd", False), centered_wd=group.get("centered_wd", 0.0),
                       centered_wd_mode=group.get("centered_wd_mode", "float8"),
                       stochastic_rounding=self.stochastic_rounding,
                       kourkoutas=kk, kourkoutas_apply=not bc,
                       spectral=group.get("adam_spectral_normalization", False))

    def _muon_hp(self, group, p):
        raise NotImplementedError

    def _normuon_hp(self, group):
        """(1 - beta2, eps) of NorMuon's row-wise second moment."""
        raise NotImplementedError

    def _step_params(self, gi, group, params):
        for p in params:
            self._init_state(p, group)
        adam = [p for p in params if not self.state[p]["is_muon"]]
        muon = [p for p in params if self.state[p]["is_muon"]]
        if adam:
            by_dtype = {}
            for p in adam:
                by_dtype.setdefault((p.dtype, p.device), []).append(p)
            if self.kourkoutas_helper is not None:
                # once per step, before the first auxiliary-Adam param (Muon_adv.py:382-384)
                self.kourkoutas_helper.maybe_prepare(self.state[adam[0]]["step"], adam[0].device)
            if self._test_noise is not None:
                self._adam_runner.test_noise = {k: v for k, v in self._test_noise.items()
                                                if any(id(p) == k for p in adam)}
            for (dt, dev), ps_all in by_dtype.items():
                # factored tensors compute in float32; under adam_nnmf_factor
                # the 1-D params of the group keep adam_state_precision
                parts = {}
                for p in ps_all:
                    parts.setdefault(bool(self.state[p].get("factored", False)), []).append(p)
                for fac, ps in parts.items():
                    cfg = self._adam_cfg(group, factored=fac)
                    key = (gi, dt, dev, fac, tuple(id(p) for p in ps))
                    self._adam_runner.run(key, ps, [self.state[p] for p in ps], [self._tid(p) for p in ps], cfg)
            self._adam_runner.test_noise = None
        for p in muon:
            hp = self._muon_hp(group, p)
            t = self._mstep.get(id(p), 0)
            self._mstep[id(p)] = t + 1
            nz = None if self._test_noise is None else self._test_noise.get(id(p), {})
            st = self.state[p]
            self._muon_runner.step_matrix(p, st, adamuon=self._adamuon, tensor_id=self._tid(p), step=t,
                                          noise=nz, sr=self.stochastic_rounding,
                                          precision=group["actual_state_precision"],
                                          normuon=self._normuon_hp(group) if "normuon_v" in st else None,
                                          mars_factor=(group["mars_gamma"] * hp["beta1"] / (1.0 - hp["beta1"])
                                                       if "last_grad" in st else None),
                                          vfact=bool(st.get("factored_2nd", False)),
                                          low_rank=group["ortho_rank"] if group.get("low_rank_ortho", False) else None,
                                          **hp)

    @torch.no_grad()
    def step_parameter(self, p: torch.Tensor, group: dict, i: int | None = None):
        if p.grad is None:
            return
        gi = next(k for k, g in enumerate(self.param_groups) if g is group)
        self._step_params(gi, group, [p])

    @torch.no_grad()
    def step(self, closure=None):
        loss = None
        if closure is not None:
            with torch.enable_grad():
                loss = closure()
        # chains of an earlier step that gave up are reported here, without a sync
        self._muon_runner.errors.check()
        for gi, group in enumerate(self.param_groups):
            params = [p for p in group["params"] if p.grad is not None]
            if params:
                self._step_params(gi, group, params)
        self._muon_runner.after_step()
        self._test_noise = None
        return loss

    def check_errors(self):
        """Synchronise and raise if a kernel of this optimizer reported a bounded wait that gave up."""
        self._adam_runner.check_errors()
        self._muon_runner.check_errors()

    def set_test_noise(self, noise):
        """Use the reference's random integers for the next step only:
        {param: {'momentum_buffer' | 'second_momentum_buffer' | 'exp_avg' |
        'exp_avg_sq' | 'param': int tensor}}.  None restores Philox."""
        self._test_noise = None if noise is None else {id(p): v for p, v in noise.items()}

    @property
    def launch_count(self):
        return self._adam_runner.launch_count + self._muon_runner.launch_count
