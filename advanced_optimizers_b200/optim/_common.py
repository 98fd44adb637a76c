"""Pieces shared by the optimizer classes."""
from __future__ import annotations

import torch


def reject(cond, what: str):
    """Options the B200 kernels do not implement fail loudly (no fallback)."""
    if cond:
        raise NotImplementedError(f"{what} is not supported by the B200 optimizer kernels")


class ErrorWatch:
    """Device error words of one runner (one int32 per device) that its
    kernels set when a bounded wait gives up, surfaced without a per-step
    synchronisation: after every launch the word is copied into pinned host
    memory behind a CUDA event, and the next launch (or `check(sync=True)`)
    raises once such a copy shows it set.  A step whose kernels gave up has
    left its parameters partly updated; the error says so at the following
    step at the latest."""

    def __init__(self, what: str):
        self.what = what
        self.words = {}   # device -> [device word, pinned copy, event or None]

    def word(self, device, existing: torch.Tensor | None = None) -> torch.Tensor:
        """The device's error word (`existing`, if given, becomes it)."""
        w = self.words.get(device)
        if w is None or (existing is not None and w[0] is not existing):
            w = [existing if existing is not None else torch.zeros(1, dtype=torch.int32, device=device),
                 torch.zeros(1, dtype=torch.int32, pin_memory=True), None]
            self.words[device] = w
        return w[0]

    def after_launch(self, device) -> None:
        w = self.words.get(device)
        if w is None:
            return
        w[1].copy_(w[0], non_blocking=True)
        ev = torch.cuda.Event()
        ev.record(torch.cuda.current_stream(device))
        w[2] = ev

    def check(self, sync: bool = False) -> None:
        for dev, w in self.words.items():
            if sync:
                torch.cuda.synchronize(dev)
                bad = int(w[0].item()) != 0
            else:
                ev = w[2]
                if ev is None or not ev.query():
                    continue
                bad = int(w[1][0]) != 0
            if bad:
                from .. import _lib as L
                raise L.AdvOptError(f"{self.what} gave up waiting for its shared-memory copies (bounded wait); "
                                    "the parameters of that step are only partly updated")


def fix_loaded_state_dtype(state: dict, p: torch.Tensor, group: dict) -> None:
    """state_util.fix_loaded_state_dtype (state_util.py:181-263): undo
    torch's load_state_dict casting of quantised / factored states."""
    mode = group.get("centered_wd_mode", "full")
    if state.get("is_muon") is False:
        # auxiliary Adam state of Muon_adv / AdaMuon_adv: its own precision key
        req = group.get("adam_state_precision", "auto")
        actual = group.get("adam_actual_state_precision", req)
    else:
        req = group.get("state_precision", "auto")
        actual = group.get("actual_state_precision", req)
    # a 'factored' group keeps float32 states for its 1-D params too (the
    # reference would cast them to the param dtype here: its group records
    # 'auto' as the actual precision)
    is_factored = state.get("factored", False) or actual == "factored" or req == "factored"
    if actual == "fp32":
        base = torch.float32
    elif actual == "bf16_sr":
        base = torch.bfloat16
    elif actual == "int8_sr":
        base = torch.uint8
    else:
        base = torch.float32 if is_factored else p.dtype
    skipped = p.numel() == 0 or getattr(p, "_is_dora_scale", False)
    uint8_keys = {"sign", "sign_slow", "sign_buf", "shifter"}
    fp32_keys = {"mu_m_nmf", "mv_m_nmf", "mu_v_nmf", "mv_v_nmf", "mu_m_slow_nmf", "mv_m_slow_nmf",
                 "mu_mbuf_nmf", "mv_mbuf_nmf", "mu_b_nmf", "normuon_v", "mu_vbuf_nmf", "mv_vbuf_nmf"}
    for key, val in list(state.items()):
        if not isinstance(val, torch.Tensor):
            continue
        if key == "anchor_data":
            if skipped or mode == "full":
                if val.dtype != p.dtype:
                    state[key] = val.to(p.dtype)
            elif mode in ("int8", "int4"):
                if val.dtype != torch.int8:
                    state[key] = val.to(torch.int8)
            elif mode == "float8":
                if val.dtype != torch.float8_e4m3fn:
                    state[key] = val.to(torch.float8_e4m3fn)
        elif key in ("anchor_scale", "anchor_min"):
            if val.dtype != p.dtype:
                state[key] = val.to(p.dtype)
        elif key in uint8_keys:
            if val.dtype != torch.uint8:
                state[key] = val.to(torch.uint8)
        elif key in fp32_keys or (key.endswith("_scale") and key != "anchor_scale"):
            if val.dtype != torch.float32:
                state[key] = val.to(torch.float32)
        elif val.is_floating_point():
            if key in ("s", "p0"):
                if val.dtype != p.dtype:
                    state[key] = val.to(p.dtype)
            elif val.dtype != base and key != "wd_scaler":
                state[key] = val.to(base)
        elif actual == "int8_sr" and val.dtype not in (torch.int8, torch.uint8):
            state[key] = val.to(torch.uint8 if key in ("exp_avg_sq", "second_momentum_buffer") else torch.int8)
        if state[key].device != p.device:
            state[key] = state[key].to(p.device)
        if not state[key].is_contiguous():
            state[key] = state[key].contiguous()


def load_state_dict_exact(optimizer, state_dict: dict) -> None:
    """torch.optim.Optimizer.load_state_dict followed by the reference's dtype
    repair (param_update.post_process_loaded_state).  torch casts every state
    tensor of a floating-point parameter to the parameter's dtype on load, so
    a bf16 model's float32 block scales and factors would come back rounded
    to bf16 (and int8 codes through bf16) before the repair widens them
    again; here every loaded state tensor keeps the exact value and dtype it
    was saved with, and the repair then only fixes states saved in another
    dtype (checkpoints written by other code)."""
    saved = state_dict.get("state", {})
    torch.optim.Optimizer.load_state_dict(optimizer, state_dict)
    params = [p for g in optimizer.param_groups for p in g["params"]]
    for idx, st in saved.items():
        if not isinstance(idx, int) or idx >= len(params):
            continue
        p = params[idx]
        live = optimizer.state.get(p)
        if live is None:
            continue
        for key, val in st.items():
            if torch.is_tensor(val) and key in live and key != "step":
                live[key] = val.detach().to(device=p.device, copy=True)
    post_process_loaded_state(optimizer)


def post_process_loaded_state(optimizer) -> None:
    """param_update.post_process_loaded_state (param_update.py:395-409)."""
    for group in optimizer.param_groups:
        for p in group["params"]:
            st = optimizer.state.get(p)
            if st:
                fix_loaded_state_dtype(st, p, group)
