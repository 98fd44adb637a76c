"""GPU test helpers: torch <-> fixture conversion."""
import numpy as np
import torch


def to_torch(arr, dt, device="cuda"):
    arr = np.ascontiguousarray(arr)
    if dt == "bf16" or arr.dtype == np.uint16:
        return torch.from_numpy(arr.view(np.int16).copy()).view(torch.bfloat16).to(device)
    return torch.from_numpy(arr.copy()).to(device)


def to_numpy(t):
    t = t.detach().cpu().contiguous()
    if t.dtype == torch.bfloat16:
        return t.view(torch.int16).numpy().view(np.uint16).copy()
    if t.dtype == torch.float8_e4m3fn:
        return t.view(torch.uint8).numpy().copy()
    return t.numpy().copy()


def _as_like(arr, like: torch.Tensor):
    arr = np.ascontiguousarray(arr)
    if like.dtype == torch.bfloat16:
        src = torch.from_numpy(arr.astype(np.uint16).view(np.int16).copy()).view(torch.bfloat16)
    elif like.dtype == torch.float8_e4m3fn:
        src = torch.from_numpy(arr.astype(np.uint8).copy()).view(torch.float8_e4m3fn)
    else:
        src = torch.from_numpy(arr.copy()).to(like.dtype)
    return src.reshape(like.shape).to(like.device)


def load_state(opt, p, z, step, i):
    """Overwrite p's optimizer state with the fixture's values after `step`
    (step < 0: the initial state)."""
    st = opt.state[p]
    pre = f"st_{step}_{i}_" if step >= 0 else f"st0_{i}_"
    for key, val in list(st.items()):
        fk = pre + key
        if torch.is_tensor(val) and fk in z.files:
            val.copy_(_as_like(z[fk], val))
    if step >= 0 and f"st_{step}_{i}_step" in z.files:
        st["step"] = int(z[f"st_{step}_{i}_step"])
