"""Device-side helpers for the host layer: small table uploads through a
pinned ring, the CUDA stream handle, and dtype checks.  PyTorch is used only
for device memory and streams."""
from __future__ import annotations

import numpy as np
import torch


def require_cuda_tensor(t: torch.Tensor, what: str):
    if not t.is_cuda:
        raise NotImplementedError(f"{what}: tensors must live on a CUDA device (no CPU fallback)")
    if t.is_sparse:
        raise NotImplementedError(f"{what}: sparse gradients are not supported")
    if not t.is_contiguous():
        raise NotImplementedError(f"{what}: tensors must be contiguous")


def dtype_code(dt: torch.dtype) -> int:
    if dt == torch.float32:
        return 0
    if dt == torch.bfloat16:
        return 1
    raise NotImplementedError(f"parameter dtype {dt} is not supported (float32 and bfloat16 are)")


def stream_handle(device) -> int:
    return torch.cuda.current_stream(device).cuda_stream


def ptr(t) -> int:
    return 0 if t is None else int(t.data_ptr())


def aligned16(*ts) -> bool:
    return all(t is None or (t.data_ptr() % 16 == 0) for t in ts)


class DeviceTable:
    """A device buffer refreshed from host bytes each step.  Uploads go
    through a ring of pinned host buffers; a slot is reused only after the
    copy that last read it has completed (an event per slot)."""

    def __init__(self, nbytes: int, device, ring: int = 2):
        self.nbytes = int(nbytes)
        self.device = device
        self.dev = torch.empty(max(1, self.nbytes), dtype=torch.uint8, device=device)
        self.host = [torch.empty(max(1, self.nbytes), dtype=torch.uint8, pin_memory=True) for _ in range(ring)]
        self.events = [None] * ring
        self.slot = 0

    @property
    def ptr(self) -> int:
        return int(self.dev.data_ptr())

    def upload(self, arr: np.ndarray):
        b = arr.view(np.uint8).reshape(-1)
        assert b.size <= self.nbytes
        i = self.slot
        self.slot = (i + 1) % len(self.host)
        if self.events[i] is not None:
            self.events[i].synchronize()
        h = self.host[i]
        h.numpy()[: b.size] = b
        self.dev[: b.size].copy_(h[: b.size], non_blocking=True)
        ev = torch.cuda.Event()
        ev.record(torch.cuda.current_stream(self.device))
        self.events[i] = ev


def upload_static(arr: np.ndarray, device) -> torch.Tensor:
    """One-off upload of a table that does not change between steps."""
    b = np.ascontiguousarray(arr).view(np.uint8).reshape(-1)
    t = torch.from_numpy(b.copy())
    return t.to(device)
