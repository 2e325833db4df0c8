"""Helpers for the GPU tests: move numpy arrays to device buffers (torch is used
only for device memory and streams) and back."""
import numpy as np


def to_dev(torch, arr: np.ndarray, pad: int = 0):
    """Device copy of `arr` as a flat uint8 tensor (plus `pad` spare bytes)."""
    b = np.ascontiguousarray(arr).view(np.uint8).ravel()
    t = torch.empty(b.size + pad, dtype=torch.uint8, device="cuda")
    if b.size:
        t[: b.size].copy_(torch.from_numpy(b.copy()))
    return t


def empty_dev(torch, nbytes: int, fill: int = 0xA5):
    t = torch.empty(max(nbytes, 1), dtype=torch.uint8, device="cuda")
    t.fill_(fill)
    return t


def from_dev(t, dtype, shape=None, nbytes=None):
    a = t.cpu().numpy()
    if nbytes is not None:
        a = a[:nbytes]
    a = a.view(dtype)
    return a.reshape(shape) if shape is not None else a
