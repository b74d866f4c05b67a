"""Argument normalisation shared by the drop-in wrappers."""

from __future__ import annotations

import torch

_F32 = torch.float32


def require_cuda_f32(name: str, *tensors) -> None:
    """The reference's device/dtype guards (``wave_backward.py:1001-1006``): CUDA tensors only;
    this library computes in fp32 only."""
    for t in tensors:
        if t is None:
            continue
        if t.device.type != "cuda":
            raise RuntimeError(f"{name} requires CUDA tensors")
        if t.dtype != _F32:
            raise RuntimeError(f"{name} supports fp32 tensors only (got {t.dtype})")


def i64(t):
    return None if t is None else (t if (t.dtype == torch.int64 and t.is_contiguous()) else
                                   t.to(torch.int64).contiguous())


def i32(t):
    return None if t is None else (t if (t.dtype == torch.int32 and t.is_contiguous()) else
                                   t.to(torch.int32).contiguous())


def f32(t):
    return None if t is None else (t if (t.dtype == _F32 and t.is_contiguous()) else
                                   t.to(_F32).contiguous())


def u8(mask):
    """bool/int mask -> contiguous uint8 view (no copy for contiguous bool)."""
    if mask is None:
        return None
    if mask.dtype == torch.bool:
        return mask.contiguous().view(torch.uint8)
    return (mask != 0).contiguous().view(torch.uint8)


def rows_of(t, G: int, S: int):
    """A per-item parameter as a contiguous [G,S] tensor (the reference's ``as_item_state``)."""
    if t.ndim == 2 and tuple(t.shape) == (G, S):
        return f32(t)
    if t.numel() == S:
        return f32(t.reshape(1, S)).expand(G, S).contiguous() if G > 1 else f32(t.reshape(1, S))
    if t.numel() == G:
        return f32(t.reshape(G, 1)).expand(G, S).contiguous()
    if t.numel() == 1:
        return f32(t.reshape(1, 1)).expand(G, S).contiguous()
    raise ValueError(f"parameter of shape {tuple(t.shape)} is not [G,S], [S], [G] or scalar")


def state_rows(t, S: int):
    """Parameter -> (contiguous [rows,S] tensor, row stride): one shared row -> stride 0.

    Mirrors the addressing of the forward split-reduction wrappers (``dts_fused.py:11-16``
    ``_load_rate`` with ``:193-194``; ``dts_tangent.py:112-113``): a 2-D tensor whose second
    dimension is not 1 ([1,S] or [G,S]) holds state-indexed rows; anything else -- [G], [G,1], a
    scalar, and also a 1-D [S] tensor -- is one value per item row (the value at the item's index),
    broadcast over S."""
    if t.ndim == 2 and int(t.shape[1]) != 1:
        if int(t.shape[1]) != S:
            raise ValueError(f"state-indexed DTS parameters must have S = {S} columns, got {tuple(t.shape)}")
        t = f32(t)
        return t, (0 if int(t.shape[0]) == 1 else S)
    vals = f32(t.reshape(-1))
    g = int(vals.numel())
    full = vals.reshape(g, 1).expand(g, S).contiguous()
    return full, (0 if g == 1 else S)
