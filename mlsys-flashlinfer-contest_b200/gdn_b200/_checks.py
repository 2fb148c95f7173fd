"""Argument checks of the Python entry points, mirroring the reference's
TVM-FFI validation (gdn_decode/solution/python/gdn_decode_utils.h:16-122 and
gdn_prefill/solution/python/cuda_utils.h:42-127): ValueError for device,
layout and shape problems, TypeError for dtypes."""
from __future__ import annotations

import torch

HEAD = 128


def cuda_contig(name, t):
    if not isinstance(t, torch.Tensor):
        raise TypeError(f"{name} must be a torch.Tensor")
    if t.device.type != "cuda":
        raise ValueError(f"{name} must be a CUDA tensor")
    if not t.is_contiguous():
        raise ValueError(f"{name} must be contiguous")


def dim(name, t, d):
    if t.dim() != d:
        raise ValueError(f"{name} must be a {d}D tensor")


def dtype(name, t, dt):
    if t.dtype != dt:
        raise TypeError(f"{name} must be {str(dt).replace('torch.', '')}")


def same_device(ref, **named):
    for n, t in named.items():
        if t is not None and t.device != ref.device:
            raise ValueError(f"q and {n} must be on the same device")


def resolve_scale(scale) -> float:
    if scale is None:
        return 0.0
    if isinstance(scale, torch.Tensor):
        scale = float(scale.item())
    return float(scale)
