"""PyTorch RMSNorm for explicit testing and comparison.

``rmsnorm`` is the ``reference.rmsnorm`` of lipengfei1409/bysj
(``python/reference/rmsnorm.py:9-48``, validation messages included).
``rmsnorm_per_degree`` is the per-degree weight extension: ``rmsnorm`` applied
to each degree slice ``x[..., l*l:(l+1)*(l+1), :]`` with weight row ``w[l]``.
Plain PyTorch on any device; the CUDA kernels never call it.
"""
from __future__ import annotations

import math

import torch


def _check(x: torch.Tensor, scale: torch.Tensor | None, eps: float) -> float:
    if not isinstance(x, torch.Tensor):
        raise TypeError("RMSNorm input must be a tensor")
    if x.dtype != torch.float32:
        raise TypeError("RMSNorm requires float32 input")
    if x.ndim < 1:
        raise ValueError("RMSNorm input must have at least one dimension")
    if x.shape[-1] <= 0:
        raise ValueError("RMSNorm feature dimension must be positive")
    if not x.is_contiguous():
        raise ValueError("RMSNorm input must be contiguous")
    if scale is not None:
        if not isinstance(scale, torch.Tensor):
            raise TypeError("RMSNorm scale must be a tensor or None")
        if scale.dtype != torch.float32:
            raise TypeError("RMSNorm scale must be float32")
        if tuple(scale.shape) != (x.shape[-1],):
            raise ValueError("RMSNorm scale must have shape (feature_dim,)")
        if scale.device != x.device:
            raise ValueError("RMSNorm input and scale must share a device")
        if not scale.is_contiguous():
            raise ValueError("RMSNorm scale must be contiguous")
    try:
        value = float(eps)
    except (TypeError, ValueError) as error:
        raise ValueError("RMSNorm eps must be a finite positive number") from error
    if not math.isfinite(value) or value <= 0.0:
        raise ValueError("RMSNorm eps must be a finite positive number")
    return value


def rmsnorm(x: torch.Tensor, scale: torch.Tensor | None = None, eps: float = 1.0e-6):
    """``x * rsqrt(mean(x**2, -1) + eps) * scale`` (no bias), differentiable."""
    eps = _check(x, scale, eps)
    out = x * torch.rsqrt(x.square().mean(dim=-1, keepdim=True) + eps)
    return out if scale is None else out * scale


def rmsnorm_per_degree(x: torch.Tensor, weight: torch.Tensor, eps: float = 1.0e-6):
    """RMSNorm over the last axis with weight row ``floor(sqrt(i))`` for component i.

    ``x`` is ``(..., (L+1)**2, C)`` and ``weight`` ``(L+1, C)``.
    """
    levels = weight.shape[0]
    if x.shape[-2] != levels * levels:
        raise ValueError("per-degree RMSNorm needs x.shape[-2] == (L+1)**2")
    pieces = [
        rmsnorm(x[..., l * l:(l + 1) * (l + 1), :].contiguous(), weight[l].contiguous(), eps)
        for l in range(levels)
    ]
    return torch.cat(pieces, dim=-2)


__all__ = ["rmsnorm", "rmsnorm_per_degree"]
