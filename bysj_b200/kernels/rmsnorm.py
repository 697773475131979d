"""Last-axis RMSNorm on B200, with input and scale gradients.

Python face of the reference's ``python/kernels/rmsnorm.py`` (validation
messages and autograd contract, lines 15-85).  Two additive widenings:

* ``x`` may be bfloat16 (the output keeps the input dtype; statistics and
  scaling are computed in fp32).  Gradients are float32-only, as in the
  reference.
* ``scale`` may be a per-degree table of shape ``(L+1, feature_dim)`` when
  ``x.shape[-2] == (L+1)**2``: component ``i`` of the irreps axis uses weight
  row ``floor(sqrt(i))``.  The normalisation axis is still the last one only.
"""
from __future__ import annotations

import math

import torch

from .native import _extension, require_dcu


def _degree_table_ok(x: torch.Tensor, scale: torch.Tensor) -> bool:
    return (
        scale.ndim == 2
        and x.ndim >= 2
        and scale.shape[1] == x.shape[-1]
        and x.shape[-2] == scale.shape[0] * scale.shape[0]
    )


def _validate(x: torch.Tensor, scale: torch.Tensor | None, eps: float) -> float:
    if not isinstance(x, torch.Tensor):
        raise TypeError("RMSNorm input must be a tensor")
    if x.dtype not in (torch.float32, torch.bfloat16):
        raise TypeError("RMSNorm requires float32 (or bfloat16) input")
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
        if tuple(scale.shape) != (x.shape[-1],) and not _degree_table_ok(x, scale):
            raise ValueError(
                "RMSNorm scale must have shape (feature_dim,) or, per degree, "
                "(L+1, feature_dim) with x.shape[-2] == (L+1)**2"
            )
        if scale.device != x.device:
            raise ValueError("RMSNorm input and scale must share a device")
        if not scale.is_contiguous():
            raise ValueError("RMSNorm scale must be contiguous")
    try:
        eps = float(eps)
    except (TypeError, ValueError) as error:
        raise ValueError("RMSNorm eps must be a finite positive number") from error
    if not math.isfinite(eps) or eps <= 0.0:
        raise ValueError("RMSNorm eps must be a finite positive number")
    return eps


class _RMSNormFunction(torch.autograd.Function):
    @staticmethod
    def forward(ctx, x: torch.Tensor, scale: torch.Tensor, eps: float):
        output, inverse_rms = _extension("rmsnorm_forward").rmsnorm_forward(x, scale, float(eps))
        ctx.save_for_backward(x, scale, inverse_rms)
        ctx.has_scale = scale.numel() != 0
        return output

    @staticmethod
    def backward(ctx, grad_output: torch.Tensor):
        x, scale, inverse_rms = ctx.saved_tensors
        if x.dtype != torch.float32:
            raise RuntimeError("RMSNorm gradients are implemented for float32 input only")
        need_scale_grad = ctx.has_scale and ctx.needs_input_grad[1]
        grad_x, grad_scale = _extension("rmsnorm_backward").rmsnorm_backward(
            grad_output.contiguous(), x, scale, inverse_rms, need_scale_grad
        )
        return (
            grad_x if ctx.needs_input_grad[0] else None,
            grad_scale if need_scale_grad else None,
            None,
        )


def rmsnorm(x: torch.Tensor, scale: torch.Tensor | None = None, eps: float = 1.0e-6) -> torch.Tensor:
    """Last-axis RMSNorm ``x * rsqrt(mean(x**2) + eps) * scale`` on a B200.

    Contiguous float32 (or bfloat16) input with arbitrary leading dimensions,
    optional float32 ``scale`` of shape ``(x.shape[-1],)`` or the per-degree
    ``(L+1, x.shape[-1])`` table, finite positive ``eps``; no bias.
    """
    eps = _validate(x, scale, eps)
    scale_tensor = scale if scale is not None else x.new_empty((0,), dtype=torch.float32)
    require_dcu(x, scale_tensor)
    return _RMSNormFunction.apply(x, scale_tensor, eps)


def rmsnorm_available() -> bool:
    """Whether this process can run the RMSNorm entry points."""
    try:
        require_dcu()
        extension = _extension("rmsnorm_forward")
        return hasattr(extension, "rmsnorm_backward")
    except (ImportError, OSError, RuntimeError):
        return False


__all__ = ["rmsnorm", "rmsnorm_available"]
