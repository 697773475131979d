"""Fused rotate-back aggregation on B200 (the flash seam of DeepMD's SO(2) block).

``rotate_back_aggregate`` takes the argument list the reference records for
DeepMD's ``SO2Convolution._flash_atten_fn`` (``docs/deepmd-fused-dispatch.md``
lines 127-128 of lipengfei1409/bysj, marked there as not yet wired): the edge
messages in each edge's local frame are rotated back by the edge's
block-diagonal rotation, weighted by the attention coefficients (and an
optional per-edge rescale) and summed into their destination -- one pass, the
rotated messages never reach HBM.  Forward only (the seam is an inference
path); the validation order and exception types follow the other wrappers.
"""
from __future__ import annotations

import torch

from .native import _extension, require_dcu


def rotation_width(lmax: int) -> int:
    """Packed rotation row length: sum over degrees 0..lmax of (2l+1)^2."""
    return (lmax + 1) * (2 * lmax + 1) * (2 * lmax + 3) // 3


def _validate(x_local, rotation, rotate_inv_rescale, attn_alpha, order, row_ptr, dst, lmax,
              heads):
    named = (("x_local", x_local), ("rotation", rotation), ("attn_alpha", attn_alpha),
             ("row_ptr", row_ptr), ("dst", dst))
    for name, tensor in named:
        if not isinstance(tensor, torch.Tensor):
            raise TypeError(f"rotate-back {name} must be a tensor")
    for name, tensor in (("rotate_inv_rescale", rotate_inv_rescale), ("order", order)):
        if tensor is not None and not isinstance(tensor, torch.Tensor):
            raise TypeError(f"rotate-back {name} must be a tensor or None")
    floats = [x_local, rotation, attn_alpha] + ([rotate_inv_rescale]
                                                if rotate_inv_rescale is not None else [])
    if any(t.dtype != torch.float32 for t in floats):
        raise TypeError("rotate-back value tensors must be float32")
    if any(t.dtype != torch.int64 for t in (row_ptr, dst) + ((order,) if order is not None
                                                              else ())):
        raise TypeError("rotate-back row_ptr, dst and order must be int64")
    lmax, heads = int(lmax), int(heads)
    if not 0 <= lmax <= 3:
        raise ValueError("rotate-back lmax must be in [0, 3]")
    if x_local.ndim != 3 or x_local.shape[1] != (lmax + 1) ** 2:
        raise ValueError("rotate-back x_local must have shape (n_edges, (lmax+1)^2, channels)")
    n_edges, _, channels = x_local.shape
    if tuple(rotation.shape) != (n_edges, rotation_width(lmax)):
        raise ValueError("rotate-back rotation must have shape (n_edges, sum_l (2l+1)^2)")
    if heads <= 0 or channels % heads:
        raise ValueError("rotate-back heads must divide the channels")
    if tuple(attn_alpha.shape) != (n_edges, heads):
        raise ValueError("rotate-back attn_alpha must have shape (n_edges, heads)")
    if rotate_inv_rescale is not None and rotate_inv_rescale.numel() != n_edges:
        raise ValueError("rotate-back rotate_inv_rescale must have one value per edge")
    if row_ptr.ndim != 1 or row_ptr.numel() < 1:
        raise ValueError("rotate-back row_ptr must be a one-dimensional exclusive prefix sum")
    if tuple(dst.shape) != (n_edges,):
        raise ValueError("rotate-back dst must have shape (n_edges,)")
    if order is not None and tuple(order.shape) != (n_edges,):
        raise ValueError("rotate-back order must have shape (n_edges,)")
    present = [t for t in (x_local, rotation, rotate_inv_rescale, attn_alpha, order, row_ptr,
                           dst) if t is not None]
    if not all(t.is_contiguous() for t in present):
        raise ValueError("rotate-back inputs must be contiguous")
    if len({t.device for t in present}) != 1:
        raise ValueError("all rotate-back inputs must share a device")
    if any(t.requires_grad for t in floats):
        raise RuntimeError("rotate_back_aggregate is forward-only (an inference seam)")
    return lmax, heads


def rotate_back_aggregate(x_local, rotation, rotate_inv_rescale, attn_alpha, order, row_ptr,
                          dst, lmax, heads):
    """``out[n, l*l+b, c] = sum_{dst(e)=n} alpha[e, c//dh] * rescale[e] * sum_a
    D_{e,l}[a, b] * x_local[e, l*l+a, c]`` on a B200 -> ``[N, (lmax+1)^2, C]``.

    ``rotation`` packs each edge's block-diagonal rotation per degree (block l
    row-major, ``x_local = D x_global``); ``row_ptr`` is the destination CSR
    prefix sum and ``order`` the slot -> edge permutation when the edges are
    not stored grouped (``None`` otherwise); ``dst`` is the destination of
    each edge (validated for shape only, like the reference's other native
    paths: index values are trusted).
    """
    lmax, heads = _validate(x_local, rotation, rotate_inv_rescale, attn_alpha, order, row_ptr,
                            dst, lmax, heads)
    require_dcu(x_local, rotation, attn_alpha, row_ptr)
    return _extension("rotate_back_aggregate_forward").rotate_back_aggregate_forward(
        x_local, rotation, rotate_inv_rescale, attn_alpha, row_ptr, order, lmax, heads)


__all__ = ["rotate_back_aggregate", "rotation_width"]
