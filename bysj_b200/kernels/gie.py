"""GIE zonal scatter on B200.

Python face of the reference's ``python/kernels/gie.py`` (validation and
autograd contract, lines 11-93).  ``dst`` may be in any order: the extension
derives the destination CSR view on the device (boundary kernel for sorted
input, histogram + stable sort otherwise) and then runs the atomic-free
segmented kernel, which normalises after the destination sum.
"""
from __future__ import annotations

import torch

from . import segment as _segment
from .native import _extension, require_dcu


def _validate(zonal, radial, dst, radial_slot, inv_sqrt_deg):
    named = (
        ("zonal", zonal),
        ("radial", radial),
        ("dst", dst),
        ("radial_slot", radial_slot),
        ("inv_sqrt_deg", inv_sqrt_deg),
    )
    for name, tensor in named:
        if not isinstance(tensor, torch.Tensor):
            raise TypeError(f"GIE {name} must be a tensor")
    if any(t.dtype != torch.float32 for t in (zonal, radial, inv_sqrt_deg)):
        raise TypeError("GIE value tensors must be float32")
    if dst.dtype != torch.int64 or radial_slot.dtype != torch.int64:
        raise TypeError("GIE dst and radial_slot must be int64")
    if zonal.ndim != 2:
        raise ValueError("GIE zonal must have shape (n_edges, n_rows)")
    if radial.ndim != 3 or radial.shape[0] != zonal.shape[0]:
        raise ValueError("GIE radial must have shape (n_edges, n_radial, channels)")
    n_edges, n_rows = zonal.shape
    if tuple(dst.shape) != (n_edges,):
        raise ValueError("GIE dst must have shape (n_edges,)")
    if tuple(radial_slot.shape) != (n_rows,):
        raise ValueError("GIE radial_slot must have shape (n_rows,)")
    if inv_sqrt_deg.ndim not in (1, 3) or (
        inv_sqrt_deg.ndim == 3 and tuple(inv_sqrt_deg.shape[1:]) != (1, 1)
    ):
        raise ValueError("GIE inv_sqrt_deg must have shape (n_nodes,) or (n_nodes, 1, 1)")
    if n_rows and radial.shape[1] == 0:
        raise ValueError("GIE radial must contain slots when zonal rows are present")
    if n_edges and inv_sqrt_deg.shape[0] == 0:
        raise ValueError("GIE degree normalization must contain destination nodes")
    tensors = (zonal, radial, dst, radial_slot, inv_sqrt_deg)
    if not all(t.is_contiguous() for t in tensors):
        raise ValueError("GIE inputs must be contiguous")
    if len({t.device for t in tensors}) != 1:
        raise ValueError("all GIE inputs must share a device")


class _GIEZonalScatterFunction(torch.autograd.Function):
    @staticmethod
    def forward(ctx, zonal, radial, dst, radial_slot, inv_sqrt_deg, dst_offsets):
        output = _extension("gie_zonal_scatter_forward").gie_zonal_scatter_forward(
            zonal, radial, dst, radial_slot, inv_sqrt_deg, dst_offsets
        )
        ctx.save_for_backward(zonal, radial, dst, radial_slot, inv_sqrt_deg, dst_offsets)
        return output

    @staticmethod
    def backward(ctx, grad_output):
        zonal, radial, dst, radial_slot, inv_sqrt_deg, dst_offsets = ctx.saved_tensors
        grad_zonal, grad_radial, grad_inv = _extension(
            "gie_zonal_scatter_backward"
        ).gie_zonal_scatter_backward(
            grad_output.contiguous(), zonal, radial, dst, radial_slot, inv_sqrt_deg, dst_offsets
        )
        needs = ctx.needs_input_grad
        return (
            grad_zonal if needs[0] else None,
            grad_radial if needs[1] else None,
            None,
            None,
            grad_inv if needs[4] else None,
            None,
        )


def _validate_dst_offsets(dst_offsets, dst, n_nodes):
    if not isinstance(dst_offsets, torch.Tensor):
        raise TypeError("GIE dst_offsets must be a tensor")
    if dst_offsets.dtype != torch.int64:
        raise TypeError("GIE dst_offsets must be int64")
    if tuple(dst_offsets.shape) != (n_nodes + 1,):
        raise ValueError("GIE dst_offsets must have shape (n_nodes + 1,)")
    if not dst_offsets.is_contiguous():
        raise ValueError("GIE inputs must be contiguous")
    if dst_offsets.device != dst.device:
        raise ValueError("all GIE inputs must share a device")


def zonal_scatter(zonal, radial, dst, radial_slot, inv_sqrt_deg, *, dst_offsets=None):
    """DPA4 geometric-initial-embedding zonal scatter on a B200.

    ``out[n, r+1, c] = inv[n] * sum_{dst[e]=n} zonal[e, r] * radial[e,
    radial_slot[r], c]``; row zero is reserved (zero).  Value tensors are
    contiguous float32, indices contiguous int64 and in range.  Gradients are
    defined for zonal, radial and the inverse degree, not for the indices.

    ``dst_offsets`` (an addition to the reference signature): when ``dst`` is
    already grouped (non-decreasing) and its CSR is at hand -- ``[n_nodes +
    1]`` int64, ``dst_offsets[n]`` = the number of edges with ``dst < n``, as
    ``segment_offsets(dst, n_nodes)`` returns -- pass it, and the operator
    uses it as given instead of deriving the CSR on the device and reading
    its flags back (no host wait; the same kernels and bits).  It is trusted
    like the other indices; with grouping checks on, it is compared with the
    CSR of ``dst``.
    """
    _validate(zonal, radial, dst, radial_slot, inv_sqrt_deg)
    if dst_offsets is not None:
        _validate_dst_offsets(dst_offsets, dst, inv_sqrt_deg.shape[0])
    require_dcu(zonal, radial, dst, radial_slot, inv_sqrt_deg)
    if _segment._should_check(None):
        _segment.check_indices(values=radial_slot, value_limit=radial.shape[1],
                               name="GIE radial_slot")
        _segment.check_indices(values=dst, value_limit=inv_sqrt_deg.shape[0], name="GIE dst")
        if dst_offsets is not None:
            _segment.check_indices(dst_offsets, dst.shape[0], name="GIE dst_offsets")
            derived, flags = _extension("segment_offsets").segment_offsets(
                dst, inv_sqrt_deg.shape[0])
            if flags & _segment._FLAG_UNSORTED or not torch.equal(derived, dst_offsets):
                raise ValueError("GIE dst_offsets: not the CSR of a grouped dst")
    return _GIEZonalScatterFunction.apply(zonal, radial, dst, radial_slot, inv_sqrt_deg,
                                          dst_offsets)


def gie_zonal_scatter(zonal, radial, dst, radial_slot, inv_sqrt_deg, *, dst_offsets=None):
    """Alias naming the DPA4 stage this primitive belongs to."""
    return zonal_scatter(zonal, radial, dst, radial_slot, inv_sqrt_deg,
                         dst_offsets=dst_offsets)


def gie_available() -> bool:
    """Whether this process can run both GIE entry points."""
    try:
        require_dcu()
        extension = _extension("gie_zonal_scatter_forward")
        return hasattr(extension, "gie_zonal_scatter_backward")
    except (ImportError, OSError, RuntimeError):
        return False


__all__ = ["gie_available", "gie_zonal_scatter", "zonal_scatter"]
