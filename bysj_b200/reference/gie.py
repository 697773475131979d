"""PyTorch GIE zonal scatter for explicit testing and comparison.

Part of the ``reference.*`` API of lipengfei1409/bysj
(``python/reference/gie.py:7-67``, same names, signatures and messages):
the radial row of each zonal row's slot is gathered, weighted by the zonal
coefficient, summed into ``out[:, 1:, :]`` with ``index_add_`` over ``dst``
(any order) and only then scaled by the inverse degree; row zero stays zero.
Plain PyTorch on any device; the CUDA kernels never call it.
"""
from __future__ import annotations

import torch


def _check(zonal, radial, dst, radial_slot, inv_sqrt_deg):
    named = (zonal, radial, dst, radial_slot, inv_sqrt_deg)
    if not isinstance(zonal, torch.Tensor) or not isinstance(radial, torch.Tensor):
        raise TypeError("GIE zonal and radial inputs must be tensors")
    if not isinstance(dst, torch.Tensor) or not isinstance(radial_slot, torch.Tensor):
        raise TypeError("GIE dst and radial_slot must be tensors")
    if not isinstance(inv_sqrt_deg, torch.Tensor):
        raise TypeError("GIE inv_sqrt_deg must be a tensor")
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
    if not all(t.is_contiguous() for t in named):
        raise ValueError("GIE inputs must be contiguous")
    if len({t.device for t in named}) != 1:
        raise ValueError("all GIE inputs must share a device")
    if n_rows and radial.shape[1] == 0:
        raise ValueError("GIE radial must contain slots when zonal rows are present")
    if n_edges and inv_sqrt_deg.shape[0] == 0:
        raise ValueError("GIE degree normalization must contain destination nodes")


def zonal_scatter_reference(zonal, radial, dst, radial_slot, inv_sqrt_deg):
    """``out[n, r+1, c] = inv[n] * sum_{dst[e]=n} zonal[e,r] * radial[e, slot[r], c]``."""
    _check(zonal, radial, dst, radial_slot, inv_sqrt_deg)
    inverse = inv_sqrt_deg.reshape(-1)
    n_edges, n_rows = zonal.shape
    nodes, channels = inverse.shape[0], radial.shape[2]
    if n_edges and (bool((dst < 0).any()) or bool((dst >= nodes).any())):
        raise ValueError("GIE dst values must be within the node range")
    if n_rows and (bool((radial_slot < 0).any()) or bool((radial_slot >= radial.shape[1]).any())):
        raise ValueError("GIE radial_slot values must be within the radial range")
    out = radial.new_zeros((nodes, n_rows + 1, channels))
    if n_edges and n_rows and channels:
        picked = radial.gather(1, radial_slot.reshape(1, n_rows, 1).expand(n_edges, n_rows, channels))
        out[:, 1:, :].index_add_(0, dst, zonal.unsqueeze(-1) * picked)
    return out * inverse.reshape(nodes, 1, 1)


gie_zonal_scatter_reference = zonal_scatter_reference

__all__ = ["gie_zonal_scatter_reference", "zonal_scatter_reference"]
