"""PyTorch segmented operators for explicit testing and comparison.

The ``reference.*`` functions of lipengfei1409/bysj
``python/reference/segment.py`` -- the executable specification its kernels
are checked against -- with the same ATen operation sequence (zero-init +
``index_add_`` over ``dst``, per-segment ``amax``):

* ``segment_sum_reference``      <- segment.py:57-78
* ``segment_softmax_reference``  <- segment.py:81-136
* ``force_assembly_reference``   <- segment.py:139-160
* ``segment_attention_reference`` -- the composition softmax -> weighted sum
  (segment.py:81-136 then :57-78), which the reference only has as two calls.

Plain PyTorch on any device; the CUDA kernels never call it.
"""
from __future__ import annotations

import torch


def _n_segments(offsets: torch.Tensor) -> int:
    if offsets.dim() != 1 or offsets.numel() < 2:
        raise ValueError("offsets must be a one-dimensional prefix sum of at least two entries")
    return int(offsets.numel()) - 1


def _grouping(dst: torch.Tensor, offsets: torch.Tensor, n_edges: int, name: str) -> int:
    """Type, shape, range and CSR-consistency checks (segment.py:32-54)."""
    if dst.dtype != torch.int64:
        raise TypeError(f"{name} dst must be int64")
    if dst.ndim != 1 or dst.shape[0] != n_edges:
        raise ValueError(f"{name} dst must have shape (n_edges,)")
    if offsets.dtype != torch.int64:
        raise TypeError(f"{name} offsets must be int64")
    nodes = _n_segments(offsets)
    if dst.numel() and (int(dst.min()) < 0 or int(dst.max()) >= nodes):
        raise ValueError(f"{name} dst values must be within the node range")
    sizes = torch.bincount(dst, minlength=nodes) if dst.numel() else dst.new_zeros(nodes)
    prefix = torch.zeros(nodes + 1, dtype=torch.int64)
    prefix[1:] = torch.cumsum(sizes, 0)
    if not torch.equal(prefix, offsets.cpu()):
        raise ValueError("offsets must be the exclusive prefix sum of the dst group sizes")
    return nodes


def _accumulate(rows: int, index: torch.Tensor, values: torch.Tensor) -> torch.Tensor:
    """Zero-initialised destination rows plus ``index_add_`` of ``values``."""
    out = values.new_zeros((rows,) + tuple(values.shape[1:]))
    if values.shape[0]:
        out.index_add_(0, index, values)
    return out


def segment_sum_reference(src, dst, offsets, edge_scale=None, node_scale=None):
    """``out[n] = node_scale[n] * sum_{dst(e)=n} edge_scale[e] * src[e]``."""
    if src.dtype != torch.float32:
        raise TypeError("segment sum src must be float32")
    if src.ndim != 2:
        raise ValueError("segment sum src must have shape (n_edges, channels)")
    nodes = _n_segments(offsets)
    _grouping(dst, offsets, src.shape[0], "segment sum")
    if edge_scale is not None and (
        edge_scale.dtype != torch.float32 or tuple(edge_scale.shape) != (src.shape[0],)
    ):
        raise ValueError("segment sum edge_scale must be float32 with shape (n_edges,)")
    if node_scale is not None and (
        node_scale.dtype != torch.float32 or node_scale.numel() != nodes
    ):
        raise ValueError("segment sum node_scale must be float32 with one value per segment")
    terms = src if edge_scale is None else src * edge_scale.reshape(-1, 1)
    out = _accumulate(nodes, dst, terms)
    return out if node_scale is None else out * node_scale.reshape(nodes, 1)


def _gated(logit: torch.Tensor, env: torch.Tensor) -> torch.Tensor:
    """``logit + 2 ln env`` where ``env > 0``, ``-inf`` elsewhere."""
    keep = (env > 0).reshape(-1, 1)
    shifted = logit + 2.0 * torch.log(env.clamp_min(1e-30)).reshape(-1, 1)
    return torch.where(keep, shifted, torch.full_like(logit, float("-inf")))


def segment_softmax_reference(logit, env, dst, offsets, null_logit=None):
    """Per-segment, per-channel gated softmax with an optional null mass.

    Returns ``(alpha, null_alpha)``; ``null_alpha`` is ``None`` without a
    null logit.  A segment whose maximum is ``-inf`` gets zero weights.
    """
    if logit.dtype != torch.float32 or env.dtype != torch.float32:
        raise TypeError("segment softmax logit and env must be float32")
    if logit.ndim != 2 or tuple(env.shape) != (logit.shape[0],):
        raise ValueError("segment softmax expects logit (n_edges, channels) and env (n_edges,)")
    n_edges, channels = logit.shape
    nodes = _n_segments(offsets)
    _grouping(dst, offsets, n_edges, "segment softmax")
    if null_logit is not None and (
        null_logit.dtype != torch.float32 or tuple(null_logit.shape) != (nodes, channels)
    ):
        raise ValueError("segment softmax null_logit must be float32 (n_nodes, channels)")

    eff = _gated(logit, env)
    peak = torch.full((nodes, channels), float("-inf"), dtype=logit.dtype)
    if n_edges:
        index = dst.reshape(-1, 1).expand(n_edges, channels).contiguous()
        peak.scatter_reduce_(0, index, eff, reduce="amax", include_self=True)
    if null_logit is not None:
        peak = torch.maximum(peak, null_logit)
    finite = peak > float("-inf")
    if n_edges:
        weights = torch.where(
            finite.index_select(0, dst), torch.exp(eff - peak.index_select(0, dst)),
            torch.zeros_like(eff),
        )
    else:
        weights = eff
    total = _accumulate(nodes, dst, weights) if n_edges else logit.new_zeros((nodes, channels))
    if null_logit is not None:
        null_weight = torch.where(finite, torch.exp(null_logit - peak), torch.zeros_like(peak))
    else:
        null_weight = torch.zeros_like(total)
    total = total + null_weight
    safe = torch.where(total > 0, total, torch.ones_like(total))
    alpha = weights / safe.index_select(0, dst) if n_edges else weights
    return alpha, (null_weight / safe if null_logit is not None else None)


def segment_attention_reference(logit, value, dst, offsets, env=None, null_logit=None):
    """``out[n, h, s, k] = sum_{dst(e)=n} alpha[e, h] * value[e, s, h*dh + k]``.

    ``alpha`` from :func:`segment_softmax_reference` (``env`` defaults to
    ones, i.e. no gating); the weighted rows are summed with ``index_add_``.
    ``value`` may be bfloat16: it is widened to float32 first.
    """
    n_edges, heads = logit.shape
    _, comps, channels = value.shape
    dh = channels // heads
    if env is None:
        env = torch.ones(n_edges, dtype=torch.float32)
    alpha, _ = segment_softmax_reference(logit, env, dst, offsets, null_logit)
    rows = value.to(torch.float32).reshape(n_edges, comps, heads, dh)
    weighted = rows * alpha.reshape(n_edges, 1, heads, 1)
    out = _accumulate(_n_segments(offsets), dst, weighted)
    return out.permute(0, 2, 1, 3).contiguous()


def force_assembly_reference(grad_edge, edge_vec, src, dst, dst_offsets, src_offsets):
    """``F_k = sum_{dst=k} g_e - sum_{src=k} g_e`` and ``W_k = sum_{src=k} -g_e (x) v_e``."""
    if grad_edge.dtype != torch.float32 or grad_edge.ndim != 2 or grad_edge.shape[1] != 3:
        raise ValueError("force assembly grad_edge must be float32 (n_edges, 3)")
    if edge_vec.shape != grad_edge.shape:
        raise ValueError("force assembly edge_vec must match grad_edge")
    n_edges = grad_edge.shape[0]
    nodes = _n_segments(dst_offsets)
    _grouping(dst, dst_offsets, n_edges, "force assembly destination")
    _grouping(src, src_offsets, n_edges, "force assembly source")
    if _n_segments(src_offsets) != nodes:
        raise ValueError("force assembly offsets must describe the same atom count")
    force = _accumulate(nodes, dst, grad_edge)
    if n_edges:
        force.index_add_(0, src, -grad_edge)
    outer = -(grad_edge.unsqueeze(2) * edge_vec.unsqueeze(1)).reshape(n_edges, 9)
    virial = _accumulate(nodes, src, outer)
    return force, virial


def _rotation_offsets(lmax: int) -> list[int]:
    offs, acc = [], 0
    for l in range(lmax + 1):
        offs.append(acc)
        acc += (2 * l + 1) ** 2
    return offs + [acc]


def rotate_back_aggregate_reference(x_local, rotation, rotate_inv_rescale, attn_alpha, order,
                                    row_ptr, dst, lmax, heads):
    """Rotate-back + attention weighting + destination sum (the flash seam).

    The argument list is the one the reference records for DeepMD's
    ``SO2Convolution._flash_atten_fn`` (``docs/deepmd-fused-dispatch.md:127``):
    ``x_local`` [E, (lmax+1)^2, C] edge messages in each edge's local frame,
    ``rotation`` [E, sum_l (2l+1)^2] the block-diagonal rotation packed per
    degree (block l row-major, ``x_local = D x_global``), ``rotate_inv_rescale``
    [E] or None a per-edge factor applied with the inverse rotation,
    ``attn_alpha`` [E, heads] the attention weights, ``order`` / ``row_ptr``
    the destination CSR view (``order`` may be None), ``dst`` [E]:

    ``out[n, l*l + b, c] = sum_{dst(e)=n} alpha[e, c // dh] * rescale[e] *
    sum_a D_{e,l}[a, b] * x_local[e, l*l + a, c]``, ``dh = C / heads``.
    """
    if x_local.dtype != torch.float32 or x_local.ndim != 3:
        raise ValueError("rotate-back x_local must be float32 (n_edges, (lmax+1)^2, channels)")
    n_edges, comps, channels = x_local.shape
    if comps != (lmax + 1) ** 2:
        raise ValueError("rotate-back x_local must have (lmax+1)^2 components")
    offs = _rotation_offsets(lmax)
    if rotation.dtype != torch.float32 or tuple(rotation.shape) != (n_edges, offs[-1]):
        raise ValueError("rotate-back rotation must be float32 (n_edges, sum_l (2l+1)^2)")
    if heads <= 0 or channels % heads:
        raise ValueError("rotate-back heads must divide the channels")
    if attn_alpha.dtype != torch.float32 or tuple(attn_alpha.shape) != (n_edges, heads):
        raise ValueError("rotate-back attn_alpha must be float32 (n_edges, heads)")
    nodes = _n_segments(row_ptr)
    _grouping(dst, row_ptr, n_edges, "rotate-back")
    y = torch.empty_like(x_local)
    for l in range(lmax + 1):
        m = 2 * l + 1
        blk = rotation[:, offs[l]:offs[l + 1]].reshape(n_edges, m, m)
        y[:, l * l:(l + 1) ** 2, :] = torch.bmm(blk.transpose(1, 2), x_local[:, l * l:(l + 1) ** 2, :])
    weight = attn_alpha.repeat_interleave(channels // heads, dim=1).unsqueeze(1)
    if rotate_inv_rescale is not None:
        weight = weight * rotate_inv_rescale.reshape(n_edges, 1, 1)
    return _accumulate(nodes, dst, y * weight)


__all__ = [
    "force_assembly_reference",
    "rotate_back_aggregate_reference",
    "segment_attention_reference",
    "segment_softmax_reference",
    "segment_sum_reference",
]
