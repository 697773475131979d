"""Destination-segmented operators over a CSR edge list (B200 / sm_100a).

Python face of the reference's ``python/kernels/segment.py``: the same
functions, argument order, keyword defaults, validation (``TypeError`` for a
wrong type or dtype, ``ValueError`` for shape / contiguity / device / range,
both raised before any device work) and autograd behaviour.  Underneath, each
call is one launch sequence of the hand-written kernels in
``bysj_b200/csrc`` through the C ABI of ``libbysj_b200.so``:

``segment_offsets``
    device boundary / histogram kernels, integer-exact (reference
    ``segment.py:46-57``).
``segment_sum``
    merge-path partitioned, 16-byte streaming loads, deterministic
    (``segment.py:283-297``).
``segment_softmax``
    gated softmax with null mass, deterministic (``segment.py:300-311``).
``force_assembly``
    two-sided force / virial walk with fp64 sums (``segment.py:314-332``).

Layout contract (unchanged): ``dst`` is non-decreasing and ``offsets`` is its
exclusive prefix sum, or ``order`` permutes the natural edge order into that
grouping.  The optional full CSR check (``check_grouping=True`` or
``DPA4_CHECK_GROUPING=1``) recomputes the offsets on the device.
"""
from __future__ import annotations

import os

import torch

from .native import _extension, require_dcu

_CHECK_GROUPING = os.environ.get("DPA4_CHECK_GROUPING", "0").strip().lower() in {
    "1",
    "true",
    "yes",
    "on",
}

_FLAG_OUT_OF_RANGE = 1
_FLAG_UNSORTED = 2


def segment_offsets(dst: torch.Tensor, n_nodes: int) -> torch.Tensor:
    """Exclusive prefix sum of the destination group sizes of an edge list.

    Runs on the device: a destination-sorted list takes the one-pass boundary
    kernel, any other order the histogram + scan kernels.  Out-of-range
    destinations raise ``ValueError`` (detected on the device; reading the
    flag back synchronises, as the reference's min/max check does).
    """
    if not isinstance(dst, torch.Tensor):
        raise TypeError("segment offsets require a tensor of destinations")
    if dst.dtype != torch.int64:
        raise TypeError("segment offsets require int64 destinations")
    if int(n_nodes) <= 0:
        raise ValueError("segment offsets require a positive node count")
    if dst.ndim != 1:
        raise ValueError("segment offsets require a one-dimensional dst")
    require_dcu(dst)
    extension = _extension("segment_offsets")
    offsets, flags = extension.segment_offsets(dst.contiguous(), int(n_nodes))
    if flags & _FLAG_OUT_OF_RANGE:
        raise ValueError("destination values must be within the node range")
    return offsets


def destination_csr(dst: torch.Tensor, n_nodes: int) -> tuple[torch.Tensor, torch.Tensor | None]:
    """Destination CSR view ``(offsets, order)`` of an edge list in any order.

    Replaces the seam's ``bincount`` + ``argsort`` (reference
    ``python/model/fused_deepmd.py:111-124``) with device kernels: the
    boundary kernel when ``dst`` is already non-decreasing (``order`` is then
    ``None``: the edges are their own grouping, so the segmented operators
    read them in place), otherwise the histogram for the offsets and the
    stable device grouping for ``order`` (bit-identical to
    ``torch.argsort(dst, stable=True)``).  One flag word is read back, as in
    :func:`segment_offsets`.
    """
    if not isinstance(dst, torch.Tensor):
        raise TypeError("destination CSR requires a tensor of destinations")
    if dst.dtype != torch.int64:
        raise TypeError("destination CSR requires int64 destinations")
    if int(n_nodes) <= 0:
        raise ValueError("destination CSR requires a positive node count")
    if dst.ndim != 1:
        raise ValueError("destination CSR requires a one-dimensional dst")
    require_dcu(dst)
    extension = _extension("segment_offsets")
    dst = dst.contiguous()
    offsets, flags = extension.segment_offsets(dst, int(n_nodes))
    if flags & _FLAG_OUT_OF_RANGE:
        raise ValueError("destination values must be within the node range")
    if not flags & _FLAG_UNSORTED:
        return offsets, None
    order, _, flags = _extension("group_by_key").group_by_key(dst, int(n_nodes))
    if flags & _FLAG_OUT_OF_RANGE:  # pragma: no cover - checked above
        raise ValueError("destination values must be within the node range")
    return offsets, order


def group_by_source(src: torch.Tensor, n_nodes: int) -> tuple[torch.Tensor, torch.Tensor]:
    """Stable ``(order, offsets)`` pair that groups an edge list by source atom."""
    if not isinstance(src, torch.Tensor):
        raise TypeError("group_by_source requires a tensor of sources")
    if src.dtype != torch.int64:
        raise TypeError("group_by_source requires int64 sources")
    if int(n_nodes) <= 0:
        raise ValueError("group_by_source requires a positive node count")
    require_dcu(src)
    extension = _extension("group_by_key")
    order, offsets, flags = extension.group_by_key(src.contiguous(), int(n_nodes))
    if flags & _FLAG_OUT_OF_RANGE:
        raise ValueError("source values must be within the node range")
    return order, offsets


def _validate_order(order, edges, name):
    if order is None:
        return None
    if not isinstance(order, torch.Tensor) or order.dtype != torch.int64:
        raise TypeError(f"{name} order must be an int64 tensor")
    if tuple(order.shape) != (edges,):
        raise ValueError(f"{name} order must have shape (n_edges,)")
    if not order.is_contiguous():
        raise ValueError(f"{name} order must be contiguous")
    return order


def _present(*tensors):
    return [t for t in tensors if t is not None]


def _validate_segment_sum(src, dst, offsets, edge_scale, node_scale, order=None):
    for name, tensor in (("src", src), ("dst", dst), ("offsets", offsets)):
        if not isinstance(tensor, torch.Tensor):
            raise TypeError(f"segment sum {name} must be a tensor")
    if src.dtype not in (torch.float32, torch.bfloat16):
        raise TypeError("segment sum src must be float32 (or bfloat16)")
    if dst.dtype != torch.int64 or offsets.dtype != torch.int64:
        raise TypeError("segment sum dst and offsets must be int64")
    if src.ndim != 2:
        raise ValueError("segment sum src must have shape (n_edges, channels)")
    edges = int(src.shape[0])
    if tuple(dst.shape) != (edges,):
        raise ValueError("segment sum dst must have shape (n_edges,)")
    if offsets.ndim != 1 or offsets.numel() < 2:
        raise ValueError("segment sum offsets must be a one-dimensional prefix sum")
    n_nodes = int(offsets.numel()) - 1
    if edge_scale is not None:
        if not isinstance(edge_scale, torch.Tensor) or edge_scale.dtype != torch.float32:
            raise TypeError("segment sum edge_scale must be a float32 tensor")
        if tuple(edge_scale.shape) != (edges,):
            raise ValueError("segment sum edge_scale must have shape (n_edges,)")
    if node_scale is not None:
        if not isinstance(node_scale, torch.Tensor) or node_scale.dtype != torch.float32:
            raise TypeError("segment sum node_scale must be a float32 tensor")
        if node_scale.numel() != n_nodes:
            raise ValueError("segment sum node_scale must have one value per segment")
    _validate_order(order, edges, "segment sum")
    present = _present(src, dst, offsets, order, edge_scale, node_scale)
    if not all(t.is_contiguous() for t in present):
        raise ValueError("segment sum inputs must be contiguous")
    if len({t.device for t in present}) != 1:
        raise ValueError("all segment sum inputs must share a device")
    return n_nodes


def _validate_segment_softmax(logit, env, offsets, null_logit, order=None):
    for name, tensor in (("logit", logit), ("env", env), ("offsets", offsets)):
        if not isinstance(tensor, torch.Tensor):
            raise TypeError(f"segment softmax {name} must be a tensor")
    if logit.dtype != torch.float32 or env.dtype != torch.float32:
        raise TypeError("segment softmax logit and env must be float32")
    if offsets.dtype != torch.int64:
        raise TypeError("segment softmax offsets must be int64")
    if logit.ndim != 2:
        raise ValueError("segment softmax logit must have shape (n_edges, channels)")
    if tuple(env.shape) != (int(logit.shape[0]),):
        raise ValueError("segment softmax env must have shape (n_edges,)")
    if offsets.ndim != 1 or offsets.numel() < 2:
        raise ValueError("segment softmax offsets must be a one-dimensional prefix sum")
    n_nodes, channels = int(offsets.numel()) - 1, int(logit.shape[1])
    if null_logit is not None:
        if not isinstance(null_logit, torch.Tensor) or null_logit.dtype != torch.float32:
            raise TypeError("segment softmax null_logit must be a float32 tensor")
        if tuple(null_logit.shape) != (n_nodes, channels):
            raise ValueError("segment softmax null_logit must have shape (n_nodes, channels)")
    _validate_order(order, int(logit.shape[0]), "segment softmax")
    present = _present(logit, env, offsets, order, null_logit)
    if not all(t.is_contiguous() for t in present):
        raise ValueError("segment softmax inputs must be contiguous")
    if len({t.device for t in present}) != 1:
        raise ValueError("all segment softmax inputs must share a device")
    return n_nodes, channels


def _validate_force_assembly(grad_edge, edge_vec, dst_offsets, src_offsets, src_order):
    named = (
        ("grad_edge", grad_edge),
        ("edge_vec", edge_vec),
        ("dst_offsets", dst_offsets),
        ("src_offsets", src_offsets),
        ("src_order", src_order),
    )
    for name, tensor in named:
        if not isinstance(tensor, torch.Tensor):
            raise TypeError(f"force assembly {name} must be a tensor")
    if grad_edge.dtype != torch.float32 or edge_vec.dtype != torch.float32:
        raise TypeError("force assembly grad_edge and edge_vec must be float32")
    if grad_edge.dim() != 2 or grad_edge.shape[1] != 3:
        raise ValueError("force assembly grad_edge must have shape (n_edges, 3)")
    if edge_vec.shape != grad_edge.shape:
        raise ValueError("force assembly edge_vec must match grad_edge")
    for name, tensor in (("dst_offsets", dst_offsets), ("src_offsets", src_offsets)):
        if tensor.dtype != torch.int64 or tensor.ndim != 1 or tensor.numel() < 2:
            raise ValueError(f"force assembly {name} must be an int64 prefix sum")
    if dst_offsets.numel() != src_offsets.numel():
        raise ValueError("force assembly offsets must describe the same atom count")
    if src_order.dtype != torch.int64 or tuple(src_order.shape) != (int(grad_edge.shape[0]),):
        raise ValueError("force assembly src_order must be int64 with shape (n_edges,)")
    present = [grad_edge, edge_vec, dst_offsets, src_offsets, src_order]
    if not all(t.is_contiguous() for t in present):
        raise ValueError("force assembly inputs must be contiguous")
    if len({t.device for t in present}) != 1:
        raise ValueError("all force assembly inputs must share a device")
    return int(dst_offsets.numel()) - 1


def _should_check(explicit):
    """Grouping validation is opt-in: it costs a pass over the edge list."""
    return _CHECK_GROUPING if explicit is None else bool(explicit)


_INDEX_MESSAGES = (
    (1, "offsets must be an exclusive prefix sum from 0 to n_edges"),
    (2, "order must be a permutation of the edge indices"),
    (4, "index values must be within range"),
)


def check_indices(offsets=None, n_edges=0, *, order=None, values=None, value_limit=0,
                  name="segment operator") -> None:
    """Device index guard: raises ``ValueError`` naming every violated invariant.

    The kernels trust their indices; this checks what they trust -- offsets a
    CSR prefix sum ending at ``n_edges``, ``order`` a permutation of the edges,
    ``values`` inside ``[0, value_limit)`` -- in one device pass and one flag
    read back.  Run by the operators when grouping validation is asked for
    (``check_grouping=True`` or ``DPA4_CHECK_GROUPING=1``).
    """
    word = _extension("check_indices").check_indices(offsets, int(n_edges), order, values,
                                                     int(value_limit))
    if word:
        broken = "; ".join(text for bit, text in _INDEX_MESSAGES if word & bit)
        raise ValueError(f"{name}: {broken}")


def _check_csr(dst: torch.Tensor, offsets: torch.Tensor, n_nodes: int, name: str) -> None:
    expected = segment_offsets(dst, n_nodes)
    if not torch.equal(expected, offsets):
        raise ValueError(
            f"{name} requires the natural edge order grouped by destination; "
            "offsets must be the exclusive prefix sum of the dst group sizes"
        )


class _SegmentSumFunction(torch.autograd.Function):
    @staticmethod
    def forward(ctx, src, dst, offsets, edge_scale, node_scale, order):
        out = _extension("segment_sum_forward").segment_sum_forward(
            src, offsets, edge_scale, node_scale, order
        )
        ctx.save_for_backward(src, dst, offsets, edge_scale, node_scale, order)
        ctx.needs_node_scale_grad = node_scale is not None and node_scale.requires_grad
        ctx.src_dtype = src.dtype
        return out

    @staticmethod
    def backward(ctx, grad_output):
        src, dst, offsets, edge_scale, node_scale, order = ctx.saved_tensors
        grad_src, grad_node_scale = _extension("segment_sum_backward").segment_sum_backward(
            grad_output.contiguous(),
            src,
            dst,
            offsets,
            edge_scale,
            node_scale,
            ctx.needs_node_scale_grad,
            order,
        )
        if ctx.src_dtype != grad_src.dtype:
            grad_src = grad_src.to(ctx.src_dtype)
        scale_grad = grad_node_scale.reshape(node_scale.shape) if ctx.needs_node_scale_grad else None
        return grad_src, None, None, None, scale_grad, None


class _SegmentSoftmaxFunction(torch.autograd.Function):
    @staticmethod
    def forward(ctx, logit, env, offsets, order):
        alpha, _ = _extension("segment_softmax_forward").segment_softmax_forward(
            logit, env, offsets, None, order
        )
        ctx.save_for_backward(alpha, env, offsets, order)
        return alpha

    @staticmethod
    def backward(ctx, grad_alpha):
        alpha, env, offsets, order = ctx.saved_tensors
        grad_logit, _, grad_env = _extension("segment_softmax_backward").segment_softmax_backward(
            alpha, grad_alpha.contiguous(), env, offsets, None, None, order
        )
        return grad_logit, grad_env, None, None


class _SegmentSoftmaxNullFunction(torch.autograd.Function):
    @staticmethod
    def forward(ctx, logit, env, offsets, null_logit, order):
        alpha, null_alpha = _extension("segment_softmax_forward").segment_softmax_forward(
            logit, env, offsets, null_logit, order
        )
        ctx.save_for_backward(alpha, null_alpha, env, offsets, order)
        return alpha, null_alpha

    @staticmethod
    def backward(ctx, grad_alpha, grad_null_alpha):
        alpha, null_alpha, env, offsets, order = ctx.saved_tensors
        grad_alpha = torch.zeros_like(alpha) if grad_alpha is None else grad_alpha.contiguous()
        grad_null_alpha = (
            torch.zeros_like(null_alpha) if grad_null_alpha is None else grad_null_alpha.contiguous()
        )
        grad_logit, grad_null_logit, grad_env = _extension(
            "segment_softmax_backward"
        ).segment_softmax_backward(
            alpha, grad_alpha, env, offsets, null_alpha, grad_null_alpha, order
        )
        return grad_logit, grad_env, None, grad_null_logit, None


def segment_sum(src, dst, offsets, edge_scale=None, node_scale=None, *, order=None,
                check_grouping=None):
    """``out[n] = node_scale[n] * sum_{dst(e)=n} edge_scale[e] * src[e]``.

    ``src`` is contiguous float32 (or bfloat16, read as is and summed in
    fp32) ``(n_edges, channels)``; ``dst`` int64 ``(n_edges,)``
    non-decreasing, ``offsets`` its exclusive prefix sum.  The output is
    float32.  Gradients are defined for ``src`` and ``node_scale``, never for
    the indices; ``edge_scale`` has none (as in the reference).
    """
    n_nodes = _validate_segment_sum(src, dst, offsets, edge_scale, node_scale, order)
    require_dcu(src, dst, offsets, edge_scale, node_scale, order)
    if _should_check(check_grouping):
        check_indices(offsets, src.shape[0], order=order, name="segment sum")
        if order is None:
            _check_csr(dst, offsets, n_nodes, "segment sum")
    return _SegmentSumFunction.apply(src, dst, offsets, edge_scale, node_scale, order)


def segment_softmax(logit, env, offsets, null_logit=None, *, order=None, check_grouping=None):
    """Gated destination-segmented softmax over the incoming edges.

    Returns ``alpha`` ``(n_edges, channels)``; with ``null_logit`` also the
    per-channel null mass ``(n_nodes, channels)``.  Edges with a non-positive
    envelope carry no mass.  With ``check_grouping`` (or
    ``DPA4_CHECK_GROUPING=1``) the offsets and ``order`` are checked on the
    device first (the softmax receives no ``dst`` to compare the grouping to).
    """
    _validate_segment_softmax(logit, env, offsets, null_logit, order)
    require_dcu(logit, env, offsets, null_logit, order)
    if _should_check(check_grouping):
        check_indices(offsets, logit.shape[0], order=order, name="segment softmax")
    if null_logit is None:
        return _SegmentSoftmaxFunction.apply(logit, env, offsets, order)
    return _SegmentSoftmaxNullFunction.apply(logit, env, offsets, null_logit, order)


def force_assembly(grad_edge, edge_vec, src, dst, dst_offsets, src_offsets=None, src_order=None):
    """Assemble ``(force, virial)`` from per-edge energy gradients.

    ``F_k = sum_{dst=k} g - sum_{src=k} g`` and ``W_k = -sum_{src=k} g (x) v``
    with fp64 accumulation.  ``src_order`` / ``src_offsets`` group the edges
    by source atom; when omitted they are derived from ``src`` (one stable
    sort -- cache them when this runs per step).  Inference only: no autograd.
    """
    n_nodes = int(dst_offsets.numel()) - 1
    if src_order is None or src_offsets is None:
        order, offsets = group_by_source(src, n_nodes)
        src_order = order if src_order is None else src_order
        src_offsets = offsets if src_offsets is None else src_offsets
    _validate_force_assembly(grad_edge, edge_vec, dst_offsets, src_offsets, src_order)
    require_dcu(grad_edge, edge_vec, dst_offsets, src_offsets, src_order)
    if _CHECK_GROUPING:
        check_indices(dst_offsets, grad_edge.shape[0], name="force assembly destination")
        check_indices(src_offsets, grad_edge.shape[0], order=src_order,
                      name="force assembly source")
    return _extension("force_assembly").force_assembly(
        grad_edge, edge_vec, dst_offsets, src_offsets, src_order
    )


def segment_available() -> bool:
    """Whether this process can run all the segmented entry points."""
    required = (
        "segment_sum_forward",
        "segment_sum_backward",
        "segment_softmax_forward",
        "segment_softmax_backward",
        "force_assembly",
    )
    try:
        require_dcu()
        extension = _extension("segment_sum_forward")
    except (ImportError, OSError, RuntimeError):
        return False
    return all(hasattr(extension, name) for name in required)


__all__ = [
    "force_assembly",
    "group_by_source",
    "segment_available",
    "segment_offsets",
    "segment_softmax",
    "segment_sum",
]
