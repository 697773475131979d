"""Fused gated segment softmax + weighted segment sum (inference).

The reference has no single operator for this: it is the composition of
``segment_softmax`` (``python/reference/segment.py:81-136``) with a weighted
``segment_sum`` (``:57-78``), i.e. the attention aggregation of an SO(2)
block.  Here it is one kernel that never writes the weights to memory:

    alpha[e, h]     = gated softmax of logit[:, h] over seg(n)
    out[n, h, s, k] = sum_{e in seg(n)} alpha[e, h] * value[e, s, h*(C/H) + k]
"""
from __future__ import annotations

import torch

from . import segment as _segment
from .native import _extension, require_dcu
from .segment import _validate_order


def _validate(logit, value, offsets, env, null_logit, order):
    for name, tensor in (("logit", logit), ("value", value), ("offsets", offsets)):
        if not isinstance(tensor, torch.Tensor):
            raise TypeError(f"segment attention {name} must be a tensor")
    if logit.dtype != torch.float32:
        raise TypeError("segment attention logit must be float32")
    if value.dtype not in (torch.float32, torch.bfloat16):
        raise TypeError("segment attention value must be float32 or bfloat16")
    if offsets.dtype != torch.int64:
        raise TypeError("segment attention offsets must be int64")
    if logit.ndim != 2:
        raise ValueError("segment attention logit must have shape (n_edges, heads)")
    if value.ndim != 3 or value.shape[0] != logit.shape[0]:
        raise ValueError("segment attention value must have shape (n_edges, components, channels)")
    heads, channels = int(logit.shape[1]), int(value.shape[2])
    if heads <= 0 or heads > 32 or channels % heads:
        raise ValueError("segment attention needs 1..32 heads dividing the channel count")
    if offsets.ndim != 1 or offsets.numel() < 2:
        raise ValueError("segment attention offsets must be a one-dimensional prefix sum")
    n_nodes = int(offsets.numel()) - 1
    if env is not None:
        if not isinstance(env, torch.Tensor) or env.dtype != torch.float32:
            raise TypeError("segment attention env must be a float32 tensor")
        if tuple(env.shape) != (int(logit.shape[0]),):
            raise ValueError("segment attention env must have shape (n_edges,)")
    if null_logit is not None:
        if not isinstance(null_logit, torch.Tensor) or null_logit.dtype != torch.float32:
            raise TypeError("segment attention null_logit must be a float32 tensor")
        if tuple(null_logit.shape) != (n_nodes, heads):
            raise ValueError("segment attention null_logit must have shape (n_nodes, heads)")
    _validate_order(order, int(logit.shape[0]), "segment attention")
    present = [t for t in (logit, value, offsets, env, null_logit, order) if t is not None]
    if not all(t.is_contiguous() for t in present):
        raise ValueError("segment attention inputs must be contiguous")
    if len({t.device for t in present}) != 1:
        raise ValueError("all segment attention inputs must share a device")
    return n_nodes


def segment_attention(logit, value, offsets, env=None, null_logit=None, *, order=None):
    """Attention aggregation ``[N, H, S, C/H]`` over destination segments.

    ``logit`` float32 ``(n_edges, H)``; ``value`` float32 or bfloat16
    ``(n_edges, S, C)`` with ``H | C``; ``offsets`` the destination CSR
    prefix sum; optional ``env`` (edges with ``env <= 0`` carry no mass, the
    others get ``+2 ln env`` on their logit), ``null_logit`` ``(N, H)`` and
    ``order``.  Output float32.  Inference only (no autograd).
    """
    _validate(logit, value, offsets, env, null_logit, order)
    require_dcu(logit, value, offsets, env, null_logit, order)
    if _segment._should_check(None):
        _segment.check_indices(offsets, logit.shape[0], order=order, name="segment attention")
    return _extension("segment_attention_forward").segment_attention_forward(
        logit, value, offsets, env, null_logit, order
    )


__all__ = ["segment_attention"]
