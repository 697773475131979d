"""float64 NumPy ground truth and exact integer CSR helpers (test infrastructure only).

The fp32 reference oracle sums with ``index_add_`` in edge order; the device
kernels sum in CSR order with split segments combined in partition order, so
neither is a bit baseline for the other at large sizes.  As the reference's
own device tests do (``tests/csrc/accuracy/test_segment_ops_accuracy.py:127-144``),
large-size parity is judged against a float64 evaluation of the same formula.

Integer helpers (exact):
* ``segment_offsets``  <- python/kernels/segment.py:46-57 (bincount + cumsum)
* ``group_by_source``  <- python/kernels/segment.py:60-71 (stable argsort)
"""
from __future__ import annotations

import numpy as np


def segment_offsets(dst: np.ndarray, n_nodes: int) -> np.ndarray:
    dst = np.asarray(dst, dtype=np.int64)
    if dst.size and (dst.min() < 0 or dst.max() >= n_nodes):
        raise ValueError("destination values must be within the node range")
    counts = np.bincount(dst, minlength=n_nodes).astype(np.int64)
    return np.concatenate([np.zeros(1, np.int64), np.cumsum(counts)])


def group_by_source(src: np.ndarray, n_nodes: int) -> tuple[np.ndarray, np.ndarray]:
    src = np.asarray(src, dtype=np.int64)
    return np.argsort(src, kind="stable").astype(np.int64), segment_offsets(src, n_nodes)


def dst_from_offsets(offsets: np.ndarray) -> np.ndarray:
    offsets = np.asarray(offsets, dtype=np.int64)
    return np.repeat(np.arange(offsets.size - 1, dtype=np.int64), np.diff(offsets))


def _rows(n: int, index: np.ndarray, values: np.ndarray) -> np.ndarray:
    out = np.zeros((n,) + values.shape[1:], dtype=np.float64)
    np.add.at(out, index, values)
    return out


def segment_sum(src, dst, n_nodes, edge_scale=None, node_scale=None) -> np.ndarray:
    v = np.asarray(src, dtype=np.float64)
    if edge_scale is not None:
        v = v * np.asarray(edge_scale, dtype=np.float64)[:, None]
    out = _rows(n_nodes, np.asarray(dst), v)
    if node_scale is not None:
        out = out * np.asarray(node_scale, dtype=np.float64).reshape(n_nodes, 1)
    return out


def gated_logit(logit, env) -> np.ndarray:
    logit = np.asarray(logit, dtype=np.float64)
    if env is None:
        return logit
    env = np.asarray(env, dtype=np.float64)
    keep = env > 0
    with np.errstate(divide="ignore", invalid="ignore"):
        shifted = logit + 2.0 * np.log(np.where(keep, env, 1.0))[:, None]
    return np.where(keep[:, None], shifted, -np.inf)


def segment_softmax(logit, env, dst, n_nodes, null_logit=None):
    """(alpha, null_alpha) in float64; all-masked segments give zeros."""
    eff = gated_logit(logit, env)
    dst = np.asarray(dst)
    channels = eff.shape[1]
    peak = np.full((n_nodes, channels), -np.inf)
    np.maximum.at(peak, dst, eff)
    if null_logit is not None:
        peak = np.maximum(peak, np.asarray(null_logit, dtype=np.float64))
    finite = np.isfinite(peak)
    with np.errstate(invalid="ignore", over="ignore"):
        w = np.where(finite[dst], np.exp(eff - np.where(finite, peak, 0.0)[dst]), 0.0)
        w = np.where(np.isfinite(eff), w, 0.0)
    total = _rows(n_nodes, dst, w)
    if null_logit is not None:
        nl = np.asarray(null_logit, dtype=np.float64)
        w0 = np.where(finite, np.exp(nl - np.where(finite, peak, 0.0)), 0.0)
    else:
        w0 = np.zeros_like(total)
    total = total + w0
    safe = np.where(total > 0, total, 1.0)
    return w / safe[dst], (w0 / safe if null_logit is not None else None)


def segment_attention(logit, value, dst, n_nodes, env=None, null_logit=None) -> np.ndarray:
    alpha, _ = segment_softmax(logit, env, dst, n_nodes, null_logit)
    value = np.asarray(value, dtype=np.float64)
    e, s, c = value.shape
    h = alpha.shape[1]
    rows = value.reshape(e, s, h, c // h) * alpha[:, None, :, None]
    out = _rows(n_nodes, np.asarray(dst), rows)
    return np.ascontiguousarray(out.transpose(0, 2, 1, 3))


def force_assembly(grad_edge, edge_vec, src, dst, n_nodes):
    g = np.asarray(grad_edge, dtype=np.float64)
    v = np.asarray(edge_vec, dtype=np.float64)
    force = _rows(n_nodes, np.asarray(dst), g) - _rows(n_nodes, np.asarray(src), g)
    outer = -(g[:, :, None] * v[:, None, :]).reshape(-1, 9)
    return force, _rows(n_nodes, np.asarray(src), outer)


def rmsnorm(x, scale=None, eps=1e-6, per_degree=False) -> tuple[np.ndarray, np.ndarray]:
    """(y, inv_rms) in float64; ``per_degree`` uses weight row floor(sqrt(i))."""
    x = np.asarray(x, dtype=np.float64)
    inv = 1.0 / np.sqrt(np.mean(x * x, axis=-1, keepdims=True) + eps)
    y = x * inv
    if scale is not None:
        w = np.asarray(scale, dtype=np.float64)
        if per_degree:
            comps = x.shape[-2]
            levels = np.floor(np.sqrt(np.arange(comps))).astype(np.int64)
            y = y * w[levels]
        else:
            y = y * w
    return y, inv.reshape(-1)


def zonal_scatter(zonal, radial, dst, radial_slot, inv_sqrt_deg) -> np.ndarray:
    z = np.asarray(zonal, dtype=np.float64)
    r = np.asarray(radial, dtype=np.float64)
    slot = np.asarray(radial_slot, dtype=np.int64)
    inv = np.asarray(inv_sqrt_deg, dtype=np.float64).reshape(-1)
    n = inv.shape[0]
    e, rows = z.shape
    c = r.shape[2]
    out = np.zeros((n, rows + 1, c))
    if e and rows:
        msg = z[:, :, None] * r[:, slot, :]
        np.add.at(out[:, 1:, :], np.asarray(dst), msg)
    return out * inv[:, None, None]


def rotation_block_offsets(lmax: int) -> list[int]:
    """Start of each degree's block in a packed rotation row: sum_{l'<l} (2l'+1)^2."""
    offs, acc = [], 0
    for l in range(lmax + 1):
        offs.append(acc)
        acc += (2 * l + 1) ** 2
    return offs + [acc]


def rotate_back_aggregate(x_local, rotation, rescale, alpha, dst, n_nodes, lmax, heads):
    """float64 truth of the fused rotate-back aggregation.

    ``out[n, l*l + b, c] = sum_{dst(e)=n} alpha[e, c // dh] * rescale[e] *
    sum_a D_{e,l}[a, b] * x_local[e, l*l + a, c]`` with ``D_{e,l}`` the
    degree-l block of edge e's packed rotation (row-major, ``x_local = D
    x_global`` per block, so the rotate-back is the transpose)."""
    x = np.asarray(x_local, dtype=np.float64)
    rot = np.asarray(rotation, dtype=np.float64)
    a = np.asarray(alpha, dtype=np.float64)
    e, comps, channels = x.shape
    dh = channels // heads
    offs = rotation_block_offsets(lmax)
    y = np.zeros_like(x)
    for l in range(lmax + 1):
        m = 2 * l + 1
        blk = rot[:, offs[l]:offs[l + 1]].reshape(e, m, m)
        y[:, l * l:(l + 1) ** 2, :] = np.einsum("eab,eac->ebc", blk, x[:, l * l:(l + 1) ** 2, :])
    w = np.repeat(a, dh, axis=1)[:, None, :]
    if rescale is not None:
        w = w * np.asarray(rescale, dtype=np.float64).reshape(e, 1, 1)
    return _rows(n_nodes, np.asarray(dst), y * w)


def edge_chain(terms, shape, activation=None) -> np.ndarray:
    """float64 truth of the one-pass elementwise chain:
    ``act(sum_t coef_t * a_t * b_t)`` with NumPy broadcasting to ``shape``."""
    out = np.zeros(tuple(shape), dtype=np.float64)
    for term in terms:
        coef, a = term[0], np.asarray(term[1], dtype=np.float64)
        value = coef * np.broadcast_to(a, shape)
        if len(term) == 3:
            value = value * np.broadcast_to(np.asarray(term[2], dtype=np.float64), shape)
        out = out + value
    if activation == "silu":
        return out / (1.0 + np.exp(-out))
    if activation == "sigmoid":
        return 1.0 / (1.0 + np.exp(-out))
    return out


__all__ = [
    "dst_from_offsets",
    "edge_chain",
    "rotate_back_aggregate",
    "rotation_block_offsets",
    "force_assembly",
    "gated_logit",
    "group_by_source",
    "rmsnorm",
    "segment_attention",
    "segment_offsets",
    "segment_softmax",
    "segment_sum",
    "zonal_scatter",
]
