"""Pure-Python loop versions of the operators, for tiny inputs only.

Test infrastructure: these are the "independent loop" checks the reference's
host tests use (``tests/python/test_segment_ops_reference.py:49-61,116-145,
199-212``, ``tests/python/test_gie.py:68-87``) written once as functions, so the
torch and NumPy oracles can be checked against an implementation that shares
no code with them.
"""
from __future__ import annotations

import math


def segment_sum(src, offsets, edge_scale=None, node_scale=None):
    nodes = len(offsets) - 1
    channels = len(src[0]) if src else 0
    out = [[0.0] * channels for _ in range(nodes)]
    for n in range(nodes):
        for e in range(offsets[n], offsets[n + 1]):
            w = 1.0 if edge_scale is None else edge_scale[e]
            for c in range(channels):
                out[n][c] += w * src[e][c]
        if node_scale is not None:
            out[n] = [v * node_scale[n] for v in out[n]]
    return out


def segment_softmax(logit, env, offsets, null_logit=None):
    nodes = len(offsets) - 1
    channels = len(logit[0]) if logit else (len(null_logit[0]) if null_logit else 0)
    alpha = [[0.0] * channels for _ in logit]
    null_alpha = [[0.0] * channels for _ in range(nodes)] if null_logit is not None else None
    for n in range(nodes):
        edges = range(offsets[n], offsets[n + 1])
        for c in range(channels):
            kept = [(e, logit[e][c] + 2.0 * math.log(env[e])) for e in edges if env[e] > 0]
            values = [v for _, v in kept]
            if null_logit is not None:
                values.append(null_logit[n][c])
            if not values:
                continue
            peak = max(values)
            if peak == -math.inf:
                continue
            weights = [(e, math.exp(v - peak)) for e, v in kept]
            w0 = math.exp(null_logit[n][c] - peak) if null_logit is not None else 0.0
            total = w0 + sum(w for _, w in weights)
            for e, w in weights:
                alpha[e][c] = w / total
            if null_alpha is not None:
                null_alpha[n][c] = w0 / total
    return alpha, null_alpha


def force_assembly(grad_edge, edge_vec, src, dst, nodes):
    force = [[0.0] * 3 for _ in range(nodes)]
    virial = [[0.0] * 9 for _ in range(nodes)]
    for e, g in enumerate(grad_edge):
        for r in range(3):
            force[dst[e]][r] += g[r]
            force[src[e]][r] -= g[r]
            for c in range(3):
                virial[src[e]][3 * r + c] -= g[r] * edge_vec[e][c]
    return force, virial


def zonal_scatter(zonal, radial, dst, radial_slot, inv):
    nodes = len(inv)
    rows = len(radial_slot)
    channels = len(radial[0][0]) if radial else 0
    out = [[[0.0] * channels for _ in range(rows + 1)] for _ in range(nodes)]
    for e in range(len(zonal)):
        n = dst[e]
        for r, s in enumerate(radial_slot):
            for c in range(channels):
                out[n][r + 1][c] += zonal[e][r] * radial[e][s][c]
    for n in range(nodes):
        for r in range(rows + 1):
            out[n][r] = [v * inv[n] for v in out[n][r]]
    return out


def rotate_back_aggregate(x_local, rotation, rescale, alpha, dst, nodes, lmax, heads):
    """Loop form of the fused rotate-back aggregation (tiny inputs only)."""
    comps = (lmax + 1) ** 2
    channels = len(x_local[0][0]) if x_local else 0
    dh = channels // heads
    out = [[[0.0] * channels for _ in range(comps)] for _ in range(nodes)]
    for e in range(len(x_local)):
        off = 0
        s = 1.0 if rescale is None else rescale[e]
        for l in range(lmax + 1):
            m = 2 * l + 1
            for b in range(m):
                for c in range(channels):
                    acc = 0.0
                    for a in range(m):
                        acc += rotation[e][off + a * m + b] * x_local[e][l * l + a][c]
                    out[dst[e]][l * l + b][c] += alpha[e][c // dh] * s * acc
            off += m * m
    return out


__all__ = ["force_assembly", "rotate_back_aggregate", "segment_softmax", "segment_sum",
           "zonal_scatter"]
