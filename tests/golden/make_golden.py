"""Generate golden input/output fixtures by running the reference's own code.

Run once, in a container where the reference project is mounted::

    python tests/golden/make_golden.py /path/to/lipengfei1409-bysj

It imports the reference's pure-PyTorch ``reference`` package and its
``kernels.segment.segment_offsets`` / ``group_by_source`` (both run on the
CPU), evaluates them on small seeded inputs, and writes ``*.npz`` files next
to this script.  Nothing at test time reads the reference tree: the tests only
load these fixtures.  Autograd gradients of the reference functions are stored
too, so the closed-form backward kernels have a pinned target.
"""
from __future__ import annotations

import sys
from pathlib import Path

import numpy as np
import torch

HERE = Path(__file__).resolve().parent


def _graph(sizes):
    dst = torch.repeat_interleave(torch.arange(len(sizes)), torch.tensor(sizes))
    offsets = torch.zeros(len(sizes) + 1, dtype=torch.int64)
    offsets[1:] = torch.cumsum(torch.tensor(sizes), 0)
    return dst.long(), offsets


def _np(t):
    return None if t is None else t.detach().cpu().numpy()


def main(reference_root: str) -> None:
    sys.path.insert(0, str(Path(reference_root) / "python"))
    from kernels.segment import group_by_source, segment_offsets  # reference code
    from reference.gie import zonal_scatter_reference
    from reference.rmsnorm import rmsnorm
    from reference.segment import (
        force_assembly_reference,
        segment_softmax_reference,
        segment_sum_reference,
    )

    gen = torch.Generator().manual_seed(20261201)

    # --- CSR helpers --------------------------------------------------------
    sizes = torch.randint(0, 9, (50,), generator=gen).tolist()
    sizes[3] = 0
    sizes[17] = 40  # one heavy segment
    dst, _ = _graph(sizes)
    src = torch.randint(0, 50, (dst.numel(),), generator=gen)
    order, src_off = group_by_source(src, 50)
    np.savez_compressed(
        HERE / "csr.npz",
        dst=_np(dst), offsets=_np(segment_offsets(dst, 50)),
        src=_np(src), src_order=_np(order), src_offsets=_np(src_off),
    )

    # --- segment_sum (+ autograd gradients) ---------------------------------
    sizes = [3, 0, 5, 1, 12, 0, 7, 2, 30, 4]
    dst, offsets = _graph(sizes)
    e = dst.numel()
    srcv = torch.randn(e, 24, generator=gen).requires_grad_(True)
    escale = (torch.rand(e, generator=gen) + 0.5)
    nscale = (torch.rand(len(sizes), generator=gen) + 0.5).requires_grad_(True)
    out = segment_sum_reference(srcv, dst, offsets, escale, nscale)
    up = torch.randn(out.shape, generator=gen)
    g_src, g_ns = torch.autograd.grad(out, (srcv, nscale), up)
    np.savez_compressed(
        HERE / "segment_sum.npz", dst=_np(dst), offsets=_np(offsets), src=_np(srcv),
        edge_scale=_np(escale), node_scale=_np(nscale), out=_np(out), upstream=_np(up),
        grad_src=_np(g_src), grad_node_scale=_np(g_ns),
    )

    # --- segment_softmax with masked edges and null mass ---------------------
    sizes = [4, 0, 6, 1, 9, 3, 25, 2]
    dst, offsets = _graph(sizes)
    e = dst.numel()
    logit = (torch.randn(e, 8, generator=gen) * 2).requires_grad_(True)
    env = torch.rand(e, generator=gen) * 1.2 - 0.2  # some edges <= 0
    env[5] = 0.0
    env_var = env.clone().requires_grad_(True)
    null = torch.randn(len(sizes), 8, generator=gen).requires_grad_(True)
    alpha, null_alpha = segment_softmax_reference(logit, env_var, dst, offsets, null)
    ga = torch.randn(alpha.shape, generator=gen)
    gn = torch.randn(null_alpha.shape, generator=gen)
    g_logit, g_env, g_null = torch.autograd.grad((alpha, null_alpha), (logit, env_var, null),
                                                 (ga, gn))
    alpha_nonull, _ = segment_softmax_reference(logit, env, dst, offsets)
    np.savez_compressed(
        HERE / "segment_softmax.npz", dst=_np(dst), offsets=_np(offsets), logit=_np(logit),
        env=_np(env), null_logit=_np(null), alpha=_np(alpha), null_alpha=_np(null_alpha),
        grad_alpha=_np(ga), grad_null_alpha=_np(gn), grad_logit=_np(g_logit),
        grad_env=_np(g_env), grad_null_logit=_np(g_null), alpha_nonull=_np(alpha_nonull),
    )

    # --- fused softmax + weighted sum (composition of two reference calls) --
    sizes = [5, 2, 0, 11, 7, 1, 16]
    dst, offsets = _graph(sizes)
    e = dst.numel()
    heads, comps, channels = 8, 4, 16
    logit = torch.randn(e, heads, generator=gen) * 2
    value = torch.randn(e, comps, channels, generator=gen)
    alpha, _ = segment_softmax_reference(logit, torch.ones(e), dst, offsets)
    rows = (value.reshape(e, comps, heads, channels // heads)
            * alpha.reshape(e, 1, heads, 1)).reshape(e, -1)
    summed = segment_sum_reference(rows, dst, offsets)
    attn = summed.reshape(len(sizes), comps, heads, channels // heads).permute(0, 2, 1, 3)
    np.savez_compressed(
        HERE / "segment_attention.npz", dst=_np(dst), offsets=_np(offsets), logit=_np(logit),
        value=_np(value), out=_np(attn.contiguous()),
    )

    # --- force assembly ------------------------------------------------------
    sizes = [3, 1, 0, 6, 2, 9, 4]
    dst, dst_off = _graph(sizes)
    e = dst.numel()
    src = torch.randint(0, len(sizes), (e,), generator=gen)
    order, src_off = group_by_source(src, len(sizes))
    grad_edge = torch.randn(e, 3, generator=gen) * 0.1
    edge_vec = torch.randn(e, 3, generator=gen)
    force, virial = force_assembly_reference(grad_edge, edge_vec, src, dst, dst_off, src_off)
    np.savez_compressed(
        HERE / "force_assembly.npz", dst=_np(dst), dst_offsets=_np(dst_off), src=_np(src),
        src_order=_np(order), src_offsets=_np(src_off), grad_edge=_np(grad_edge),
        edge_vec=_np(edge_vec), force=_np(force), virial=_np(virial),
    )

    # --- RMSNorm (forward + gradients), tail widths --------------------------
    cases = {}
    for tag, shape in (("w17", (3, 2, 17)), ("w128", (6, 16, 128)), ("w257", (2, 3, 257))):
        x = torch.randn(*shape, generator=gen).requires_grad_(True)
        scale = torch.randn(shape[-1], generator=gen).requires_grad_(True)
        y = rmsnorm(x, scale, eps=1e-5)
        up = torch.randn(y.shape, generator=gen)
        gx, gs = torch.autograd.grad(y, (x, scale), up)
        cases.update({f"{tag}_x": _np(x), f"{tag}_scale": _np(scale), f"{tag}_y": _np(y),
                      f"{tag}_upstream": _np(up), f"{tag}_grad_x": _np(gx),
                      f"{tag}_grad_scale": _np(gs)})
    # per-degree weights: the reference rmsnorm applied per degree slice
    x = torch.randn(5, 16, 128, generator=gen)
    w = torch.rand(4, 128, generator=gen) + 0.5
    y = torch.cat([rmsnorm(x[:, l * l:(l + 1) ** 2, :].contiguous(), w[l].contiguous())
                   for l in range(4)], dim=1)
    cases.update({"deg_x": _np(x), "deg_w": _np(w), "deg_y": _np(y)})
    np.savez_compressed(HERE / "rmsnorm.npz", **cases)

    # --- GIE zonal scatter with unsorted, colliding destinations -------------
    e, n = 40, 6
    dst = torch.randint(0, n, (e,), generator=gen)
    zonal = torch.randn(e, 15, generator=gen).requires_grad_(True)
    radial = torch.randn(e, 4, 16, generator=gen).requires_grad_(True)
    slot = torch.tensor([1, 1, 1, 2, 2, 2, 2, 2, 3, 3, 3, 3, 3, 3, 3])
    inv = (torch.rand(n, generator=gen) + 0.3).requires_grad_(True)
    out = zonal_scatter_reference(zonal, radial, dst, slot, inv)
    up = torch.randn(out.shape, generator=gen)
    gz, gr, gi = torch.autograd.grad(out, (zonal, radial, inv), up)
    np.savez_compressed(
        HERE / "gie.npz", dst=_np(dst), zonal=_np(zonal), radial=_np(radial), slot=_np(slot),
        inv=_np(inv), out=_np(out), upstream=_np(up), grad_zonal=_np(gz), grad_radial=_np(gr),
        grad_inv=_np(gi),
    )
    print("wrote", sorted(p.name for p in HERE.glob("*.npz")))


if __name__ == "__main__":
    if len(sys.argv) != 2:
        raise SystemExit("usage: make_golden.py <reference project root>")
    main(sys.argv[1])
