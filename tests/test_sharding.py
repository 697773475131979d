"""Host logic of the multi-GPU decompositions, on CPU with gloo ranks.

The destination-range partition of ``force_assembly`` (source partials of all
atoms on every rank, summed by a reduce-scatter, destination sums added
locally) must reproduce the single-device result; the per-rank compute steps
are CPU stand-ins here, the CUDA entry points are checked in the GPU suite.
"""
from __future__ import annotations

import os
import socket

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from oracle import truth
from bysj_b200 import sharding as S
from bysj_b200 import workloads as W


def cpu_group_by_source(src, n):
    order = torch.argsort(src, stable=True)
    off = torch.zeros(n + 1, dtype=torch.int64)
    off[1:] = torch.cumsum(torch.bincount(src, minlength=n), 0)
    return order, off


def cpu_src_partial(g, v, soff, order):
    n = soff.numel() - 1
    owner = torch.repeat_interleave(torch.arange(n), soff[1:] - soff[:-1])
    gs, vs = g[order].double(), v[order].double()
    part = torch.zeros(n, 12, dtype=torch.float64)
    part[:, :3].index_add_(0, owner, -gs)
    part[:, 3:].index_add_(0, owner, -(gs[:, :, None] * vs[:, None, :]).reshape(-1, 9))
    return part


def cpu_dst_add(g, doff, summed):
    n = doff.numel() - 1
    owner = torch.repeat_interleave(torch.arange(n), doff[1:] - doff[:-1])
    force = summed[:, :3].index_add(0, owner, g.double())
    return force.float(), summed[:, 3:].float()


def offsets_of(dst, n):
    off = torch.zeros(n + 1, dtype=torch.int64)
    off[1:] = torch.cumsum(torch.bincount(dst, minlength=n), 0)
    return off


def test_frame_share_covers_each_frame_once():
    for world in (1, 2, 3, 8):
        got = sorted(f for r in range(world) for f in S.frame_share(13, r, world))
        assert got == list(range(13))
    with pytest.raises(ValueError):
        S.frame_share(4, 2, 2)


@pytest.mark.parametrize("parts", [1, 2, 3, 4, 8])
def test_edge_balanced_bounds(parts):
    g = W.c1_box()
    off = offsets_of(g.dst, g.n_atoms)
    b = S.edge_balanced_bounds(off, parts)
    assert b[0] == 0 and b[-1] == g.n_atoms and len(b) == parts + 1
    assert all(b[i] <= b[i + 1] for i in range(parts))
    per = [int(off[b[i + 1]] - off[b[i]]) for i in range(parts)]
    widest = int((off[1:] - off[:-1]).max())
    assert sum(per) == g.n_edges
    assert max(per) - min(per) <= 2 * widest


def test_edge_balanced_bounds_empty_and_skewed():
    off = torch.tensor([0, 0, 0, 100, 100, 101], dtype=torch.int64)
    b = S.edge_balanced_bounds(off, 4)
    assert b[0] == 0 and b[-1] == 5 and all(b[i] <= b[i + 1] for i in range(4))
    assert S.edge_balanced_bounds(torch.zeros(4, dtype=torch.int64), 2) == [0, 0, 3]


def test_padded_offsets_layout():
    off = torch.tensor([0, 2, 2, 5, 9, 10], dtype=torch.int64)   # 5 atoms
    got = S.padded_offsets(off, [0, 2, 5], 3)
    # rank 0: atoms 0,1 then one empty row; rank 1: atoms 2,3,4
    assert got.tolist() == [0, 2, 2, 2, 5, 9, 10]


def test_partition_single_rank_matches_truth():
    g = W.c1_box()
    off = offsets_of(g.dst, g.n_atoms)
    gen = torch.Generator().manual_seed(3)
    grad = torch.randn(g.n_edges, 3, generator=gen)
    parts = [S.make_partition(off, g.src, r, 3, group_by_source=cpu_group_by_source)
             for r in range(3)]
    assert sum(p.n_edges for p in parts) == g.n_edges
    partials = [cpu_src_partial(p.edges(grad), p.edges(g.edge_vec), p.src_offsets, p.src_order)
                for p in parts]
    assert all(x.shape == (3 * parts[0].chunk, 12) for x in partials)
    total = torch.stack(partials).sum(0)
    force, virial = [], []
    for p in parts:
        f, v = S.force_assembly_partitioned(
            p.edges(grad), p.edges(g.edge_vec), p, src_partial=cpu_src_partial,
            dst_add=cpu_dst_add,
            combine=lambda _, q: total[q.rank * q.chunk:(q.rank + 1) * q.chunk])
        force.append(f)
        virial.append(v)
    tf, tv = truth.force_assembly(grad.numpy(), g.edge_vec.numpy(), g.src.numpy(),
                                  g.dst.numpy(), g.n_atoms)
    np.testing.assert_allclose(torch.cat(force).numpy(), tf, rtol=1e-5, atol=1e-5)
    np.testing.assert_allclose(torch.cat(virial).numpy(), tv, rtol=1e-5, atol=1e-5)


def test_force_exchange_call_order():
    g = W.c1_box()
    off = offsets_of(g.dst, g.n_atoms)
    p = S.make_partition(off, g.src, 0, 1, group_by_source=cpu_group_by_source)
    ex = S.ForceExchange(p, src_partial=cpu_src_partial, dst_add=cpu_dst_add,
                         combine=lambda x, q: x)
    with pytest.raises(RuntimeError):
        ex.finish()
    grad = torch.zeros(g.n_edges, 3)
    ex.start(grad, g.edge_vec)
    with pytest.raises(RuntimeError):
        ex.start(grad, g.edge_vec)
    f, v = ex.finish()
    assert f.shape == (g.n_atoms, 3) and v.shape == (g.n_atoms, 9)
    with pytest.raises(ValueError):
        S.make_partition(off, g.src[:10], 0, 2, group_by_source=cpu_group_by_source)


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _worker(rank, world, port, out_dir):
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        g = W.c1_box()
        off = offsets_of(g.dst, g.n_atoms)
        gen = torch.Generator().manual_seed(11)
        grad = torch.randn(g.n_edges, 3, generator=gen)
        part = S.make_partition(off, g.src, rank, world, group_by_source=cpu_group_by_source)
        force, virial = S.force_assembly_partitioned(
            part.edges(grad), part.edges(g.edge_vec), part,
            src_partial=cpu_src_partial, dst_add=cpu_dst_add)
        torch.save({"force": force, "virial": virial, "begin": part.atom_begin},
                   os.path.join(out_dir, f"rank{rank}.pt"))
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("world", [2, 3])
def test_partitioned_force_with_gloo_ranks(tmp_path, world):
    mp.start_processes(_worker, args=(world, _free_port(), str(tmp_path)), nprocs=world,
                       join=True, start_method="spawn")
    parts = sorted((torch.load(tmp_path / f"rank{r}.pt") for r in range(world)),
                   key=lambda d: d["begin"])
    force = torch.cat([p["force"] for p in parts])
    virial = torch.cat([p["virial"] for p in parts])
    g = W.c1_box()
    gen = torch.Generator().manual_seed(11)
    grad = torch.randn(g.n_edges, 3, generator=gen)
    tf, tv = truth.force_assembly(grad.numpy(), g.edge_vec.numpy(), g.src.numpy(),
                                  g.dst.numpy(), g.n_atoms)
    np.testing.assert_allclose(force.numpy(), tf, rtol=1e-5, atol=1e-5)
    np.testing.assert_allclose(virial.numpy(), tv, rtol=1e-5, atol=1e-5)


def test_single_partition_needs_no_process_group():
    g = W.c1_box()
    off = offsets_of(g.dst, g.n_atoms)
    p = S.make_partition(off, g.src, 0, 1, group_by_source=cpu_group_by_source)
    gen = torch.Generator().manual_seed(5)
    grad = torch.randn(g.n_edges, 3, generator=gen)
    assert not dist.is_initialized()
    f, v = S.force_assembly_partitioned(grad, g.edge_vec, p, src_partial=cpu_src_partial,
                                        dst_add=cpu_dst_add)
    tf, tv = truth.force_assembly(grad.numpy(), g.edge_vec.numpy(), g.src.numpy(),
                                  g.dst.numpy(), g.n_atoms)
    np.testing.assert_allclose(f.numpy(), tf, rtol=1e-5, atol=1e-5)
    np.testing.assert_allclose(v.numpy(), tv, rtol=1e-5, atol=1e-5)


def _leaving_worker(rank, world, port, out_dir, how):
    # Both ranks run one partitioned step; rank 1 then leaves between steps
    # (``exit``: its process ends, nothing of it in flight; ``stall``: it stays
    # alive but never joins the next step) and rank 0 tries a second step,
    # which must end with an error within the group's 5 s timeout.
    import time

    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    S.init_process_group("gloo", timeout_s=5.0, rank=rank, world_size=world)
    g = W.c1_box()
    off = offsets_of(g.dst, g.n_atoms)
    grad = torch.randn(g.n_edges, 3, generator=torch.Generator().manual_seed(2))
    part = S.make_partition(off, g.src, rank, world, group_by_source=cpu_group_by_source)

    def step():
        return S.force_assembly_partitioned(part.edges(grad), part.edges(g.edge_vec), part,
                                            src_partial=cpu_src_partial, dst_add=cpu_dst_add)

    step()
    if rank == 1:
        if how == "stall":
            time.sleep(12.0)
        os._exit(0)  # leaves between steps without a goodbye
    t0 = time.monotonic()
    outcome = {"raised": False}
    try:
        step()
    except Exception as error:  # noqa: BLE001 - the test records whatever surfaced
        outcome = {"raised": True, "type": type(error).__name__, "message": str(error)[:200]}
    outcome["seconds"] = time.monotonic() - t0
    torch.save(outcome, os.path.join(out_dir, "rank0.pt"))
    os._exit(0)


@pytest.mark.parametrize("how", ["exit", "stall"])
def test_rank_leaving_between_steps_gives_a_clean_error(tmp_path, how):
    mp.start_processes(_leaving_worker, args=(2, _free_port(), str(tmp_path), how), nprocs=2,
                       join=True, start_method="spawn")
    outcome = torch.load(tmp_path / "rank0.pt")
    assert outcome["raised"], outcome
    assert outcome["seconds"] < 11.0, outcome
    print("rank 0 after its peer left:", outcome)
