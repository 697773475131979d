"""Destination-range partition over NCCL on two B200s (skipped below 2 GPUs).

Two ranks, one process per GPU, split a 6144-atom water box by destination
ranges and assemble forces with ``sharding.ForceExchange``: source partials in
float64, one NCCL reduce-scatter, destination sums added locally.  Each rank
checks that three repeated exchanges give bit-identical forces and virials
and that they equal the single-device ``force_assembly`` of the whole box
(the float64 exchange rounds each sum to float32 once, as one device does).
"""
from __future__ import annotations

import os
import socket

import pytest
import torch
import torch.multiprocessing as mp

pytestmark = pytest.mark.gpu


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _rank(rank, world, port, out_dir):
    import datetime

    import torch.distributed as dist

    from bysj_b200 import _C
    from bysj_b200 import kernels as K
    from bysj_b200 import sharding as S
    from bysj_b200 import workloads as W

    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    device = torch.device("cuda", rank)
    torch.cuda.set_device(device)
    dist.init_process_group("nccl", rank=rank, world_size=world, device_id=device,
                            timeout=datetime.timedelta(seconds=60))
    result = {"rank": rank}
    try:
        g = W.water_box(6144, density=0.1, seed=3, device=device)
        off = K.segment_offsets(g.dst, g.n_atoms)
        gen = torch.Generator(device=device).manual_seed(5)
        grad = torch.randn(g.n_edges, 3, device=device, generator=gen) * 2.0
        part = S.make_partition(off, g.src, rank, world)
        ex = S.ForceExchange(part)
        runs = []
        for _ in range(3):
            ex.start(part.edges(grad).contiguous(), part.edges(g.edge_vec).contiguous())
            f, v = ex.finish()
            runs.append((f.clone(), v.clone()))
        torch.cuda.synchronize()
        result["repeat_identical"] = all(torch.equal(runs[0][0], r[0]) and
                                         torch.equal(runs[0][1], r[1]) for r in runs[1:])
        order, soff = K.group_by_source(g.src, g.n_atoms)
        f_ref, v_ref = _C.force_assembly(grad, g.edge_vec, off, soff, order)
        f, v = runs[0]
        result["max_err"] = max(float((f - part.atoms(f_ref)).abs().max()),
                                float((v - part.atoms(v_ref)).abs().max()))
        result["max_ulp_scale"] = float(part.atoms(f_ref).abs().max())
        result["n_local"] = part.n_local
    finally:
        torch.save(result, os.path.join(out_dir, f"rank{rank}.pt"))
        dist.destroy_process_group()


def test_partitioned_force_assembly_on_two_gpus(tmp_path):
    if not torch.cuda.is_available() or torch.cuda.device_count() < 2:
        pytest.skip("needs two GPUs")
    env = {"NCCL_NVLS_ENABLE": os.environ.get("NCCL_NVLS_ENABLE", "0")}
    os.environ.update(env)
    mp.start_processes(_rank, args=(2, _free_port(), str(tmp_path)), nprocs=2, join=True,
                       start_method="spawn")
    for r in range(2):
        res = torch.load(tmp_path / f"rank{r}.pt")
        assert res["n_local"] > 0
        assert res["repeat_identical"], res
        # one float32 rounding of float64 sums on both sides: at most an ulp apart
        assert res["max_err"] <= 2.0 ** -22 * max(1.0, res["max_ulp_scale"]), res
