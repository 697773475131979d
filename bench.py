#!/usr/bin/env python
"""Benchmark of the B200 segmented-operator path (one JSON line on rank 0).

Headline workload ("C3", the fused-attention configuration): aggregation on
a 24576-atom water-like periodic box (density 0.1 / A^3, rcut 6 A, ~2.22 M
dst-sorted edges); logits fp32 [E, 8] drawn N(0, 2) (variance 2), values
fp32 [E, 16, 64] drawn N(0, 1).  One step = ``segment_offsets`` (device
boundary kernels) -> ``segment_attention`` (fused gated softmax + weighted
segment sum) producing [N, 8, 16, 8].  The metric is edges/s.

* ``value``: device throughput, inputs resident in HBM, CUDA events around K
  back-to-back steps (inputs are 9.1 GB per frame, far larger than the 126 MB
  L2, so no flush is needed), barrier + synchronize on both sides, max over
  ranks.  With N GPUs each rank processes its own frame per step ("weak").
* ``e2e``: the same metric through the public API (``bysj_b200.kernels``)
  from pinned host buffers: H2D of dst / logits / values, the two calls, D2H
  of the output, all inside the timed region.
* ``roofline``: the attention kernel's algorithmic bytes per launch over its
  average launch time (events on its stream), against MEASURED_PEAKS.json.
* ``cpu_baseline``: the reference's PyTorch oracle (restated under
  ``oracle/``) on the host cores, on the whole frame; ``check``: the public
  API's output of the e2e steps against that oracle output, elementwise at
  rtol 1e-5 / atol 1e-6 (computed outside every timed region).
* ``chain`` and ``partition``: the default run also measures the two other
  multi-GPU workloads (below) on the same ranks, at most 10 timed steps each,
  and attaches their lines.
* ``ops``: per-operator roofline lines for the other configs at N = 1:
  segment_offsets, group_by_source, bf16-value attention, standalone
  softmax, segment_sum, force_assembly (Morton and random atom order),
  zonal_scatter, RMSNorm fp32/bf16, the backward operators, and a small
  launch-bound step replayed from a CUDA graph.  ``--only OP`` times one.
* ``--mode chain``: 64 independent frames of the full chain (offsets ->
  RMSNorm -> fused attention -> zonal scatter -> source grouping -> force
  assembly, fp32, C = 32) sharded over the ranks; frames/s ("strong").
  Each rank alternates its frames over two CUDA streams and interleaves
  their stages (``--chain-streams 1`` runs them one after another).
* ``--mode partition``: one 500k-atom box split by destination ranges over
  the ranks (strong scaling; force partials reduce-scattered over NCCL).

``--impl reference`` times the CPU oracle instead (rank 0 only) on the whole
frame every step and reports the same metric and config.
"""
from __future__ import annotations

import argparse
import gc
import json
import os
import statistics
import subprocess
import sys
import threading
import time
from pathlib import Path

import torch

ROOT = Path(__file__).resolve().parent
sys.path.insert(0, str(ROOT))

METRIC = "edges/s (fused segment softmax + weighted sum, 24576-atom C3 frame)"
UNIT = "edges/s"
FALLBACK_HBM_GBS = 6650.0


def parse_args():
    p = argparse.ArgumentParser(description=__doc__.splitlines()[0])
    p.add_argument("--gpus", type=int, default=1)
    p.add_argument("--steps", type=int, default=200)
    p.add_argument("--warmup", type=int, default=5)
    p.add_argument("--impl", choices=("ours", "reference"), default="ours")
    p.add_argument("--values", choices=("f32", "bf16"), default="f32")
    p.add_argument("--seed", type=int, default=0)
    p.add_argument("--no-e2e", action="store_true")
    p.add_argument("--no-ops", action="store_true")
    p.add_argument("--no-cpu", action="store_true")
    p.add_argument("--no-extra", action="store_true",
                   help="skip the chain and partition lines of the default run")
    p.add_argument("--profile-small", action="store_true",
                   help="tiny frame for ncu captures (not a bench number)")
    p.add_argument("--only", choices=sorted(OPS),
                   help="time one operator on its own (per-op line only, no headline)")
    p.add_argument("--atoms", type=int, default=24576,
                   help="atoms of the synthetic box used by --only")
    p.add_argument("--mode", choices=("frames", "chain", "partition"), default="frames",
                   help="frames: one C3 frame per rank (default); chain: the full operator "
                        "chain over 64 frames sharded across the ranks; partition: one large "
                        "box split by destination-atom ranges, force partials reduce-scattered")
    p.add_argument("--chain-frames", type=int, default=64,
                   help="frames of the job in --mode chain")
    p.add_argument("--chain-streams", type=int, default=2,
                   help="CUDA streams per rank that --mode chain alternates frames over")
    p.add_argument("--partition-atoms", type=int, default=500_000,
                   help="atoms of the box used by --mode partition")
    return p.parse_args()


# ---------------------------------------------------------------------------
# distributed plumbing
# ---------------------------------------------------------------------------

class Dist:
    def __init__(self):
        self.world = int(os.environ.get("WORLD_SIZE", "1"))
        self.rank = int(os.environ.get("RANK", "0"))
        self.local = int(os.environ.get("LOCAL_RANK", "0"))
        self.pg = None

    def setup(self, backend: str):
        if self.world > 1:
            from bysj_b200 import sharding as S

            kwargs = {}
            if backend == "nccl":
                device = torch.device("cuda", self.local)
                torch.cuda.set_device(device)
                kwargs["device_id"] = device
            # bounded: a rank that dies makes the others' next collective raise
            self.pg = S.init_process_group(backend, timeout_s=120.0, **kwargs)

    def barrier(self):
        if self.pg is not None:
            self.pg.barrier()

    def max(self, value: float) -> float:
        if self.pg is None:
            return value
        t = torch.tensor([value], dtype=torch.float64, device="cuda")
        self.pg.all_reduce(t, op=self.pg.ReduceOp.MAX)
        return float(t.item())

    def sum(self, value: float) -> float:
        if self.pg is None:
            return value
        t = torch.tensor([value], dtype=torch.float64, device="cuda")
        self.pg.all_reduce(t, op=self.pg.ReduceOp.SUM)
        return float(t.item())

    def close(self):
        if self.pg is not None:
            self.pg.destroy_process_group()


# ---------------------------------------------------------------------------
# clocks
# ---------------------------------------------------------------------------

class ClockSampler:
    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, device: torch.device):
        try:
            uuid = str(torch.cuda.get_device_properties(device).uuid)
            self.gpu = uuid if uuid.startswith("GPU-") else f"GPU-{uuid}"
        except (AttributeError, RuntimeError):
            self.gpu = str(device.index or 0)
        self.proc = None
        self.lines: list[str] = []
        self.thread = None

    def start(self):
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", f"--id={self.gpu}", f"--query-gpu={self.FIELDS}",
                 "--format=csv,noheader,nounits", "-lms", "50"],
                stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
        except (FileNotFoundError, OSError):
            self.proc = None
            return
        self.thread = threading.Thread(target=self._read, daemon=True)
        self.thread.start()
        time.sleep(0.3)

    def _read(self):
        for line in self.proc.stdout:
            self.lines.append(line.strip())

    def stop(self) -> dict:
        if self.proc is None:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["nvidia-smi unavailable"]}
        time.sleep(0.2)
        self.proc.terminate()
        try:
            self.proc.wait(timeout=5)
        except subprocess.TimeoutExpired:
            self.proc.kill()
        sm, smax, reasons = [], [], set()
        names = ("hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap")
        for line in self.lines:
            parts = [x.strip() for x in line.split(",")]
            if len(parts) < 9:
                continue
            try:
                sm.append(float(parts[1]))
                smax.append(float(parts[2]))
            except ValueError:
                continue
            for name, flag in zip(names, parts[5:9]):
                if flag.lower().startswith("active"):
                    reasons.add(name)
        if not sm:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["no samples"]}
        loaded = [s for s in sm if s > 0.5 * max(sm)] or sm
        return {"sm_mhz": statistics.median(loaded), "sm_max_mhz": max(smax),
                "reasons": sorted(reasons), "samples": len(sm)}


def measured_peak() -> tuple[float, str]:
    path = ROOT / "MEASURED_PEAKS.json"
    try:
        data = json.loads(path.read_text())
        return float(data["hbm_gbs"]), "measured (MEASURED_PEAKS.json hbm_gbs)"
    except (OSError, KeyError, ValueError):
        return FALLBACK_HBM_GBS, "fallback 6.65 TB/s (no MEASURED_PEAKS.json)"


def profiled_traffic_per_edge(name: str) -> float | None:
    """``traffic_bytes_per_edge: X`` from the committed ncu summary, if any."""
    path = ROOT / "profiles" / f"{name}.md"
    try:
        for line in path.read_text().splitlines():
            if line.strip().startswith("traffic_bytes_per_edge:"):
                return float(line.split(":", 1)[1].split()[0])
    except (OSError, ValueError):
        return None
    return None


# ---------------------------------------------------------------------------
# workload
# ---------------------------------------------------------------------------

def make_frame(device, seed, values_dtype, small=False):
    from bysj_b200 import workloads as W

    g = W.water_box(1536, density=0.1, seed=seed, device=device) if small else \
        W.c3_box(device=device, seed=seed)
    gen = torch.Generator(device=device).manual_seed(seed + 17)
    logit = torch.randn(g.n_edges, 8, device=device, generator=gen) * (2.0 ** 0.5)
    value = torch.randn(g.n_edges, 16, 64, device=device, generator=gen)
    if values_dtype == "bf16":
        value = value.to(torch.bfloat16)
    return g, logit.contiguous(), value.contiguous()


def c3_config(n_atoms, n_edges, values, world):
    """The headline workload's `config` object (both arms report the same one)."""
    return {"workload": "C3 fused attention: segment_offsets -> segment_attention",
            "n_atoms": n_atoms, "n_edges_per_frame": n_edges, "heads": 8, "components": 16,
            "channels": 64, "values": values, "frames_per_gpu_per_step": 1,
            "parallelism": f"frame-sharded x{world} (no collective)",
            "l2": "inputs (~9.1 GB fp32 values) larger than L2; no flush"}


def attention_bytes(e, n, value_elem_bytes):
    return e * (8 * 4 + 16 * 64 * value_elem_bytes) + n * 16 * 64 * 4 + 8 * (n + 1)


def cpu_frame_rate(g, logit, value, out_public=None, repeats=2):
    """The reference's PyTorch oracle on the WHOLE frame on the host cores.

    Returns the ``cpu_baseline`` object (edges/s of one full frame, median of
    ``repeats`` after one untimed run) and, when ``out_public`` (the public
    API's [N, 8, 16, 8] output of the same frame, on the host) is given, the
    ``check`` object: that output against the oracle's, elementwise at the
    spec's rtol 1e-5 / atol 1e-6.  The oracle is only the checker here and
    the timed CPU baseline; nothing on the GPU path calls it."""
    sys.path.insert(0, str(ROOT / "oracle"))
    from reference import segment_attention_reference

    cores = os.cpu_count() or 1
    torch.set_num_threads(cores)
    dst = g.dst.cpu()
    offsets = torch.zeros(g.n_atoms + 1, dtype=torch.int64)
    offsets[1:] = torch.cumsum(torch.bincount(dst, minlength=g.n_atoms), 0)
    lg = logit.cpu()
    val = value.float().cpu()
    want = segment_attention_reference(lg, val, dst, offsets)  # untimed first run
    times = []
    for _ in range(repeats):
        t0 = time.perf_counter()
        segment_attention_reference(lg, val, dst, offsets)
        times.append(time.perf_counter() - t0)
    per = statistics.median(times)
    cpu = {
        "value": g.n_edges / per,
        "unit": UNIT,
        "cores": cores,
        "kind": "port",
        "sample": f"the whole frame ({g.n_atoms} segments, {g.n_edges} edges): "
                  f"oracle.reference.segment_attention_reference (the reference's "
                  f"python/reference chain, restated) on CPU, torch threads="
                  f"{torch.get_num_threads()}, median of {repeats} after one untimed run",
        "seconds_per_frame": per,
    }
    check = None
    if out_public is not None:
        got = out_public.reshape(want.shape)
        diff = (got.double() - want.double()).abs()
        bound = 1e-6 + 1e-5 * want.double().abs()
        check = {"against": "fp32 oracle (reference.segment_attention_reference) on the whole "
                            "frame, output of the public API (e2e path)",
                 "elements": int(want.numel()), "rtol": 1e-5, "atol": 1e-6,
                 "outside_tolerance": int((diff > bound).sum()),
                 "max_abs_err": float(diff.max()),
                 "max_err_over_bound": float((diff / bound).max()),
                 "max_abs_value": float(want.abs().max())}
    return cpu, check


# ---------------------------------------------------------------------------
# per-op measurements (N = 1, rank 0)
# ---------------------------------------------------------------------------

class Flusher:
    """Evicts a small working set from L2 between timed launches.

    Writes 512 MB (4x the 126 MB L2), then reads another 256 MB so that the
    lines left in L2 are clean: the next timed kernel starts with none of its
    inputs cached and pays no write-back of the flush's own dirty lines.
    """

    def __init__(self, device):
        self.buf = torch.empty(512 * 1024 * 1024 // 4, dtype=torch.float32, device=device)
        self.clean = torch.ones(256 * 1024 * 1024 // 4, dtype=torch.float32, device=device)

    def __call__(self):
        self.buf.fill_(1.0)
        self.clean.sum()


def time_launches(fn, iters, flush=None):
    """Trimmed mean CUDA-event time of `fn` over `iters` launches (L2 flushed
    before each when `flush` is given): the fastest and slowest tenth (at
    least one each) are dropped.  Single launches of a few tens of
    microseconds land on a coarse grid of event timestamps, so a median sits
    on a grid point while a mean does not; the trimming keeps a rare stalled
    iteration (operators that wait on the host) out of the mean.  One untimed
    call first: an operator's first call pays for caching its workspace."""
    if flush is not None:
        flush()
    fn()
    torch.cuda.synchronize()
    times = []
    for _ in range(iters):
        if flush is not None:
            flush()
        a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        a.record()
        fn()
        b.record()
        b.synchronize()
        times.append(a.elapsed_time(b) / 1e3)
    times.sort()
    cut = max(1, len(times) // 10) if len(times) > 2 else 0
    return statistics.mean(times[cut:len(times) - cut])


def op_line(name, alg_bytes, seconds, peak, edges=None, extra=None):
    gbs = alg_bytes / seconds / 1e9
    line = {"us": seconds * 1e6, "alg_bytes": int(alg_bytes), "achieved_gbs": round(gbs, 1),
            "frac": round(gbs / peak, 4)}
    if edges:
        line["edges_per_s"] = edges / seconds
    if extra:
        line.update(extra)
    return name, line


def _op_offsets(ctx):
    from bysj_b200 import _C

    g, n, e = ctx["g"], ctx["g"].n_atoms, ctx["g"].n_edges
    flags = ctx["flags"]
    t = time_launches(lambda: _C.segment_offsets_device(g.dst, n, flags), ctx["iters"],
                      ctx["flush"])
    return op_line("segment_offsets", 8 * e + 8 * (n + 1), t, ctx["peak"], e,
                   {"note": "one fused check + boundary launch, L2 flushed"})


def _op_group(ctx):
    from bysj_b200 import _C

    g, n, e = ctx["g"], ctx["g"].n_atoms, ctx["g"].n_edges
    t = time_launches(lambda: _C.group_by_key(g.src, n), ctx["iters"], ctx["flush"])
    t_sort = time_launches(lambda: torch.argsort(g.src, stable=True), ctx["iters"], ctx["flush"])
    return op_line("group_by_source", 8 * e + 8 * e + 8 * (n + 1), t, ctx["peak"], e,
                   {"note": "histogram, scan, scatter, per-group sort; includes the flag "
                            "read back; L2 flushed",
                    "torch_argsort_stable_us": t_sort * 1e6})


def _op_attention_bf16(ctx):
    from bysj_b200 import _C

    e, n = ctx["g"].n_edges, ctx["g"].n_atoms
    vb = ctx["value32"]().to(torch.bfloat16)
    t = time_launches(lambda: _C.segment_attention_forward(ctx["logit"](), vb, ctx["offsets"]),
                      ctx["iters"])
    return op_line("segment_attention_bf16", attention_bytes(e, n, 2), t, ctx["peak"], e)


def _op_softmax(ctx):
    from bysj_b200 import _C

    e, n = ctx["g"].n_edges, ctx["g"].n_atoms
    env = torch.ones(e, device=ctx["device"])
    logit = ctx["logit"]()
    t = time_launches(lambda: _C.segment_softmax_forward(logit, env, ctx["offsets"]),
                      ctx["iters"], ctx["flush"])
    return op_line("segment_softmax_h8", e * (32 + 4 + 32) + 8 * (n + 1), t, ctx["peak"], e,
                   {"note": "standalone alpha output, L2 flushed"})


def _op_softmax_hub(ctx):
    """Standalone softmax (H = 8) on the C3 segment sizes with one extra hub
    segment of 100,000 edges in the middle of the frame; per-edge time is
    compared with the uniform C3 line."""
    from bysj_b200 import _C

    g, n = ctx["g"], ctx["g"].n_atoms
    device = ctx["device"]
    sizes = (ctx["offsets"][1:] - ctx["offsets"][:-1]).clone()
    sizes[n // 2] += 100_000
    off = torch.zeros(n + 1, dtype=torch.int64, device=device)
    off[1:] = torch.cumsum(sizes, 0)
    e = int(off[-1])
    gen = torch.Generator(device=device).manual_seed(94)
    logit = torch.randn(e, 8, device=device, generator=gen) * 2 ** 0.5
    env = torch.ones(e, device=device)
    t = time_launches(lambda: _C.segment_softmax_forward(logit, env, off), ctx["iters"],
                      ctx["flush"])
    return op_line("segment_softmax_h8_hub", e * (32 + 4 + 32) + 8 * (n + 1), t, ctx["peak"], e,
                   {"note": "C3 sizes plus one 100,000-edge segment; L2 flushed"})


def _op_segment_sum(ctx):
    from bysj_b200 import _C

    e, n = ctx["g"].n_edges, ctx["g"].n_atoms
    device = ctx["device"]
    src = ctx["value32"]().reshape(e, -1)
    ws = torch.rand(e, device=device) + 0.5
    ns = torch.rand(n, device=device) + 0.5
    t = time_launches(lambda: _C.segment_sum_forward(src, ctx["offsets"], ws, ns), ctx["iters"])
    return op_line("segment_sum_c1024", e * (4096 + 4) + n * (4096 + 4) + 8 * (n + 1), t,
                   ctx["peak"], e)


def _op_force(ctx, shuffled=False):
    from bysj_b200 import _C
    from bysj_b200 import kernels as K

    g, e, n = ctx["g"], ctx["g"].n_edges, ctx["g"].n_atoms
    gen = torch.Generator(device=ctx["device"]).manual_seed(99)
    grad = torch.randn(e, 3, device=ctx["device"], generator=gen) * 0.1
    src, unit, offsets, name = g.src, g.unit, ctx["offsets"], "force_assembly"
    if shuffled:
        # the same system with atoms numbered in random order: neighbours' rows
        # are scattered over the whole array (worst case for the source gather)
        label = torch.randperm(n, device=ctx["device"], generator=gen)
        dst, src = label[g.dst], label[src]
        perm = torch.argsort(dst * n + src)
        dst, src, unit = dst[perm].contiguous(), src[perm].contiguous(), unit[perm].contiguous()
        offsets = _C.segment_offsets_device(dst, n, ctx["flags"])
        name = "force_assembly_random_order"
    order, soff = K.group_by_source(src, n)
    fa = lambda: _C.force_assembly(grad, unit, offsets, soff, order)  # noqa: E731
    fa_bytes = e * (12 + 12 + 8) + n * (16 + 12 + 36)
    t_cold = time_launches(fa, ctx["iters"], ctx["flush"])
    t_warm = time_launches(fa, ctx["iters"])
    return op_line(name, fa_bytes, t_cold, ctx["peak"], e,
                   {"note": "L2 flushed before each launch (cold)", "warm_us": t_warm * 1e6,
                    "warm_frac": round(fa_bytes / t_warm / 1e9 / ctx["peak"], 4)})


def _op_zonal(ctx):
    from bysj_b200 import _C
    from bysj_b200 import workloads as W

    g, e, n = ctx["g"], ctx["g"].n_edges, ctx["g"].n_atoms
    device = ctx["device"]
    gen = torch.Generator(device=device).manual_seed(98)
    zonal = W.real_sph_zonal(g.unit)
    radial = torch.randn(e, 4, 64, device=device, generator=gen)
    slot = W.degree_slots().to(device)
    inv = torch.rsqrt(torch.bincount(g.dst, minlength=n).float() + 1.0)
    t = time_launches(lambda: _C.gie_zonal_scatter_forward(zonal, radial, g.dst, slot, inv),
                      ctx["iters"])
    return op_line("zonal_scatter", e * (60 + 8 + 256 * 3) + n * (4096 + 4), t, ctx["peak"], e,
                   {"note": "includes the device CSR view of dst; its flags word is read as soon "
                            "as the CSR kernel is done, while the operator runs"})


def _op_rmsnorm(ctx, dtype):
    from bysj_b200 import _C

    n = ctx["g"].n_atoms
    device = ctx["device"]
    gen = torch.Generator(device=device).manual_seed(97)
    x = torch.randn(n, 16, 128, device=device, generator=gen).to(dtype)
    w = torch.rand(4, 128, device=device, generator=gen) + 0.5
    t = time_launches(lambda: _C.rmsnorm_forward(x, w, 1e-6), ctx["iters"], ctx["flush"])
    size = 4 if dtype == torch.float32 else 2
    name = "rmsnorm_f32" if dtype == torch.float32 else "rmsnorm_bf16"
    return op_line(name, 2 * n * 16 * 128 * size + 4 * n * 16 + 2048, t, ctx["peak"], None,
                   {"rows": n * 16, "note": "per-degree weights [4,128], L2 flushed"})


def _op_segment_sum_bwd(ctx):
    from bysj_b200 import _C

    g, e, n = ctx["g"], ctx["g"].n_edges, ctx["g"].n_atoms
    device = ctx["device"]
    src = ctx["value32"]().reshape(e, -1)
    ws = torch.rand(e, device=device) + 0.5
    ns = torch.rand(n, device=device) + 0.5
    grad = torch.randn(n, src.shape[1], device=device)
    t = time_launches(lambda: _C.segment_sum_backward(grad, src, g.dst, ctx["offsets"], ws, ns,
                                                      True), ctx["iters"])
    c = src.shape[1] * 4
    return op_line("segment_sum_bwd_c1024", e * (2 * c + 4) + n * (c + 8) + 8 * (n + 1), t,
                   ctx["peak"], e, {"note": "grad_src and grad_node_scale"})


def _op_softmax_bwd(ctx):
    from bysj_b200 import _C

    e, n = ctx["g"].n_edges, ctx["g"].n_atoms
    env = torch.rand(e, device=ctx["device"]) * 0.9 + 0.1
    alpha, _ = _C.segment_softmax_forward(ctx["logit"](), env, ctx["offsets"])
    grad = torch.randn_like(alpha)
    t = time_launches(lambda: _C.segment_softmax_backward(alpha, grad, env, ctx["offsets"]),
                      ctx["iters"], ctx["flush"])
    return op_line("segment_softmax_bwd_h8", e * (32 * 3 + 4 + 4) + 8 * (n + 1), t, ctx["peak"],
                   e, {"note": "grad_logit and grad_env, L2 flushed"})


def _op_rmsnorm_bwd(ctx):
    from bysj_b200 import _C

    n = ctx["g"].n_atoms
    device = ctx["device"]
    x = torch.randn(n, 16, 128, device=device)
    w = torch.rand(128, device=device) + 0.5
    y, inv = _C.rmsnorm_forward(x, w, 1e-6)
    grad = torch.randn_like(x)
    t = time_launches(lambda: _C.rmsnorm_backward(grad, x, w, inv, True), ctx["iters"],
                      ctx["flush"])
    rows = n * 16
    return op_line("rmsnorm_bwd_f32", rows * (3 * 512 + 4) + 2 * 512, t, ctx["peak"], None,
                   {"rows": rows, "note": "gx and grad_scale, L2 flushed"})


def _op_zonal_bwd(ctx):
    from bysj_b200 import _C
    from bysj_b200 import workloads as W

    g, e, n = ctx["g"], ctx["g"].n_edges, ctx["g"].n_atoms
    device = ctx["device"]
    gen = torch.Generator(device=device).manual_seed(98)
    zonal = W.real_sph_zonal(g.unit)
    radial = torch.randn(e, 4, 64, device=device, generator=gen)
    slot = W.degree_slots().to(device)
    inv = torch.rsqrt(torch.bincount(g.dst, minlength=n).float() + 1.0)
    grad = torch.randn(n, 16, 64, device=device, generator=gen)
    t = time_launches(lambda: _C.gie_zonal_scatter_backward(grad, zonal, radial, g.dst, slot,
                                                            inv), ctx["iters"])
    return op_line("zonal_scatter_bwd", e * (60 + 8 + 768 + 60 + 1024) + n * (4096 + 8), t,
                   ctx["peak"], e,
                   {"note": "grad_zonal, grad_radial (all 4 slots written), grad_inv; includes "
                            "the device CSR view of dst"})


def _op_rotate(ctx):
    """Fused rotate-back aggregation on the C3 frame: messages [E,16,64] fp32
    (the value rows), packed orthogonal rotations [E,84], attention weights
    [E,8] normalised per segment, per-edge rescale -> [N,16,64]."""
    from bysj_b200 import kernels as K

    g, e, n = ctx["g"], ctx["g"].n_edges, ctx["g"].n_atoms
    device = ctx["device"]
    gen = torch.Generator().manual_seed(96)
    blocks = []
    for l in range(4):
        q, _ = torch.linalg.qr(torch.randn(4096, 2 * l + 1, 2 * l + 1, generator=gen,
                                           dtype=torch.float64))
        blocks.append(q.reshape(4096, -1))
    pool = torch.cat(blocks, 1).float().to(device)
    rot = pool[torch.arange(e, device=device) % 4096].contiguous()
    logit = ctx["logit"]()
    peak = torch.full((n, 8), -float("inf"), device=device).scatter_reduce(
        0, g.dst[:, None].expand(-1, 8), logit, "amax")
    w = torch.exp(logit - peak[g.dst])
    alpha = (w / torch.zeros_like(peak).index_add_(0, g.dst, w)[g.dst]).contiguous()
    scale = torch.rand(e, device=device) + 0.5
    x = ctx["value32"]()
    off = ctx["offsets"]
    t = time_launches(lambda: K.rotate_back_aggregate(x, rot, scale, alpha, None, off, g.dst, 3,
                                                      8), ctx["iters"])
    return op_line("rotate_back_aggregate", e * (4096 + 336 + 32 + 4) + n * 4096 + 8 * (n + 1),
                   t, ctx["peak"], e,
                   {"note": "rotate-back (84 coefficients per edge) + weighting + destination "
                            "sum in one pass; inputs larger than L2"})


def _op_chain(ctx):
    """One-pass edge-stream chain x + y * gate + residual over [E, 9, 64] fp32
    (the gate [E, 1, 64] broadcast over the components) on the C3 edge
    count, beside the same chain as eager torch passes."""
    from bysj_b200 import kernels as K

    e = ctx["g"].n_edges
    device = ctx["device"]
    gen = torch.Generator(device=device).manual_seed(95)
    x, y, res = (torch.randn(e, 9, 64, device=device, generator=gen) for _ in range(3))
    gate = torch.randn(e, 1, 64, device=device, generator=gen)
    terms = [(1.0, x), (1.0, y, gate), (1.0, res)]
    t = time_launches(lambda: K.edge_chain(terms, (e, 9, 64)), ctx["iters"])
    t_eager = time_launches(lambda: x + y * gate + res, ctx["iters"])
    row = 9 * 64 * 4
    return op_line("edge_chain", e * (4 * row + 64 * 4), t, ctx["peak"], e,
                   {"eager_us": t_eager * 1e6,
                    "note": "3 terms (2 full streams + gated stream), 1 output, one pass; "
                            "eager_us = torch x + y * gate + res (3 passes)"})


def _op_small_step_graph(ctx):
    """A launch-bound step on the 192-atom C1 box, eager and as a CUDA-graph replay."""
    from bysj_b200 import _C
    from bysj_b200 import kernels as K
    from bysj_b200 import workloads as W

    device = ctx["device"]
    g = W.c1_box(device=device)
    e, n = g.n_edges, g.n_atoms
    gen = torch.Generator(device=device).manual_seed(23)
    logit = torch.randn(e, 8, device=device, generator=gen)
    value = torch.randn(e, 16, 64, device=device, generator=gen)
    env = torch.rand(e, device=device, generator=gen) + 0.05
    grad = torch.randn(e, 3, device=device, generator=gen) * 0.1
    x = torch.randn(n, 16, 128, device=device, generator=gen)
    w = torch.rand(4, 128, device=device, generator=gen) + 0.5
    order, soff = K.group_by_source(g.src, n)
    flags = torch.zeros(1, dtype=torch.int32, device=device)

    def step():
        off = _C.segment_offsets_device(g.dst, n, flags)
        _C.segment_attention_forward(logit, value, off)
        _C.segment_softmax_forward(logit, env, off)
        _C.force_assembly(grad, g.unit, off, soff, order)
        _C.rmsnorm_forward(x, w, 1e-6)

    reps = 20
    side = torch.cuda.Stream()
    side.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(side):
        step()
    torch.cuda.current_stream().wait_stream(side)
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph):
        step()
    t_eager = time_launches(lambda: [step() for _ in range(reps)], ctx["iters"]) / reps
    t_graph = time_launches(lambda: [graph.replay() for _ in range(reps)], ctx["iters"]) / reps
    del graph
    alg = (e * (32 + 4096) + n * 4096 + e * (32 + 4 + 32) + e * 32 + n * 64
           + 2 * n * 16 * 128 * 4 + 8 * e + 8 * (n + 1))
    return op_line("c1_step_graph", alg, t_graph, ctx["peak"], e,
                   {"eager_us": t_eager * 1e6,
                    "note": "offsets + attention + softmax + force + RMSNorm on the 192-atom "
                            "C1 box (17.7k edges, launch-bound); us = one CUDA-graph replay, "
                            "eager_us = the same launches issued one by one"})


OPS = {
    "offsets": _op_offsets,
    "c1_step_graph": _op_small_step_graph,
    "group": _op_group,
    "attention_bf16": _op_attention_bf16,
    "softmax": _op_softmax,
    "softmax_hub": _op_softmax_hub,
    "segment_sum": _op_segment_sum,
    "force": _op_force,
    "force_random_order": lambda ctx: _op_force(ctx, shuffled=True),
    "zonal": _op_zonal,
    "rmsnorm": lambda ctx: _op_rmsnorm(ctx, torch.float32),
    "rmsnorm_bf16": lambda ctx: _op_rmsnorm(ctx, torch.bfloat16),
    "segment_sum_bwd": _op_segment_sum_bwd,
    "softmax_bwd": _op_softmax_bwd,
    "rmsnorm_bwd": _op_rmsnorm_bwd,
    "zonal_bwd": _op_zonal_bwd,
    "rotate": _op_rotate,
    "chain": _op_chain,
}


def op_context(g, device, peak, logit=None, value32=None, iters=20):
    """Shared inputs of the per-op lines; logits / values built on demand."""
    from bysj_b200 import _C

    flags = torch.zeros(1, dtype=torch.int32, device=device)
    cache = {}

    def lazy(name, make):
        def get():
            if name not in cache:
                cache[name] = make()
            return cache[name]
        return get

    gen = torch.Generator(device=device).manual_seed(17)
    return {
        "g": g, "device": device, "peak": peak, "iters": iters, "flags": flags,
        "flush": Flusher(device),
        "offsets": _C.segment_offsets_device(g.dst, g.n_atoms, flags),
        "logit": (lambda: logit) if logit is not None else lazy(
            "logit", lambda: torch.randn(g.n_edges, 8, device=device, generator=gen) * 2 ** 0.5),
        "value32": (lambda: value32) if value32 is not None else lazy(
            "value", lambda: torch.randn(g.n_edges, 16, 64, device=device, generator=gen)),
    }


def measure_ops(g, logit, value32, device, peak, iters=20, only=None):
    ctx = op_context(g, device, peak, logit, value32, iters)
    out = {}
    for name, fn in OPS.items():
        if only is not None and name != only:
            continue
        key, line = fn(ctx)
        out[key] = line
    return out


# ---------------------------------------------------------------------------
# arms
# ---------------------------------------------------------------------------

def run_reference(args, dist):
    """The reference's CPU path on the whole C3 frame, rank 0 only.

    The reference's own implementation of this path is its PyTorch
    ``reference.*`` chain (its HIP kernels need a Hygon DCU); it is restated
    under ``oracle/`` and timed here with all host threads on every step's full
    frame (2.2 M edges, 9.1 GB of fp32 values), inputs drawn from a CPU
    generator with the headline's shapes and distributions."""
    if dist.rank != 0:
        return
    from bysj_b200 import workloads as W

    cores = os.cpu_count() or 1
    torch.set_num_threads(cores)
    g = W.c3_box(device="cpu", seed=args.seed)
    gen = torch.Generator().manual_seed(args.seed + 17)
    e = g.n_edges
    logit = torch.randn(e, 8, generator=gen) * (2.0 ** 0.5)
    value = torch.randn(e, 16, 64, generator=gen)
    sys.path.insert(0, str(ROOT / "oracle"))
    from reference import segment_attention_reference

    dst = g.dst.contiguous()
    off = torch.zeros(g.n_atoms + 1, dtype=torch.int64)
    off[1:] = torch.cumsum(torch.bincount(dst, minlength=g.n_atoms), 0)
    for _ in range(args.warmup):
        segment_attention_reference(logit, value, dst, off)
    t0 = time.perf_counter()
    for _ in range(args.steps):
        segment_attention_reference(logit, value, dst, off)
    per = (time.perf_counter() - t0) / args.steps
    rate = e / per
    sample = (f"the whole frame per step ({g.n_atoms} segments, {e} edges); "
              "oracle.reference.segment_attention_reference (the reference's python/reference "
              f"softmax + weighted segment_sum chain, restated) on CPU, torch threads="
              f"{torch.get_num_threads()}")
    line = {
        "impl": "reference", "metric": METRIC, "value": rate, "unit": UNIT,
        "n_gpus": args.gpus, "steps": args.steps, "warmup": args.warmup,
        "ms_per_step": per * 1e3, "higher_is_better": True, "scaling": "weak",
        "vs_baseline": None, "dtype": "f32", "data": "synthetic",
        "config": c3_config(g.n_atoms, g.n_edges, "f32", args.gpus),
        "cpu_baseline": {"value": rate, "unit": UNIT, "cores": cores, "kind": "port",
                         "sample": sample},
        "e2e": {"value": rate, "unit": UNIT, "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)


def run_ours(args, dist):
    from bysj_b200 import _C
    from bysj_b200 import kernels as K

    device = torch.device("cuda", dist.local)
    torch.cuda.set_device(device)
    seed = args.seed + 1000 * dist.rank
    g, logit, value = make_frame(device, seed, args.values, small=args.profile_small)
    e, n = g.n_edges, g.n_atoms
    elem = 2 if args.values == "bf16" else 4
    flags = torch.zeros(1, dtype=torch.int32, device=device)

    def step(events=None):
        offsets = _C.segment_offsets_device(g.dst, n, flags)
        if events is not None:
            events[0].record()
        out = _C.segment_attention_forward(logit, value, offsets)
        if events is not None:
            events[1].record()
        return out

    for _ in range(args.warmup):
        step()
    torch.cuda.synchronize()
    pairs = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True))
             for _ in range(args.steps)]
    clocks = ClockSampler(device)
    clocks.start()
    dist.barrier()
    torch.cuda.synchronize()
    torch.cuda.profiler.start()  # ncu --profile-from-start off captures from here
    start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    start.record()
    for i in range(args.steps):
        step(pairs[i])
    end.record()
    torch.cuda.synchronize()
    torch.cuda.profiler.stop()
    dist.barrier()
    clock_info = clocks.stop()
    step_s = start.elapsed_time(end) / 1e3 / args.steps
    kernel_s = statistics.mean(a.elapsed_time(b) for a, b in pairs) / 1e3
    if int(flags.item()) != 0:
        raise RuntimeError(f"segment_offsets flagged the edge list: {int(flags.item())}")
    step_max = dist.max(step_s)
    edges_total = dist.sum(float(e))
    value_rate = edges_total / step_max

    # e2e through the public API from pinned host buffers
    e2e = None
    if not args.no_e2e:
        h_dst = g.dst.cpu().pin_memory()
        h_logit = logit.cpu().pin_memory()
        h_value = torch.empty(value.shape, dtype=value.dtype, pin_memory=True)
        h_value.copy_(value)
        h_out = torch.empty((n, 8, 16, 8), dtype=torch.float32, pin_memory=True)
        d_dst, d_logit, d_value = torch.empty_like(g.dst), torch.empty_like(logit), \
            torch.empty_like(value)
        del value  # keep one device copy of the 9 GB values
        torch.cuda.empty_cache()

        def e2e_step():
            d_dst.copy_(h_dst, non_blocking=True)
            d_logit.copy_(h_logit, non_blocking=True)
            d_value.copy_(h_value, non_blocking=True)
            offsets = K.segment_offsets(d_dst, n)
            out = K.segment_attention(d_logit, d_value, offsets)
            h_out.copy_(out, non_blocking=True)
            torch.cuda.current_stream().synchronize()

        e2e_step()
        k2 = max(2, min(args.steps, 5))
        dist.barrier()
        torch.cuda.synchronize()
        a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        a.record()
        for _ in range(k2):
            e2e_step()
        b.record()
        torch.cuda.synchronize()
        e2e_s = dist.max(a.elapsed_time(b) / 1e3 / k2)
        e2e = {"value": edges_total / e2e_s, "unit": UNIT,
               "h2d_bytes_per_step": int(h_dst.numel() * 8 + h_logit.numel() * 4
                                         + h_value.numel() * elem),
               "d2h_bytes_per_step": int(h_out.numel() * 4), "steps": k2,
               "ms_per_step": e2e_s * 1e3,
               "path": "bysj_b200.kernels.segment_offsets + segment_attention, pinned host "
                       "buffers, H2D + D2H inside the timed region"}
        value = d_value

    peak, peak_src = measured_peak()
    alg = attention_bytes(e, n, elem)
    achieved = alg / kernel_s / 1e9
    per_edge = profiled_traffic_per_edge("segment_attention_c3")
    roofline = {"bound": "hbm", "achieved": round(achieved, 1), "peak": peak, "unit": "GB/s",
                "frac": round(achieved / peak, 4),
                "traffic": (per_edge * e) if per_edge is not None else None,
                "kernel": "segment_attention_kernel", "alg_bytes_per_launch": int(alg),
                "kernel_ms": kernel_s * 1e3, "peak_source": peak_src}

    ops = cpu = None
    if dist.world == 1 and not args.no_ops and not args.profile_small:
        value32 = value if value.dtype == torch.float32 else value.float()
        torch.cuda.profiler.start()
        ops = measure_ops(g, logit, value32, device, peak)
        torch.cuda.profiler.stop()
    check = None
    if dist.rank == 0 and dist.world == 1 and not args.no_cpu and not args.profile_small:
        # the public API's output of the e2e steps (or one more device step)
        out_public = h_out if e2e is not None else step().cpu()
        cpu, check = cpu_frame_rate(g, logit, value, out_public)

    if dist.rank == 0:
        line = {
            "metric": METRIC, "value": value_rate, "unit": UNIT, "n_gpus": dist.world,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": step_max * 1e3,
            "higher_is_better": True, "scaling": "weak", "vs_baseline": None,
            "dtype": "f32" if args.values == "f32" else "bf16-in/f32-acc", "data": "synthetic",
            "config": c3_config(n, e, args.values, dist.world),
            "roofline": roofline,
            "cpu_baseline": cpu,
            "e2e": e2e,
            "clocks": clock_info,
            "gpu_launches": 2 * args.steps * dist.world,
        }
        if check is not None:
            line["check"] = check
        if ops:
            line["ops"] = ops
        return line
    return None


CHAIN_CHANNELS = 32


def chain_inputs(g, seed, device, channels=CHAIN_CHANNELS):
    """One C5 frame: the C3 geometry with C = 32 features for every operator
    of the chain (node features [N,16,C], per-degree weights [4,C], logits
    [E,8], values [E,16,C], zonal [E,15] from the unit vectors, radial
    [E,4,C], dE/dr [E,3])."""
    from bysj_b200 import workloads as W

    gen = torch.Generator(device=device).manual_seed(seed)
    n, e = g.n_atoms, g.n_edges
    return {
        "g": g, "n": n, "e": e,
        "x": torch.randn(n, 16, channels, device=device, generator=gen),
        "scale": torch.rand(4, channels, device=device, generator=gen) + 0.5,
        "logit": torch.randn(e, 8, device=device, generator=gen) * (2.0 ** 0.5),
        "value": torch.randn(e, 16, channels, device=device, generator=gen),
        "zonal": W.real_sph_zonal(g.unit).contiguous(),
        "radial": torch.randn(e, 4, channels, device=device, generator=gen),
        "slot": W.degree_slots().to(device),
        "inv": torch.rsqrt(torch.bincount(g.dst, minlength=n).float() + 1.0),
        "grad": torch.randn(e, 3, device=device, generator=gen) * 0.1,
    }


def chain_frame(f):
    """The full chain of one frame through the public API, as a user calls it:
    CSR of dst -> RMSNorm of the node features -> fused softmax + weighted sum
    -> GIE zonal scatter -> source grouping -> force assembly."""
    from bysj_b200 import kernels as K

    g = f["g"]
    offsets = K.segment_offsets(g.dst, f["n"])
    h = K.rmsnorm(f["x"], f["scale"], 1.0e-6)
    agg = K.segment_attention(f["logit"], f["value"], offsets)
    z = K.zonal_scatter(f["zonal"], f["radial"], g.dst, f["slot"], f["inv"], dst_offsets=offsets)
    order, soff = K.group_by_source(g.src, f["n"])
    force, virial = K.force_assembly(f["grad"], g.unit, g.src, g.dst, offsets, soff, order)
    return h, agg, z, force, virial


# The same calls in stages, for the two-stream pipeline of run_chain: the
# read-backs of the public API (the offsets flags, the grouping range flag)
# wait on their own stream only, so a frame's wait overlaps the other
# stream's kernels.  The GIE takes the frame's destination CSR from the
# offsets stage, so it reads nothing back.
def chain_offsets(f, st):
    from bysj_b200 import kernels as K

    st["offsets"] = K.segment_offsets(f["g"].dst, f["n"])


def chain_node_ops(f, st):
    from bysj_b200 import kernels as K

    st["h"] = K.rmsnorm(f["x"], f["scale"], 1.0e-6)
    st["agg"] = K.segment_attention(f["logit"], f["value"], st["offsets"])


def chain_zonal(f, st):
    from bysj_b200 import kernels as K

    g = f["g"]
    st["z"] = K.zonal_scatter(f["zonal"], f["radial"], g.dst, f["slot"], f["inv"],
                              dst_offsets=st["offsets"])


def chain_forces(f, st):
    from bysj_b200 import kernels as K

    g = f["g"]
    order, soff = K.group_by_source(g.src, f["n"])
    st["force"] = K.force_assembly(f["grad"], g.unit, g.src, g.dst, st["offsets"], soff, order)


def chain_pipelined(frames, streams):
    """Frames on alternating streams, their stages interleaved so that every
    host wait has the other stream's kernels queued: offsets and node
    operators of frame i, then the grouping and forces of frame i-1, then the
    GIE of frame i."""
    main = torch.cuda.current_stream()
    for s in streams:
        s.wait_stream(main)
    pending = None
    for i, f in enumerate(frames):
        s, st = streams[i % len(streams)], {}
        with torch.cuda.stream(s):
            chain_offsets(f, st)
            chain_node_ops(f, st)
        if pending is not None:
            with torch.cuda.stream(pending[0]):
                chain_forces(pending[1], pending[2])
        with torch.cuda.stream(s):
            chain_zonal(f, st)
        pending = (s, f, st)
    if pending is not None:
        with torch.cuda.stream(pending[0]):
            chain_forces(pending[1], pending[2])
    for s in streams:
        main.wait_stream(s)


def chain_bytes(e, n, c=CHAIN_CHANNELS):
    """Algorithmic bytes of one chain frame (each input read once, each output
    written once, per operator)."""
    offsets = 8 * e + 8 * (n + 1)
    rms = 2 * n * 16 * c * 4 + 4 * n * 16 + 4 * 4 * c
    attention = e * (8 * 4 + 16 * c * 4) + n * 16 * c * 4 + 8 * (n + 1)
    zonal = e * (15 * 4 + 8 + 3 * c * 4) + n * (16 * c * 4 + 4)
    group = 8 * e + 8 * e + 8 * (n + 1)
    force = e * (12 + 12 + 8) + n * (16 + 12 + 36)
    return offsets + rms + attention + zonal + group + force


def count_library_kernels(fn) -> int | None:
    """Kernels of this library (names in namespace bysj) that one call of `fn`
    launches, from a CUDA-activity profile of that call; None when the
    profiler is unavailable."""
    try:
        from torch.profiler import ProfilerActivity, profile

        with profile(activities=[ProfilerActivity.CUDA]) as prof:
            fn()
            torch.cuda.synchronize()
        return sum(1 for ev in prof.events()
                   if ev.device_type == torch.autograd.DeviceType.CUDA and "bysj" in ev.name)
    except Exception:  # noqa: BLE001 -- the count is a report, not a gate
        return None


def run_chain(args, dist):
    """C5(a): 64 independent 24576-atom frames of the full chain, fp32, C = 32,
    frames r, r + P, ... on rank r, no communication ("strong": the 64 frames
    are the fixed job).  Each rank holds two synthetic frames (two seeded
    geometries and feature sets) and its frames alternate between them; every
    frame's inputs (~5.9 GB) exceed L2, so a re-used frame is read from HBM
    like a new one."""
    from bysj_b200 import sharding as S
    from bysj_b200 import workloads as W

    device = torch.device("cuda", dist.local)
    torch.cuda.set_device(device)
    frames = S.frame_share(args.chain_frames, dist.rank, dist.world)
    sets = []
    for k in range(2):
        seed = args.seed + 1000 * dist.rank + 97 * k
        sets.append(chain_inputs(W.c3_box(device=device, seed=seed), seed + 5, device))

    streams = [torch.cuda.Stream(device=device) for _ in range(max(1, args.chain_streams))]

    def step():
        if len(streams) == 1:
            for i, _ in enumerate(frames):
                chain_frame(sets[i % 2])
        else:
            chain_pipelined([sets[i % 2] for i, _ in enumerate(frames)], streams)

    for _ in range(args.warmup):
        step()
    torch.cuda.synchronize()
    per_frame_kernels = count_library_kernels(lambda: chain_frame(sets[0]))
    clocks = ClockSampler(device)
    clocks.start()
    dist.barrier()
    torch.cuda.synchronize()
    start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    start.record()
    for _ in range(args.steps):
        step()
    end.record()
    torch.cuda.synchronize()
    dist.barrier()
    clock_info = clocks.stop()
    step_max = dist.max(start.elapsed_time(end) / 1e3 / args.steps)
    frames_total = args.chain_frames
    e_mean = sum(s["e"] for s in sets) / 2
    n = sets[0]["n"]
    peak, peak_src = measured_peak()
    # per-frame device time on the slowest rank: its frames run back to back
    frame_s = step_max / max(1, len(S.frame_share(frames_total, 0, dist.world)))
    achieved = chain_bytes(e_mean, n) / frame_s / 1e9
    if dist.rank == 0:
        line = {
            "metric": "frames/s (full fused chain, 24576-atom frames, fp32, C = 32)",
            "value": frames_total / step_max, "unit": "frames/s", "n_gpus": dist.world,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": step_max * 1e3,
            "higher_is_better": True, "scaling": "strong", "vs_baseline": None,
            "dtype": "f32", "data": "synthetic",
            "config": {"workload": "C5(a) 64 independent frames, full chain",
                       "chain": "segment_offsets -> rmsnorm -> segment_attention -> "
                                "zonal_scatter -> group_by_source -> force_assembly",
                       "frames_per_step": frames_total, "n_atoms": n,
                       "n_edges_per_frame": int(e_mean), "channels": CHAIN_CHANNELS,
                       "parallelism": f"frame-sharded x{dist.world} (no collective)",
                       "streams": (f"{len(streams)} CUDA streams per rank, consecutive "
                                   "frames alternating, their stages interleaved"
                                   if len(streams) > 1 else "one stream"),
                       "l2": "each frame's inputs (~5.9 GB) exceed L2; no flush"},
            "edges_per_s": frames_total * e_mean / step_max,
            "ms_per_frame": frame_s * 1e3,
            "roofline": {"bound": "hbm", "achieved": round(achieved, 1), "peak": peak,
                         "unit": "GB/s", "frac": round(achieved / peak, 4), "traffic": None,
                         "kernel": "whole chain: the sum of its operators' algorithmic bytes "
                                   "per frame over the frame's device time",
                         "peak_source": peak_src},
            "clocks": clock_info,
            "gpu_launches": (None if per_frame_kernels is None
                             else per_frame_kernels * frames_total * args.steps),
        }
        return line
    return None


def run_partition(args, dist):
    """One large box split by destination-atom ranges over the ranks ("strong").

    Per step and rank, the full chain of C5(b): ``force_assembly_src_partial``
    over the local edges (all atoms' source sums, written in the padded
    exchange layout), NCCL reduce-scatter of those partials (asynchronous, on
    NCCL's stream); meanwhile the local operators -- RMSNorm of the local
    atoms' node features [N_r, 16, 32], ``segment_attention`` over the local
    edges (values fp32 [E_r, 16, 32], logits [E_r, 8]) and the GIE zonal
    scatter of the local edges into the local atoms (radial [E_r, 4, 32]);
    then the wait and ``force_assembly_dst_add`` for the local atoms
    (dE/dr fp32 [E, 3]).
    """
    from bysj_b200 import _C
    from bysj_b200 import kernels as K
    from bysj_b200 import sharding as S
    from bysj_b200 import workloads as W

    device = torch.device("cuda", dist.local)
    torch.cuda.set_device(device)
    g = W.water_box(args.partition_atoms, density=0.1, seed=args.seed, device=device)
    n, e_total = g.n_atoms, g.n_edges
    offsets = K.segment_offsets(g.dst, n)
    part = S.make_partition(offsets, g.src, dist.rank, dist.world)
    e = part.n_edges
    gen = torch.Generator(device=device).manual_seed(args.seed + 31)
    grad_all = torch.randn(e_total, 3, device=device, generator=gen) * 0.1
    vec_all = g.edge_vec
    grad, vec = part.edges(grad_all).contiguous(), part.edges(vec_all).contiguous()
    gen.manual_seed(args.seed + 1000 * dist.rank + 37)
    logit = torch.randn(e, 8, device=device, generator=gen) * (2.0 ** 0.5)
    value = torch.randn(e, 16, 32, device=device, generator=gen)
    x_local = torch.randn(part.n_local, 16, 32, device=device, generator=gen)
    scale = torch.rand(4, 32, device=device, generator=gen) + 0.5
    zonal = W.real_sph_zonal(part.edges(g.unit).contiguous()).contiguous()
    radial = torch.randn(e, 4, 32, device=device, generator=gen)
    dst_local = (part.edges(g.dst) - part.atom_begin).contiguous()
    inv_local = torch.rsqrt(torch.bincount(dst_local, minlength=part.n_local).float() + 1.0)
    slot = W.degree_slots().to(device)
    ex = S.ForceExchange(part)

    def local_ops(events=None):
        h = K.rmsnorm(x_local, scale, 1.0e-6)
        if events is not None:
            events[0].record()
        out = _C.segment_attention_forward(logit, value, part.dst_offsets)
        if events is not None:
            events[1].record()
        z = K.zonal_scatter(zonal, radial, dst_local, slot, inv_local,
                            dst_offsets=part.dst_offsets)
        return h, out, z

    def step(events=None):
        ex.start(grad, vec)
        outs = local_ops(events)
        return outs, ex.finish()

    for _ in range(args.warmup):
        step()
    torch.cuda.synchronize()
    # this rank's kernels per step: the local operators (counted from a
    # profile of one call, no collective inside) + the two force kernels
    local_kernels = count_library_kernels(local_ops)
    launches = dist.sum(float(local_kernels + 2)) if local_kernels is not None else None
    pairs = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True))
             for _ in range(args.steps)]
    # one event after each step: this rank's step durations, to tell a uniform
    # slowdown from a few slow steps; the allocator's counters over the same
    # region show whether a step had to return cached blocks and map new ones
    marks = [torch.cuda.Event(enable_timing=True) for _ in range(args.steps)]
    clocks = ClockSampler(device)
    clocks.start()
    dist.barrier()
    torch.cuda.synchronize()
    stats0 = torch.cuda.memory_stats(device)
    start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    start.record()
    for i in range(args.steps):
        _, (force, virial) = step(pairs[i])
        marks[i].record()
    end.record()
    torch.cuda.synchronize()
    dist.barrier()
    clock_info = clocks.stop()
    stats1 = torch.cuda.memory_stats(device)
    free_b, total_b = torch.cuda.mem_get_info(device)
    step_max = dist.max(start.elapsed_time(end) / 1e3 / args.steps)
    kernel_s = statistics.mean(a.elapsed_time(b) for a, b in pairs) / 1e3
    step_ms = [a.elapsed_time(b) for a, b in zip([start] + marks[:-1], marks)]
    allocator = {key: int(stats1.get(key, 0) - stats0.get(key, 0))
                 for key in ("num_alloc_retries", "num_device_alloc", "num_device_free")}
    allocator.update(reserved_gb=round(torch.cuda.memory_reserved(device) / 1e9, 2),
                     free_gb=round(free_b / 1e9, 2), total_gb=round(total_b / 1e9, 2))

    # check: repeated steps give bit-identical forces (fixed reduction orders
    # on every rank and in the collective) ...
    force = force.clone()
    virial = virial.clone()
    _, (force2, virial2) = step()
    torch.cuda.synchronize()
    same = float(torch.equal(force, force2) and torch.equal(virial, virial2))
    repeat_same = dist.sum(same) == float(dist.world)
    del force2, virial2
    # the GIE was given the partition's destination CSR: the same output as
    # deriving it from dst_local (the public API's own path)
    z_given = local_ops()[2]
    z_derived = K.zonal_scatter(zonal, radial, dst_local, slot, inv_local)
    csr_same = dist.sum(float(torch.equal(z_given, z_derived))) == float(dist.world)
    del z_given, z_derived
    # ... and this rank's forces match the single-device assembly of the whole box
    order, soff = K.group_by_source(g.src, n)
    f_ref, v_ref = _C.force_assembly(grad_all, vec_all, offsets, soff, order)
    err = max(float((force - part.atoms(f_ref)).abs().max()) if part.n_local else 0.0,
              float((virial - part.atoms(v_ref)).abs().max()) if part.n_local else 0.0)
    err = dist.max(err)
    force_scale = float(f_ref.abs().max())
    del f_ref, v_ref, order, soff

    # what the overlapped step is made of: the force exchange (source partials,
    # reduce-scatter, destination sums) and the local operators, each timed
    # alone on the caller's stream (max over ranks; every rank runs both)
    def timed_alone(fn, reps=5):
        dist.barrier()
        torch.cuda.synchronize()
        a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        a.record()
        for _ in range(reps):
            fn()
        b.record()
        torch.cuda.synchronize()
        return dist.max(a.elapsed_time(b) / 1e3 / reps)

    def exchange_only():
        ex.start(grad, vec)
        ex.finish()

    exchange_s = timed_alone(exchange_only)
    local_s = timed_alone(local_ops)

    peak, peak_src = measured_peak()
    alg = e * (32 + 16 * 32 * 4) + part.n_local * 16 * 32 * 4 + 8 * (part.n_local + 1)
    achieved = alg / kernel_s / 1e9
    if dist.rank == 0:
        line = {
            "metric": f"edges/s (dst-partitioned {n}-atom box: full chain)",
            "value": e_total / step_max, "unit": UNIT, "n_gpus": dist.world,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": step_max * 1e3,
            "higher_is_better": True, "scaling": "strong", "vs_baseline": None,
            "dtype": "f32", "data": "synthetic",
            "config": {"workload": "C5(b) one box, dst-range partition",
                       "n_atoms": n, "n_edges": e_total, "edges_rank0": e,
                       "atoms_rank0": part.n_local, "heads": 8, "components": 16,
                       "channels": 32, "exchange_rows": part.world * part.chunk,
                       "chain": "rmsnorm -> segment_attention -> zonal_scatter (local); "
                                "force_assembly (source partials reduce-scattered)",
                       "parallelism": f"dst-range partition x{dist.world}, NCCL reduce-scatter "
                                      "of [N, 12] force partials overlapped with the local "
                                      "operators",
                       "l2": "inputs larger than L2; no flush"},
            "roofline": {"bound": "hbm", "achieved": round(achieved, 1), "peak": peak,
                         "unit": "GB/s", "frac": round(achieved / peak, 4), "traffic": None,
                         "kernel": "segment_attention_kernel (rank 0)",
                         "kernel_ms": kernel_s * 1e3, "peak_source": peak_src},
            "check": {"max_abs_err_vs_single_device": err, "max_abs_force": force_scale,
                      "bit_identical_repeat": repeat_same,
                      "zonal_given_csr_equal": csr_same,
                      "exchange": "float64 source partials, NCCL reduce-scatter (sum)",
                      "nccl_algo": os.environ.get("NCCL_ALGO", "default"),
                      "nccl_proto": os.environ.get("NCCL_PROTO", "default")},
            "breakdown": {"exchange_ms": exchange_s * 1e3, "local_ms": local_s * 1e3,
                          "note": "each part timed alone (max over ranks); the timed step "
                                  "overlaps the exchange with the local operators"},
            "steps_rank0_ms": {"min": round(min(step_ms), 3),
                               "median": round(statistics.median(step_ms), 3),
                               "max": round(max(step_ms), 3),
                               "each": [round(t, 2) for t in step_ms]},
            "allocator_rank0": allocator,
            "clocks": clock_info,
            "gpu_launches": None if launches is None else int(launches) * args.steps,
        }
        return line
    return None


def run_only(args):
    """One operator on a box of ``--atoms`` atoms (profiling / tuning aid)."""
    from bysj_b200 import workloads as W

    device = torch.device("cuda", 0)
    torch.cuda.set_device(device)
    g = W.water_box(args.atoms, density=0.1, seed=args.seed, device=device)
    peak, _ = measured_peak()
    torch.cuda.synchronize()
    torch.cuda.profiler.start()
    ops = measure_ops(g, None, None, device, peak, iters=max(args.steps, 1), only=args.only)
    torch.cuda.profiler.stop()
    print(json.dumps({"only": args.only, "atoms": g.n_atoms, "edges": g.n_edges, "ops": ops}),
          flush=True)


def extra_args(args):
    """Arguments of the chain and partition lines that the default run adds:
    the same job, at most 10 timed steps after 3-5 warm-up steps."""
    extra = argparse.Namespace(**vars(args))
    extra.steps = max(1, min(args.steps, 10))
    extra.warmup = max(3, min(args.warmup, 5))
    return extra


def main():
    args = parse_args()
    dist = Dist()
    if args.impl == "reference":
        run_reference(args, dist)
        return
    # No automatic garbage collection while measuring (as timeit does): a
    # full collection pauses the host for tens of ms, and a step whose host
    # waits on the device once per step (a public-API read-back) turns that
    # pause into device idle time.  Collected explicitly between lines.
    gc.disable()
    if args.only:
        run_only(args)
        return
    dist.setup("nccl")
    try:
        if args.mode == "frames":
            line = run_ours(args, dist)
            if not args.no_extra and not args.profile_small:
                # the two other multi-GPU workloads (the 64-frame chain and the
                # partitioned box), same ranks, same collective order on every
                # rank; their own timings and checks.
                # They run after the headline and the per-op lines, which are
                # measured on a fresh allocator: run first, the partition's
                # ~130 GB left the op lines measurably slower later in the
                # same process (the GIE forward 345 -> 357 us).
                gc.collect()
                torch.cuda.empty_cache()
                chain = run_chain(extra_args(args), dist)
                gc.collect()
                torch.cuda.empty_cache()
                part = run_partition(extra_args(args), dist)
                if line is not None:
                    line["chain"] = chain
                    line["partition"] = part
        else:
            line = {"partition": run_partition, "chain": run_chain}[args.mode](args, dist)
        if line is not None:
            print(json.dumps(line), flush=True)
    finally:
        dist.close()


if __name__ == "__main__":
    main()
