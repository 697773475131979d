"""Seeded synthetic water-like systems and their neighbour lists.

The reference measures on a 3000-atom water box that DeepMD builds neighbour
lists for; DeepMD is not part of this slice, so benchmarks and tests use
synthetic stand-ins with the same statistics: atoms placed uniformly at random
(from a seed) in a cubic periodic box at a chosen number density, types
O:H = 1:2, and every directed pair (i != j) closer than ``rcut`` under the
minimum-image convention.  Edges are sorted by destination, then source, so
the list is in the CSR layout the segmented operators expect.

``edge_vec = r[src] - r[dst]`` (minimum image), ``unit = edge_vec / |edge_vec|``.
Building uses a cell list on whichever device is given (a GPU makes the
2.2 M-edge and 45 M-edge systems take seconds).

Atom numbering: by default atoms are renumbered in Morton (z-curve) order of
their position, the way MD engines keep atoms spatially sorted for cache
locality (LAMMPS re-bins atoms periodically); a node's neighbours then have
nearby indices.  ``spatial_sort=False`` keeps the random draw order, the worst
case for operators that gather rows by source atom.
"""
from __future__ import annotations

import math
from dataclasses import dataclass

import torch


@dataclass
class Graph:
    n_atoms: int
    box: float
    pos: torch.Tensor       # [N, 3] float64
    types: torch.Tensor     # [N] int64 (0 = O, 1 = H)
    src: torch.Tensor       # [E] int64
    dst: torch.Tensor       # [E] int64, non-decreasing
    edge_vec: torch.Tensor  # [E, 3] float32
    unit: torch.Tensor      # [E, 3] float32

    @property
    def n_edges(self) -> int:
        return int(self.dst.numel())


def box_length(n_atoms: int, density: float) -> float:
    return (n_atoms / density) ** (1.0 / 3.0)


def _pairs_bruteforce(pos: torch.Tensor, box: float, rcut: float):
    n = pos.shape[0]
    d = pos[None, :, :] - pos[:, None, :]          # d[i, j] = r_j - r_i
    d = d - box * torch.round(d / box)
    r2 = (d * d).sum(-1)
    mask = (r2 < rcut * rcut) & ~torch.eye(n, dtype=torch.bool, device=pos.device)
    dst, src = mask.nonzero(as_tuple=True)         # edge: src -> dst
    return dst, src


def _pairs_cells(pos: torch.Tensor, box: float, rcut: float):
    n = pos.shape[0]
    device = pos.device
    cells = int(math.floor(box / rcut))
    cell_len = box / cells
    cidx = torch.clamp((pos / cell_len).floor().long(), 0, cells - 1)
    flat = (cidx[:, 0] * cells + cidx[:, 1]) * cells + cidx[:, 2]
    order = torch.argsort(flat, stable=True)
    counts = torch.bincount(flat, minlength=cells ** 3)
    width = int(counts.max())
    starts = torch.zeros(cells ** 3 + 1, dtype=torch.long, device=device)
    starts[1:] = torch.cumsum(counts, 0)
    sorted_flat = flat[order]
    rank = torch.arange(n, device=device) - starts[sorted_flat]
    table = torch.full((cells ** 3, width), -1, dtype=torch.long, device=device)
    table[sorted_flat, rank] = order
    grid = torch.arange(cells, device=device)
    cx, cy, cz = torch.meshgrid(grid, grid, grid, indexing="ij")
    cx, cy, cz = cx.reshape(-1), cy.reshape(-1), cz.reshape(-1)
    dsts, srcs = [], []
    for ox in (-1, 0, 1):
        for oy in (-1, 0, 1):
            for oz in (-1, 0, 1):
                nb = (((cx + ox) % cells) * cells + (cy + oy) % cells) * cells + (cz + oz) % cells
                a = table[:, :, None].expand(-1, width, width)      # dst candidates
                b = table[nb][:, None, :].expand(-1, width, width)  # src candidates
                ok = (a >= 0) & (b >= 0) & (a != b)
                ai, bi = a[ok], b[ok]
                d = pos[bi] - pos[ai]
                d = d - box * torch.round(d / box)
                keep = (d * d).sum(-1) < rcut * rcut
                dsts.append(ai[keep])
                srcs.append(bi[keep])
    return torch.cat(dsts), torch.cat(srcs)


def _morton_order(pos: torch.Tensor, box: float, bits: int = 10) -> torch.Tensor:
    """Permutation sorting positions along a 3-D z-curve of 2^bits bins per axis."""
    bins = 1 << bits
    cell = torch.clamp((pos / box * bins).floor().long(), 0, bins - 1)
    code = torch.zeros(pos.shape[0], dtype=torch.long, device=pos.device)
    for b in range(bits):
        for axis in range(3):
            code |= ((cell[:, axis] >> b) & 1) << (3 * b + axis)
    return torch.argsort(code, stable=True)


def water_box(n_atoms: int, *, density: float = 0.1, box: float | None = None,
              rcut: float = 6.0, seed: int = 0, device: str | torch.device = "cpu",
              spatial_sort: bool = True) -> Graph:
    """Uniform random water-like box and its dst-sorted directed neighbour list."""
    length = float(box) if box is not None else box_length(n_atoms, density)
    if length < 2.0 * rcut:
        raise ValueError("the minimum-image convention needs box >= 2 * rcut")
    gen = torch.Generator().manual_seed(seed)
    pos = torch.rand(n_atoms, 3, generator=gen, dtype=torch.float64) * length
    if spatial_sort:
        pos = pos[_morton_order(pos, length)].contiguous()
    pos = pos.to(device)
    types = (torch.arange(n_atoms) % 3 != 0).long().to(device)
    if math.floor(length / rcut) >= 3:
        dst, src = _pairs_cells(pos, length, rcut)
    else:
        dst, src = _pairs_bruteforce(pos, length, rcut)
    key = dst * n_atoms + src
    perm = torch.argsort(key)
    dst, src = dst[perm].contiguous(), src[perm].contiguous()
    vec = pos[src] - pos[dst]
    vec = vec - length * torch.round(vec / length)
    unit = vec / vec.norm(dim=-1, keepdim=True)
    return Graph(n_atoms, length, pos, types, src, dst,
                 vec.to(torch.float32).contiguous(), unit.to(torch.float32).contiguous())


def c1_box(device="cpu", seed: int = 0) -> Graph:
    """Plumbing configuration: 192 atoms in a 12.4 A box, rcut 6 A (~17k edges)."""
    return water_box(192, box=12.4, seed=seed, device=device)


def c3_box(device="cpu", seed: int = 0, spatial_sort: bool = True) -> Graph:
    """Headline geometry: 24576 atoms at 0.1 / A^3 (L ~ 62.65 A), ~2.2 M edges."""
    return water_box(24576, density=0.1, seed=seed, device=device, spatial_sort=spatial_sort)


def real_sph_zonal(unit: torch.Tensor, lmax: int = 3) -> torch.Tensor:
    """Per-row geometric coupling for the GIE scatter: [E, (lmax+1)^2 - 1].

    Real spherical harmonics of the edge direction evaluated by the standard
    associated-Legendre recurrences (unnormalised), rows l = 1..lmax,
    m = -l..l.  Any deterministic function of the direction serves the
    operator (it takes the coefficients as input); this one has the right
    shape and smoothness.
    """
    x, y, z = unit[:, 0].double(), unit[:, 1].double(), unit[:, 2].double()
    rows = []
    for l in range(1, lmax + 1):
        for m in range(-l, l + 1):
            am = abs(m)
            # P_l^{|m|}(z) via the recurrence in l at fixed m.
            pmm = torch.ones_like(z)
            somx2 = torch.sqrt(torch.clamp(1.0 - z * z, min=0.0))
            fact = 1.0
            for _ in range(am):
                pmm = -pmm * fact * somx2
                fact += 2.0
            if l == am:
                plm = pmm
            else:
                pmmp1 = z * (2 * am + 1) * pmm
                if l == am + 1:
                    plm = pmmp1
                else:
                    for ll in range(am + 2, l + 1):
                        pll = (z * (2 * ll - 1) * pmmp1 - (ll + am - 1) * pmm) / (ll - am)
                        pmm, pmmp1 = pmmp1, pll
                    plm = pmmp1
            phi = torch.atan2(y, x)
            if m > 0:
                rows.append(plm * torch.cos(m * phi))
            elif m < 0:
                rows.append(plm * torch.sin(am * phi))
            else:
                rows.append(plm)
    return torch.stack(rows, dim=1).to(torch.float32).contiguous()


def degree_slots(lmax: int = 3, zero_based: bool = False) -> torch.Tensor:
    """``radial_slot[r] = l(r+1)`` (or ``l - 1``) for rows r = 0..(lmax+1)^2-2."""
    comps = (lmax + 1) ** 2
    levels = [int(math.isqrt(i)) for i in range(1, comps)]
    return torch.tensor([l - 1 if zero_based else l for l in levels], dtype=torch.int64)


__all__ = ["Graph", "box_length", "c1_box", "c3_box", "degree_slots", "real_sph_zonal",
           "water_box"]
