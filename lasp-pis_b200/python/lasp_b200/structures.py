"""Seeded synthetic structures for the benchmark configurations, and ARC I/O.

C1  64-atom simple-cubic cell (a = 9 A), species {H, C, N, O}
C2  1,000-atom triclinic cell, Poisson-disk positions, 10 species with p ~ 1/Z
C3  10,000-atom perturbed FCC cube (46.4 A), 10 species uniform
C4  a batch of independent triclinic cells of 32..256 atoms (species Z = 1..20)
C5  ~200,000-atom perturbed BCC Fe/Ni/Cr slab (125 x 125 x 128 A)

Positions and cells are rounded to float32, the precision the C ABI takes.  Every
generator re-jitters atoms that have a pair distance within 1e-4 A of the 6 A cutoff, so
that float32 and float64 neighbour enumerations agree (the reference's boundary-band
policy, lapis/docs/PAIR_OP.md:76-82).  No public dataset is involved.

The ARC writer/reader follow the BIOSYM/LASP layout the reference parses
(chemio/src/arc.cpp:35-93): ``PBC=ON``, a title line, ``PBC a b c alpha beta gamma``, one
``El x y z CORE ...`` line per atom and a double ``end`` per frame.
"""
from __future__ import annotations

import math
from dataclasses import dataclass
from pathlib import Path

import numpy as np
from scipy.spatial import cKDTree

CUTOFF = 6.0
BAND = 1e-4
TEN = (1, 3, 6, 7, 8, 11, 12, 14, 16, 26)
SYMBOLS = ("X H He Li Be B C N O F Ne Na Mg Al Si P S Cl Ar K Ca Sc Ti V Cr Mn Fe Co Ni Cu Zn Ga Ge "
           "As Se Br Kr Rb Sr Y Zr Nb Mo Tc Ru Rh Pd Ag Cd In Sn Sb Te I Xe Cs Ba La Ce Pr Nd Pm Sm "
           "Eu Gd Tb Dy Ho Er Tm Yb Lu Hf Ta W Re Os Ir Pt Au Hg Tl Pb Bi Po At Rn Fr Ra Ac Th Pa U "
           "Np Pu Am Cm Bk Cf Es Fm Md No Lr Rf Db Sg Bh Hs Mt Ds Rg Cn Nh Fl Mc Lv Ts Og").split()


@dataclass
class Structure:
    positions: np.ndarray   # float32 [n, 3], Angstrom
    numbers: np.ndarray     # int32 [n]
    cell: np.ndarray        # float32 [3, 3], lattice vectors are rows

    @property
    def size(self) -> int:
        return int(self.numbers.size)


def _pairs_within(frac, cell, r):
    """All periodic pairs (i, j, distance) with distance <= r (brute over 27 images)."""
    pos = frac @ cell
    out_i, out_j, out_d = [], [], []
    tree = cKDTree(pos)
    shifts = np.array(np.meshgrid(*[(-1, 0, 1)] * 3, indexing="ij")).reshape(3, -1).T
    for s in shifts:
        other = cKDTree(pos + s @ cell)
        pairs = tree.sparse_distance_matrix(other, r, output_type="coo_matrix")
        keep = ~((pairs.row == pairs.col) & (not s.any()))
        out_i.append(pairs.row[keep])
        out_j.append(pairs.col[keep])
        out_d.append(pairs.data[keep])
    return np.concatenate(out_i), np.concatenate(out_j), np.concatenate(out_d)


def _finish(frac, numbers, cell, rng, dmin, max_rounds=50):
    """Round to float32; nudge atoms (0.01 A) inside the cutoff band or closer than dmin."""
    cell32 = cell.astype(np.float32)
    cell64 = cell32.astype(np.float64)
    for _ in range(max_rounds):
        pos32 = (frac @ cell64).astype(np.float32)
        f = pos32.astype(np.float64) @ np.linalg.inv(cell64)
        i, j, d = _pairs_within(f - np.floor(f), cell64, CUTOFF + 2 * BAND)
        bad = (np.abs(d - CUTOFF) <= BAND) | (d < dmin - 0.05)
        if not bad.any():
            return Structure(pos32, numbers.astype(np.int32), cell32)
        move = np.unique(np.concatenate([i[bad], j[bad]]))
        frac[move] += rng.normal(scale=0.01, size=(move.size, 3)) @ np.linalg.inv(cell64)
    raise RuntimeError("could not place atoms outside the cutoff band")


def _poisson(rng, cell, n, dmin):
    """Periodic random sequential placement with minimum separation dmin."""
    inv = np.linalg.inv(cell)
    heights = 1.0 / np.linalg.norm(inv, axis=0)
    grid = np.maximum(1, np.floor(heights / dmin).astype(int))
    bins: dict[tuple, list] = {}
    pts = []
    shifts = np.array(np.meshgrid(*[(-1, 0, 1)] * 3, indexing="ij")).reshape(3, -1).T
    tries = 0
    while len(pts) < n:
        tries += 1
        if tries > 400 * n:
            raise RuntimeError("Poisson-disk placement failed")
        f = rng.random(3)
        b = tuple((f * grid).astype(int) % grid)
        ok = True
        for s in shifts:
            nb = tuple((np.array(b) + s) % grid)
            for g in bins.get(nb, ()):
                df = f - pts[g]
                df -= np.round(df)
                if np.linalg.norm(df @ cell) < dmin:
                    ok = False
                    break
            if not ok:
                break
        if ok:
            bins.setdefault(b, []).append(len(pts))
            pts.append(f)
    return np.array(pts)


def c1(seed=101):
    rng = np.random.default_rng(seed)
    cell = np.eye(3) * 9.0
    g = (np.stack(np.meshgrid(*[np.arange(4)] * 3, indexing="ij"), -1).reshape(-1, 3) + 0.5) / 4
    frac = g + rng.normal(scale=0.1, size=g.shape) / 9.0
    z = rng.choice([1, 6, 7, 8], size=64)
    return _finish(frac, z, cell, rng, 1.6)


def c2(seed=102):
    rng = np.random.default_rng(seed)
    cell = np.array([[22.0, 0, 0], [6, 21, 0], [4, 5, 20]])
    frac = _poisson(rng, cell, 1000, 1.8)
    p = 1.0 / np.array(TEN)
    z = rng.choice(TEN, size=1000, p=p / p.sum())
    return _finish(frac, z, cell, rng, 1.8)


def c3(seed=103):
    rng = np.random.default_rng(seed)
    side = 46.4
    base = np.array([[0, 0, 0], [0.5, 0.5, 0], [0.5, 0, 0.5], [0, 0.5, 0.5]])
    cells = np.stack(np.meshgrid(*[np.arange(14)] * 3, indexing="ij"), -1).reshape(-1, 1, 3)
    sites = ((cells + base).reshape(-1, 3)) / 14.0
    sites = sites[rng.choice(len(sites), size=10000, replace=False)]
    frac = sites + rng.normal(scale=0.15, size=sites.shape) / side
    z = rng.choice(TEN, size=10000)
    return _finish(frac, z, np.eye(3) * side, rng, 0.5)


def c5(seed=105):
    rng = np.random.default_rng(seed)
    dims = np.array([46, 46, 47])
    lengths = np.array([125.0, 125.0, 128.0])
    base = np.array([[0, 0, 0], [0.5, 0.5, 0.5]])
    cells = np.stack(np.meshgrid(*[np.arange(d) for d in dims], indexing="ij"), -1).reshape(-1, 1, 3)
    sites = (cells + base).reshape(-1, 3) / dims
    frac = sites + rng.normal(scale=0.1, size=sites.shape) / lengths
    z = rng.choice([26, 28, 24], size=len(sites), p=[0.7, 0.2, 0.1])
    return _finish(frac, z, np.diag(lengths), rng, 0.5)


def random_cell(rng, n, volume_per_atom=12.0):
    """Random triclinic cell of the given volume whose plane heights exceed the cutoff."""
    vol = volume_per_atom * n
    for _ in range(1000):
        lengths = rng.uniform(0.8, 1.25, 3)
        angles = np.radians(rng.uniform(70, 110, 3))
        h = cell_from_parameters(*lengths, *np.degrees(angles))
        h *= (vol / abs(np.linalg.det(h))) ** (1 / 3)
        heights = 1.0 / np.linalg.norm(np.linalg.inv(h), axis=0)
        if heights.min() > CUTOFF + 0.05:
            return h
    return np.eye(3) * vol ** (1 / 3)


def c4_cell(index, seed=104):
    """Cell ``index`` of the C4 batch: N ~ U{32..256}, Z ~ U{1..20}, d_min 1.7 A."""
    rng = np.random.default_rng([seed, index])
    n = int(rng.integers(32, 257))
    cell = random_cell(rng, n)
    frac = _poisson(rng, cell, n, 1.7)
    z = rng.integers(1, 21, size=n)
    return _finish(frac, z, cell, rng, 1.7)


def cell_from_parameters(a, b, c, alpha, beta, gamma):
    """Lattice rows from lengths and angles (degrees): a along x, b in the xy plane."""
    rad = math.pi / 180
    ca, cb, cg, sg = math.cos(alpha * rad), math.cos(beta * rad), math.cos(gamma * rad), math.sin(gamma * rad)
    cx = c * cb
    cy = c * (ca - cb * cg) / sg
    return np.array([[a, 0, 0], [b * cg, b * sg, 0], [cx, cy, math.sqrt(c * c - cx * cx - cy * cy)]])


def parameters(cell):
    cell = np.asarray(cell, np.float64)
    la = np.linalg.norm(cell, axis=1)

    def ang(i, j):
        return math.degrees(math.acos(float(cell[i] @ cell[j] / (la[i] * la[j]))))
    return (*la, ang(1, 2), ang(0, 2), ang(0, 1))


def write_arc(path, frames, title="synthetic"):
    lines = ["!BIOSYM archive 2", "PBC=ON"]
    for s in frames:
        lines += [f"{title} {s.size}", "!DATE"]
        lines.append("PBC " + " ".join(f"{x:.10f}" for x in parameters(s.cell)))
        for k, (z, p) in enumerate(zip(s.numbers, s.positions.astype(np.float64))):
            lines.append(f"{SYMBOLS[z]} {p[0]:.9f} {p[1]:.9f} {p[2]:.9f} CORE {k + 1} X X 0 {k + 1}")
        lines += ["end", "end"]
    Path(path).write_text("\n".join(lines) + "\n")


GENERATORS = {"C1": c1, "C2": c2, "C3": c3, "C5": c5}


def load(name: str, cache_dir: str | Path) -> Structure:
    """Generate (or load the cached) seeded structure for config C1/C2/C3/C5."""
    cache = Path(cache_dir) / f"{name}.npz"
    if cache.exists():
        d = np.load(cache)
        return Structure(d["positions"], d["numbers"], d["cell"])
    s = GENERATORS[name]()
    cache.parent.mkdir(parents=True, exist_ok=True)
    np.savez(cache, positions=s.positions, numbers=s.numbers, cell=s.cell)
    return s


def _c4_arrays(index):
    s = c4_cell(index)
    return s.positions, s.numbers, s.cell


def load_c4(cache_dir: str | Path, count: int = 4096, workers: int | None = None) -> list[Structure]:
    """The C4 batch (cells 0..count-1 of c4_cell), generated in a spawn-context process pool
    (CPU only) and cached as C4_<count>.npz."""
    cache = Path(cache_dir) / f"C4_{count}.npz"
    if cache.exists():
        d = np.load(cache)
        off = d["offsets"]
        return [Structure(d["positions"][off[k]:off[k + 1]], d["numbers"][off[k]:off[k + 1]], d["cells"][k])
                for k in range(count)]
    import multiprocessing as mp
    import os
    with mp.get_context("spawn").Pool(workers or os.cpu_count() or 1) as pool:
        parts = pool.map(_c4_arrays, range(count), chunksize=16)
    cells = [Structure(p, z, c) for p, z, c in parts]
    offsets = np.concatenate([[0], np.cumsum([c.size for c in cells])])
    cache.parent.mkdir(parents=True, exist_ok=True)
    np.savez(cache, positions=np.concatenate([c.positions for c in cells]),
             numbers=np.concatenate([c.numbers for c in cells]), cells=np.stack([c.cell for c in cells]),
             offsets=offsets)
    return cells


def density_sample(n_atoms: int, seed: int = 203) -> Structure:
    """A smaller cube cut from the C3 process (same density, lattice, jitter, species)."""
    rng = np.random.default_rng(seed)
    m = max(2, round((n_atoms / 4 / (10000 / 10976)) ** (1 / 3)))
    side = 46.4 / 14 * m
    base = np.array([[0, 0, 0], [0.5, 0.5, 0], [0.5, 0, 0.5], [0, 0.5, 0.5]])
    cells = np.stack(np.meshgrid(*[np.arange(m)] * 3, indexing="ij"), -1).reshape(-1, 1, 3)
    sites = ((cells + base).reshape(-1, 3)) / m
    sites = sites[rng.choice(len(sites), size=min(n_atoms, len(sites)), replace=False)]
    frac = sites + rng.normal(scale=0.15, size=sites.shape) / side
    z = rng.choice(TEN, size=len(sites))
    return _finish(frac, z, np.eye(3) * side, rng, 0.5)
