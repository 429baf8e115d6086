"""Seeded synthetic MH1-shaped model archive (random weights, real MH1 shapes).

The shapes are the ones the reference loader enforces (mace/src/mh1.cu:672-734): 512-wide
species embedding, 128-channel messages, 9728-wide pre-gate node features, 8192-wide
gated features, 2 interaction layers with 4 / 10 tensor-product paths, correlation-3
products, 10 Bessel functions, radial MLP 10->64->64->64 with LayerNorm+SiLU, ZBL and the
Agnesi distance transform.  Irrep ordering follows MACE's ``tp_out_irreps_with_instructions``
followed by ``Irreps.sort()`` (instructions in (input irrep, harmonic, output) order,
output blocks sorted by (l, parity)), and the coupling values are real 3j symbols times a
path weight, like mace/src/weights.cpp:200-240.  Product terms are symmetrised sparse cubic
polynomials extracted like mace/src/weights.cpp:241-303, built from equivariant 3j
contractions so that the model is rotation invariant.
"""
from __future__ import annotations

import itertools
import json
from pathlib import Path

import numpy as np

from . import archive, so3

SEED = 20261201
SPECIES = tuple(range(1, 31))
PARITY = {0: 1, 1: -1, 2: 1, 3: -1}          # hidden irreps are 0e, 1o, 2e, 3o


def _irreps_offsets(irreps):
    """irreps: list of (mul, l) -> list of (mul, l, offset, component)."""
    out, off, comp = [], 0, 0
    for mul, l in irreps:
        out.append((mul, l, off, comp))
        off += mul * (2 * l + 1)
        comp += 2 * l + 1
    return out


def _linear(rng, ins, outs, scale=1.0):
    """Equivariant linear: one path per (input block, output block) with equal l."""
    ib, ob = _irreps_offsets(ins), _irreps_offsets(outs)
    fan = {}
    for mi, li, _, _ in ib:
        for j, (mo, lo, _, _) in enumerate(ob):
            if li == lo:
                fan[j] = fan.get(j, 0) + mi
    paths, weights = [], []
    for mi, li, oi, _ in ib:
        for j, (mo, lo, oo, _) in enumerate(ob):
            if li != lo:
                continue
            w = rng.normal(size=(mi, mo)) * scale / np.sqrt(fan[j])
            paths += [oi, oo, mi, mo, 2 * li + 1, sum(x.size for x in weights)]
            weights.append(w.ravel())
    dims = [ib[-1][2] + ib[-1][0] * (2 * ib[-1][1] + 1), ob[-1][2] + ob[-1][0] * (2 * ob[-1][1] + 1)]
    return {"dims": np.array(dims), "paths": np.array(paths), "weight": np.concatenate(weights)}


def _radial(rng, species, depth, outputs):
    r = {
        "source": rng.normal(size=(species, 64)) * 0.5,
        "target": rng.normal(size=(species, 64)) * 0.5,
        "radial": rng.normal(size=(64, 10)) / np.sqrt(10),
        "0.weight": rng.normal(size=(64, 1034)) / np.sqrt(1034),
    }
    for k in range(depth):
        if k:
            r[f"{3 * k}.weight"] = rng.normal(size=(64, 64)) / 8.0
        r[f"{3 * k}.bias"] = rng.normal(size=64) * 0.1
        r[f"{3 * k + 1}.weight"] = 1.0 + rng.normal(size=64) * 0.1
        r[f"{3 * k + 1}.bias"] = rng.normal(size=64) * 0.1
    r[f"{3 * depth}.weight"] = rng.normal(size=(outputs, 64)) / 8.0
    r[f"{3 * depth}.bias"] = rng.normal(size=outputs) * 0.1
    return r


def tp_layout(layer: int):
    """Paths (l_in, l_sh, l_out) in instruction order, output blocks sorted (MACE)."""
    ins = [0] if layer == 0 else [0, 1]
    paths = []
    for li in ins:
        for ls in range(4):
            for lo in range(abs(li - ls), li + ls + 1):
                if lo <= 3 and PARITY[li] * PARITY[ls] == PARITY[lo]:
                    paths.append((li, ls, lo))
    order = sorted(range(len(paths)), key=lambda k: (paths[k][2], k))
    comp, out_start = 0, {}
    for k in order:
        out_start[k] = comp
        comp += 2 * paths[k][2] + 1
    in_start = {0: 0, 1: 1}
    return paths, out_start, in_start, comp


def _tensor_product(layer: int):
    paths, out_start, in_start, ncomp = tp_layout(layer)
    terms, values = [], []
    for p, (li, ls, lo) in enumerate(paths):
        c = so3.wigner_3j(li, ls, lo)
        weight = np.float32(np.sqrt((2 * lo + 1) / (1 + layer)))
        for a, b, cc in itertools.product(*(range(n) for n in c.shape)):
            if abs(c[a, b, cc]) > 1e-14:
                terms.append([p, in_start[li] + a, ls * ls + b, out_start[p] + cc])
                values.append(np.float32(c[a, b, cc]) * weight)
    return {"dims": np.array([len(paths), 1 if layer == 0 else 4, ncomp]),
            "terms": np.array(terms).ravel(), "values": np.array(values, np.float32)}


def _block(l):
    return range(l * l, (l + 1) * (l + 1))


def _coupling_paths(out_l):
    """Ordered coupling tensors over the 16 product-input components per degree."""
    paths = {1: [], 2: [], 3: []}
    nout = 2 * out_l + 1
    t = np.zeros((nout, 16))
    for m in range(nout):
        t[m, out_l * out_l + m] = 1
    paths[1].append(t)
    for l1 in range(4):
        for l2 in range(l1, 4):
            if PARITY[l1] * PARITY[l2] != PARITY[out_l]:
                continue
            c = so3.wigner_3j(l1, l2, out_l)
            if not c.any():
                continue
            t = np.zeros((nout, 16, 16))
            for a, b, m in itertools.product(range(2 * l1 + 1), range(2 * l2 + 1), range(nout)):
                t[m, l1 * l1 + a, l2 * l2 + b] = c[a, b, m]
            paths[2].append(t)
    for l1 in range(4):
        for l2 in range(l1, 4):
            for big in range(abs(l1 - l2), min(3, l1 + l2) + 1):
                for l3 in range(4):
                    if PARITY[l1] * PARITY[l2] * PARITY[l3] != PARITY[out_l]:
                        continue
                    c1, c2 = so3.wigner_3j(l1, l2, big), so3.wigner_3j(big, l3, out_l)
                    if not (c1.any() and c2.any()):
                        continue
                    inner = np.einsum("abM,Mcm->mabc", c1, c2)
                    t = np.zeros((nout, 16, 16, 16))
                    t[:, l1 * l1:(l1 + 1) ** 2, l2 * l2:(l2 + 1) ** 2, l3 * l3:(l3 + 1) ** 2] = inner
                    paths[3].append(t)
    return paths


def _polynomial(rng, layer):
    """Symmetric-contraction terms {out, degree, a, b, c} and per-channel coefficients."""
    terms, coefficients = [], []
    contractions = [(0, 0)] if layer else [(0, 0), (1, 1)]      # (output l, output offset)
    for out_l, out_offset in contractions:
        paths = _coupling_paths(out_l)
        for degree in (1, 2, 3):
            ts = paths[degree]
            w = rng.normal(size=(len(ts), 512)) / np.sqrt(len(ts)) * (1.0, 0.3, 0.05)[degree - 1]
            for m in range(2 * out_l + 1):
                for idx in itertools.combinations_with_replacement(range(16), degree):
                    coupling = np.zeros(len(ts))
                    for perm in set(itertools.permutations(idx)):
                        coupling += np.array([t[(m,) + perm] for t in ts])
                    coupling[np.abs(coupling) < 1e-12] = 0
                    if not coupling.any():
                        continue
                    coeff = coupling @ w
                    if np.abs(coeff).max() < 1e-12:
                        continue
                    full = list(idx) + [-1] * (3 - degree)
                    terms.append([out_offset + m, degree] + full)
                    coefficients.append(coeff)
    return {"terms": np.array(terms).ravel(), "coefficients": np.concatenate(coefficients)}


def make_records(seed: int = SEED, species=SPECIES) -> dict[str, np.ndarray]:
    rng = np.random.default_rng(seed)
    s = len(species)
    rec: dict[str, np.ndarray] = {}
    rec["atomic_numbers"] = np.array(species)
    rec["embedding"] = rng.normal(size=(s, 512))
    rec["e0"] = rng.uniform(-10, -1, size=s)
    rec["constants"] = np.array([6.0, np.sqrt(2.0 / 6.0), 5.0, 1.0805, 0.9183, 4.5791, 0.8, -0.05,
                                 0.300, 0.4543, 6.0, 1.6790, 1.8484, 1.6790])
    rec["bessel"] = np.arange(1, 11) * np.pi / 6.0
    rec["radii"] = rng.uniform(0.5, 1.6, size=119)
    rec["zbl.radii"] = rng.uniform(0.5, 1.1, size=119)
    rec["zbl.c"] = np.array([0.1818, 0.5099, 0.2802, 0.02817])
    pre = [(2048, 0), (512, 1), (512, 2), (512, 3)]
    gated = [(512, 0), (512, 1), (512, 2), (512, 3)]
    for k in range(2):
        p = f"layer{k}"
        node = [(512, 0)] if k == 0 else [(512, 0), (512, 1)]
        up = [(128, 0)] if k == 0 else [(128, 0), (128, 1)]
        hidden = [(512, 0), (512, 1)] if k == 0 else [(512, 0)]
        tp_paths, out_start, _, ncomp = tp_layout(k)
        message = [(128, tp_paths[q][2]) for q in sorted(out_start, key=out_start.get)]
        parts = {
            "linear_up": _linear(rng, node, up),
            "linear_res": _linear(rng, up, pre),
            "linear_1": _linear(rng, message, pre),
            "linear_2": _linear(rng, gated, gated, 0.6),
            "skip_tp": _linear(rng, node, hidden),
            "product.linear": _linear(rng, hidden, hidden),
        }
        for name, lin in parts.items():
            for key, value in lin.items():
                rec[f"{p}.{name}.{key}"] = value
        rec[f"{p}.norm"] = np.array([1.0, 1.0])
        for key, value in _tensor_product(k).items():
            rec[f"{p}.tp.{key}"] = value
        for key, value in _radial(rng, s, 3, len(tp_paths) * 128).items():
            rec[f"{p}.radial.{key}"] = value
        for key, value in _radial(rng, s, 1, 1).items():
            rec[f"{p}.density.{key}"] = value
        for key, value in _polynomial(rng, k).items():
            rec[f"{p}.product.{key}"] = value
    for name, ins, outs in (("readout0", [(512, 0), (512, 1)], [(1, 0)]),
                            ("readout1.up", [(512, 0)], [(16, 0)]),
                            ("readout1.down", [(16, 0)], [(1, 0)])):
        for key, value in _linear(rng, ins, outs).items():
            rec[f"{name}.{key}"] = value
    return {k: np.asarray(v) for k, v in rec.items()}


def manifest(records: dict[str, np.ndarray], seed: int) -> dict:
    return {
        "seed": seed,
        "species": [int(z) for z in records["atomic_numbers"]],
        "constants": [float(x) for x in records["constants"].astype(np.float32)],
        "tp_terms": [int(records[f"layer{k}.tp.values"].size) for k in range(2)],
        "product_terms": [int(records[f"layer{k}.product.terms"].size // 5) for k in range(2)],
        "parameter_floats": int(sum(v.size for v in records.values())),
    }


def write_archive(path: str | Path, seed: int = SEED) -> dict:
    """Write the seeded archive (and ``<path>.json`` manifest) unless already current."""
    path = Path(path)
    meta = Path(str(path) + ".json")
    if path.exists() and meta.exists():
        info = json.loads(meta.read_text())
        if info.get("seed") == seed and info.get("generator") == GENERATOR_VERSION:
            return info
    records = make_records(seed)
    path.parent.mkdir(parents=True, exist_ok=True)
    archive.write(path, records)
    info = manifest(records, seed)
    info["generator"] = GENERATOR_VERSION
    meta.write_text(json.dumps(info, indent=1) + "\n")
    return info


GENERATOR_VERSION = 1
