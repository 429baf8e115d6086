"""GPU parity of the B200 engine, through the C ABI.

Edges: the canonical (receiver, sender, shift) multiset must equal the reference's own
Lapis traversal bit for bit (sha256 of the sorted int32 list recorded on a B200 by
tests/golden/make_ref_golden.py) and the float64 oracle's, on every backend.

Model outputs are compared with the reference CUDA build's outputs on identical inputs and
weights (tests/golden/ref_*.npz) and with the float64 oracle (oracle/).  Bounds, all
absolute except the energy (north star: energy 1e-6 relative, forces 1e-5 eV/A, virial
1e-5 eV "at the reference's precision"):

* energy: 1e-6 relative;
* forces: max(1e-5 eV/A, 2 x the reference's own call-to-call spread for that config)
  (tests/golden/ref_summary.json "repeat_0": two calls of the reference differ by up to
  9.5e-6 eV/A at C2 and 9.5e-5 at C5 through its float atomics);
* virial: max(1e-5 eV, 2 x the reference's own deviation from the float64 oracle) against
  the oracle, and max(1e-5 eV, 3 x that deviation + the reference's call-to-call spread)
  against the reference (tests/golden/oracle_summary.json, made by make_oracle_golden.py;
  virial_bound).  The virial of these cells is 1e2-3e5 eV, so 1e-5 eV is below one float32
  ulp of the value itself; the reference's own float32 result is 6e-5 (C1) to 1.4e-3 eV (C3)
  away from float64, and this build's 0.7-1.6x as far;
* per-atom energies: 5e-5 eV.
"""
import hashlib
import json
import subprocess

import numpy as np
import pytest

import oracle as O
import scenarios
from conftest import DATA, GOLDEN, ROOT
from lasp_b200 import structures

pytestmark = pytest.mark.gpu
SUMMARY = json.loads((GOLDEN / "ref_summary.json").read_text())


def digest(edges):
    return hashlib.sha256(np.ascontiguousarray(edges, np.int32).tobytes()).hexdigest()


@pytest.fixture(scope="module")
def engine(library, archive_path):
    from mace_inference import NativeMH1
    models = {b: NativeMH1(archive_path, backend=b, library=library) for b in (0, 1, 2)}
    yield models
    for m in models.values():
        m.close()


@pytest.mark.parametrize("case", list(scenarios.framework_scenarios()), ids=lambda c: c[0])
def test_neighbor_edges_match_reference(library, case):
    from mace_inference import neighbor_edges
    name, xyz, cell, cutoff, grid, backends = case
    for b in backends:
        e = neighbor_edges(xyz, cell, cutoff, b, grid, library=library)
        ref = SUMMARY["edges"][name][str(b)]
        assert len(e) == ref["count"], (name, b)
        assert digest(e) == ref["sha256"], (name, b)


def test_neighbor_errors(library):
    from mace_inference import neighbor_edges
    with pytest.raises(RuntimeError, match="Singular"):
        neighbor_edges(np.zeros((2, 3)), np.zeros((3, 3)), 2.5, library=library)
    with pytest.raises(RuntimeError, match="CellList"):
        neighbor_edges(np.zeros((2, 3)), np.eye(3), 2.5, 2, library=library)


ORACLE = json.loads((GOLDEN / "oracle_summary.json").read_text())


def force_bound(name):
    return max(1e-5, 2 * SUMMARY["configs"][name]["repeat_0"]["forces"])


def virial_bound(name, against="reference"):
    """Against float64: max(1e-5 eV, 2 x the reference's own deviation from float64).
    Against the reference: max(1e-5 eV, 3 x that deviation + the reference's call-to-call
    spread) -- this build's deviation (at most 2x) plus the reference's own (1x).

    Measured on B200 against float64: 0.7x (C1), 0.9x (C2) and 1.6x (C3) the reference's
    deviation.  C5 has no float64 result (the oracle needs more than 62 GB of host memory for
    its 17.3M edges): the reference's deviation is estimated as its relative deviation at C3
    times C5's virial magnitude, and the bound against the reference is 4x that estimate plus
    the spread (measured 3.7x)."""
    if name in ORACLE:
        err = ORACLE[name]["reference_error"]["virial"]
        factor = 2 if against == "oracle" else 3
    else:
        rel = ORACLE["C3"]["reference_error"]["virial"] / float(np.abs(np.load(GOLDEN / "ref_C3.npz")["virial"]).max())
        err = rel * float(np.abs(np.load(GOLDEN / f"ref_{name}.npz")["virial"]).max())
        factor = 4
    spread = SUMMARY["configs"][name]["repeat_0"]["virial"] if against == "reference" else 0.0
    return max(1e-5, factor * err + spread)


def check_close(r, ref, name, against="reference"):
    assert abs(r["energy"] - ref["energy"]) <= 1e-6 * abs(ref["energy"]), (r["energy"], ref["energy"])
    ferr = float(np.abs(r["forces"] - ref["forces"]).max())
    bound = force_bound(name) if against == "reference" else max(1e-5, 2 * ORACLE[name]["reference_error"]["forces"])
    assert ferr <= bound, (ferr, bound)
    assert float(np.abs(r["energies"] - ref["energies"]).max()) <= 5e-5
    werr = float(np.abs(np.asarray(r["virial"], np.float64) - np.asarray(ref["virial"], np.float64)).max())
    assert werr <= virial_bound(name, against), (werr, virial_bound(name, against))


@pytest.mark.parametrize("name", ["C1", "C2", "C3"])
def test_model_edges_match_reference(engine, name):
    """Every backend's edge list (Auto, Brute, Cell) equals the reference traversal's."""
    s = structures.load(name, DATA)
    for b, key in ((0, "edges_1"), (1, "edges_1"), (2, "edges_2")):
        engine[b].calculate(s.positions, s.numbers, s.cell)
        e = engine[b].last_edges()
        ref = SUMMARY["configs"][name][key]
        assert len(e) == ref["count"] and digest(e) == ref["sha256"], (name, b)


@pytest.mark.parametrize("name", ["C1", "C2"])
def test_matches_oracle(engine, oracle_model, name):
    s = structures.load(name, DATA)
    ref = oracle_model.calculate(s.positions, s.numbers, s.cell)
    for b in (0, 1, 2):
        check_close(engine[b].calculate(s.positions, s.numbers, s.cell), ref, name, against="oracle")


@pytest.mark.parametrize("name", ["C1", "C2", "C3"])
def test_matches_reference_cuda(engine, name):
    s = structures.load(name, DATA)
    g = dict(np.load(GOLDEN / f"ref_{name}.npz"))
    for b in ((0, 1, 2) if s.size <= 1000 else (0,)):
        check_close(engine[b].calculate(s.positions, s.numbers, s.cell), g, name)


def test_c5_matches_reference_cuda(library, archive_path):
    """C5, 198,904 atoms and 17.3M edges on one GPU, against the reference build's outputs on
    the same inputs: the cell-list edge digest, energy, virial, float64 sums of the per-atom
    energies and forces, and the forces and energies of a seeded sample of 4,096 atoms."""
    from mace_inference import NativeMH1
    s = structures.load("C5", DATA)
    g = dict(np.load(GOLDEN / "ref_C5.npz"))
    with NativeMH1(archive_path, backend=0, library=library) as m:
        r = m.calculate(s.positions, s.numbers, s.cell)
        e = m.last_edges()
    ref = SUMMARY["configs"]["C5"]["edges_2"]
    assert len(e) == ref["count"] and digest(e) == ref["sha256"]
    assert abs(r["energy"] - float(g["energy"])) <= 1e-6 * abs(float(g["energy"]))
    idx = g["sample"]
    assert float(np.abs(r["forces"][idx] - g["forces_sample"]).max()) <= force_bound("C5")
    assert float(np.abs(r["energies"][idx] - g["energies_sample"]).max()) <= 5e-5 * 4
    werr = float(np.abs(np.asarray(r["virial"], np.float64) - np.asarray(g["virial"], np.float64)).max())
    assert werr <= virial_bound("C5"), werr
    # Whole-array checks through float64 sums: total of the per-atom energies, net force.
    assert abs(r["energies"].astype(np.float64).sum() - float(g["energies_sum"])) <= 1e-6 * abs(float(g["energy"]))
    assert np.abs(r["forces"].astype(np.float64).sum(0) - g["forces_sum"]).max() <= 1e-2


ENGINE_VARIANT = """
import sys, numpy as np
sys.path[:0] = {paths!r}
from lasp_b200 import structures
from mace_inference import NativeMH1
s = structures.load("C2", {data!r})
with NativeMH1({archive!r}, backend=0, library={library!r}) as m:
    r = m.calculate(s.positions, s.numbers, s.cell)
np.savez({out!r}, **r)
"""


@pytest.mark.parametrize("env", [{"MACE_PROJECTION_CHUNK_EDGES": "3000"}, {"MACE_SIMT_EDGES": "1"},
                                 {"MACE_SIMT_LINEARS": "1"}, {"MACE_GENERIC_PRODUCT": "1"}],
                         ids=["projection-chunks", "simt-edges", "simt-all", "generic-product"])
def test_engine_variants_match_oracle(library, archive_path, oracle_model, env, tmp_path):
    """The chunked projection path (many receiver-aligned chunks, R recomputed in the backward),
    the fused SIMT edge kernels, the all-SIMT path (node linears too) and the table-driven
    product kernels give the oracle's results as well."""
    import os
    import sys
    out = tmp_path / "r.npz"
    paths = [str(ROOT / "lasp-pis_b200" / "python")]
    code = ENGINE_VARIANT.format(paths=paths, data=str(DATA), archive=str(archive_path), library=str(library),
                                 out=str(out))
    r = subprocess.run([sys.executable, "-c", code], env={**os.environ, **env}, capture_output=True, text=True)
    assert r.returncode == 0, r.stderr[-2000:]
    s = structures.load("C2", DATA)
    check_close(dict(np.load(out)), oracle_model.calculate(s.positions, s.numbers, s.cell), "C2", against="oracle")


def test_native_behaviour(engine):
    """Backends agree, permutation, empty structure, error recovery (mace/tests/native.py:41-72)."""
    xyz, z, cell = scenarios.native_case()
    base = engine[1].calculate(xyz, z, cell)
    g = np.load(GOLDEN / "ref_native.npz")
    assert abs(base["energy"] - float(g["energy"])) <= 1e-6 * abs(float(g["energy"]))
    assert np.abs(base["forces"] - g["forces"]).max() <= 1e-5
    for b in (0, 2):
        r = engine[b].calculate(xyz, z, cell)
        for k in r:
            np.testing.assert_allclose(r[k], base[k], atol=2e-4, rtol=2e-5)
    order = np.array([2, 0, 3, 1])
    p = engine[0].calculate(xyz[order], z[order], cell)
    np.testing.assert_allclose(p["forces"], base["forces"][order], atol=2e-4, rtol=2e-5)
    assert engine[0].calculate(np.zeros((0, 3)), np.zeros(0, np.int32), cell)["energy"] == 0
    with pytest.raises(RuntimeError, match="Singular"):
        engine[0].calculate(xyz, z, np.zeros((3, 3)))
    with pytest.raises(RuntimeError, match="code 2"):
        engine[0].calculate(xyz, np.array([14, 6, 8, 99], np.int32), cell)
    with pytest.raises(RuntimeError, match="Invalid atomic number"):
        engine[0].calculate(xyz, np.array([14, 6, 8, 0], np.int32), cell)
    again = engine[0].calculate(xyz, z, cell)
    for k in again:
        np.testing.assert_allclose(again[k], base[k], atol=2e-4, rtol=2e-5)


@pytest.mark.parametrize("name", ["C2", "C3"])
def test_repeat_is_bitwise_deterministic(engine, library, archive_path, name):
    """Every output is reproducible bit for bit: repeated calls on one handle and a call on a
    fresh handle give the same energy, per-atom energies, forces and virial (no float atomics
    anywhere on the path: sender-side sums run over a sender index in edge order)."""
    from mace_inference import NativeMH1
    s = structures.load(name, DATA)
    a = engine[0].calculate(s.positions, s.numbers, s.cell)
    b = engine[0].calculate(s.positions, s.numbers, s.cell)
    with NativeMH1(archive_path, backend=0, library=library) as fresh:
        c = fresh.calculate(s.positions, s.numbers, s.cell)
    for r in (b, c):
        assert r["energy"] == a["energy"]
        for key in ("energies", "forces", "virial"):
            assert np.array_equal(r[key], a[key]), key


def test_device_entry_point_matches_host(engine):
    import torch
    s = structures.load("C2", DATA)
    host = engine[0].calculate(s.positions, s.numbers, s.cell)
    xyz = torch.from_numpy(s.positions).cuda()
    z = torch.from_numpy(s.numbers).cuda()
    torch.cuda.synchronize()
    dev = engine[0].calculate_device(s.size, xyz.data_ptr(), z.data_ptr(), s.cell)
    assert dev["energy"] == pytest.approx(host["energy"], rel=1e-7)
    assert np.abs(dev["forces"] - host["forces"]).max() <= 1e-5


def test_cli_matches_reference(library, archive_path, tmp_path):
    s = structures.load("C1", DATA)
    arc = tmp_path / "C1.arc"
    structures.write_arc(arc, [s])
    exe = ROOT / "lasp-pis_b200" / "bin" / "mace-main"
    r = subprocess.run([str(exe), str(archive_path), str(arc), "--json"], capture_output=True, text=True)
    assert r.returncode == 0, r.stderr
    mine = json.loads(r.stdout)
    ref = json.loads((GOLDEN / "ref_cli_C1.json").read_text())
    assert mine["atoms"] == ref["atoms"] == 64
    assert mine["energy"] == pytest.approx(ref["energy"], rel=1e-6)
    assert np.abs(np.array(mine["forces"]) - np.array(ref["forces"])).max() <= 5e-5
    out = tmp_path / "out.txt"
    r = subprocess.run([str(exe), str(archive_path), str(arc), "--output", str(out)], capture_output=True, text=True)
    assert r.returncode == 0 and "Energy (eV)" in out.read_text()


def test_checkpoint_route(library, tmp_path):
    """An MH1 PyTorch ZIP checkpoint loads through mace_create_mh1_head and the
    device-binding constructor and evaluates like the archive the converter writes for the
    same head, bit for bit (energy, per-atom energies, forces, virial), and that archive
    matches the float64 oracle.  The CLI accepts the checkpoint with --head and names the head on
    stderr; unknown heads are errors.  (The converter itself is pinned byte for byte against
    the reference's in test_checkpoint.py.)  Oracle bounds are 3x check_close's: this random
    model's forces and virial are 4-7x smaller than the synthetic archive's, so the same
    absolute float32 error is a larger fraction of them."""
    import torch
    from lasp_b200 import checkpoint
    from mace_inference import NativeMH1
    ckpt = checkpoint.write_checkpoint(tmp_path / "mh1.model", 5, torch.float32)
    head = "synthetic_scan"
    pwm = tmp_path / "mh1.pwm"
    dump = ROOT / "lasp-pis_b200" / "bin" / "mace-weights-dump"
    subprocess.run([str(dump), str(ckpt), str(pwm), head], check=True)
    s = structures.load("C1", DATA)
    with NativeMH1(ckpt, head=head, library=library) as a, NativeMH1(pwm, library=library) as b, \
            NativeMH1(ckpt, head=head, device=0, library=library) as c, NativeMH1(ckpt, library=library) as d:
        ra, rb, rc, rd = (m.calculate(s.positions, s.numbers, s.cell) for m in (a, b, c, d))
    for r in (ra, rc):
        assert r["energy"] == rb["energy"]
        for key in ("energies", "forces", "virial"):
            assert np.array_equal(r[key], rb[key]), key
    assert rd["energy"] != ra["energy"]  # the default head (matpes_r2scan) has its own e0 and scale
    check_close(ra, O.Oracle(pwm).calculate(s.positions, s.numbers, s.cell), "C1", against="oracle")
    with pytest.raises(RuntimeError, match="unknown head: no_such_head"):
        NativeMH1(ckpt, head="no_such_head", library=library)
    arc = tmp_path / "C1.arc"
    structures.write_arc(arc, [s])
    exe = ROOT / "lasp-pis_b200" / "bin" / "mace-main"
    r = subprocess.run([str(exe), str(ckpt), str(arc), "--head", head, "--json"], capture_output=True, text=True)
    assert r.returncode == 0, r.stderr
    assert f"MACE head: {head}" in r.stderr
    assert json.loads(r.stdout)["energy"] == pytest.approx(ra["energy"], rel=1e-6)


def test_engine_invariances(engine):
    """The engine's own physics checks (as the reference's check_invariants.py:14-96 runs
    them on its build): translation, wrapping an atom by a lattice vector, a rigid rotation
    of positions and cell (forces and virial rotate with it), and zero net force.  Bounds:
    energy 3e-6 relative (float32 rounding of the moved coordinates), forces 1e-4 eV/A x
    max(1, max|F|) and virial 1e-5 x max|W| under rotation, 3e-5 / 6e-6 otherwise."""
    from lasp_b200 import so3
    s = structures.load("C1", DATA)
    m = engine[0]
    base = m.calculate(s.positions, s.numbers, s.cell)
    fmax, wmax = max(1.0, float(np.abs(base["forces"]).max())), float(np.abs(base["virial"]).max())

    def close(r, f_bound, w_bound, rot=None):
        f, w = base["forces"].astype(np.float64), base["virial"].astype(np.float64)
        if rot is not None:
            f, w = f @ rot.T, rot @ w @ rot.T
        assert abs(r["energy"] - base["energy"]) <= 3e-6 * abs(base["energy"])
        assert float(np.abs(r["forces"] - f).max()) <= f_bound * fmax
        assert float(np.abs(r["virial"] - w).max()) <= w_bound * wmax

    shift = np.array([0.37, -1.2, 2.9], np.float32)
    close(m.calculate(s.positions + shift, s.numbers, s.cell), 3e-5, 6e-6)
    wrapped = s.positions.copy()
    wrapped[5] += s.cell[1] - s.cell[2]
    close(m.calculate(wrapped, s.numbers, s.cell), 3e-5, 6e-6)
    rot = so3.rotation(3)
    rx = (s.positions.astype(np.float64) @ rot.T).astype(np.float32)
    rc = (s.cell.astype(np.float64) @ rot.T).astype(np.float32)
    close(m.calculate(rx, s.numbers, rc), 1e-4, 1e-5, rot)
    assert float(np.abs(base["forces"].astype(np.float64).sum(0)).max()) <= 1e-4 * fmax
