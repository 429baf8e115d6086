"""CPU tests of the parity oracle: pinned against the reference's golden outputs.

The fixtures in tests/golden/ were recorded by running the reference's own CUDA build
(oracle/_ref, compiled from its sources) on a B200 with tests/golden/make_ref_golden.py,
and the e3nn coupling table extracted from the reference by tests/golden/extract_cg.py.
"""
import hashlib
import json

import numpy as np
import pytest

import oracle as O
import scenarios
from conftest import DATA, GOLDEN
from lasp_b200 import archive, so3, structures, synth

SUMMARY = json.loads((GOLDEN / "ref_summary.json").read_text())


def digest(edges):
    return hashlib.sha256(np.ascontiguousarray(edges, np.int32).tobytes()).hexdigest()


def test_coupling_table_matches_reference_cg():
    ref = {}
    for line in (GOLDEN / "cg_e3nn044.txt").read_text().split("\n"):
        if line.strip():
            v = line.split()
            ref[tuple(int(x) for x in v[:6])] = float(v[6])
    mine = {r[:6]: r[6] for r in so3.coupling_table()}
    assert set(mine) == set(ref)
    for k, v in ref.items():
        assert mine[k] == pytest.approx(v, abs=2e-7), k


def test_archive_round_trip(archive_path):
    rec = archive.read(archive_path)
    again = archive.decode(archive.encode(rec))
    assert rec.keys() == again.keys()
    for k in rec:
        assert np.array_equal(rec[k], again[k])
    info = json.loads((DATA / "mh1_synth.pwm.json").read_text())
    assert info["tp_terms"] == [16, 86]
    assert rec["layer1.tp.dims"].tolist() == [10, 4, 40]


@pytest.mark.parametrize("case", list(scenarios.framework_scenarios()), ids=lambda c: c[0])
def test_oracle_edges_match_reference_traversal(case):
    name, xyz, cell, cutoff, grid, backends = case
    for b in backends:
        e, d = O.edges(xyz, cell, cutoff, b)
        ref = SUMMARY["edges"][name][str(b)]
        assert len(e) == ref["count"]
        assert digest(e) == ref["sha256"]
        assert len(np.unique(e, axis=0)) == len(e)


def test_edge_semantics():
    box = np.eye(3, dtype=np.float32) * 8
    e, _ = O.edges(np.array([[0, 0, 0], [2.5, 0, 0]], np.float32), box, 2.5)
    assert len(e) == 2                       # inclusive cutoff
    for count in (1, 17, 145):
        xyz = np.ones((count, 3), np.float32)
        xyz[:, 0] += np.arange(count, dtype=np.float32) * np.float32(1e-4)
        e, _ = O.edges(xyz, box, 0.5)
        assert len(e) == count * (count - 1)
    with pytest.raises(RuntimeError, match="Singular"):
        O.edges(np.zeros((2, 3), np.float32), np.zeros((3, 3), np.float32), 2.5)
    with pytest.raises(RuntimeError, match="CellList"):
        O.edges(np.zeros((2, 3), np.float32), np.eye(3, dtype=np.float32), 2.5, backend=2)


@pytest.mark.parametrize("name", ["C1", "C2", "C3"])
def test_oracle_config_edges_match_reference(name):
    s = structures.load(name, DATA)
    e, _ = O.edges(s.positions, s.cell)
    ref = SUMMARY["configs"][name]["edges_1"]
    assert len(e) == ref["count"] and digest(e) == ref["sha256"]


@pytest.mark.parametrize("name", ["C1", "C2"])
def test_oracle_matches_reference_outputs(oracle_model, name):
    """Float64 oracle vs the reference's float32 CUDA outputs on identical inputs."""
    s = structures.load(name, DATA)
    r = oracle_model.calculate(s.positions, s.numbers, s.cell)
    g = np.load(GOLDEN / f"ref_{name}.npz")
    assert abs(g["energy"] - r["energy"]) <= 1e-6 * abs(r["energy"])
    fmax = np.abs(r["forces"]).max()
    assert np.abs(g["forces"] - r["forces"]).max() <= 1e-5 * max(1.0, fmax)
    assert np.abs(g["energies"] - r["energies"]).max() <= 5e-5
    assert np.abs(g["virial"] - r["virial"]).max() <= 1e-6 * np.abs(r["virial"]).max()


def test_oracle_native_case_matches_reference(oracle_model):
    xyz, z, cell = scenarios.native_case()
    r = oracle_model.calculate(xyz, z, cell)
    g = np.load(GOLDEN / "ref_native.npz")
    assert abs(g["energy"] - r["energy"]) <= 1e-6 * abs(r["energy"])
    assert np.abs(g["forces"] - r["forces"]).max() <= 1e-5


def test_oracle_finite_differences(oracle_model):
    s = structures.load("C1", DATA)
    x, cell = s.positions.astype(np.float64), s.cell.astype(np.float64)
    r = oracle_model.calculate(x, s.numbers, cell)
    h = 4e-3
    for i, k in [(3, 0), (22, 1), (40, 2)]:
        xp, xm = x.copy(), x.copy()
        xp[i, k] += h
        xm[i, k] -= h
        step = float(np.float32(xp[i, k]) - np.float32(xm[i, k]))
        ep = oracle_model.calculate(xp, s.numbers, cell)["energy"]
        em = oracle_model.calculate(xm, s.numbers, cell)["energy"]
        assert r["forces"][i, k] == pytest.approx(-(ep - em) / step, abs=2e-4)
    for a, b in [(0, 0), (1, 2)]:
        def energy(eps):
            f = np.eye(3)
            f[a, b] += eps
            return oracle_model.calculate(x @ f.T, s.numbers, cell @ f.T)["energy"]
        eps = 1e-3
        assert r["virial"][a, b] == pytest.approx(-(energy(eps) - energy(-eps)) / (2 * eps), rel=2e-3, abs=0.05)


def test_oracle_invariances(oracle_model):
    s = structures.load("C1", DATA)
    r = oracle_model.calculate(s.positions, s.numbers, s.cell)
    rot = so3.rotation(3)
    rr = oracle_model.calculate(s.positions @ rot.T, s.numbers, s.cell @ rot.T)
    assert rr["energy"] == pytest.approx(r["energy"], rel=1e-8)
    assert np.abs(rr["forces"] - r["forces"] @ rot.T).max() < 1e-5
    p = np.random.default_rng(0).permutation(s.size)
    rp = oracle_model.calculate(s.positions[p], s.numbers[p], s.cell)
    assert rp["energy"] == pytest.approx(r["energy"], rel=1e-12)
    assert np.abs(rp["forces"] - r["forces"][p]).max() < 1e-9
    assert np.abs(r["forces"].sum(0)).max() < 1e-8
    shifted = oracle_model.calculate(s.positions + np.float32(9.0), s.numbers, s.cell)
    assert shifted["energy"] == pytest.approx(r["energy"], rel=1e-7)


def test_oracle_errors(oracle_model):
    xyz, z, cell = scenarios.native_case()
    with pytest.raises(RuntimeError, match="Singular"):
        oracle_model.calculate(xyz, z, np.zeros((3, 3)))
    with pytest.raises(RuntimeError, match="code 2"):
        oracle_model.calculate(xyz, np.array([14, 6, 8, 99], np.int32), cell)
    empty = oracle_model.calculate(np.zeros((0, 3)), np.zeros(0, np.int32), cell)
    assert empty["energy"] == 0


def test_structure_generators_avoid_cutoff_band():
    for name in ("C1", "C2"):
        s = structures.load(name, DATA)
        f = s.positions.astype(float) @ np.linalg.inv(s.cell.astype(float))
        _, _, d = structures._pairs_within(f - np.floor(f), s.cell.astype(float), 6.001)
        assert np.all(np.abs(d - 6.0) > structures.BAND)


def test_arc_round_trip(tmp_path):
    s = structures.load("C1", DATA)
    path = tmp_path / "c1.arc"
    structures.write_arc(path, [s, s])
    text = path.read_text()
    assert text.count("CORE") == 2 * s.size and text.count("\nend\nend") == 2
    a, b, c, al, be, ga = structures.parameters(s.cell)
    assert np.allclose(structures.cell_from_parameters(a, b, c, al, be, ga), s.cell, atol=1e-5)
    assert synth.SEED == 20261201
