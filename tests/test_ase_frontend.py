"""The ASE frontend (mace_inference.MH1Calculator) against the reference's contract
(mace/python/mace_inference/calculator.py:10-94): implemented properties, stress =
-virial / volume in Voigt order, three periodic axes required, evaluate() bypassing the
cache, close / context-manager lifecycle.

ASE is not installed in this image.  When it is absent, a stand-in with the three names the
calculator imports is installed for these tests only: ``Calculator`` (whose ``calculate``
copies the atoms, as ASE's does), ``all_changes`` and ``full_3x3_to_voigt_6_stress``
(ASE's published Voigt order xx, yy, zz, yz, xz, xy of the symmetrised matrix).
"""
import importlib
import sys
import types

import numpy as np
import pytest

from conftest import DATA


def _install_ase_stand_in():
    """Installs the stand-in when ASE is absent; returns the module names it added."""
    try:
        import ase  # noqa: F401
        return []
    except ImportError:
        pass

    class Calculator:
        implemented_properties = []

        def __init__(self, **kwargs):
            self.results, self.atoms, self.parameters = {}, None, dict(kwargs)

        def calculate(self, atoms=None, properties=("energy",), system_changes=()):
            if atoms is not None:
                self.atoms = atoms.copy()

    def full_3x3_to_voigt_6_stress(m):
        m = np.asarray(m)
        return np.array([m[0, 0], m[1, 1], m[2, 2], (m[1, 2] + m[2, 1]) / 2, (m[0, 2] + m[2, 0]) / 2,
                         (m[0, 1] + m[1, 0]) / 2])

    mods = {n: types.ModuleType(n) for n in ("ase", "ase.calculators", "ase.calculators.calculator", "ase.stress")}
    mods["ase.calculators.calculator"].Calculator = Calculator
    mods["ase.calculators.calculator"].all_changes = ["positions", "numbers", "cell", "pbc"]
    mods["ase.stress"].full_3x3_to_voigt_6_stress = full_3x3_to_voigt_6_stress
    sys.modules.update(mods)
    return list(mods)


class Atoms:
    """The part of ase.Atoms the calculator reads."""

    def __init__(self, positions, numbers, cell, pbc=True):
        self.positions = np.asarray(positions, np.float64)
        self.numbers = np.asarray(numbers)
        self.cell = types.SimpleNamespace(array=np.asarray(cell, np.float64))
        self.pbc = np.array([pbc] * 3 if np.isscalar(pbc) else pbc)

    def get_volume(self):
        return abs(np.linalg.det(self.cell.array))

    def copy(self):
        return Atoms(self.positions.copy(), self.numbers.copy(), self.cell.array.copy(), self.pbc.copy())

    def __len__(self):
        return len(self.numbers)


@pytest.fixture(scope="module")
def calculator_module():
    added = _install_ase_stand_in()
    import mace_inference.calculator as calc
    yield importlib.reload(calc)
    for name in added:
        sys.modules.pop(name, None)
    if added:
        sys.modules.pop("mace_inference.calculator", None)


class FakeNative:
    calls = 0

    def __init__(self, model, backend=0, library=None, head=None):
        self.model, self.head, self.closed = model, head, False

    def calculate(self, xyz, z, cell):
        FakeNative.calls += 1
        n = len(z)
        virial = np.array([[1.0, 2.0, 3.0], [2.5, 5.0, 6.0], [3.5, 6.5, 9.0]], np.float32)
        return dict(energy=-1.5 * n, energies=np.full(n, -1.5, np.float32), forces=np.zeros((n, 3), np.float32),
                    virial=virial)

    def close(self):
        self.closed = True


def test_calculator_contract(calculator_module, monkeypatch):
    monkeypatch.setattr(calculator_module, "NativeMH1", FakeNative)
    cell = np.diag([2.0, 3.0, 4.0])
    atoms = Atoms(np.zeros((2, 3)), [1, 8], cell)
    calc = calculator_module.MH1Calculator("model.pwm", head="matpes_r2scan")
    assert calc.implemented_properties == ["energy", "energies", "forces", "stress"]
    assert calc.native.head == "matpes_r2scan"
    before = FakeNative.calls
    r = calc.evaluate(atoms)
    calc.evaluate(atoms)
    assert FakeNative.calls == before + 2  # no cache
    v = np.array([[1.0, 2.0, 3.0], [2.5, 5.0, 6.0], [3.5, 6.5, 9.0]]) / -24.0
    assert np.allclose(r["stress"], [v[0, 0], v[1, 1], v[2, 2], (v[1, 2] + v[2, 1]) / 2, (v[0, 2] + v[2, 0]) / 2,
                                     (v[0, 1] + v[1, 0]) / 2])
    calc.calculate(atoms)
    assert calc.results["energy"] == -3.0 and calc.atoms is not atoms
    with pytest.raises(ValueError, match="three periodic axes"):
        calc.evaluate(Atoms(np.zeros((2, 3)), [1, 8], cell, pbc=[True, True, False]))
    native = calc.native
    with calc:
        pass
    assert native.closed and calc.native is None
    with pytest.raises(RuntimeError, match="Calculator is closed"):
        calc.evaluate(atoms)


@pytest.mark.gpu
def test_calculator_on_gpu(calculator_module, library, archive_path):
    """The real engine behind the calculator: the same numbers as NativeMH1."""
    from lasp_b200 import structures
    from mace_inference import NativeMH1
    s = structures.load("C1", DATA)
    atoms = Atoms(s.positions, s.numbers, s.cell)
    with calculator_module.MH1Calculator(archive_path, library=library) as calc, \
            NativeMH1(archive_path, library=library) as native:
        r = calc.evaluate(atoms)
        ref = native.calculate(s.positions, s.numbers, s.cell)
    assert r["energy"] == ref["energy"] and np.array_equal(r["energies"], ref["energies"])
    assert np.abs(r["forces"] - ref["forces"]).max() <= 1e-6 * max(1.0, float(np.abs(ref["forces"]).max()))
    vol = abs(np.linalg.det(s.cell.astype(np.float64)))
    w = -ref["virial"].astype(np.float64) / vol
    assert np.allclose(r["stress"][:3], np.diag(w), rtol=1e-5, atol=1e-9)
