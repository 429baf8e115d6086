"""ASE calculator over the C ABI (same surface as the reference's MH1Calculator,
mace/python/mace_inference/calculator.py:10-94): energy, energies, forces and
stress = -virial / volume in Voigt order; ``evaluate`` bypasses the ASE cache."""
import numpy as np
from ase.calculators.calculator import Calculator, all_changes
from ase.stress import full_3x3_to_voigt_6_stress

from .native import NativeMH1


class MH1Calculator(Calculator):
    implemented_properties = ["energy", "energies", "forces", "stress"]

    def __init__(self, model, *, backend="auto", library=None, head=None, **kwargs):
        super().__init__(**kwargs)
        self.native = NativeMH1(model, backend=backend, library=library, head=head)

    def close(self):
        if getattr(self, "native", None):
            self.native.close()
            self.native = None

    def __enter__(self):
        return self

    def __exit__(self, *args):
        self.close()

    def __del__(self):
        self.close()

    def evaluate(self, atoms):
        """Always execute, bypassing ASE's geometry cache (for trajectory replay)."""
        if not getattr(self, "native", None):
            raise RuntimeError("Calculator is closed")
        if not np.all(atoms.pbc):
            raise ValueError("v1 requires three periodic axes")
        r = self.native.calculate(atoms.positions, atoms.numbers, atoms.cell.array)
        r["stress"] = full_3x3_to_voigt_6_stress(-r["virial"] / atoms.get_volume())
        return r

    def calculate(self, atoms=None, properties=("energy",), system_changes=all_changes):
        super().calculate(atoms, properties, system_changes)
        self.results = self.evaluate(self.atoms)

    @property
    def diagnostics(self):
        return self.native.diagnostics
