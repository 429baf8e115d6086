"""Record the float64 oracle's outputs and the reference's own float32 error (no GPU).

For each config, runs the float64 CPU oracle (oracle/) on the seeded structure and archive and
compares it with the REFERENCE build's outputs already committed here (ref_<config>.npz, made
by make_ref_golden.py on a B200).  Writes oracle_summary.json:

    {config: {"oracle": {"energy", "virial"[9]},
              "reference_error": {"energy_rel", "forces", "energies", "virial"}}}

The reference's error against float64 is the scale of "the reference's precision" that the
GPU parity tests use for their bounds (tests/test_mh1_gpu.py).  For C5 the reference fixture
holds forces and energies for a seeded sample of atoms; the errors are taken over that sample.

    python tests/golden/make_oracle_golden.py                 # C1, C2, C3
    python tests/golden/make_oracle_golden.py --configs C5 --merge
    python tests/golden/make_oracle_golden.py --configs C5 --merge --oracle-npz C5=<file.npz>

--oracle-npz reuses an oracle result saved earlier with numpy.savez (energy, energies,
forces, virial) instead of recomputing it (C5 takes tens of minutes on 8 cores).
"""
from __future__ import annotations

import argparse
import json
import sys
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent
ROOT = HERE.parents[1]
sys.path[:0] = [str(ROOT / "lasp-pis_b200" / "python"), str(ROOT / "oracle")]
from lasp_b200 import structures, synth  # noqa: E402

DATA = ROOT / "lasp-pis_b200" / "data"


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--configs", default="C1,C2,C3")
    ap.add_argument("--merge", action="store_true")
    ap.add_argument("--oracle-npz", action="append", default=[], help="CONFIG=path of a saved oracle result")
    args = ap.parse_args()
    saved = dict(x.split("=", 1) for x in args.oracle_npz)
    out = HERE / "oracle_summary.json"
    summary = json.loads(out.read_text()) if args.merge and out.exists() else {}
    archive = DATA / "mh1_synth.pwm"
    synth.write_archive(archive)
    import oracle
    oracle.build()
    model = oracle.Oracle(archive)
    for name in args.configs.split(","):
        s = structures.load(name, DATA)
        o = dict(np.load(saved[name])) if name in saved else model.calculate(s.positions, s.numbers, s.cell)
        g = dict(np.load(HERE / f"ref_{name}.npz"))
        if "sample" in g:
            idx = g["sample"]
            f_ref, e_ref, f_o, e_o = g["forces_sample"], g["energies_sample"], o["forces"][idx], o["energies"][idx]
        else:
            f_ref, e_ref, f_o, e_o = g["forces"], g["energies"], o["forces"], o["energies"]
        summary[name] = {
            "oracle": {"energy": float(o["energy"]), "virial": np.asarray(o["virial"], np.float64).ravel().tolist()},
            "reference_error": {
                "energy_rel": float(abs(float(g["energy"]) - float(o["energy"])) / abs(float(o["energy"]))),
                "forces": float(np.abs(f_ref.astype(np.float64) - f_o).max()),
                "energies": float(np.abs(e_ref.astype(np.float64) - e_o).max()),
                "virial": float(np.abs(np.asarray(g["virial"], np.float64).ravel()
                                       - np.asarray(o["virial"], np.float64).ravel()).max()),
            },
        }
        print(name, json.dumps(summary[name]["reference_error"]), flush=True)
    out.write_text(json.dumps(summary, indent=1) + "\n")


if __name__ == "__main__":
    main()
