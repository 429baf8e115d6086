"""Record golden outputs of the REFERENCE CUDA build (oracle/_ref) on a B200.

Runs the reference's own ``libmace.so`` (built from its sources by oracle/ref/Makefile)
through its C ABI on the seeded synthetic archive and configs, plus its Lapis traversal
(oracle/_ref/libref_edges.so) on the neighbour scenarios, and writes the results to
``<out>/`` (default: this folder) as .npz / .json files.  The committed fixtures in
tests/golden/ were produced by running this script on a B200:

    python tests/golden/make_ref_golden.py                      # C1-C3, scenarios, CLI
    python tests/golden/make_ref_golden.py --configs C5 --merge # adds C5 to ref_summary.json

Structures above 20,000 atoms (C5) are stored compactly: energy, virial, float64 sums of the
per-atom energies and forces, and the forces and energies of a seeded sample of 4,096 atoms.
Their edge digest comes from the reference's cell-list traversal only (brute force over
200,000 atoms is not a useful fixture).

Only this script and the tests read oracle/_ref.
"""
from __future__ import annotations

import argparse
import ctypes as ct
import hashlib
import json
import os
import subprocess
import sys
import time
from pathlib import Path

import numpy as np

ROOT = Path(__file__).resolve().parents[2]
sys.path[:0] = [str(ROOT / "lasp-pis_b200" / "python"), str(ROOT / "tests" / "golden")]
from lasp_b200 import structures, synth  # noqa: E402
import scenarios  # noqa: E402

REF = ROOT / "oracle" / "_ref"
DATA = ROOT / "lasp-pis_b200" / "data"


class RefMH1:
    def __init__(self, lib, archive, backend):
        self.lib = lib
        self.h = lib.mace_create_mh1(str(archive).encode(), backend)
        if not self.h:
            raise RuntimeError(lib.mace_last_error().decode())

    def calc(self, xyz, z, cell):
        xyz = np.ascontiguousarray(xyz, np.float32).reshape(-1, 3)
        z = np.ascontiguousarray(z, np.int32)
        cell = np.ascontiguousarray(cell, np.float32).reshape(3, 3)
        e = np.zeros(1)
        a = np.zeros(len(z), np.float32)
        f = np.zeros((len(z), 3), np.float32)
        v = np.zeros((3, 3), np.float32)
        if self.lib.mace_calculate(self.h, len(z), *[x.ctypes.data for x in (xyz, z, cell, e, a, f, v)]):
            raise RuntimeError(self.lib.mace_last_error().decode())
        return dict(energy=e[0], energies=a, forces=f, virial=v)

    def diagnostics(self):
        buf = ct.create_string_buffer(1 << 16)
        self.lib.mace_diagnostics(self.h, buf, len(buf))
        return json.loads(buf.value)

    def close(self):
        self.lib.mace_destroy(self.h)


def load_ref():
    lib = ct.CDLL(str(REF / "libmace_ref.so"))
    lib.mace_create_mh1.argtypes = [ct.c_char_p, ct.c_int]
    lib.mace_create_mh1.restype = ct.c_void_p
    lib.mace_last_error.restype = ct.c_char_p
    lib.mace_destroy.argtypes = [ct.c_void_p]
    lib.mace_calculate.argtypes = [ct.c_void_p, ct.c_int] + [ct.c_void_p] * 7
    lib.mace_diagnostics.argtypes = [ct.c_void_p, ct.c_void_p, ct.c_size_t]
    return lib


def load_edges():
    lib = ct.CDLL(str(REF / "libref_edges.so"))
    lib.ref_edges.argtypes = [ct.c_int, ct.c_void_p, ct.c_void_p, ct.c_void_p, ct.c_int, ct.c_float, ct.c_int64,
                              ct.c_int64, ct.c_void_p]
    lib.ref_edges.restype = ct.c_int64
    lib.ref_edges_error.restype = ct.c_char_p
    return lib


def ref_edge_list(lib, xyz, cell, backend, cutoff=6.0, grid_bytes=0):
    xyz = np.ascontiguousarray(xyz, np.float32)
    z = np.ones(len(xyz), np.int32)
    cell = np.ascontiguousarray(cell, np.float32)
    cap = 1 << 16
    while True:
        out = np.zeros((cap, 5), np.int32)
        n = lib.ref_edges(len(xyz), xyz.ctypes.data, z.ctypes.data, cell.ctypes.data, backend, cutoff,
                          grid_bytes, cap, out.ctypes.data)
        if n < 0:
            raise RuntimeError(lib.ref_edges_error().decode())
        if n <= cap:
            return out[:n]
        cap = int(n)


def digest(edges):
    return hashlib.sha256(np.ascontiguousarray(edges, np.int32).tobytes()).hexdigest()


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--out", default=str(Path(__file__).resolve().parent))
    ap.add_argument("--configs", default="C1,C2,C3")
    ap.add_argument("--timing-calls", type=int, default=20)
    ap.add_argument("--merge", action="store_true",
                    help="add the configs to the existing ref_summary.json in --out instead of rewriting it "
                         "(skips the scenarios and the CLI case)")
    args = ap.parse_args()
    out = Path(args.out)
    out.mkdir(parents=True, exist_ok=True)
    archive = DATA / "mh1_synth.pwm"
    info = synth.write_archive(archive)
    lib, elib = load_ref(), load_edges()
    if args.merge:
        summary = json.loads((out / "ref_summary.json").read_text())
    else:
        summary = {"archive": info, "nproc": os.cpu_count(), "configs": {}, "edges": {}}
        # Neighbour scenarios (reference traversal on the GPU).
        for name, xyz, cell, cutoff, grid, backends in scenarios.framework_scenarios():
            rec = {}
            for b in backends:
                e = ref_edge_list(elib, xyz, cell, b, cutoff, grid)
                rec[str(b)] = {"count": int(len(e)), "sha256": digest(e)}
            summary["edges"][name] = rec
    for name in args.configs.split(","):
        s = structures.load(name, DATA)
        rec = {"atoms": s.size}
        large = s.size > 20000
        for b in ((2,) if large else (1, 2)):
            e = ref_edge_list(elib, s.positions, s.cell, b)
            rec[f"edges_{b}"] = {"count": int(len(e)), "sha256": digest(e)}
            del e
        backends = (0, 1, 2) if s.size <= 1000 else (0,)
        results = {}
        for b in backends:
            m = RefMH1(lib, archive, b)
            r1 = m.calc(s.positions, s.numbers, s.cell)
            r2 = m.calc(s.positions, s.numbers, s.cell)
            rec[f"repeat_{b}"] = {
                "energy": float(abs(r1["energy"] - r2["energy"])),
                "forces": float(np.abs(r1["forces"] - r2["forces"]).max()),
                "virial": float(np.abs(r1["virial"] - r2["virial"]).max()),
            }
            results[b] = r1
            if b == backends[0]:
                times = []
                for _ in range(3):
                    m.calc(s.positions, s.numbers, s.cell)
                for _ in range(args.timing_calls):
                    t = time.perf_counter()
                    m.calc(s.positions, s.numbers, s.cell)
                    times.append(time.perf_counter() - t)
                med = float(np.median(times))
                rec["timing"] = {"median_s": med, "atoms_evals_per_s": s.size / med,
                                 "device_ms": m.diagnostics()["device_ms"], "calls": args.timing_calls}
                rec["diagnostics"] = m.diagnostics()
            m.close()
        b0 = backends[0]
        r0 = results[b0]
        if large:
            idx = np.sort(np.random.default_rng(4096).choice(s.size, 4096, replace=False)).astype(np.int32)
            np.savez_compressed(out / f"ref_{name}.npz", energy=r0["energy"], virial=r0["virial"], sample=idx,
                                forces_sample=r0["forces"][idx], energies_sample=r0["energies"][idx],
                                energies_sum=np.float64(r0["energies"].astype(np.float64).sum()),
                                forces_sum=r0["forces"].astype(np.float64).sum(0),
                                forces_abs_sum=np.float64(np.abs(r0["forces"].astype(np.float64)).sum()),
                                forces_abs_max=np.float64(np.abs(r0["forces"]).max()))
        else:
            np.savez_compressed(out / f"ref_{name}.npz", energy=r0["energy"], energies=r0["energies"],
                                forces=r0["forces"], virial=r0["virial"])
        for b in backends[1:]:
            rec[f"backend_{b}_vs_{b0}"] = {
                "energy": float(abs(results[b]["energy"] - results[b0]["energy"])),
                "forces": float(np.abs(results[b]["forces"] - results[b0]["forces"]).max()),
            }
        summary["configs"][name] = rec
        print(name, json.dumps(rec)[:400], flush=True)
    if args.merge:
        (out / "ref_summary.json").write_text(json.dumps(summary, indent=1) + "\n")
        print("done")
        return
    # C-ABI behaviour case (native.py-like) and the CLI on C1.
    xyz, z, cell = scenarios.native_case()
    m = RefMH1(lib, archive, 1)
    r = m.calc(xyz, z, cell)
    np.savez_compressed(out / "ref_native.npz", **r)
    m.close()
    arc = out / "C1.arc"
    structures.write_arc(arc, [structures.load("C1", DATA)])
    cli = subprocess.run([str(REF / "mace-main-ref"), str(archive), str(arc), "--json"], capture_output=True,
                         text=True)
    (out / "ref_cli_C1.json").write_text(cli.stdout)
    summary["cli_returncode"] = cli.returncode
    (out / "ref_summary.json").write_text(json.dumps(summary, indent=1) + "\n")
    print("done")


if __name__ == "__main__":
    main()
