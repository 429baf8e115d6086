"""Lapis PairOp extension API and its Lennard-Jones example (reference: lapis/include/lapis/pair.cuh,
lapis/docs/PAIR_OP.md, lapis/examples/lj/lj.cu, lapis/tests/framework.cu).

CPU: an external CUDA client in the shape of the reference's packaging check
(tools/check_packages.py:70-82) compiles against include/lapis/pair.cuh for sm_100a, and the
library exports the LJ entry point.
GPU: the native framework test (edge semantics through an edge-collecting operation, tile
boundaries, inclusive cutoff, LJ derivatives, reuse, single flight, resource and geometry
errors) and LJ energies/forces/virial against a float64 enumeration of all periodic images
(tolerance: 1e-5 relative energy, 1e-4 relative to max|F| and max|W|).
"""
import ctypes as ct
import shutil
import subprocess

import numpy as np
import pytest

from conftest import ROOT

EXTENSION = r"""
#include <lapis/pair.cuh>
struct Op {
  static constexpr int threads = 32, tile_edges = 4, scratch_alignment = 16;
  static const char *name() { return "external"; }
  struct State {};
  lapis::WorkspaceSpec plan(int) const { return {}; }
  void setup(lapis::Context &, void *) {}
  void postprocess(lapis::Context &, void *) {}
  __device__ void prepare(int, State &, void *) {}
  template <class Tile> __device__ void consume(int, const Tile &, State &, void *) {}
  __device__ void finalize(int, State &, void *) {}
};
void launch(lapis::Context &ctx) { lapis::execute(ctx, Op{}); }
"""


@pytest.mark.skipif(shutil.which("nvcc") is None, reason="nvcc absent")
def test_external_extension_compiles(tmp_path):
    src = tmp_path / "extension.cu"
    src.write_text(EXTENSION)
    r = subprocess.run(["nvcc", "-std=c++17", "-gencode", "arch=compute_100a,code=sm_100a", "-I",
                        str(ROOT / "include"), "-c", str(src), "-o", str(tmp_path / "extension.o")],
                       capture_output=True, text=True)
    assert r.returncode == 0, r.stderr[-3000:]


def test_library_exports_lj(library):
    lib = ct.CDLL(str(library))
    assert hasattr(lib, "lapis_lj_calculate")


def lj_reference(xyz, cell, eps, sigma, rc):
    """Force-shifted LJ over every periodic image within rc (float64): half of each directed
    edge's energy and virial to the receiver, the full edge force on the receiver."""
    n = len(xyz)
    inv = np.linalg.inv(cell)
    heights = 1.0 / np.linalg.norm(inv, axis=0)
    images = np.ceil(rc / heights).astype(int)
    a6 = (sigma / rc) ** 6
    uc, duc = 4 * eps * (a6 * a6 - a6), 24 * eps * (a6 - 2 * a6 * a6) / rc
    e = np.zeros(n)
    f = np.zeros((n, 3))
    w = np.zeros((3, 3))
    shifts = np.array([(x, y, z) for x in range(-images[0], images[0] + 1)
                       for y in range(-images[1], images[1] + 1) for z in range(-images[2], images[2] + 1)])
    for i in range(n):
        d = xyz[None, :, :] + (shifts @ cell)[:, None, :] - xyz[i]
        r2 = (d ** 2).sum(-1)
        ok = r2 <= rc * rc
        ok[np.all(shifts == 0, axis=1), i] = False
        d, r2 = d[ok], r2[ok]
        r = np.sqrt(r2)
        q6 = (sigma * sigma / r2) ** 3
        u = 4 * eps * (q6 * q6 - q6) - uc - (r - rc) * duc
        du = 24 * eps * (q6 - 2 * q6 * q6) / r - duc
        e[i] = 0.5 * u.sum()
        f[i] = (du[:, None] * d / r[:, None]).sum(0)
        w -= 0.5 * np.einsum("e,ek,el->kl", du / r, d, d)
    return e.sum(), e, f, w


def lj_call(library, xyz, z, cell, eps, sigma, rc, backend=0):
    lib = ct.CDLL(str(library))
    f = lib.lapis_lj_calculate
    f.restype = ct.c_int
    P = np.ctypeslib.ndpointer
    f.argtypes = [ct.c_int, P(np.float32), P(np.int32), P(np.float32), ct.c_float, ct.c_float, ct.c_float,
                  ct.c_int, ct.POINTER(ct.c_double), P(np.float32), P(np.float32), P(np.float32)]
    n = len(xyz)
    energy = ct.c_double()
    per = np.zeros(n, np.float32)
    force = np.zeros((n, 3), np.float32)
    vir = np.zeros(9, np.float32)
    rc_ = f(n, np.ascontiguousarray(xyz, np.float32), np.ascontiguousarray(z, np.int32),
            np.ascontiguousarray(cell, np.float32).ravel(), eps, sigma, rc, backend, ct.byref(energy), per, force,
            vir)
    if rc_:
        lib.mace_last_error.restype = ct.c_char_p
        raise RuntimeError(lib.mace_last_error().decode())
    return energy.value, per, force, vir.reshape(3, 3)


@pytest.mark.gpu
def test_framework_native():
    exe = ROOT / "lasp-pis_b200" / "bin" / "lapis-framework"
    r = subprocess.run([str(exe)], capture_output=True, text=True, timeout=300)
    assert r.returncode == 0, r.stdout + r.stderr
    assert "resource limits and geometry errors passed" in r.stdout


@pytest.mark.gpu
@pytest.mark.parametrize("backend", [0, 1, 2])
def test_lj_matches_float64(library, backend):
    rng = np.random.default_rng(7)
    cell = np.array([[9.0, 0.0, 0.0], [1.2, 8.5, 0.0], [-0.7, 0.9, 9.4]])
    n = 120
    frac = rng.random((n, 3))
    xyz = (frac @ cell).astype(np.float32)
    # keep pairs apart (no overlapping atoms) for a well-conditioned potential
    for _ in range(200):
        d = xyz[:, None, :] - xyz[None, :, :]
        d -= np.round(d @ np.linalg.inv(cell)) @ cell
        r = np.sqrt((d ** 2).sum(-1)) + np.eye(n) * 10
        bad = np.argwhere(r < 1.0)
        if not len(bad):
            break
        xyz[bad[:, 0]] += rng.normal(scale=0.3, size=(len(bad), 3)).astype(np.float32)
    z = np.full(n, 18, np.int32)
    e, per, f, w = lj_call(library, xyz, z, cell, 0.8, 1.1, 3.0, backend)
    re, rper, rf, rw = lj_reference(xyz.astype(np.float64), cell.astype(np.float32).astype(np.float64), 0.8, 1.1,
                                    3.0)
    assert abs(e - re) <= 1e-5 * abs(re) + 1e-6
    assert np.abs(per - rper).max() <= 1e-5 * np.abs(rper).max() + 1e-6
    assert np.abs(f - rf).max() <= 1e-4 * np.abs(rf).max()
    assert np.abs(w - rw).max() <= 1e-4 * np.abs(rw).max()
