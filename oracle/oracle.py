"""ctypes binding of the CPU float64 oracle (liboracle_mh1.so).

TEST INFRASTRUCTURE ONLY: imported by tests/, __graft_entry__.smoke() and the CPU-baseline
leg of bench.py.  It restates the reference's MH1 evaluation and neighbour semantics
(see mh1_oracle.c for the per-function reference citations).
"""
from __future__ import annotations

import ctypes as ct
import subprocess
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent
LIB = HERE / "liboracle_mh1.so"


def build() -> Path:
    subprocess.run(["make", "-s", "-C", str(HERE)], check=True)
    return LIB


_lib = None


def lib():
    global _lib
    if _lib is None:
        if not LIB.exists():
            build()
        l = ct.CDLL(str(LIB))
        l.oracle_load.argtypes = [ct.c_char_p, ct.c_char_p, ct.c_int]
        l.oracle_load.restype = ct.c_void_p
        l.oracle_free.argtypes = [ct.c_void_p]
        l.oracle_edges.argtypes = [ct.c_int, ct.c_void_p, ct.c_void_p, ct.c_float, ct.c_int, ct.c_int64,
                                   ct.c_void_p, ct.c_void_p, ct.c_char_p, ct.c_int]
        l.oracle_edges.restype = ct.c_int64
        l.oracle_calculate.argtypes = [ct.c_void_p, ct.c_int] + [ct.c_void_p] * 3 + [ct.c_int] + \
            [ct.c_void_p] * 4 + [ct.c_char_p, ct.c_int]
        l.oracle_calculate.restype = ct.c_int
        l.oracle_threads.argtypes = [ct.c_int]
        l.oracle_threads.restype = ct.c_int
        _lib = l
    return _lib


def threads(n: int = 0) -> int:
    return lib().oracle_threads(n)


def _f32(a, shape=None):
    a = np.ascontiguousarray(a, dtype=np.float32)
    return a.reshape(shape) if shape else a


def edges(xyz, cell, cutoff=6.0, backend=0):
    """Canonically sorted directed edges: int32 [E, 5] (i, j, sx, sy, sz), float32 d [E, 3]."""
    xyz = _f32(xyz, (-1, 3))
    cell = _f32(cell, (3, 3))
    err = ct.create_string_buffer(512)
    n = xyz.shape[0]
    count = lib().oracle_edges(n, xyz.ctypes.data, cell.ctypes.data, cutoff, backend, 0, None, None, err, 512)
    if count < 0:
        raise RuntimeError(err.value.decode())
    out = np.zeros((count, 5), np.int32)
    disp = np.zeros((count, 3), np.float32)
    lib().oracle_edges(n, xyz.ctypes.data, cell.ctypes.data, cutoff, backend, count, out.ctypes.data,
                       disp.ctypes.data, err, 512)
    return out, disp


class Oracle:
    """Float64 MH1 restatement: calculate() mirrors mace_calculate()'s outputs."""

    def __init__(self, archive):
        err = ct.create_string_buffer(512)
        self.handle = lib().oracle_load(str(archive).encode(), err, 512)
        if not self.handle:
            raise RuntimeError(err.value.decode())

    def calculate(self, xyz, z, cell, backend=0):
        xyz = _f32(xyz, (-1, 3))
        z = np.ascontiguousarray(z, dtype=np.int32)
        cell = _f32(cell, (3, 3))
        n = z.size
        energy = np.zeros(1)
        atomic = np.zeros(n)
        forces = np.zeros((n, 3))
        virial = np.zeros((3, 3))
        err = ct.create_string_buffer(512)
        rc = lib().oracle_calculate(self.handle, n, xyz.ctypes.data, z.ctypes.data, cell.ctypes.data, backend,
                                    energy.ctypes.data, atomic.ctypes.data, forces.ctypes.data,
                                    virial.ctypes.data, err, 512)
        if rc:
            raise RuntimeError(err.value.decode())
        return dict(energy=float(energy[0]), energies=atomic, forces=forces, virial=virial)

    def close(self):
        if self.handle:
            lib().oracle_free(self.handle)
            self.handle = None

    def __del__(self):
        self.close()
