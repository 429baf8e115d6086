"""ctypes binding of the C ABI (include/mace/c_api.h); raises RuntimeError on failure."""
from __future__ import annotations

import ctypes as ct
import json

import numpy as np

from .library import library_path

_libs: dict[str, ct.CDLL] = {}


def load(path=None) -> ct.CDLL:
    path = str(path or library_path())
    if path in _libs:
        return _libs[path]
    lib = ct.CDLL(path)
    lib.mace_create_mh1.argtypes = [ct.c_char_p, ct.c_int]
    lib.mace_create_mh1.restype = ct.c_void_p
    lib.mace_create_mh1_head.argtypes = [ct.c_char_p, ct.c_int, ct.c_char_p]
    lib.mace_create_mh1_head.restype = ct.c_void_p
    lib.mace_create_mh1_device.argtypes = [ct.c_char_p, ct.c_int, ct.c_int]
    lib.mace_create_mh1_device.restype = ct.c_void_p
    lib.mace_create_mh1_device_head.argtypes = [ct.c_char_p, ct.c_int, ct.c_char_p, ct.c_int]
    lib.mace_create_mh1_device_head.restype = ct.c_void_p
    lib.mace_destroy.argtypes = [ct.c_void_p]
    lib.mace_destroy.restype = None
    lib.mace_last_error.restype = ct.c_char_p
    lib.mace_calculate.argtypes = [ct.c_void_p, ct.c_int] + [ct.c_void_p] * 7
    lib.mace_calculate.restype = ct.c_int
    lib.mace_calculate_device.argtypes = [ct.c_void_p, ct.c_int] + [ct.c_void_p] * 7
    lib.mace_calculate_device.restype = ct.c_int
    lib.mace_create_mh1_domain.argtypes = [ct.c_char_p, ct.c_int, ct.c_int, ct.c_int, ct.c_int, ct.c_char_p]
    lib.mace_create_mh1_domain.restype = ct.c_void_p
    lib.mace_nccl_unique_id.argtypes = [ct.c_void_p]
    lib.mace_nccl_unique_id.restype = ct.c_int
    lib.mace_calculate_batch.argtypes = [ct.c_void_p, ct.c_int] + [ct.c_void_p] * 8
    lib.mace_calculate_batch.restype = ct.c_int
    lib.mace_diagnostics.argtypes = [ct.c_void_p, ct.c_void_p, ct.c_size_t]
    lib.mace_diagnostics.restype = ct.c_int
    lib.mace_profile.argtypes = [ct.c_void_p, ct.c_int]
    lib.mace_profile.restype = ct.c_int
    lib.mace_last_edges.argtypes = [ct.c_void_p, ct.c_void_p, ct.c_longlong]
    lib.mace_last_edges.restype = ct.c_longlong
    lib.lapis_neighbor_edges.argtypes = [ct.c_int, ct.c_void_p, ct.c_void_p, ct.c_float, ct.c_int, ct.c_longlong,
                                         ct.c_void_p, ct.c_longlong]
    lib.lapis_neighbor_edges.restype = ct.c_longlong
    lib.mace_check_model.argtypes = [ct.c_char_p, ct.c_char_p]
    lib.mace_check_model.restype = ct.c_int
    _libs[path] = lib
    return lib


def _error(lib) -> str:
    return lib.mace_last_error().decode()


def neighbor_edges(xyz, cell, cutoff=6.0, backend=0, grid_bytes=0, library=None):
    """Canonical directed edges int32 [E, 5] (receiver, sender, sx, sy, sz) of the Lapis list."""
    lib = load(library)
    xyz = np.ascontiguousarray(xyz, np.float32).reshape(-1, 3)
    cell = np.ascontiguousarray(cell, np.float32).reshape(3, 3)
    count = lib.lapis_neighbor_edges(len(xyz), xyz.ctypes.data, cell.ctypes.data, cutoff, backend, grid_bytes,
                                     None, 0)
    if count < 0:
        raise RuntimeError(_error(lib))
    out = np.zeros((max(count, 1), 5), np.int32)
    lib.lapis_neighbor_edges(len(xyz), xyz.ctypes.data, cell.ctypes.data, cutoff, backend, grid_bytes,
                             out.ctypes.data, count)
    return out[:count]


def check_model(model, head=None, library=None) -> None:
    """Parse and validate a model (archive or MH1 checkpoint for ``head``) as the
    constructors do, without a GPU; raises RuntimeError with the loader's message."""
    lib = load(library)
    if lib.mace_check_model(str(model).encode(), None if head is None else head.encode()):
        raise RuntimeError(_error(lib))


def nccl_unique_id(library=None) -> bytes:
    """A new 128-byte NCCL id for ``NativeMH1(..., domain=(rank, world, id))`` (make it on one
    rank and pass it to all)."""
    lib = load(library)
    buf = ct.create_string_buffer(128)
    if lib.mace_nccl_unique_id(buf):
        raise RuntimeError(_error(lib))
    return buf.raw


class NativeMH1:
    """One MH1 handle: ``calculate(xyz, z, cell)`` -> energy, energies, forces, virial.

    ``domain=(rank, world, nccl_id)`` decomposes each structure across ``world`` ranks (one
    process per GPU, ``device`` required): every rank calls with the same full structure and
    gets the full result; calls are collective."""

    def __init__(self, archive, backend=0, library=None, device=None, head=None, domain=None):
        self.lib = load(library)
        b = {"auto": 0, "brute": 1, "cell": 2}.get(backend, backend)
        if domain is not None:
            rank, world, nccl_id = domain
            if device is None or len(nccl_id) != 128:
                raise ValueError("domain decomposition needs a device and a 128-byte NCCL id")
            self.handle = self.lib.mace_create_mh1_domain(str(archive).encode(), b, device, rank, world,
                                                          ct.c_char_p(bytes(nccl_id)))
        elif device is not None:
            self.handle = self.lib.mace_create_mh1_device_head(
                str(archive).encode(), b, None if head is None else head.encode(), device)
        elif head is not None:
            self.handle = self.lib.mace_create_mh1_head(str(archive).encode(), b, head.encode())
        else:
            self.handle = self.lib.mace_create_mh1(str(archive).encode(), b)
        if not self.handle:
            raise RuntimeError(_error(self.lib))

    def _call(self, fn, n, xyz_ptr, z_ptr, cell):
        cell = np.ascontiguousarray(cell, np.float32).reshape(3, 3)
        energy = np.zeros(1, np.float64)
        atomic = np.zeros(n, np.float32)
        forces = np.zeros((n, 3), np.float32)
        virial = np.zeros((3, 3), np.float32)
        if fn(self.handle, n, xyz_ptr, z_ptr, cell.ctypes.data, energy.ctypes.data, atomic.ctypes.data,
              forces.ctypes.data, virial.ctypes.data):
            raise RuntimeError(_error(self.lib))
        return dict(energy=float(energy[0]), energies=atomic, forces=forces, virial=virial)

    def calculate(self, xyz, z, cell):
        xyz = np.ascontiguousarray(xyz, np.float32).reshape(-1, 3)
        z = np.ascontiguousarray(z, np.int32)
        return self._call(self.lib.mace_calculate, len(z), xyz.ctypes.data, z.ctypes.data, cell)

    def calculate_batch(self, cells):
        """Independent periodic cells in one call: ``cells`` is a sequence of (xyz, Z, cell).
        Returns one result dict per cell (as calculate)."""
        sizes = np.array([len(z) for _, z, _ in cells], np.int32)
        total = int(sizes.sum())
        xyz = np.ascontiguousarray(np.concatenate([np.asarray(x, np.float32).reshape(-1, 3) for x, _, _ in cells])
                                   if total else np.zeros((0, 3), np.float32), np.float32)
        z = np.ascontiguousarray(np.concatenate([np.asarray(q, np.int32) for _, q, _ in cells])
                                 if total else np.zeros(0, np.int32), np.int32)
        h = np.ascontiguousarray(np.stack([np.asarray(c, np.float32).reshape(3, 3) for _, _, c in cells])
                                 if len(cells) else np.zeros((0, 3, 3), np.float32), np.float32)
        count = len(cells)
        energies = np.zeros(max(count, 1), np.float64)
        per_atom = np.zeros(max(total, 1), np.float32)
        forces = np.zeros((max(total, 1), 3), np.float32)
        virials = np.zeros((max(count, 1), 3, 3), np.float32)
        if self.lib.mace_calculate_batch(self.handle, count, sizes.ctypes.data, xyz.ctypes.data, z.ctypes.data,
                                         h.ctypes.data, energies.ctypes.data, per_atom.ctypes.data,
                                         forces.ctypes.data, virials.ctypes.data):
            raise RuntimeError(_error(self.lib))
        out, first = [], 0
        for c, n in enumerate(sizes):
            out.append({"energy": float(energies[c]), "energies": per_atom[first:first + n].copy(),
                        "forces": forces[first:first + n].copy(), "virial": virials[c].copy()})
            first += int(n)
        return out

    def calculate_device(self, n, xyz_ptr, z_ptr, cell):
        """Device-resident inputs (raw device pointers on the handle's GPU)."""
        return self._call(self.lib.mace_calculate_device, n, xyz_ptr, z_ptr, cell)

    def profile(self, enable=True):
        if self.lib.mace_profile(self.handle, int(enable)):
            raise RuntimeError(_error(self.lib))

    def last_edges(self):
        count = self.lib.mace_last_edges(self.handle, None, 0)
        if count < 0:
            raise RuntimeError(_error(self.lib))
        out = np.zeros((max(count, 1), 5), np.int32)
        self.lib.mace_last_edges(self.handle, out.ctypes.data, count)
        return out[:count]

    @property
    def diagnostics(self):
        buf = ct.create_string_buffer(1 << 16)
        if self.lib.mace_diagnostics(self.handle, buf, len(buf)):
            raise RuntimeError(_error(self.lib))
        return json.loads(buf.value)

    def close(self):
        if getattr(self, "handle", None):
            self.lib.mace_destroy(self.handle)
            self.handle = None

    def __enter__(self):
        return self

    def __exit__(self, *args):
        self.close()

    def __del__(self):
        self.close()
