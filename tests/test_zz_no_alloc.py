"""GPU test of lapis_neighbor_list_static, the neighbour-list entry point that allocates no
GPU memory (for callers that own all device memory and cannot let a library allocate).

The test (not the entry point) allocates the caller's device buffers with torch, calls the
entry point through the C ABI twice in a row on different structures (the larger first, so a
stale count from the first call would show up in the second), and checks each edge list
against the existing allocating entry point (lapis_neighbor_edges) exactly -- edge sets are
compared bit for bit, as in the other neighbour tests -- and each displacement against the
positions and image shift to 1e-4 A.  It lives in its own file, collected last.
"""
import ctypes as ct

import numpy as np
import pytest

from conftest import DATA
from lasp_b200 import structures

pytestmark = pytest.mark.gpu
MAX_ATOMS = 16384


def bind(library):
    lib = ct.CDLL(str(library))
    lib.lapis_neighbor_list_static.argtypes = [ct.c_int, ct.c_void_p, ct.c_void_p, ct.c_void_p, ct.c_float,
                                               ct.c_void_p, ct.c_void_p, ct.c_void_p, ct.c_void_p, ct.c_longlong,
                                               ct.c_void_p]
    lib.lapis_neighbor_list_static.restype = ct.c_longlong
    lib.mace_last_error.restype = ct.c_char_p
    return lib


def static_edges(lib, s, capacity):
    import torch
    n = s.size
    xyz = torch.from_numpy(np.ascontiguousarray(s.positions)).cuda()
    z = torch.from_numpy(np.ascontiguousarray(s.numbers)).cuda()
    row = torch.full((n + 1,), -7, dtype=torch.int32, device="cuda")
    sender = torch.empty(capacity, dtype=torch.int32, device="cuda")
    shift = torch.empty(capacity * 3, dtype=torch.int32, device="cuda")
    vec = torch.empty(capacity * 4, dtype=torch.float32, device="cuda")
    cell = np.ascontiguousarray(s.cell, np.float32)
    torch.cuda.synchronize()
    count = lib.lapis_neighbor_list_static(n, xyz.data_ptr(), z.data_ptr(), cell.ctypes.data, 6.0, row.data_ptr(),
                                           sender.data_ptr(), shift.data_ptr(), vec.data_ptr(), capacity, None)
    assert count >= 0, lib.mace_last_error().decode()
    return count, row.cpu().numpy(), sender.cpu().numpy(), shift.cpu().numpy().reshape(-1, 3), \
        vec.cpu().numpy().reshape(-1, 4)


def check_against_allocating_entry(library, lib, s):
    from mace_inference import neighbor_edges
    expected = neighbor_edges(s.positions, s.cell, 6.0, 1, library=library)
    count, row, sender, shift, vec = static_edges(lib, s, capacity=len(expected) + 64)
    assert count == len(expected)
    assert row[0] == 0 and row[-1] == count and np.all(np.diff(row) >= 0)
    receiver = np.repeat(np.arange(s.size, dtype=np.int32), np.diff(row))
    got = np.concatenate([receiver[:, None], sender[:count, None], shift[:count]], axis=1)
    order = np.lexsort(got.T[::-1])
    assert np.array_equal(got[order], expected)
    x = s.positions.astype(np.float64)
    d = x[sender[:count]] + shift[:count] @ s.cell.astype(np.float64) - x[receiver]
    assert np.abs(d - vec[:count, :3]).max() < 1e-4
    assert np.abs(np.linalg.norm(vec[:count, :3], axis=1) - vec[:count, 3]).max() < 1e-5
    return count


def test_static_neighbor_list_matches_allocating_entry_twice(library):
    lib = bind(library)
    big, small = structures.load("C2", DATA), structures.load("C1", DATA)
    assert check_against_allocating_entry(library, lib, big) == 97006
    assert check_against_allocating_entry(library, lib, small) == 5126


def test_static_neighbor_list_limits(library):
    lib = bind(library)
    cell = np.eye(3, dtype=np.float32) * 30
    row = ct.c_int(0)
    assert lib.lapis_neighbor_list_static(MAX_ATOMS + 1, None, None, cell.ctypes.data, 6.0, ct.addressof(row),
                                          None, None, None, 0, None) == -1
    assert "16384" in lib.mace_last_error().decode()
    s = structures.load("C1", DATA)
    count, row, *_ = static_edges(lib, s, capacity=10)
    assert count == 5126 and row[-1] == 5126
