"""Neighbour-list scenarios shared by the golden-fixture script and the tests.

The scenario shapes follow the reference's edge-multiset tests
(lapis/tests/framework.cu:109-158, 217-250): cubic cells of 1.6 / 2.7 / 5.3 / 9.1 A, a
triclinic cell, unwrapped coordinates, a sparse 200 A cell with a 1024-byte grid budget, 145
clustered atoms and an empty cell, all at a 2.5 A cutoff; then fully accepted candidate
batches of 1..145 atoms (queue boundaries) and the inclusive cutoff.  Coordinates are drawn
here from numpy with a fixed seed (the reference uses its own generator).
"""
from __future__ import annotations

import numpy as np


def framework_scenarios():
    """Yield (name, xyz float32 [n,3], cell float32 [3,3], cutoff, grid_bytes, backends)."""
    rng = np.random.default_rng(123)
    for scenario in range(8):
        n = 0 if scenario == 7 else 145 if scenario == 6 else 11
        h = 1.6 if scenario == 0 else 2.7 if scenario == 1 else 5.3 if scenario == 2 else 9.1
        cell = np.array([[h, 0, 0], [2.0 if scenario == 3 else 0.0, h, 0],
                         [-1.0 if scenario == 3 else 0.0, 1.0 if scenario == 3 else 0.0, h]])
        if scenario == 5:
            cell = np.diag([200.0, 210.0, 220.0])
        f = rng.uniform(0.01, 0.99, size=(n, 3))
        if scenario == 6:
            f *= 0.1
        if scenario == 4:
            f[:, 0] += np.arange(n) % 3 - 1
        cell = cell.astype(np.float32)
        xyz = (f.astype(np.float32) @ cell).astype(np.float32)
        backends = [1, 0] + ([2] if h >= 2.5 and scenario != 0 else [])
        yield f"scenario{scenario}", xyz, cell, 2.5, (1024 if scenario == 5 else 0), backends
    box = np.eye(3, dtype=np.float32) * 8
    for count in (1, 2, 17, 18, 33, 34, 35, 128, 129, 144, 145):
        xyz = np.ones((count, 3), np.float32)
        xyz[:, 0] += np.arange(count, dtype=np.float32) * np.float32(1e-4)
        yield f"queue{count}", xyz, box, 0.5, 0, [0]
    for label, x in (("inclusive", np.float32(2.5)), ("above", np.nextafter(np.float32(2.5), np.float32(3))),
                     ("below", np.nextafter(np.float32(2.5), np.float32(2)))):
        xyz = np.array([[0, 0, 0], [x, 0, 0]], np.float32)
        yield f"cutoff_{label}", xyz, box, 2.5, 0, [0]


def native_case():
    """Four atoms in a triclinic cell (the C-ABI check of mace/tests/native.py:41-72)."""
    cell = np.array([[8.4, 0, 0], [1.1, 8.7, 0], [-0.8, 0.4, 9.2]], np.float32)
    xyz = np.array([[1, 1, 1], [2.5, 1.2, 1], [2.3, 2.7, 1.3], [3.1, 3.1, 1.5]], np.float32)
    z = np.array([14, 6, 8, 1], np.int32)
    return xyz, z, cell
