"""Real spherical harmonics (l <= 3) and real-basis Wigner 3j symbols, in numpy.

The spherical-harmonic polynomials follow the e3nn "component" convention that the
reference evaluates on the device (mace/src/mh1_math.cuh:54-86): l=1 is (x, y, z) and
every degree l is scaled by sqrt(2l+1).  The 3j symbols are computed numerically as the
one-dimensional invariant subspace of D^l1 (x) D^l2 (x) D^l3, with the representation
matrices D^l(R) fitted from those same polynomials, and normalised to unit Frobenius
norm like e3nn's ``wigner_3j``.  The tests
compare the resulting table with the e3nn 0.4.4 constants the reference ships
(mace/src/cg.inc, produced by mace/tools/generate_cg.py).
"""
from __future__ import annotations

import functools
import itertools

import numpy as np

S3 = np.sqrt(3.0)


def sh(v: np.ndarray) -> np.ndarray:
    """Component-normalised real harmonics of the unit vectors v[..., 3] -> [..., 16]."""
    x, y, z = v[..., 0], v[..., 1], v[..., 2]
    yy = y * y
    xxzz = x * x + z * z
    out = np.empty(v.shape[:-1] + (16,))
    out[..., 0] = 1.0
    out[..., 1], out[..., 2], out[..., 3] = x, y, z
    s4 = S3 * x * z
    s8 = S3 / 2 * (z * z - x * x)
    out[..., 4] = s4
    out[..., 5] = S3 * x * y
    out[..., 6] = yy - 0.5 * xxzz
    out[..., 7] = S3 * y * z
    out[..., 8] = s8
    out[..., 9] = np.sqrt(5.0 / 6.0) * (s4 * z + s8 * x)
    out[..., 10] = np.sqrt(5.0) * s4 * y
    out[..., 11] = np.sqrt(3.0 / 8.0) * (4 * yy - xxzz) * x
    out[..., 12] = 0.5 * y * (2 * yy - 3 * xxzz)
    out[..., 13] = np.sqrt(3.0 / 8.0) * z * (4 * yy - xxzz)
    out[..., 14] = np.sqrt(5.0) * s8 * y
    out[..., 15] = np.sqrt(5.0 / 6.0) * (s8 * z - s4 * x)
    for l in (1, 2, 3):
        out[..., l * l:(l + 1) * (l + 1)] *= np.sqrt(2 * l + 1)
    return out


def _random_rotation(rng: np.random.Generator) -> np.ndarray:
    q, r = np.linalg.qr(rng.normal(size=(3, 3)))
    q *= np.sign(np.diag(r))
    if np.linalg.det(q) < 0:
        q[:, 0] = -q[:, 0]
    return q


def wigner_d(l: int, rot: np.ndarray) -> np.ndarray:
    """D^l(R) with Y_l(R v) = D^l(R) Y_l(v), fitted by least squares."""
    rng = np.random.default_rng(7)
    v = rng.normal(size=(64, 3))
    v /= np.linalg.norm(v, axis=1, keepdims=True)
    sl = slice(l * l, (l + 1) * (l + 1))
    a = sh(v)[:, sl]
    b = sh(v @ rot.T)[:, sl]
    d, *_ = np.linalg.lstsq(a, b, rcond=None)
    return d.T


@functools.lru_cache(maxsize=None)
def wigner_3j(l1: int, l2: int, l3: int) -> np.ndarray:
    """Real-basis 3j tensor C[a, b, c] of unit Frobenius norm (zero if not a triangle)."""
    dims = (2 * l1 + 1, 2 * l2 + 1, 2 * l3 + 1)
    if not abs(l1 - l2) <= l3 <= l1 + l2:
        return np.zeros(dims)
    rng = np.random.default_rng(11)
    rows = []
    for _ in range(4):
        rot = _random_rotation(rng)
        k = np.kron(np.kron(wigner_d(l1, rot), wigner_d(l2, rot)), wigner_d(l3, rot))
        rows.append(k - np.eye(k.shape[0]))
    _, s, vt = np.linalg.svd(np.concatenate(rows))
    c = vt[-1].reshape(dims)
    c[np.abs(c) < 1e-9] = 0.0
    c /= np.linalg.norm(c)
    flat = c.ravel()
    k = int(np.argmax(np.abs(flat) > np.abs(flat).max() - 1e-9))
    # Sign convention: the entry of largest magnitude (first in (a, b, c) order among
    # ties) is positive.  This reproduces every e3nn 0.4.4 coupling in the reference table.
    c *= np.sign(flat[k])
    return c


def rotation(seed: int) -> np.ndarray:
    return _random_rotation(np.random.default_rng(seed))


def coupling_table():
    """Rows (l1, l2, lo, a, b, c, value) for l1 <= 1, l2 <= 3, lo <= 3 in cg.inc's order."""
    rows = []
    for l1 in (0, 1):
        for l2 in range(4):
            for lo in range(abs(l1 - l2), min(3, l1 + l2) + 1):
                c = wigner_3j(l1, l2, lo)
                for a, b, cc in itertools.product(*(range(n) for n in c.shape)):
                    if abs(c[a, b, cc]) > 1e-14:
                        rows.append((l1, l2, lo, a, b, cc, float(c[a, b, cc])))
    return rows
