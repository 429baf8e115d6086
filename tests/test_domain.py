"""Spatial domain decomposition across GPUs (one process per GPU, NCCL).

Two ranks evaluate the same structure decomposed (each owns half of the atoms, exchanges
layer-1 ghost features, their gradients and ghost forces) and both must return the full
single-GPU result: energy 1e-6 relative, forces 1e-5 x max(1, |F|), per-atom energies 5e-5,
virial 2e-6 x max|W| (float32 summation order differs).  Needs two GPUs; skipped otherwise.
"""
import numpy as np
import pytest

from conftest import DATA, ROOT
from lasp_b200 import structures

pytestmark = pytest.mark.gpu


def _rank(rank, world, archive, library, nccl_id, names, out):
    import sys
    sys.path.insert(0, str(ROOT / "lasp-pis_b200" / "python"))
    from mace_inference import NativeMH1
    results = {}
    with NativeMH1(archive, backend=0, library=library, device=rank, domain=(rank, world, nccl_id)) as m:
        for name in names:
            s = structures.load(name, DATA)
            for _ in range(2):  # a repeated call reuses the exchange plan and buffers
                r = m.calculate(s.positions, s.numbers, s.cell)
            results[name] = r
    out.put((rank, results))


def _close(a, b):
    assert abs(a["energy"] - b["energy"]) <= 1e-6 * abs(b["energy"])
    assert np.abs(a["forces"] - b["forces"]).max() <= 1e-5 * max(1.0, float(np.abs(b["forces"]).max()))
    assert np.abs(a["energies"] - b["energies"]).max() <= 5e-5
    assert np.abs(a["virial"] - b["virial"]).max() <= 2e-6 * float(np.abs(b["virial"]).max())


def test_two_rank_decomposition_matches_single_gpu(library, archive_path):
    import torch
    if torch.cuda.device_count() < 2:
        pytest.skip("needs two GPUs")
    import torch.multiprocessing as mp
    from mace_inference import NativeMH1, nccl_unique_id
    names = ["C2", "C3"]
    with NativeMH1(archive_path, backend=0, library=library, device=0) as m:
        single = {}
        for name in names:
            s = structures.load(name, DATA)
            single[name] = m.calculate(s.positions, s.numbers, s.cell)
    nccl_id = nccl_unique_id(library)
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    procs = [ctx.Process(target=_rank, args=(r, 2, str(archive_path), str(library), nccl_id, names, q))
             for r in range(2)]
    for p in procs:
        p.start()
    got = dict(q.get(timeout=300) for _ in procs)
    for p in procs:
        p.join(timeout=120)
        assert p.exitcode == 0
    for name in names:
        for rank in (0, 1):
            _close(got[rank][name], single[name])
