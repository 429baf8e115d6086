"""Spatial domain decomposition across GPUs (one process per GPU, NCCL).

Two ranks evaluate the same structure decomposed -- each builds the neighbour rows of the
atoms it owns only, exchanges layer-1 ghost features, their gradients and ghost forces -- and
both must return the full single-GPU result (the same engine; only float32 summation order
differs): energy 1e-6 relative, forces 1e-5 eV/A, per-atom energies 5e-5 eV, virial within
the parity tests' bound for the config.  A rank that stops taking part (it stays alive
between calls, with nothing in flight) makes its peer's next call fail within
MACE_DOMAIN_TIMEOUT_S: the peer aborts its communicator instead of waiting for ever, and the
domain stays failed.  NVLS is off (NCCL_NVLS_ENABLE=0).  Needs two GPUs; skipped otherwise.
"""
import os
import time

import numpy as np
import pytest

from conftest import DATA, ROOT
from lasp_b200 import structures
from test_mh1_gpu import virial_bound

pytestmark = pytest.mark.gpu


def _rank(rank, world, archive, library, nccl_id, names, out):
    import sys
    os.environ["NCCL_NVLS_ENABLE"] = "0"
    sys.path.insert(0, str(ROOT / "lasp-pis_b200" / "python"))
    from mace_inference import NativeMH1
    results = {}
    with NativeMH1(archive, backend=0, library=library, device=rank, domain=(rank, world, nccl_id)) as m:
        for name in names:
            s = structures.load(name, DATA)
            for _ in range(2):  # a repeated call rebuilds the plan and reuses the buffers
                r = m.calculate(s.positions, s.numbers, s.cell)
            results[name] = r
    out.put((rank, results))


def _close(a, b, name):
    assert abs(a["energy"] - b["energy"]) <= 1e-6 * abs(b["energy"])
    assert np.abs(a["forces"] - b["forces"]).max() <= 1e-5
    assert np.abs(a["energies"] - b["energies"]).max() <= 5e-5
    assert np.abs(np.asarray(a["virial"], np.float64) - b["virial"]).max() <= virial_bound(name)


def _spawn(target, args_of, world):
    import torch.multiprocessing as mp
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    procs = [ctx.Process(target=target, args=args_of(r, q)) for r in range(world)]
    for p in procs:
        p.start()
    return procs, q


def test_two_rank_decomposition_matches_single_gpu(library, archive_path):
    import torch
    if torch.cuda.device_count() < 2:
        pytest.skip("needs two GPUs")
    from mace_inference import NativeMH1, nccl_unique_id
    names = ["C2", "C3"]
    with NativeMH1(archive_path, backend=0, library=library, device=0) as m:
        single = {}
        for name in names:
            s = structures.load(name, DATA)
            single[name] = m.calculate(s.positions, s.numbers, s.cell)
    nccl_id = nccl_unique_id(library)
    procs, q = _spawn(_rank, lambda r, q: (r, 2, str(archive_path), str(library), nccl_id, names, q), 2)
    got = dict(q.get(timeout=300) for _ in procs)
    for p in procs:
        p.join(timeout=120)
        assert p.exitcode == 0
    for name in names:
        for rank in (0, 1):
            _close(got[rank][name], single[name], name)


def _rank_that_stops(rank, world, archive, library, nccl_id, out):
    import sys
    os.environ["NCCL_NVLS_ENABLE"] = "0"
    os.environ["MACE_DOMAIN_TIMEOUT_S"] = "5"
    sys.path.insert(0, str(ROOT / "lasp-pis_b200" / "python"))
    from mace_inference import NativeMH1
    s = structures.load("C2", DATA)
    m = NativeMH1(archive, backend=0, library=library, device=rank, domain=(rank, world, nccl_id))
    m.calculate(s.positions, s.numbers, s.cell)  # both ranks take part in the first call
    if rank == 1:
        # Leaves between calls: nothing in flight, never joins the next call.
        out.put((rank, "left", 0.0, ""))
        out.close()
        out.join_thread()
        time.sleep(20)
        os._exit(0)
    t0 = time.monotonic()
    try:
        m.calculate(s.positions, s.numbers, s.cell)
        status, message = "returned", ""
    except RuntimeError as e:
        status, message = "error", str(e)
    dt = time.monotonic() - t0
    try:  # the domain stays failed: the next call is refused at once
        m.calculate(s.positions, s.numbers, s.cell)
        again = "returned"
    except RuntimeError as e:
        again = str(e)
    m.close()
    out.put((rank, status, dt, message + " | " + again))
    out.close()
    out.join_thread()
    os._exit(0)


def test_peer_that_stops_times_out_cleanly(library, archive_path):
    import torch
    if torch.cuda.device_count() < 2:
        pytest.skip("needs two GPUs")
    from mace_inference import nccl_unique_id
    nccl_id = nccl_unique_id(library)
    procs, q = _spawn(_rank_that_stops, lambda r, q: (r, 2, str(archive_path), str(library), nccl_id, q), 2)
    got = {}
    for _ in procs:
        rank, status, dt, message = q.get(timeout=120)
        got[rank] = (status, dt, message)
    for p in procs:
        p.join(timeout=60)
    status, dt, message = got[0]
    assert status == "error", got
    assert "did not take part" in message and "failed earlier" in message, message
    assert 4.0 <= dt <= 60.0, dt
