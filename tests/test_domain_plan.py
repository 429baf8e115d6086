"""The exchange plan of the domain decomposition, on CPU (host rules, gloo ranks) and on one GPU.

Rank r of W owns the ids [n r / W, n (r + 1) / W).  Its ghosts are the foreign senders of its
edges (ascending); its sends to peer q are its receivers with an edge from one of q's atoms
(ascending).  Because every edge has its reverse, rank r's sends to q must equal q's ghost
block from r element for element -- the owner ships exactly the rows the peer stores, in the
peer's order.  The CPU tests check that rule on the float64 oracle's edge lists with the
library's host implementation (lapis_exchange_plan_host), also across gloo ranks that
exchange their lists; a rank that never sends makes its peer fail within the deadline
instead of waiting forever.  The GPU test checks that the device plan (the partitioned
neighbour list and plan kernels of a decomposed evaluation, lapis_exchange_plan) equals the
host rules on the same rows and that the ranks' rows together are the full edge list.
"""
import ctypes as ct
import datetime
import os
import time

import numpy as np
import pytest

import oracle as O
from conftest import DATA
from lasp_b200 import structures


def _lib(library):
    lib = ct.CDLL(str(library))
    lib.lapis_exchange_plan_host.argtypes = [ct.c_int] * 3 + [ct.c_void_p] * 6 + [ct.c_longlong]
    lib.lapis_exchange_plan_host.restype = ct.c_int
    lib.lapis_exchange_plan.argtypes = [ct.c_int, ct.c_void_p, ct.c_void_p, ct.c_float, ct.c_int, ct.c_int] + \
        [ct.c_void_p] * 7 + [ct.c_longlong]
    lib.lapis_exchange_plan.restype = ct.c_longlong
    lib.mace_last_error.restype = ct.c_char_p
    return lib


def bounds(n, world):
    return [n * r // world for r in range(world + 1)]


def local_rows(edges, n, rank, world):
    """CSR of rank's receivers from a canonical [E, 5] edge list (receiver-sorted)."""
    b = bounds(n, world)
    mine = edges[(edges[:, 0] >= b[rank]) & (edges[:, 0] < b[rank + 1])]
    counts = np.bincount(mine[:, 0] - b[rank], minlength=b[rank + 1] - b[rank])
    row = np.concatenate([[0], np.cumsum(counts)]).astype(np.int32)
    return row, np.ascontiguousarray(mine[:, 1], np.int32)


def host_plan(lib, n, rank, world, row, sender):
    sc, gc = np.zeros(world, np.int32), np.zeros(world, np.int32)
    cap = max(n, len(sender), 1)
    ghosts, sends = np.zeros(cap, np.int32), np.zeros(cap, np.int32)
    assert lib.lapis_exchange_plan_host(n, rank, world, row.ctypes.data, sender.ctypes.data, sc.ctypes.data,
                                        gc.ctypes.data, ghosts.ctypes.data, sends.ctypes.data, cap) == 0, \
        lib.mace_last_error()
    return split_plan(sc, gc, ghosts, sends, rank, world)


def split_plan(sc, gc, ghosts, sends, rank, world):
    """Per-peer lists: sends[q] and ghost blocks ghost[q] (empty for q == rank)."""
    out_s, out_g, a, b = {}, {}, 0, 0
    for q in range(world):
        out_s[q] = sends[a:a + sc[q]].copy()
        out_g[q] = ghosts[b:b + gc[q]].copy()
        a += sc[q]
        b += gc[q]
    return out_s, out_g


def check_pairwise(plans, world):
    for r in range(world):
        for q in range(world):
            if q == r:
                assert len(plans[r][0][q]) == 0 and len(plans[r][1][q]) == 0
                continue
            np.testing.assert_array_equal(plans[r][0][q], plans[q][1][r])


@pytest.fixture(scope="module")
def c2_edges():
    s = structures.load("C2", DATA)
    O.build()
    return s.size, O.edges(s.positions, s.cell, 6.0)[0]


@pytest.mark.parametrize("world", [2, 3, 4, 7])
def test_host_plan_is_pairwise_consistent(library, c2_edges, world):
    n, edges = c2_edges
    lib = _lib(library)
    plans = [host_plan(lib, n, r, world, *local_rows(edges, n, r, world)) for r in range(world)]
    check_pairwise(plans, world)
    for r in range(world):
        b = bounds(n, world)
        ghosts = np.concatenate([plans[r][1][q] for q in range(world)])
        _, sender = local_rows(edges, n, r, world)
        foreign = np.unique(sender[(sender < b[r]) | (sender >= b[r + 1])])
        np.testing.assert_array_equal(ghosts, foreign)  # ascending, each owner's block contiguous


def _gloo_rank(rank, world, port, n, edges, library, skip_send, out):
    import torch
    import torch.distributed as dist
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    # A generous timeout while the ranks start; the exchange runs in a group with a 3 s one.
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=120))
    group = dist.new_group(backend="gloo", timeout=datetime.timedelta(seconds=3))
    lib = _lib(library)
    sends, ghosts = host_plan(lib, n, rank, world, *local_rows(edges, n, rank, world))
    try:
        reqs = []
        for q in range(world):
            if q == rank or (skip_send and rank == 1):
                continue
            reqs.append(dist.isend(torch.from_numpy(sends[q].astype(np.int64)), q, group=group))
        got = {}
        t0 = time.monotonic()
        for q in range(world):
            if q == rank:
                continue
            buf = torch.zeros(len(ghosts[q]), dtype=torch.int64)
            dist.recv(buf, q, group=group)
            got[q] = buf.numpy()
        for r in reqs:
            r.wait()
        ok = all(np.array_equal(got[q], ghosts[q]) for q in got)
        out.put((rank, "ok" if ok else "mismatch", 0.0))
    except RuntimeError as e:
        out.put((rank, "error: " + str(e).splitlines()[0][:200], time.monotonic() - t0))
    out.close()
    out.join_thread()  # the result reaches the parent before this process leaves
    if skip_send and rank == 1:
        time.sleep(6)  # stays alive, never sends, until the peer has given up
    os._exit(0)


def _run_gloo(world, library, c2_edges, skip_send=False):
    import multiprocessing as mp
    import socket
    n, edges = c2_edges
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        port = s.getsockname()[1]
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    procs = [ctx.Process(target=_gloo_rank, args=(r, world, port, n, edges, str(library), skip_send, q))
             for r in range(world)]
    for p in procs:
        p.start()
    results = {}
    for _ in range(world):
        rank, status, dt = q.get(timeout=60)
        results[rank] = (status, dt)
    for p in procs:
        p.join(timeout=30)
    return results


@pytest.mark.parametrize("world", [2, 3])
def test_plan_exchange_over_gloo(library, c2_edges, world):
    results = _run_gloo(world, library, c2_edges)
    assert all(status == "ok" for status, _ in results.values()), results


def test_rank_that_never_sends_times_out(library, c2_edges):
    """Rank 1 computes its plan but never sends: rank 0's receive fails after the 3 s group
    timeout with an error instead of waiting for ever."""
    results = _run_gloo(2, library, c2_edges, skip_send=True)
    status, dt = results[0]
    assert status.startswith("error"), status
    assert dt < 30, dt


@pytest.mark.gpu
@pytest.mark.parametrize("name", ["C2", "C3"])
@pytest.mark.parametrize("world", [2, 4, 8])
def test_device_plan_matches_host_rules(library, name, world):
    """The device plan of every rank equals the host rules applied to that rank's device rows;
    the ranks' plans agree pairwise; together the ranks' rows hold every edge once."""
    from mace_inference import neighbor_edges
    lib = _lib(library)
    s = structures.load(name, DATA)
    n = s.size
    xyz = np.ascontiguousarray(s.positions, np.float32)
    cell = np.ascontiguousarray(s.cell, np.float32)
    plans, pairs = [], []
    for r in range(world):
        sc, gc = np.zeros(world, np.int32), np.zeros(world, np.int32)
        E = lib.lapis_exchange_plan(n, xyz.ctypes.data, cell.ctypes.data, 6.0, r, world, sc.ctypes.data,
                                    gc.ctypes.data, None, None, None, None, None, 0)
        assert E >= 0, lib.mace_last_error()
        cap = max(E, n)
        b = bounds(n, world)
        i2o = np.zeros(n, np.int32)
        row = np.zeros(b[r + 1] - b[r] + 1, np.int32)
        sender, ghosts, sends = (np.zeros(cap, np.int32) for _ in range(3))
        assert lib.lapis_exchange_plan(n, xyz.ctypes.data, cell.ctypes.data, 6.0, r, world, sc.ctypes.data,
                                       gc.ctypes.data, i2o.ctypes.data, row.ctypes.data, sender.ctypes.data,
                                       ghosts.ctypes.data, sends.ctypes.data, cap) == E
        device = split_plan(sc, gc, ghosts, sends, r, world)
        host = host_plan(lib, n, r, world, row, sender[:E].copy())
        for q in range(world):
            np.testing.assert_array_equal(device[0][q], host[0][q])
            np.testing.assert_array_equal(device[1][q], host[1][q])
        plans.append(device)
        recv = np.repeat(np.arange(b[r], b[r + 1]), np.diff(row))
        pairs.append(np.stack([i2o[recv], i2o[sender[:E]]], 1))
    check_pairwise(plans, world)
    full = neighbor_edges(s.positions, s.cell, 6.0, library=library)[:, :2]
    mine = np.concatenate(pairs)
    mine = mine[np.lexsort((mine[:, 1], mine[:, 0]))]
    full = full[np.lexsort((full[:, 1], full[:, 0]))]
    np.testing.assert_array_equal(mine, full)
