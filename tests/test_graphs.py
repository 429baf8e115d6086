"""CUDA-graph replay of the evaluation (B200 GPU).

A handle records its kernels into a CUDA graph on the second call whose prepared geometry
(atom and edge counts, cell, workspace pointers) equals the previous call's, and replays the
graph on later such calls.  A replay must give the same results as launching the kernels
directly, bit for bit -- also for new coordinates with the same key (a rigid translation
keeps every distance, so the edge count stays), since the graph reads the positions from
device memory.  A call with another key runs directly again.  Direct results come from a
child process with MACE_CUDA_GRAPHS=0.
"""
import json
import os
import subprocess
import sys

import numpy as np
import pytest

from conftest import DATA, ROOT
from lasp_b200 import structures

pytestmark = pytest.mark.gpu

DIRECT = """
import sys, json, numpy as np
sys.path[:0] = {paths!r}
from lasp_b200 import structures
from mace_inference import NativeMH1
s = structures.load({name!r}, {data!r})
out = {{}}
with NativeMH1({archive!r}, backend=0, library={library!r}) as m:
    for tag, shift in (("base", 0.0), ("moved", 0.731)):
        r = m.calculate(s.positions + np.float32(shift), s.numbers, s.cell)
        assert m.diagnostics["graph"] == "direct"
        for k, v in r.items():
            out[tag + "." + k] = v
np.savez({out!r}, **out)
"""


@pytest.mark.parametrize("name", ["C1", "C2"])
def test_replay_matches_direct_launches(library, archive_path, name, tmp_path):
    from mace_inference import NativeMH1
    out = tmp_path / "direct.npz"
    code = DIRECT.format(paths=[str(ROOT / "lasp-pis_b200" / "python")], name=name, data=str(DATA),
                         archive=str(archive_path), library=str(library), out=str(out))
    r = subprocess.run([sys.executable, "-c", code], env={**os.environ, "MACE_CUDA_GRAPHS": "0"},
                       capture_output=True, text=True)
    assert r.returncode == 0, r.stderr[-2000:]
    ref = dict(np.load(out))
    s = structures.load(name, DATA)
    modes = []
    with NativeMH1(archive_path, backend=0, library=library) as m:
        for k in range(4):
            res = m.calculate(s.positions, s.numbers, s.cell)
            modes.append(m.diagnostics["graph"])
            for key in ("energies", "forces", "virial"):
                assert np.array_equal(res[key], ref["base." + key]), (k, key)
            assert res["energy"] == float(ref["base.energy"])
        assert modes[-2:] == ["recorded", "replayed"] or modes[-1] == "replayed", modes
        launches = m.diagnostics["launches"]
        assert launches > 0
        moved = m.calculate(s.positions + np.float32(0.731), s.numbers, s.cell)
        assert m.diagnostics["graph"] == "replayed"
        for key in ("energies", "forces", "virial"):
            assert np.array_equal(moved[key], ref["moved." + key]), key
        other = structures.load("C1" if name == "C2" else "C2", DATA)
        m.calculate(other.positions, other.numbers, other.cell)
        assert m.diagnostics["graph"] == "direct"
