"""Host-side input parsing: the ARC reader (CPU).

This build's reader (lasp-pis_b200/csrc/mace/arc.cpp, through bin/mace-host-bench arc-dump)
must parse every frame to the same elements, titles, periodicity and float64 positions and
cell as the reference's chemio::read_frame (oracle/_ref/host-bench-ref, built from the
reference's chemio/src/arc.cpp), and fail with the same message on the same malformed input.
The reference's own checks (chemio/tests/arc.cpp) are asserted on this build directly, so
the test still pins behaviour where the reference tools are not built.
"""
import json
import math
import subprocess

import numpy as np
import pytest

from conftest import DATA, ROOT

OURS = ROOT / "lasp-pis_b200" / "bin" / "mace-host-bench"
REF = ROOT / "oracle" / "_ref" / "host-bench-ref"

FRAME = ("Energy 0 0 -1\n!DATE\nPBC 21.9552 15.2646 6.877 91.8679 68.0603 72.9361\n"
         "Ti 1 2 3 CORE 1 X X 0 1\nO -1 0 2 CORE 1 X X 0 2\nend\nend\n")
GOOD = {
    "two_frames": "!BIOSYM archive 2\nPBC=ON\n" + FRAME + FRAME,
    "crlf_tabs": ("PBC=ON\r\nt \"quoted\" \\ title\r\nPBC\t5 6 7\t90 90 90\r\n"
                  "Fe\t0.5 0.25 1e-3 CORE\r\nNi 1.5 2.5 -0.125 CORE x\r\nEND\r\nend"),
    "open_boundaries": "PBC=OFF\nmolecule\nC 0 0 0 CORE\nH 0.6 0.6 0.6 CORE\nend\nend\n\n",
    "comments_between": "! header\nPBC=ON\n! c\nPBC 3 3 3 90 90 120\n! c2\nSi 0 0 0 CORE\nend\nend\n",
}
BAD = {
    "bad_number": "PBC=ON\nPBC 1 1 1 90 90 90\nO x 0 0 CORE 1 X X 0 1\nend\nend\n",
    "bad_element": "PBC=ON\nPBC 1 1 1 90 90 90\nXx 0 0 0 CORE 1 X X 0 1\nend\nend\n",
    "one_end": "PBC=ON\nPBC 1 1 1 90 90 90\nO 0 0 0 CORE 1 X X 0 1\nend\n",
    "bad_cell": "PBC=ON\nPBC 1 1 1 1 1 179\n",
    "empty": "",
    "atom_before_cell": "PBC=ON\ntitle\nO 0 0 0 CORE 1 X X 0 1\nend\nend\n",
    "header_in_frame": "PBC=OFF\nt\nO 0 0 0 CORE\nend\nPBC=ON\nend\n",
    "nonfinite": "PBC=OFF\nt\nO inf 0 0 CORE\nend\nend\n",
    "trailing_garbage": "PBC=OFF\nt\nO 1.0x 0 0 CORE\nend\nend\n",
    "second_title": "PBC=OFF\nt\nt2\nO 0 0 0 CORE\nend\nend\n",
}


@pytest.fixture(scope="module")
def tool():
    if not OURS.exists():
        subprocess.run(["make", "-s", "-C", str(ROOT / "lasp-pis_b200"), str(OURS)], check=True)
    return OURS


def dump(exe, path, frame=0):
    r = subprocess.run([str(exe), "arc-dump", str(path), str(frame)], capture_output=True, text=True)
    return r.returncode, (json.loads(r.stdout) if r.returncode == 0 else r.stderr.strip())


def test_reference_arc_checks(tool, tmp_path):
    """chemio/tests/arc.cpp's assertions: two frames, elements, a coordinate of frame 1, the
    c length and the alpha angle of the triclinic cell."""
    path = tmp_path / "t.arc"
    path.write_text(GOOD["two_frames"])
    rc, f0 = dump(tool, path, 0)
    assert rc == 0 and f0["elements"] == [22, 8]
    rc, f1 = dump(tool, path, 1)
    assert rc == 0 and f1["positions"][3] == -1
    c = np.array(f0["cell"]).reshape(3, 3)
    assert abs(np.linalg.norm(c[2]) - 6.877) < 1e-12
    cos_alpha = c[1] @ c[2] / (np.linalg.norm(c[1]) * np.linalg.norm(c[2]))
    assert abs(math.degrees(math.acos(cos_alpha)) - 91.8679) < 1e-10
    rc, err = dump(tool, path, 2)
    assert rc == 1 and "frame index out of range" in err
    for name in ("bad_number", "bad_element", "one_end", "bad_cell"):
        path.write_text(BAD[name])
        assert dump(tool, path)[0] == 1, name


@pytest.mark.parametrize("name", sorted(GOOD))
def test_parses_like_reference(tool, tmp_path, name):
    path = tmp_path / f"{name}.arc"
    path.write_text(GOOD[name], newline="")
    frames = GOOD[name].count("CORE") // 2 if name == "two_frames" else 1
    for frame in range(frames):
        rc, mine = dump(tool, path, frame)
        assert rc == 0, mine
        if REF.exists():
            assert dump(REF, path, frame) == (0, mine)
    if name == "open_boundaries":
        assert mine["pbc"] == [0, 0, 0] and mine["cell"] == [0] * 9
    if name == "crlf_tabs":
        assert mine["elements"] == [26, 28] and mine["positions"][2] == 1e-3
        assert mine["title"] == 't "quoted" \\ title\r'


@pytest.mark.parametrize("name", sorted(BAD))
def test_rejects_like_reference(tool, tmp_path, name):
    path = tmp_path / f"{name}.arc"
    path.write_text(BAD[name])
    rc, err = dump(tool, path)
    assert rc == 1 and err.startswith(str(path)), err
    if REF.exists():
        assert dump(REF, path) == (1, err)


def test_config_files_parse_like_reference(tool, tmp_path):
    """C1-C3 as ARC files: every float64 coordinate and cell entry, element and title."""
    from lasp_b200 import structures
    for name in ("C1", "C2", "C3"):
        s = structures.load(name, DATA)
        path = tmp_path / f"{name}.arc"
        structures.write_arc(path, [s])
        rc, mine = dump(tool, path)
        assert rc == 0 and len(mine["elements"]) == s.size
        assert np.allclose(np.array(mine["positions"]).reshape(-1, 3), s.positions, atol=1e-5)
        if REF.exists():
            assert dump(REF, path) == (0, mine)


def test_bench_host_mode(tool):
    """bench.py --host prints one JSON line with every host step for this build's arm and, with
    --impl reference, for the reference's (when its tools are built)."""
    import sys
    for impl in ("ours", "reference"):
        r = subprocess.run([sys.executable, str(ROOT / "bench.py"), "--host", "--steps", "2", "--impl", impl],
                           capture_output=True, text=True, timeout=600)
        assert r.returncode == 0, r.stderr
        line = json.loads(r.stdout.strip().splitlines()[-1])
        if impl == "reference" and "unavailable" in line:
            continue
        assert line["impl"] == impl and line["unit"] == "ms" and line["higher_is_better"] is False
        assert set(line["steps"]) == {"arc_C1", "arc_C2", "arc_C3", "arc_C5", "convert_checkpoint"}
        assert line["steps"]["arc_C5"]["units"] == 198904
        assert line["steps"]["convert_checkpoint"]["units"] == 25621837
        assert all(v["median_ms"] > 0 for v in line["steps"].values())


def test_mutated_arc_files_match_reference(tool, tmp_path):
    """Seeded mutations of the C1 ARC file (digits, signs, separators, keywords, random
    bytes): this build never crashes and, where the reference's reader is built, returns
    exactly its result or its error message for every one."""
    import random
    from lasp_b200 import structures
    base_path = tmp_path / "C1.arc"
    structures.write_arc(base_path, [structures.load("C1", DATA)])
    base = base_path.read_bytes()
    rng = random.Random(3)
    path = tmp_path / "m.arc"
    for it in range(200):
        p = bytearray(base)
        for _ in range(rng.randint(1, 5)):
            k = rng.randrange(len(p))
            p[k] = rng.choice(b" \t\n\r0123456789.-+eEx!PBCORend") if rng.random() < 0.8 else rng.randrange(256)
        path.write_bytes(bytes(p))
        mine = subprocess.run([str(tool), "arc-dump", str(path), "0"], capture_output=True)
        assert mine.returncode in (0, 1), (it, mine.returncode)
        if REF.exists():
            ref = subprocess.run([str(REF), "arc-dump", str(path), "0"], capture_output=True)
            assert (mine.returncode, mine.stdout, mine.stderr) == (ref.returncode, ref.stdout, ref.stderr), it
