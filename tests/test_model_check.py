"""Model validation without a GPU: mace_check_model runs the loader's every parse and
validation step (mace/src/mh1.cu:626-734 for archives, mace/src/weights.cpp:305-393 for
checkpoints) in host memory.  Valid models pass; each defect gets the loader's own message;
mutated archives are accepted or rejected but never crash the process.
"""
import ctypes as ct
import json
import struct
import subprocess
import sys
from pathlib import Path

import numpy as np
import pytest
import torch


@pytest.fixture(scope="module")
def lib(library):
    lib = ct.CDLL(str(library))
    lib.mace_check_model.argtypes = [ct.c_char_p, ct.c_char_p]
    lib.mace_check_model.restype = ct.c_int
    lib.mace_last_error.restype = ct.c_char_p
    return lib


def check(lib, path, head=None):
    rc = lib.mace_check_model(str(path).encode(), None if head is None else head.encode())
    return rc, lib.mace_last_error().decode()


def test_valid_models_pass(lib, archive_path, tmp_path):
    from lasp_b200 import checkpoint
    assert check(lib, archive_path) == (0, "")
    ckpt = checkpoint.write_checkpoint(tmp_path / "m.model", 4, torch.float32)
    for head in (None, "synthetic_pbe", "synthetic_scan"):
        assert check(lib, ckpt, head) == (0, "")
    rc, err = check(lib, ckpt, "nope")
    assert rc == -1 and err == "unsupported MH1 checkpoint: unknown head: nope"
    rc, err = check(lib, archive_path, "matpes_r2scan")
    assert rc == -1 and "head selection requires an original checkpoint" in err
    rc, err = check(lib, tmp_path / "missing.pwm")
    assert rc == -1 and err.startswith("Cannot open MH1 archive")


def test_python_helper(library, archive_path, tmp_path):
    from mace_inference import check_model
    check_model(archive_path, library=library)
    with pytest.raises(RuntimeError, match="Invalid MH1 archive magic"):
        bad = tmp_path / "bad.pwm"
        bad.write_bytes(b"PWMH1002" + archive_path.read_bytes()[8:])
        check_model(bad, library=library)


def defects():
    """(name, edit of the records or the bytes, expected message fragment)."""
    def drop(key):
        return lambda r: r.pop(key)

    def setv(key, fn):
        def edit(r):
            r[key] = fn(r[key].copy())
        return edit

    def nan_at(a):
        a[3] = np.nan
        return a

    return [
        ("missing_embedding", drop("embedding"), "Invalid MH1 tensor size: embedding"),
        ("linear_dims", setv("layer0.linear_up.dims", lambda a: a + 1), "Unsupported MH1 linear dimensions: layer0.linear_up"),
        ("nonfinite", setv("layer1.linear_2.weight", nan_at), "Nonfinite MH1 tensor: layer1.linear_2.weight"),
        ("constants", setv("constants", lambda a: a[:13]), "Unsupported MH1 constants"),
        ("cutoff", setv("constants", lambda a: np.concatenate([[5.0], a[1:]])), "Unsupported MH1 constants"),
        ("duplicate_z", setv("atomic_numbers", lambda a: np.concatenate([[a[1]], a[1:]])), "Invalid MH1 element map"),
        ("path_bounds", setv("layer0.linear_res.paths", lambda a: np.concatenate([[a[0] + 10**6], a[1:]])),
         "Invalid linear path: layer0.linear_res"),
    ]


@pytest.mark.parametrize("case", defects(), ids=lambda c: c[0])
def test_defects_are_reported(lib, archive_path, tmp_path, case):
    from lasp_b200 import archive
    name, edit, message = case
    records = archive.read(archive_path)
    edit(records)
    path = tmp_path / f"{name}.pwm"
    archive.write(path, records)
    rc, err = check(lib, path)
    assert rc == -1 and message in err, err


def test_malformed_files_are_reported(lib, archive_path, tmp_path):
    blob = archive_path.read_bytes()
    for name, data, message in (("magic", b"PWMH1002" + blob[8:], "Invalid MH1 archive magic"),
                                ("truncated", blob[:len(blob) // 2], "Truncated MH1 archive"),
                                ("count", blob[:8] + struct.pack("<I", 0) + blob[12:], "Invalid MH1 tensor count"),
                                ("short", blob[:10], "")):
        path = tmp_path / f"{name}.pwm"
        path.write_bytes(data)
        rc, err = check(lib, path)
        assert rc == -1 and message in err, (name, err)


MUTATE = r'''
import ctypes as ct, random, struct, sys
lib = ct.CDLL(sys.argv[1])
lib.mace_check_model.argtypes = [ct.c_char_p, ct.c_char_p]
lib.mace_last_error.restype = ct.c_char_p
blob = open(sys.argv[2], "rb").read()
heads, pos = [], 12
for _ in range(struct.unpack_from("<I", blob, 8)[0]):
    n, size = struct.unpack_from("<IQ", blob, pos)
    heads.append((pos, 12 + n))
    pos += 12 + n + size
rng = random.Random(int(sys.argv[4]))
accepted = 0
for it in range(int(sys.argv[5])):
    p = bytearray(blob)
    for _ in range(rng.randint(1, 3)):
        if rng.random() < 0.7:   # a record header: its name length, byte size or name
            start, length = rng.choice(heads)
            p[start + rng.randrange(length)] = rng.randrange(256)
        else:
            p[rng.randrange(len(p))] = rng.randrange(256)
    open(sys.argv[3], "wb").write(p)
    accepted += lib.mace_check_model(sys.argv[3].encode(), None) == 0
    print(it, flush=True)
print("accepted", accepted, flush=True)
'''


def test_mutated_archives_never_crash(library, archive_path, tmp_path):
    r = subprocess.run([sys.executable, "-c", MUTATE, str(library), str(archive_path), str(tmp_path / "m.pwm"),
                        "2026", "120"], capture_output=True, text=True, timeout=900)
    assert r.returncode == 0, (r.returncode, r.stdout[-200:], r.stderr[-500:])
    assert r.stdout.strip().splitlines()[-1].startswith("accepted")


REF_CREATE = r'''
import ctypes as ct, json, sys
lib = ct.CDLL(sys.argv[1])
lib.mace_create_mh1_head.argtypes = [ct.c_char_p, ct.c_int, ct.c_char_p]
lib.mace_create_mh1_head.restype = ct.c_void_p
lib.mace_last_error.restype = ct.c_char_p
lib.mace_destroy.argtypes = [ct.c_void_p]
out = []
for path in sys.argv[2:]:
    h = lib.mace_create_mh1_head(path.encode(), 0, None)
    out.append(None if h else lib.mace_last_error().decode())
    if h:
        lib.mace_destroy(h)
print(json.dumps(out))
'''


@pytest.mark.gpu
def test_loader_errors_match_reference_library(lib, archive_path, tmp_path):
    """On a GPU: the reference's own library (oracle/_ref/libmace_ref.so, built from its
    sources) rejects every defective archive above with the message mace_check_model and this
    build's constructor give, and accepts the valid one."""
    from lasp_b200 import archive
    from mace_inference import NativeMH1
    ref_lib = Path(__file__).resolve().parents[1] / "oracle" / "_ref" / "libmace_ref.so"
    if not ref_lib.exists():
        pytest.skip("reference library not built")
    paths = [archive_path]
    for name, edit, _ in defects():
        records = archive.read(archive_path)
        edit(records)
        paths.append(tmp_path / f"{name}.pwm")
        archive.write(paths[-1], records)
    blob = archive_path.read_bytes()
    for name, data in (("magic", b"PWMH1002" + blob[8:]), ("truncated", blob[:len(blob) // 2])):
        paths.append(tmp_path / f"{name}.pwm")
        paths[-1].write_bytes(data)
    r = subprocess.run([sys.executable, "-c", REF_CREATE, str(ref_lib)] + [str(p) for p in paths],
                       capture_output=True, text=True, timeout=600)
    assert r.returncode == 0, r.stderr[-500:]
    theirs = json.loads(r.stdout.strip().splitlines()[-1])
    for path, ref_err in zip(paths, theirs):
        rc, err = check(lib, path)
        assert (rc == 0) == (ref_err is None) and (ref_err is None or err == ref_err), (path.name, err, ref_err)
        if ref_err is not None:
            with pytest.raises(RuntimeError) as e:
                NativeMH1(path, device=0)
            assert str(e.value) == ref_err
