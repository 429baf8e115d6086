"""The MH1 checkpoint route: ZIP/pickle reader and checkpoint -> archive converter (CPU).

Follows the reference's own checks for this path: checkpoint/tests/reader.py (stored and
deflated records, ZIP64 end records, truncation and CRC corruption), checkpoint/tests/
reader.cpp (inert reducers, malformed pickles, strided views; here tests/native/
checkpoint_reader.cpp) and mace/tests/check_checkpoint.py (every head converted byte for
byte like the reference, a changed-weight checkpoint, an unknown head).  The byte-for-byte
reference is the reference's converter compiled from its sources (oracle/_ref, when built)
and the SHA-256 digests it produced for the seeded checkpoints (tests/golden/checkpoint_ref.json).
"""
import hashlib
import io
import json
import struct
import subprocess
import zipfile

import numpy as np
import pytest
import torch

from conftest import GOLDEN, ROOT

BIN = ROOT / "lasp-pis_b200" / "bin"
DUMP = BIN / "mace-weights-dump"
READER = BIN / "checkpoint-reader"
REF_DUMP = ROOT / "oracle" / "_ref" / "mace-weights-dump-ref"
GOLD = json.loads((GOLDEN / "checkpoint_ref.json").read_text())


@pytest.fixture(scope="module")
def tools():
    if not (DUMP.exists() and READER.exists()):
        subprocess.run(["make", "-s", "-C", str(ROOT / "lasp-pis_b200"), str(DUMP), str(READER)], check=True)
    return DUMP, READER


@pytest.fixture(scope="module")
def checkpoints(tmp_path_factory):
    from lasp_b200 import checkpoint
    out = {}
    for name, case in GOLD["cases"].items():
        path = tmp_path_factory.mktemp("ckpt") / f"mh1_{name}.model"
        checkpoint.write_checkpoint(path, case["seed"], getattr(torch, case["dtype"]))
        out[name] = path
    return out


def run(*args):
    return subprocess.run([str(a) for a in args], capture_output=True, text=True)


def convert(model, out, head=None, tool=DUMP):
    r = run(tool, model, out, *([head] if head is not None else []))
    return r.returncode, r.stderr.strip()


# ------------------------------------------------------------------------------- reader

def zip_fixture(compression):
    mem = io.BytesIO()
    with zipfile.ZipFile(mem, "w", compression=compression) as z:
        with z.open("archive/data.pkl", "w", force_zip64=True) as f:
            f.write(b"\x80\x02N.")
        z.writestr("archive/byteorder", "little")
    return mem.getvalue()


def with_zip64_end(data):
    """The same archive ending in a ZIP64 end record, locator and saturated classic end record."""
    end = len(data) - 22
    _, _, _, count, _, size, offset, _ = struct.unpack("<IHHHHIIH", data[end:])
    zip64 = struct.pack("<IQHHIIQQQQ", 0x06064B50, 44, 45, 45, 0, 0, count, count, size, offset)
    locator = struct.pack("<IIQI", 0x07064B50, 0, end, 1)
    eocd = struct.pack("<IHHHHIIH", 0x06054B50, 0, 0, 0xFFFF, 0xFFFF, 0xFFFFFFFF, 0xFFFFFFFF, 0)
    return data[:end] + zip64 + locator + eocd


@pytest.mark.parametrize("compression", [zipfile.ZIP_STORED, zipfile.ZIP_DEFLATED])
def test_zip_reader_fixtures(tools, tmp_path, compression):
    _, reader = tools
    data = zip_fixture(compression)
    path = tmp_path / "fixture.zip"
    for good in (data, with_zip64_end(data)):
        path.write_bytes(good)
        r = run(reader, path)
        assert r.returncode == 0, r.stderr
    end = len(data) - 22
    offset = struct.unpack("<I", data[end + 16:end + 20])[0]
    truncated = data[:-8]
    bad_crc = data[:offset + 16] + b"\0\0\0\0" + data[offset + 20:]
    for bad, why in ((truncated, "end record"), (bad_crc, "checksum")):
        path.write_bytes(bad)
        r = run(reader, "--open", path)
        assert r.returncode == 1 and why in r.stderr, (why, r.stderr)


def test_zip_reader_rejects_unsupported(tools, tmp_path):
    _, reader = tools
    path = tmp_path / "x.zip"
    mem = io.BytesIO()
    with zipfile.ZipFile(mem, "w", compression=zipfile.ZIP_BZIP2) as z:
        z.writestr("archive/data.pkl", b"\x80\x02N.")
    path.write_bytes(mem.getvalue())
    assert "unsupported ZIP compression" in run(reader, "--open", path).stderr
    mem = io.BytesIO()
    with zipfile.ZipFile(mem, "w") as z:
        z.writestr("data.pkl", b"\x80\x02N.")
    path.write_bytes(mem.getvalue())
    assert "root directory" in run(reader, "--open", path).stderr
    mem = io.BytesIO()
    with zipfile.ZipFile(mem, "w") as z:
        z.writestr("archive/data.pkl", b"\x80\x02N.")
        z.writestr("archive/byteorder", "big")
    path.write_bytes(mem.getvalue())
    assert "little-endian" in run(reader, "--open", path).stderr


def test_deep_and_cyclic_pickles(tools, tmp_path):
    """200,000 nested lists and a list that contains itself decode and are released without
    exhausting the call stack (the reference's recursive release overflows it on the first)."""
    _, reader = tools
    n = 200000
    for name, pickle in (("deep", b"\x80\x02" + b"]" * n + b"a" * (n - 1) + b"."),
                         ("cycle", b"\x80\x02]q\x00h\x00a.")):
        path = tmp_path / f"{name}.zip"
        with zipfile.ZipFile(path, "w") as z:
            z.writestr("archive/data.pkl", pickle)
        r = run(reader, "--open", path)
        assert r.returncode == 0, (name, r.returncode, r.stderr)
        r = run(DUMP, path, tmp_path / "o.pwm")
        assert r.returncode == 1 and "unsupported MH1 checkpoint" in r.stderr, (name, r.stderr)


def test_torch_save_decodes(tools, tmp_path):
    """A plain torch.save file (parameters, buffers, OrderedDicts, sets, memo references)."""
    _, reader = tools
    m = torch.nn.Sequential(torch.nn.Linear(3, 4), torch.nn.LayerNorm(4), torch.nn.SiLU())
    path = tmp_path / "seq.pt"
    torch.save(m, path)
    r = run(reader, "--open", path)
    assert r.returncode == 0, r.stderr


def test_module_tree_tensors_match_state_dict(tools, tmp_path):
    """Every parameter and buffer reachable through _parameters / _buffers / _modules, with
    torch's state_dict names, shapes and values (the reference's checkpoint_inspect view)."""
    from lasp_b200 import checkpoint
    _, reader = tools
    model = checkpoint.build_model(9, torch.float32)
    path = checkpoint.save(model, tmp_path / "m.model")
    r = run(reader, "--tensors", path)
    assert r.returncode == 0, r.stderr
    head, *lines = r.stdout.splitlines()
    state = model.state_dict()
    assert head == f"mace.modules.models ScaleShiftMACE {len(state)} tensors"
    seen = {}
    for line in lines:
        name, shape, first = line.split(" ")
        seen[name] = ([int(d) for d in shape.strip("[]").split(",") if d], float(first))
    assert seen.keys() == state.keys()
    for name, t in state.items():
        assert seen[name][0] == list(t.shape), name
        assert seen[name][1] == (float(t.flatten()[0]) if t.numel() else 0.0), name


# ---------------------------------------------------------------------------- converter

def records(data: bytes):
    assert data[:8] == b"PWMH1001"
    (count,) = struct.unpack("<I", data[8:12])
    out, at = {}, 12
    for _ in range(count):
        n, size = struct.unpack("<IQ", data[at:at + 12])
        name = data[at + 12:at + 12 + n].decode()
        out[name] = data[at + 12 + n:at + 12 + n + size]
        at += 12 + n + size
    assert at == len(data)
    return out


@pytest.mark.parametrize("case", ["float64", "float32"])
def test_conversion_matches_reference_digests(tools, checkpoints, tmp_path, case):
    """Every head converts to the bytes the reference's converter wrote for it."""
    for head, gold in GOLD["cases"][case]["heads"].items():
        out = tmp_path / f"{head}.pwm"
        rc, err = convert(checkpoints[case], out, head)
        assert rc == 0, err
        data = out.read_bytes()
        assert len(data) == gold["bytes"] and hashlib.sha256(data).hexdigest() == gold["sha256"], head


def test_default_head_is_matpes_r2scan(tools, checkpoints, tmp_path):
    rc, err = convert(checkpoints["float64"], tmp_path / "d.pwm")
    assert rc == 0, err
    gold = GOLD["cases"]["float64"]["heads"]["matpes_r2scan"]["sha256"]
    assert hashlib.sha256((tmp_path / "d.pwm").read_bytes()).hexdigest() == gold


def test_converted_archive_is_a_valid_model(tools, checkpoints, tmp_path):
    """The converted archive has the record set and shapes the loader validates, and the
    float64 oracle evaluates it to finite energies, forces and virial."""
    import oracle
    from lasp_b200 import structures
    out = tmp_path / "m.pwm"
    assert convert(checkpoints["float64"], out)[0] == 0
    rec = records(out.read_bytes())
    assert len(rec) == 117
    dims = np.frombuffer(rec["layer1.linear_1.dims"], np.int32)
    assert list(dims) == [5120, 9728]
    assert np.frombuffer(rec["layer1.tp.dims"], np.int32).tolist() == [10, 4, 40]
    oracle.build()
    s = structures.load("C1", ROOT / "lasp-pis_b200" / "data")
    r = oracle.Oracle(out).calculate(s.positions, s.numbers, s.cell)
    assert np.isfinite(r["energy"]) and np.isfinite(r["forces"]).all() and np.isfinite(r["virial"]).all()
    assert np.abs(r["forces"].sum(axis=0)).max() < 1e-8 * max(1.0, np.abs(r["forces"]).max())


@pytest.mark.skipif(not REF_DUMP.exists(), reason="reference converter not built here")
def test_changed_weights_match_reference(tools, tmp_path):
    """A changed-weight checkpoint (check_checkpoint.py's second case) converts like the
    reference's converter does, record for record."""
    from lasp_b200 import checkpoint
    model = checkpoint.build_model(11, torch.float32)
    with torch.no_grad():
        model.node_embedding.linear.weight[0] += 0.125
        model.interactions[1].conv_tp_weights.net[3].weight[2, 5] -= 0.5
    path = checkpoint.save(model, tmp_path / "changed.model")
    for head in ("matpes_r2scan", "synthetic_scan"):
        assert convert(path, tmp_path / "a.pwm", head)[0] == 0
        assert convert(path, tmp_path / "b.pwm", head, REF_DUMP)[0] == 0
        a, b = records((tmp_path / "a.pwm").read_bytes()), records((tmp_path / "b.pwm").read_bytes())
        assert a.keys() == b.keys()
        for key in a:
            assert a[key] == b[key], key


def broken(kind):
    """A checkpoint with one defect, and the converter message it must produce."""
    from lasp_b200 import checkpoint
    m = checkpoint.build_model(3, torch.float32)
    if kind == "heads":
        m.heads = m.heads[:5]
        return m, "expected six-head MH1 architecture"
    if kind == "nonfinite":
        with torch.no_grad():
            m.interactions[0].linear_up.weight[7] = float("nan")
        return m, "nonfinite tensor value"
    if kind == "eps":
        m.interactions[0].conv_tp_weights.net[1].eps = 1e-6
        return m, "radial LayerNorm epsilon"
    if kind == "connection":
        inst = m.interactions[1].conv_tp.instructions
        inst[2] = inst[2]._replace(connection_mode="uuu")
        return m, "tensor product connectivity"
    if kind == "gate":
        m.interactions[1].equivariant_nonlin.act_gates.acts[0].cst = 1.5
        return m, "different gate normalization"
    if kind == "cutoff":
        m.radial_embedding.apply_cutoff = True
        return m, "radial cutoff"
    if kind == "root":
        return m.interactions[0], "expected ScaleShiftMACE"
    if kind == "scalar_text":
        m.radial_embedding.apply_cutoff = "no"
        return m, "invalid tensor metadata"
    raise ValueError(kind)


@pytest.mark.parametrize("kind", ["heads", "nonfinite", "eps", "connection", "gate", "cutoff", "root", "scalar_text"])
def test_conversion_errors(tools, tmp_path, kind):
    from lasp_b200 import checkpoint
    model, message = broken(kind)
    path = checkpoint.save(model, tmp_path / "bad.model")
    rc, err = convert(path, tmp_path / "o.pwm")
    assert rc == 1 and message in err, err
    if REF_DUMP.exists():
        rc_ref, err_ref = convert(path, tmp_path / "r.pwm", tool=REF_DUMP)
        assert rc_ref == 1 and err_ref == err


def test_head_rules(tools, checkpoints, archive_path, tmp_path):
    rc, err = convert(checkpoints["float32"], tmp_path / "o.pwm", "no_such_head")
    assert rc == 1 and "unknown head: no_such_head" in err
    rc, err = convert(archive_path, tmp_path / "o.pwm", "matpes_r2scan")
    assert rc == 1 and "head selection requires an original checkpoint" in err
    rc, err = convert(archive_path, tmp_path / "o.pwm")
    assert rc == 0 and (tmp_path / "o.pwm").read_bytes() == archive_path.read_bytes()
    assert run(DUMP).returncode == 1


def test_cg_table_matches_reference_constants():
    """The converter's compiled coupling table equals e3nn 0.4.4's float32 constants, row for row."""
    import re
    text = (ROOT / "lasp-pis_b200" / "csrc" / "mace" / "cg_table.h").read_text()
    rows = re.findall(r"\{(\d), (\d), (\d), (\d), (\d), (\d), (\S+)f\}", text)
    ref = [line.split() for line in (GOLDEN / "cg_e3nn044.txt").read_text().splitlines() if line.strip()]
    assert len(rows) == len(ref)
    for mine, theirs in zip(rows, ref):
        assert mine[:6] == tuple(theirs[:6])
        assert np.float32(float.fromhex(mine[6])) == np.float32(float(theirs[6]))


def test_generated_tables_are_current(tmp_path):
    """The compiled tables (coupling constants, tensor-product and product-basis layouts)
    equal what their generators produce now."""
    import sys
    gen = ROOT / "lasp-pis_b200" / "csrc" / "mace"
    for script, header in (("gen_cg_table.py", "cg_table.h"), ("gen_tp_table.py", "tp_table.h"),
                           ("gen_product_table.py", "product_table.h")):
        subprocess.run([sys.executable, str(gen / script), str(tmp_path)], check=True)
        assert (tmp_path / header).read_text() == (gen / header).read_text(), header


def test_mutated_checkpoints_fail_cleanly(tools, tmp_path):
    """Seeded byte mutations of a torch.save file -- inside its pickle (re-zipped with valid
    checksums) and in the raw ZIP -- are either decoded or rejected with an error: the
    reader never crashes on them."""
    import random
    _, reader = tools
    buf = io.BytesIO()
    torch.save(torch.nn.Sequential(torch.nn.Linear(3, 4), torch.nn.LayerNorm(4)), buf)
    data = buf.getvalue()
    src = zipfile.ZipFile(io.BytesIO(data))
    names = src.namelist()
    pkl_name = next(n for n in names if n.endswith("data.pkl"))
    pkl = src.read(pkl_name)
    rng = random.Random(2026)
    path = tmp_path / "m.zip"
    for it in range(300):
        if it % 2 == 0:
            p = bytearray(pkl)
            for _ in range(rng.randint(1, 4)):
                p[rng.randrange(len(p))] = rng.randrange(256)
            out = io.BytesIO()
            with zipfile.ZipFile(out, "w") as w:
                for n in names:
                    w.writestr(n, bytes(p) if n == pkl_name else src.read(n))
            path.write_bytes(out.getvalue())
        else:
            p = bytearray(data)
            for _ in range(rng.randint(1, 3)):
                k = rng.randrange(len(p)) if rng.random() < 0.5 else len(p) - 1 - rng.randrange(600)
                p[k] = rng.randrange(256)
            path.write_bytes(bytes(p))
        r = run(reader, "--open", path)
        assert r.returncode in (0, 1), (it, r.returncode, r.stderr)


def _random_value(rng, depth=0):
    """Random data of the kinds a checkpoint pickles: ints (|x| < 2^52), floats, bools, None,
    ASCII text, bytes, tuples, lists, sets, dicts with text or int keys, OrderedDicts."""
    import collections
    kinds = ["int", "float", "bool", "none", "str", "bytes"] + (["tuple", "list", "set", "dict", "odict"]
                                                               if depth < 4 else [])
    k = rng.choice(kinds)
    if k == "int":
        return rng.choice([rng.randrange(256), rng.randrange(65536), rng.randrange(-2**31, 2**31),
                           rng.randrange(-2**52, 2**52)])
    if k == "float":
        return rng.choice([rng.uniform(-1e6, 1e6), rng.random() * 1e-300, -0.0, float(rng.randrange(100))])
    if k == "bool":
        return rng.random() < 0.5
    if k == "none":
        return None
    if k == "str":
        return "".join(rng.choice("abcXYZ_.019 ") for _ in range(rng.randrange(0, 300)))
    if k == "bytes":
        return bytes(rng.randrange(256) for _ in range(rng.randrange(0, 300)))
    n = rng.randrange(0, 6)
    if k in ("tuple", "list"):
        items = [_random_value(rng, depth + 1) for _ in range(n)]
        return tuple(items) if k == "tuple" else items
    if k == "set":
        return {rng.randrange(-1000, 1000) for _ in range(n)}
    keys = [rng.choice([str(rng.randrange(1000)), rng.randrange(-1000, 1000)]) for _ in range(n)]
    d = {key: _random_value(rng, depth + 1) for key in keys}
    return collections.OrderedDict(d) if k == "odict" else d


def _expected(value):
    """What the decoder must produce for a value, in the reader's JSON form."""
    if isinstance(value, bool):
        return int(value)
    if isinstance(value, bytes):
        return value.decode("latin1")
    if isinstance(value, (list, tuple)):
        return [_expected(v) for v in value]
    if isinstance(value, set):
        return [_expected(v) for v in value]
    if isinstance(value, dict):
        return {str(k): _expected(v) for k, v in value.items()}
    return value


def test_pickle_layer_matches_python_pickle(tools, tmp_path):
    """Seeded random values pickled by Python (protocol 2, with memo references for shared
    and repeated objects) decode to the same data: every container, number, text and byte."""
    import pickle
    import random
    _, reader = tools
    rng = random.Random(4242)
    path = tmp_path / "v.zip"
    for it in range(150):
        value = _random_value(rng)
        shared = [value, value] if rng.random() < 0.3 else value  # memo BINGET of a shared object
        with zipfile.ZipFile(path, "w") as z:
            z.writestr("archive/data.pkl", pickle.dumps(shared, protocol=2))
        r = run(reader, "--tree", path)
        assert r.returncode == 0, (it, r.stderr)
        assert _same(json.loads(r.stdout), _expected(shared)), it


def _same(got, want):
    """Structural equality; numbers equal as doubles, including the sign of zero."""
    import math
    if isinstance(want, (int, float)) and not isinstance(want, bool):
        return isinstance(got, float) and got == float(want) and math.copysign(1, got) == math.copysign(1, want)
    if isinstance(want, list):
        return isinstance(got, list) and len(got) == len(want) and all(map(_same, got, want))
    if isinstance(want, dict):
        return isinstance(got, dict) and got.keys() == want.keys() and all(_same(got[k], want[k]) for k in want)
    return got == want



@pytest.mark.parametrize("protocol", [4, 5])
def test_newer_pickle_protocols_convert_the_same(tools, tmp_path, protocol):
    """torch.save with pickle protocol 4 or 5 (frames, memoize, stack globals) converts to the
    same archive as the default protocol 2."""
    from lasp_b200 import checkpoint
    case = GOLD["cases"]["float64"]
    model = checkpoint.build_model(case["seed"], torch.float64)
    path = tmp_path / f"p{protocol}.model"
    with checkpoint._registered():
        torch.save(model, path, pickle_protocol=protocol)
    rc, err = convert(path, tmp_path / "o.pwm")
    assert rc == 0, err
    digest = hashlib.sha256((tmp_path / "o.pwm").read_bytes()).hexdigest()
    assert digest == case["heads"]["matpes_r2scan"]["sha256"]


def _structural_mutation(rng, model):
    """One seeded structural defect of the module tree: a parameter one element short, a
    changed instruction field, a changed irreps block, a removed child module, a truncated
    buffer, a transposed matrix, or shuffled heads.  Returns a label, or None if not applied."""
    from lasp_b200 import checkpoint

    def modules(m, prefix=""):
        out = [(prefix, m)]
        for n, c in m._modules.items():
            if c is not None:
                out += modules(c, prefix + n + ".")
        return out

    name, mod = rng.choice(modules(model))
    kind = rng.randrange(7)
    if kind == 0 and mod._parameters:
        k = rng.choice(list(mod._parameters))
        t = mod._parameters[k]
        if t is not None and t.numel() > 1:
            mod._parameters[k] = torch.nn.Parameter(t.data.flatten()[:-1].clone(), requires_grad=False)
            return f"short {name}{k}"
    if kind == 1 and getattr(mod, "instructions", None):
        i = rng.randrange(len(mod.instructions))
        inst = mod.instructions[i]
        f = rng.randrange(len(inst))
        v = inst[f]
        if isinstance(v, bool):
            v = not v
        elif isinstance(v, int):
            v += rng.choice([-1, 1, 7])
        elif isinstance(v, float):
            v *= 2
        elif isinstance(v, str):
            v = "uuw"
        elif isinstance(v, tuple):
            v = (v[0] + 1,) + v[1:]
        mod.instructions[i] = inst._replace(**{inst._fields[f]: v})
        return f"instruction {name}{i}.{inst._fields[f]}"
    attrs = [a for a in ("irreps_in", "irreps_out", "irreps_in1", "irreps_in2") if hasattr(mod, a)]
    if kind == 2 and attrs:
        attr = rng.choice(attrs)
        blocks = [(mul, ir[0], ir[1]) for mul, ir in getattr(mod, attr)]
        j = rng.randrange(len(blocks))
        mul, l, p = blocks[j]
        blocks[j] = rng.choice([(mul + 1, l, p), (mul, min(l + 1, 3), p), (mul, l, -p), (0, l, p)])
        setattr(mod, attr, checkpoint._Irreps(blocks))
        return f"irreps {name}{attr}"
    if kind == 3 and mod._modules:
        k = rng.choice(list(mod._modules))
        del mod._modules[k]
        return f"removed {name}{k}"
    if kind == 4 and mod._buffers:
        k = rng.choice(list(mod._buffers))
        t = mod._buffers[k]
        if t is not None:
            mod._buffers[k] = t.reshape(-1)[:t.numel() - 1].clone() if t.numel() > 1 else t * 2
            return f"buffer {name}{k}"
    if kind == 5 and mod._parameters:
        k = rng.choice(list(mod._parameters))
        t = mod._parameters[k]
        if t is not None and t.dim() == 2:
            mod._parameters[k] = torch.nn.Parameter(t.data.t().contiguous(), requires_grad=False)
            return f"transposed {name}{k}"
    if kind == 6:
        model.heads = list(model.heads)
        rng.shuffle(model.heads)
        return "shuffled heads"
    return None


def test_structural_defects_match_reference(tools, tmp_path):
    """Seeded structural defects of the module tree (one or two each, random head): this
    build never crashes and, where the reference's converter is built, gives its exit code,
    its message and, when it converts, its archive bytes."""
    import copy
    import random
    from lasp_b200 import checkpoint
    base = checkpoint.build_model(3, torch.float32)
    rng = random.Random(2)
    path = tmp_path / "s.model"
    for it in range(25):
        model = copy.deepcopy(base)
        labels = [_structural_mutation(rng, model) for _ in range(rng.randint(1, 2))]
        checkpoint.save(model, path)
        head = rng.choice([None] + list(checkpoint.HEADS))
        rc, err = convert(path, tmp_path / "a.pwm", head)
        assert rc in (0, 1), (it, labels, err)
        if REF_DUMP.exists():
            assert convert(path, tmp_path / "b.pwm", head, REF_DUMP) == (rc, err), (it, labels)
            if rc == 0:
                assert (tmp_path / "a.pwm").read_bytes() == (tmp_path / "b.pwm").read_bytes(), (it, labels)
