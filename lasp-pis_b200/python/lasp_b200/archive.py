"""PWMH1001 model archives: the flat record format the MH1 loader reads.

Layout (mace/src/weights.cpp:81-91 writes it, mace/src/mh1.cu:630-671 reads it):
``b"PWMH1001"``, ``u32 count``, then per record ``u32 name_len, u64 byte_size, name,
bytes``.  Records are little-endian float32 except ``atomic_numbers`` and names ending in
``.dims``, ``.paths`` or ``.terms``, which are int32.  Names are unique; the writer emits
them in sorted order like the reference's ``std::map``.
"""
from __future__ import annotations

import struct
from pathlib import Path

import numpy as np

MAGIC = b"PWMH1001"


def is_index_record(name: str) -> bool:
    return name == "atomic_numbers" or name.endswith((".dims", ".paths", ".terms"))


def encode(records: dict[str, np.ndarray]) -> bytes:
    out = [MAGIC, struct.pack("<I", len(records))]
    for name in sorted(records):
        value = np.asarray(records[name])
        dtype = np.int32 if is_index_record(name) else np.float32
        data = np.ascontiguousarray(value, dtype=dtype).tobytes()
        key = name.encode()
        out += [struct.pack("<IQ", len(key), len(data)), key, data]
    return b"".join(out)


def decode(blob: bytes) -> dict[str, np.ndarray]:
    if blob[:8] != MAGIC:
        raise ValueError("Invalid MH1 archive magic")
    (count,) = struct.unpack_from("<I", blob, 8)
    pos, records = 12, {}
    for _ in range(count):
        n, size = struct.unpack_from("<IQ", blob, pos)
        pos += 12
        name = blob[pos:pos + n].decode()
        pos += n
        dtype = np.int32 if is_index_record(name) else np.float32
        records[name] = np.frombuffer(blob[pos:pos + size], dtype=dtype).copy()
        pos += size
    return records


def write(path: str | Path, records: dict[str, np.ndarray]) -> None:
    Path(path).write_bytes(encode(records))


def read(path: str | Path) -> dict[str, np.ndarray]:
    return decode(Path(path).read_bytes())
