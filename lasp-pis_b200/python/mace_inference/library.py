import os
from pathlib import Path


def library_path(filename="libmace.so"):
    """MACE_LIBRARY if set, else the in-tree build (lasp-pis_b200/lib/libmace.so)."""
    override = os.environ.get("MACE_LIBRARY")
    if override:
        return Path(override)
    return Path(__file__).resolve().parents[2] / "lib" / filename
