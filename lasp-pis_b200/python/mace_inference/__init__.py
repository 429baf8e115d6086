"""Python frontend of the B200 MACE MH1 engine (ctypes over libmace.so's C ABI).

Mirrors the reference frontend (mace/python/mace_inference): ``MH1Calculator`` is the ASE
calculator (importable only when ``ase`` is installed) and ``library_path`` locates the
library (``MACE_LIBRARY`` overrides).  ``NativeMH1`` is the same binding without ASE.
"""
from .library import library_path
from .native import NativeMH1, check_model, nccl_unique_id, neighbor_edges

__all__ = ["NativeMH1", "check_model", "library_path", "nccl_unique_id", "neighbor_edges"]
try:  # ase is optional
    from .calculator import MH1Calculator  # noqa: F401
    __all__.append("MH1Calculator")
except ImportError:
    pass
