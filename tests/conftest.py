import sys
from pathlib import Path

import pytest

ROOT = Path(__file__).resolve().parents[1]
for p in (ROOT / "lasp-pis_b200" / "python", ROOT / "oracle", ROOT / "tests" / "golden", ROOT):
    if str(p) not in sys.path:
        sys.path.insert(0, str(p))

DATA = ROOT / "lasp-pis_b200" / "data"
GOLDEN = ROOT / "tests" / "golden"


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA GPU (B200)")


@pytest.fixture(scope="session")
def archive_path():
    from lasp_b200 import synth
    path = DATA / "mh1_synth.pwm"
    synth.write_archive(path)
    return path


@pytest.fixture(scope="session")
def oracle_model(archive_path):
    import oracle
    oracle.build()
    return oracle.Oracle(archive_path)


LIB = ROOT / "lasp-pis_b200" / "lib" / "libmace.so"


@pytest.fixture(scope="session")
def library():
    """Build (if needed) and return the path of the B200 libmace.so."""
    import subprocess
    if not LIB.exists():
        subprocess.run(["make", "-s", "-C", str(ROOT / "lasp-pis_b200"), "-j8"], check=True)
    return LIB
