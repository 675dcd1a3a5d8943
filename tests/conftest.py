import pathlib
import subprocess
import sys

import pytest

REPO = pathlib.Path(__file__).resolve().parent.parent
if str(REPO) not in sys.path:
    sys.path.insert(0, str(REPO))


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a B200 (sm_100a) GPU")
    config.addinivalue_line("markers", "slow: long-running case")


@pytest.fixture(scope="session")
def oracle():
    """The CPU restatement (test infrastructure only), built on demand."""
    if not (REPO / "oracle" / "build" / "liboracle.so").exists():
        subprocess.run(["make", "-C", str(REPO / "oracle")], check=True, capture_output=True)
    from tests import oracle_lib
    return oracle_lib


@pytest.fixture(scope="session")
def gpu():
    """The library with a usable device; GPU tests fail loudly if the native code is absent."""
    from tensorforge_b200 import _lib
    import ctypes as C
    n = C.c_int(0)
    rc = _lib.lib().tforge_device_count(C.byref(n))
    assert rc == 0 and n.value > 0, f"no CUDA device visible (status {rc})"
    return _lib
