import ctypes
import re
import sys
from pathlib import Path

import pytest

ROOT = Path(__file__).resolve().parent.parent
if str(ROOT) not in sys.path:
    sys.path.insert(0, str(ROOT))

HEADER = ROOT / "include" / "flashlite_b200.h"
LIBRARY = ROOT / "flashlite_b200" / "libflashlite_b200.so"


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a B200 (sm_100a) GPU")
    config.addinivalue_line("markers", "slow: long-running case")


def header_functions() -> list[str]:
    """Names of the functions the C header declares."""
    text = HEADER.read_text()
    text = re.sub(r"/\*.*?\*/", "", text, flags=re.S)
    return re.findall(r"^\s*(?:const\s+)?[a-z_0-9]+\s*\*?\s*(fl_[a-z0-9_]+)\s*\(", text, flags=re.M)


@pytest.fixture(scope="session")
def header_fns():
    return header_functions()


@pytest.fixture(scope="session")
def cuda():
    import torch

    if not torch.cuda.is_available():
        pytest.skip("CUDA device not available")
    major, _ = torch.cuda.get_device_capability(0)
    if major != 10:
        pytest.skip("kernels are built for sm_100a only")
    return torch.device("cuda:0")


@pytest.fixture(scope="session")
def fl_lib():
    """The C-ABI library via ctypes, with argument types declared."""
    lib = ctypes.CDLL(str(LIBRARY))
    p, i64, f32, i32 = ctypes.c_void_p, ctypes.c_int64, ctypes.c_float, ctypes.c_int
    for name in ("fl_flash2_fwd", "fl_naive_fwd"):
        fn = getattr(lib, name)
        fn.argtypes = [p, p, p, p, i64, i64, i64, i64, f32, i32, p]
        fn.restype = i32
    lib.fl_flash2_fwd_block.argtypes = [p, p, p, p, p, i64, i64, i64, i64, i64, i64, f32, i32, i32, p]
    lib.fl_flash2_fwd_block.restype = i32
    lib.fl_ring_finalize.argtypes = [p, p, i64, p]
    lib.fl_ring_finalize.restype = i32
    lib.fl_status_str.argtypes = [i32]
    lib.fl_status_str.restype = ctypes.c_char_p
    lib.fl_last_error.restype = ctypes.c_char_p
    lib.fl_version.restype = ctypes.c_char_p
    lib.fl_device_error.argtypes = [p, ctypes.POINTER(ctypes.c_uint32)]
    lib.fl_device_error.restype = i32
    lib.fl_selftest_bounded_wait.argtypes = [ctypes.c_uint64, p, p]
    lib.fl_selftest_bounded_wait.restype = i32
    return lib
