"""The C-ABI library loads and exports every symbol include/rngd_b200.h declares (no GPU needed)."""
import ctypes
import os
import re

from tests.conftest import REPO

HEADER = os.path.join(REPO, "include", "rngd_b200.h")
SO = os.path.join(REPO, "rngd-pd_b200", "rngd_pd", "_rngd_b200.so")


def declared():
    src = open(HEADER).read()
    src = re.sub(r"/\*.*?\*/", "", src, flags=re.S)
    return sorted(set(re.findall(r"^\s*(?:int|int32_t|void)\s+(rngd_\w+)\s*\(", src, flags=re.M)))


def test_header_declares_entry_points():
    names = declared()
    assert "rngd_last_error" in names and "rngd_decode_layers" in names
    assert len(names) >= 10


def test_library_exports_every_declared_symbol():
    lib = ctypes.CDLL(SO)
    missing = [n for n in declared() if not hasattr(lib, n)]
    assert not missing, f"declared but not exported: {missing}"


def test_last_error_and_argument_checks_without_gpu():
    """Argument validation runs on the host: a bad call fails with a message, no launch."""
    lib = ctypes.CDLL(SO)
    lib.rngd_gemv_bf16.restype = ctypes.c_int
    st = lib.rngd_gemv_bf16(None, 4, 8, None, 8, 1, None, 4, 0, None)
    assert st == -1
    buf = ctypes.create_string_buffer(256)
    assert lib.rngd_last_error(buf, 256) == 0
    assert b"null" in buf.value
    assert lib.rngd_abi_version() >= 1


def test_package_import_needs_library(tmp_path):
    """The product refuses to import without its CUDA library (no fallback path)."""
    import rngd_pd._lib as L
    src = open(L.__file__).read()
    ns = {"__file__": str(tmp_path / "_lib.py"), "__name__": "probe"}
    try:
        exec(compile(src, "probe", "exec"), ns)
    except ImportError as e:
        assert "no fallback" in str(e)
    else:
        raise AssertionError("import without the library should fail")
