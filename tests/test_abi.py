"""The C-ABI library builds, loads without a GPU and exports every entry point include/*.h declares."""
import ctypes
import re

from conftest import REPO


def declared_symbols():
    names = set()
    for h in (REPO / "include").glob("*.h"):
        text = re.sub(r"/\*.*?\*/", "", h.read_text(), flags=re.S)
        names |= set(re.findall(r"\b(plamo_\w+)\s*\(", text))
    return names


def test_library_exports_declared_symbols(pkg):
    pkg.build.build()
    lib = ctypes.CDLL(str(pkg.runtime.LIB_PATH))
    names = declared_symbols()
    assert len(names) >= 30
    missing = [n for n in sorted(names) if not hasattr(lib, n)]
    assert not missing, missing


def test_open_without_device_fails_cleanly(pkg, micro_dir):
    """No CUDA device here: plamo_open reports an error instead of falling back to the CPU."""
    import pytest
    with pytest.raises(pkg.PlamoError):
        pkg.Runtime(micro_dir, context=32)
