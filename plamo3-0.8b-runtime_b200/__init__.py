"""B200-native (sm_100a) backend for the PLaMo-3 0.8B decoder hot path.

The compute path lives in `libplamo_cuda.so` (hand-written CUDA for sm_100a behind a C ABI,
include/plamo.h). This package holds the host-side mirror of the reference's `Runtime` /
`Batch` interface (runtime.py, over ctypes), the seeded synthetic model writer
(synthetic.py), the lossless `.p12` codec (packing.py) and the build step (build.py).

The directory name is not a Python identifier; load it with `load_package()` from a path, or
via importlib with the name `plamo_b200` (as tests/, bench.py and __graft_entry__ do).
"""
from . import packing, synthetic  # noqa: F401

__all__ = ["packing", "synthetic", "runtime", "build"]


def __getattr__(name):
    if name in ("runtime", "build"):
        import importlib
        return importlib.import_module(f"{__name__}.{name}")
    if name in ("Runtime", "Batch", "decode_batch", "PlamoError"):
        import importlib
        return getattr(importlib.import_module(f"{__name__}.runtime"), name)
    raise AttributeError(name)
