"""tinygiant_b200 — B200-native drop-in for TinyGiant's fused quantized MoE
expert path (csrc/libtinygiant.c of andrew-the-drawer/tinygiant).

The product is the C-ABI shared library `libtinygiant.so` built from
`csrc/` (CUDA for sm_100a + host C++).  This package locates, builds and
binds it; `_lib.load_tinygiant_lib` mirrors the reference's ctypes loader.
There is no CPU compute path: without a GPU every compute call reports an
error through `tg_cuda_last_error`, which `check()` turns into an exception.
"""
import ctypes

from ._lib import ABI, EXT, find_library, load_tinygiant_lib

__all__ = ["ABI", "EXT", "find_library", "load", "check", "TinyGiantCudaError", "FMT", "ACT"]

FMT = {"q4_k": 0, "float16": 1, "q6_k": 2, "mxfp4": 3, "q8_0": 4}
ACT = {"silu": 0, "gptoss": 1}

_LIB = None


class TinyGiantCudaError(RuntimeError):
    pass


def load(build_if_missing=True):
    """The bound library (built in-tree on first use if absent)."""
    global _LIB
    if _LIB is None:
        path = find_library()
        if path is None and build_if_missing:
            from .build import build
            path = build()
        if path is None:
            raise TinyGiantCudaError("libtinygiant.so not found; run python -m tinygiant_b200.build")
        _LIB = load_tinygiant_lib(path)
    return _LIB


def last_error(lib=None):
    lib = lib or load()
    buf = ctypes.create_string_buffer(512)
    code = lib.tg_cuda_last_error(buf, len(buf))
    return code, buf.value.decode(errors="replace")


def check(lib=None):
    """Raises TinyGiantCudaError if the previous call failed."""
    code, msg = last_error(lib)
    if code:
        raise TinyGiantCudaError(f"[{code}] {msg}")
