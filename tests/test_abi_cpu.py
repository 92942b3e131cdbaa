"""The product library's C ABI without a GPU: it loads, exports every symbol
include/tinygiant.h declares (the reference's 21 among them), answers the
host-only queries, and fails loudly (no CPU fallback) on compute calls when
no device is visible."""
import ctypes
import os
import re
import sys
from pathlib import Path

import numpy as np
import pytest

import tinygiant_b200 as tg
from tinygiant_b200 import _lib

ROOT = Path(__file__).resolve().parents[1]


def declared_symbols():
    text = (ROOT / "include" / "tinygiant.h").read_text()
    text = re.sub(r"/\*.*?\*/", "", text, flags=re.S)
    return sorted(set(re.findall(r"\b(tg_\w+)\s*\(", text)))


def test_header_declares_reference_abi():
    decl = set(declared_symbols())
    assert len(_lib.ABI) == 21
    missing = set(_lib.ABI) - decl
    assert not missing, missing


def test_library_exports_every_declared_symbol(lib):
    for name in declared_symbols():
        assert hasattr(lib, name), name


def test_loader_mirrors_reference_search(lib):
    path = _lib.find_library()
    assert path is not None and path.name == "libtinygiant.so"
    again = _lib.load_tinygiant_lib(path)
    for name, (args, res) in _lib.ABI.items():
        assert getattr(again, name).argtypes == args


def test_reference_loader_binds_this_library(lib):
    """tinygiant/_lib.py of the reference (when the checkout is present)
    loads this .so unchanged."""
    from oracle import oracle as O
    ref = O.reference_dir()
    if not (ref / "tinygiant" / "_lib.py").exists():
        pytest.skip("reference checkout not present")
    import importlib.util
    spec = importlib.util.spec_from_file_location("ref_lib", ref / "tinygiant" / "_lib.py")
    mod = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(mod)
    loaded = mod.load_tinygiant_lib(_lib.find_library())
    assert loaded is not None


def test_host_queries(lib):
    for fmt, cols, want in ((0, 2048, 1152), (2, 768, 630), (3, 2880, 1530), (4, 2880, 3060), (1, 100, 200),
                            (7, 100, 200)):
        assert lib.tg_row_bytes(fmt, cols) == want
    lib.tg_set_threads(6)
    assert lib.tg_get_threads() == 6
    lib.tg_set_threads(1)
    assert lib.tg_get_threads() == 1


def test_compute_without_gpu_fails_loudly(lib):
    if lib.tg_cuda_device_count() > 0:
        pytest.skip("a GPU is visible")
    rows, cols = 4, 256
    mat = np.zeros(rows * 144, np.uint8)
    x = np.ones(cols, np.float32)
    out = np.full(rows, 42.0, np.float32)
    lib.tg_matmul_q4k(mat.ctypes.data, x.ctypes.data, out.ctypes.data, rows, cols)
    code, msg = tg.last_error(lib)
    assert code != 0 and "CUDA" in msg
    assert np.all(out == 42.0)      # outputs untouched, nothing computed on the CPU
    with pytest.raises(tg.TinyGiantCudaError):
        lib.tg_matmul_q4k(mat.ctypes.data, x.ctypes.data, out.ctypes.data, rows, cols)
        tg.check(lib)


def test_bad_arguments_are_rejected_before_the_gpu(lib):
    out = np.full(256, 3.0, np.float32)
    x = np.ones(256, np.float32)
    mat = np.zeros(256 * 144, np.uint8)
    lib.tg_matmul_q4k(mat.ctypes.data, x.ctypes.data, out.ctypes.data, 4, 200)   # 200 is not a multiple of 256
    code, msg = tg.last_error(lib)
    assert code != 0 and "multiple" in msg
    assert np.all(out == 3.0)


def test_packers_match_gguf_decoders():
    """The packers write the block layouts the reference decodes: gguf-py's
    independent decoders read back exactly the values of our numpy decoders."""
    gguf = pytest.importorskip("gguf")
    from gguf import GGMLQuantizationType as T
    from gguf.quants import dequantize
    from tinygiant_b200 import quants as Q
    rng = np.random.default_rng(9)
    w = rng.standard_normal((64, 512)).astype(np.float32) * 0.02
    p4, p6 = Q.pack_q4k(w), Q.pack_q6k(w)
    d4, d6 = Q.dequant_q4k(p4, 64, 512), Q.dequant_q6k(p6, 64, 512)
    np.testing.assert_array_equal(d4, dequantize(p4.reshape(64, -1), T.Q4_K))
    np.testing.assert_array_equal(d6, dequantize(p6.reshape(64, -1), T.Q6_K))
    # the fits are tight: rms error well under the weight spread
    assert np.sqrt(np.mean((d4 - w) ** 2)) < 0.12 * w.std()
    assert np.sqrt(np.mean((d6 - w) ** 2)) < 0.03 * w.std()
    assert np.array_equal(p4, Q.pack_q4k(w))   # deterministic


def test_decoders_match_golden_gguf_fixture():
    from conftest import golden
    from tinygiant_b200 import quants as Q
    g = golden("gguf")
    for name, fmt, cols in (("q4k", 0, 512), ("q6k", 2, 512), ("mxfp4", 3, 64)):
        ours = Q.DEQUANT[fmt](g[f"{name}_mat"], 8, cols)
        np.testing.assert_array_equal(ours, g[f"{name}_deq"])


def test_noalloc_return_code_is_the_reported_error(lib):
    """tg_cuda_matmul_q4k_noalloc returns the same code that
    tg_cuda_last_error reports, for size errors and (without a GPU) for the
    missing device; nothing is written to the output."""
    out = np.full(8, 5.0, np.float32)
    x = np.ones(256, np.float32)
    mat = np.zeros(8 * 144, np.uint8)
    for rows, cols in ((8, 200), (8, 65536 + 256), (0, 256)):
        rc = lib.tg_cuda_matmul_q4k_noalloc(mat.ctypes.data, x.ctypes.data, out.ctypes.data, rows, cols, None)
        code, msg = tg.last_error(lib)
        assert rc == code == 3, (rc, code, msg)
    if lib.tg_cuda_device_count() == 0:
        rc = lib.tg_cuda_matmul_q4k_noalloc(mat.ctypes.data, x.ctypes.data, out.ctypes.data, 8, 256, None)
        code, msg = tg.last_error(lib)
        assert rc != 0 and rc == code, (rc, code, msg)
    assert np.all(out == 5.0)


def test_numpy_packers_golden():
    """The numpy Q4_K / Q6_K packers against committed packed bytes
    (tests/golden/packers.npz), edge blocks included: all-zero, all-positive,
    constant, tiny and huge values."""
    from conftest import golden
    from tinygiant_b200 import quants as Q
    g = golden("packers")
    np.testing.assert_array_equal(Q.pack_q4k(g["w"]), g["q4k"])
    np.testing.assert_array_equal(Q.pack_q6k(g["w"]), g["q6k"])


def test_bindings_match_the_reference_loader_signatures():
    """tinygiant_b200._lib.ABI gives each of the 21 symbols the argtypes and
    restype that the reference's loader gives it (tests/golden/ref_abi.json,
    recorded from tinygiant/_lib.py by tests/golden/make_ref_abi.py)."""
    import ctypes
    import json
    from pathlib import Path
    ref = json.loads((Path(__file__).resolve().parent / "golden" / "ref_abi.json").read_text())
    assert set(ref) == set(_lib.ABI)
    for name, (args, res) in _lib.ABI.items():
        assert [t.__name__ for t in args] == ref[name]["argtypes"], name
        assert (None if res is None else res.__name__) == ref[name]["restype"], name
