"""ctypes bindings for the CPU checkers built by oracle/Makefile.

TEST INFRASTRUCTURE ONLY: imported by tests/, by __graft_entry__.smoke() and
by bench.py's cpu_baseline / --impl reference leg.  The product library
(tinygiant_b200) never imports this module.

Two checkers share one binding:
  * ``load_oracle()``  -> oracle/libtg_oracle.so, this repo's scalar
    restatement of csrc/libtinygiant.c, plus tgo_* test hooks (Q8 blocks,
    per-sub-block int32 sums);
  * ``load_reference()`` -> oracle/_ref/libtinygiant_ref.so, the reference's
    own csrc/libtinygiant.c compiled unmodified on x86 through
    oracle/neon_shim/arm_neon.h (None when it was not built).

Argument types follow tinygiant/_lib.py:39-93 of the reference.
"""
import ctypes
import os
import subprocess
from pathlib import Path

import numpy as np

VP = ctypes.c_void_p
CI = ctypes.c_int
CF = ctypes.c_float

HERE = Path(__file__).resolve().parent
ORACLE_SO = HERE / "libtg_oracle.so"
REF_SO = HERE / "_ref" / "libtinygiant_ref.so"

Q8_BLOCK_BYTES = 296          # float scale, int32 sum, int32 bsums[8], int8 qs[256]
Q8_DTYPE = np.dtype([("scale", "<f4"), ("sum", "<i4"), ("bsums", "<i4", (8,)), ("qs", "i1", (256,))])
assert Q8_DTYPE.itemsize == Q8_BLOCK_BYTES

# The hot-path symbols both checkers export, with the reference's ctypes
# signatures (restype None unless given).
_SIGS = {
    "tg_expert_forward": ([VP, VP, VP, CF, CI, CI], None),
    "tg_expert_forward_mixed": ([VP, VP, VP, CI, VP, VP, CF, CI, CI], None),
    "tg_matmul_q4k": ([VP, VP, VP, CI, CI], None),
    "tg_matmul_q6k": ([VP, VP, VP, CI, CI], None),
    "tg_rms_norm": ([VP, VP, VP, CI, CF], None),
    "tg_f32_matvec": ([VP, VP, VP, CI, CI], None),
    "tg_f16_matvec": ([VP, VP, VP, CI, CI], None),
    "tg_moe_forward_rows_v2": ([VP, VP, VP, CI, VP, VP, VP, VP, CI, CI, VP, VP, VP, CI, CI, CI], None),
    "tg_matmul": ([CI, VP, VP, VP, VP, CI, CI], None),
    "tg_row_bytes": ([CI, CI], ctypes.c_size_t),
    "tg_set_threads": ([CI], None),
    "tg_get_threads": ([], CI),
    "tg_expert_forward_rows": ([VP, VP, VP, CI, VP, VP, VP, CI, CI, CI], None),
    "tg_moe_forward_rows": ([VP, VP, VP, VP, CI, VP, VP, VP, CI, CI, CI], None),
    "tg_moe_forward": ([VP, VP, CI, VP, VP, CI, CI], None),
}

_HOOKS = {
    "tgo_q8_block_bytes": ([], ctypes.c_size_t),
    "tgo_quantize_q8": ([VP, VP, CI], None),
    "tgo_row_isums": ([CI, VP, VP, CI, VP], CI),
    "tgo_rows_dot": ([CI, VP, CI, CI, VP, CI, CI, VP], None),
    "tgo_act": ([CI, CF, CF], CF),
}


def reference_dir():
    """The reference checkout: $TG_REFERENCE_DIR, else `reference` beside this
    repository.  Only the CPU checkers are built from it; nothing reads it at
    run time on a GPU host."""
    return Path(os.environ.get("TG_REFERENCE_DIR", HERE.parent.parent / "reference"))


def build(quiet=True):
    """Runs oracle/Makefile (the _ref targets only where the reference exists)."""
    targets = ["libtg_oracle.so"]
    ref = reference_dir()
    if Path(ref, "csrc", "libtinygiant.c").exists():
        targets.append("ref")
    subprocess.run(["make", "-C", str(HERE), f"REF={ref}", *targets], check=True,
                   stdout=subprocess.DEVNULL if quiet else None)


def _bind(lib, sigs):
    for name, (args, res) in sigs.items():
        fn = getattr(lib, name)
        fn.argtypes = args
        fn.restype = res
    return lib


def load_oracle():
    if not ORACLE_SO.exists():
        build()
    lib = _bind(ctypes.CDLL(str(ORACLE_SO)), {**_SIGS, **_HOOKS})
    assert lib.tgo_q8_block_bytes() == Q8_BLOCK_BYTES
    return lib


def load_reference():
    """The reference's own kernels (compiled through the NEON shim), or None."""
    if not REF_SO.exists():
        return None
    return _bind(ctypes.CDLL(str(REF_SO)), _SIGS)


def ptr(a):
    return None if a is None else a.ctypes.data


def quantize_q8(lib, x):
    """x: float32 [..., ncols] -> structured Q8 blocks [..., nblocks]."""
    x = np.ascontiguousarray(x, dtype=np.float32)
    ncols = x.shape[-1]
    nb = (ncols + 255) // 256
    rows = x.reshape(-1, ncols)
    out = np.zeros((rows.shape[0], nb), dtype=Q8_DTYPE)
    for i in range(rows.shape[0]):
        lib.tgo_quantize_q8(rows[i].ctypes.data, out[i].ctypes.data, ncols)
    return out.reshape(x.shape[:-1] + (nb,))


def pointer_array(arrays, ctype=VP):
    """A ctypes array of the data pointers of numpy arrays (None -> NULL)."""
    return (ctype * len(arrays))(*[None if a is None else a.ctypes.data for a in arrays])


def moe_forward_rows_v2(lib, gates, ups, downs, gate_fmt, down_fmts, gb, ub, db, act, row_w, xs, out,
                        embed_dim, inter_dim):
    """Calls tg_moe_forward_rows_v2 exactly as tinygiant/engine.py:323-340 does."""
    n = len(gates)
    k = xs.shape[0]
    gp, upp, dp = pointer_array(gates), pointer_array(ups), pointer_array(downs)
    fm = (ctypes.c_int * n)(*down_fmts)
    bias = [None, None, None]
    keep = []
    for i, b in enumerate((gb, ub, db)):
        if b is not None:
            arr = pointer_array(b)
            keep.append(arr)
            bias[i] = ctypes.addressof(arr)
    lib.tg_moe_forward_rows_v2(ctypes.addressof(gp), ctypes.addressof(upp), ctypes.addressof(dp), gate_fmt,
                               ctypes.addressof(fm), bias[0], bias[1], bias[2], act, n,
                               row_w.ctypes.data, xs.ctypes.data, out.ctypes.data, k, embed_dim, inter_dim)
    return out
