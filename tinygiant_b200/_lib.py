"""ctypes loader for libtinygiant.so — the reference loader's interface.

`find_library()` and `load_tinygiant_lib(lib_path)` behave as the
reference's tinygiant/_lib.py:9-95: the same search order, the same 21
symbols with the same argtypes/restype.  `load_tinygiant_lib` additionally
binds the library's extension entry points (tg_cuda_*, tg_layer_*).
"""
import ctypes
from pathlib import Path

VP = ctypes.c_void_p
CI = ctypes.c_int
CF = ctypes.c_float
SZ = ctypes.c_size_t

# The reference ABI (tinygiant/_lib.py:39-93): name -> (argtypes, restype).
ABI = {
    "tg_expert_forward": ([VP, VP, VP, CF, CI, CI], None),
    "tg_expert_forward_mixed": ([VP, VP, VP, CI, VP, VP, CF, CI, CI], None),
    "tg_matmul_q4k": ([VP, VP, VP, CI, CI], None),
    "tg_matmul_q6k": ([VP, VP, VP, CI, CI], None),
    "tg_rms_norm": ([VP, VP, VP, CI, CF], None),
    "tg_f32_matvec": ([VP, VP, VP, CI, CI], None),
    "tg_f16_matvec": ([VP, VP, VP, CI, CI], None),
    "tg_attention_decode": ([VP, VP, VP, VP, VP, VP, VP, VP, CI, CI, VP, VP, VP, VP, CI, CI, CI, CI, CI], None),
    "tg_attention_decode_q4": ([VP, VP, VP, VP, VP, VP, VP, VP, CI, CI, VP, VP, VP, VP, CI, CI, CI, CI, CI], None),
    "tg_prefetch": ([VP, SZ], None),
    "tg_prefetch_batch": ([VP, VP, CI], None),
    "tg_mlock": ([VP, SZ], CI),
    "tg_attention_v2": ([CI, CI, CI, CI, VP, VP, VP, VP, VP, VP, VP, VP, VP, VP, VP, VP, VP, CI, CI, CI, VP, VP, VP,
                         VP, CI, CI, CI, CI, CI, CF], None),
    "tg_moe_forward_rows_v2": ([VP, VP, VP, CI, VP, VP, VP, VP, CI, CI, VP, VP, VP, CI, CI, CI], None),
    "tg_matmul": ([CI, VP, VP, VP, VP, CI, CI], None),
    "tg_row_bytes": ([CI, CI], SZ),
    "tg_set_threads": ([CI], None),
    "tg_get_threads": ([], CI),
    "tg_expert_forward_rows": ([VP, VP, VP, CI, VP, VP, VP, CI, CI, CI], None),
    "tg_moe_forward_rows": ([VP, VP, VP, VP, CI, VP, VP, VP, CI, CI, CI], None),
    "tg_transformer_layer": ([VP, VP, VP, VP, VP, VP, VP, VP, VP, VP, CI, CI, VP, VP, VP, VP, VP, VP, VP, CI, VP,
                              CI, CI, CI, CI, CI, CI], None),
}

# Exported by the reference's C library but not registered by its loader;
# bound here so Python callers get checked pointer arguments.
EXTRA_ABI = {
    "tg_moe_forward": ([VP, VP, CI, VP, VP, CI, CI], None),
}

# Extensions of this library (include/tinygiant.h).
EXT = {
    "tg_cuda_last_error": ([ctypes.c_char_p, SZ], CI),
    "tg_cuda_set_device": ([CI], CI),
    "tg_cuda_set_stream": ([VP], None),
    "tg_cuda_register": ([VP, SZ], CI),
    "tg_cuda_unregister": ([VP], CI),
    "tg_cuda_registry_clear": ([], None),
    "tg_cuda_registry_bytes": ([], SZ),
    "tg_cuda_registry_stats": ([VP, VP, VP], None),
    "tg_cuda_set_weight_check": ([CI], CI),
    "tg_cuda_launch_count": ([], ctypes.c_uint64),
    "tg_cuda_device_count": ([], CI),
    "tg_cuda_debug_quantize_q8": ([VP, CI, CI, VP], CI),
    "tg_cuda_debug_row_isums": ([CI, VP, CI, CI, VP, VP], CI),
    "tg_cuda_debug_div_check": ([ctypes.c_longlong, ctypes.c_uint, VP], CI),
    "tg_layer_create": ([CI, VP, VP, VP, CI, VP, VP, VP, VP, CI, CI, CI, VP, VP, CI, CI], VP),
    "tg_layer_create_shard": ([CI, VP, VP, VP, CI, VP, VP, VP, VP, CI, CI, CI, VP, VP, CI, CI, CI, CI], VP),
    "tg_layer_clone": ([VP], VP),
    "tg_layer_destroy": ([VP], None),
    "tg_layer_expert_bytes": ([VP, CI], SZ),
    "tg_layer_forward_dev": ([VP, VP, VP, VP, VP, CI, CI, VP], CI),
    "tg_layer_set_fused": ([VP, CI], CI),
    "tg_layer_ep_handle": ([VP, VP], CI),
    "tg_layer_ep_connect": ([VP, VP], CI),
    "tg_layer_ep_reset": ([VP], CI),
    "tg_layer_set_tc": ([VP, CI], CI),
    "tg_layer_set_router": ([VP, VP, VP], CI),
    "tg_cuda_step_trace": ([VP], CI),
    "tg_cuda_step_trace_warps": ([], CI),
    "tg_cuda_tc_trace": ([VP], CI),
    "tg_cuda_debug_step_fault": ([CI, CI], CI),
    "tg_cuda_debug_tc_isums": ([VP, VP], CI),
    "tg_layer_forward": ([VP, VP, VP, CI, CI], CI),
    "tg_layer_last_routing": ([VP, CI, VP, VP], CI),
    "tg_stack_forward_dev": ([VP, CI, VP, CI, VP], CI),
    "tg_cuda_graph_begin": ([], CI),
    "tg_cuda_graph_end": ([], VP),
    "tg_cuda_graph_launch": ([VP], CI),
    "tg_cuda_graph_destroy": ([VP], None),
    "tg_cuda_stream": ([], VP),
    "tg_cuda_synchronize": ([], CI),
    "tg_cuda_matmul_q4k_noalloc": ([VP, VP, VP, CI, CI, VP], CI),
}


def find_library():
    """Same search order as the reference: the package directory, then the
    repository root."""
    pkg_dir = Path(__file__).parent
    repo_dir = pkg_dir.parent
    for path in (pkg_dir / "libtinygiant.dylib", pkg_dir / "libtinygiant.so",
                 repo_dir / "libtinygiant.dylib", repo_dir / "libtinygiant.so"):
        if path.exists():
            return path
    return None


def _bind(lib, table, optional=False):
    for name, (args, res) in table.items():
        fn = getattr(lib, name, None) if optional else getattr(lib, name)
        if fn is None:
            continue
        fn.argtypes = args
        fn.restype = res


def load_tinygiant_lib(lib_path=None):
    """Loads the library; returns None if it cannot be found (as the reference
    does).  A missing ABI symbol raises AttributeError."""
    if lib_path is None:
        lib_path = find_library()
    if lib_path is None:
        return None
    lib = ctypes.CDLL(str(lib_path))
    _bind(lib, ABI)
    _bind(lib, EXTRA_ABI, optional=True)
    _bind(lib, EXT, optional=True)
    return lib
