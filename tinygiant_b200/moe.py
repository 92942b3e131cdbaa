"""Host-side mirror of the reference engine's MoE call.

`moe_forward_rows_v2` builds the ctypes pointer arrays exactly as
tinygiant/engine.py:323-340 does and calls the library; `moe_layer_forward`
adds the routing and union step of engine.py:297-318 (via synth.route) in
front of it, for one layer and T rows.
"""
import ctypes

import numpy as np

from . import synth


def _ptrs(arrays):
    return (ctypes.c_void_p * len(arrays))(*[None if a is None else a.ctypes.data for a in arrays])


def moe_forward_rows_v2(lib, gates, ups, downs, gate_fmt, down_fmts, gate_bias, up_bias, down_bias, act, row_w,
                        inputs, output, embed_dim, inter_dim):
    """One tg_moe_forward_rows_v2 call; `output` [k, D] accumulates."""
    n = len(gates)
    k = inputs.shape[0]
    row_w = np.ascontiguousarray(row_w, dtype=np.float32)
    inputs = np.ascontiguousarray(inputs, dtype=np.float32)
    assert output.flags["C_CONTIGUOUS"] and output.dtype == np.float32
    gp, upp, dp = _ptrs(gates), _ptrs(ups), _ptrs(downs)
    fm = (ctypes.c_int * n)(*down_fmts)
    keep, bias = [], []
    for b in (gate_bias, up_bias, down_bias):
        if b is None:
            bias.append(None)
        else:
            arr = _ptrs(b)
            keep.append(arr)
            bias.append(ctypes.addressof(arr))
    lib.tg_moe_forward_rows_v2(ctypes.addressof(gp), ctypes.addressof(upp), ctypes.addressof(dp), gate_fmt,
                               ctypes.addressof(fm), bias[0], bias[1], bias[2], act, n, row_w.ctypes.data,
                               inputs.ctypes.data, output.ctypes.data, k, embed_dim, inter_dim)
    return output


def moe_layer_forward(lib, layer, N, output=None):
    """Route rows N [T, D] through `layer` and run the MoE call, as one
    iteration of the engine's layer loop does.  Returns output [T, D]."""
    N = np.ascontiguousarray(np.atleast_2d(N), dtype=np.float32)
    experts, row_w, _, _ = synth.route(layer, N)
    if output is None:
        output = np.zeros_like(N)
    sel = [int(e) for e in experts]
    return moe_forward_rows_v2(lib, [layer.gates[e] for e in sel], [layer.ups[e] for e in sel],
                               [layer.downs[e] for e in sel], layer.gate_fmt, [layer.down_fmts[e] for e in sel],
                               None, None, None, layer.act, row_w, N, output, layer.embed_dim, layer.inter_dim)
