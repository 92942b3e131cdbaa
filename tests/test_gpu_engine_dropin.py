"""The drop-in path as the reference engine drives it: this library loaded
with exactly the ctypes signatures that the reference's loader
(tinygiant/_lib.py load_tinygiant_lib) gives each symbol — recorded in
tests/golden/ref_abi.json — and called with the engine's own MoE sequence
(tinygiant/engine.py:281-341): numpy RMSNorm, router logits, top-k by
descending logit, softmax over the selected, the union of experts ascending
by id, dense row weights, a zero-filled output, pointer arrays built per
call, then tg_moe_forward_rows_v2 with host pointers.  Checked against the
oracle within 1e-4 of max|ref|."""
import ctypes
import json
from pathlib import Path

import numpy as np
import pytest

import tinygiant_b200 as tg
from tinygiant_b200 import synth

pytestmark = pytest.mark.gpu
TOL = 1e-4
ABI = Path(__file__).resolve().parent / "golden" / "ref_abi.json"


def _bind_like_reference(path):
    lib = ctypes.CDLL(str(path))
    for name, sig in json.loads(ABI.read_text()).items():
        fn = getattr(lib, name)
        fn.argtypes = [getattr(ctypes, t) for t in sig["argtypes"]]
        fn.restype = None if sig["restype"] is None else getattr(ctypes, sig["restype"])
    return lib


def _engine_moe(lib, layer, X, eps=1e-6):
    """One layer of the engine's MoE block on rows X [k, D]; returns moe_out."""
    k, D = X.shape
    N = (X / np.sqrt(np.mean(X * X, axis=-1, keepdims=True) + np.float32(eps))).astype(np.float32)
    union = {}
    for r in range(k):
        logits = layer.router_w @ N[r]
        idx = np.argpartition(logits, -layer.top_k)[-layer.top_k:]
        idx = idx[np.argsort(logits[idx])[::-1]]
        sel = logits[idx]
        e = np.exp(sel - sel.max())
        w = (e / e.sum()).astype(np.float32)
        for ei, wt in zip(idx, w):
            union.setdefault(int(ei), {})[r] = float(wt)
    experts = sorted(union)
    n = len(experts)
    row_w = np.zeros((n, k), np.float32)
    for ei, e in enumerate(experts):
        for r, wt in union[e].items():
            row_w[ei, r] = wt
    gate_ptrs = (ctypes.c_void_p * n)(*[layer.gates[e].ctypes.data for e in experts])
    up_ptrs = (ctypes.c_void_p * n)(*[layer.ups[e].ctypes.data for e in experts])
    down_ptrs = (ctypes.c_void_p * n)(*[layer.downs[e].ctypes.data for e in experts])
    fmts = (ctypes.c_int * n)(*[layer.down_fmts[e] for e in experts])
    moe_out = np.empty((k, D), np.float32)
    moe_out.fill(0)
    lib.tg_moe_forward_rows_v2(ctypes.addressof(gate_ptrs), ctypes.addressof(up_ptrs), ctypes.addressof(down_ptrs),
                               layer.gate_fmt, ctypes.addressof(fmts), None, None, None, layer.act, n,
                               row_w.ctypes.data, N.ctypes.data, moe_out.ctypes.data, k, D, layer.inter_dim)
    return moe_out


@pytest.fixture(scope="module")
def ref_bound(gpu):
    return _bind_like_reference(tg.find_library())


@pytest.fixture(scope="module")
def layers():
    return {"qwen": synth.qwen_layer(seed=1, layer=3, n_experts=32),
            "gptoss": synth.gptoss_layer(seed=3, layer=1, n_experts=16)}


@pytest.mark.parametrize("kind,k", [("qwen", 1), ("qwen", 4), ("qwen", 8), ("gptoss", 1), ("gptoss", 3)])
def test_engine_sequence_vs_oracle(ref_bound, oracle, layers, kind, k):
    L = layers[kind]
    X = np.random.default_rng([77, k]).standard_normal((k, L.embed_dim)).astype(np.float32)
    got = _engine_moe(ref_bound, L, X)
    tg.check(tg.load())
    want = _engine_moe(oracle, L, X)
    err = float(np.max(np.abs(got.astype(np.float64) - want)) / np.max(np.abs(want)))
    assert err <= TOL


def test_engine_residual_loop_two_layers(ref_bound, oracle, layers):
    """X += MoE(X) over two layers with the same buffers reused, as the
    engine's layer loop does (engine.py:339-341)."""
    L = layers["qwen"]
    L2 = synth.qwen_layer(seed=1, layer=4, n_experts=32)
    X0 = np.random.default_rng(78).standard_normal((2, 2048)).astype(np.float32)
    outs = []
    for lib in (ref_bound, oracle):
        X = X0.copy()
        for lay in (L, L2):
            X += _engine_moe(lib, lay, X)
        outs.append(X)
    tg.check(tg.load())
    err = float(np.max(np.abs(outs[0].astype(np.float64) - outs[1])) / np.max(np.abs(outs[1])))
    assert err <= TOL
