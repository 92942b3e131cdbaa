"""The CPU oracle against golden vectors recorded from the reference itself
(tests/golden/make_golden.py): bit-exact on every fixture."""
import ctypes

import numpy as np
import pytest

from conftest import golden
from oracle import oracle as O


def bits(a):
    return np.ascontiguousarray(a, dtype=np.float32).view(np.uint32)


def q8_of(lib, x):
    return O.quantize_q8(lib, x).view(np.uint8).reshape(x.shape[0], -1)


@pytest.mark.parametrize("case", ["normal_2048", "partial_2880", "inter_768", "zeros_and_single", "ties", "tiny",
                                  "n32"])
def test_q8_blocks_bitexact(oracle, case):
    g = golden("q8")
    x = g[f"x_{case}"]
    assert np.array_equal(q8_of(oracle, x), g[f"q8_{case}"])


def test_dots_x1_x4_bitexact(oracle):
    g = golden("dots")
    keys = sorted({k.rsplit("_", 1)[0] for k in g})
    for key in keys:
        fmt, cols = int(key.split("_")[0][1:]), int(key.split("_")[1][1:])
        mat, xs = g[f"{key}_mat"], g[f"{key}_x"]
        rows = g[f"{key}_x1"].shape[1]
        q8 = O.quantize_q8(oracle, xs)
        for mode, ref in ((0, g[f"{key}_x1"]), (1, g[f"{key}_x4"])):
            out = np.zeros((4, rows), np.float32)
            oracle.tgo_rows_dot(fmt, mat.ctypes.data, rows, cols, q8.ctypes.data, 4, mode, out.ctypes.data)
            assert np.array_equal(bits(out), bits(ref)), (key, mode)


def test_act_bitexact(oracle):
    g = golden("act")
    for act in (0, 1):
        got = np.array([oracle.tgo_act(act, a, b) for a, b in zip(g["g"], g["u"])], np.float32)
        assert np.array_equal(bits(got), bits(g[f"act{act}"]))


def moe_case(g, name):
    gf, D, I, k, act, biased = (int(v) for v in g[f"{name}_meta"])
    dfs = [int(v) for v in g[f"{name}_dfmts"]]
    E = len(dfs)
    c = dict(gf=gf, D=D, I=I, k=k, act=act, dfs=dfs, rw=g[f"{name}_rw"], x=g[f"{name}_x"], init=g[f"{name}_init"],
             out=g[f"{name}_out"], gates=[g[f"{name}_gate{e}"] for e in range(E)],
             ups=[g[f"{name}_up{e}"] for e in range(E)], downs=[g[f"{name}_down{e}"] for e in range(E)])
    for b in ("gb", "ub", "db"):
        c[b] = [g[f"{name}_{b}{e}"] for e in range(E)] if biased else None
    return c


MOE_CASES = ["silu_mixed", "silu_f16down", "gptoss_bias", "q80_gate", "q6k_gate_k1"]


@pytest.mark.parametrize("name", MOE_CASES)
@pytest.mark.parametrize("threads", [1, 4])
def test_moe_v2_bitexact(oracle, name, threads):
    c = moe_case(golden("moe"), name)
    oracle.tg_set_threads(threads)
    out = c["init"].copy()
    O.moe_forward_rows_v2(oracle, c["gates"], c["ups"], c["downs"], c["gf"], c["dfs"], c["gb"], c["ub"], c["db"],
                          c["act"], c["rw"], c["x"], out, c["D"], c["I"])
    oracle.tg_set_threads(1)
    assert np.array_equal(bits(out), bits(c["out"]))


def test_expert_entries_bitexact(oracle):
    g = golden("expert")
    D, I = 256, 256
    o = g["fwd_init"].copy()
    oracle.tg_expert_forward(g["fwd_q4"].ctypes.data, g["fwd_x"].ctypes.data, o.ctypes.data, 0.375, D, I)
    assert np.array_equal(bits(o), bits(g["fwd_out"]))
    for dfmt in (0, 1, 2):
        o = np.zeros(D, np.float32)
        oracle.tg_expert_forward_mixed(g["mixed_gate"].ctypes.data, g["mixed_up"].ctypes.data,
                                       g[f"mixed_down{dfmt}"].ctypes.data, dfmt, g["fwd_x"].ctypes.data,
                                       o.ctypes.data, 0.5, D, I)
        assert np.array_equal(bits(o), bits(g[f"mixed_out{dfmt}"])), dfmt
    for k in (1, 3, 6):
        o = np.zeros((k, D), np.float32)
        oracle.tg_expert_forward_rows(g["mixed_gate"].ctypes.data, g["mixed_up"].ctypes.data,
                                      g[f"rows{k}_down"].ctypes.data, 2, g[f"rows{k}_x"].ctypes.data, o.ctypes.data,
                                      g[f"rows{k}_w"].ctypes.data, k, D, I)
        assert np.array_equal(bits(o), bits(g[f"rows{k}_out"])), k
    experts = [g[f"moef_e{i}"] for i in range(3)]
    arr = O.pointer_array(experts)
    o = np.full(D, 7.0, np.float32)
    oracle.tg_moe_forward(ctypes.addressof(arr), g["moef_w"].ctypes.data, 3, g["fwd_x"].ctypes.data, o.ctypes.data,
                          D, I)
    assert np.array_equal(bits(o), bits(g["moef_out"]))


def test_matmul_entries_bitexact(oracle):
    g = golden("matmul")
    for fmt in (0, 2, 3, 4, 1):
        key = f"f{fmt}"
        rows, cols = (int(v) for v in g[key + "_shape"])
        for bias, ref in ((g[key + "_bias"], g[key + "_out_bias"]), (None, g[key + "_out_nobias"])):
            o = np.zeros(rows, np.float32)
            oracle.tg_matmul(fmt, g[key + "_mat"].ctypes.data, O.ptr(bias), g[key + "_x"].ctypes.data, o.ctypes.data,
                             rows, cols)
            assert np.array_equal(bits(o), bits(ref)), (fmt, bias is None)
    for name, fn, cols in (("q4k", oracle.tg_matmul_q4k, 2048), ("q6k", oracle.tg_matmul_q6k, 768)):
        ref = g[f"mm_{name}_out"]
        o = np.zeros(ref.shape[0], np.float32)
        fn(g[f"mm_{name}_mat"].ctypes.data, g[f"mm_{name}_x"].ctypes.data, o.ctypes.data, ref.shape[0], cols)
        assert np.array_equal(bits(o), bits(ref)), name
    o = np.zeros(33, np.float32)
    oracle.tg_f32_matvec(g["f32_A"].ctypes.data, g["f32_x"].ctypes.data, o.ctypes.data, 33, 77)
    assert np.array_equal(bits(o), bits(g["f32_out"]))
    o = np.zeros(33, np.float32)
    oracle.tg_f16_matvec(g["f16_A"].ctypes.data, g["f32_x"].ctypes.data, o.ctypes.data, 33, 77)
    assert np.array_equal(bits(o), bits(g["f16_out"]))
    o = np.zeros(2050, np.float32)
    oracle.tg_rms_norm(g["rms_x"].ctypes.data, g["rms_w"].ctypes.data, o.ctypes.data, 2050, 1e-6)
    assert np.array_equal(bits(o), bits(g["rms_out"]))


def test_row_bytes(oracle):
    for fmt, cols, want in ((0, 2048, 1152), (2, 768, 630), (3, 2880, 1530), (4, 2880, 3060), (1, 100, 200),
                            (9, 100, 200)):
        assert oracle.tg_row_bytes(fmt, cols) == want


@pytest.mark.parametrize("name", ["qwen", "zipf", "gptoss"])
def test_router_matches_reference_router(name):
    """synth.route restates tinygiant/router.py: same top-k order, same weights."""
    from tinygiant_b200 import synth
    g = golden("router")
    W = g[f"{name}_W"]
    b = g[f"{name}_b"] if f"{name}_b" in g else None
    k = g[f"{name}_idx"].shape[1]
    layer = synth.MoeLayer(W.shape[1], 0, 0, 0, k, router_w=W, router_b=b)
    _, _, idx, wts = synth.route(layer, g[f"{name}_N"])
    assert np.array_equal(idx, g[f"{name}_idx"])
    np.testing.assert_allclose(wts, g[f"{name}_wts"], rtol=1e-6, atol=0)
