"""Parity of the sm_100a kernels with the reference, through the C ABI.

Bar:
  * Q8 blocks and per-sub-block int32 dot sums: bit-exact;
  * matvec outputs (no activation in between): bit-exact, because the
    kernels repeat the reference's float association;
  * anything that passes through the activation's expf: max|err| / max|ref|
    <= 1e-4 (TOL below) — CUDA's expf and glibc's may differ in the last bit.
The comparison targets are the golden fixtures recorded from the reference
itself and, at larger shapes, the CPU oracle (bit-exact to the reference).
"""
import ctypes

import numpy as np
import pytest

import tinygiant_b200 as tg
from conftest import golden
from oracle import oracle as O
from tinygiant_b200 import moe as M
from tinygiant_b200 import quants as Q
from tinygiant_b200 import synth

pytestmark = pytest.mark.gpu

TOL = 1e-4


def bits(a):
    return np.ascontiguousarray(a, dtype=np.float32).view(np.uint32)


def rel_err(got, ref):
    scale = float(np.max(np.abs(ref)))
    return float(np.max(np.abs(got.astype(np.float64) - ref))) / (scale if scale > 0 else 1.0)


def ok(lib):
    tg.check(lib)


# ---- Q8 quantizer and integer sums ---------------------------------------

@pytest.mark.parametrize("case", ["normal_2048", "partial_2880", "inter_768", "zeros_and_single", "ties", "tiny",
                                  "n32"])
def test_q8_blocks_bitexact_vs_reference(gpu, case):
    g = golden("q8")
    x = g[f"x_{case}"]
    nb = (x.shape[1] + 255) // 256
    out = np.zeros((x.shape[0], nb), O.Q8_DTYPE)
    assert gpu.tg_cuda_debug_quantize_q8(x.ctypes.data, x.shape[0], x.shape[1], out.ctypes.data) == 0
    ok(gpu)
    assert np.array_equal(out.view(np.uint8).reshape(x.shape[0], -1), g[f"q8_{case}"])


def test_q8_blocks_bitexact_random_scales(gpu, oracle):
    rng = np.random.default_rng(11)
    for scale in (1e-20, 1e-3, 1.0, 1e4, 1e30):
        x = (rng.standard_normal((5, 2880)) * scale).astype(np.float32)
        out = np.zeros((5, 12), O.Q8_DTYPE)
        gpu.tg_cuda_debug_quantize_q8(x.ctypes.data, 5, 2880, out.ctypes.data)
        ok(gpu)
        assert np.array_equal(out.view(np.uint8), O.quantize_q8(oracle, x).view(np.uint8)), scale


@pytest.mark.parametrize("fmt,cols", [(0, 2048), (0, 768), (2, 768), (2, 2048), (3, 2880), (4, 2880)])
def test_int32_sub_block_sums_bitexact(gpu, oracle, fmt, cols):
    from tests.golden.make_golden import GEN
    rng = np.random.default_rng(100 + fmt)
    rows = 37
    mat = GEN[fmt](rng, rows, cols)
    x = (rng.standard_normal(cols) * 2).astype(np.float32)
    xq = O.quantize_q8(oracle, x[None])[0]
    want = np.zeros((rows, 16 * cols // 32), np.int32)
    rb = Q.row_bytes(fmt, cols)
    n = 0
    for r in range(rows):
        n = oracle.tgo_row_isums(fmt, mat[r * rb:].ctypes.data, xq.ctypes.data, cols, want[r].ctypes.data)
    got = np.zeros((rows, n), np.int32)
    per = gpu.tg_cuda_debug_row_isums(fmt, mat.ctypes.data, rows, cols, xq.ctypes.data, got.ctypes.data)
    ok(gpu)
    assert per == n
    assert np.array_equal(got, want[:, :n])


# ---- matvecs: bit-exact ------------------------------------------------

def test_matmul_entries_bitexact_vs_reference(gpu):
    g = golden("matmul")
    for fmt in (0, 2, 3, 4, 1):
        key = f"f{fmt}"
        rows, cols = (int(v) for v in g[key + "_shape"])
        for bias, ref in ((g[key + "_bias"], g[key + "_out_bias"]), (None, g[key + "_out_nobias"])):
            o = np.zeros(rows, np.float32)
            gpu.tg_matmul(fmt, g[key + "_mat"].ctypes.data, O.ptr(bias), g[key + "_x"].ctypes.data, o.ctypes.data,
                          rows, cols)
            ok(gpu)
            assert np.array_equal(bits(o), bits(ref)), (fmt, bias is None)
    for name, fn, cols in (("q4k", gpu.tg_matmul_q4k, 2048), ("q6k", gpu.tg_matmul_q6k, 768)):
        ref = g[f"mm_{name}_out"]
        o = np.zeros(ref.shape[0], np.float32)
        fn(g[f"mm_{name}_mat"].ctypes.data, g[f"mm_{name}_x"].ctypes.data, o.ctypes.data, ref.shape[0], cols)
        ok(gpu)
        assert np.array_equal(bits(o), bits(ref)), name
    o = np.zeros(33, np.float32)
    gpu.tg_f32_matvec(g["f32_A"].ctypes.data, g["f32_x"].ctypes.data, o.ctypes.data, 33, 77)
    ok(gpu)
    assert np.array_equal(bits(o), bits(g["f32_out"]))
    o = np.zeros(33, np.float32)
    gpu.tg_f16_matvec(g["f16_A"].ctypes.data, g["f32_x"].ctypes.data, o.ctypes.data, 33, 77)
    ok(gpu)
    assert np.array_equal(bits(o), bits(g["f16_out"]))
    o = np.zeros(2050, np.float32)
    gpu.tg_rms_norm(g["rms_x"].ctypes.data, g["rms_w"].ctypes.data, o.ctypes.data, 2050, 1e-6)
    ok(gpu)
    assert np.array_equal(bits(o), bits(g["rms_out"]))


def test_dots_x1_bitexact_vs_reference(gpu):
    """Every golden x1 dot (one row, one input) through tg_matmul's no-bias
    path, which is the reference's x1 kernel plus +0.f."""
    g = golden("dots")
    for key in sorted({k.rsplit("_", 1)[0] for k in g}):
        fmt, cols = int(key.split("_")[0][1:]), int(key.split("_")[1][1:])
        rows = g[f"{key}_x1"].shape[1]
        for t in range(4):
            o = np.zeros(rows, np.float32)
            x = np.ascontiguousarray(g[f"{key}_x"][t])
            fn = {0: gpu.tg_matmul_q4k, 2: gpu.tg_matmul_q6k}.get(fmt)
            if fn is not None:
                fn(g[f"{key}_mat"].ctypes.data, x.ctypes.data, o.ctypes.data, rows, cols)
                want = g[f"{key}_x1"][t]
            else:
                gpu.tg_matmul(fmt, g[f"{key}_mat"].ctypes.data, None, x.ctypes.data, o.ctypes.data, rows, cols)
                want = g[f"{key}_x1"][t] + np.float32(0)
            ok(gpu)
            assert np.array_equal(bits(o), bits(want)), (key, t)


@pytest.mark.parametrize("fmt,rows,cols", [(0, 768, 2048), (2, 2048, 768), (3, 2880, 2880), (4, 512, 2880)])
def test_matvec_full_size_bitexact_vs_oracle(gpu, oracle, fmt, rows, cols):
    from tests.golden.make_golden import GEN
    rng = np.random.default_rng(7 + fmt)
    mat = GEN[fmt](rng, rows, cols)
    x = rng.standard_normal(cols).astype(np.float32)
    bias = rng.standard_normal(rows).astype(np.float32)
    want, got = np.zeros(rows, np.float32), np.zeros(rows, np.float32)
    oracle.tg_matmul(fmt, mat.ctypes.data, bias.ctypes.data, x.ctypes.data, want.ctypes.data, rows, cols)
    gpu.tg_matmul(fmt, mat.ctypes.data, bias.ctypes.data, x.ctypes.data, got.ctypes.data, rows, cols)
    ok(gpu)
    assert np.array_equal(bits(got), bits(want))


# ---- expert / MoE entries: through the activation ------------------------

def test_expert_entries_vs_reference(gpu):
    g = golden("expert")
    D, I = 256, 256
    o = g["fwd_init"].copy()
    gpu.tg_expert_forward(g["fwd_q4"].ctypes.data, g["fwd_x"].ctypes.data, o.ctypes.data, 0.375, D, I)
    ok(gpu)
    assert rel_err(o, g["fwd_out"]) <= TOL
    for dfmt in (0, 1, 2):
        o = np.zeros(D, np.float32)
        gpu.tg_expert_forward_mixed(g["mixed_gate"].ctypes.data, g["mixed_up"].ctypes.data,
                                    g[f"mixed_down{dfmt}"].ctypes.data, dfmt, g["fwd_x"].ctypes.data, o.ctypes.data,
                                    0.5, D, I)
        ok(gpu)
        assert rel_err(o, g[f"mixed_out{dfmt}"]) <= TOL, dfmt
    for k in (1, 3, 6):
        o = np.zeros((k, D), np.float32)
        gpu.tg_expert_forward_rows(g["mixed_gate"].ctypes.data, g["mixed_up"].ctypes.data,
                                   g[f"rows{k}_down"].ctypes.data, 2, g[f"rows{k}_x"].ctypes.data, o.ctypes.data,
                                   g[f"rows{k}_w"].ctypes.data, k, D, I)
        ok(gpu)
        assert rel_err(o, g[f"rows{k}_out"]) <= TOL, k
    experts = [g[f"moef_e{i}"] for i in range(3)]
    arr = O.pointer_array(experts)
    o = np.full(D, 7.0, np.float32)
    gpu.tg_moe_forward(ctypes.addressof(arr), g["moef_w"].ctypes.data, 3, g["fwd_x"].ctypes.data, o.ctypes.data, D, I)
    ok(gpu)
    assert rel_err(o, g["moef_out"]) <= TOL


@pytest.mark.parametrize("name", ["silu_mixed", "silu_f16down", "gptoss_bias", "q80_gate", "q6k_gate_k1"])
def test_moe_v2_vs_reference(gpu, name):
    from test_oracle_golden import moe_case
    c = moe_case(golden("moe"), name)
    out = c["init"].copy()
    M.moe_forward_rows_v2(gpu, c["gates"], c["ups"], c["downs"], c["gf"], c["dfs"], c["gb"], c["ub"], c["db"],
                          c["act"], c["rw"], c["x"], out, c["D"], c["I"])
    ok(gpu)
    assert rel_err(out, c["out"]) <= TOL


@pytest.fixture(scope="module")
def qwen_small():
    """16 experts of the C2 layer (seed 1), with its router cut to 16 rows."""
    L = synth.qwen_layer(seed=1, n_experts=16)
    return L


@pytest.mark.parametrize("T", [1, 2, 5, 8])
def test_moe_qwen_shapes_vs_oracle(gpu, oracle, qwen_small, T):
    rng = np.random.default_rng(50 + T)
    N = synth.rms_norm(rng.standard_normal((T, 2048)).astype(np.float32))
    init = (rng.standard_normal((T, 2048)) * 0.01).astype(np.float32)
    want = M.moe_layer_forward(oracle, qwen_small, N, init.copy())
    got = M.moe_layer_forward(gpu, qwen_small, N, init.copy())
    ok(gpu)
    assert rel_err(got, want) <= TOL


@pytest.mark.parametrize("T", [1, 3])
def test_moe_gptoss_shapes_vs_oracle(gpu, oracle, T):
    L = synth.gptoss_layer(seed=3, n_experts=6)
    rng = np.random.default_rng(70 + T)
    N = synth.rms_norm(rng.standard_normal((T, 2880)).astype(np.float32))
    want = M.moe_layer_forward(oracle, L, N)
    got = M.moe_layer_forward(gpu, L, N)
    ok(gpu)
    assert rel_err(got, want) <= TOL


def test_c1_expert_forward_vs_oracle(gpu, oracle):
    buf = synth.c1_expert(seed=0)
    x = np.random.default_rng(0).standard_normal(2048).astype(np.float32)
    want, got = np.zeros(2048, np.float32), np.zeros(2048, np.float32)
    oracle.tg_expert_forward(buf.ctypes.data, x.ctypes.data, want.ctypes.data, 1.0, 2048, 768)
    gpu.tg_expert_forward(buf.ctypes.data, x.ctypes.data, got.ctypes.data, 1.0, 2048, 768)
    ok(gpu)
    assert rel_err(got, want) <= TOL


# ---- semantics and edge cases --------------------------------------------

def _tiny_layer(rng, E=3, D=256, I=256):
    from tests.golden.make_golden import rand_q4k, rand_q6k
    return ([rand_q4k(rng, I, D) for _ in range(E)], [rand_q4k(rng, I, D) for _ in range(E)],
            [rand_q6k(rng, D, I) for _ in range(E)])


def test_moe_edge_cases(gpu, oracle):
    rng = np.random.default_rng(3)
    gates, ups, downs = _tiny_layer(rng)
    x = rng.standard_normal((4, 256)).astype(np.float32)
    rw = np.zeros((3, 4), np.float32)
    # row 1 uses no expert; expert 2 is unused; -0.0 counts as zero
    rw[0, 0], rw[1, 0], rw[0, 2], rw[1, 3], rw[2, 1] = 0.5, 0.25, 1.0, 0.75, -0.0
    for lib in (oracle, gpu):
        out = np.full((4, 256), 1.5, np.float32)
        M.moe_forward_rows_v2(lib, gates, ups, downs, 0, [2, 2, 2], None, None, None, 0, rw, x, out, 256, 256)
        if lib is oracle:
            want = out
        else:
            ok(gpu)
            got = out
    assert np.all(got[1] == 1.5)
    assert rel_err(got, want) <= TOL
    # no experts at all: output untouched
    out = np.full((4, 256), 2.0, np.float32)
    M.moe_forward_rows_v2(gpu, [], [], [], 0, [], None, None, None, 0, np.zeros((0, 4), np.float32), x, out, 256, 256)
    ok(gpu)
    assert np.all(out == 2.0)


def test_registry_sees_changed_weights(gpu, oracle):
    rng = np.random.default_rng(5)
    from tests.golden.make_golden import rand_q4k
    mat = rand_q4k(rng, 64, 512)
    x = rng.standard_normal(512).astype(np.float32)
    a = np.zeros(64, np.float32)
    gpu.tg_matmul_q4k(mat.ctypes.data, x.ctypes.data, a.ctypes.data, 64, 512)
    mat[:] = rand_q4k(rng, 64, 512)            # same address, new bytes
    b, want = np.zeros(64, np.float32), np.zeros(64, np.float32)
    gpu.tg_matmul_q4k(mat.ctypes.data, x.ctypes.data, b.ctypes.data, 64, 512)
    oracle.tg_matmul_q4k(mat.ctypes.data, x.ctypes.data, want.ctypes.data, 64, 512)
    ok(gpu)
    assert np.array_equal(bits(b), bits(want))
    assert not np.array_equal(a, b)


def _registry_stats(lib):
    r, e, n = ctypes.c_uint64(), ctypes.c_uint64(), ctypes.c_size_t()
    lib.tg_cuda_registry_stats(ctypes.byref(r), ctypes.byref(e), ctypes.byref(n))
    return r.value, e.value, n.value


def test_registry_sees_any_changed_byte_and_reused_addresses(gpu, oracle):
    """An unregistered host matrix is fingerprinted whole on every call (the
    default policy): one
    nibble rewritten anywhere (here in the middle of a block, away from the
    matrix's first, middle and last 32 bytes) is uploaded again.  The same
    host address reused with another shape drops the old entry and reuses its
    HBM."""
    rng = np.random.default_rng(15)
    from tests.golden.make_golden import rand_q4k
    rows, cols = 64, 512
    mat = rand_q4k(rng, rows, cols)
    x = rng.standard_normal(cols).astype(np.float32)

    def run(lib, m, r, c):
        o = np.zeros(r, np.float32)
        lib.tg_matmul_q4k(m.ctypes.data, x[:c].ctypes.data, o.ctypes.data, r, c)
        return o

    assert gpu.tg_cuda_set_weight_check(2) == 2     # the default: every byte
    run(gpu, mat, rows, cols)
    ok(gpu)
    re0, ev0, _ = _registry_stats(gpu)
    for off in (1000, 144 * 37 + 100, mat.nbytes - 40):   # nibble bytes of blocks 6, 37 and the last
        mat[off] ^= 0x5A
        got, want = run(gpu, mat, rows, cols), run(oracle, mat, rows, cols)
        ok(gpu)
        assert np.array_equal(bits(got), bits(want)), off
    re1, _, _ = _registry_stats(gpu)
    assert re1 - re0 == 3
    got = run(gpu, mat, rows, cols)      # unchanged bytes: no upload
    ok(gpu)
    assert _registry_stats(gpu)[0] == re1
    # the same buffer as a 32 x 1024 matrix: the 64 x 512 entry is dropped
    mat2 = mat.reshape(-1)[: 32 * 4 * 144]
    assert mat2.ctypes.data == mat.ctypes.data
    mat2[:] = rand_q4k(rng, 32, 1024)
    x = rng.standard_normal(1024).astype(np.float32)
    got, want = run(gpu, mat2, 32, 1024), run(oracle, mat2, 32, 1024)
    ok(gpu)
    assert np.array_equal(bits(got), bits(want))
    assert _registry_stats(gpu)[1] > ev0
    # the sampled policy misses an edit away from its samples; the
    # registered-range path never checks
    assert gpu.tg_cuda_set_weight_check(1) == 2
    try:
        base = run(gpu, mat2, 32, 1024)
        mat2[1000] ^= 0x5A
        assert np.array_equal(bits(run(gpu, mat2, 32, 1024)), bits(base))
        mat2[0] ^= 0x01                             # inside the sample: seen
        got, want = run(gpu, mat2, 32, 1024), run(oracle, mat2, 32, 1024)
        ok(gpu)
        assert np.array_equal(bits(got), bits(want))
    finally:
        gpu.tg_cuda_set_weight_check(2)


def test_unsupported_formats_fail_loudly(gpu):
    rng = np.random.default_rng(6)
    gates, ups, downs = _tiny_layer(rng, E=1)
    x = rng.standard_normal((1, 256)).astype(np.float32)
    out = np.full((1, 256), 9.0, np.float32)
    rw = np.ones((1, 1), np.float32)
    M.moe_forward_rows_v2(gpu, gates, ups, downs, 1, [2], None, None, None, 0, rw, x, out, 256, 256)  # F16 gate
    code, msg = tg.last_error(gpu)
    assert code != 0 and "gate format" in msg
    M.moe_forward_rows_v2(gpu, gates, ups, downs, 0, [7], None, None, None, 0, rw, x, out, 256, 256)  # bad down fmt
    code, msg = tg.last_error(gpu)
    assert code != 0
    assert np.all(out == 9.0)


def test_launches_are_counted(gpu):
    before = gpu.tg_cuda_launch_count()
    rng = np.random.default_rng(8)
    from tests.golden.make_golden import rand_q4k
    mat = rand_q4k(rng, 8, 256)
    x = np.ones(256, np.float32)
    o = np.zeros(8, np.float32)
    gpu.tg_matmul_q4k(mat.ctypes.data, x.ctypes.data, o.ctypes.data, 8, 256)
    ok(gpu)
    assert gpu.tg_cuda_launch_count() > before


def test_step_division_is_exact(gpu):
    """The fused step divides x by the RMS norm as x * RN_double(1 / d)
    rounded to fp32; on 2^26 pseudo-random operand pairs (half of them near
    1, the rest any bit pattern) that equals IEEE fp32 division bit for bit."""
    bad = ctypes.c_ulonglong(123)
    assert gpu.tg_cuda_debug_div_check(1 << 26, 12345, ctypes.byref(bad)) == 0, tg.last_error(gpu)
    assert bad.value == 0
