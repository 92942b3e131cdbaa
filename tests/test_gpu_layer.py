"""The GPU-routed layer path (tg_layer_*): routing on the device against the
reference router, expert outputs against the oracle, the residual stack and
CUDA-graph replay.  Tolerance as in test_gpu_parity (1e-4 of max|ref|)."""
import ctypes

import numpy as np
import pytest

import tinygiant_b200 as tg
from oracle import oracle as O
from tinygiant_b200 import moe as M
from tinygiant_b200 import synth
from tinygiant_b200.layer import ResidentLayer

pytestmark = pytest.mark.gpu
TOL = 1e-4


def rel_err(got, ref):
    s = float(np.max(np.abs(ref)))
    return float(np.max(np.abs(got.astype(np.float64) - ref))) / (s if s > 0 else 1.0)


def routing_agrees(layer, N, idx, w):
    """Same experts in the same order and weights within 1e-5, except where
    the reference's logits tie to within 1e-5 (fp32 order differences)."""
    _, _, ridx, rw = synth.route(layer, N)
    for t in range(N.shape[0]):
        if not np.array_equal(ridx[t], idx[t]):
            logits = layer.router_w @ N[t] + (0 if layer.router_b is None else layer.router_b)
            gaps = np.abs(np.diff(np.sort(logits)[::-1][:layer.top_k + 1]))
            assert gaps.min() < 1e-5, (t, ridx[t], idx[t])
        else:
            np.testing.assert_allclose(w[t], rw[t], rtol=1e-5, atol=1e-7)


@pytest.fixture(scope="module")
def qwen16(gpu):
    L = synth.qwen_layer(seed=1, n_experts=16)
    return L, ResidentLayer(L, max_tokens=8, lib=gpu)


@pytest.mark.parametrize("T", [1, 3, 8])
def test_layer_matches_reference_pipeline(gpu, oracle, qwen16, T):
    L, R = qwen16
    rng = np.random.default_rng(200 + T)
    N = synth.rms_norm(rng.standard_normal((T, 2048)).astype(np.float32))
    got = R.forward(N, normalize=False)          # route N as given, like the engine
    idx, w = R.last_routing(T)
    routing_agrees(L, N, idx, w)
    want = M.moe_layer_forward(oracle, L, N)
    assert rel_err(got, want) <= TOL


@pytest.mark.parametrize("T", [1, 3, 8])
def test_fused_step_matches_three_kernel_path(gpu, qwen16, T):
    """The single-kernel step and the three-kernel step route and compute alike."""
    L, R = qwen16
    x = np.random.default_rng(300 + T).standard_normal((T, 2048)).astype(np.float32)
    outs, routes = [], []
    for fused in (True, False):
        R.set_fused(fused)
        outs.append(R.forward(x, normalize=True))
        routes.append(R.last_routing(T))
    R.set_fused(True)
    N = synth.rms_norm(x)
    for idx, w in routes:
        routing_agrees(L, N, idx, w)
    if np.array_equal(routes[0][0], routes[1][0]):
        assert rel_err(outs[0], outs[1]) <= TOL


@pytest.mark.parametrize("T", [1, 5])
def test_fused_step_bit_exact_vs_gpu_abi_path(gpu, qwen16, T):
    """Given the step's own routing, its output equals the reference-ABI call
    as this library runs it on the GPU (tg_moe_forward_rows_v2) on the same
    rows bit for bit (a GPU-vs-GPU check; the oracle checks are in
    test_gpu_full_configs.py): the dots, the
    activation and the ordered combine are the same arithmetic."""
    L, R = qwen16
    N = synth.rms_norm(np.random.default_rng(400 + T).standard_normal((T, 2048)).astype(np.float32))
    got = R.forward(N, normalize=False)
    idx, w = R.last_routing(T)
    sel = sorted({int(idx[t, j]) for t in range(T) for j in range(L.top_k) if w[t, j] != 0})
    row_w = np.zeros((len(sel), T), np.float32)
    for t in range(T):
        for j in range(L.top_k):
            if w[t, j] != 0:
                row_w[sel.index(int(idx[t, j])), t] = w[t, j]
    want = np.zeros_like(N)
    M.moe_forward_rows_v2(gpu, [L.gates[e] for e in sel], [L.ups[e] for e in sel], [L.downs[e] for e in sel],
                          L.gate_fmt, [L.down_fmts[e] for e in sel], None, None, None, L.act, row_w, N, want,
                          L.embed_dim, L.inter_dim)
    tg.check(gpu)
    np.testing.assert_array_equal(got.view(np.uint32), want.view(np.uint32))


@pytest.fixture(scope="module")
def gptoss8(gpu):
    L = synth.gptoss_layer(seed=3, n_experts=8)
    return L, ResidentLayer(L, max_tokens=4, lib=gpu)


@pytest.mark.parametrize("T", [1, 3])
def test_fused_step_bit_exact_vs_gpu_abi_path_mxfp4(gpu, gptoss8, T):
    """The MXFP4 (gpt-oss) fused step, whose rows are split over half warps
    with the sub-block fold chained through the lanes, equals the GPU
    reference-ABI call on the step's own routing bit for bit."""
    L, R = gptoss8
    N = synth.rms_norm(np.random.default_rng(500 + T).standard_normal((T, L.embed_dim)).astype(np.float32))
    got = R.forward(N, normalize=False)
    idx, w = R.last_routing(T)
    sel = sorted({int(idx[t, j]) for t in range(T) for j in range(L.top_k) if w[t, j] != 0})
    row_w = np.zeros((len(sel), T), np.float32)
    for t in range(T):
        for j in range(L.top_k):
            if w[t, j] != 0:
                row_w[sel.index(int(idx[t, j])), t] = w[t, j]
    want = np.zeros_like(N)
    M.moe_forward_rows_v2(gpu, [L.gates[e] for e in sel], [L.ups[e] for e in sel], [L.downs[e] for e in sel],
                          L.gate_fmt, [L.down_fmts[e] for e in sel], None, None, None, L.act, row_w, N, want,
                          L.embed_dim, L.inter_dim)
    tg.check(gpu)
    np.testing.assert_array_equal(got.view(np.uint32), want.view(np.uint32))


@pytest.fixture(scope="module")
def qwen16_batch(gpu):
    L = synth.qwen_layer(seed=1, n_experts=16)
    return L, ResidentLayer(L, max_tokens=96, lib=gpu)


def _abi_with_routing(gpu, L, N, idx, w):
    T = N.shape[0]
    sel = sorted({int(idx[t, j]) for t in range(T) for j in range(L.top_k) if w[t, j] != 0})
    row_w = np.zeros((len(sel), T), np.float32)
    for t in range(T):
        for j in range(L.top_k):
            if w[t, j] != 0:
                row_w[sel.index(int(idx[t, j])), t] = w[t, j]
    want = np.zeros_like(N)
    M.moe_forward_rows_v2(gpu, [L.gates[e] for e in sel], [L.ups[e] for e in sel], [L.downs[e] for e in sel],
                          L.gate_fmt, [L.down_fmts[e] for e in sel], None, None, None, L.act, row_w, N, want,
                          L.embed_dim, L.inter_dim)
    tg.check(gpu)
    return want


@pytest.mark.parametrize("T", [20, 64, 96])
def test_tensor_core_step_bit_exact_vs_gpu_abi_path(gpu, qwen16_batch, T):
    """Batched steps on the tcgen05 grouped GEMMs (exact per-sub-block int32
    sums read back from tensor memory, the reference's fp32 folds, the
    ordered combine) equal the GPU reference-ABI call on the step's routing."""
    L, R = qwen16_batch
    N = synth.rms_norm(np.random.default_rng(600 + T).standard_normal((T, 2048)).astype(np.float32))
    got = R.forward(N, normalize=False)
    idx, w = R.last_routing(T)
    want = _abi_with_routing(gpu, L, N, idx, w)
    np.testing.assert_array_equal(got.view(np.uint32), want.view(np.uint32))


def test_tensor_core_step_equals_matvec_step(gpu, qwen16_batch):
    L, R = qwen16_batch
    x = np.random.default_rng(700).standard_normal((40, 2048)).astype(np.float32)
    outs = []
    for tc in (True, False):
        R.set_tc(tc)
        outs.append(R.forward(x, normalize=True))
    R.set_tc(True)
    np.testing.assert_array_equal(outs[0].view(np.uint32), outs[1].view(np.uint32))


@pytest.fixture(scope="module")
def gptoss_batch(gpu):
    L = synth.gptoss_layer(seed=3, n_experts=32)
    return L, ResidentLayer(L, max_tokens=40, lib=gpu)


@pytest.mark.parametrize("T", [12, 40])
def test_tensor_core_step_bit_exact_vs_gpu_abi_path_mxfp4(gpu, gptoss_batch, T):
    """MXFP4 (gpt-oss, D = I = 2880: the last Q8 block of a row holds two
    live sub-blocks) on the tcgen05 grouped GEMMs: codes unpacked to int8 in
    shared memory, one int8 MMA per 32-value sub-block; T = 12 over 32
    experts leaves one or two active rows per expert, T = 40 up to a dozen."""
    L, R = gptoss_batch
    N = synth.rms_norm(np.random.default_rng(800 + T).standard_normal((T, L.embed_dim)).astype(np.float32))
    got = R.forward(N, normalize=False)
    idx, w = R.last_routing(T)
    want = _abi_with_routing(gpu, L, N, idx, w)
    np.testing.assert_array_equal(got.view(np.uint32), want.view(np.uint32))


def test_tensor_core_step_mxfp4_vs_oracle_and_matvec(gpu, oracle, gptoss_batch):
    L, R = gptoss_batch
    N = synth.rms_norm(np.random.default_rng(900).standard_normal((16, L.embed_dim)).astype(np.float32))
    outs = []
    for tc in (True, False):
        R.set_tc(tc)
        outs.append(R.forward(N, normalize=False))
    R.set_tc(True)
    np.testing.assert_array_equal(outs[0].view(np.uint32), outs[1].view(np.uint32))
    idx, w = R.last_routing(16)
    routing_agrees(L, N, idx, w)
    assert rel_err(outs[0], M.moe_layer_forward(oracle, L, N)) <= TOL


def test_fused_step_more_experts_than_sms(gpu, oracle):
    """200 experts: some CTAs hold two router rows."""
    L = synth.qwen_layer(seed=7, n_experts=200, D=512, I=256)
    R = ResidentLayer(L, max_tokens=4, lib=gpu)
    N = synth.rms_norm(np.random.default_rng(8).standard_normal((4, 512)).astype(np.float32))
    got = R.forward(N, normalize=False)
    idx, w = R.last_routing(4)
    routing_agrees(L, N, idx, w)
    want = M.moe_layer_forward(oracle, L, N)
    assert rel_err(got, want) <= TOL
    R.close()


def test_layer_rmsnorm_in_kernel(gpu, oracle, qwen16):
    L, R = qwen16
    x = np.random.default_rng(9).standard_normal((2, 2048)).astype(np.float32) * 3
    got = R.forward(x, normalize=True)
    want = M.moe_layer_forward(oracle, L, synth.rms_norm(x))
    assert rel_err(got, want) <= TOL


def test_layer_zipf_bias_and_clone(gpu, oracle):
    L = synth.qwen_layer(seed=2, n_experts=16, router_bias=synth.zipf_bias(seed=2, n_experts=16))
    R = ResidentLayer(L, max_tokens=4, lib=gpu)
    C = R.clone()
    N = synth.rms_norm(np.random.default_rng(3).standard_normal((4, 2048)).astype(np.float32))
    a = R.forward(N, normalize=False)
    b = C.forward(N, normalize=False)
    assert np.array_equal(a, b)
    want = M.moe_layer_forward(oracle, L, N)
    assert rel_err(a, want) <= TOL
    C.close()
    R.close()


def test_layer_gptoss_top4(gpu, oracle):
    L = synth.gptoss_layer(seed=3, n_experts=8)
    R = ResidentLayer(L, max_tokens=2, lib=gpu)
    N = synth.rms_norm(np.random.default_rng(5).standard_normal((2, 2880)).astype(np.float32))
    got = R.forward(N, normalize=False)
    want = M.moe_layer_forward(oracle, L, N)
    assert rel_err(got, want) <= TOL
    R.close()


def test_layer_shards_sum_to_whole(gpu, qwen16):
    """Expert-parallel shards: the parts of 4 shards add up to the whole layer."""
    L, R = qwen16
    N = synth.rms_norm(np.random.default_rng(6).standard_normal((3, 2048)).astype(np.float32))
    whole = R.forward(N, normalize=False)
    parts = [ResidentLayer(L, max_tokens=8, lib=gpu, shard=s, n_shards=4) for s in range(4)]
    total = sum(p.forward(N, normalize=False).astype(np.float64) for p in parts)
    assert rel_err(total, whole) <= 1e-6 * 10
    for p in parts:
        p.close()


def test_stack_of_clones_with_own_routers(gpu, oracle):
    """C5's construction: layers cloned from one set of experts, each given
    its own router by tg_layer_set_router, run as a device stack."""
    torch = pytest.importorskip("torch")
    import copy
    L = synth.qwen_layer(seed=4, n_experts=12)
    base = ResidentLayer(L, max_tokens=1, lib=gpu)
    res = [base, base.clone(), base.clone()]
    layers = []
    for l, r in enumerate(res):
        Ll = copy.copy(L)
        Ll.router_w = (np.random.default_rng([9, l]).standard_normal((12, 2048)) * 0.02).astype(np.float32)
        r.set_router(Ll.router_w)
        layers.append(Ll)
    x0 = np.random.default_rng(5).standard_normal((1, 2048)).astype(np.float32)
    want = x0.copy()
    for Ll in layers:
        want = want + M.moe_layer_forward(oracle, Ll, synth.rms_norm(want))
    stream = torch.cuda.Stream()
    gpu.tg_cuda_set_stream(ctypes.c_void_p(stream.cuda_stream))
    try:
        hs = (ctypes.c_void_p * 3)(*[r.h for r in res])
        x = torch.from_numpy(x0.copy()).cuda()
        with torch.cuda.stream(stream):
            assert gpu.tg_stack_forward_dev(hs, 3, ctypes.c_void_p(x.data_ptr()), 1, None) == 0
        torch.cuda.synchronize()
        tg.check(gpu)
        assert rel_err(x.cpu().numpy(), want) <= TOL
    finally:
        gpu.tg_cuda_set_stream(None)
        for r in res:
            r.close()


def test_stack_forward_and_graph_replay(gpu, oracle):
    torch = pytest.importorskip("torch")
    layers = [synth.qwen_layer(seed=4, layer=l, n_experts=12) for l in range(3)]
    res = [ResidentLayer(L, max_tokens=1, lib=gpu) for L in layers]
    x0 = np.random.default_rng(4).standard_normal((1, 2048)).astype(np.float32)
    # reference: x += moe(rmsnorm(x)) per layer, engine order
    want = x0.copy()
    for L in layers:
        want = want + M.moe_layer_forward(oracle, L, synth.rms_norm(want))
    stream = torch.cuda.Stream()
    gpu.tg_cuda_set_stream(ctypes.c_void_p(stream.cuda_stream))
    try:
        hs = (ctypes.c_void_p * 3)(*[r.h for r in res])
        x = torch.from_numpy(x0.copy()).cuda()
        with torch.cuda.stream(stream):
            assert gpu.tg_stack_forward_dev(hs, 3, ctypes.c_void_p(x.data_ptr()), 1, None) == 0
        torch.cuda.synchronize()
        tg.check(gpu)
        got = x.cpu().numpy()
        assert rel_err(got, want) <= TOL
        # the same stack captured in a graph and replayed
        x2 = torch.from_numpy(x0.copy()).cuda()
        g = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g, stream=stream):
            gpu.tg_stack_forward_dev(hs, 3, ctypes.c_void_p(x2.data_ptr()), 1, None)
        x2.copy_(torch.from_numpy(x0))
        with torch.cuda.stream(stream):
            g.replay()
        torch.cuda.synchronize()
        tg.check(gpu)
        assert np.array_equal(x2.cpu().numpy(), got)
        del g
    finally:
        gpu.tg_cuda_set_stream(None)
        for r in res:
            r.close()


@pytest.mark.parametrize("kind", ["q4k", "mxfp4"])
def test_tensor_core_int32_sums_bit_exact_vs_oracle(gpu, oracle, kind):
    """The tcgen05 grouped GEMM's int32 sub-block sums (read back from tensor
    memory) equal the oracle's (tgo_row_isums) bit for bit for every gate and
    up row of every active (expert, token) row of a batched step (T = 16):
    Q4_K sub-blocks of 32 values, and MXFP4 sub-blocks at D = 2880, whose
    last Q8 block holds two live sub-blocks."""
    import torch
    from tinygiant_b200 import quants as Q
    if kind == "q4k":
        L = synth.qwen_layer(seed=7, n_experts=8, top_k=2)
    else:
        L = synth.gptoss_layer(seed=3, layer=2, n_experts=8, top_k=2)
    T, D, I = 16, L.embed_dim, L.inter_dim
    nsb, rb = D // 32, Q.row_bytes(L.gate_fmt, D)
    R = ResidentLayer(L, max_tokens=T, lib=gpu)
    buf = torch.full((T * L.top_k * 2 * I * nsb,), -(2 ** 31), dtype=torch.int32, device="cuda")
    try:
        gpu.tg_cuda_debug_tc_isums(ctypes.c_void_p(buf.data_ptr()), None)
        N = synth.rms_norm(np.random.default_rng([71, T]).standard_normal((T, D)).astype(np.float32))
        R.forward(N, normalize=False)          # a fresh layer: its graph is captured with the hook on
    finally:
        gpu.tg_cuda_debug_tc_isums(None, None)
        R_idx, R_w = R.last_routing(T)
        R.close()
    dbg = buf.cpu().numpy().reshape(T * L.top_k, 2, I, nsb)
    xq = O.quantize_q8(oracle, N)
    sel = sorted({int(R_idx[t, j]) for t in range(T) for j in range(L.top_k) if R_w[t, j] != 0})
    p = 0
    want = np.zeros((I, nsb), np.int32)
    for e in sel:
        toks = [t for t in range(T) if any(int(R_idx[t, j]) == e and R_w[t, j] != 0 for j in range(L.top_k))]
        for t in toks:
            xt = np.ascontiguousarray(xq[t])
            for mat, Mx in enumerate((L.gates[e], L.ups[e])):
                for r in range(I):
                    oracle.tgo_row_isums(L.gate_fmt, Mx[r * rb:].ctypes.data, xt.ctypes.data, D, want[r].ctypes.data)
                np.testing.assert_array_equal(dbg[p, mat], want, err_msg=f"expert {e} token {t} matrix {mat}")
            p += 1
    assert p > T   # every token's rows were checked


def test_tensor_core_role_trace(gpu):
    """tg_cuda_tc_trace: one batched step fills the per-CTA role counters of
    both grouped-GEMM passes; on every CTA with units the units and steps
    match the unit count and steps per unit, and no role waited longer than
    its own span."""
    import torch
    L = synth.qwen_layer(seed=5, n_experts=16)
    T = 48
    R = ResidentLayer(L, max_tokens=T, lib=gpu)
    N = synth.rms_norm(np.random.default_rng(48).standard_normal((T, 2048)).astype(np.float32))
    try:
        R.forward(N, normalize=False)   # graph captured without the hook
        grid = gpu.tg_cuda_tc_trace(None)
        assert grid > 0
        buf = torch.zeros(2 * grid * 16, dtype=torch.int64, device="cuda")
        gpu.tg_cuda_tc_trace(ctypes.c_void_p(buf.data_ptr()))
        R2 = R.clone()                  # a fresh layer: its graph is captured with the hook on
        try:
            R2.forward(N, normalize=False)
        finally:
            gpu.tg_cuda_tc_trace(None)
            R2.close()
        tg.check(gpu)
    finally:
        R.close()
    v = buf.cpu().numpy().reshape(2, grid, 16)
    for p, steps_per_unit in ((0, 2048 // 256), (1, 2 * (768 // 256))):
        units, steps = v[p, :, 13], v[p, :, 14]
        busy = units > 0
        assert busy.any()
        np.testing.assert_array_equal(steps[busy], units[busy] * steps_per_unit)
        for wait, span in ((0, 1), (2, 4), (3, 4), (10, 12), (11, 12)):
            assert (v[p, busy, wait] <= v[p, busy, span]).all()
        assert (v[p, busy, 12] > 0).all()
