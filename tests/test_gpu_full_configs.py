"""Parity at BASELINE.json's full configurations, against the CPU oracle
(oracle/tg_oracle.c, itself bit-exact to the reference's compiled C on the
golden vectors), through the product library's C ABI on the GPU.

  C2  one Qwen3-30B-A3B layer, 128 experts, seed 1, T = 1: the fused step
      (tg_layer_forward with the RMS norm on the device)
  C3  the same shapes with the Zipf(1.1) router bias, seed 2, T = 8 (fused
      step), 64 and 512 (routing kernels + tcgen05 grouped GEMMs)
  v2  the reference-ABI entry tg_moe_forward_rows_v2 on the GPU at k = 64
      and 512 rows over all 128 experts' routing (engine.py:297-341)
  C4  gpt-oss-120b-shaped MXFP4 layer, 128 experts, seed 3, T = 1 and 32
  C1  tg_expert_forward and the same expert as a one-expert resident layer
      (the C1 bench line's device path)

Bar: routing identical to the reference router restated in numpy (top-k
ids in order, weights within rtol 1e-5 except across logit ties) and fp32
outputs within max|err| / max|ref| <= 1e-4 (TOL).  The oracle runs with
every host thread (its thread partition leaves results unchanged).
"""
import os

import numpy as np
import pytest

import tinygiant_b200 as tg
from tinygiant_b200 import moe as M
from tinygiant_b200 import quants as Q
from tinygiant_b200 import synth
from tinygiant_b200.layer import ResidentLayer

pytestmark = pytest.mark.gpu
TOL = 1e-4


def rel_err(got, ref):
    s = float(np.max(np.abs(ref)))
    return float(np.max(np.abs(got.astype(np.float64) - ref))) / (s if s > 0 else 1.0)


def routing_agrees(layer, N, idx, w):
    """Same experts in the same order and weights within rtol 1e-5, except
    where the reference's logits tie to within 1e-5 (fp32 order)."""
    _, _, ridx, rw = synth.route(layer, N)
    for t in range(N.shape[0]):
        if not np.array_equal(ridx[t], idx[t]):
            logits = layer.router_w @ N[t] + (0 if layer.router_b is None else layer.router_b)
            gaps = np.abs(np.diff(np.sort(logits)[::-1][:layer.top_k + 1]))
            assert gaps.min() < 1e-5, (t, ridx[t], idx[t])
        else:
            np.testing.assert_allclose(w[t], rw[t], rtol=1e-5, atol=1e-7)


@pytest.fixture(scope="module")
def threaded_oracle(oracle):
    oracle.tg_set_threads(os.cpu_count() or 1)
    yield oracle
    oracle.tg_set_threads(1)


@pytest.fixture(scope="module")
def c2(gpu):
    L = synth.qwen_layer(seed=1)
    R = ResidentLayer(L, max_tokens=8, lib=gpu)
    yield L, R
    R.close()


@pytest.fixture(scope="module")
def c3(gpu):
    L = synth.qwen_layer(seed=2, router_bias=synth.zipf_bias(seed=2))
    R = ResidentLayer(L, max_tokens=512, lib=gpu)
    yield L, R
    R.close()


@pytest.fixture(scope="module")
def c4(gpu):
    L = synth.gptoss_layer(seed=3)
    R = ResidentLayer(L, max_tokens=32, lib=gpu)
    yield L, R
    R.close()


def _inputs(seed, T, D):
    return np.random.default_rng([seed, 13]).standard_normal((T, D)).astype(np.float32)


@pytest.mark.parametrize("seed", [0, 1, 2, 3])
def test_c2_full_layer_fused_step_vs_oracle(gpu, threaded_oracle, c2, seed):
    """C2 at full size, T = 1, normalised on the device (the bench's step)."""
    L, R = c2
    x = _inputs(100 + seed, 1, 2048)
    got = R.forward(x, normalize=True)
    N = synth.rms_norm(x)
    idx, w = R.last_routing(1)
    routing_agrees(L, N, idx, w)
    want = M.moe_layer_forward(threaded_oracle, L, N)
    assert rel_err(got, want) <= TOL


@pytest.mark.parametrize("T", [8, 64, 512])
def test_c3_zipf_layer_vs_oracle(gpu, threaded_oracle, c3, T):
    """C3 at full size: T = 8 on the fused step, 64 and 512 on the routing
    kernels + tcgen05 grouped GEMMs, Zipf-skewed expert load."""
    L, R = c3
    N = synth.rms_norm(_inputs(200 + T, T, 2048))
    got = R.forward(N, normalize=False)
    idx, w = R.last_routing(T)
    routing_agrees(L, N, idx, w)
    want = M.moe_layer_forward(threaded_oracle, L, N)
    assert rel_err(got, want) <= TOL


@pytest.mark.parametrize("k", [64, 512])
def test_moe_forward_rows_v2_many_rows_vs_oracle(gpu, threaded_oracle, c3, k):
    """The reference-ABI entry on the GPU with the engine's argument
    construction at k = 64 and 512 rows (every expert of the union, dense
    row weights, output accumulated into a nonzero start)."""
    L, _ = c3
    rng = np.random.default_rng(300 + k)
    N = synth.rms_norm(rng.standard_normal((k, 2048)).astype(np.float32))
    init = (rng.standard_normal((k, 2048)) * 0.01).astype(np.float32)
    want = M.moe_layer_forward(threaded_oracle, L, N, init.copy())
    got = M.moe_layer_forward(gpu, L, N, init.copy())
    tg.check(gpu)
    assert rel_err(got, want) <= TOL


def test_moe_forward_rows_vs_oracle(gpu, threaded_oracle, c2):
    """tg_moe_forward_rows (Q4_K gate, SiLU, no biases; libtinygiant.c:1439-1448)."""
    import ctypes
    L, _ = c2
    N = synth.rms_norm(_inputs(400, 3, 2048))
    experts, row_w, _, _ = synth.route(L, N)
    sel = [int(e) for e in experts]
    outs = []
    for lib in (gpu, threaded_oracle):
        P = ctypes.c_void_p
        g = (P * len(sel))(*[L.gates[e].ctypes.data for e in sel])
        u = (P * len(sel))(*[L.ups[e].ctypes.data for e in sel])
        d = (P * len(sel))(*[L.downs[e].ctypes.data for e in sel])
        f = (ctypes.c_int * len(sel))(*[L.down_fmts[e] for e in sel])
        rw = np.ascontiguousarray(row_w, np.float32)
        out = np.zeros_like(N)
        lib.tg_moe_forward_rows(ctypes.addressof(g), ctypes.addressof(u), ctypes.addressof(d), ctypes.addressof(f),
                                len(sel), rw.ctypes.data, N.ctypes.data, out.ctypes.data, 3, 2048, 768)
        outs.append(out)
    tg.check(gpu)
    assert rel_err(outs[0], outs[1]) <= TOL


@pytest.mark.parametrize("T", [1, 32])
def test_c4_full_layer_vs_oracle(gpu, threaded_oracle, c4, T):
    """C4 at full size (128 MXFP4 experts, top-4, gpt-oss activation): T = 1
    on the fused step, 32 on the tcgen05 grouped GEMMs."""
    L, R = c4
    N = synth.rms_norm(_inputs(500 + T, T, 2880))
    got = R.forward(N, normalize=False)
    idx, w = R.last_routing(T)
    routing_agrees(L, N, idx, w)
    want = M.moe_layer_forward(threaded_oracle, L, N)
    assert rel_err(got, want) <= TOL


def test_c1_one_expert_layer_equals_expert_forward(gpu, threaded_oracle):
    """The C1 bench's device path (the expert as a one-expert layer, no norm,
    weight 1) equals tg_expert_forward bit for bit and the oracle within TOL."""
    e0 = synth.c1_expert(seed=0)
    D, I = 2048, 768
    gb = Q.row_bytes(Q.FMT_Q4K, D) * I
    L1 = synth.MoeLayer(D, I, Q.FMT_Q4K, 0, 1, gates=[e0[:gb]], ups=[e0[gb:2 * gb]], downs=[e0[2 * gb:]],
                        down_fmts=[Q.FMT_Q4K], router_w=np.zeros((1, D), np.float32))
    R = ResidentLayer(L1, max_tokens=1, lib=gpu)
    try:
        x = _inputs(600, 1, D)
        got = R.forward(x, normalize=False)
        ref = np.zeros(D, np.float32)
        gpu.tg_expert_forward(e0.ctypes.data, x.ctypes.data, ref.ctypes.data, 1.0, D, I)
        want = np.zeros(D, np.float32)
        threaded_oracle.tg_expert_forward(e0.ctypes.data, x.ctypes.data, want.ctypes.data, 1.0, D, I)
        tg.check(gpu)
        np.testing.assert_array_equal(got[0].view(np.uint32), ref.view(np.uint32))
        assert rel_err(got[0], want) <= TOL
    finally:
        R.close()
