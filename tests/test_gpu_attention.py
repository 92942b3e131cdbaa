"""Attention decode steps on the GPU (tg_attention_v2, tg_attention_decode,
tg_attention_decode_q4) against the reference's own C (oracle/_ref, built
from its source), over a sequence of positions that appends to the KV
cache: the outputs and the KV rows written back into the caller's arrays
agree within 1e-4 of max|ref| (fp32 softmax, norms and sums in another
order).  A cache the caller filled on the host before the first GPU call is
uploaded to the device mirror."""
import ctypes

import numpy as np
import pytest

from oracle import oracle as O
from tinygiant_b200 import quants as Q
from tinygiant_b200._lib import ABI

pytestmark = pytest.mark.gpu
TOL = 1e-4
D, H, KH, HD, KV_MAX = 512, 8, 2, 64, 24


@pytest.fixture(scope="module")
def ref():
    if not O.REF_SO.exists():
        pytest.skip("oracle/_ref/libtinygiant_ref.so not built")
    lib = ctypes.CDLL(str(O.REF_SO))
    for name in ("tg_attention_v2", "tg_attention_decode", "tg_attention_decode_q4", "tg_transformer_layer",
                 "tg_set_threads"):
        fn = getattr(lib, name)
        fn.argtypes, fn.restype = ABI[name] if name in ABI else ([ctypes.c_int], None)
    lib.tg_set_threads(4)
    return lib


def rel_err(got, want):
    s = float(np.max(np.abs(want)))
    return float(np.max(np.abs(got.astype(np.float64) - want))) / (s if s > 0 else 1.0)


def rope_tables():
    half = HD // 2
    inv = 1.0 / (10000.0 ** (np.arange(half) * 2.0 / HD))
    ang = np.arange(KV_MAX)[:, None] * inv[None, :]
    return np.cos(ang).astype(np.float32), np.sin(ang).astype(np.float32)


def weights(rng, fmt, rows, cols):
    w = (rng.standard_normal((rows, cols)) * 0.05).astype(np.float32)
    if fmt == Q.FMT_Q4K:
        return Q.pack_q4k(w)
    if fmt == Q.FMT_Q6K:
        return Q.pack_q6k(w)
    if fmt == Q.FMT_F16:
        return np.ascontiguousarray(w.astype(np.float16)).view(np.uint8).reshape(-1)
    return w   # fp32


def p(a):
    return None if a is None else a.ctypes.data


def run_sequence(gpu, ref, call, steps, prefill=0, seed=0):
    """call(lib, kvk, kvv, kv_len, x, out) for positions 0 .. steps-1 on both
    libraries (the first `prefill` positions on the reference only, then its
    cache copied into the GPU's)."""
    rng = np.random.default_rng(seed)
    caches = {}
    for name in ("ref", "gpu"):
        caches[name] = (np.zeros((KH, KV_MAX, HD), np.float32), np.zeros((KH, KV_MAX, HD), np.float32))
    for pos in range(steps):
        x = rng.standard_normal(D).astype(np.float32)
        outs = {}
        for name, lib in (("ref", ref), ("gpu", gpu)):
            if name == "gpu" and pos < prefill:
                continue
            if name == "gpu" and pos == prefill:
                if prefill:
                    caches["gpu"][0][:] = caches["ref"][0]
                    caches["gpu"][1][:] = caches["ref"][1]
                # a cache written on the host (or new at a reused address):
                # drop any device mirror of it, as the API asks
                gpu.tg_cuda_unregister(p(caches["gpu"][0]))
                gpu.tg_cuda_unregister(p(caches["gpu"][1]))
            out = np.zeros(D, np.float32)
            call(lib, caches[name][0], caches[name][1], pos, x, out)
            outs[name] = out
        if pos < prefill:
            continue
        msg = ctypes.create_string_buffer(512)
        assert gpu.tg_cuda_last_error(msg, 512) == 0, msg.value
        assert rel_err(outs["gpu"], outs["ref"]) <= TOL, pos
        for c in (0, 1):
            assert rel_err(caches["gpu"][c][:, pos], caches["ref"][c][:, pos]) <= TOL, (pos, c)
    for c in (0, 1):
        assert rel_err(caches["gpu"][c][:, :steps], caches["ref"][c][:, :steps]) <= TOL


@pytest.mark.parametrize("window,sinks,prefill", [(0, False, 0), (5, True, 0), (0, True, 3)])
def test_attention_v2_matches_reference(gpu, ref, window, sinks, prefill):
    rng = np.random.default_rng(10 + window)
    fq, fk, fv, fo = Q.FMT_Q4K, Q.FMT_Q6K, Q.FMT_F16, Q.FMT_Q4K
    wq, wk, wv, wo = (weights(rng, fq, H * HD, D), weights(rng, fk, KH * HD, D), weights(rng, fv, KH * HD, D),
                      weights(rng, fo, D, H * HD))
    bq, bk, bv, bo = [(rng.standard_normal(n) * 0.1).astype(np.float32) for n in (H * HD, KH * HD, KH * HD, D)]
    qn, kn = [(1.0 + 0.1 * rng.standard_normal(HD)).astype(np.float32) for _ in range(2)]
    sk = (rng.standard_normal(H)).astype(np.float32) if sinks else None
    cos, sin = rope_tables()

    def call(lib, kvk, kvv, pos, x, out):
        lib.tg_attention_v2(fq, fk, fv, fo, p(wq), p(wk), p(wv), p(wo), p(bq), p(bk), p(bv), p(bo), p(qn), p(kn),
                            p(sk), p(kvk), p(kvv), pos, KV_MAX, window, p(cos), p(sin), p(x), p(out),
                            D, H, KH, HD, pos, 1e-6)

    run_sequence(gpu, ref, call, steps=10, prefill=prefill, seed=window)


def test_attention_decode_f32_matches_reference(gpu, ref):
    rng = np.random.default_rng(21)
    wq, wk, wv, wo = (weights(rng, None, H * HD, D), weights(rng, None, KH * HD, D), weights(rng, None, KH * HD, D),
                      weights(rng, None, D, H * HD))
    qn, kn = [(1.0 + 0.1 * rng.standard_normal(HD)).astype(np.float32) for _ in range(2)]
    cos, sin = rope_tables()

    def call(lib, kvk, kvv, pos, x, out):
        lib.tg_attention_decode(p(wq), p(wk), p(wv), p(wo), p(qn), p(kn), p(kvk), p(kvv), pos, KV_MAX, p(cos), p(sin),
                                p(x), p(out), D, H, KH, HD, pos)

    run_sequence(gpu, ref, call, steps=8, seed=1)


def test_attention_decode_q4_matches_reference(gpu, ref):
    rng = np.random.default_rng(22)
    wq, wk = weights(rng, Q.FMT_Q4K, H * HD, D), weights(rng, Q.FMT_Q4K, KH * HD, D)
    wv, wo = weights(rng, Q.FMT_F16, KH * HD, D), weights(rng, Q.FMT_Q4K, D, H * HD)
    qn, kn = [(1.0 + 0.1 * rng.standard_normal(HD)).astype(np.float32) for _ in range(2)]
    cos, sin = rope_tables()

    def call(lib, kvk, kvv, pos, x, out):
        lib.tg_attention_decode_q4(p(wq), p(wk), p(wv), p(wo), p(qn), p(kn), p(kvk), p(kvv), pos, KV_MAX, p(cos),
                                   p(sin), p(x), p(out), D, H, KH, HD, pos)

    run_sequence(gpu, ref, call, steps=8, seed=2)


@pytest.mark.parametrize("window,sinks", [(0, True), (700, False)])
def test_attention_long_context_matches_reference(gpu, ref, window, sinks):
    """A 1,000-position context, filled on the host, split over several CTAs
    per head on the GPU (and a sliding window of 700)."""
    rng = np.random.default_rng(41 + window)
    L0, kv_max, steps = 1000, 1008, 3
    fq = fk = fv = fo = Q.FMT_Q4K
    wq, wk, wv, wo = (weights(rng, fq, H * HD, D), weights(rng, fk, KH * HD, D), weights(rng, fv, KH * HD, D),
                      weights(rng, fo, D, H * HD))
    qn, kn = [(1.0 + 0.1 * rng.standard_normal(HD)).astype(np.float32) for _ in range(2)]
    sk = rng.standard_normal(H).astype(np.float32) if sinks else None
    half = HD // 2
    ang = np.arange(kv_max)[:, None] * (1.0 / (10000.0 ** (np.arange(half) * 2.0 / HD)))[None, :]
    cos, sin = np.cos(ang).astype(np.float32), np.sin(ang).astype(np.float32)
    kv0 = [(rng.standard_normal((KH, kv_max, HD)) * 0.5).astype(np.float32) for _ in range(2)]
    caches = {n: [c.copy() for c in kv0] for n in ("ref", "gpu")}
    for c in caches["gpu"]:
        gpu.tg_cuda_unregister(p(c))
    for pos in range(L0, L0 + steps):
        x = rng.standard_normal(D).astype(np.float32)
        outs = {}
        for name, lib in (("ref", ref), ("gpu", gpu)):
            out = np.zeros(D, np.float32)
            kk, vv = caches[name]
            lib.tg_attention_v2(fq, fk, fv, fo, p(wq), p(wk), p(wv), p(wo), None, None, None, None, p(qn), p(kn),
                                p(sk), p(kk), p(vv), pos, kv_max, window, p(cos), p(sin), p(x), p(out),
                                D, H, KH, HD, pos, 1e-6)
            outs[name] = out
        msg = ctypes.create_string_buffer(512)
        assert gpu.tg_cuda_last_error(msg, 512) == 0, msg.value
        assert rel_err(outs["gpu"], outs["ref"]) <= TOL, pos


def test_transformer_layer_matches_reference(gpu, ref):
    """x += attention(rms_norm(x)); x += sum_e w_e expert_e(rms_norm(x)), the
    experts pre-routed (Q4_K gate/up, Q4_K or F16 down), over 4 positions."""
    rng = np.random.default_rng(31)
    I = 256
    wq, wk, wv, wo = (weights(rng, None, H * HD, D), weights(rng, None, KH * HD, D), weights(rng, None, KH * HD, D),
                      weights(rng, None, D, H * HD))
    an, fn = [(1.0 + 0.1 * rng.standard_normal(D)).astype(np.float32) for _ in range(2)]
    qn, kn = [(1.0 + 0.1 * rng.standard_normal(HD)).astype(np.float32) for _ in range(2)]
    cos, sin = rope_tables()
    f16 = [0, 1, 0]
    gates = [weights(rng, Q.FMT_Q4K, I, D) for _ in f16]
    ups = [weights(rng, Q.FMT_Q4K, I, D) for _ in f16]
    downs = [weights(rng, Q.FMT_F16 if f else Q.FMT_Q4K, D, I) for f in f16]
    VPA = ctypes.c_void_p * len(f16)
    gp, up_, dp = VPA(*[p(a) for a in gates]), VPA(*[p(a) for a in ups]), VPA(*[p(a) for a in downs])
    isf = (ctypes.c_int * len(f16))(*f16)
    ew = np.array([0.5, 0.3, 0.2], np.float32)
    caches = {n: (np.zeros((KH, KV_MAX, HD), np.float32), np.zeros((KH, KV_MAX, HD), np.float32))
              for n in ("ref", "gpu")}
    for c in caches["gpu"]:
        gpu.tg_cuda_unregister(p(c))
    for pos in range(4):
        x0 = rng.standard_normal(D).astype(np.float32)
        xs = {}
        for name, lib in (("ref", ref), ("gpu", gpu)):
            x = x0.copy()
            lib.tg_transformer_layer(p(wq), p(wk), p(wv), p(wo), p(an), p(qn), p(kn), p(fn), p(caches[name][0]),
                                     p(caches[name][1]), pos, KV_MAX, p(cos), p(sin), ctypes.addressof(gp),
                                     ctypes.addressof(up_), ctypes.addressof(dp), ctypes.addressof(isf), p(ew),
                                     len(f16), p(x), D, I, H, KH, HD, pos)
            xs[name] = x
        msg = ctypes.create_string_buffer(512)
        assert gpu.tg_cuda_last_error(msg, 512) == 0, msg.value
        assert rel_err(xs["gpu"], xs["ref"]) <= TOL, pos
        assert rel_err(caches["gpu"][0][:, pos], caches["ref"][0][:, pos]) <= TOL


def test_attention_rejects_bad_shapes(gpu):
    x = np.zeros(D, np.float32)
    out = np.ones(D, np.float32)
    kv = np.zeros((KH, KV_MAX, HD), np.float32)
    cos, sin = rope_tables()
    w = np.zeros((H * HD, D), np.float32)
    gpu.tg_attention_decode(p(w), p(w), p(w), p(w), p(cos[0]), p(cos[0]), p(kv), p(kv), KV_MAX, KV_MAX, p(cos),
                            p(sin), p(x), p(out), D, H, KH, HD, 0)   # kv_len == kv_max
    assert gpu.tg_cuda_last_error(None, 0) != 0
    assert np.all(out == 1.0)
