"""Writes the golden fixtures in tests/golden/ from the REFERENCE itself.

    python tests/golden/make_golden.py          (needs the reference checkout: TG_REFERENCE_DIR)

Sources, all run in this container:
  * oracle/_ref/libtinygiant_ref_hooks.so — the reference's
    csrc/libtinygiant.c compiled unmodified (through oracle/neon_shim) with
    its static quantize_q8 / dot_fmt / dot_fmt_x4 / act_fn exported;
  * oracle/_ref/libtinygiant_ref.so — the same source as a library, for the
    exported entry points (tg_moe_forward_rows_v2, tg_expert_forward*, ...);
  * the reference's tinygiant.router.Router, imported from the checkout;
  * gguf-py's dequantize (independent block decoder, pinned version in
    fixtures' metadata).
Inputs are drawn from fixed numpy seeds and stored with the outputs, so the
fixtures do not depend on any generator at test time.
"""
import ctypes
import os
import sys
from pathlib import Path

import numpy as np

ROOT = Path(__file__).resolve().parents[2]
sys.path.insert(0, str(ROOT))
from oracle import oracle as O  # noqa: E402

OUT = Path(__file__).resolve().parent
REF = Path(os.environ.get("TG_REFERENCE_DIR", Path(__file__).resolve().parents[3] / "reference"))

VP, CI, CF = ctypes.c_void_p, ctypes.c_int, ctypes.c_float


def hooks():
    lib = ctypes.CDLL(str(ROOT / "oracle" / "_ref" / "libtinygiant_ref_hooks.so"))
    lib.refh_q8_block_bytes.restype = ctypes.c_size_t
    lib.refh_quantize_q8.argtypes = [VP, VP, CI]
    lib.refh_dot.argtypes = [CI, VP, VP, CI]
    lib.refh_dot.restype = CF
    lib.refh_dot_x4.argtypes = [CI, VP, VP, VP, VP, VP, CI, VP]
    lib.refh_act.argtypes = [CI, CF, CF]
    lib.refh_act.restype = CF
    assert lib.refh_q8_block_bytes() == O.Q8_BLOCK_BYTES
    return lib


def ref_q8(h, x):
    x = np.ascontiguousarray(x, np.float32)
    nb = (x.shape[-1] + 255) // 256
    out = np.zeros((x.shape[0], nb), O.Q8_DTYPE)
    for i in range(x.shape[0]):
        h.refh_quantize_q8(x[i].ctypes.data, out[i].ctypes.data, x.shape[-1])
    return out


# ---- weight generators (random blocks with sane fp16 scales) ----------

def rand_q4k(rng, rows, cols):
    nb = rows * cols // 256
    b = rng.integers(0, 256, size=(nb, 144), dtype=np.uint8)
    b[:, 0:2] = rng.uniform(0.002, 0.02, nb).astype(np.float16).view(np.uint8).reshape(nb, 2)
    b[:, 2:4] = rng.uniform(0.0005, 0.004, nb).astype(np.float16).view(np.uint8).reshape(nb, 2)
    return b.reshape(-1)


def rand_q6k(rng, rows, cols):
    nb = rows * cols // 256
    b = rng.integers(0, 256, size=(nb, 210), dtype=np.uint8)
    b[:, 192:208] = rng.integers(-60, 61, size=(nb, 16)).astype(np.int8).view(np.uint8)
    b[:, 208:210] = rng.uniform(0.0002, 0.002, nb).astype(np.float16).view(np.uint8).reshape(nb, 2)
    return b.reshape(-1)


def rand_mxfp4(rng, rows, cols):
    nsub = rows * cols // 32
    b = rng.integers(0, 256, size=(nsub, 17), dtype=np.uint8)
    b[:, 0] = rng.integers(116, 124, size=nsub)
    return b.reshape(-1)


def rand_q80(rng, rows, cols):
    nsub = rows * cols // 32
    b = rng.integers(0, 256, size=(nsub, 34), dtype=np.uint8)
    b[:, 0:2] = rng.uniform(0.001, 0.01, nsub).astype(np.float16).view(np.uint8).reshape(nsub, 2)
    return b.reshape(-1)


def rand_f16(rng, rows, cols):
    return (rng.standard_normal((rows, cols)) * 0.05).astype(np.float16).view(np.uint8).reshape(-1)


GEN = {0: rand_q4k, 1: rand_f16, 2: rand_q6k, 3: rand_mxfp4, 4: rand_q80}


def q8_cases(h):
    rng = np.random.default_rng(101)
    cases = {}
    x = rng.standard_normal((4, 2048)).astype(np.float32)
    cases["normal_2048"] = x
    cases["partial_2880"] = rng.standard_normal((3, 2880)).astype(np.float32) * 3
    cases["inter_768"] = (rng.standard_normal((2, 768)) * 0.01).astype(np.float32)
    z = np.zeros((2, 512), np.float32)
    z[1, 300] = -2.5                           # one non-zero value in the second block
    cases["zeros_and_single"] = z
    # exact ties: amax 127 makes inv = 1, so x.5 values round half to even
    t = np.tile(np.arange(-128, 128, dtype=np.float32) * 0.5, (1, 1))
    t[0, 0] = 127.0
    cases["ties"] = t
    cases["tiny"] = (rng.standard_normal((2, 256)) * 1e-30).astype(np.float32)
    cases["n32"] = rng.standard_normal((2, 32)).astype(np.float32)
    out = {}
    for name, xv in cases.items():
        out[f"x_{name}"] = xv
        out[f"q8_{name}"] = ref_q8(h, xv).view(np.uint8).reshape(xv.shape[0], -1)
    np.savez_compressed(OUT / "q8.npz", **out)


def dot_cases(h):
    rng = np.random.default_rng(202)
    out = {}
    for fmt, cols in ((0, 2048), (2, 768), (3, 2880), (4, 2880), (0, 768), (2, 512), (3, 320)):
        rows = 12
        mat = GEN[fmt](rng, rows, cols)
        rb = len(mat) // rows
        xs = (rng.standard_normal((4, cols)) * rng.uniform(0.1, 3)).astype(np.float32)
        q8 = ref_q8(h, xs)
        x1 = np.zeros((4, rows), np.float32)
        x4 = np.zeros((4, rows), np.float32)
        for r in range(rows):
            row = mat[r * rb:(r + 1) * rb]
            for t in range(4):
                x1[t, r] = h.refh_dot(fmt, row.ctypes.data, q8[t].ctypes.data, cols)
            o = np.zeros(4, np.float32)
            h.refh_dot_x4(fmt, row.ctypes.data, *[q8[t].ctypes.data for t in range(4)], cols, o.ctypes.data)
            x4[:, r] = o
        key = f"f{fmt}_c{cols}"
        out[f"{key}_mat"] = mat
        out[f"{key}_x"] = xs
        out[f"{key}_x1"] = x1
        out[f"{key}_x4"] = x4
    np.savez_compressed(OUT / "dots.npz", **out)


def act_cases(h):
    g = np.array([-30, -7.5, -1, -1e-3, 0, 1e-3, 0.5, 1, 6.9, 7, 7.1, 50], np.float32)
    u = np.array([-9, -7, -0.5, 0, 2, 8, 1, -3, 7.5, 0.25, -7.25, 3], np.float32)
    out = {"g": g, "u": u}
    for act in (0, 1):
        out[f"act{act}"] = np.array([h.refh_act(act, a, b) for a, b in zip(g, u)], np.float32)
    np.savez_compressed(OUT / "act.npz", **out)


def moe_cases(ref):
    """tg_moe_forward_rows_v2 on small shapes from the reference library."""
    rng = np.random.default_rng(303)
    out = {}
    specs = [
        # name, gate_fmt, down fmts, D, I, k, act, biases
        ("silu_mixed", 0, [0, 2, 2, 2], 256, 256, 6, 0, False),
        ("silu_f16down", 0, [1, 2], 256, 256, 3, 0, False),
        ("gptoss_bias", 3, [3, 3, 3], 160, 288, 5, 1, True),
        ("q80_gate", 4, [4, 2], 256, 256, 2, 0, True),
        ("q6k_gate_k1", 2, [2, 0, 2], 256, 256, 1, 0, False),
    ]
    for name, gf, dfs, D, I, k, act, biased in specs:
        E = len(dfs)
        gates = [GEN[gf](rng, I, D) for _ in range(E)]
        ups = [GEN[gf](rng, I, D) for _ in range(E)]
        downs = [GEN[f](rng, D, I) for f in dfs]
        rw = np.zeros((E, k), np.float32)
        for r in range(k):
            for e in rng.choice(E, size=min(E, 2 + r % 2), replace=False):
                rw[e, r] = rng.uniform(0.05, 0.6)
        xs = (rng.standard_normal((k, D)) * 0.7).astype(np.float32)
        gb = [(rng.standard_normal(I) * 0.3).astype(np.float32) for _ in range(E)] if biased else None
        ub = [(rng.standard_normal(I) * 0.3).astype(np.float32) for _ in range(E)] if biased else None
        db = [(rng.standard_normal(D) * 0.05).astype(np.float32) for _ in range(E)] if biased else None
        init = (rng.standard_normal((k, D)) * 0.1).astype(np.float32)   # output accumulates
        o = init.copy()
        O.moe_forward_rows_v2(ref, gates, ups, downs, gf, dfs, gb, ub, db, act, rw, xs, o, D, I)
        p = f"{name}_"
        out.update({p + "meta": np.array([gf, D, I, k, act, int(biased)], np.int64), p + "dfmts": np.array(dfs),
                    p + "rw": rw, p + "x": xs, p + "init": init, p + "out": o})
        for e in range(E):
            out[p + f"gate{e}"] = gates[e]
            out[p + f"up{e}"] = ups[e]
            out[p + f"down{e}"] = downs[e]
            if biased:
                out[p + f"gb{e}"], out[p + f"ub{e}"], out[p + f"db{e}"] = gb[e], ub[e], db[e]
    np.savez_compressed(OUT / "moe.npz", **out)


def expert_cases(ref):
    rng = np.random.default_rng(404)
    D, I = 256, 256
    out = {}
    q4 = np.concatenate([rand_q4k(rng, I, D), rand_q4k(rng, I, D), rand_q4k(rng, D, I)])
    x = (rng.standard_normal(D) * 0.8).astype(np.float32)
    o = (rng.standard_normal(D) * 0.1).astype(np.float32)
    out["fwd_q4"], out["fwd_x"], out["fwd_init"] = q4, x, o.copy()
    ref.tg_expert_forward(q4.ctypes.data, x.ctypes.data, o.ctypes.data, 0.375, D, I)
    out["fwd_out"] = o
    gate, up = rand_q4k(rng, I, D), rand_q4k(rng, I, D)
    out["mixed_gate"], out["mixed_up"] = gate, up
    for dfmt in (0, 1, 2):
        down = GEN[dfmt](rng, D, I)
        o = np.zeros(D, np.float32)
        ref.tg_expert_forward_mixed(gate.ctypes.data, up.ctypes.data, down.ctypes.data, dfmt, x.ctypes.data,
                                    o.ctypes.data, 0.5, D, I)
        out[f"mixed_down{dfmt}"], out[f"mixed_out{dfmt}"] = down, o
    for k in (1, 3, 6):
        down = rand_q6k(rng, D, I)
        xs = (rng.standard_normal((k, D)) * 0.8).astype(np.float32)
        w = rng.uniform(0.1, 1.0, k).astype(np.float32)
        o = np.zeros((k, D), np.float32)
        ref.tg_expert_forward_rows(gate.ctypes.data, up.ctypes.data, down.ctypes.data, 2, xs.ctypes.data,
                                   o.ctypes.data, w.ctypes.data, k, D, I)
        out[f"rows{k}_down"], out[f"rows{k}_x"], out[f"rows{k}_w"], out[f"rows{k}_out"] = down, xs, w, o
    experts = [np.concatenate([rand_q4k(rng, I, D), rand_q4k(rng, I, D), rand_q4k(rng, D, I)]) for _ in range(3)]
    w = np.array([0.5, 0.3, 0.2], np.float32)
    o = np.full(D, 7.0, np.float32)      # tg_moe_forward zeroes its output first
    arr = O.pointer_array(experts)
    ref.tg_moe_forward(ctypes.addressof(arr), w.ctypes.data, 3, x.ctypes.data, o.ctypes.data, D, I)
    for i, e in enumerate(experts):
        out[f"moef_e{i}"] = e
    out["moef_w"], out["moef_out"] = w, o
    np.savez_compressed(OUT / "expert.npz", **out)


def matmul_cases(ref):
    rng = np.random.default_rng(505)
    out = {}
    for fmt, cols in ((0, 512), (2, 512), (3, 544), (4, 544), (1, 200)):
        rows = 20
        mat = GEN[fmt](rng, rows, cols)
        x = rng.standard_normal(cols).astype(np.float32)
        bias = rng.standard_normal(rows).astype(np.float32)
        o_b = np.zeros(rows, np.float32)
        o_n = np.zeros(rows, np.float32)
        ref.tg_matmul(fmt, mat.ctypes.data, bias.ctypes.data, x.ctypes.data, o_b.ctypes.data, rows, cols)
        ref.tg_matmul(fmt, mat.ctypes.data, None, x.ctypes.data, o_n.ctypes.data, rows, cols)
        key = f"f{fmt}"
        out.update({key + "_mat": mat, key + "_x": x, key + "_bias": bias, key + "_out_bias": o_b,
                    key + "_out_nobias": o_n, key + "_shape": np.array([rows, cols])})
    for name, fn, fmt, cols in (("q4k", ref.tg_matmul_q4k, 0, 2048), ("q6k", ref.tg_matmul_q6k, 2, 768)):
        rows = 24
        mat = GEN[fmt](rng, rows, cols)
        x = rng.standard_normal(cols).astype(np.float32)
        o = np.zeros(rows, np.float32)
        fn(mat.ctypes.data, x.ctypes.data, o.ctypes.data, rows, cols)
        out.update({f"mm_{name}_mat": mat, f"mm_{name}_x": x, f"mm_{name}_out": o})
    A = rng.standard_normal((33, 77)).astype(np.float32)
    x = rng.standard_normal(77).astype(np.float32)
    o = np.zeros(33, np.float32)
    ref.tg_f32_matvec(A.ctypes.data, x.ctypes.data, o.ctypes.data, 33, 77)
    out.update({"f32_A": A, "f32_x": x, "f32_out": o})
    A16 = rand_f16(rng, 33, 77)
    o = np.zeros(33, np.float32)
    ref.tg_f16_matvec(A16.ctypes.data, x.ctypes.data, o.ctypes.data, 33, 77)
    out.update({"f16_A": A16, "f16_out": o})
    xn = rng.standard_normal(2050).astype(np.float32)
    wn = rng.uniform(0.5, 1.5, 2050).astype(np.float32)
    o = np.zeros(2050, np.float32)
    ref.tg_rms_norm(xn.ctypes.data, wn.ctypes.data, o.ctypes.data, 2050, ctypes.c_float(1e-6))
    out.update({"rms_x": xn, "rms_w": wn, "rms_out": o})
    np.savez_compressed(OUT / "matmul.npz", **out)


def router_cases():
    sys.path.insert(0, str(REF))
    from tinygiant.router import Router  # the reference's own router
    rng = np.random.default_rng(606)
    out = {}
    for name, E, D, k, biased in (("qwen", 128, 256, 8, False), ("zipf", 128, 256, 8, True),
                                  ("gptoss", 64, 160, 4, False)):
        W = (rng.standard_normal((E, D)) * 0.02).astype(np.float32)
        b = (-1.1 * np.log(rng.permutation(E) + 1)).astype(np.float32) if biased else None
        r = Router([W], k, biases=[b] if biased else None)
        N = rng.standard_normal((6, D)).astype(np.float32)
        idx = np.zeros((6, k), np.int64)
        wts = np.zeros((6, k), np.float32)
        for t in range(6):
            lg = r.logits(0, N[t])
            i, w = r.select(lg)
            idx[t], wts[t] = i, w
        out.update({f"{name}_W": W, f"{name}_N": N, f"{name}_idx": idx, f"{name}_wts": wts})
        if biased:
            out[f"{name}_b"] = b
    np.savez_compressed(OUT / "router.npz", **out)


def gguf_cases():
    """Block decodes by gguf-py (an independent decoder) for layout checks."""
    import gguf
    from gguf import GGMLQuantizationType as T
    from gguf.quants import dequantize
    rng = np.random.default_rng(707)
    out = {"gguf_version": np.array(gguf.__version__ if hasattr(gguf, "__version__") else "unknown")}
    for name, fmt, t, cols in (("q4k", 0, T.Q4_K, 512), ("q6k", 2, T.Q6_K, 512), ("mxfp4", 3, T.MXFP4, 64),
                               ("q80", 4, T.Q8_0, 64)):
        mat = GEN[fmt](rng, 8, cols)
        out[f"{name}_mat"] = mat
        out[f"{name}_deq"] = dequantize(mat.reshape(8, -1), t).astype(np.float32)
    np.savez_compressed(OUT / "gguf.npz", **out)


def main():
    O.build()
    h = hooks()
    ref = O.load_reference()
    assert ref is not None, "oracle/_ref/libtinygiant_ref.so was not built"
    ref.tg_set_threads(4)
    q8_cases(h)
    dot_cases(h)
    act_cases(h)
    moe_cases(ref)
    expert_cases(ref)
    matmul_cases(ref)
    router_cases()
    gguf_cases()
    for p in sorted(OUT.glob("*.npz")):
        print(f"{p.name:12s} {p.stat().st_size:>9d} bytes")


if __name__ == "__main__":
    main()
