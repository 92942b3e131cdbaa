"""Phase timeline of the fused layer step (diagnostics).

The fused step kernel (tg_step.cu) can record, per CTA, SM-clock timestamps
at its phase boundaries and, per warp, the cycles its weight ring spent
waiting, computing and issuing copies (tg_cuda_step_trace).  This module
runs steps of a resident layer with tracing on and reports the median and
maximum over CTAs / warps of each phase, in microseconds (cycles are
converted with the CTA's own global-timer span).

    python -m tinygiant_b200.steptrace [--experts 128] [--copies 4] [--tokens 1] [--gptoss]
"""
import argparse
import ctypes

import numpy as np

PHASES = [
    ("launch -> inputs ready", 0, 1),
    ("R: x + router rows (w0)", 1, 3),
    ("R1: sums, partial logits (w0)", 3, 16),
    ("R2: rr, logits (CTA)", 16, 17),
    ("logits poll (w0)", 2, 9),
    ("top-k, softmax (+plan) (w0)", 9, 14),
    ("  sort network (w0)", 9, 22),
    ("  top-k rounds (w0)", 22, 23),
    ("  softmax (w0)", 23, 24),
    ("  plan T=1 (w0)", 24, 14),
    ("R3: Q8 of N (first R3 warp)", 20, 18),
    ("S / R3 CTA sync (w0)", 14, 21),
    ("plan (T>1)", 21, 4),
    ("phase A (warp 0)", 4, 5),
    ("hidden poll (warp 0)", 5, 6),
    ("Q8 of hidden (warp 0)", 6, 15),
    ("CTA sync", 15, 7),
    ("phase B (warp 0)", 7, 8),
]
WARP = ["A wait", "A compute", "A issue", "B wait", "B compute", "B issue"]
SLOTS = 32   # trace words per CTA


def trace(lib, step, n_steps=1):
    """Runs `step()` n_steps times with tracing on; returns (phases, warps,
    counts): dicts name -> array over CTAs / warps (last step); phases and
    warps in microseconds (cycles are converted with the CTA's own
    global-timer span), counts in polls."""
    import torch

    grid = lib.tg_cuda_step_trace(None)
    buf = torch.zeros(grid * SLOTS + grid * 16 * 8, dtype=torch.int64, device="cuda")
    torch.cuda.synchronize()
    lib.tg_cuda_step_trace(ctypes.c_void_p(buf.data_ptr()))
    try:
        for _ in range(n_steps):
            step()
        torch.cuda.synchronize()
    finally:
        lib.tg_cuda_step_trace(None)
    v = buf.cpu().numpy().astype(np.int64)
    t = v[: grid * SLOTS].reshape(grid, SLOTS)
    span_ns = (t[:, 13] - t[:, 12]).astype(np.float64)
    span_cyc = (t[:, 8] - t[:, 0]).astype(np.float64)
    cyc_per_us = np.median(span_cyc / np.maximum(span_ns, 1.0)) * 1000.0
    phases = {name: (t[:, b] - t[:, a]) / cyc_per_us for name, a, b in PHASES}
    phases["whole step (CTA)"] = span_ns / 1000.0
    wv = v[grid * SLOTS:].reshape(grid * 16, 8)
    w = wv[:, :6] / cyc_per_us
    warps = {name: w[:, i] for i, name in enumerate(WARP)}
    warps["A end -> hidden ready"] = wv[:, 7] / cyc_per_us
    counts = {"logits polls (CTA)": t[:, 19], "hidden polls (warp)": wv[:, 6]}
    return phases, warps, counts


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--experts", type=int, default=128)
    ap.add_argument("--copies", type=int, default=4)
    ap.add_argument("--tokens", type=int, default=1)
    ap.add_argument("--gptoss", action="store_true", help="the gpt-oss-shaped MXFP4 layer (C4) instead of Qwen3 (C2)")
    a = ap.parse_args()
    import torch

    import tinygiant_b200 as tg
    from tinygiant_b200 import synth
    from tinygiant_b200.layer import ResidentLayer

    lib = tg.load()
    L = synth.gptoss_layer(seed=3, n_experts=a.experts) if a.gptoss else synth.qwen_layer(seed=1, n_experts=a.experts)
    base = ResidentLayer(L, max_tokens=a.tokens, lib=lib)
    lays = [base] + [base.clone() for _ in range(a.copies - 1)]
    stream = torch.cuda.Stream()
    lib.tg_cuda_set_stream(ctypes.c_void_p(stream.cuda_stream))
    x = torch.randn(a.tokens, L.embed_dim, device="cuda")
    out = torch.zeros_like(x)
    it = [0]

    def step():
        lay = lays[it[0] % len(lays)]
        it[0] += 1
        lib.tg_layer_forward_dev(lay.h, ctypes.c_void_p(x.data_ptr()), None, None, ctypes.c_void_p(out.data_ptr()),
                                 a.tokens, 1, None)

    try:
        with torch.cuda.stream(stream):
            for _ in range(20):
                step()
            torch.cuda.synchronize()
            for tag, n in (("one step after idle", 1), ("last of 8 back-to-back steps", 8)):
                phases, warps, counts = trace(lib, step, n)
                print(f"== {tag}")
                for name, d in phases.items():
                    print(f"  {name:28s} median {np.median(d):7.2f} us   max {d.max():7.2f}")
                for name, d in warps.items():
                    print(f"  per-warp {name:21s} median {np.median(d):7.2f} us   max {d.max():7.2f}")
                for name, d in counts.items():
                    print(f"  {name:28s} median {np.median(d):7.1f}      max {d.max():7.0f}")
        tg.check(lib)
    finally:
        lib.tg_cuda_set_stream(None)


if __name__ == "__main__":
    main()
