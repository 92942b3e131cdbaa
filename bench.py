"""Benchmark: MoE-layer decode tok/s and fused quant-matvec HBM GB/s on B200.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]
                    [--config c2|c3|c4|c5|attn|cache] [--tokens T] [--layers L]

Default workload (the headline configuration, "C2"): one Qwen3-30B-A3B-shaped MoE
layer at batch 1 — 128 experts (Q4_K gate/up 768x2048, Q6_K down 2048x768),
fp32 router [128 x 2048], top-8 softmax, weights from seed 1, x ~ N(0, 1).
A step is one layer-token: rmsnorm -> router -> top-8 -> 8 experts on the
GPU.  Synthetic data; every expert of every copy is HBM-resident.

Timing (device): W warm-up steps, then K steps captured in one CUDA graph,
bracketed by barrier + synchronize, CUDA events on the library's stream, max
over ranks.  Steps cycle through R HBM copies of the layer (6.3 GB at R=16),
so each step's 24.5 MB of experts were last touched 15 steps (~390 MB of
traffic) earlier and are not L2-resident.

e2e: the same step through the C-ABI entry tg_layer_forward with host
buffers (x in, MoE output back), host<->device copies inside the timed region.

Multi-GPU (torchrun), --parallel dp (default): every GPU holds the layer
and serves its own tokens; no collective on the data path, per-GPU work is
fixed ("weak").  --parallel ep: experts sharded by id (e % N == rank), router
replicated, one NCCL all-reduce of the [T, D] output per step; total work is
fixed ("strong").

--impl reference: the reference's own CPU path on the host cores — its router
(restated in synth.route, checked against tinygiant/router.py) + its
csrc/libtinygiant.c tg_moe_forward_rows_v2 (oracle/_ref, compiled from the
reference's source) with every host thread.
"""
import argparse
import ctypes
import json
import os
import statistics
import subprocess
import sys
import threading
import time
from pathlib import Path

import numpy as np

ROOT = Path(__file__).resolve().parent
sys.path.insert(0, str(ROOT))

METRIC = "MoE-layer decode tok/s; fused quant-matvec HBM GB/s vs ~8 TB/s B200 peak"
UNIT = "tok/s"
R_COPIES = 16
DTYPES = {"c2": "int8xQ4_K/Q6_K (int32 accumulate), fp32 combine",
          "c3": "int8xQ4_K/Q6_K (int32 accumulate), fp32 combine",
          "c4": "int8xMXFP4 (int32 accumulate), fp32 combine",
          "c5": "int8xQ4_K/Q6_K (int32 accumulate), fp32 combine"}


def parse():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=2000)
    ap.add_argument("--warmup", type=int, default=10)
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--config", default="c2", choices=["c2", "c3", "c4", "c5", "attn", "cache"],
                    help="c2-c5: the MoE workloads; attn: one attention decode step (tg_attention_v2); "
                         "cache: an expert-cache directory loaded into HBM")
    ap.add_argument("--tokens", type=int, default=None)
    ap.add_argument("--copies", type=int, default=R_COPIES)
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--parallel", default="dp", choices=["dp", "ep"])
    ap.add_argument("--layers", type=int, default=None,
                    help="C4 / C5: layers in the stack (default 36 / 48; C4 with 1: one layer over HBM copies)")
    ap.add_argument("--matvec", action="store_true",
                    help="batched steps (T > 8) on the matvec kernels instead of the tcgen05 grouped GEMMs")
    ap.add_argument("--ep-nccl", action="store_true",
                    help="expert parallel: sum the shards with an NCCL all-reduce instead of inside the step kernel")
    return ap.parse_args()


# ---- workload ------------------------------------------------------------

def make_layer(cfg):
    from tinygiant_b200 import synth
    if cfg == "c4":
        return synth.gptoss_layer(seed=3)
    if cfg == "c3":
        return synth.qwen_layer(seed=2, router_bias=synth.zipf_bias(seed=2))
    return synth.qwen_layer(seed=1)


def workload_desc(cfg, T, R, L):
    names = {
        "c2": "C2: one Qwen3-30B-A3B MoE layer (128 experts, Q4_K gate/up, Q6_K down, top-8, D=2048, I=768)",
        "c3": "C3: Qwen3-30B-A3B MoE layer with Zipf(1.1)-skewed router bias",
        "c4": "C4: gpt-oss-120b-shaped MXFP4 MoE layer (128 experts, top-4, D=I=2880)",
        "c4s": "C4: gpt-oss-120b-shaped MXFP4 MoE stack (128 experts per layer, top-4, D=I=2880, per-layer routers, "
               "residual add)",
        "c5": "C5: Qwen3-30B-A3B MoE-FFN stack (C2 experts per layer, per-layer routers, residual add)",
    }
    return {"workload": names[cfg], "tokens_per_step": T, "experts": L.n_experts, "top_k": L.top_k,
            "embed_dim": L.embed_dim, "inter_dim": L.inter_dim, "layer_copies": R,
            "l2": f"inputs larger than L2: steps cycle {R} HBM copies of the layer",
            "step": "rmsnorm + router + top-k softmax + experts (gate/up/act/down/combine)"}


def step_inputs(n, T, D, seed=4):
    rng = np.random.default_rng([seed, 7])
    return rng.standard_normal((n, T, D)).astype(np.float32)


def algorithmic_bytes(L, xs):
    """Per step: each distinct selected expert's weight bytes once + the fp32
    router + x in and out; routing by the reference router."""
    from tinygiant_b200 import synth
    eb = L.expert_bytes(0)
    out = []
    for x in xs:
        experts, _, _, _ = synth.route(L, synth.rms_norm(x))
        out.append(len(experts) * eb + L.router_w.nbytes + 2 * x.nbytes)
    return np.array(out, dtype=np.float64)


def stack_routers(n_layers, E, D, seed=4):
    """C5's per-layer routers: fp32 N(0, 0.02) [E, D], layer l from seed (seed, l)."""
    return [(np.random.default_rng([seed, 11, l]).standard_normal((E, D)) * 0.02).astype(np.float32)
            for l in range(n_layers)]


def stack_bytes(L, n_layers, T, uniq=None):
    """A stack step: every layer reads each distinct selected expert once
    (T = 1 selects top_k distinct experts; for T > 1, uniq = the mean distinct
    experts per layer, read back from the layers' routing), its router and
    x in / out."""
    u = L.top_k if T == 1 else uniq
    return float(n_layers * (u * L.expert_bytes(0) + L.router_w.nbytes + 2 * T * L.embed_dim * 4))


# ---- clocks ------------------------------------------------------------------

class ClockSampler:
    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, device):
        self.device = device
        self.proc = None
        self.lines = []

    def start(self):
        try:
            self.proc = subprocess.Popen(["nvidia-smi", "-i", str(self.device), f"--query-gpu={self.FIELDS}",
                                          "--format=csv,noheader,nounits", "-lms", "100"],
                                         stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
            self.t = threading.Thread(target=self._read, daemon=True)
            self.t.start()
        except OSError:
            self.proc = None

    def _read(self):
        for line in self.proc.stdout:
            self.lines.append(line.strip())

    def stop(self):
        if not self.proc:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["nvidia-smi unavailable"]}
        self.proc.terminate()
        try:
            self.proc.wait(timeout=5)
        except subprocess.TimeoutExpired:
            self.proc.kill()
        self.t.join(timeout=2)
        sm, mx, reasons = [], [], set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for ln in self.lines:
            p = [v.strip() for v in ln.split(",")]
            if len(p) < 9:
                continue
            try:
                sm.append(float(p[1]))
                mx.append(float(p[2]))
            except ValueError:
                continue
            for n, v in zip(names, p[5:9]):
                if v.lower().startswith("active"):
                    reasons.add(n)
        return {"sm_mhz": statistics.median(sm) if sm else None, "sm_max_mhz": max(mx) if mx else None,
                "reasons": sorted(reasons), "samples": len(sm)}


def measured_peak():
    p = ROOT / "MEASURED_PEAKS.json"
    if p.exists():
        d = json.loads(p.read_text())
        return float(d["hbm_gbs"]), "measured (MEASURED_PEAKS.json hbm_gbs)"
    return 6650.0, "fallback 6.65 TB/s"


def traffic_from_profiles():
    p = ROOT / "profiles" / "traffic.json"
    if p.exists():
        try:
            return json.loads(p.read_text())
        except ValueError:
            return None
    return None


# ---- CPU baseline (reference arm / cpu_baseline) ---------------------------

def cpu_reference_run(L, xs, budget_s=12.0, max_steps=None):
    """The reference's CPU path per step: its router + its C MoE call."""
    from oracle import oracle as O
    from tinygiant_b200 import moe, synth
    lib = O.load_reference()
    kind = "reference"
    if lib is None:
        lib, kind = O.load_oracle(), "port"
    cores = os.cpu_count() or 1
    lib.tg_set_threads(cores)
    out = np.zeros_like(xs[0])
    moe.moe_layer_forward(lib, L, synth.rms_norm(xs[0]), out)    # warm
    n, t0 = 0, time.perf_counter()
    while True:
        x = xs[n % len(xs)]
        moe.moe_layer_forward(lib, L, synth.rms_norm(x), out)
        n += 1
        el = time.perf_counter() - t0
        if (max_steps and n >= max_steps) or (not max_steps and el >= budget_s):
            break
    lib.tg_set_threads(1)
    T = xs.shape[1]
    return {"value": n * T / el, "unit": UNIT, "cores": cores, "kind": kind,
            "sample": f"{n} steps x {T} token(s) of the same workload, {el:.1f} s; "
                      f"{'reference csrc/libtinygiant.c built from source (NEON via oracle/neon_shim)' if kind == 'reference' else 'oracle port (tg_oracle.c)'}"
                      f" + numpy router, all {cores} host threads"}, el / n


def run_reference(a):
    rank = int(os.environ.get("RANK", "0"))
    if rank != 0:
        return
    cfg = a.config
    T = a.tokens or 1
    L = make_layer(cfg)
    xs = step_inputs(max(a.warmup, 1) + a.steps, T, L.embed_dim)
    # warm-up steps, untimed
    from oracle import oracle as O
    from tinygiant_b200 import moe, synth
    lib = O.load_reference()
    kind = "reference"
    if lib is None:
        lib, kind = O.load_oracle(), "port"
    cores = os.cpu_count() or 1
    lib.tg_set_threads(cores)
    out = np.zeros_like(xs[0])
    if is_stack(a):
        # the engine's layer loop: x += MoE_l(rmsnorm(x)) for each layer's router
        import copy
        stack = []
        for rw in stack_routers(n_layers(a), L.n_experts, L.embed_dim):
            Ll = copy.copy(L)
            Ll.router_w = rw
            stack.append(Ll)

        def one(x):
            x = x.copy()
            for Ll in stack:
                o = np.zeros_like(x)
                moe.moe_layer_forward(lib, Ll, synth.rms_norm(x), o)
                x += o
            return x
    else:
        def one(x):
            moe.moe_layer_forward(lib, L, synth.rms_norm(x), out)
    for i in range(a.warmup):
        one(xs[i])
    t0 = time.perf_counter()
    for i in range(a.steps):
        one(xs[a.warmup + i])
    el = time.perf_counter() - t0
    value = a.steps * T / el
    line = {"impl": "reference", "metric": METRIC, "value": value, "unit": UNIT, "n_gpus": a.gpus, "steps": a.steps,
            "warmup": a.warmup, "ms_per_step": el / a.steps * 1e3, "higher_is_better": True, "scaling": "strong",
            "vs_baseline": None, "dtype": DTYPES.get(cfg, DTYPES["c2"]), "data": "synthetic",
            "config": {**workload_desc("c4s" if cfg == "c4" and is_stack(a) else cfg, T, 1, L),
                       **({"layers": n_layers(a)} if is_stack(a) else {})},
            "cpu_baseline": {"value": value, "unit": UNIT, "cores": cores, "kind": kind,
                             "sample": f"{a.steps} steps x {T} token(s); numpy router + "
                                       f"{'csrc/libtinygiant.c (reference source, NEON via oracle/neon_shim)' if kind == 'reference' else 'oracle port'}"
                                       f", tg_set_threads({cores})"},
            "e2e": {"value": value, "unit": UNIT, "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}
    print(json.dumps(line), flush=True)


def quiet_nccl():
    """Keep NCCL's banner ("NCCL version ...") off stdout, which carries only the
    JSON line; INFO / TRACE debugging still goes through."""
    if os.environ.get("NCCL_DEBUG", "").upper() not in ("INFO", "TRACE"):
        os.environ["NCCL_DEBUG"] = "WARN"


# ---- our arm ---------------------------------------------------------------

def run_ours(a):
    import torch
    import torch.distributed as dist

    import tinygiant_b200 as tg
    from tinygiant_b200.layer import ResidentLayer

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if world != a.gpus:
        a.gpus = world
    torch.cuda.set_device(local)
    if world > 1:
        from datetime import timedelta
        quiet_nccl()
        dist.init_process_group("nccl", timeout=timedelta(seconds=120), device_id=torch.device("cuda", local))
    lib = tg.load()
    lib.tg_cuda_set_device(local)
    stream = torch.cuda.Stream()
    lib.tg_cuda_set_stream(ctypes.c_void_p(stream.cuda_stream))

    cfg = a.config
    T = a.tokens or 1
    L = make_layer(cfg)
    D = L.embed_dim
    R = max(1, a.copies)
    ep = world > 1 and a.parallel == "ep"
    base = ResidentLayer(L, max_tokens=T, lib=lib, shard=rank if ep else 0, n_shards=world if ep else 1)
    layers = [base] + [base.clone() for _ in range(R - 1)]
    if a.matvec:
        for lay in layers:
            lay.set_tc(False)
    tg.check(lib)
    # expert parallel at decode size: the shards' parts are combined inside
    # the step kernel over NVLink (no all-reduce launch) unless --ep-nccl
    in_kernel = ep and T <= 8 and not a.ep_nccl
    if in_kernel:
        for lay in layers:
            lay.ep_connect()

    S = a.warmup + a.steps
    # data-parallel ranks serve different tokens; expert-parallel ranks the same ones
    xs_host = step_inputs(S, T, D, seed=4 if ep or world == 1 else 4 + 1000 * rank)
    xs = torch.from_numpy(xs_host).to(f"cuda:{local}")
    out = torch.zeros((T, D), dtype=torch.float32, device=f"cuda:{local}")

    def step(i):
        lay = layers[i % R]
        lib.tg_layer_forward_dev(lay.h, xs[i].data_ptr(), None, None, out.data_ptr(), T, 1, None)
        if ep and not in_kernel:
            dist.all_reduce(out)

    # warm-up (also exercises every copy once)
    with torch.cuda.stream(stream):
        for i in range(a.warmup):
            step(i)
    torch.cuda.synchronize()
    tg.check(lib)

    # capture the K timed steps in one graph
    g = torch.cuda.CUDAGraph()
    launches0 = lib.tg_cuda_launch_count()
    with torch.cuda.graph(g, stream=stream):
        for i in range(a.warmup, S):
            step(i)
    launches = lib.tg_cuda_launch_count() - launches0
    tg.check(lib)
    # one untimed replay so the graph's first-launch cost is not timed
    g.replay()
    torch.cuda.synchronize()

    # Clocks are sampled over a ~1.5 s soak of untimed replays of the same
    # graph and the timed replay that follows it (the timed region alone is
    # shorter than nvidia-smi's sampling period).
    clocks = ClockSampler(local)
    clocks.start()
    t_soak = time.perf_counter()
    with torch.cuda.stream(stream):
        while time.perf_counter() - t_soak < 1.5:
            g.replay()
            torch.cuda.synchronize()
    ev0, ev1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    if world > 1:
        dist.barrier()
    torch.cuda.synchronize()
    with torch.cuda.stream(stream):
        ev0.record(stream)
        g.replay()
        ev1.record(stream)
    torch.cuda.synchronize()
    ms = ev0.elapsed_time(ev1)
    if world > 1:
        t = torch.tensor([ms], device=f"cuda:{local}")
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        ms = float(t.item())
    clk = clocks.stop()
    tg.check(lib)

    ms_step = ms / a.steps
    ranks_tokens = 1 if ep else world   # data-parallel ranks each process their own tokens
    value = ranks_tokens * a.steps * T / (ms / 1e3)
    line = None
    if rank == 0:
        nbytes = algorithmic_bytes(L, xs_host[a.warmup:])
        achieved = ranks_tokens * nbytes.sum() / (ms / 1e3) / 1e9
        peak, peak_src = measured_peak()
        peak *= world            # whole-job bytes against every GPU's HBM
        tr = traffic_from_profiles()
        roof = {"bound": "hbm", "achieved": achieved, "peak": peak, "unit": "GB/s", "frac": achieved / peak,
                "traffic": (tr or {}).get(cfg),
                "kernel": "fused MoE layer step (router + gate/up + down kernels), per step",
                "algorithmic_bytes_per_step": float(nbytes.mean()), "peak_source": peak_src}
        line = {"metric": METRIC, "value": value, "unit": UNIT, "n_gpus": world, "steps": a.steps,
                "warmup": a.warmup, "ms_per_step": ms_step, "higher_is_better": True,
                "scaling": "strong" if ep or world == 1 else "weak",
                "vs_baseline": None, "dtype": DTYPES.get(cfg, DTYPES["c2"]),
                "data": "synthetic (seeded weights and inputs)",
                "config": {**workload_desc(cfg, T, R, L), "parallelism": f"ep{world}" if ep else f"dp{world}",
                           "expert_path": "fused step kernel" if T <= 8 else
                                          ("matvec kernels" if a.matvec else "tcgen05 grouped GEMMs"),
                           **({"ep_combine": "in the step kernel over NVLink" if in_kernel else "NCCL all-reduce"}
                              if ep else {})},
                "gbps": achieved, "clocks": clk, "roofline": roof, "gpu_launches": int(launches)}

    # e2e: one GPU through the C-ABI entry tg_layer_forward with host buffers
    # (synchronous, x in / MoE output out every step); several GPUs through
    # tg_layer_forward_dev with each step's x copied from pinned host memory
    # and its output read back, plus the all-reduce for ep; max over ranks.
    e2e = None
    if world == 1:
        xh = [np.ascontiguousarray(x) for x in xs_host]
        outh = np.zeros((T, D), np.float32)
        for i in range(min(a.warmup, S)):
            layers[i % R].forward(xh[i], outh)
        t0 = time.perf_counter()
        for i in range(a.warmup, S):
            lib.tg_layer_forward(layers[i % R].h, xh[i].ctypes.data, outh.ctypes.data, T, 1)
        el = time.perf_counter() - t0
        tg.check(lib)
        e2e = {"value": a.steps * T / el, "unit": UNIT, "h2d_bytes_per_step": int(xh[0].nbytes),
               "d2h_bytes_per_step": int(outh.nbytes), "api": "tg_layer_forward (C ABI, host buffers)",
               "ms_per_step": el / a.steps * 1e3}
    else:
        xpin = torch.from_numpy(xs_host).pin_memory()
        opin = torch.zeros((T, D), dtype=torch.float32).pin_memory()
        xd = torch.empty((T, D), dtype=torch.float32, device=f"cuda:{local}")

        def e2e_step(i):
            with torch.cuda.stream(stream):
                xd.copy_(xpin[i], non_blocking=True)
                lib.tg_layer_forward_dev(layers[i % R].h, xd.data_ptr(), None, None, out.data_ptr(), T, 1, None)
                if ep and not in_kernel:
                    dist.all_reduce(out)
                opin.copy_(out, non_blocking=True)
            stream.synchronize()

        for i in range(min(a.warmup, S)):
            e2e_step(i)
        dist.barrier()
        t0 = time.perf_counter()
        for i in range(a.warmup, S):
            e2e_step(i)
        el = time.perf_counter() - t0
        t = torch.tensor([el], device=f"cuda:{local}")
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        el = float(t.item())
        tg.check(lib)
        e2e = {"value": ranks_tokens * a.steps * T / el, "unit": UNIT, "h2d_bytes_per_step": int(xs_host[0].nbytes),
               "d2h_bytes_per_step": int(opin.numel() * 4),
               "api": "tg_layer_forward_dev per rank, pinned host copies" +
                      (" + NCCL all-reduce" if ep and not in_kernel else " (shards combined in the step kernel)" if ep else ""),
               "ms_per_step": el / a.steps * 1e3}
    if rank == 0:
        line["e2e"] = e2e
        if world == 1 and not a.no_cpu_baseline:
            cb, _ = cpu_reference_run(L, xs_host[a.warmup:], budget_s=12.0)
            line["cpu_baseline"] = cb
        print(json.dumps(line), flush=True)
    del g
    for lay in layers:
        lay.close()
    if world > 1:
        dist.destroy_process_group()


def is_stack(a):
    return a.config == "c5" or (a.config == "c4" and n_layers(a) > 1)


def n_layers(a):
    return a.layers if a.layers is not None else {"c4": 36, "c5": 48}.get(a.config, 1)


def run_stack(a):
    """C4 / C5: T tokens through an n-layer stack (x += MoE(rmsnorm(x)) per
    layer) per step."""
    import torch
    import torch.distributed as dist

    import tinygiant_b200 as tg
    from tinygiant_b200 import synth
    from tinygiant_b200.layer import ResidentLayer

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    a.gpus = world
    torch.cuda.set_device(local)
    if world > 1:
        from datetime import timedelta
        quiet_nccl()
        dist.init_process_group("nccl", timeout=timedelta(seconds=120), device_id=torch.device("cuda", local))
    lib = tg.load()
    lib.tg_cuda_set_device(local)
    stream = torch.cuda.Stream()
    lib.tg_cuda_set_stream(ctypes.c_void_p(stream.cuda_stream))
    cfg = a.config
    T, NL = a.tokens or 1, n_layers(a)
    ep = world > 1 and a.parallel == "ep"
    L = make_layer(cfg)
    D = L.embed_dim
    base = ResidentLayer(L, max_tokens=T, lib=lib, shard=rank if ep else 0, n_shards=world if ep else 1)
    layers = [base] + [base.clone() for _ in range(NL - 1)]
    for lay, rw in zip(layers, stack_routers(NL, L.n_experts, D)):
        lay.set_router(rw)
    if a.matvec:
        for lay in layers:
            lay.set_tc(False)
    tg.check(lib)
    # expert parallel at decode size: every layer's shards are combined inside
    # its step kernel over NVLink, so the stack runs as on one GPU
    in_kernel = ep and T <= 8 and not a.ep_nccl
    if in_kernel:
        for lay in layers:
            lay.ep_connect()
    handles = (ctypes.c_void_p * NL)(*[lay.h for lay in layers])
    S = a.warmup + a.steps
    xs_host = step_inputs(S, T, D, seed=4 if ep or world == 1 else 4 + 1000 * rank)
    xs = torch.from_numpy(xs_host).to(f"cuda:{local}")
    xb = [torch.zeros((T, D), dtype=torch.float32, device=f"cuda:{local}") for _ in range(4)]

    def step(i):
        if not ep or in_kernel:
            xb[0].copy_(xs[i])
            lib.tg_stack_forward_dev(handles, NL, xb[0].data_ptr(), T, None)
            return
        # expert parallel: each layer's MoE parts are summed before the next layer reads them
        x, xn, m0, m1 = xb
        x.copy_(xs[i])
        for l, lay in enumerate(layers):
            lib.tg_layer_forward_dev(lay.h, x.data_ptr(), m0.data_ptr() if l else None,
                                     xn.data_ptr() if l else None, m1.data_ptr(), T, 1, None)
            dist.all_reduce(m1)
            if l:
                x, xn = xn, x
            m0, m1 = m1, m0
        x.add_(m0)
        if x.data_ptr() != xb[0].data_ptr():
            xb[0].copy_(x)

    with torch.cuda.stream(stream):
        for i in range(a.warmup):
            step(i)
    torch.cuda.synchronize()
    tg.check(lib)
    g = torch.cuda.CUDAGraph()
    launches0 = lib.tg_cuda_launch_count()
    with torch.cuda.graph(g, stream=stream):
        for i in range(a.warmup, S):
            step(i)
    launches = lib.tg_cuda_launch_count() - launches0
    tg.check(lib)
    g.replay()
    torch.cuda.synchronize()
    clocks = ClockSampler(local)
    clocks.start()
    t_soak = time.perf_counter()
    with torch.cuda.stream(stream):
        while time.perf_counter() - t_soak < 1.5:
            g.replay()
            torch.cuda.synchronize()
    ev0, ev1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    if world > 1:
        dist.barrier()
    torch.cuda.synchronize()
    with torch.cuda.stream(stream):
        ev0.record(stream)
        g.replay()
        ev1.record(stream)
    torch.cuda.synchronize()
    ms = ev0.elapsed_time(ev1)
    if world > 1:
        t = torch.tensor([ms], device=f"cuda:{local}")
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        ms = float(t.item())
    clk = clocks.stop()
    tg.check(lib)
    ranks_tokens = 1 if ep else world
    value = ranks_tokens * a.steps * T / (ms / 1e3)

    # e2e: x from pinned host memory, the stack, x back, every step (one GPU,
    # or every rank for data parallel; max over ranks)
    xpin = torch.from_numpy(xs_host).pin_memory()
    opin = torch.zeros((T, D), dtype=torch.float32).pin_memory()

    def e2e_step(i):
        with torch.cuda.stream(stream):
            xs[i].copy_(xpin[i], non_blocking=True)
            step(i)
            opin.copy_(xb[0], non_blocking=True)
        stream.synchronize()

    for i in range(min(a.warmup, S)):
        e2e_step(i)
    if world > 1:
        dist.barrier()
    t0 = time.perf_counter()
    for i in range(a.warmup, S):
        e2e_step(i)
    el = time.perf_counter() - t0
    if world > 1:
        t = torch.tensor([el], device=f"cuda:{local}")
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        el = float(t.item())
    tg.check(lib)
    # distinct experts per layer (T > 1): from every layer's routing of the last step
    uniq = None
    if T > 1:
        per = []
        for lay in layers:
            idx, w = lay.last_routing(T)
            per.append(len({int(e) for e, ww in zip(idx.ravel(), w.ravel()) if ww != 0}))
        uniq = float(np.mean(per))
    if rank == 0:
        nbytes = stack_bytes(L, NL, T, uniq)
        achieved = ranks_tokens * a.steps * nbytes / (ms / 1e3) / 1e9
        peak, peak_src = measured_peak()
        peak *= world
        roof = {"bound": "hbm", "achieved": achieved, "peak": peak, "unit": "GB/s", "frac": achieved / peak,
                "traffic": None, "kernel": f"fused MoE layer step x {NL} layers per token",
                "algorithmic_bytes_per_step": nbytes, "peak_source": peak_src}
        desc = workload_desc("c4s" if cfg == "c4" else "c5", T, 1, L)
        desc.update({"layers": NL, "l2": f"inputs larger than L2: {NL} distinct layers resident "
                                       f"({NL * L.n_experts * L.expert_bytes(0) / 1e9 / (world if ep else 1):.1f} GB "
                                       f"of experts per GPU)",
                     "step": f"{T} token(s) through the stack: per layer rmsnorm + router + top-k + experts + "
                             f"residual add",
                     "expert_path": "fused step kernel" if T <= 8 else
                                    ("matvec kernels" if a.matvec else "tcgen05 grouped GEMMs"),
                     **({"distinct_experts_per_layer": uniq} if uniq is not None else {}),
                     **({"ep_combine": "in the step kernel over NVLink" if in_kernel else "NCCL all-reduce"}
                        if ep else {})})
        line = {"metric": METRIC, "value": value, "unit": UNIT, "n_gpus": world, "steps": a.steps,
                "warmup": a.warmup, "ms_per_step": ms / a.steps, "higher_is_better": True,
                "scaling": "strong" if ep or world == 1 else "weak", "vs_baseline": None,
                "dtype": DTYPES[cfg], "data": "synthetic (seeded weights and inputs)",
                "config": {**desc, "parallelism": f"ep{world}" if ep else f"dp{world}"},
                "gbps": achieved, "clocks": clk, "roofline": roof, "gpu_launches": int(launches),
                "e2e": {"value": ranks_tokens * a.steps * T / el, "unit": UNIT,
                        "h2d_bytes_per_step": int(T * D * 4), "d2h_bytes_per_step": int(T * D * 4),
                        "api": "tg_stack_forward_dev with pinned host copies" if not ep or in_kernel else
                               "tg_layer_forward_dev per layer + NCCL all-reduce, pinned host copies",
                        "ms_per_step": el / a.steps * 1e3}}
        print(json.dumps(line), flush=True)
    del g
    for lay in layers:
        lay.close()
    if world > 1:
        dist.destroy_process_group()


# ---- around the path: attention decode and expert-cache loading ----------------

def run_attn(a):
    """One Qwen3-30B-A3B-shaped attention decode step (D 2048, 32 query / 4 KV
    heads of 128, Q4_K q/k/o, Q6_K v, QK norm) per token through the C-ABI
    tg_attention_v2 with host buffers, the context starting at --tokens
    positions (default 1024) and growing by one per call; beside it the
    reference's own C (oracle/_ref) on the same inputs, all host threads."""
    import torch  # noqa: F401  (CUDA context first)

    import tinygiant_b200 as tg
    from oracle import oracle as O
    from tinygiant_b200 import quants as Q
    from tinygiant_b200._lib import ABI

    if int(os.environ.get("RANK", "0")) != 0:
        return
    D, H, KH, HD, KV_MAX = 2048, 32, 4, 128, 4096
    L0 = a.tokens or 1024
    rng = np.random.default_rng([9, 1])
    mats = {"q": (Q.FMT_Q4K, H * HD, D), "k": (Q.FMT_Q4K, KH * HD, D), "v": (Q.FMT_Q6K, KH * HD, D),
            "o": (Q.FMT_Q4K, D, H * HD)}
    W = {}
    for k, (f, r, c) in mats.items():
        w = (rng.standard_normal((r, c)) * 0.02).astype(np.float32)
        W[k] = Q.pack_q4k(w) if f == Q.FMT_Q4K else Q.pack_q6k(w)
    qn, kn = [(1.0 + 0.1 * rng.standard_normal(HD)).astype(np.float32) for _ in range(2)]
    half = HD // 2
    ang = np.arange(KV_MAX)[:, None] * (1.0 / (1e6 ** (np.arange(half) * 2.0 / HD)))[None, :]
    cos, sin = np.cos(ang).astype(np.float32), np.sin(ang).astype(np.float32)
    kv0 = [(rng.standard_normal((KH, KV_MAX, HD)) * 0.5).astype(np.float32) for _ in range(2)]
    n_calls = a.warmup + a.steps
    xs = rng.standard_normal((n_calls, D)).astype(np.float32)

    def p(x):
        return None if x is None else x.ctypes.data

    def call(lib, kv, pos, x, out):
        lib.tg_attention_v2(mats["q"][0], mats["k"][0], mats["v"][0], mats["o"][0], p(W["q"]), p(W["k"]), p(W["v"]),
                            p(W["o"]), None, None, None, None, p(qn), p(kn), None, p(kv[0]), p(kv[1]), pos, KV_MAX, 0,
                            p(cos), p(sin), p(x), p(out), D, H, KH, HD, pos, 1e-6)

    lib = tg.load()
    ours_kv = [k.copy() for k in kv0]
    out = np.zeros(D, np.float32)
    for i in range(a.warmup):
        call(lib, ours_kv, L0 + i, xs[i], out)
    tg.check(lib)
    t0 = time.perf_counter()
    for i in range(a.warmup, n_calls):
        call(lib, ours_kv, L0 + i, xs[i], out)
    el = time.perf_counter() - t0
    tg.check(lib)
    ours_last = out.copy()

    # the reference's C on the same sequence (a bounded sample), and the
    # parity of the last step
    ref = ctypes.CDLL(str(O.REF_SO)) if O.REF_SO.exists() else None
    cpu = None
    err = None
    if ref is not None:
        ref.tg_attention_v2.argtypes, ref.tg_attention_v2.restype = ABI["tg_attention_v2"]
        ref.tg_set_threads.argtypes = [ctypes.c_int]
        cores = os.cpu_count() or 1
        ref.tg_set_threads(cores)
        ref_kv = [k.copy() for k in kv0]
        rout = np.zeros(D, np.float32)
        n, t1 = 0, time.perf_counter()
        for i in range(n_calls):
            call(ref, ref_kv, L0 + i, xs[i], rout)
            n += 1
            if i >= a.warmup and time.perf_counter() - t1 > 20.0:
                break
        rel = time.perf_counter() - t1
        if n == n_calls:
            err = float(np.max(np.abs(ours_last - rout)) / max(float(np.max(np.abs(rout))), 1e-30))
        cpu = {"value": n / rel, "unit": "tok/s", "cores": cores, "kind": "reference",
               "sample": f"{n} steps from context {L0}; csrc/libtinygiant.c tg_attention_v2 (NEON via oracle/neon_shim)"}
    wbytes = sum(w.nbytes for w in W.values())
    kvb = lambda pos: 2 * KH * (pos + 1) * HD * 4
    nbytes = float(np.mean([wbytes + kvb(L0 + i) for i in range(a.warmup, n_calls)]))
    ms = el / a.steps * 1e3
    peak, peak_src = measured_peak()
    achieved = nbytes / (ms / 1e3) / 1e9
    line = {"metric": "attention decode step tok/s (one layer)", "value": a.steps / el, "unit": "tok/s",
            "n_gpus": 1, "steps": a.steps, "warmup": a.warmup, "ms_per_step": ms, "higher_is_better": True,
            "scaling": "strong", "vs_baseline": None, "dtype": "int8xQ4_K/Q6_K projections, fp32 attention",
            "data": "synthetic (seeded weights, KV cache and inputs)",
            "config": {"workload": "Qwen3-30B-A3B attention decode: D 2048, 32 q / 4 kv heads x 128, Q4_K q/k/o, "
                                   "Q6_K v, QK norm, RoPE", "context_start": L0, "kv_max": KV_MAX,
                       "api": "tg_attention_v2 (C ABI, host buffers; the KV cache is the caller's host array, "
                              "mirrored in HBM)"},
            "roofline": {"bound": "hbm", "achieved": achieved, "peak": peak, "unit": "GB/s", "frac": achieved / peak,
                         "traffic": None, "algorithmic_bytes_per_step": nbytes, "peak_source": peak_src},
            "e2e": {"value": a.steps / el, "unit": "tok/s", "h2d_bytes_per_step": int(D * 4 + HD * 4),
                    "d2h_bytes_per_step": int(D * 4 + 2 * KH * HD * 4), "ms_per_step": ms},
            "cpu_baseline": cpu, "parity_last_step_rel_err": err}
    print(json.dumps(line), flush=True)


def run_cache(a):
    """--layers C2-shaped layers (default 2) written as an expert-cache
    directory (the relayout format), then mapped and made resident in HBM:
    GB/s of expert bytes from the (warm) page cache into HBM, and the first
    layer's output checked against the same layer built in memory."""
    import tempfile

    import torch  # noqa: F401

    import tinygiant_b200 as tg
    from tinygiant_b200 import expert_cache, synth
    from tinygiant_b200.layer import ResidentLayer

    if int(os.environ.get("RANK", "0")) != 0:
        return
    n = a.layers or 2
    lib = tg.load()
    layers = [synth.qwen_layer(seed=1, layer=l) for l in range(n)]
    with tempfile.TemporaryDirectory() as d:
        expert_cache.write_cache(d, layers)
        t0 = time.perf_counter()
        got = expert_cache.stack_from_cache(d, [L.router_w for L in layers])
        res = [ResidentLayer(G, max_tokens=1, lib=lib) for G in got]
        lib.tg_cuda_synchronize()
        el = time.perf_counter() - t0
        tg.check(lib)
        nbytes = float(sum(G.n_experts * G.expert_bytes(0) for G in got))
        x = np.random.default_rng(3).standard_normal((1, layers[0].embed_dim)).astype(np.float32)
        mem = ResidentLayer(layers[0], max_tokens=1, lib=lib)
        same = bool(np.array_equal(res[0].forward(x).view(np.uint32), mem.forward(x).view(np.uint32)))
        for r in res + [mem]:
            r.close()
    line = {"metric": "expert-cache load into HBM GB/s", "value": nbytes / el / 1e9, "unit": "GB/s", "n_gpus": 1,
            "steps": 1, "warmup": 0, "ms_per_step": el * 1e3, "higher_is_better": True, "scaling": "strong",
            "vs_baseline": None, "dtype": "raw GGUF blocks (Q4_K, Q6_K)", "data": "synthetic C2 layers written as "
            "layer_NNN.q4.bin + index.json in a temporary directory (warm page cache)",
            "config": {"workload": f"{n} Qwen3-30B-A3B MoE layers, 128 experts each", "bytes": nbytes,
                       "api": "tinygiant_b200.expert_cache.stack_from_cache + ResidentLayer"},
            "first_layer_bit_identical": same}
    print(json.dumps(line), flush=True)


def main():
    a = parse()
    if a.config == "attn":
        run_attn(a)
        return
    if a.config == "cache":
        run_cache(a)
        return
    if a.impl == "reference":
        run_reference(a)
    elif is_stack(a):
        run_stack(a)
    else:
        run_ours(a)


if __name__ == "__main__":
    main()
