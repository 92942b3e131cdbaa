"""Benchmark: MoE-layer decode tok/s and fused quant-matvec HBM GB/s on B200.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]
                    [--config c1|c2|c3|c4|c5|attn|cache|trace] [--tokens T] [--layers L]

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
buffers (x in, MoE output back), host<->device copies inside the timed
region.  e2e_engine: the reference engine's own call sequence per step —
numpy RMSNorm + router + top-k + union (engine.py:281-318) and
tg_moe_forward_rows_v2 with host pointers (engine.py:323-341).

Multi-GPU (torchrun): --parallel ep (the default for N > 1) shards the experts
by id (e % N == rank) with the router replicated; decode-sized steps sum the
shards' parts inside the step kernel over NVLink (--ep-nccl: one NCCL
all-reduce instead); total work is fixed ("strong").  --parallel dp: every
GPU holds the whole layer and serves its own tokens ("weak").

C1 (--config c1): one all-Q4_K expert (tg_expert_forward) over 64 copies
(170 MB); the device-timed step is that expert as a one-expert resident layer
without normalisation (weight 1), e2e is tg_expert_forward with host buffers.

--impl reference: the reference's own CPU path on the host cores — its router
(restated in synth.route, checked against tinygiant/router.py) + its
csrc/libtinygiant.c tg_moe_forward_rows_v2 (oracle/_ref, compiled from the
reference's source) with every host thread, over the same R copies of the
layer in host memory.
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
C1_COPIES = 64      # C1: 64 x 2.65 MB = 170 MB of experts, beyond the 126 MB L2
DTYPES = {"c1": "int8xQ4_K (int32 accumulate), fp32 combine",
          "c2": "int8xQ4_K/Q6_K (int32 accumulate), fp32 combine",
          "c3": "int8xQ4_K/Q6_K (int32 accumulate), fp32 combine",
          "c4": "int8xMXFP4 (int32 accumulate), fp32 combine",
          "c5": "int8xQ4_K/Q6_K (int32 accumulate), fp32 combine"}


def parse():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=2000)
    ap.add_argument("--warmup", type=int, default=10)
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--config", default="c2", choices=["c1", "c2", "c3", "c4", "c5", "attn", "cache", "trace"],
                    help="c1-c5: the MoE workloads; attn: one attention decode step (tg_attention_v2); "
                         "cache: an expert-cache directory loaded into HBM; trace: the fused step's phase "
                         "timeline (diagnostics, no bench line)")
    ap.add_argument("--tokens", type=int, default=None)
    ap.add_argument("--copies", type=int, default=R_COPIES)
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--parallel", default=None, choices=["dp", "ep"],
                    help="with several GPUs: ep (default) shards the experts by id, dp runs replicas")
    ap.add_argument("--gptoss", action="store_true", help="--config trace: the C4 layer instead of C2")
    ap.add_argument("--experts", type=int, default=None, help="--config trace: experts in the layer")
    ap.add_argument("--layers", type=int, default=None,
                    help="C4 / C5: layers in the stack (default 36 / 48; C4 with 1: one layer over HBM copies)")
    ap.add_argument("--matvec", action="store_true",
                    help="batched steps (T > 8) on the matvec kernels instead of the tcgen05 grouped GEMMs")
    ap.add_argument("--ep-nccl", action="store_true",
                    help="expert parallel: sum the shards with an NCCL all-reduce instead of inside the step kernel")
    a = ap.parse_args()
    if a.parallel is None:
        a.parallel = "ep" if int(os.environ.get("WORLD_SIZE", "1")) > 1 else "dp"
    return a


# ---- workload ------------------------------------------------------------

def make_layer(cfg):
    from tinygiant_b200 import synth
    if cfg == "c4":
        return synth.gptoss_layer(seed=3)
    if cfg == "c3":
        return synth.qwen_layer(seed=2, router_bias=synth.zipf_bias(seed=2))
    return synth.qwen_layer(seed=1)


def host_copies(L, R):
    """R copies of layer L whose expert byte arrays are distinct host arrays
    (the router is shared): the CPU arms cycle them as the GPU arm cycles its
    R HBM copies."""
    import copy
    out = [L]
    for _ in range(R - 1):
        c = copy.copy(L)
        c.gates = [g.copy() for g in L.gates]
        c.ups = [u.copy() for u in L.ups]
        c.downs = [d.copy() for d in L.downs]
        out.append(c)
    return out


def workload_desc(cfg, T, R, L):
    """The `config` of a bench line; both arms report the same one."""
    names = {
        "c1": "C1: one Qwen3-30B-A3B-shaped expert SwiGLU FFN (all Q4_K: gate/up 768x2048, down 2048x768), "
              "tg_expert_forward, weight 1",
        "c2": "C2: one Qwen3-30B-A3B MoE layer (128 experts, Q4_K gate/up, Q6_K down, top-8, D=2048, I=768)",
        "c3": "C3: Qwen3-30B-A3B MoE layer with Zipf(1.1)-skewed router bias",
        "c4": "C4: gpt-oss-120b-shaped MXFP4 MoE layer (128 experts, top-4, D=I=2880)",
        "c4s": "C4: gpt-oss-120b-shaped MXFP4 MoE stack (128 experts per layer, top-4, D=I=2880, per-layer routers, "
               "residual add)",
        "c5": "C5: Qwen3-30B-A3B MoE-FFN stack (C2 experts per layer, per-layer routers, residual add)",
    }
    if cfg == "c1":
        return {"workload": names[cfg], "tokens_per_step": 1, "embed_dim": 2048, "inter_dim": 768,
                "expert_copies": R,
                "l2": f"inputs larger than L2: steps cycle {R} copies of the expert ({R * 2.654208:.0f} MB; "
                      f"HBM on the GPU arm, host memory on the reference arm)",
                "step": "one expert: gate/up, SiLU, down, out += 1.0 * y"}
    return {"workload": names[cfg], "tokens_per_step": T, "experts": L.n_experts, "top_k": L.top_k,
            "embed_dim": L.embed_dim, "inter_dim": L.inter_dim, "layer_copies": R,
            "l2": f"inputs larger than L2: steps cycle {R} copies of the layer (HBM on the GPU arm, host memory "
                  f"on the reference arm)",
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


def measured_int8_peak():
    """Dense int8 tensor ops/s: twice the measured bf16 GEMM rate (the
    nominal int8 : bf16 dense ratio of B200, 4.5 : 2.25 POPS), burst figure."""
    p = ROOT / "MEASURED_PEAKS.json"
    if p.exists():
        d = json.loads(p.read_text())
        return 2.0 * float(d["bf16_tflops"]), "2 x measured bf16 cuBLAS (MEASURED_PEAKS.json bf16_tflops)"
    return 2.0 * 1590.0, "2 x fallback 1.59 PFLOP/s bf16"


def batched_ops(L, xs):
    """Per step: int8 multiply-adds x 2 of the active (expert, token) rows'
    gate, up and down dots (3 D I each), from the reference routing."""
    from tinygiant_b200 import synth
    out = []
    for x in xs:
        _, row_w, _, _ = synth.route(L, synth.rms_norm(x))
        out.append(2.0 * float(np.count_nonzero(row_w)) * 3 * L.embed_dim * L.inter_dim)
    return np.array(out)


def traffic_from_profiles():
    p = ROOT / "profiles" / "traffic.json"
    if p.exists():
        try:
            return json.loads(p.read_text())
        except ValueError:
            return None
    return None


# ---- CPU baseline (reference arm / cpu_baseline) ---------------------------

def reference_lib():
    """The reference's own C (oracle/_ref, kind "reference"), else the oracle
    port (kind "port")."""
    from oracle import oracle as O
    lib = O.load_reference()
    if lib is None:
        return O.load_oracle(), "port"
    return lib, "reference"


def ref_source(kind):
    return ("csrc/libtinygiant.c built from the reference source (NEON via oracle/neon_shim)"
            if kind == "reference" else "oracle port (oracle/tg_oracle.c)")


def cpu_step(cfg, lib, copies, routers=None):
    """One step of the reference's CPU path, as fn(i, x) -> output: C1 its
    tg_expert_forward on copy i % R; a layer its router (synth.route, the
    engine's numpy sequence) + tg_moe_forward_rows_v2 on layer copy i % R; a
    stack (routers given) x += MoE_l(rmsnorm(x)) for each layer's router."""
    import copy
    from tinygiant_b200 import moe, synth
    R = len(copies)
    if cfg == "c1":
        out = np.zeros(2048, np.float32)

        def one(i, x):
            out[:] = 0.0
            lib.tg_expert_forward(copies[i % R].ctypes.data, x.ctypes.data, out.ctypes.data, 1.0, 2048, 768)
            return out
        return one
    if routers is not None:
        stack = []
        for rw in routers:
            Ll = copy.copy(copies[0])
            Ll.router_w = rw
            stack.append(Ll)

        def one(i, x):
            x = x.copy()
            for Ll in stack:
                o = np.zeros_like(x)
                moe.moe_layer_forward(lib, Ll, synth.rms_norm(x), o)
                x += o
            return x
        return one

    def one(i, x):
        out = np.zeros_like(x)
        return moe.moe_layer_forward(lib, copies[i % R], synth.rms_norm(x), out)
    return one


def cpu_reference_run(cfg, copies, xs, budget_s=12.0, routers=None):
    """The cpu_baseline leg: the reference's CPU path on the same workload,
    all host threads, for about budget_s seconds of steps."""
    lib, kind = reference_lib()
    cores = os.cpu_count() or 1
    lib.tg_set_threads(cores)
    one = cpu_step(cfg, lib, copies, routers)
    one(0, xs[0])    # warm
    n, t0 = 0, time.perf_counter()
    while True:
        one(n, xs[n % len(xs)])
        n += 1
        el = time.perf_counter() - t0
        if el >= budget_s:
            break
    lib.tg_set_threads(1)
    T = 1 if cfg == "c1" else xs.shape[1]
    return {"value": n * T / el, "unit": UNIT, "cores": cores, "kind": kind,
            "sample": f"{n} steps x {T} token(s) of the same workload, {el:.1f} s; {ref_source(kind)}"
                      f"{'' if cfg == 'c1' else ' + numpy router'}, all {cores} host threads"}


def run_reference(a):
    """--impl reference: the reference's CPU path on this arm's config,
    metric and unit; rank 0 only."""
    rank = int(os.environ.get("RANK", "0"))
    if rank != 0:
        return
    cfg = a.config
    T = 1 if cfg == "c1" else (a.tokens or 1)
    from tinygiant_b200 import synth
    stack = is_stack(a)
    if cfg == "c1":
        R = max(1, a.copies if a.copies != R_COPIES else C1_COPIES)
        e0 = synth.c1_expert(seed=0)
        copies = [e0] + [e0.copy() for _ in range(R - 1)]
        xs = step_inputs(max(a.warmup, 1) + a.steps, 1, 2048)[:, 0]
        desc = workload_desc("c1", 1, R, None)
        routers = None
    else:
        L = make_layer(cfg)
        R = 1 if stack else max(1, a.copies)
        copies = host_copies(L, R)
        xs = step_inputs(max(a.warmup, 1) + a.steps, T, L.embed_dim)
        routers = stack_routers(n_layers(a), L.n_experts, L.embed_dim) if stack else None
        desc = stack_desc(cfg, T, n_layers(a), L) if stack else workload_desc(cfg, T, R, L)
    lib, kind = reference_lib()
    cores = os.cpu_count() or 1
    lib.tg_set_threads(cores)
    one = cpu_step(cfg, lib, copies, routers)
    for i in range(a.warmup):
        one(i, xs[i])
    t0 = time.perf_counter()
    for i in range(a.steps):
        one(a.warmup + i, xs[a.warmup + i])
    el = time.perf_counter() - t0
    value = a.steps * T / el
    line = {"impl": "reference", "metric": METRIC, "value": value, "unit": UNIT, "n_gpus": a.gpus, "steps": a.steps,
            "warmup": a.warmup, "ms_per_step": el / a.steps * 1e3, "higher_is_better": True,
            "scaling": scaling_of(a, cfg), "vs_baseline": None, "dtype": DTYPES.get(cfg, DTYPES["c2"]),
            "data": "synthetic (seeded weights and inputs)", "config": desc,
            "cpu_baseline": {"value": value, "unit": UNIT, "cores": cores, "kind": kind,
                             "sample": f"{a.steps} steps x {T} token(s) of this workload; {ref_source(kind)}"
                                       f"{'' if cfg == 'c1' else ' + numpy router'}, tg_set_threads({cores})"},
            "e2e": {"value": value, "unit": UNIT, "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}
    print(json.dumps(line), flush=True)


def scaling_of(a, cfg):
    """"strong" when the job's total work is fixed as GPUs are added (one GPU,
    or experts sharded), "weak" for data-parallel replicas."""
    world = int(os.environ.get("WORLD_SIZE", "1"))
    return "weak" if world > 1 and a.parallel == "dp" else "strong"


def quiet_nccl():
    """Keep NCCL's banner ("NCCL version ...") off stdout, which carries only the
    JSON line; INFO / TRACE debugging still goes through."""
    if os.environ.get("NCCL_DEBUG", "").upper() not in ("INFO", "TRACE"):
        os.environ["NCCL_DEBUG"] = "WARN"


# ---- our arm ---------------------------------------------------------------

def setup_gpu(a):
    """Per-rank set-up: device, process group (N > 1), library and its stream."""
    import torch
    import torch.distributed as dist

    import tinygiant_b200 as tg
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
    return world, rank, local, lib, stream


def time_graph(lib, step, first, last, stream, world, local):
    """Captures steps first .. last-1 in one CUDA graph, replays it once
    untimed, soaks ~1.5 s of replays while nvidia-smi samples the clocks, then
    times one replay with CUDA events on the library's stream (barrier +
    synchronize on both sides; the max over ranks).  Returns (ms, our kernel
    launches in the graph, clocks, graph)."""
    import torch
    import torch.distributed as dist

    import tinygiant_b200 as tg
    g = torch.cuda.CUDAGraph()
    launches0 = lib.tg_cuda_launch_count()
    with torch.cuda.graph(g, stream=stream):
        for i in range(first, last):
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
    return ms, int(launches), clk, g


def max_over_ranks(v, world, local):
    if world == 1:
        return v
    import torch
    import torch.distributed as dist
    t = torch.tensor([v], device=f"cuda:{local}", dtype=torch.float64)
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t.item())


def ep_balance(L, xs, world):
    """Expert parallel (e % world == rank): per step the largest number of
    distinct selected experts that one GPU holds, averaged over the steps."""
    from tinygiant_b200 import synth
    per = []
    for x in xs:
        experts, _, _, _ = synth.route(L, synth.rms_norm(x))
        counts = np.bincount(np.asarray(experts) % world, minlength=world)
        per.append(int(counts.max()))
    return float(np.mean(per)), int(max(per))


def engine_e2e(lib, L, xs, R, warm):
    """The reference engine's own call sequence per step on one GPU: numpy
    RMSNorm + router + top-k + expert union and row weights (synth.route,
    engine.py:281-318), then tg_moe_forward_rows_v2 with host pointers and a
    zero-filled host output (engine.py:323-341).  The R host copies of the
    layer are registered as immutable (tg_cuda_register, as an integration
    does for its mapped expert files) and uploaded by one warm call each."""
    import tinygiant_b200 as tg
    from tinygiant_b200 import moe, synth
    copies = host_copies(L, R)
    for c in copies:
        for arr in c.gates + c.ups + c.downs:
            if lib.tg_cuda_register(arr.ctypes.data, arr.nbytes) != 0:
                tg.check(lib)
        allw = np.ones((c.n_experts, 1), np.float32)
        o = np.zeros((1, c.embed_dim), np.float32)
        moe.moe_forward_rows_v2(lib, c.gates, c.ups, c.downs, c.gate_fmt, c.down_fmts, None, None, None, c.act,
                                allw, xs[0][:1], o, c.embed_dim, c.inter_dim)
    tg.check(lib)
    for i in range(warm):
        moe.moe_layer_forward(lib, copies[i % R], synth.rms_norm(xs[i]))
    t0 = time.perf_counter()
    for i in range(warm, len(xs)):
        moe.moe_layer_forward(lib, copies[i % R], synth.rms_norm(xs[i]))
    el = time.perf_counter() - t0
    tg.check(lib)
    n = len(xs) - warm
    T = xs.shape[1]
    for c in copies:
        for arr in c.gates + c.ups + c.downs:
            lib.tg_cuda_unregister(arr.ctypes.data)
    return {"value": n * T / el, "unit": UNIT, "h2d_bytes_per_step": int(xs[0].nbytes),
            "d2h_bytes_per_step": int(xs[0].nbytes),
            "api": "engine sequence: numpy rmsnorm + router + top-k + union, then tg_moe_forward_rows_v2 "
                   "(reference ABI, host pointers)", "ms_per_step": el / n * 1e3}


def run_ours(a):
    import torch
    import torch.distributed as dist

    import tinygiant_b200 as tg
    from tinygiant_b200.layer import ResidentLayer

    world, rank, local, lib, stream = setup_gpu(a)
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

    # warm-up: the W steps, and at least one step on every copy
    with torch.cuda.stream(stream):
        for i in range(max(a.warmup, R)):
            step(i % S)
    torch.cuda.synchronize()
    tg.check(lib)
    ms, launches, clk, g = time_graph(lib, step, a.warmup, S, stream, world, local)

    ms_step = ms / a.steps
    ranks_tokens = 1 if ep else world   # data-parallel ranks each process their own tokens
    value = ranks_tokens * a.steps * T / (ms / 1e3)
    line = None
    if rank == 0:
        nbytes = algorithmic_bytes(L, xs_host[a.warmup:])
        achieved = ranks_tokens * nbytes.sum() / (ms / 1e3) / 1e9
        peak1, peak_src = measured_peak()
        peak = peak1 * world            # whole-job bytes against every GPU's HBM
        tr = traffic_from_profiles()
        roof = {"bound": "hbm", "achieved": achieved, "peak": peak, "unit": "GB/s", "frac": achieved / peak,
                "traffic": (tr or {}).get(cfg) if world == 1 else None,
                "traffic_source": "dram__bytes_read.sum + dram__bytes_write.sum per launch from an earlier ncu "
                                  "capture of this workload (profiles/traffic.json), not this run",
                "kernel": "fused MoE layer step (one kernel: router + gate/up + down), per step" if T <= 8 else
                          "batched MoE layer step (routing kernels + grouped GEMMs), per step",
                "algorithmic_bytes_per_step": float(nbytes.mean()), "peak_source": peak_src}
        line = {"metric": METRIC, "value": value, "unit": UNIT, "n_gpus": world, "steps": a.steps,
                "warmup": a.warmup, "ms_per_step": ms_step, "higher_is_better": True,
                "scaling": scaling_of(a, cfg), "vs_baseline": None, "dtype": DTYPES.get(cfg, DTYPES["c2"]),
                "data": "synthetic (seeded weights and inputs)", "config": workload_desc(cfg, T, R, L),
                "parallelism": f"ep{world}" if ep else f"dp{world}",
                "expert_path": "fused step kernel" if T <= 8 else
                               ("matvec kernels" if a.matvec else "tcgen05 grouped GEMMs"),
                "gbps": achieved, "clocks": clk, "roofline": roof, "gpu_launches": launches}
        if T > 8:
            # batched steps: the tensor-pipe roofline of the grouped GEMMs
            ops = batched_ops(L, xs_host[a.warmup:])
            tops = ranks_tokens * ops.sum() / (ms / 1e3) / 1e12
            ipeak, ipsrc = measured_int8_peak()
            ipeak *= world
            line["roofline"] = {"bound": "tensor", "achieved": tops, "peak": ipeak, "unit": "TOPS (int8)",
                                "frac": tops / ipeak, "traffic": None,
                                "kernel": "batched MoE layer step (routing kernels + tcgen05 kind::i8 grouped "
                                          "GEMMs), per step", "ops_per_step": float(ops.mean()),
                                "peak_source": ipsrc, "hbm": roof}
        if ep:
            mean_max, worst = ep_balance(L, xs_host[a.warmup:], world)
            busiest = mean_max * L.expert_bytes(0) + L.router_w.nbytes + 2 * T * D * 4
            line["ep"] = {"combine": "in the step kernel over NVLink" if in_kernel else "NCCL all-reduce",
                          "shard_rule": "expert e on GPU e % N",
                          "max_local_experts_per_step": {"mean": mean_max, "max": worst},
                          "busiest_gpu_hbm_frac": busiest / (ms_step / 1e3) / 1e9 / peak1}

    # e2e: one GPU through the C-ABI entry tg_layer_forward with host buffers
    # (synchronous, x in / MoE output out every step); several GPUs through
    # tg_layer_forward_dev with each step's x copied from pinned host memory
    # and its output read back, plus the all-reduce for ep; max over ranks.
    if world == 1:
        xh = [np.ascontiguousarray(x) for x in xs_host]
        outh = np.zeros((T, D), np.float32)
        # every copy's per-layer graph is instantiated before the timed calls
        for i in range(max(a.warmup, R)):
            layers[i % R].forward(xh[i % S], outh)
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

        for i in range(max(a.warmup, R)):
            e2e_step(i % S)
        dist.barrier()
        t0 = time.perf_counter()
        for i in range(a.warmup, S):
            e2e_step(i)
        el = max_over_ranks(time.perf_counter() - t0, world, local)
        tg.check(lib)
        e2e = {"value": ranks_tokens * a.steps * T / el, "unit": UNIT, "h2d_bytes_per_step": int(xs_host[0].nbytes),
               "d2h_bytes_per_step": int(opin.numel() * 4),
               "api": "tg_layer_forward_dev per rank, pinned host copies" +
                      (" + NCCL all-reduce" if ep and not in_kernel else " (shards combined in the step kernel)" if ep else ""),
               "ms_per_step": el / a.steps * 1e3}
    del g
    for lay in layers:
        lay.close()
    if rank == 0:
        line["e2e"] = e2e
        if world == 1 and T <= 8:
            line["e2e_engine"] = engine_e2e(lib, L, xs_host, R, max(a.warmup, 1))
        if world == 1 and not a.no_cpu_baseline:
            line["cpu_baseline"] = cpu_reference_run(cfg, host_copies(L, R), xs_host[a.warmup:], budget_s=12.0)
        print(json.dumps(line), flush=True)
    if world > 1:
        dist.destroy_process_group()


def run_c1(a):
    """C1: one all-Q4_K expert.  Device-timed: the expert as a one-expert
    resident layer stepped without normalisation (router weight 1, so the step
    writes 1.0 * y, what tg_expert_forward adds to a zeroed output), cycling
    64 HBM copies.  e2e: tg_expert_forward with host buffers, cycling 64 host
    copies (uploaded on first sight)."""
    import torch

    import tinygiant_b200 as tg
    from tinygiant_b200 import quants as Q, synth
    from tinygiant_b200.layer import ResidentLayer

    world, rank, local, lib, stream = setup_gpu(a)
    R = max(1, a.copies if a.copies != R_COPIES else C1_COPIES)
    D, I = 2048, 768
    e0 = synth.c1_expert(seed=0)
    gb = Q.row_bytes(Q.FMT_Q4K, D) * I
    L1 = synth.MoeLayer(D, I, Q.FMT_Q4K, 0, 1, gates=[e0[:gb]], ups=[e0[gb:2 * gb]], downs=[e0[2 * gb:]],
                        down_fmts=[Q.FMT_Q4K], router_w=np.zeros((1, D), np.float32))
    base = ResidentLayer(L1, max_tokens=1, lib=lib)
    layers = [base] + [base.clone() for _ in range(R - 1)]
    tg.check(lib)
    S = a.warmup + a.steps
    xs_host = step_inputs(S, 1, D, seed=4 + 1000 * rank)
    xs = torch.from_numpy(xs_host).to(f"cuda:{local}")
    out = torch.zeros((1, D), dtype=torch.float32, device=f"cuda:{local}")

    def step(i):
        lib.tg_layer_forward_dev(layers[i % R].h, xs[i].data_ptr(), None, None, out.data_ptr(), 1, 0, None)

    with torch.cuda.stream(stream):
        for i in range(max(a.warmup, R)):
            step(i % S)
    torch.cuda.synchronize()
    tg.check(lib)
    ms, launches, clk, g = time_graph(lib, step, a.warmup, S, stream, world, local)
    del g
    for lay in layers:
        lay.close()
    ms_step = ms / a.steps
    # e2e through the reference ABI: tg_expert_forward(x, out += y) on host copies
    # the copies are registered as immutable, as an integration registers its
    # mapped expert files (unregistered host weights are fingerprinted per call)
    copies = [e0] + [e0.copy() for _ in range(R - 1)]
    for c in copies:
        if lib.tg_cuda_register(c.ctypes.data, c.nbytes) != 0:
            tg.check(lib)
    xh = [np.ascontiguousarray(x[0]) for x in xs_host]
    outh = np.zeros(D, np.float32)
    for i in range(R):
        lib.tg_expert_forward(copies[i].ctypes.data, xh[i % S].ctypes.data, outh.ctypes.data, 1.0, D, I)
    tg.check(lib)
    t0 = time.perf_counter()
    for i in range(a.warmup, S):
        outh[:] = 0.0
        lib.tg_expert_forward(copies[i % R].ctypes.data, xh[i].ctypes.data, outh.ctypes.data, 1.0, D, I)
    el = max_over_ranks(time.perf_counter() - t0, world, local)
    tg.check(lib)
    for c in copies:
        lib.tg_cuda_unregister(c.ctypes.data)
    if rank == 0:
        nbytes = float(e0.nbytes + 3 * D * 4)   # weights, x, out, the layer's router row
        achieved = world * nbytes / (ms_step / 1e3) / 1e9
        peak, peak_src = measured_peak()
        peak *= world
        line = {"metric": METRIC, "value": world * a.steps / (ms / 1e3), "unit": UNIT, "n_gpus": world,
                "steps": a.steps, "warmup": a.warmup, "ms_per_step": ms_step, "higher_is_better": True,
                "scaling": "weak" if world > 1 else "strong", "vs_baseline": None, "dtype": DTYPES["c1"],
                "data": "synthetic (seeded weights and inputs)", "config": workload_desc("c1", 1, R, None),
                "parallelism": f"dp{world}", "expert_path": "fused step kernel (one expert, weight 1)",
                "gbps": achieved, "clocks": clk,
                "roofline": {"bound": "hbm", "achieved": achieved, "peak": peak, "unit": "GB/s",
                             "frac": achieved / peak, "traffic": None,
                             "kernel": "fused step kernel on a one-expert layer, per call",
                             "algorithmic_bytes_per_step": nbytes, "peak_source": peak_src},
                "gpu_launches": launches,
                "e2e": {"value": world * a.steps / el, "unit": UNIT, "h2d_bytes_per_step": D * 4,
                        "d2h_bytes_per_step": D * 4,
                        "api": "tg_expert_forward (reference ABI, host buffers; expert copies registered)",
                        "ms_per_step": el / a.steps * 1e3}}
        if world == 1 and not a.no_cpu_baseline:
            line["cpu_baseline"] = cpu_reference_run("c1", copies, xs_host[a.warmup:, 0], budget_s=12.0)
        print(json.dumps(line), flush=True)
    if world > 1:
        import torch.distributed as dist
        dist.destroy_process_group()


def is_stack(a):
    return a.config == "c5" or (a.config == "c4" and n_layers(a) > 1)


def n_layers(a):
    return a.layers if a.layers is not None else {"c4": 36, "c5": 48}.get(a.config, 1)


def stack_desc(cfg, T, NL, L):
    """The `config` of a C4 / C5 stack line (both arms)."""
    desc = workload_desc("c4s" if cfg == "c4" else "c5", T, 1, L)
    desc.pop("layer_copies")
    desc.update({"layers": NL,
                 "l2": f"inputs larger than L2: {NL} layers with per-layer routers ({NL} HBM copies of the experts "
                       f"on the GPU arm, one host copy on the reference arm)",
                 "step": f"{T} token(s) through the stack: per layer rmsnorm + router + top-k + experts + "
                         f"residual add"})
    return desc


def run_stack(a):
    """C4 / C5: T tokens through an n-layer stack (x += MoE(rmsnorm(x)) per
    layer) per step."""
    import torch
    import torch.distributed as dist

    import tinygiant_b200 as tg
    from tinygiant_b200.layer import ResidentLayer

    world, rank, local, lib, stream = setup_gpu(a)
    cfg = a.config
    T, NL = a.tokens or 1, n_layers(a)
    ep = world > 1 and a.parallel == "ep"
    L = make_layer(cfg)
    D = L.embed_dim
    base = ResidentLayer(L, max_tokens=T, lib=lib, shard=rank if ep else 0, n_shards=world if ep else 1)
    layers = [base] + [base.clone() for _ in range(NL - 1)]
    routers = stack_routers(NL, L.n_experts, D)
    for lay, rw in zip(layers, routers):
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
    ms, launches, clk, g = time_graph(lib, step, a.warmup, S, stream, world, local)
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
    el = max_over_ranks(time.perf_counter() - t0, world, local)
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
        line = {"metric": METRIC, "value": value, "unit": UNIT, "n_gpus": world, "steps": a.steps,
                "warmup": a.warmup, "ms_per_step": ms / a.steps, "higher_is_better": True,
                "scaling": scaling_of(a, cfg), "vs_baseline": None,
                "dtype": DTYPES[cfg], "data": "synthetic (seeded weights and inputs)",
                "config": stack_desc(cfg, T, NL, L), "parallelism": f"ep{world}" if ep else f"dp{world}",
                "expert_path": "fused step kernel" if T <= 8 else
                               ("matvec kernels" if a.matvec else "tcgen05 grouped GEMMs"),
                "experts_per_gpu_gb": NL * L.n_experts * L.expert_bytes(0) / 1e9 / (world if ep else 1),
                **({"distinct_experts_per_layer": uniq} if uniq is not None else {}),
                **({"ep": {"combine": "in the step kernel over NVLink" if in_kernel else "NCCL all-reduce",
                           "shard_rule": "expert e on GPU e % N"}} if ep else {}),
                "gbps": achieved, "clocks": clk, "roofline": roof, "gpu_launches": launches,
                "e2e": {"value": ranks_tokens * a.steps * T / el, "unit": UNIT,
                        "h2d_bytes_per_step": int(T * D * 4), "d2h_bytes_per_step": int(T * D * 4),
                        "api": "tg_stack_forward_dev with pinned host copies" if not ep or in_kernel else
                               "tg_layer_forward_dev per layer + NCCL all-reduce, pinned host copies",
                        "ms_per_step": el / a.steps * 1e3}}
        if world == 1 and not a.no_cpu_baseline:
            line["cpu_baseline"] = cpu_reference_run(cfg, [L], xs_host[a.warmup:], budget_s=12.0, routers=routers)
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


# ---- diagnostics: the fused step's phase timeline ---------------------------

TRACE_PHASES = [
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
    ("  CTA barrier (w0, T > 5)", 5, 25),
    ("  poll of its block (w0, T > 2)", 25, 26),
    ("  Q8 + publish (w0, T > 2)", 26, 6),
    ("Q8 of hidden (warp 0)", 6, 15),
    ("  flags poll (w0, T > 2)", 6, 27),
    ("  copy (w0, T > 2)", 27, 15),
    ("CTA sync", 15, 7),
    ("phase B (warp 0)", 7, 8),
]
TRACE_WARP = ["A wait", "A compute", "A issue", "B wait", "B compute", "B issue"]
TRACE_SLOTS = 32   # trace words per CTA


def step_trace(lib, step, n_steps=1):
    """Runs step() n_steps times with the step kernel's trace hook
    (tg_cuda_step_trace) on; returns (phases, warps, counts): name -> array
    over CTAs / warps for the last step, in microseconds (SM cycles converted
    with each CTA's own global-timer span) or poll counts."""
    import torch
    grid = lib.tg_cuda_step_trace(None)
    nw = lib.tg_cuda_step_trace_warps()
    buf = torch.zeros(grid * TRACE_SLOTS + grid * nw * 8, dtype=torch.int64, device="cuda")
    torch.cuda.synchronize()
    lib.tg_cuda_step_trace(ctypes.c_void_p(buf.data_ptr()))
    try:
        for _ in range(n_steps):
            step()
        torch.cuda.synchronize()
    finally:
        lib.tg_cuda_step_trace(None)
    v = buf.cpu().numpy().astype(np.int64)
    t = v[: grid * TRACE_SLOTS].reshape(grid, TRACE_SLOTS)
    span_ns = (t[:, 13] - t[:, 12]).astype(np.float64)
    span_cyc = (t[:, 8] - t[:, 0]).astype(np.float64)
    cyc_per_us = np.median(span_cyc / np.maximum(span_ns, 1.0)) * 1000.0
    # phases whose marks this step does not set (other T) are left out
    phases = {name: (t[:, b] - t[:, a]) / cyc_per_us for name, a, b in TRACE_PHASES if t[:, a].all() and t[:, b].all()}
    phases["whole step (CTA)"] = span_ns / 1000.0
    wv = v[grid * TRACE_SLOTS:].reshape(grid * nw, 8)
    wv = wv[wv.any(axis=1)]   # records of warps a narrower step does not have stay zero
    w = wv[:, :6] / cyc_per_us
    warps = {name: w[:, i] for i, name in enumerate(TRACE_WARP)}
    warps["A total"] = w[:, 0] + w[:, 1] + w[:, 2]
    warps["A end -> hidden ready"] = wv[:, 7] / cyc_per_us
    counts = {"logits polls (CTA)": t[:, 19], "hidden polls (warp)": wv[:, 6]}
    return phases, warps, counts


TC_TRACE = ["producer: waits for a free weight stage", "producer: span",
            "MMA: waits for A/B operands", "MMA: waits for a free accumulator", "MMA: span",
            "unpack: waits for weights", "unpack: waits for a free A/B stage", "unpack: waits for free epilogue data",
            "unpack: waits for row tails", "unpack: span",
            "epilogue: waits for its data", "epilogue: waits for accumulators", "epilogue: span"]


def run_tc_trace(a, T):
    """--config trace --tokens T > 8 [--gptoss]: the tensor-core GEMMs' role
    counters per CTA (kilocycles; percentiles over CTAs) for one batched step
    of C3 (or C4 with --gptoss).  Diagnostics only."""
    import torch

    import tinygiant_b200 as tg
    from tinygiant_b200.layer import ResidentLayer

    lib = tg.load()
    L = make_layer("c4" if a.gptoss else "c3")
    lay = ResidentLayer(L, max_tokens=T, lib=lib)
    stream = torch.cuda.Stream()
    lib.tg_cuda_set_stream(ctypes.c_void_p(stream.cuda_stream))
    x = torch.randn(T, L.embed_dim, device="cuda")
    out = torch.zeros_like(x)
    try:
        with torch.cuda.stream(stream):
            for _ in range(3):
                lib.tg_layer_forward_dev(lay.h, ctypes.c_void_p(x.data_ptr()), None, None,
                                         ctypes.c_void_p(out.data_ptr()), T, 1, None)
            torch.cuda.synchronize()
            grid = lib.tg_cuda_tc_trace(None)
            buf = torch.zeros(2 * grid * 16, dtype=torch.int64, device="cuda")
            torch.cuda.synchronize()
            lib.tg_cuda_tc_trace(ctypes.c_void_p(buf.data_ptr()))
            lib.tg_layer_forward_dev(lay.h, ctypes.c_void_p(x.data_ptr()), None, None,
                                     ctypes.c_void_p(out.data_ptr()), T, 1, None)
            torch.cuda.synchronize()
            lib.tg_cuda_tc_trace(None)
        tg.check(lib)
        v = buf.cpu().numpy().reshape(2, grid, 16).astype(np.float64)
        for p, name in enumerate(("gate/up", "down")):
            print(f"== {name} GEMM, T = {T}: units per CTA median {np.median(v[p, :, 13]):.0f}, "
                  f"steps per CTA median {np.median(v[p, :, 14]):.0f}")
            print(f"  {'(kcycles)':44s}{'min':>8s}{'p10':>8s}{'median':>8s}{'p90':>8s}{'max':>8s}")
            for i, n in enumerate(TC_TRACE):
                q = np.percentile(v[p, :, i] / 1000.0, [0, 10, 50, 90, 100])
                print(f"  {n:44s}" + "".join(f"{x:8.1f}" for x in q))
    finally:
        lib.tg_cuda_set_stream(None)
        lay.close()


def run_trace(a):
    """--config trace [--gptoss] [--experts E] [--copies R] [--tokens T]: the
    fused step's phase timeline (percentiles over CTAs / warps), after one
    idle step and for the last of 8 back-to-back steps; with T > 8 the
    tensor-core GEMMs' role counters (run_tc_trace).  Diagnostics only."""
    import torch
    if (a.tokens or 1) > 8:
        run_tc_trace(a, a.tokens)
        return

    import tinygiant_b200 as tg
    from tinygiant_b200 import synth
    from tinygiant_b200.layer import ResidentLayer

    lib = tg.load()
    E = a.experts or 128
    T = a.tokens or 1
    R = a.copies if a.copies != R_COPIES else 4
    L = synth.gptoss_layer(seed=3, n_experts=E) if a.gptoss else synth.qwen_layer(seed=1, n_experts=E)
    base = ResidentLayer(L, max_tokens=T, lib=lib)
    lays = [base] + [base.clone() for _ in range(R - 1)]
    stream = torch.cuda.Stream()
    lib.tg_cuda_set_stream(ctypes.c_void_p(stream.cuda_stream))
    x = torch.randn(T, L.embed_dim, device="cuda")
    out = torch.zeros_like(x)
    it = [0]

    def step():
        lay = lays[it[0] % len(lays)]
        it[0] += 1
        lib.tg_layer_forward_dev(lay.h, ctypes.c_void_p(x.data_ptr()), None, None, ctypes.c_void_p(out.data_ptr()),
                                 T, 1, None)

    try:
        with torch.cuda.stream(stream):
            for _ in range(20):
                step()
            torch.cuda.synchronize()
            for tag, n in (("one step after idle", 1), ("last of 8 back-to-back steps", 8)):
                phases, warps, counts = step_trace(lib, step, n)
                print(f"== {tag}")
                print(f"  {'':37s}{'min':>8s}{'p10':>8s}{'median':>8s}{'p90':>8s}{'max':>8s}")

                def row(name, d, fmt="8.2f"):
                    q = np.percentile(d, [0, 10, 50, 90, 100])
                    print(f"  {name:37s}" + "".join(format(x, fmt) for x in q))
                for name, d in phases.items():
                    row(name + " (us)", d)
                for name, d in warps.items():
                    row("per-warp " + name + " (us)", d)
                for name, d in counts.items():
                    row(name, d, "8.0f")
        tg.check(lib)
    finally:
        lib.tg_cuda_set_stream(None)
        for lay in lays:
            lay.close()


def main():
    a = parse()
    if a.config == "attn":
        run_attn(a)
        return
    if a.config == "cache":
        run_cache(a)
        return
    if a.config == "trace":
        run_trace(a)
        return
    if a.impl == "reference":
        run_reference(a)
    elif a.config == "c1":
        run_c1(a)
    elif is_stack(a):
        run_stack(a)
    else:
        run_ours(a)


if __name__ == "__main__":
    main()
