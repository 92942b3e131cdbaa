"""Expert-parallel layers across ranks: experts e with e % world == rank on
each rank, the parts summed by one all-reduce (the multi-GPU plan of the
layer path).  The decomposition is checked on CPU ranks over gloo with the
oracle standing in for the GPU kernels; on a box with two GPUs the same is
run through the library over NCCL."""
import os
import socket

import numpy as np
import pytest

TOL = 1e-5


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _layer():
    from tinygiant_b200 import synth
    return synth.qwen_layer(seed=11, n_experts=8, D=512, I=256, top_k=3)


def _rows():
    from tinygiant_b200 import synth
    return synth.rms_norm(np.random.default_rng(12).standard_normal((3, 512)).astype(np.float32))


def _shard_part(lib, layer, N, rank, world):
    """This rank's experts' share of the layer output (oracle or library)."""
    from tinygiant_b200 import moe as M
    from tinygiant_b200 import synth
    experts, row_w, _, _ = synth.route(layer, N)
    keep = [i for i, e in enumerate(experts) if int(e) % world == rank]
    out = np.zeros_like(N)
    if keep:
        sel = [int(experts[i]) for i in keep]
        M.moe_forward_rows_v2(lib, [layer.gates[e] for e in sel], [layer.ups[e] for e in sel],
                              [layer.downs[e] for e in sel], layer.gate_fmt, [layer.down_fmts[e] for e in sel],
                              None, None, None, layer.act, np.ascontiguousarray(row_w[keep]), N, out,
                              layer.embed_dim, layer.inter_dim)
    return out


def _gloo_rank(rank, world, port, q):
    import torch
    import torch.distributed as dist
    from datetime import timedelta
    from oracle import oracle as O
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=timedelta(seconds=60))
    try:
        lib = O.load_oracle()
        L, N = _layer(), _rows()
        part = torch.from_numpy(_shard_part(lib, L, N, rank, world))
        dist.all_reduce(part)
        if rank == 0:
            whole = _shard_part(lib, L, N, 0, 1)
            q.put(float(np.max(np.abs(part.numpy() - whole)) / np.max(np.abs(whole))))
    finally:
        dist.destroy_process_group()


def test_expert_shards_sum_to_whole_gloo():
    import torch.multiprocessing as mp
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_gloo_rank, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout=120)
    assert all(p.exitcode == 0 for p in procs), [p.exitcode for p in procs]
    assert q.get(timeout=5) <= TOL


def _nccl_rank(rank, world, port, q, in_kernel=False):
    import ctypes

    import torch
    import torch.distributed as dist
    from datetime import timedelta
    import tinygiant_b200 as tg
    from tinygiant_b200.layer import ResidentLayer
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), NCCL_NVLS_ENABLE="0")
    torch.cuda.set_device(rank)
    dist.init_process_group("nccl", rank=rank, world_size=world, timeout=timedelta(seconds=60),
                            device_id=torch.device("cuda", rank))
    try:
        lib = tg.load()
        lib.tg_cuda_set_device(rank)
        L, N = _layer(), _rows()
        shard = ResidentLayer(L, max_tokens=N.shape[0], lib=lib, shard=rank, n_shards=world)
        if in_kernel:
            shard.ep_connect()
        x = torch.from_numpy(N).cuda()
        out = torch.zeros_like(x)
        stream = torch.cuda.current_stream()
        lib.tg_cuda_set_stream(ctypes.c_void_p(stream.cuda_stream))
        for _ in range(3 if in_kernel else 1):   # repeated steps reuse the receive blocks (new epochs)
            assert lib.tg_layer_forward_dev(shard.h, ctypes.c_void_p(x.data_ptr()), None, None,
                                            ctypes.c_void_p(out.data_ptr()), N.shape[0], 0, None) == 0
        if not in_kernel:
            dist.all_reduce(out)
        torch.cuda.synchronize()
        tg.check(lib)
        if rank == 0:
            whole = ResidentLayer(L, max_tokens=N.shape[0], lib=lib).forward(N, normalize=False)
            got = out.cpu().numpy()
            q.put(float(np.max(np.abs(got - whole)) / np.max(np.abs(whole))))
        lib.tg_cuda_set_stream(None)
        shard.close()
    finally:
        dist.destroy_process_group()


@pytest.mark.gpu
@pytest.mark.parametrize("in_kernel", [False, True])
def test_expert_shards_two_gpus(in_kernel):
    """Two GPUs, one process each: the shards' parts summed by an NCCL
    all-reduce, or inside the step kernel over NVLink (tg_layer_ep_connect),
    equal the unsharded layer."""
    import torch
    if torch.cuda.device_count() < 2:
        pytest.skip("needs two GPUs")
    import torch.multiprocessing as mp
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_nccl_rank, args=(r, 2, port, q, in_kernel)) for r in range(2)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout=180)
    assert all(p.exitcode == 0 for p in procs), [p.exitcode for p in procs]
    assert q.get(timeout=5) <= TOL


# ---- failure agreement across shards (layer.EpStepper) ----------------------

class _FakeShardLayer:
    """Stands in for a ResidentLayer: its epoch is the count of steps since
    the last reset, as the step kernel's launch counter is."""

    def __init__(self):
        self.epoch = 0
        self.resets = 0

    def ep_reset(self):
        self.epoch = 0
        self.resets += 1


def _stepper_rank(rank, world, port, q, fail_at, peer_sees_failure):
    import torch
    import torch.distributed as dist
    from datetime import timedelta
    from tinygiant_b200.layer import EpStepper
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=timedelta(seconds=60))
    try:
        lay = _FakeShardLayer()
        stepper = EpStepper([lay])
        log = []
        for i in range(1, 7):
            def step():
                lay.epoch += 1
                epochs = [None] * world
                dist.all_gather_object(epochs, lay.epoch)
                if rank == 1 and i == fail_at:
                    lay.epoch = 0          # the failing shard's runtime resets only itself
                    raise RuntimeError("injected: a wait ran out")
                # the in-kernel combine only completes when every shard tags the same epoch
                same = len(set(epochs)) == 1
                return same and not (peer_sees_failure and i == fail_at)
            ok = stepper(step)
            epochs = [None] * world
            dist.all_gather_object(epochs, lay.epoch)
            log.append((ok, tuple(epochs)))
        if rank == 0:
            q.put((log, lay.resets, stepper.resets))
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("peer_sees_failure", [False, True])
def test_ep_stepper_resyncs_epochs_on_cpu_ranks(peer_sees_failure):
    """Rank 1's step fails at step 3 (its runtime resets its own epochs); with
    or without rank 0 seeing a failure of its own, both shards agree the step
    failed, both restart their epochs, and every later step succeeds with
    equal epochs on both."""
    import torch.multiprocessing as mp
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_stepper_rank, args=(r, 2, port, q, 3, peer_sees_failure)) for r in range(2)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout=120)
    assert all(p.exitcode == 0 for p in procs), [p.exitcode for p in procs]
    log, resets, stepper_resets = q.get(timeout=5)
    assert [ok for ok, _ in log] == [True, True, False, True, True, True]
    assert resets == 1 and stepper_resets == 1
    for ok, epochs in log:
        assert len(set(epochs)) == 1
    assert [e[0] for _, e in log] == [1, 2, 0, 1, 2, 3]


def _skip_rank(rank, world, port, q):
    import ctypes

    import torch
    import torch.distributed as dist
    from datetime import timedelta
    import tinygiant_b200 as tg
    from tinygiant_b200.layer import EpStepper, ResidentLayer
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), NCCL_NVLS_ENABLE="0")
    torch.cuda.set_device(rank)
    dist.init_process_group("nccl", rank=rank, world_size=world, timeout=timedelta(seconds=60),
                            device_id=torch.device("cuda", rank))
    log = []
    try:
        lib = tg.load()
        lib.tg_cuda_set_device(rank)
        L, N = _layer(), _rows()
        shard = ResidentLayer(L, max_tokens=N.shape[0], lib=lib, shard=rank, n_shards=world)
        shard.ep_connect()
        lib.tg_cuda_set_stream(None)
        lib.tg_cuda_debug_step_fault(-1, 1 << 14)     # waits give up after ~ms, not ~1 s
        x = torch.from_numpy(N).cuda()
        out = torch.zeros_like(x)
        torch.cuda.synchronize()
        stepper = EpStepper([shard])
        oks = []
        for i in range(5):
            def step():
                if rank == 1 and i == 2:
                    log.append((i, "skipped"))
                    return True                      # this shard does not launch step 2
                rc = lib.tg_layer_forward_dev(shard.h, ctypes.c_void_p(x.data_ptr()), None, None,
                                              ctypes.c_void_p(out.data_ptr()), N.shape[0], 0, None)
                sync = lib.tg_cuda_synchronize()
                code, msg = tg.last_error(lib)
                log.append((i, rc, sync, code, msg))
                return rc == 0 and sync == 0 and code == 0
            oks.append(stepper(step))
        lib.tg_cuda_debug_step_fault(-1, 0)
        err = None
        if rank == 0:
            whole = ResidentLayer(L, max_tokens=N.shape[0], lib=lib).forward(N, normalize=False)
            got = out.cpu().numpy()
            err = float(np.max(np.abs(got - whole)) / np.max(np.abs(whole)))
        shard.close()
        q.put((rank, oks, err, log + stepper.errors))
    except Exception as ex:             # reported to the test, which fails on it
        q.put((rank, None, None, log + [repr(ex)]))
    finally:
        dist.destroy_process_group()


@pytest.mark.gpu
def test_shard_that_skips_a_step_makes_its_peer_time_out_then_both_recover():
    """Two GPUs, the in-kernel combine: shard 1 skips step 2 (between steps,
    nothing of it in flight); shard 0's combine poll runs out and is reported
    (device error 2 at site 38); EpStepper restarts both shards' epochs and
    steps 3 and 4 give the unsharded layer's output."""
    import torch
    if torch.cuda.device_count() < 2:
        pytest.skip("needs two GPUs")
    import torch.multiprocessing as mp
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_skip_rank, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout=180)
    assert all(p.exitcode == 0 for p in procs), [p.exitcode for p in procs]
    res = dict((m[0], m[1:]) for m in (q.get(timeout=5), q.get(timeout=5)))
    oks0, err, log0 = res[0]
    oks1, _, log1 = res[1]
    assert oks0 == oks1 == [True, True, False, True, True], (log0, log1)
    step2 = [e for e in log0 if e[0] == 2][0]
    assert step2[3] == 202 and "site 38" in step2[4], step2
    assert err <= TOL
