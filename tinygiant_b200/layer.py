"""Python handle for a resident MoE layer routed on the GPU.

Wraps tg_layer_* of libtinygiant.so: all experts of a synth.MoeLayer (or any
expert byte arrays) go to HBM once; a step runs rmsnorm -> router -> top-k
-> experts entirely on the device.
"""
import ctypes

import numpy as np

from . import check, load


class ResidentLayer:
    def __init__(self, layer, max_tokens=1, lib=None, handle=None, shard=0, n_shards=1):
        self.lib = lib or load()
        self.layer = layer
        self.max_tokens = max_tokens
        self.D, self.I, self.E, self.k = layer.embed_dim, layer.inter_dim, layer.n_experts, layer.top_k
        if handle is not None:
            self.h = handle
            return
        P = ctypes.c_void_p
        self._g = (P * self.E)(*[a.ctypes.data for a in layer.gates])
        self._u = (P * self.E)(*[a.ctypes.data for a in layer.ups])
        self._d = (P * self.E)(*[a.ctypes.data for a in layer.downs])
        self._f = (ctypes.c_int * self.E)(*layer.down_fmts)
        self._rw = np.ascontiguousarray(layer.router_w, dtype=np.float32)
        self._rb = None if layer.router_b is None else np.ascontiguousarray(layer.router_b, dtype=np.float32)
        self.shard, self.n_shards = shard, n_shards
        self.h = self.lib.tg_layer_create_shard(self.E, ctypes.addressof(self._g), ctypes.addressof(self._u),
                                                ctypes.addressof(self._d), layer.gate_fmt, ctypes.addressof(self._f),
                                                None, None, None, layer.act, self.D, self.I, self._rw.ctypes.data,
                                                None if self._rb is None else self._rb.ctypes.data, self.k,
                                                max_tokens, shard, n_shards)
        if not self.h:
            check(self.lib)
            raise RuntimeError("tg_layer_create failed")

    def clone(self):
        h = self.lib.tg_layer_clone(self.h)
        if not h:
            check(self.lib)
        r = ResidentLayer(self.layer, self.max_tokens, self.lib, handle=h)
        r.shard, r.n_shards = self.shard, self.n_shards
        return r

    def set_router(self, router_w, router_b=None):
        """A new fp32 router [E, D] (and bias [E]) for this layer."""
        self._rw2 = np.ascontiguousarray(router_w, dtype=np.float32)
        self._rb2 = None if router_b is None else np.ascontiguousarray(router_b, dtype=np.float32)
        rc = self.lib.tg_layer_set_router(self.h, self._rw2.ctypes.data,
                                          None if self._rb2 is None else self._rb2.ctypes.data)
        check(self.lib)
        if rc != 0:
            raise RuntimeError("tg_layer_set_router failed")

    def ep_connect(self):
        """Expert-parallel shards (one process per GPU, torch.distributed
        initialised): exchange the shards' receive-block handles and map them,
        so decode-sized steps combine the shards' parts inside the step kernel
        over NVLink and return the whole layer's output on every shard."""
        import torch.distributed as dist
        h = ctypes.create_string_buffer(64)
        if self.lib.tg_layer_ep_handle(self.h, h) != 0:
            check(self.lib)
            raise RuntimeError("tg_layer_ep_handle failed")
        handles = [None] * self.n_shards
        dist.all_gather_object(handles, bytes(h.raw))
        self._ep_handles = ctypes.create_string_buffer(b"".join(handles), 64 * self.n_shards)
        if self.lib.tg_layer_ep_connect(self.h, self._ep_handles) != 0:
            check(self.lib)
            raise RuntimeError("tg_layer_ep_connect failed")

    def ep_reset(self):
        """Restart this layer's step epochs at 1 (tg_layer_ep_reset); see
        EpStepper for when shards call it."""
        if self.lib.tg_layer_ep_reset(self.h) != 0:
            check(self.lib)
            raise RuntimeError("tg_layer_ep_reset failed")

    def set_tc(self, on=True):
        """Tensor-core grouped GEMMs (default) or matvec kernels for batched steps (T > 8)."""
        return bool(self.lib.tg_layer_set_tc(self.h, int(bool(on))))

    def set_fused(self, on=True):
        """Fused single-kernel steps (default) or the three-kernel path."""
        return bool(self.lib.tg_layer_set_fused(self.h, int(bool(on))))

    def expert_bytes(self, e):
        return self.lib.tg_layer_expert_bytes(self.h, e)

    def forward(self, x, out=None, normalize=True):
        """Host arrays: out [T, D] += experts(rmsnorm(x))."""
        x = np.ascontiguousarray(np.atleast_2d(x), dtype=np.float32)
        if out is None:
            out = np.zeros_like(x)
        rc = self.lib.tg_layer_forward(self.h, x.ctypes.data, out.ctypes.data, x.shape[0], int(normalize))
        check(self.lib)
        if rc != 0:
            raise RuntimeError("tg_layer_forward failed")
        return out

    def last_routing(self, T):
        idx = np.zeros((T, self.k), np.int32)
        w = np.zeros((T, self.k), np.float32)
        self.lib.tg_layer_last_routing(self.h, T, idx.ctypes.data, w.ctypes.data)
        return idx, w

    def close(self):
        if self.h:
            self.lib.tg_layer_destroy(self.h)
            self.h = None


class EpStepper:
    """Agreement on the outcome of expert-parallel steps across shards.

    The shards of a layer combine their parts inside the step kernel, each
    word tagged with the step's epoch (the layer's launch count), so every
    shard must count the same steps.  A shard whose step fails (a bounded
    wait ran out because a peer did not step, or any device error) resets its
    own exchange state; its peers, whose steps may have failed or not, keep
    counting.  So after every step the shards all-reduce a failure flag over
    the host process group (torch.distributed, any backend), and on any
    failure every shard resets the layers' epochs between two barriers
    (ep_reset) and reports the step as failed; the next step starts at epoch
    1 everywhere.

    step: a callable running one step on this shard and returning True on
    success (it synchronises and checks the device status itself); layers:
    objects with ep_reset() (ResidentLayer).  The collectives are the same on
    every shard and in the same order, whatever the outcome.
    """

    def __init__(self, layers, group=None):
        self.layers = list(layers)
        self.group = group
        self.resets = 0
        self.errors = []           # (step number, repr of the exception) of steps that raised

    def __call__(self, step):
        import torch
        import torch.distributed as dist
        try:
            ok = bool(step())
        except Exception as ex:    # a failed step is reported to the peers, never skipped
            self.errors.append((self.resets, repr(ex)))
            ok = False
        backend = dist.get_backend(self.group)
        dev = torch.device("cuda", torch.cuda.current_device()) if backend == "nccl" else torch.device("cpu")
        flag = torch.tensor([0 if ok else 1], dtype=torch.int32, device=dev)
        dist.all_reduce(flag, op=dist.ReduceOp.MAX, group=self.group)
        if int(flag.item()) == 0:
            return True
        dist.barrier(group=self.group)
        for lay in self.layers:
            lay.ep_reset()
        dist.barrier(group=self.group)
        self.resets += 1
        return False
