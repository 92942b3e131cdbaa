"""Failure detection without a GPU fault: every wait in the fused step kernel
is bounded, and a wait that runs out is reported through the device status
and tg_cuda_last_error, after which the library is usable again.

The failure is made by the test itself, never by a fault: a debug knob
(tg_cuda_debug_step_fault) shortens the poll limit to a few thousand polls
and makes one CTA skip publishing its router logits, so every CTA's logits
poll runs out.  The 2-GPU test stops one shard between steps (it simply does
not launch one step) so that its peer's in-kernel combine times out; the
host-side agreement (layer.EpStepper) then restarts both shards' epochs and
the next steps are correct again."""
import ctypes

import numpy as np
import pytest

import tinygiant_b200 as tg
from tinygiant_b200 import synth
from tinygiant_b200.layer import ResidentLayer

pytestmark = pytest.mark.gpu


@pytest.fixture
def layer16(gpu):
    L = synth.qwen_layer(seed=1, n_experts=16)
    R = ResidentLayer(L, max_tokens=2, lib=gpu)
    yield L, R
    R.close()
    gpu.tg_cuda_debug_step_fault(-1, 0)


def _dev_step(lib, R, x, out):
    rc = lib.tg_layer_forward_dev(R.h, ctypes.c_void_p(x.data_ptr()), None, None, ctypes.c_void_p(out.data_ptr()),
                                  x.shape[0], 1, None)
    assert rc == 0, tg.last_error(lib)
    return lib.tg_cuda_synchronize()


def test_step_poll_timeout_is_reported_then_the_next_step_is_clean(gpu, layer16):
    import torch
    L, R = layer16
    x = torch.from_numpy(np.random.default_rng(31).standard_normal((2, 2048)).astype(np.float32)).cuda()
    out = torch.zeros_like(x)
    lib = gpu
    lib.tg_cuda_set_stream(None)
    assert _dev_step(lib, R, x, out) == 0
    tg.check(lib)
    want = out.cpu().numpy().copy()
    # CTA 5 publishes no logits; polls give up after 4096 tries (~ms)
    lib.tg_cuda_debug_step_fault(5, 4096)
    out.fill_(7.0)
    assert _dev_step(lib, R, x, out) != 0
    code, msg = tg.last_error(lib)
    assert code == 202 and "device error 2" in msg and "site 31" in msg, (code, msg)
    # the knob off: the same layer steps cleanly and gives the same output
    lib.tg_cuda_debug_step_fault(-1, 0)
    out.zero_()
    assert _dev_step(lib, R, x, out) == 0
    tg.check(lib)
    np.testing.assert_array_equal(out.cpu().numpy().view(np.uint32), want.view(np.uint32))
