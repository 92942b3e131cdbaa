"""tg_cuda_matmul_q4k_noalloc, the allocation-free Q4_K matvec, against the
existing entry point tg_matmul_q4k (host buffers) on the same inputs.

The file name sorts last so the test also runs after every other GPU test
(with the library's context, registry and scratch already set up); it must
pass just as well alone in a fresh process."""
import ctypes

import numpy as np
import pytest

pytestmark = pytest.mark.gpu

MAX_COLS = 65536


def _q4k_matrix(rng, rows, cols):
    from tinygiant_b200 import quants as Q
    return Q.pack_q4k(rng.standard_normal((rows, cols)).astype(np.float32))


def _host_matmul(lib, mat, x, rows, cols):
    out = np.empty(rows, np.float32)
    lib.tg_matmul_q4k(mat.ctypes.data, x.ctypes.data, out.ctypes.data, rows, cols)
    return out


def _last_error(lib):
    buf = ctypes.create_string_buffer(512)
    code = lib.tg_cuda_last_error(buf, 512)
    return code, buf.value.decode()


def test_noalloc_matches_tg_matmul_q4k_two_calls_in_a_row(gpu):
    import torch

    lib = gpu
    rng = np.random.default_rng(20261201)
    cases = [(300, 2048), (96, MAX_COLS)]
    mats = [_q4k_matrix(rng, r, c) for r, c in cases]
    xs = [rng.standard_normal(c).astype(np.float32) for _, c in cases]
    want = [_host_matmul(lib, m, x, r, c) for m, x, (r, c) in zip(mats, xs, cases)]

    dev = torch.device("cuda", 0)
    d_mats = [torch.from_numpy(m).to(dev) for m in mats]
    d_xs = [torch.from_numpy(x).to(dev) for x in xs]
    d_outs = [torch.full((r,), float("nan"), device=dev) for r, _ in cases]
    stream = torch.cuda.Stream(device=dev)
    torch.cuda.synchronize(dev)

    def call(i):
        r, c = cases[i]
        return lib.tg_cuda_matmul_q4k_noalloc(d_mats[i].data_ptr(), d_xs[i].data_ptr(), d_outs[i].data_ptr(), r, c,
                                              ctypes.c_void_p(stream.cuda_stream))

    # Two calls in a row on one stream, no synchronisation between them: the
    # second overwrites the scratch only after the first has read it.
    for _ in range(2):
        for t in d_outs:
            t.fill_(float("nan"))
        torch.cuda.synchronize(dev)
        assert call(0) == 0, _last_error(lib)
        assert call(1) == 0, _last_error(lib)
        stream.synchronize()
        for i in range(2):
            got = d_outs[i].cpu().numpy()
            np.testing.assert_array_equal(got.view(np.uint32), want[i].view(np.uint32))

    # Once set up, further calls allocate no device memory.  The free-memory
    # figure is device-wide, so another process can move it: any device
    # allocation takes at least 2 MiB, so a drop of 1 MiB or more in every
    # one of three tries fails the test.
    drops = []
    for _ in range(3):
        free0 = torch.cuda.mem_get_info(dev)[0]
        assert call(0) == 0 and call(1) == 0
        stream.synchronize()
        drops.append(free0 - torch.cuda.mem_get_info(dev)[0])
        if drops[-1] < (1 << 20):
            break
    assert min(drops) < (1 << 20), drops


def test_noalloc_rejects_sizes_beyond_its_scratch(gpu):
    import torch

    lib = gpu
    dev = torch.device("cuda", 0)
    cols = MAX_COLS + 256
    mat = torch.zeros(8 * lib.tg_row_bytes(0, cols), dtype=torch.uint8, device=dev)
    x = torch.zeros(cols, device=dev)
    out = torch.zeros(8, device=dev)
    rc = lib.tg_cuda_matmul_q4k_noalloc(mat.data_ptr(), x.data_ptr(), out.data_ptr(), 8, cols, None)
    assert rc == 3
    code, msg = _last_error(lib)
    assert code == 3 and "65536" in msg
    # Host memory is refused before anything is launched.
    h = np.zeros(256, np.float32)
    rc = lib.tg_cuda_matmul_q4k_noalloc(mat.data_ptr(), h.ctypes.data, out.data_ptr(), 8, 256, None)
    assert rc == 3 and "device memory" in _last_error(lib)[1]
