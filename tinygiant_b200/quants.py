"""Host-side block formats: packers, generators and numpy decoders.

Layouts are TinyGiant's (csrc/libtinygiant.c): Q4_K 144-byte blocks of 256
values (fp16 d, fp16 dmin, 12 bytes of 6-bit scales/mins, 128 bytes of
nibbles), Q6_K 210-byte blocks (ql[128], qh[64], int8 scales[16], fp16 d),
MXFP4 17-byte blocks of 32 (e8m0 exponent, 16 bytes of e2m1 nibbles).
The packers run in the library (tg_pack_q4k / tg_pack_q6k); the decoders
here restate the reference's decode for building float references.
"""
import numpy as np

from . import load

FMT_Q4K, FMT_F16, FMT_Q6K, FMT_MXFP4, FMT_Q80 = 0, 1, 2, 3, 4
BLOCK = {FMT_Q4K: (256, 144), FMT_Q6K: (256, 210), FMT_MXFP4: (32, 17), FMT_Q80: (32, 34)}
MXFP4_KVALUES = np.array([0, 1, 2, 3, 4, 6, 8, 12, 0, -1, -2, -3, -4, -6, -8, -12], dtype=np.int8)


def row_bytes(fmt, cols):
    """tg_row_bytes (libtinygiant.c:596-606)."""
    if fmt in BLOCK:
        n, b = BLOCK[fmt]
        return (cols // n) * b
    return cols * 2


def _pack(fn, fmt, w):
    w = np.ascontiguousarray(w, dtype=np.float32)
    rows, cols = w.shape
    if cols % 256:
        raise ValueError("cols must be a multiple of 256")
    out = np.empty(rows * row_bytes(fmt, cols), dtype=np.uint8)
    fn(w.ctypes.data, rows, cols, out.ctypes.data)
    return out


def pack_q4k(w):
    return _pack(load().tg_pack_q4k, FMT_Q4K, w)


def pack_q6k(w):
    return _pack(load().tg_pack_q6k, FMT_Q6K, w)


def mxfp4_random(rows, cols, rng, exp_lo=119, exp_hi=123):
    """MXFP4 rows with e8m0 exponents uniform in [exp_lo, exp_hi] (i.e. scale
    exponents exp-127 in [-8, -4] by default) and uniform random codes."""
    nsub = rows * (cols // 32)
    b = np.empty((nsub, 17), dtype=np.uint8)
    b[:, 0] = rng.integers(exp_lo, exp_hi + 1, size=nsub, dtype=np.uint8)
    b[:, 1:] = rng.integers(0, 256, size=(nsub, 16), dtype=np.uint8)
    return b.reshape(-1)


# ---- numpy decoders (reference decode restated) ------------------------

def _f16(u8pair):
    return u8pair.copy().view(np.float16).astype(np.float32).reshape(-1)


def dequant_q4k(data, rows, cols):
    """value = d*sc*q - dmin*m, float32 as libtinygiant.c's test decoder
    (test_libtinygiant.c:111-130)."""
    b = np.asarray(data, dtype=np.uint8).reshape(-1, 144)
    d = _f16(b[:, 0:2])[:, None]
    dmin = _f16(b[:, 2:4])[:, None]
    s = b[:, 4:16].astype(np.int32)
    sc = np.empty((b.shape[0], 8), np.int32)
    mn = np.empty((b.shape[0], 8), np.int32)
    sc[:, :4] = s[:, 0:4] & 63
    mn[:, :4] = s[:, 4:8] & 63
    sc[:, 4:] = (s[:, 8:12] & 0xF) | ((s[:, 0:4] >> 6) << 4)
    mn[:, 4:] = (s[:, 8:12] >> 4) | ((s[:, 4:8] >> 6) << 4)
    qs = b[:, 16:144].reshape(-1, 4, 32)
    q = np.empty((b.shape[0], 256), np.float32)
    for g in range(4):
        q[:, 64 * g:64 * g + 32] = qs[:, g] & 0xF
        q[:, 64 * g + 32:64 * g + 64] = qs[:, g] >> 4
    scale = (d * sc.astype(np.float32)).repeat(32, axis=1)
    minv = (dmin * mn.astype(np.float32)).repeat(32, axis=1)
    return (scale * q - minv).reshape(rows, cols)


def dequant_q6k(data, rows, cols):
    b = np.asarray(data, dtype=np.uint8).reshape(-1, 210)
    ql = b[:, 0:128].astype(np.int32)
    qh = b[:, 128:192].astype(np.int32)
    sc = b[:, 192:208].view(np.int8).astype(np.float32)
    d = _f16(b[:, 208:210])[:, None]
    q = np.empty((b.shape[0], 256), np.int32)
    for h in range(2):
        for l in range(32):
            a, c, hh = ql[:, 64 * h + l], ql[:, 64 * h + 32 + l], qh[:, 32 * h + l]
            q[:, 128 * h + l] = (a & 15) | ((hh & 3) << 4)
            q[:, 128 * h + l + 32] = (c & 15) | (((hh >> 2) & 3) << 4)
            q[:, 128 * h + l + 64] = (a >> 4) | (((hh >> 4) & 3) << 4)
            q[:, 128 * h + l + 96] = (c >> 4) | ((hh >> 6) << 4)
    scale = (d * sc).repeat(16, axis=1)
    return (scale * (q - 32).astype(np.float32)).reshape(rows, cols)


def e8m0_half(e):
    e = np.asarray(e, dtype=np.uint32)
    bits = np.where(e < 2, np.uint32(0x00200000) << e, (e - 1) << 23).astype(np.uint32)
    return bits.view(np.float32)


def dequant_mxfp4(data, rows, cols):
    """Doubled e2m1 code * 2^(e-128), i.e. the reference's value convention."""
    b = np.asarray(data, dtype=np.uint8).reshape(-1, 17)
    d = e8m0_half(b[:, 0])[:, None]
    codes = b[:, 1:]
    v = np.empty((b.shape[0], 32), np.float32)
    v[:, :16] = MXFP4_KVALUES[codes & 15]
    v[:, 16:] = MXFP4_KVALUES[codes >> 4]
    return (v * d).reshape(rows, cols)


DEQUANT = {FMT_Q4K: dequant_q4k, FMT_Q6K: dequant_q6k, FMT_MXFP4: dequant_mxfp4}
