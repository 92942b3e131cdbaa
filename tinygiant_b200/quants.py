"""Host-side block formats: packers, generators and numpy decoders.

Layouts are TinyGiant's (csrc/libtinygiant.c): Q4_K 144-byte blocks of 256
values (fp16 d, fp16 dmin, 12 bytes of 6-bit scales/mins, 128 bytes of
nibbles), Q6_K 210-byte blocks (ql[128], qh[64], int8 scales[16], fp16 d),
MXFP4 17-byte blocks of 32 (e8m0 exponent, 16 bytes of e2m1 nibbles).
The packers (numpy, host only) make the synthetic weights; the reference
has no quantizer, so they fill its block layouts with a plain per-sub-block
fit.  The decoders restate the reference's decode for building float
references.  Nothing here is on the GPU path, and nothing here loads the
product library.
"""
import numpy as np

FMT_Q4K, FMT_F16, FMT_Q6K, FMT_MXFP4, FMT_Q80 = 0, 1, 2, 3, 4
BLOCK = {FMT_Q4K: (256, 144), FMT_Q6K: (256, 210), FMT_MXFP4: (32, 17), FMT_Q80: (32, 34)}
MXFP4_KVALUES = np.array([0, 1, 2, 3, 4, 6, 8, 12, 0, -1, -2, -3, -4, -6, -8, -12], dtype=np.int8)


def row_bytes(fmt, cols):
    """tg_row_bytes (libtinygiant.c:596-606)."""
    if fmt in BLOCK:
        n, b = BLOCK[fmt]
        return (cols // n) * b
    return cols * 2


# ---- packers ----------------------------------------------------------------
#
#   Q4_K : value ~= d*sc_j*q - dmin*m_j, q in [0,15]; per 32-value sub-block
#          lo = min(min(x), 0), scale_j = (max(x) - lo)/15, min_j = -lo; the
#          block's d = max(scale_j)/63 and dmin = max(min_j)/63 are stored as
#          fp16, and sc_j, m_j are 6-bit roundings against them
#          (layout: csrc/libtinygiant.c:139-155, 210-222).
#   Q6_K : value ~= d*sc_j*(q - 32), q-32 in [-32,31]; per 16-value
#          sub-block scale_j = v/-32 with v its first largest-magnitude value;
#          d = max|scale_j|/127 (fp16), sc_j an int8 rounding
#          (layout: csrc/libtinygiant.c:382-401).
# All arithmetic is fp32 with round-to-nearest-even, so the bytes are a
# deterministic function of the weights.

def _f16_round(x):
    """fp32 -> nearest-even fp16 -> fp32 (the stored scale and its value)."""
    h = np.asarray(x, dtype=np.float32).astype(np.float16)
    return h, h.astype(np.float32)


def _chain(v, better, start=None):
    """Left fold over the last axis of v keeping `cur` while better(cur, next)
    holds, else taking `next` (so ties, +0 against -0 included, go to the later
    element): the fmin / fmax chains of the C fit."""
    cur = v[..., 0] if start is None else start
    for j in range(0 if start is not None else 1, v.shape[-1]):
        cur = np.where(better(cur, v[..., j]), cur, v[..., j])
    return cur.astype(np.float32)


def _rint_clip(v, lo, hi):
    return np.clip(np.rint(v), lo, hi).astype(np.int32)


def _pack_q4k_blocks(x):
    """x: fp32 [nb, 256] -> uint8 [nb, 144]."""
    nb = x.shape[0]
    xs = x.reshape(nb, 8, 32)
    lo, hi = _chain(xs, np.less), _chain(xs, np.greater)
    lo = np.where(lo > 0, np.float32(0), lo).astype(np.float32)
    scale = ((hi - lo) / np.float32(15)).astype(np.float32)
    minv = (-lo).astype(np.float32)
    max_scale = _chain(scale, np.greater, np.zeros(nb, np.float32))
    max_min = _chain(minv, np.greater, np.zeros(nb, np.float32))
    dh, d = _f16_round(max_scale / np.float32(63))
    mh, dmin = _f16_round(max_min / np.float32(63))
    with np.errstate(divide="ignore", invalid="ignore"):
        sc = np.where(d[:, None] > 0, _rint_clip(scale / d[:, None], 0, 63), 0).astype(np.int32)
        mn = np.where(dmin[:, None] > 0, _rint_clip(minv / dmin[:, None], 0, 63), 0).astype(np.int32)
        step = (d[:, None] * sc.astype(np.float32)).astype(np.float32)
        off = (dmin[:, None] * mn.astype(np.float32)).astype(np.float32)
        q = np.where(step[:, :, None] > 0,
                     _rint_clip((xs + off[:, :, None]) / step[:, :, None], 0, 15), 0).astype(np.uint8)
    out = np.zeros((nb, 144), np.uint8)
    out[:, 0:2] = dh.view(np.uint8).reshape(nb, 2)
    out[:, 2:4] = mh.view(np.uint8).reshape(nb, 2)
    s = np.zeros((nb, 12), np.int32)
    s[:, 0:4] = sc[:, 0:4] & 63
    s[:, 4:8] = mn[:, 0:4] & 63
    s[:, 8:12] = (sc[:, 4:8] & 0xF) | ((mn[:, 4:8] & 0xF) << 4)
    s[:, 0:4] |= (sc[:, 4:8] >> 4) << 6
    s[:, 4:8] |= (mn[:, 4:8] >> 4) << 6
    out[:, 4:16] = s.astype(np.uint8)
    q = q.reshape(nb, 4, 2, 32)
    out[:, 16:144] = (q[:, :, 0, :] | (q[:, :, 1, :] << 4)).reshape(nb, 128)
    return out


def _pack_q6k_blocks(x):
    nb = x.shape[0]
    xs = x.reshape(nb, 16, 16)
    idx = np.abs(xs).argmax(axis=2)
    v = np.take_along_axis(xs, idx[:, :, None], axis=2)[:, :, 0]
    scale = (v / np.float32(-32)).astype(np.float32)
    max_abs = _chain(np.abs(scale), np.greater, np.zeros(nb, np.float32))
    dh, d = _f16_round(max_abs / np.float32(127))
    with np.errstate(divide="ignore", invalid="ignore"):
        sc = np.where(d[:, None] > 0, _rint_clip(scale / d[:, None], -127, 127), 0).astype(np.int32)
        step = (d[:, None] * sc.astype(np.float32)).astype(np.float32)
        l = np.where(step[:, :, None] != 0, _rint_clip(xs / step[:, :, None], -32, 31), 0)
    q = (l + 32).astype(np.int32).reshape(nb, 2, 4, 32)   # [h][quarter][l]
    q1, q2, q3, q4 = q[:, :, 0], q[:, :, 1], q[:, :, 2], q[:, :, 3]
    out = np.zeros((nb, 210), np.uint8)
    ql = np.concatenate([(q1 & 15) | ((q3 & 15) << 4), (q2 & 15) | ((q4 & 15) << 4)], axis=2)  # [nb][2][64]
    out[:, 0:128] = ql.reshape(nb, 128).astype(np.uint8)
    qh = (q1 >> 4) | ((q2 >> 4) << 2) | ((q3 >> 4) << 4) | ((q4 >> 4) << 6)
    out[:, 128:192] = qh.reshape(nb, 64).astype(np.uint8)
    out[:, 192:208] = sc.astype(np.int8).view(np.uint8)
    out[:, 208:210] = dh.view(np.uint8).reshape(nb, 2)
    return out


def _pack(blocks_fn, fmt, w):
    w = np.ascontiguousarray(w, dtype=np.float32)
    if w.ndim != 2 or w.shape[1] % 256:
        raise ValueError("weights must be [rows, cols] with cols a multiple of 256")
    rows, cols = w.shape
    out = blocks_fn(w.reshape(-1, 256))
    assert out.nbytes == rows * row_bytes(fmt, cols)
    return out.reshape(-1)


def pack_q4k(w):
    """fp32 [rows, cols] -> Q4_K rows (144-byte blocks), uint8."""
    return _pack(_pack_q4k_blocks, FMT_Q4K, w)


def pack_q6k(w):
    """fp32 [rows, cols] -> Q6_K rows (210-byte blocks), uint8."""
    return _pack(_pack_q6k_blocks, FMT_Q6K, w)


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
