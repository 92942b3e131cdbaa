/*
 * tg_oracle.c — CPU restatement of TinyGiant's fused quantized MoE path.
 *
 * TEST INFRASTRUCTURE ONLY.  This file is the parity checker for the CUDA
 * library in tinygiant_b200/.  It is loaded by tests/, by
 * __graft_entry__.smoke() and by bench.py's cpu_baseline leg, and by nothing
 * on the product path.  It is pinned against the reference itself: the
 * reference's csrc/libtinygiant.c compiled unmodified through
 * oracle/neon_shim/arm_neon.h into oracle/_ref/libtinygiant_ref.so
 * (tests/test_oracle_golden.py), and against gguf-py's independent block
 * decoders (tests/golden/).
 *
 * Every function restates the reference algorithm in scalar C with the same
 * block layouts, the same integer sub-block sums and the same float
 * association order (build with -ffp-contract=off so a*b+c is never fused).
 * Citations are csrc/libtinygiant.c:line in andrew-the-drawer/tinygiant.
 *
 * Exports the hot-path subset of the reference C-ABI (same names, argument
 * lists and += semantics) plus tgo_* hooks that expose the internal Q8 blocks
 * and per-sub-block int32 dot sums for bit-exact comparison.
 */
#include <math.h>
#include <pthread.h>
#include <stdatomic.h>
#include <stdint.h>
#include <stdlib.h>
#include <string.h>

#define QK_K 256
#define Q4K_BSIZE 144
#define Q6K_BSIZE 210
#define MXFP4_BSIZE 17
#define Q80_BSIZE 34
#define MM_CHUNK 64
#define MOE_INTER_CHUNK 96
#define MOE_EMBED_CHUNK 256

enum { FMT_Q4K = 0, FMT_F16 = 1, FMT_Q6K = 2, FMT_MXFP4 = 3, FMT_Q80 = 4 };
enum { ACT_SILU = 0, ACT_GPTOSS = 1 };

/* 296-byte activation block (libtinygiant.c:159-164). */
typedef struct {
    float scale;
    int32_t sum;
    int32_t bsums[8];
    int8_t qs[QK_K];
} q8_block;

static inline int q8_nblocks(int n) { return (n + QK_K - 1) / QK_K; }

/* ------------------------------------------------------------------ */
/* Parallel-for over independent tasks (libtinygiant.c:26-124).  Each output
 * element is written by exactly one task, so results do not depend on the
 * thread count.  A tiny fork/join pool is enough for a checker.            */

typedef void (*task_fn)(void *ctx, size_t i);
static int g_threads = 1;

typedef struct {
    task_fn fn;
    void *ctx;
    size_t n;
    atomic_size_t next;
} pf_job;

static void *pf_worker(void *p) {
    pf_job *j = p;
    for (;;) {
        size_t i = atomic_fetch_add(&j->next, 1);
        if (i >= j->n) break;
        j->fn(j->ctx, i);
    }
    return NULL;
}

static void parallel_for(size_t n, task_fn fn, void *ctx) {
    if (g_threads <= 1 || n <= 1) {
        for (size_t i = 0; i < n; i++) fn(ctx, i);
        return;
    }
    pf_job job = { fn, ctx, n, 0 };
    int nw = g_threads - 1;
    pthread_t th[256];
    if (nw > 255) nw = 255;
    for (int t = 0; t < nw; t++) pthread_create(&th[t], NULL, pf_worker, &job);
    pf_worker(&job);
    for (int t = 0; t < nw; t++) pthread_join(th[t], NULL);
}

void tg_set_threads(int n) { g_threads = n < 1 ? 1 : n; }   /* libtinygiant.c:85-102 */
int tg_get_threads(void) { return g_threads; }              /* libtinygiant.c:104 */

/* ------------------------------------------------------------------ */
/* Scalar decoders. */

/* IEEE half -> float with subnormals (libtinygiant.c:128-137).  Restated bit
 * for bit, including the reference's handling of exponent 31 (inf/NaN): it
 * sets e = 255 and shifts (255 + 112) << 23, which wraps in uint32 and yields
 * a small negative finite value rather than inf/NaN.                        */
static inline float f16_to_f32(uint16_t h) {
    uint32_t s = (uint32_t)(h & 0x8000u) << 16, e = (h >> 10) & 0x1Fu, m = h & 0x3FFu;
    if (e == 0) {
        if (m == 0) { float r; memcpy(&r, &s, 4); return r; }
        while (!(m & 0x400u)) { m <<= 1; e--; }
        e++;
        m &= ~0x400u;
    } else if (e == 31) {
        e = 255;
    }
    uint32_t f = s | ((e + 112u) << 23) | (m << 13);
    float r; memcpy(&r, &f, 4); return r;
}

static inline uint16_t rd16(const uint8_t *p) { uint16_t v; memcpy(&v, p, 2); return v; }

/* 6-bit scale/min pair j of a Q4_K block's 12 scale bytes (libtinygiant.c:146-155). */
static inline void scale_min_k4(int j, const uint8_t *s, int *sc, int *m) {
    if (j < 4) {
        *sc = s[j] & 63;
        *m = s[j + 4] & 63;
    } else {
        *sc = (s[j + 4] & 0xF) | ((s[j - 4] >> 6) << 4);
        *m = (s[j + 4] >> 4) | ((s[j] >> 6) << 4);
    }
}

/* Doubled e2m1 code table and e8m0 -> 2^(e-128) (libtinygiant.c:514-519). */
static const int8_t kvalues_mxfp4[16] = { 0, 1, 2, 3, 4, 6, 8, 12, 0, -1, -2, -3, -4, -6, -8, -12 };
static inline float e8m0_half(uint8_t e) {
    uint32_t bits = e < 2 ? (0x00200000u << e) : ((uint32_t)(e - 1) << 23);
    float f; memcpy(&f, &bits, 4); return f;
}

/* ------------------------------------------------------------------ */
/* Q8 quantizer (libtinygiant.c:169-208): per 256-block amax, scale = amax/127,
 * inv = 127/amax (0 if amax == 0), q = round-half-even(x*inv), bsums per 32,
 * a partial last block zero-padded.                                         */

static inline int32_t round_half_even(float x) {
    /* x*inv lies in [-127.5, 127.5]; rintf under the default rounding mode is
     * round-to-nearest-even, matching FCVTNS, which also maps NaN to 0. */
    return x != x ? 0 : (int32_t)rintf(x);
}

static void quantize_q8(const float *x, q8_block *out, int ncols) {
    int nb = q8_nblocks(ncols);
    for (int b = 0; b < nb; b++) {
        const float *xb = x + (size_t)b * QK_K;
        int n = ncols - b * QK_K < QK_K ? ncols - b * QK_K : QK_K;
        float amax = 0.f;
        for (int i = 0; i < n; i++) {
            float a = fabsf(xb[i]);
            if (a != a || a > amax) amax = a;   /* FMAX keeps a NaN */
        }
        float sc = amax / 127.f;
        float inv = amax > 0 ? 127.f / amax : 0.f;
        out[b].scale = sc;
        int32_t total = 0;
        for (int j = 0; j < 8; j++) {
            int32_t s = 0;
            if (j * 32 < n) {
                for (int i = j * 32; i < (j + 1) * 32; i++) {
                    int32_t q = round_half_even(xb[i] * inv);
                    out[b].qs[i] = (int8_t)q;
                    s += q;
                }
            } else {
                memset(out[b].qs + j * 32, 0, 32);
            }
            out[b].bsums[j] = s;
            total += s;
        }
        out[b].sum = total;
    }
}

/* ------------------------------------------------------------------ */
/* Integer sub-block sums.  These are the exact int32 values the NEON code
 * forms with vdotq_s32 + vaddvq_s32; the GPU must reproduce them bit for bit. */

/* Q4_K block: 8 sums, sub-block 2g = low nibbles of qs[32g..32g+31] against
 * x[64g..64g+31], 2g+1 = high nibbles against x[64g+32..] (libtinygiant.c:243-261). */
static inline void q4k_isums(const uint8_t *bl, const int8_t *xq, int32_t out[8]) {
    const uint8_t *qs = bl + 16;
    for (int g = 0; g < 4; g++) {
        int32_t lo = 0, hi = 0;
        for (int j = 0; j < 32; j++) {
            uint8_t v = qs[32 * g + j];
            lo += (int32_t)(v & 0xF) * xq[64 * g + j];
            hi += (int32_t)(v >> 4) * xq[64 * g + 32 + j];
        }
        out[2 * g] = lo;
        out[2 * g + 1] = hi;
    }
}

/* Q6_K block: 16 sums of 16 values in the reference's visiting order
 * (half h, l-chunk c, quarter k) -> index (h*2 + c)*4 + k; the value at
 * position 128h + 32k + 16c + i has scale sc[8h + c + 2k] (libtinygiant.c:384-439). */
static inline int q6k_value(const uint8_t *bl, int h, int l, int k) {
    const uint8_t *ql = bl + 64 * h, *qh = bl + 128 + 32 * h;
    int v;
    switch (k) {
        case 0: v = (ql[l] & 0xF) | ((qh[l] & 3) << 4); break;
        case 1: v = (ql[l + 32] & 0xF) | (((qh[l] >> 2) & 3) << 4); break;
        case 2: v = (ql[l] >> 4) | (((qh[l] >> 4) & 3) << 4); break;
        default: v = (ql[l + 32] >> 4) | ((qh[l] >> 6) << 4); break;
    }
    return v - 32;
}

static inline void q6k_isums(const uint8_t *bl, const int8_t *xq, int32_t out[16]) {
    for (int h = 0; h < 2; h++)
        for (int c = 0; c < 2; c++)
            for (int k = 0; k < 4; k++) {
                int32_t s = 0;
                for (int i = 0; i < 16; i++) {
                    int l = 16 * c + i;
                    s += q6k_value(bl, h, l, k) * xq[128 * h + 32 * k + l];
                }
                out[(h * 2 + c) * 4 + k] = s;
            }
}

/* MXFP4 sub-block: low nibbles -> values 0..15, high -> 16..31 (libtinygiant.c:522-546). */
static inline int32_t mxfp4_isum(const uint8_t *bl, const int8_t *xq) {
    int32_t s = 0;
    for (int i = 0; i < 16; i++) {
        s += kvalues_mxfp4[bl[1 + i] & 0xF] * xq[i];
        s += kvalues_mxfp4[bl[1 + i] >> 4] * xq[16 + i];
    }
    return s;
}

/* Q8_0 sub-block (libtinygiant.c:576-590). */
static inline int32_t q80_isum(const uint8_t *bl, const int8_t *xq) {
    const int8_t *q = (const int8_t *)(bl + 2);
    int32_t s = 0;
    for (int i = 0; i < 32; i++) s += q[i] * xq[i];
    return s;
}

/* ------------------------------------------------------------------ */
/* Row dot products with the reference's float association. */

/* One row, one input (libtinygiant.c:223-272). */
static float dot_q4k(const uint8_t *row, const q8_block *xq, int bpr) {
    float total = 0;
    for (int b = 0; b < bpr; b++) {
        const uint8_t *bl = row + (size_t)b * Q4K_BSIZE;
        float d = f16_to_f32(rd16(bl)), dmin = f16_to_f32(rd16(bl + 2));
        int32_t is[8];
        q4k_isums(bl, xq[b].qs, is);
        float bs = 0;
        for (int g = 0; g < 4; g++) {
            int sl, ml, sh, mh;
            scale_min_k4(2 * g, bl + 4, &sl, &ml);
            scale_min_k4(2 * g + 1, bl + 4, &sh, &mh);
            bs += d * (float)sl * (float)is[2 * g] - dmin * (float)ml * (float)xq[b].bsums[2 * g];
            bs += d * (float)sh * (float)is[2 * g + 1] - dmin * (float)mh * (float)xq[b].bsums[2 * g + 1];
        }
        total += xq[b].scale * bs;
    }
    return total;
}

/* One row against four inputs: the per-group terms are summed before being
 * added to the block sum (libtinygiant.c:276-337). */
static void dot_q4k_x4(const uint8_t *row, const q8_block *const xq[4], int bpr, float out[4]) {
    float tot[4] = { 0, 0, 0, 0 };
    for (int b = 0; b < bpr; b++) {
        const uint8_t *bl = row + (size_t)b * Q4K_BSIZE;
        float d = f16_to_f32(rd16(bl)), dmin = f16_to_f32(rd16(bl + 2));
        float bs[4] = { 0, 0, 0, 0 };
        int32_t is[4][8];
        for (int r = 0; r < 4; r++) q4k_isums(bl, xq[r][b].qs, is[r]);
        for (int g = 0; g < 4; g++) {
            int sl, ml, sh, mh;
            scale_min_k4(2 * g, bl + 4, &sl, &ml);
            scale_min_k4(2 * g + 1, bl + 4, &sh, &mh);
            float dsl = d * (float)sl, dml = dmin * (float)ml;
            float dsh = d * (float)sh, dmh = dmin * (float)mh;
            for (int r = 0; r < 4; r++)
                bs[r] += dsl * (float)is[r][2 * g] - dml * (float)xq[r][b].bsums[2 * g]
                       + dsh * (float)is[r][2 * g + 1] - dmh * (float)xq[r][b].bsums[2 * g + 1];
        }
        for (int r = 0; r < 4; r++) tot[r] += xq[r][b].scale * bs[r];
    }
    for (int r = 0; r < 4; r++) out[r] = tot[r];
}

/* Q6_K, identical association for x1 and x4 (libtinygiant.c:403-487). */
static float dot_q6k(const uint8_t *row, const q8_block *xq, int bpr) {
    float total = 0;
    for (int b = 0; b < bpr; b++) {
        const uint8_t *bl = row + (size_t)b * Q6K_BSIZE;
        const int8_t *sc = (const int8_t *)(bl + 192);
        float d = f16_to_f32(rd16(bl + 208));
        int32_t is[16];
        q6k_isums(bl, xq[b].qs, is);
        float bs = 0;
        for (int h = 0; h < 2; h++)
            for (int c = 0; c < 2; c++)
                for (int k = 0; k < 4; k++)
                    bs += (float)sc[8 * h + c + 2 * k] * (float)is[(h * 2 + c) * 4 + k];
        total += d * xq[b].scale * bs;
    }
    return total;
}

/* MXFP4 over ncols (a multiple of 32): sub-block s pairs with Q8 block s/8
 * at offset (s%8)*32 (libtinygiant.c:533-570; x1 and x4 associate alike). */
static float dot_mxfp4(const uint8_t *row, const q8_block *xq, int ncols) {
    float total = 0;
    for (int s = 0; s < ncols / 32; s++) {
        const q8_block *xb = &xq[s >> 3];
        const uint8_t *bl = row + (size_t)s * MXFP4_BSIZE;
        total += xb->scale * e8m0_half(bl[0]) * (float)mxfp4_isum(bl, xb->qs + (s & 7) * 32);
    }
    return total;
}

static float dot_q80(const uint8_t *row, const q8_block *xq, int ncols) {
    float total = 0;
    for (int s = 0; s < ncols / 32; s++) {
        const q8_block *xb = &xq[s >> 3];
        const uint8_t *bl = row + (size_t)s * Q80_BSIZE;
        total += xb->scale * f16_to_f32(rd16(bl)) * (float)q80_isum(bl, xb->qs + (s & 7) * 32);
    }
    return total;
}

/* Exact IEEE half -> float, as the vcvt_f32_f16 instruction converts
 * (inf and NaN included). */
static inline float half_ieee(uint16_t h) {
    uint32_t s = (uint32_t)(h & 0x8000u) << 16, e = (h >> 10) & 0x1Fu, m = h & 0x3FFu, bits;
    if (e == 0) {
        if (m == 0) bits = s;
        else {
            int k = -1;
            do { m <<= 1; k++; } while (!(m & 0x400u));
            bits = s | ((uint32_t)(112 - k) << 23) | ((m & 0x3FFu) << 13);
        }
    } else if (e == 31) {
        bits = s | 0x7F800000u | (m << 13);
    } else {
        bits = s | ((e + 112u) << 23) | (m << 13);
    }
    float f; memcpy(&f, &bits, 4); return f;
}

/* f16 row with two 4-lane fused accumulators over 8-value steps (vector
 * conversion), pairwise lane reduction, then a scalar tail through
 * f16_to_f32 (libtinygiant.c:635-653). */
static float dot_f16(const uint16_t *row, const float *x, int ncols) {
    float a0[4] = { 0, 0, 0, 0 }, a1[4] = { 0, 0, 0, 0 };
    int i = 0;
    for (; i + 7 < ncols; i += 8)
        for (int l = 0; l < 4; l++) {
            a0[l] = fmaf(half_ieee(row[i + l]), x[i + l], a0[l]);
            a1[l] = fmaf(half_ieee(row[i + 4 + l]), x[i + 4 + l], a1[l]);
        }
    float s[4];
    for (int l = 0; l < 4; l++) s[l] = a0[l] + a1[l];
    float sum = (s[0] + s[1]) + (s[2] + s[3]);
    for (; i < ncols; i++) sum += f16_to_f32(row[i]) * x[i];
    return sum;
}

static void matvec_f16(const uint16_t *A, const float *x, float *out, int nrows, int ncols) {
    for (int r = 0; r < nrows; r++) out[r] = dot_f16(A + (size_t)r * ncols, x, ncols);
}

/* ------------------------------------------------------------------ */
/* Format dispatch (libtinygiant.c:594-631). */

static size_t row_bytes(int fmt, int ncols) {
    switch (fmt) {
        case FMT_Q4K: return (size_t)(ncols / QK_K) * Q4K_BSIZE;
        case FMT_Q6K: return (size_t)(ncols / QK_K) * Q6K_BSIZE;
        case FMT_MXFP4: return (size_t)(ncols / 32) * MXFP4_BSIZE;
        case FMT_Q80: return (size_t)(ncols / 32) * Q80_BSIZE;
        default: return (size_t)ncols * 2;
    }
}

size_t tg_row_bytes(int fmt, int ncols) { return row_bytes(fmt, ncols); }

static float dot_fmt(int fmt, const uint8_t *row, const q8_block *xq, const float *xf, int ncols) {
    switch (fmt) {
        case FMT_Q4K: return dot_q4k(row, xq, ncols / QK_K);
        case FMT_Q6K: return dot_q6k(row, xq, ncols / QK_K);
        case FMT_MXFP4: return dot_mxfp4(row, xq, ncols);
        case FMT_Q80: return dot_q80(row, xq, ncols);
        default: return dot_f16((const uint16_t *)row, xf, ncols);
    }
}

static void dot_fmt_x4(int fmt, const uint8_t *row, const q8_block *const xq[4], const float *const xf[4],
                       int ncols, float out[4]) {
    if (fmt == FMT_Q4K) { dot_q4k_x4(row, xq, ncols / QK_K, out); return; }
    for (int r = 0; r < 4; r++) out[r] = dot_fmt(fmt, row, xq[r], xf ? xf[r] : NULL, ncols);
}

/* ------------------------------------------------------------------ */
/* Matvecs (libtinygiant.c:341-378, 489-501, 906-931). */

typedef struct {
    int fmt;
    const uint8_t *mat;
    const q8_block *xq;
    const float *x;
    const float *bias;
    float *out;
    int nrows, ncols;
    int bias_term;   /* 1: add `bias ? bias[r] : 0.f` as qkv_rows does */
} mm_ctx;

static void mm_task(void *p, size_t i) {
    mm_ctx *c = p;
    int r0 = (int)i * MM_CHUNK, r1 = r0 + MM_CHUNK < c->nrows ? r0 + MM_CHUNK : c->nrows;
    size_t rb = row_bytes(c->fmt, c->ncols);
    for (int r = r0; r < r1; r++) {
        float v = dot_fmt(c->fmt, c->mat + (size_t)r * rb, c->xq, c->x, c->ncols);
        c->out[r] = c->bias_term ? v + (c->bias ? c->bias[r] : 0.f) : v;
    }
}

/* matmul_q4k / matmul_q6k: quantize once, 64-row tasks, no bias term
 * (libtinygiant.c:353-373, 489-496). */
static void matmul_fmt(int fmt, const uint8_t *mat, const float *x, float *out, int nrows, int ncols) {
    q8_block *xq = malloc(sizeof(q8_block) * (size_t)q8_nblocks(ncols));
    quantize_q8(x, xq, ncols);
    mm_ctx c = { fmt, mat, xq, x, NULL, out, nrows, ncols, 0 };
    parallel_for((size_t)(nrows + MM_CHUNK - 1) / MM_CHUNK, mm_task, &c);
    free(xq);
}

void tg_matmul_q4k(const uint8_t *m, const float *x, float *out, int nrows, int ncols) {
    matmul_fmt(FMT_Q4K, m, x, out, nrows, ncols);
}
void tg_matmul_q6k(const uint8_t *m, const float *x, float *out, int nrows, int ncols) {
    matmul_fmt(FMT_Q6K, m, x, out, nrows, ncols);
}
/* Generic matvec: every row gets `+ (bias ? bias[r] : 0.f)` (qkv_rows,
 * libtinygiant.c:829-834, 918-931). */
void tg_matmul(int fmt, const void *mat, const float *bias, const float *x, float *out, int nrows, int ncols) {
    q8_block *xq = malloc(sizeof(q8_block) * (size_t)q8_nblocks(ncols));
    if (fmt != FMT_F16) quantize_q8(x, xq, ncols);
    mm_ctx c = { fmt, mat, xq, x, bias, out, nrows, ncols, 1 };
    parallel_for((size_t)(nrows + MM_CHUNK - 1) / MM_CHUNK, mm_task, &c);
    free(xq);
}

void tg_f16_matvec(const uint16_t *A, const float *x, float *out, int nrows, int ncols) {
    matvec_f16(A, x, out, nrows, ncols);
}

/* f32 matvec with fused lanes (libtinygiant.c:662-676). */
void tg_f32_matvec(const float *A, const float *x, float *out, int nrows, int ncols) {
    for (int r = 0; r < nrows; r++) {
        const float *row = A + (size_t)r * ncols;
        float a0[4] = { 0, 0, 0, 0 }, a1[4] = { 0, 0, 0, 0 };
        int i = 0;
        for (; i + 7 < ncols; i += 8)
            for (int l = 0; l < 4; l++) {
                a0[l] = fmaf(row[i + l], x[i + l], a0[l]);
                a1[l] = fmaf(row[i + 4 + l], x[i + 4 + l], a1[l]);
            }
        float s[4];
        for (int l = 0; l < 4; l++) s[l] = a0[l] + a1[l];
        float sum = (s[0] + s[1]) + (s[2] + s[3]);
        for (; i < ncols; i++) sum += row[i] * x[i];
        out[r] = sum;
    }
}

/* RMSNorm with 4 fused lanes (libtinygiant.c:680-698). */
void tg_rms_norm(const float *x, const float *w, float *out, int dim, float eps) {
    float a[4] = { 0, 0, 0, 0 };
    int i = 0;
    for (; i + 3 < dim; i += 4)
        for (int l = 0; l < 4; l++) a[l] = fmaf(x[i + l], x[i + l], a[l]);
    float ss = (a[0] + a[1]) + (a[2] + a[3]);
    for (; i < dim; i++) ss += x[i] * x[i];
    float scale = 1.f / sqrtf(ss / dim + eps);
    for (i = 0; i < dim; i++) out[i] = x[i] * scale * w[i];
}

/* ------------------------------------------------------------------ */
/* Single-expert forwards (libtinygiant.c:1040-1231). */

static inline float silu_mul(float g, float u) { return g / (1.f + expf(-g)) * u; }

void tg_expert_forward(const uint8_t *q4, const float *x, float *out, float w, int D, int I) {
    int gbpr = D / QK_K, dbpr = I / QK_K;
    size_t gbytes = (size_t)I * gbpr * Q4K_BSIZE;
    const uint8_t *gate = q4, *up = q4 + gbytes, *down = q4 + 2 * gbytes;
    q8_block *xe = malloc(sizeof(q8_block) * gbpr), *xi = malloc(sizeof(q8_block) * dbpr);
    float *g = malloc(sizeof(float) * I), *u = malloc(sizeof(float) * I), *h = malloc(sizeof(float) * I);
    float *dn = malloc(sizeof(float) * D);
    quantize_q8(x, xe, D);
    for (int r = 0; r < I; r++) g[r] = dot_q4k(gate + (size_t)r * gbpr * Q4K_BSIZE, xe, gbpr);
    for (int r = 0; r < I; r++) u[r] = dot_q4k(up + (size_t)r * gbpr * Q4K_BSIZE, xe, gbpr);
    for (int i = 0; i < I; i++) h[i] = silu_mul(g[i], u[i]);
    quantize_q8(h, xi, I);
    for (int r = 0; r < D; r++) dn[r] = dot_q4k(down + (size_t)r * dbpr * Q4K_BSIZE, xi, dbpr);
    for (int i = 0; i < D; i++) out[i] += w * dn[i];
    free(xe); free(xi); free(g); free(u); free(h); free(dn);
}

/* Mixed down format: 1 = f16, 2 = Q6_K (through the Q6_K matvec), else Q4_K
 * (libtinygiant.c:1084-1128). */
void tg_expert_forward_mixed(const uint8_t *gq, const uint8_t *uq, const void *down, int dfmt,
                             const float *x, float *out, float w, int D, int I) {
    int gbpr = D / QK_K, dbpr = I / QK_K;
    q8_block *xe = malloc(sizeof(q8_block) * gbpr), *xi = malloc(sizeof(q8_block) * (dbpr + 1));
    float *g = malloc(sizeof(float) * I), *u = malloc(sizeof(float) * I), *h = malloc(sizeof(float) * I);
    float *dn = malloc(sizeof(float) * D);
    quantize_q8(x, xe, D);
    for (int r = 0; r < I; r++) g[r] = dot_q4k(gq + (size_t)r * gbpr * Q4K_BSIZE, xe, gbpr);
    for (int r = 0; r < I; r++) u[r] = dot_q4k(uq + (size_t)r * gbpr * Q4K_BSIZE, xe, gbpr);
    for (int i = 0; i < I; i++) h[i] = silu_mul(g[i], u[i]);
    if (dfmt == 1) {
        matvec_f16(down, h, dn, D, I);
    } else if (dfmt == 2) {
        matmul_fmt(FMT_Q6K, down, h, dn, D, I);
    } else {
        quantize_q8(h, xi, I);
        for (int r = 0; r < D; r++) dn[r] = dot_q4k((const uint8_t *)down + (size_t)r * dbpr * Q4K_BSIZE, xi, dbpr);
    }
    for (int i = 0; i < D; i++) out[i] += w * dn[i];
    free(xe); free(xi); free(g); free(u); free(h); free(dn);
}

/* Rows in groups of 4 via the x4 kernel whenever k > 1, padding the last
 * group with the last row; x1 only when k == 1 (libtinygiant.c:1136-1180). */
static void fmt_rows(int fmt, const uint8_t *mat, int nrows, int ncols, const q8_block *xq, int k,
                     int xq_stride, float *out, int out_stride) {
    size_t rb = row_bytes(fmt, ncols);
    if (k == 1) {
        for (int row = 0; row < nrows; row++) out[row] = dot_fmt(fmt, mat + (size_t)row * rb, xq, NULL, ncols);
        return;
    }
    for (int r0 = 0; r0 < k; r0 += 4) {
        const q8_block *p[4];
        for (int r = 0; r < 4; r++) p[r] = xq + (size_t)(r0 + r < k ? r0 + r : k - 1) * xq_stride;
        int n = k - r0 < 4 ? k - r0 : 4;
        for (int row = 0; row < nrows; row++) {
            float o[4];
            dot_fmt_x4(fmt, mat + (size_t)row * rb, p, NULL, ncols, o);
            for (int r = 0; r < n; r++) out[(size_t)(r0 + r) * out_stride + row] = o[r];
        }
    }
}

void tg_expert_forward_rows(const uint8_t *gq, const uint8_t *uq, const void *down, int dfmt,
                            const float *xs, float *out, const float *wts, int k, int D, int I) {
    int gbpr = D / QK_K, dbpr = I / QK_K;
    q8_block *xe = malloc(sizeof(q8_block) * (size_t)gbpr * k);
    float *g = malloc(sizeof(float) * (size_t)I * k), *u = malloc(sizeof(float) * (size_t)I * k);
    float *dn = malloc(sizeof(float) * (size_t)D * k);
    for (int r = 0; r < k; r++) quantize_q8(xs + (size_t)r * D, xe + (size_t)r * gbpr, D);
    fmt_rows(FMT_Q4K, gq, I, D, xe, k, gbpr, g, I);
    fmt_rows(FMT_Q4K, uq, I, D, xe, k, gbpr, u, I);
    for (size_t i = 0; i < (size_t)I * k; i++) g[i] = silu_mul(g[i], u[i]);
    if (dfmt == 1) {
        for (int r = 0; r < k; r++) matvec_f16(down, g + (size_t)r * I, dn + (size_t)r * D, D, I);
    } else {
        q8_block *xi = malloc(sizeof(q8_block) * (size_t)dbpr * k);
        for (int r = 0; r < k; r++) quantize_q8(g + (size_t)r * I, xi + (size_t)r * dbpr, I);
        fmt_rows(dfmt == 2 ? FMT_Q6K : FMT_Q4K, down, D, I, xi, k, dbpr, dn, D);
        free(xi);
    }
    for (int r = 0; r < k; r++)
        for (int i = 0; i < D; i++) out[(size_t)r * D + i] += wts[r] * dn[(size_t)r * D + i];
    free(xe); free(g); free(u); free(dn);
}

/* ------------------------------------------------------------------ */
/* Batched MoE layer (libtinygiant.c:1245-1448). */

static inline float act_fn(int act, float g, float u) {
    if (act == ACT_GPTOSS) {
        if (g > 7.f) g = 7.f;
        if (u > 7.f) u = 7.f; else if (u < -7.f) u = -7.f;
        return g / (1.f + expf(-1.702f * g)) * (u + 1.f);
    }
    return g / (1.f + expf(-g)) * u;
}

typedef struct {
    const uint8_t *const *gate;
    const uint8_t *const *up;
    const void *const *down;
    int gate_fmt;
    const int *down_fmts;
    const float *const *gb, *const *ub, *const *db;
    int act, n_exp, k, D, I, gbpr, dbpr;
    int *n_rows, *rows;
    float *wts;
    q8_block *xq_in;
    float *hidden, *partials;
    int n_ic, n_ec;
} moe_ctx;

/* Phase A task (expert, 96-row chunk of I): active rows in groups of 4, x1
 * when a group holds one row, else x4 (libtinygiant.c:1279-1327). */
static void moe_phase_a(void *p, size_t task) {
    moe_ctx *c = p;
    int e = (int)(task / c->n_ic), ch = (int)(task % c->n_ic), n = c->n_rows[e];
    if (n == 0) return;
    int r0 = ch * MOE_INTER_CHUNK, r1 = r0 + MOE_INTER_CHUNK < c->I ? r0 + MOE_INTER_CHUNK : c->I;
    int fmt = c->gate_fmt;
    size_t grow = row_bytes(fmt, c->D);
    const uint8_t *gate = c->gate[e] + r0 * grow, *up = c->up[e] + r0 * grow;
    const q8_block *xq = c->xq_in + (size_t)e * c->k * c->gbpr;
    const float *gb = c->gb ? c->gb[e] : NULL, *ub = c->ub ? c->ub[e] : NULL;
    float *hid = c->hidden + (size_t)e * c->k * c->I;
    float g[MOE_INTER_CHUNK * 4], u[MOE_INTER_CHUNK * 4];
    for (int b = 0; b < n; b += 4) {
        int m = n - b < 4 ? n - b : 4;
        if (m == 1) {
            const q8_block *x = xq + (size_t)b * c->gbpr;
            float *h = hid + (size_t)b * c->I;
            for (int r = r0; r < r1; r++) {
                float gv = dot_fmt(fmt, gate + (size_t)(r - r0) * grow, x, NULL, c->D);
                float uv = dot_fmt(fmt, up + (size_t)(r - r0) * grow, x, NULL, c->D);
                if (gb) { gv += gb[r]; uv += ub[r]; }
                h[r] = act_fn(c->act, gv, uv);
            }
            continue;
        }
        const q8_block *px[4];
        for (int j = 0; j < 4; j++) px[j] = xq + (size_t)(b + (j < m ? j : m - 1)) * c->gbpr;
        for (int r = r0; r < r1; r++) {
            dot_fmt_x4(fmt, gate + (size_t)(r - r0) * grow, px, NULL, c->D, g + (r - r0) * 4);
            dot_fmt_x4(fmt, up + (size_t)(r - r0) * grow, px, NULL, c->D, u + (r - r0) * 4);
        }
        for (int j = 0; j < m; j++) {
            float *h = hid + (size_t)(b + j) * c->I;
            for (int r = r0; r < r1; r++) {
                float gv = g[(r - r0) * 4 + j], uv = u[(r - r0) * 4 + j];
                if (gb) { gv += gb[r]; uv += ub[r]; }
                h[r] = act_fn(c->act, gv, uv);
            }
        }
    }
}

/* Phase B task (expert, 256-row chunk of D): re-quantize the hidden rows,
 * partial = wt * (down.h + bias) (libtinygiant.c:1329-1384). */
static void moe_phase_b(void *p, size_t task) {
    moe_ctx *c = p;
    int e = (int)(task / c->n_ec), ch = (int)(task % c->n_ec), n = c->n_rows[e];
    if (n == 0) return;
    int r0 = ch * MOE_EMBED_CHUNK, r1 = r0 + MOE_EMBED_CHUNK < c->D ? r0 + MOE_EMBED_CHUNK : c->D;
    const float *hid = c->hidden + (size_t)e * c->k * c->I;
    float *part = c->partials + (size_t)e * c->k * c->D;
    const float *wt = c->wts + (size_t)e * c->k;
    const float *db = c->db ? c->db[e] : NULL;
    int fmt = c->down_fmts[e], I = c->I;
    if (fmt == FMT_F16) {
        const uint16_t *w = c->down[e];
        for (int j = 0; j < n; j++)
            matvec_f16(w + (size_t)r0 * I, hid + (size_t)j * I, part + (size_t)j * c->D + r0, r1 - r0, I);
        for (int j = 0; j < n; j++)
            for (int r = r0; r < r1; r++)
                part[(size_t)j * c->D + r] = wt[j] * (part[(size_t)j * c->D + r] + (db ? db[r] : 0.f));
        return;
    }
    size_t rb = row_bytes(fmt, I);
    const uint8_t *mat = (const uint8_t *)c->down[e] + r0 * rb;
    q8_block *xq = malloc(sizeof(q8_block) * (size_t)n * c->dbpr);
    for (int j = 0; j < n; j++) quantize_q8(hid + (size_t)j * I, xq + (size_t)j * c->dbpr, I);
    for (int b = 0; b < n; b += 4) {
        int m = n - b < 4 ? n - b : 4;
        if (m == 1) {
            const q8_block *x = xq + (size_t)b * c->dbpr;
            float *o = part + (size_t)b * c->D;
            for (int r = r0; r < r1; r++) {
                float v = dot_fmt(fmt, mat + (size_t)(r - r0) * rb, x, NULL, I);
                o[r] = wt[b] * (v + (db ? db[r] : 0.f));
            }
            continue;
        }
        const q8_block *px[4];
        for (int j = 0; j < 4; j++) px[j] = xq + (size_t)(b + (j < m ? j : m - 1)) * c->dbpr;
        for (int r = r0; r < r1; r++) {
            float o[4];
            dot_fmt_x4(fmt, mat + (size_t)(r - r0) * rb, px, NULL, I, o);
            float bias = db ? db[r] : 0.f;
            for (int j = 0; j < m; j++) part[(size_t)(b + j) * c->D + r] = wt[b + j] * (o[j] + bias);
        }
    }
    free(xq);
}

/* Gather active rows per expert, phase A, phase B, then a serial combine in
 * the given expert order into the accumulated output (libtinygiant.c:1386-1437). */
void tg_moe_forward_rows_v2(const uint8_t *const *gate, const uint8_t *const *up, const void *const *down,
                            int gate_fmt, const int *down_fmts, const float *const *gb, const float *const *ub,
                            const float *const *db, int act, int n_exp, const float *row_w, const float *xs,
                            float *out, int k, int D, int I) {
    int gbpr = q8_nblocks(D), dbpr = q8_nblocks(I);
    moe_ctx c = { gate, up, down, gate_fmt, down_fmts, gb, ub, db, act, n_exp, k, D, I, gbpr, dbpr };
    c.n_rows = calloc((size_t)n_exp, sizeof(int));
    c.rows = malloc(sizeof(int) * (size_t)n_exp * k);
    c.wts = malloc(sizeof(float) * (size_t)n_exp * k);
    c.xq_in = malloc(sizeof(q8_block) * (size_t)n_exp * k * gbpr);
    c.hidden = malloc(sizeof(float) * (size_t)n_exp * k * I);
    c.partials = calloc((size_t)n_exp * k * D, sizeof(float));
    c.n_ic = (I + MOE_INTER_CHUNK - 1) / MOE_INTER_CHUNK;
    c.n_ec = (D + MOE_EMBED_CHUNK - 1) / MOE_EMBED_CHUNK;
    q8_block *xr = malloc(sizeof(q8_block) * (size_t)k * gbpr);
    for (int r = 0; r < k; r++) quantize_q8(xs + (size_t)r * D, xr + (size_t)r * gbpr, D);
    for (int e = 0; e < n_exp; e++) {
        const float *w = row_w + (size_t)e * k;
        int n = 0;
        for (int r = 0; r < k; r++) {
            if (w[r] == 0.f) continue;
            c.rows[e * k + n] = r;
            c.wts[e * k + n] = w[r];
            memcpy(c.xq_in + ((size_t)e * k + n) * gbpr, xr + (size_t)r * gbpr, sizeof(q8_block) * gbpr);
            n++;
        }
        c.n_rows[e] = n;
    }
    parallel_for((size_t)n_exp * c.n_ic, moe_phase_a, &c);
    parallel_for((size_t)n_exp * c.n_ec, moe_phase_b, &c);
    for (int e = 0; e < n_exp; e++)
        for (int j = 0; j < c.n_rows[e]; j++) {
            float *o = out + (size_t)c.rows[e * k + j] * D;
            const float *p = c.partials + ((size_t)e * k + j) * D;
            for (int i = 0; i < D; i++) o[i] += p[i];
        }
    free(xr); free(c.n_rows); free(c.rows); free(c.wts); free(c.xq_in); free(c.hidden); free(c.partials);
}

void tg_moe_forward_rows(const uint8_t *const *gate, const uint8_t *const *up, const void *const *down,
                         const int *down_fmts, int n_exp, const float *row_w, const float *xs, float *out,
                         int k, int D, int I) {
    tg_moe_forward_rows_v2(gate, up, down, FMT_Q4K, down_fmts, NULL, NULL, NULL, ACT_SILU, n_exp, row_w, xs,
                           out, k, D, I);
}

/* Zeroes the output, then runs each all-Q4_K expert (libtinygiant.c:1452-1460). */
void tg_moe_forward(const uint8_t **experts, const float *weights, int n_exp, const float *x, float *out,
                    int D, int I) {
    memset(out, 0, (size_t)D * sizeof(float));
    for (int e = 0; e < n_exp; e++) tg_expert_forward(experts[e], x, out, weights[e], D, I);
}

/* ------------------------------------------------------------------ */
/* Test hooks (no counterpart in the reference ABI). */

size_t tgo_q8_block_bytes(void) { return sizeof(q8_block); }

/* Quantizes ncols floats into q8_nblocks(ncols) 296-byte blocks. */
void tgo_quantize_q8(const float *x, void *out, int ncols) { quantize_q8(x, out, ncols); }

/* Per-sub-block int32 sums of one row against Q8 blocks:
 * Q4_K: 8 per 256-block, Q6_K: 16 per 256-block (visiting order above),
 * MXFP4 / Q8_0: 1 per 32 values.  Returns the number written. */
int tgo_row_isums(int fmt, const uint8_t *row, const void *xq_, int ncols, int32_t *out) {
    const q8_block *xq = xq_;
    int n = 0;
    if (fmt == FMT_Q4K) {
        for (int b = 0; b < ncols / QK_K; b++, n += 8) q4k_isums(row + (size_t)b * Q4K_BSIZE, xq[b].qs, out + n);
    } else if (fmt == FMT_Q6K) {
        for (int b = 0; b < ncols / QK_K; b++, n += 16) q6k_isums(row + (size_t)b * Q6K_BSIZE, xq[b].qs, out + n);
    } else if (fmt == FMT_MXFP4) {
        for (int s = 0; s < ncols / 32; s++)
            out[n++] = mxfp4_isum(row + (size_t)s * MXFP4_BSIZE, xq[s >> 3].qs + (s & 7) * 32);
    } else if (fmt == FMT_Q80) {
        for (int s = 0; s < ncols / 32; s++)
            out[n++] = q80_isum(row + (size_t)s * Q80_BSIZE, xq[s >> 3].qs + (s & 7) * 32);
    }
    return n;
}

/* Row dot with the x1 association (mode 0) or the x4 association (mode 1),
 * against already-quantized inputs. */
void tgo_rows_dot(int fmt, const uint8_t *mat, int nrows, int ncols, const void *xq_, int k, int mode, float *out) {
    const q8_block *xq = xq_;
    int bpr = q8_nblocks(ncols);
    size_t rb = row_bytes(fmt, ncols);
    for (int r = 0; r < nrows; r++) {
        const uint8_t *row = mat + (size_t)r * rb;
        if (mode == 0) {
            for (int t = 0; t < k; t++) out[(size_t)t * nrows + r] = dot_fmt(fmt, row, xq + (size_t)t * bpr, NULL, ncols);
        } else {
            for (int t0 = 0; t0 < k; t0 += 4) {
                const q8_block *p[4];
                for (int j = 0; j < 4; j++) p[j] = xq + (size_t)(t0 + j < k ? t0 + j : k - 1) * bpr;
                float o[4];
                dot_fmt_x4(fmt, row, p, NULL, ncols, o);
                for (int j = 0; j < 4 && t0 + j < k; j++) out[(size_t)(t0 + j) * nrows + r] = o[j];
            }
        }
    }
}

float tgo_act(int act, float g, float u) { return act_fn(act, g, u); }
