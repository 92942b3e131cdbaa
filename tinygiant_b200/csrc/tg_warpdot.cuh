// tg_warpdot.cuh — warp-level exact row dots of the quantized formats and the
// per-row staging helpers shared by the expert kernels (tg_moe.cu) and the
// fused layer step (tg_step.cu).
//
// A row dot is spread over the lanes of one warp (Q4_K: 4 lanes per
// 256-block, one per 64-value group; Q6_K: 8 lanes per block; MXFP4 / Q8_0:
// one lane per 32-value block).  Integer sums are exact (dp4a); the float
// terms are formed and folded in the reference's association and order
// (csrc/libtinygiant.c, see tg_dots.cuh), so each fp32 row result equals the
// reference's bit for bit.
#pragma once
#include "tg_dots.cuh"
#include "tg_ptx.cuh"

namespace tg {

constexpr unsigned FULL = 0xffffffffu;

// ---------------------------------------------------------------------
// Staging.  Rows r .. r + nr - 1 of a matrix are one contiguous byte range
// (WDesc row layout); it is moved by one bulk copy of its 16-byte-aligned
// window.  Every allocation holding weights is padded by at least 16 bytes,
// so the window stays inside it.

// Stage bytes reserved for nr rows of stride rs.
__host__ __device__ __forceinline__ uint32_t rows_stage_bytes(int rs, int nr) {
  return round16((size_t)nr * rs) + 16u;
}

struct RowPtrs {
  const uint8_t* m;
  const uint8_t* a1;
  const uint8_t* a2;
};

__device__ __forceinline__ const uint8_t* win_start(const uint8_t* p) {
  return reinterpret_cast<const uint8_t*>(reinterpret_cast<uintptr_t>(p) & ~(uintptr_t)15);
}
__device__ __forceinline__ uint32_t win_bytes(const uint8_t* p, uint32_t len) {
  const uintptr_t a = reinterpret_cast<uintptr_t>(p);
  return (uint32_t)(((a + len + 15) & ~(uintptr_t)15) - (a & ~(uintptr_t)15));
}

// Row r of W in global memory.
__device__ __forceinline__ RowPtrs row_src(const WDesc& W, int r) {
  const size_t o = (size_t)r * W.rs;
  RowPtrs p;
  p.m = W.main + o;
  p.a1 = W.aux1 ? W.aux1 + o : nullptr;
  p.a2 = W.aux2 ? W.aux2 + o : nullptr;
  return p;
}

// Row r of W as staged at dst by stage_row (rows after it follow at W.rs
// bytes each), or in global memory when dst is null.
__device__ __forceinline__ RowPtrs row_ptrs(const WDesc& W, int r, const uint8_t* dst) {
  RowPtrs p = row_src(W, r);
  if (!dst) return p;
  const uint8_t* m = dst + (reinterpret_cast<uintptr_t>(p.m) & 15);
  if (p.a1) p.a1 = m + (W.aux1 - W.main);
  if (p.a2) p.a2 = m + (W.aux2 - W.main);
  p.m = m;
  return p;
}

__device__ __forceinline__ uint32_t row_tx(const WDesc& W, int r, int nr = 1) {
  return win_bytes(W.main + (size_t)r * W.rs, (uint32_t)nr * W.rs);
}

// One lane: bulk-copies the window of rows r .. r + nr - 1 of W to dst.
__device__ __forceinline__ void stage_row(const WDesc& W, int r, uint8_t* dst, uint64_t* bar, int nr = 1) {
  const uint8_t* p = W.main + (size_t)r * W.rs;
  bulk_g2s(dst, win_start(p), win_bytes(p, (uint32_t)nr * W.rs), bar);
}

// Orders this thread's earlier shared-memory reads before a later bulk copy
// into the same bytes.
__device__ __forceinline__ void fence_proxy_async() { asm volatile("fence.proxy.async.shared::cta;" ::: "memory"); }

__device__ __forceinline__ void prefetch_l2(const void* p, uint32_t bytes) {
  asm volatile("cp.async.bulk.prefetch.L2.global [%0], %1;" ::"l"(p), "r"(bytes) : "memory");
}

__device__ __forceinline__ uint4 ld16(const void* p) { return *reinterpret_cast<const uint4*>(p); }
__device__ __forceinline__ uint2 ld8(const void* p) { return *reinterpret_cast<const uint2*>(p); }
__device__ __forceinline__ float shfl(float v, int src) { return __shfl_sync(FULL, v, src); }

// Signed byte `pos` (0..3) of w.
__device__ __forceinline__ int sbyte(uint32_t w, int pos) { return ((int)(w << (24 - 8 * pos))) >> 24; }

// The reference's f16_to_f32: the hardware conversion everywhere except the
// exponent-31 encodings, where the reference's own bit arithmetic applies.
__device__ __forceinline__ float f16_fast(uint32_t h) {
  return (h & 0x7C00u) == 0x7C00u ? f16_bits_to_f32(h) : __half2float(__ushort_as_half((unsigned short)h));
}

// Scales and mins of sub-blocks 2g and 2g+1 of a Q4_K block from its 12 scale
// bytes s0..s2 (get_scale_min_k4, csrc/libtinygiant.c:146-155).
__device__ __forceinline__ void q4k_pair_scales(int g, uint32_t s0, uint32_t s1, uint32_t s2, int& sl, int& ml,
                                                int& sh, int& mh) {
  const int P = 16 * (g & 1);
  const uint32_t y = (s0 >> P) & 0xFFFFu, z = (s1 >> P) & 0xFFFFu, w = (s2 >> P) & 0xFFFFu;
  if (g < 2) {
    sl = (int)(y & 63u);
    sh = (int)((y >> 8) & 63u);
    ml = (int)(z & 63u);
    mh = (int)((z >> 8) & 63u);
  } else {
    sl = (int)((w & 0xFu) | (((y >> 6) & 3u) << 4));
    sh = (int)(((w >> 8) & 0xFu) | (((y >> 14) & 3u) << 4));
    ml = (int)(((w >> 4) & 0xFu) | (((z >> 6) & 3u) << 4));
    mh = (int)(((w >> 12) & 0xFu) | (((z >> 14) & 3u) << 4));
  }
}

// ---------------------------------------------------------------------
// Warp row dots of one row against one token.  Every lane calls; lane 0
// returns the row's fp32 dot (the other lanes return 0).  x points at the
// token's Q8 blocks; x4 selects Q4_K's x4 association.

// Q4_K: lane = 4 * (block in pass) + group g; 8 blocks per pass.
template <typename XT>
__device__ __forceinline__ float dot_q4k(const uint8_t* m, int bpr, const XT* x, bool x4) {
  const int lane = threadIdx.x & 31, g = lane & 3, base = lane & ~3;
  float tot = 0.f;
  for (int p = 0; p < bpr; p += 8) {
    const int b = p + (lane >> 2);
    float c0 = 0.f, c1 = 0.f, sx = 0.f;
    if (b < bpr) {
      const uint8_t* blk = m + (size_t)b * Q4K_BYTES;
      const uint4 h = ld16(blk), q0 = ld16(blk + 16 + 32 * g), q1 = ld16(blk + 32 + 32 * g);
      const XT* xb = x + b;
      const int8_t* xq = xb->qs + 64 * g;
      const uint4 xa = ld16(xq), xe = ld16(xq + 16), xc = ld16(xq + 32), xd = ld16(xq + 48);
      const int2 bsv = *reinterpret_cast<const int2*>(&xb->bsums[2 * g]);
      sx = xb->scale;
      const uint32_t qw[8] = {q0.x, q0.y, q0.z, q0.w, q1.x, q1.y, q1.z, q1.w};
      const uint32_t xl[8] = {xa.x, xa.y, xa.z, xa.w, xe.x, xe.y, xe.z, xe.w};
      const uint32_t xh[8] = {xc.x, xc.y, xc.z, xc.w, xd.x, xd.y, xd.z, xd.w};
      int ilo = 0, ihi = 0;
#pragma unroll
      for (int j = 0; j < 8; j++) {
        ilo = dp4a((int)(qw[j] & 0x0F0F0F0Fu), (int)xl[j], ilo);
        ihi = dp4a((int)((qw[j] >> 4) & 0x0F0F0F0Fu), (int)xh[j], ihi);
      }
      const float d = f16_fast(h.x & 0xFFFFu), dmin = f16_fast(h.x >> 16);
      int sl, ml, sh, mh;
      q4k_pair_scales(g, h.y, h.z, h.w, sl, ml, sh, mh);
      const float dsl = fmul(d, (float)sl), dml = fmul(dmin, (float)ml);
      const float dsh = fmul(d, (float)sh), dmh = fmul(dmin, (float)mh);
      const float blo = (float)bsv.x, bhi = (float)bsv.y;
      if (x4) {
        c0 = fsub(fadd(fsub(fmul(dsl, (float)ilo), fmul(dml, blo)), fmul(dsh, (float)ihi)), fmul(dmh, bhi));
      } else {
        c0 = fsub(fmul(dsl, (float)ilo), fmul(dml, blo));
        c1 = fsub(fmul(dsh, (float)ihi), fmul(dmh, bhi));
      }
    }
    float bs;
    if (x4) {
      const float e1 = shfl(c0, base + 1), e2 = shfl(c0, base + 2), e3 = shfl(c0, base + 3);
      bs = fadd(fadd(fadd(fadd(0.f, c0), e1), e2), e3);
    } else {
      const float a1 = shfl(c0, base + 1), b1 = shfl(c1, base + 1);
      const float a2 = shfl(c0, base + 2), b2 = shfl(c1, base + 2);
      const float a3 = shfl(c0, base + 3), b3 = shfl(c1, base + 3);
      bs = fadd(fadd(fadd(fadd(fadd(fadd(fadd(fadd(0.f, c0), c1), a1), b1), a2), b2), a3), b3);
    }
    const float term = fmul(sx, bs);
    const int nb = min(8, bpr - p);
    float tv[8];
#pragma unroll
    for (int i = 0; i < 8; i++) tv[i] = shfl(term, 4 * i);
    if (lane == 0)
#pragma unroll
      for (int i = 0; i < 8; i++)
        if (i < nb) tot = fadd(tot, tv[i]);
  }
  return lane == 0 ? tot : 0.f;
}

// Q6_K: 8 lanes per block (half h = sub / 4, 8 consecutive l per lane); 4
// blocks per pass.  A block's sum of sc * isum16 is accumulated exactly in
// int32; when no partial sum can reach 2^24 that equals the reference's
// float fold, otherwise the 16 products are folded in its order.
template <typename XT>
__device__ __forceinline__ float dot_q6k(const uint8_t* m, const uint8_t* scp, const uint8_t* dp, int bpr,
                                         const XT* x) {
  const int lane = threadIdx.x & 31, sub = lane & 7, h = sub >> 2, c4 = sub & 3, lq = c4 >> 1;
  const int base = lane & ~7;
  float tot = 0.f;
  for (int p = 0; p < bpr; p += 4) {
    const int b = p + (lane >> 3);
    const bool on = b < bpr;
    int is[4] = {0, 0, 0, 0}, sck[4] = {0, 0, 0, 0};
    float d = 0.f, sx = 0.f;
    if (on) {
      const uint8_t* blk = m + (size_t)b * 192;
      const uint2 qa = ld8(blk + 64 * h + 8 * c4), qb = ld8(blk + 64 * h + 32 + 8 * c4);
      const uint2 qh = ld8(blk + 128 + 32 * h + 8 * c4);
      const uint4 sv = ld16(scp + (size_t)b * 16);
      const uint32_t dbits = (uint32_t)dp[(size_t)b * 2] | ((uint32_t)dp[(size_t)b * 2 + 1] << 8);
      const XT* xb = x + b;
      const int8_t* xq = xb->qs + 128 * h + 8 * c4;
      uint2 xk[4];
#pragma unroll
      for (int k = 0; k < 4; k++) xk[k] = ld8(xq + 32 * k);
      sx = xb->scale;
      d = f16_fast(dbits);
      const uint32_t A[2] = {qa.x, qa.y}, B[2] = {qb.x, qb.y}, H[2] = {qh.x, qh.y};
      int v[4][2];
#pragma unroll
      for (int w = 0; w < 2; w++) {
        v[0][w] = (int)((A[w] & 0x0F0F0F0Fu) | ((H[w] & 0x03030303u) << 4));
        v[1][w] = (int)((B[w] & 0x0F0F0F0Fu) | ((H[w] & 0x0C0C0C0Cu) << 2));
        v[2][w] = (int)(((A[w] >> 4) & 0x0F0F0F0Fu) | (H[w] & 0x30303030u));
        v[3][w] = (int)(((B[w] >> 4) & 0x0F0F0F0Fu) | ((H[w] >> 2) & 0x30303030u));
      }
#pragma unroll
      for (int k = 0; k < 4; k++) {
        const int raw = dp4a(v[k][0], (int)xk[k].x, dp4a(v[k][1], (int)xk[k].y, 0));
        const int xs = dp4a((int)xk[k].x, 0x01010101, dp4a((int)xk[k].y, 0x01010101, 0));
        is[k] = raw - 32 * xs;
      }
      // scales of (h, lq, k): sc[8h + lq + 2k]
      const uint32_t s0 = h ? sv.z : sv.x, s1 = h ? sv.w : sv.y;
      sck[0] = sbyte(s0, lq);
      sck[1] = sbyte(s0, lq + 2);
      sck[2] = sbyte(s1, lq);
      sck[3] = sbyte(s1, lq + 2);
    }
    int pr[4], S = 0, A = 0;
#pragma unroll
    for (int k = 0; k < 4; k++) {
      is[k] += __shfl_xor_sync(FULL, is[k], 1);
      pr[k] = (c4 & 1) ? 0 : sck[k] * is[k];
      S += pr[k];
      A += abs(pr[k]);
    }
    S += __shfl_xor_sync(FULL, S, 2);
    A += __shfl_xor_sync(FULL, A, 2);
    S += __shfl_xor_sync(FULL, S, 4);
    A += __shfl_xor_sync(FULL, A, 4);
    float bs = (float)S;
    const bool slow = on && sub == 0 && A >= (1 << 24);
    if (__any_sync(FULL, slow)) {
      float acc = 0.f;
#pragma unroll
      for (int o = 0; o < 8; o += 2)
#pragma unroll
        for (int k = 0; k < 4; k++) acc = fadd(acc, (float)__shfl_sync(FULL, pr[k], base + o));
      if (slow) bs = acc;
    }
    const float term = fmul(fmul(d, sx), bs);
    const int nb = min(4, bpr - p);
    float tv[4];
#pragma unroll
    for (int i = 0; i < 4; i++) tv[i] = shfl(term, 8 * i);
    if (lane == 0)
#pragma unroll
      for (int i = 0; i < 4; i++)
        if (i < nb) tot = fadd(tot, tv[i]);
  }
  return lane == 0 ? tot : 0.f;
}

// 4 e2m1 codes (one per byte, 0..15) -> 4 signed doubled values, in the byte
// order [v0, v2, v1, v3] (selector trick: c | c >> 12 packs the nibbles).
__device__ __forceinline__ int mxfp4_decode(uint32_t c) {
  const uint32_t sel = c | (c >> 12);
  const uint32_t pos = __byte_perm(0x03020100u, 0x0C080604u, sel & 0x7777u);   // 0,1,2,3 | 4,6,8,12
  const uint32_t neg = __byte_perm(0xFDFEFF00u, 0xF4F8FAFCu, sel & 0x7777u);   // 0,-1,-2,-3 | -4,-6,-8,-12
  return (int)__byte_perm(pos, neg, ((sel & 0x8888u) >> 1) | 0x3210u);
}

// MXFP4 (one lane per 32-value block) and Q8_0 (the same): lane 0 folds the
// lanes' terms in order.
template <int FMT, typename XT>
__device__ __forceinline__ float dot_sub32(const RowPtrs& rp, int nsub, const XT* x) {
  const int lane = threadIdx.x & 31;
  float tot = 0.f;
  for (int p = 0; p < nsub; p += 32) {
    const int u = p + lane;
    float term = 0.f;
    if (u < nsub) {
      int q[8];
      float sc;
      if constexpr (FMT == FMT_MXFP4) {
        const uint4 cv = ld16(rp.m + (size_t)u * 16);
        const uint32_t cw[4] = {cv.x, cv.y, cv.z, cv.w};
#pragma unroll
        for (int i = 0; i < 4; i++) {
          q[i] = mxfp4_decode(cw[i] & 0x0F0F0F0Fu);
          q[4 + i] = mxfp4_decode((cw[i] >> 4) & 0x0F0F0F0Fu);
        }
        sc = e8m0_half(rp.a1[u]);
      } else {
        const uint4 qa = ld16(rp.m + (size_t)u * 32), qb = ld16(rp.m + (size_t)u * 32 + 16);
        q[0] = (int)qa.x; q[1] = (int)qa.y; q[2] = (int)qa.z; q[3] = (int)qa.w;
        q[4] = (int)qb.x; q[5] = (int)qb.y; q[6] = (int)qb.z; q[7] = (int)qb.w;
        sc = f16_fast((uint32_t)rp.a2[(size_t)u * 2] | ((uint32_t)rp.a2[(size_t)u * 2 + 1] << 8));
      }
      const XT* xb = x + (u >> 3);
      const uint8_t* xv = reinterpret_cast<const uint8_t*>(xb->qs) + (u & 7) * 32;
      const uint4 xa = ld16(xv), xc = ld16(xv + 16);
      uint32_t xw[8] = {xa.x, xa.y, xa.z, xa.w, xc.x, xc.y, xc.z, xc.w};
      if constexpr (FMT == FMT_MXFP4) {
#pragma unroll
        for (int i = 0; i < 8; i++) xw[i] = __byte_perm(xw[i], 0u, 0x3120u);
      }
      int acc = 0;
#pragma unroll
      for (int i = 0; i < 8; i++) acc = dp4a(q[i], (int)xw[i], acc);
      term = fmul(fmul(xb->scale, sc), (float)acc);
    }
    const int nb = min(32, nsub - p);
#pragma unroll
    for (int i = 0; i < 32; i++) {
      const float v = shfl(term, i);
      if (lane == 0 && i < nb) tot = fadd(tot, v);
    }
  }
  return lane == 0 ? tot : 0.f;
}

template <int FMT, typename XT>
__device__ __forceinline__ float warp_dot1(const RowPtrs& rp, int cols, const XT* x, bool x4) {
  if constexpr (FMT == FMT_Q4K) return dot_q4k(rp.m, cols / QK, x, x4);
  else if constexpr (FMT == FMT_Q6K) return dot_q6k(rp.m, rp.a1, rp.a2, cols / QK, x);
  else return dot_sub32<FMT>(rp, cols / 32, x);
}

// Up to 4 tokens (lane 0 gets out[t], t < ng), one token at a time.
template <int FMT>
__device__ __forceinline__ void warp_dot(const RowPtrs& rp, int cols, const Q8Dev* const* x, int ng, bool x4,
                                         float* out) {
#pragma unroll 1
  for (int t = 0; t < ng; t++) {
    const float v = warp_dot1<FMT>(rp, cols, x[t], x4);
    if (t == 0) out[0] = v;
    else if (t == 1) out[1] = v;
    else if (t == 2) out[2] = v;
    else out[3] = v;
  }
}

// ---------------------------------------------------------------------
// One lane, one whole 256-value block: the block's term of a row dot for one
// token, folded in the reference's order inside the lane.  Rows are then
// folded over their blocks by the caller (block order, one lane).

// Q8 input block as staged in shared memory: the Q8Dev fields, the int32
// sums of each 16 values (Q6_K's bias correction, in the order the Q6_K
// block term reads them), the 32-value sums as
// fp32 (Q4_K's min terms), every field 16-byte
// aligned so it is read with 16-byte loads, and a 400-byte stride, which puts
// the blocks read by 8 consecutive lanes on distinct banks.
struct __align__(16) XQ {
  int8_t qs[QK];        // 0
  float scale;          // 256
  int32_t pad0[3];
  union {               // 272: the sums the consuming format's block terms use
    float bsf[8];       // Q4_K: 32-value sums as fp32 (exact: |bsum| <= 4064)
    int32_t xs16[16];   // Q6_K: sum of 16-value group g = 8h + 2k + lq at 4 (2h + lq) + k
  };
};
static_assert(sizeof(XQ) == 336, "XQ layout");

// Slot of the sum of 16-value group g (values 16g .. 16g + 15) in XQ.xs16.
__host__ __device__ __forceinline__ int xs16_slot(int g) { return 4 * (2 * (g >> 3) + (g & 1)) + ((g & 7) >> 1); }

// x / d correctly rounded to fp32, given yd = RN_double(1 / d).  The double
// product x * yd is within 2^-52 (relative) of x / d.  A quotient of two
// fp32 numbers that is not itself an fp32 number lies at least 2^-49
// (relative) from every fp32 rounding midpoint m: x - d m is a nonzero
// multiple of 2^min(e_x, e_d + e_m) (the exponents of the three numbers'
// last significant bits), and x = d m is impossible for a 25-bit m.  So
// rounding the product to fp32 rounds x / d.  Operands outside 2^-57 .. 2^58
// (zeros, subnormals, infinities, NaNs included) take __fdiv_rn, which keeps
// every quotient in the normal range.
__device__ __forceinline__ float div_rn_d(float x, float d, double yd) {
  const uint32_t ex = (__float_as_uint(x) >> 23) & 0xFFu, ed = (__float_as_uint(d) >> 23) & 0xFFu;
  if (ex - 70u > 114u || ed - 70u > 114u) return __fdiv_rn(x, d);
  return __double2float_rn((double)x * yd);
}

// max with NaN propagation (either operand NaN gives NaN).
__device__ __forceinline__ float fmax_nan(float a, float b) {
  float d;
  asm("max.NaN.f32 %0, %1, %2;" : "=f"(d) : "f"(a), "f"(b));
  return d;
}

// The quantizer of tg_q8.cuh (quantize_q8, csrc/libtinygiant.c:169-208) run
// by one warp into the staged form XQ, its extra field for the consuming
// format CF (Q6_K: sums of each 16 values; Q4_K: 32-value sums as fp32)
// formed from the same lane sums.  Lane l
// holds v[j] = value 8l + j of the block; positions at or past n are stored
// as 0.  The amax reduction is a tree (max is order-free); a NaN in the block
// gives the canonical NaN scale, where the reference propagates the NaN it
// met first — the block's dots are NaN either way.
//
// PERM stores each 32-value sub-block's qs in the MXFP4 order: word 2k + h
// holds values (4k + 2h, 16 + 4k + 2h, 4k + 2h + 1, 17 + 4k + 2h), the
// order in which mxfp4_isum reads a code word's nibbles.
template <bool PERM = false, int CF = FMT_Q4K>
__device__ __forceinline__ void quantize_xq(const float (&v)[8], int n, XQ* o) {
  const int lane = threadIdx.x & 31;
  float m[8];
#pragma unroll
  for (int j = 0; j < 8; j++) m[j] = 8 * lane + j < n ? fabsf(v[j]) : 0.f;
  float a = fmax_nan(fmax_nan(fmax_nan(m[0], m[1]), fmax_nan(m[2], m[3])),
                     fmax_nan(fmax_nan(m[4], m[5]), fmax_nan(m[6], m[7])));
#pragma unroll
  for (int off = 16; off > 0; off >>= 1) a = fmax_nan(a, __shfl_xor_sync(FULL, a, off));
  const float inv = a > 0.f ? __fdiv_rn(127.f, a) : 0.f;
  int q[8], s = 0;
#pragma unroll
  for (int j = 0; j < 8; j++) {
    q[j] = 0;
    if (8 * lane + j < n) {
      const float sv = __fmul_rn(v[j], inv);
      q[j] = (sv != sv) ? 0 : __float2int_rn(sv);
    }
    s += q[j];
  }
  uint32_t w0 = 0, w1 = 0;
#pragma unroll
  for (int j = 0; j < 4; j++) {
    w0 |= ((uint32_t)q[j] & 0xFFu) << (8 * j);
    w1 |= ((uint32_t)q[4 + j] & 0xFFu) << (8 * j);
  }
  if constexpr (PERM) {
    // lane l holds sub-block l / 4's values 8 (l % 4) .. + 7; lanes with
    // l % 4 < 2 take the values 16 further on from lane l + 2 and write
    // 16 bytes of the sub-block each
    const uint32_t p0 = __shfl_xor_sync(FULL, w0, 2), p1 = __shfl_xor_sync(FULL, w1, 2);
    if ((lane & 2) == 0) {
      uint4 nw;
      nw.x = __byte_perm(w0, p0, 0x5140);
      nw.y = __byte_perm(w0, p0, 0x7362);
      nw.z = __byte_perm(w1, p1, 0x5140);
      nw.w = __byte_perm(w1, p1, 0x7362);
      *reinterpret_cast<uint4*>(o->qs + 32 * (lane >> 2) + 16 * (lane & 1)) = nw;
    }
  } else {
    *reinterpret_cast<uint2*>(o->qs + 8 * lane) = make_uint2(w0, w1);
  }
  const int s16 = s + __shfl_xor_sync(FULL, s, 1);        // values 16 (l / 2) .. + 15
  const int s32 = s16 + __shfl_xor_sync(FULL, s16, 2);    // sub-block l / 4
  if constexpr (CF == FMT_Q6K) {
    if ((lane & 1) == 0) o->xs16[xs16_slot(lane >> 1)] = s16;
  } else if constexpr (CF == FMT_Q4K) {
    if ((lane & 3) == 0) o->bsf[lane >> 2] = (float)s32;
  }
  if (lane == 0) o->scale = div_rn_d(a, 127.f, 1.0 / 127.0);
}

// Exact int -> fp32 for |v| < 2^22 on the integer and fp32 pipes: the bits of
// 1.5 * 2^23 + v, minus 1.5 * 2^23.
__device__ __forceinline__ float i2f_small(int v) { return __fsub_rn(__int_as_float(0x4B400000 + v), 12582912.0f); }

// dp4a with unsigned bytes in a and signed bytes in b.
__device__ __forceinline__ int dp4a_us(uint32_t a, int b, int c) {
  int d;
  asm("dp4a.u32.s32 %0, %1, %2, %3;" : "=r"(d) : "r"(a), "r"(b), "r"(c));
  return d;
}

// Q4_K block term (dot_q4k_q8 223-272 for x1, dot_q4k_q8_x4 276-337 for x4).
// The four 64-value groups are unrolled (a loop measured slower in the step
// kernel).
__device__ __forceinline__ float q4k_block_term(const uint8_t* blk, const XQ& xb, bool x4) {
  const uint4 h = ld16(blk);
  const float d = f16_fast(h.x & 0xFFFFu), dmin = f16_fast(h.x >> 16);
  float bs = 0.f;
#pragma unroll
  for (int g = 0; g < 4; g++) {
    const uint4 q0 = ld16(blk + 16 + 32 * g), q1 = ld16(blk + 32 + 32 * g);
    const uint4 xa = ld16(xb.qs + 64 * g), xe = ld16(xb.qs + 64 * g + 16);
    const uint4 xc = ld16(xb.qs + 64 * g + 32), xd = ld16(xb.qs + 64 * g + 48);
    const float2 bf = *reinterpret_cast<const float2*>(xb.bsf + 2 * g);
    const uint32_t qw[8] = {q0.x, q0.y, q0.z, q0.w, q1.x, q1.y, q1.z, q1.w};
    const uint32_t xl[8] = {xa.x, xa.y, xa.z, xa.w, xe.x, xe.y, xe.z, xe.w};
    const uint32_t xh[8] = {xc.x, xc.y, xc.z, xc.w, xd.x, xd.y, xd.z, xd.w};
    int ilo = 0, ihi16 = 0;
#pragma unroll
    for (int j = 0; j < 8; j++) {
      ilo = dp4a_us(qw[j] & 0x0F0F0F0Fu, (int)xl[j], ilo);
      ihi16 = dp4a_us(qw[j] & 0xF0F0F0F0u, (int)xh[j], ihi16);   // 16 * (high nibbles . x)
    }
    const int ihi = ihi16 >> 4;
    int sl, ml, sh, mh;
    q4k_pair_scales(g, h.y, h.z, h.w, sl, ml, sh, mh);
    const float dsl = fmul(d, (float)sl), dml = fmul(dmin, (float)ml);
    const float dsh = fmul(d, (float)sh), dmh = fmul(dmin, (float)mh);
    const float flo = i2f_small(ilo), fhi = i2f_small(ihi);
    if (x4) {
      bs = fadd(bs, fsub(fadd(fsub(fmul(dsl, flo), fmul(dml, bf.x)), fmul(dsh, fhi)), fmul(dmh, bf.y)));
    } else {
      bs = fadd(bs, fsub(fmul(dsl, flo), fmul(dml, bf.x)));
      bs = fadd(bs, fsub(fmul(dsh, fhi), fmul(dmh, bf.y)));
    }
  }
  return fmul(xb.scale, bs);
}

// The product sc * isum16 of (half h, l-half lq, quarter k) of a Q6_K block.
__device__ __forceinline__ int q6k_prod(const uint32_t* qa, const uint32_t* qb, const uint32_t* qh, const XQ& xb,
                                        const uint32_t* sw, int xsum, int h, int lq, int k) {
  const uint4 xv = ld16(xb.qs + 128 * h + 32 * k + 16 * lq);
  const uint32_t xw[4] = {xv.x, xv.y, xv.z, xv.w};
  int raw = 0;
#pragma unroll
  for (int q = 0; q < 4; q++) {
    uint32_t v;
    if (k == 0) v = (qa[q] & 0x0F0F0F0Fu) | ((qh[q] & 0x03030303u) << 4);
    else if (k == 1) v = (qb[q] & 0x0F0F0F0Fu) | ((qh[q] & 0x0C0C0C0Cu) << 2);
    else if (k == 2) v = ((qa[q] >> 4) & 0x0F0F0F0Fu) | (qh[q] & 0x30303030u);
    else v = ((qb[q] >> 4) & 0x0F0F0F0Fu) | ((qh[q] >> 2) & 0x30303030u);
    raw = dp4a_us(v, (int)xw[q], raw);
  }
  // (q - 32) . x = q . x - 32 * sum(x) over the 16 values
  const int si = 8 * h + lq + 2 * k;
  return sbyte(sw[si >> 2], si & 3) * (raw - 32 * xsum);
}

// The reference's fp32 fold of a Q6_K block's 16 products, in order (the
// rare blocks whose partial sums may not be exact integers in fp32).
static __device__ __noinline__ float q6k_fold_slow(const uint8_t* mb, const uint32_t* sw, const XQ& xb) {
  float bs = 0.f;
  for (int hl = 0; hl < 4; hl++) {
    const int h = hl >> 1, lq = hl & 1;
    const uint4 va = ld16(mb + 64 * h + 16 * lq), vb = ld16(mb + 64 * h + 32 + 16 * lq);
    const uint4 vh = ld16(mb + 128 + 32 * h + 16 * lq);
    const uint4 xs = ld16(xb.xs16 + 4 * hl);
    const uint32_t qa[4] = {va.x, va.y, va.z, va.w}, qb[4] = {vb.x, vb.y, vb.z, vb.w};
    const uint32_t qh[4] = {vh.x, vh.y, vh.z, vh.w};
    const int xsv[4] = {(int)xs.x, (int)xs.y, (int)xs.z, (int)xs.w};
#pragma unroll
    for (int k = 0; k < 4; k++) bs = fadd(bs, (float)q6k_prod(qa, qb, qh, xb, sw, xsv[k], h, lq, k));
  }
  return bs;
}

// Q6_K block term (dot_q6k_q8 403-443): block_sum += sc * isum16 over
// (half, l = 0 / 16, quarter), then (d * sx) * block_sum.  Every product is
// an integer below 2^24 in magnitude (exact in fp32), so while the sum of
// their magnitudes stays below 2^24 every partial sum of the reference's
// fp32 fold is an exact integer and the fold equals the int32 sum; larger
// blocks replay the fold in order.  The four (half, l-half) pairs run as a
// loop (not unrolled), for a small instruction footprint.
__device__ __forceinline__ float q6k_block_term(const uint8_t* mb, const uint8_t* scb, const uint8_t* db,
                                                const XQ& xb) {
  const uint4 sv = ld16(scb);
  int S = 0, A = 0;
#pragma unroll 2
  for (int hl = 0; hl < 4; hl++) {
    const int h = hl >> 1, lq = hl & 1;
    const uint4 va = ld16(mb + 64 * h + 16 * lq), vb = ld16(mb + 64 * h + 32 + 16 * lq);
    const uint4 vh = ld16(mb + 128 + 32 * h + 16 * lq);
    const uint4 xs = ld16(xb.xs16 + 4 * hl);
    const uint32_t qa[4] = {va.x, va.y, va.z, va.w}, qb[4] = {vb.x, vb.y, vb.z, vb.w};
    const uint32_t qh[4] = {vh.x, vh.y, vh.z, vh.w};
    const int xsv[4] = {(int)xs.x, (int)xs.y, (int)xs.z, (int)xs.w};
    // scale 8h + lq + 2k: word 2h + k / 2, byte lq + 2 (k & 1)
    const uint32_t w0 = h ? sv.z : sv.x, w1 = h ? sv.w : sv.y;
    const int8_t* xq = xb.qs + 128 * h + 16 * lq;
#pragma unroll
    for (int k = 0; k < 4; k++) {
      const uint4 xv = ld16(xq + 32 * k);
      const uint32_t xw[4] = {xv.x, xv.y, xv.z, xv.w};
      int raw = 0;
#pragma unroll
      for (int q = 0; q < 4; q++) {
        uint32_t v;
        if (k == 0) v = (qa[q] & 0x0F0F0F0Fu) | ((qh[q] & 0x03030303u) << 4);
        else if (k == 1) v = (qb[q] & 0x0F0F0F0Fu) | ((qh[q] & 0x0C0C0C0Cu) << 2);
        else if (k == 2) v = ((qa[q] >> 4) & 0x0F0F0F0Fu) | (qh[q] & 0x30303030u);
        else v = ((qb[q] >> 4) & 0x0F0F0F0Fu) | ((qh[q] >> 2) & 0x30303030u);
        raw = dp4a_us(v, (int)xw[q], raw);
      }
      const int sc = sbyte(k < 2 ? w0 : w1, lq + 2 * (k & 1));
      const int p = sc * (raw - 32 * xsv[k]);
      S += p;
      A += abs(p);
    }
  }
  const uint32_t sw[4] = {sv.x, sv.y, sv.z, sv.w};
  const float bs = A < (1 << 24) ? (float)S : q6k_fold_slow(mb, sw, xb);
  const float d = f16_fast((uint32_t)db[0] | ((uint32_t)db[1] << 8));
  return fmul(fmul(d, xb.scale), bs);
}

// prmt with the PTX semantics of the selector's bit 3: the selected byte's
// sign replicated.
__device__ __forceinline__ uint32_t prmt(uint32_t a, uint32_t b, uint32_t sel) {
  uint32_t d;
  asm("prmt.b32 %0, %1, %2, %3;" : "=r"(d) : "r"(a), "r"(b), "r"(sel));
  return d;
}

// Integer dot of one MXFP4 sub-block (16 code bytes: byte i holds value i in
// its low nibble and value 16 + i in its high nibble) with x's 32 values in
// the MXFP4 order of quantize_xq<true>.  A code word used as a prmt selector
// indexes the doubled e2m1 magnitudes {0, 1, 2, 3, 4, 6, 8, 12} (csrc/
// libtinygiant.c:514) by its nibbles' low 3 bits, while a set sign bit makes
// prmt emit the (zero) sign of the entry: so the word itself gives the
// positive codes' values and the word with its sign bits flipped the
// negative codes' magnitudes, and the dot is dot(positives) - dot(negatives).
__device__ __forceinline__ int mxfp4_isum(const uint4& cv, const int8_t* xq) {
  constexpr uint32_t T0 = 0x03020100u, T1 = 0x0C080604u;
  const uint4 xa = ld16(xq), xb = ld16(xq + 16);
  const uint32_t xw[8] = {xa.x, xa.y, xa.z, xa.w, xb.x, xb.y, xb.z, xb.w};
  const uint32_t cw[4] = {cv.x, cv.y, cv.z, cv.w};
  int p = 0, m = 0;
#pragma unroll
  for (int k = 0; k < 4; k++) {
    const uint32_t c = cw[k], cn = c ^ 0x88888888u;
    p = dp4a((int)prmt(T0, T1, c), (int)xw[2 * k], p);
    m = dp4a((int)prmt(T0, T1, cn), (int)xw[2 * k], m);
    p = dp4a((int)prmt(T0, T1, c >> 16), (int)xw[2 * k + 1], p);
    m = dp4a((int)prmt(T0, T1, cn >> 16), (int)xw[2 * k + 1], m);
  }
  return p - m;
}

// Half-warp row dot of a 32-value-block format (MXFP4, Q8_0) against one
// token's Q8 blocks x (XQ; for MXFP4 in the order of quantize_xq<true>): the
// 16 lanes of half hb = lane & 16 share the row; lane h of the half forms the
// terms of sub-blocks h C .. h C + C - 1 (C = ceil(nsub / 16) <= 8), and the
// reference's left fold over sub-blocks (dot_mxfp4_q8 533-547, dot_q80_q8
// 576-590) runs through the half's lanes in order, one shuffle per lane.
// Terms past the row end are +0, whose addition leaves every partial sum of
// these folds unchanged (no term and no partial sum is -0: the products of
// positive scales with an integer sum round a zero to +0).  Both halves call
// together; every lane of a half returns its row's dot.
template <int FMT>
__device__ __forceinline__ float half_dot_sub32(const RowPtrs& rp, int nsub, const XQ* x) {
  const int lane = threadIdx.x & 31, h = lane & 15, hb = lane & 16;
  const int C = (nsub + 15) >> 4;
  float term[8];
#pragma unroll
  for (int c = 0; c < 8; c++) {
    const int u = h * C + c;
    term[c] = 0.f;
    if (c < C && u < nsub) {
      const XQ& xb = x[u >> 3];
      const int8_t* xq = xb.qs + (u & 7) * 32;
      if constexpr (FMT == FMT_MXFP4) {
        const int isum = mxfp4_isum(ld16(rp.m + (size_t)u * 16), xq);
        term[c] = fmul(fmul(xb.scale, e8m0_half(rp.a1[u])), i2f_small(isum));
      } else {
        const uint4 qa = ld16(rp.m + (size_t)u * 32), qb = ld16(rp.m + (size_t)u * 32 + 16);
        const uint4 xa = ld16(xq), xc = ld16(xq + 16);
        int acc = dp4a((int)qa.x, (int)xa.x, 0);
        acc = dp4a((int)qa.y, (int)xa.y, acc);
        acc = dp4a((int)qa.z, (int)xa.z, acc);
        acc = dp4a((int)qa.w, (int)xa.w, acc);
        acc = dp4a((int)qb.x, (int)xc.x, acc);
        acc = dp4a((int)qb.y, (int)xc.y, acc);
        acc = dp4a((int)qb.z, (int)xc.z, acc);
        acc = dp4a((int)qb.w, (int)xc.w, acc);
        const float sc = f16_fast((uint32_t)rp.a2[(size_t)u * 2] | ((uint32_t)rp.a2[(size_t)u * 2 + 1] << 8));
        term[c] = fmul(fmul(xb.scale, sc), i2f_small(acc));
      }
    }
  }
  float tot = 0.f;
#pragma unroll 1
  for (int i = 0; i < 16; i++) {
    const float prev = __shfl_sync(FULL, tot, hb | ((i + 15) & 15));
    float r = i == 0 ? 0.f : prev;
#pragma unroll
    for (int c = 0; c < 8; c++)
      if (c < C) r = fadd(r, term[c]);
    if (h == i) tot = r;
  }
  return __shfl_sync(FULL, tot, hb | 15);
}

// Row fold over lanes: lanes lead, lead + stride, ... (n of them) hold the
// block terms of one row in block order; every lane returns the left fold of
// its row, starting from 0.  n and stride must be the same on every lane.
__device__ __forceinline__ float fold_row(float term, int lead, int n, int stride = 1) {
  float tot = 0.f;
#pragma unroll 4
  for (int i = 0; i < n; i++) tot = fadd(tot, shfl(term, (lead + i * stride) & 31));
  return tot;
}

// F16 rows against fp32 inputs (lane 0): the reference's 8 fused lane chains,
// their pairwise sum, then the tail (matvec_f16, 635-653).
__device__ __forceinline__ float dot_f16_lane(const uint16_t* row, const float* x, int n) {
  float a0[4] = {0.f, 0.f, 0.f, 0.f}, a1[4] = {0.f, 0.f, 0.f, 0.f};
  int q = 0;
  for (; q + 7 < n; q += 8)
#pragma unroll
    for (int l = 0; l < 4; l++) {
      a0[l] = __fmaf_rn(half_ieee(row[q + l]), x[q + l], a0[l]);
      a1[l] = __fmaf_rn(half_ieee(row[q + 4 + l]), x[q + 4 + l], a1[l]);
    }
  float v = fadd(fadd(fadd(a0[0], a1[0]), fadd(a0[1], a1[1])), fadd(fadd(a0[2], a1[2]), fadd(a0[3], a1[3])));
  for (; q < n; q++) v = fadd(v, fmul(f16_bits_to_f32(row[q]), x[q]));
  return v;
}

}  // namespace tg
