// tg_dots.cuh — per-format "outer terms" of a quantized row dot product.
//
// The reference forms each row dot as a single left-to-right float fold
//     total = ((0 + t_0) + t_1) + ... + t_{n-1}
// over one term per 256-block (Q4_K, Q6_K) or per 32-block (MXFP4, Q8_0):
//   Q4_K : t_b = sx_b * bs_b, bs_b itself folded over the block's 4 groups
//          (x1: 223-272, x4: 276-337 of csrc/libtinygiant.c)
//   Q6_K : t_b = (d_b * sx_b) * bs_b, bs_b = fold of sc * isum16 (403-487)
//   MXFP4: t_s = (sx * e8m0_half) * isum32 (533-570)
//   Q8_0 : t_s = (sx * d) * isum32 (576-590)
// The functions below compute one term for up to 4 Q8 inputs at once.  The
// integer sums are exact (dp4a), and every float operation is a separately
// rounded __f*_rn call in the reference's order, so a fold of these terms
// in index order reproduces the reference's fp32 result bit for bit.
#pragma once
#include <cuda_fp16.h>
#include "tg_common.cuh"

namespace tg {

__device__ __forceinline__ uint4 ldg16(const void* p) { return __ldg(reinterpret_cast<const uint4*>(p)); }

__device__ __forceinline__ int dp4a(int a, int b, int c) { return __dp4a(a, b, c); }

// Q8 input view for up to 4 tokens of one 256-block.
struct Q8Ref {
  const Q8Dev* blk[4];
};

// Q4_K: the 8 exact sub-block sums of one block against one Q8 block.
// w = the block's 36 words (header in w[0..3], nibbles in w[4..35]); sums in
// the reference's order: is[2g] = low nibbles of group g (values 64g..64g+31),
// is[2g+1] = high nibbles (64g+32..64g+63) (csrc/libtinygiant.c:243-261).
__device__ __forceinline__ void q4k_isums(const uint32_t* w, const int* xw, int* is) {
#pragma unroll
  for (int g = 0; g < 4; g++) {
    int ilo = 0, ihi = 0;
#pragma unroll
    for (int j4 = 0; j4 < 8; j4++) {
      uint32_t q = w[4 + 8 * g + j4];
      ilo = dp4a((int)(q & 0x0F0F0F0Fu), __ldg(xw + 16 * g + j4), ilo);
      ihi = dp4a((int)((q >> 4) & 0x0F0F0F0Fu), __ldg(xw + 16 * g + 8 + j4), ihi);
    }
    is[2 * g] = ilo;
    is[2 * g + 1] = ihi;
  }
}

__device__ __forceinline__ void load_words(const uint8_t* p, uint32_t* w, int n16) {
#pragma unroll
  for (int i = 0; i < n16; i++) {
    uint4 v = ldg16(p + 16 * i);
    w[4 * i] = v.x; w[4 * i + 1] = v.y; w[4 * i + 2] = v.z; w[4 * i + 3] = v.w;
  }
}

// Q4_K block term for n tokens (n <= 4).  `x4` selects the x4 association.
__device__ __forceinline__ void q4k_terms(const uint8_t* bl, const Q8Ref& xr, int n, bool x4, float* out) {
  uint32_t w[36];
  load_words(bl, w, 9);
  float d = f16_bits_to_f32(w[0] & 0xFFFFu), dmin = f16_bits_to_f32(w[0] >> 16);
  int sc[8], mn[8];
#pragma unroll
  for (int j = 0; j < 8; j++) q4k_scale_min(j, w[1], w[2], w[3], sc[j], mn[j]);
  for (int t = 0; t < n; t++) {
    const Q8Dev* xb = xr.blk[t];
    int is[8];
    q4k_isums(w, reinterpret_cast<const int*>(xb->qs), is);
    float bs = 0.f;
#pragma unroll
    for (int g = 0; g < 4; g++) {
      float blo = (float)__ldg(&xb->bsums[2 * g]), bhi = (float)__ldg(&xb->bsums[2 * g + 1]);
      float dsl = fmul(d, (float)sc[2 * g]), dml = fmul(dmin, (float)mn[2 * g]);
      float dsh = fmul(d, (float)sc[2 * g + 1]), dmh = fmul(dmin, (float)mn[2 * g + 1]);
      if (x4) {
        bs = fadd(bs, fsub(fadd(fsub(fmul(dsl, (float)is[2 * g]), fmul(dml, blo)), fmul(dsh, (float)is[2 * g + 1])),
                           fmul(dmh, bhi)));
      } else {
        bs = fadd(bs, fsub(fmul(dsl, (float)is[2 * g]), fmul(dml, blo)));
        bs = fadd(bs, fsub(fmul(dsh, (float)is[2 * g + 1]), fmul(dmh, bhi)));
      }
    }
    out[t] = fmul(__ldg(&xb->scale), bs);
  }
}

// Q6_K: the 16 exact sums of 16 values of one block, in the reference's
// visiting order (half h, 16-byte chunk c, quarter k) -> is[(2h + c)*4 + k];
// value 128h + 32k + 16c + i has scale sc[8h + c + 2k] (384-439).
// w = ql[128] | qh[64] as 48 words.
__device__ __forceinline__ void q6k_isums(const uint32_t* w, const int* xw, int* is) {
#pragma unroll
  for (int h = 0; h < 2; h++) {
#pragma unroll
    for (int c = 0; c < 2; c++) {
      int a[4] = {0, 0, 0, 0};
#pragma unroll
      for (int wq = 0; wq < 4; wq++) {
        int l = 16 * c + 4 * wq;                      // byte offset within the half
        uint32_t qa = w[(64 * h + l) >> 2];           // ql[64h + l ..]
        uint32_t qb = w[(64 * h + 32 + l) >> 2];      // ql[64h + 32 + l ..]
        uint32_t qh = w[(128 + 32 * h + l) >> 2];     // qh[32h + l ..]
        uint32_t v0 = (qa & 0x0F0F0F0Fu) | ((qh & 0x03030303u) << 4);
        uint32_t v1 = (qb & 0x0F0F0F0Fu) | ((qh & 0x0C0C0C0Cu) << 2);
        uint32_t v2 = ((qa >> 4) & 0x0F0F0F0Fu) | (qh & 0x30303030u);
        uint32_t v3 = ((qb >> 4) & 0x0F0F0F0Fu) | ((qh >> 2) & 0x30303030u);
        int base = 32 * h + 4 * c + wq;               // x word of position 128h + 16c + 4wq
        a[0] = dp4a((int)__vsub4(v0, 0x20202020u), __ldg(xw + base), a[0]);
        a[1] = dp4a((int)__vsub4(v1, 0x20202020u), __ldg(xw + base + 8), a[1]);
        a[2] = dp4a((int)__vsub4(v2, 0x20202020u), __ldg(xw + base + 16), a[2]);
        a[3] = dp4a((int)__vsub4(v3, 0x20202020u), __ldg(xw + base + 24), a[3]);
      }
#pragma unroll
      for (int k = 0; k < 4; k++) is[(2 * h + c) * 4 + k] = a[k];
    }
  }
}

// Q6_K block term.  main: ql[128] | qh[64]; sc: 16 int8 scales; d: fp16.
__device__ __forceinline__ void q6k_terms(const uint8_t* mainp, const uint8_t* scp, const uint8_t* dp,
                                          const Q8Ref& xr, int n, float* out) {
  uint32_t w[48];
  load_words(mainp, w, 12);
  uint4 sv = ldg16(scp);
  uint32_t sw[4] = {sv.x, sv.y, sv.z, sv.w};
  float scf[16];
#pragma unroll
  for (int i = 0; i < 16; i++) scf[i] = (float)(int8_t)((sw[i >> 2] >> (8 * (i & 3))) & 0xFFu);
  float d = f16_bits_to_f32((uint32_t)dp[0] | ((uint32_t)dp[1] << 8));
  for (int t = 0; t < n; t++) {
    const Q8Dev* xb = xr.blk[t];
    int is[16];
    q6k_isums(w, reinterpret_cast<const int*>(xb->qs), is);
    float bs = 0.f;
#pragma unroll
    for (int h = 0; h < 2; h++)
#pragma unroll
      for (int c = 0; c < 2; c++)
#pragma unroll
        for (int k = 0; k < 4; k++) bs = fadd(bs, fmul(scf[8 * h + c + 2 * k], (float)is[(2 * h + c) * 4 + k]));
    out[t] = fmul(fmul(d, __ldg(&xb->scale)), bs);
  }
}

// Doubled e2m1 values (514).
__device__ __forceinline__ int mxfp4_val(uint32_t code) {
  constexpr uint64_t lo = 0x0C08060403020100ull;   // 0,1,2,3,4,6,8,12
  int m = (int)((lo >> (8 * (code & 7u))) & 0xFFu);
  return (code & 8u) ? -m : m;
}

// 4 e2m1 codes from the low (shift 0) or high (shift 4) nibbles of a word,
// packed as 4 signed bytes in byte order.
__device__ __forceinline__ int mxfp4_word(uint32_t w, int shift) {
  uint32_t r = 0;
#pragma unroll
  for (int i = 0; i < 4; i++) r |= ((uint32_t)mxfp4_val((w >> (8 * i + shift)) & 0xFu) & 0xFFu) << (8 * i);
  return (int)r;
}

// MXFP4: exact sum of one 32-value sub-block (codes as 4 words) against
// its 32 Q8 values (xw: 8 words).
__device__ __forceinline__ int mxfp4_isum(const uint32_t* cw, const int* xw) {
  int acc = 0;
#pragma unroll
  for (int i = 0; i < 4; i++) acc = dp4a(mxfp4_word(cw[i], 0), __ldg(xw + i), acc);
#pragma unroll
  for (int i = 0; i < 4; i++) acc = dp4a(mxfp4_word(cw[i], 4), __ldg(xw + 4 + i), acc);
  return acc;
}

// MXFP4 sub-block term: codes 16 B, e8m0 1 B; x = Q8 block s/8 at (s%8)*32.
__device__ __forceinline__ void mxfp4_terms(const uint8_t* codes, uint32_t e, int s, const Q8Ref& xr, int n,
                                            float* out) {
  uint4 cv = ldg16(codes);
  uint32_t cw[4] = {cv.x, cv.y, cv.z, cv.w};
  float dh = e8m0_half(e);
  for (int t = 0; t < n; t++) {
    const Q8Dev* xb = xr.blk[t];
    int acc = mxfp4_isum(cw, reinterpret_cast<const int*>(xb->qs) + (s & 7) * 8);
    out[t] = fmul(fmul(__ldg(&xb->scale), dh), (float)acc);
  }
}

// Q8_0: exact sum of one 32-value sub-block (8 words) against 8 Q8 words.
__device__ __forceinline__ int q80_isum(const int* qw, const int* xw) {
  int acc = 0;
#pragma unroll
  for (int i = 0; i < 8; i++) acc = dp4a(qw[i], __ldg(xw + i), acc);
  return acc;
}

// Q8_0 sub-block term: 32 int8 + fp16 d.
__device__ __forceinline__ void q80_terms(const uint8_t* q, uint32_t dbits, int s, const Q8Ref& xr, int n,
                                          float* out) {
  uint4 a = ldg16(q), b = ldg16(q + 16);
  int qw[8] = {(int)a.x, (int)a.y, (int)a.z, (int)a.w, (int)b.x, (int)b.y, (int)b.z, (int)b.w};
  float d = f16_bits_to_f32(dbits);
  for (int t = 0; t < n; t++) {
    const Q8Dev* xb = xr.blk[t];
    int acc = q80_isum(qw, reinterpret_cast<const int*>(xb->qs) + (s & 7) * 8);
    out[t] = fmul(fmul(__ldg(&xb->scale), d), (float)acc);
  }
}

// Number of outer terms per row.
__host__ __device__ __forceinline__ int terms_per_row(int fmt, int cols) {
  return (fmt == FMT_Q4K || fmt == FMT_Q6K) ? cols / QK : cols / 32;
}

// Term p of row r of matrix W for n tokens.  xq points at the tokens' Q8
// rows (qstride blocks apart); returns false for an unsupported format.
__device__ __forceinline__ bool row_terms(const WDesc& W, int r, int p, const Q8Dev* const* xrow, int n, bool x4,
                                          float* out) {
  Q8Ref xr;
  switch (W.fmt) {
    case FMT_Q4K: {
      for (int t = 0; t < n; t++) xr.blk[t] = xrow[t] + p;
      q4k_terms(W.main + (size_t)r * W.rs + (size_t)p * Q4K_BYTES, xr, n, x4, out);
      return true;
    }
    case FMT_Q6K: {
      const size_t ro = (size_t)r * W.rs;
      for (int t = 0; t < n; t++) xr.blk[t] = xrow[t] + p;
      q6k_terms(W.main + ro + (size_t)p * 192, W.aux1 + ro + (size_t)p * 16, W.aux2 + ro + (size_t)p * 2, xr, n, out);
      return true;
    }
    case FMT_MXFP4: {
      const size_t ro = (size_t)r * W.rs;
      for (int t = 0; t < n; t++) xr.blk[t] = xrow[t] + (p >> 3);
      mxfp4_terms(W.main + ro + (size_t)p * 16, __ldg(W.aux1 + ro + p), p, xr, n, out);
      return true;
    }
    case FMT_Q80: {
      const size_t ro = (size_t)r * W.rs;
      for (int t = 0; t < n; t++) xr.blk[t] = xrow[t] + (p >> 3);
      const uint8_t* dp = W.aux2 + ro + 2 * (size_t)p;
      uint32_t db = (uint32_t)__ldg(dp) | ((uint32_t)__ldg(dp + 1) << 8);
      q80_terms(W.main + ro + (size_t)p * 32, db, p, xr, n, out);
      return true;
    }
    default:
      return false;
  }
}

// f16 row . float x with the reference's lane structure (635-653): two
// 4-lane fused accumulators over 8-value steps (exact IEEE conversion, as
// vcvt_f32_f16 does), pairwise lane sum, then a scalar tail through the
// reference's own f16_to_f32.
__device__ __forceinline__ float half_ieee(uint16_t h) { return __half2float(__ushort_as_half(h)); }

__device__ __forceinline__ float dot_f16_row(const uint16_t* row, const float* x, int ncols) {
  float a0[4] = {0.f, 0.f, 0.f, 0.f}, a1[4] = {0.f, 0.f, 0.f, 0.f};
  int i = 0;
  for (; i + 7 < ncols; i += 8) {
#pragma unroll
    for (int l = 0; l < 4; l++) {
      a0[l] = __fmaf_rn(half_ieee(row[i + l]), x[i + l], a0[l]);
      a1[l] = __fmaf_rn(half_ieee(row[i + 4 + l]), x[i + 4 + l], a1[l]);
    }
  }
  float s[4];
#pragma unroll
  for (int l = 0; l < 4; l++) s[l] = fadd(a0[l], a1[l]);
  float sum = fadd(fadd(s[0], s[1]), fadd(s[2], s[3]));
  for (; i < ncols; i++) sum = fadd(sum, fmul(f16_bits_to_f32(row[i]), x[i]));
  return sum;
}

}  // namespace tg
