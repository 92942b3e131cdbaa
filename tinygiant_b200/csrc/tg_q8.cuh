// tg_q8.cuh — the Q8 activation quantizer as a CTA-wide device routine.
//
// quantize_q8 (csrc/libtinygiant.c:169-208) per 256-value block:
//   amax = max|x| (a NaN propagates, as FMAX does);  scale = amax / 127;
//   inv = amax > 0 ? 127 / amax : 0;  q = round-half-even(x * inv) (NaN -> 0);
//   bsums[j] = sum of q over values 32j..32j+31;  sum = sum of bsums;
//   positions past the row end (a partial last block) are 0.
// IEEE division and multiplication (__fdiv_rn, __fmul_rn) and __float2int_rn
// make every field bit-identical to the reference; max and integer sums are
// order-free.
#pragma once
#include "tg_common.cuh"

namespace tg {

__device__ __forceinline__ float max_nan(float a, float b) {
  if (a != a) return a;
  if (b != b) return b;
  return a > b ? a : b;
}

struct Q8Scratch {
  float wmax[8];
  int wsum[8];
};

// Called by all 256 threads of a CTA; thread t holds value v of position t
// (valid = t < n).  Writes one block.  Contains __syncthreads().
__device__ __forceinline__ void quantize_block_cta(float v, bool valid, Q8Dev* o, Q8Scratch& sh) {
  const int t = threadIdx.x, lane = t & 31, w = t >> 5;
  float a = valid ? fabsf(v) : 0.f;
#pragma unroll
  for (int off = 16; off > 0; off >>= 1) a = max_nan(a, __shfl_xor_sync(0xffffffffu, a, off));
  if (lane == 0) sh.wmax[w] = a;
  __syncthreads();
  float amax = sh.wmax[0];
#pragma unroll
  for (int i = 1; i < 8; i++) amax = max_nan(amax, sh.wmax[i]);
  const float inv = amax > 0.f ? __fdiv_rn(127.f, amax) : 0.f;
  int q = 0;
  if (valid) {
    const float s = __fmul_rn(v, inv);
    q = (s != s) ? 0 : __float2int_rn(s);
  }
  int bs = q;
#pragma unroll
  for (int off = 16; off > 0; off >>= 1) bs += __shfl_xor_sync(0xffffffffu, bs, off);
  o->qs[t] = (int8_t)q;
  if (lane == 0) {
    sh.wsum[w] = bs;
    o->bsums[w] = bs;
  }
  __syncthreads();
  if (t == 0) {
    int total = 0;
#pragma unroll
    for (int i = 0; i < 8; i++) total += sh.wsum[i];
    o->scale = __fdiv_rn(amax, 127.f);
    o->sum = total;
  }
  __syncthreads();
}

// The same quantizer run by one warp on values it holds: lane l holds v[j] =
// value 8l + j of the block (positions at or past n must be passed as 0 and
// are stored as 0).  No CTA barrier.
template <typename O>
__device__ __forceinline__ void quantize_block_warp_vals(const float* v, int n, O* o) {
  const int lane = threadIdx.x & 31;
  float a = 0.f;
#pragma unroll
  for (int j = 0; j < 8; j++)
    if (lane * 8 + j < n) a = max_nan(a, fabsf(v[j]));
#pragma unroll
  for (int off = 16; off > 0; off >>= 1) a = max_nan(a, __shfl_xor_sync(0xffffffffu, a, off));
  const float inv = a > 0.f ? __fdiv_rn(127.f, a) : 0.f;
  int q[8], s = 0;
#pragma unroll
  for (int j = 0; j < 8; j++) {
    const int i = lane * 8 + j;
    q[j] = 0;
    if (i < n) {
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
  reinterpret_cast<uint2*>(o->qs)[lane] = make_uint2(w0, w1);
  // bsums: 4 lanes per 32-value sub-block
  int bs = s;
  bs += __shfl_xor_sync(0xffffffffu, bs, 1);
  bs += __shfl_xor_sync(0xffffffffu, bs, 2);
  if ((lane & 3) == 0) o->bsums[lane >> 2] = bs;
  int tot = s;
#pragma unroll
  for (int off = 16; off > 0; off >>= 1) tot += __shfl_xor_sync(0xffffffffu, tot, off);
  if (lane == 0) {
    o->scale = __fdiv_rn(a, 127.f);
    o->sum = tot;
  }
}

// NB blocks at once, interleaved so their warp reductions overlap: lane l
// holds v[b][j] = value 8l + j of block b (positions at or past n[b] passed
// as 0); blocks with n[b] == 0 are not written.
template <int NB, typename O>
__device__ __forceinline__ void quantize_blocks_warp_vals(const float (*v)[8], const int* n, O* const* o) {
  const int lane = threadIdx.x & 31;
  float a[NB];
#pragma unroll
  for (int b = 0; b < NB; b++) {
    a[b] = 0.f;
#pragma unroll
    for (int j = 0; j < 8; j++)
      if (lane * 8 + j < n[b]) a[b] = max_nan(a[b], fabsf(v[b][j]));
  }
#pragma unroll
  for (int off = 16; off > 0; off >>= 1)
#pragma unroll
    for (int b = 0; b < NB; b++) a[b] = max_nan(a[b], __shfl_xor_sync(0xffffffffu, a[b], off));
  int s[NB], tot[NB], bs[NB];
#pragma unroll
  for (int b = 0; b < NB; b++) {
    const float inv = a[b] > 0.f ? __fdiv_rn(127.f, a[b]) : 0.f;
    int q[8];
    s[b] = 0;
#pragma unroll
    for (int j = 0; j < 8; j++) {
      q[j] = 0;
      if (lane * 8 + j < n[b]) {
        const float sv = __fmul_rn(v[b][j], inv);
        q[j] = (sv != sv) ? 0 : __float2int_rn(sv);
      }
      s[b] += q[j];
    }
    uint32_t w0 = 0, w1 = 0;
#pragma unroll
    for (int j = 0; j < 4; j++) {
      w0 |= ((uint32_t)q[j] & 0xFFu) << (8 * j);
      w1 |= ((uint32_t)q[4 + j] & 0xFFu) << (8 * j);
    }
    if (n[b] > 0) reinterpret_cast<uint2*>(o[b]->qs)[lane] = make_uint2(w0, w1);
    bs[b] = s[b];
    tot[b] = s[b];
  }
#pragma unroll
  for (int b = 0; b < NB; b++) bs[b] += __shfl_xor_sync(0xffffffffu, bs[b], 1);
#pragma unroll
  for (int b = 0; b < NB; b++) bs[b] += __shfl_xor_sync(0xffffffffu, bs[b], 2);
#pragma unroll
  for (int off = 16; off > 0; off >>= 1)
#pragma unroll
    for (int b = 0; b < NB; b++) tot[b] += __shfl_xor_sync(0xffffffffu, tot[b], off);
#pragma unroll
  for (int b = 0; b < NB; b++) {
    if (n[b] == 0) continue;
    if ((lane & 3) == 0) o[b]->bsums[lane >> 2] = bs[b];
    if (lane == 0) {
      o[b]->scale = __fdiv_rn(a[b], 127.f);
      o[b]->sum = tot[b];
    }
  }
}

// The same quantizer on a block held as two halves in 16-byte lane order:
// lane l holds values 4l..4l+3 (lo) and 128+4l..128+4l+3 (hi); positions at
// or past n are passed as 0.
template <typename O>
__device__ __forceinline__ void quantize_block_warp_f4(const float4& lo, const float4& hi, int n, O* o) {
  const int lane = threadIdx.x & 31;
  const float v[8] = {lo.x, lo.y, lo.z, lo.w, hi.x, hi.y, hi.z, hi.w};
  float a = 0.f;
#pragma unroll
  for (int j = 0; j < 8; j++)
    if ((j < 4 ? 4 * lane + j : 128 + 4 * lane + j - 4) < n) a = max_nan(a, fabsf(v[j]));
#pragma unroll
  for (int off = 16; off > 0; off >>= 1) a = max_nan(a, __shfl_xor_sync(0xffffffffu, a, off));
  const float inv = a > 0.f ? __fdiv_rn(127.f, a) : 0.f;
  int q[8], s0 = 0, s1 = 0;
#pragma unroll
  for (int j = 0; j < 8; j++) {
    const int i = j < 4 ? 4 * lane + j : 128 + 4 * lane + j - 4;
    q[j] = 0;
    if (i < n) {
      const float sv = __fmul_rn(v[j], inv);
      q[j] = (sv != sv) ? 0 : __float2int_rn(sv);
    }
    if (j < 4) s0 += q[j];
    else s1 += q[j];
  }
  uint32_t w0 = 0, w1 = 0;
#pragma unroll
  for (int j = 0; j < 4; j++) {
    w0 |= ((uint32_t)q[j] & 0xFFu) << (8 * j);
    w1 |= ((uint32_t)q[4 + j] & 0xFFu) << (8 * j);
  }
  reinterpret_cast<uint32_t*>(o->qs)[lane] = w0;
  reinterpret_cast<uint32_t*>(o->qs + 128)[lane] = w1;
  // bsums: 8 lanes per 32-value sub-block in each half
  int b0 = s0, b1 = s1;
#pragma unroll
  for (int off = 1; off < 8; off <<= 1) {
    b0 += __shfl_xor_sync(0xffffffffu, b0, off);
    b1 += __shfl_xor_sync(0xffffffffu, b1, off);
  }
  if ((lane & 7) == 0) {
    o->bsums[lane >> 3] = b0;
    o->bsums[4 + (lane >> 3)] = b1;
  }
  int tot = s0 + s1;
#pragma unroll
  for (int off = 16; off > 0; off >>= 1) tot += __shfl_xor_sync(0xffffffffu, tot, off);
  if (lane == 0) {
    o->scale = __fdiv_rn(a, 127.f);
    o->sum = tot;
  }
}

// The warp quantizer on the block at src (shared or global memory).
__device__ __forceinline__ void quantize_block_warp(const float* src, int n, Q8Dev* o) {
  const int lane = threadIdx.x & 31;
  float v[8];
#pragma unroll
  for (int j = 0; j < 8; j++) v[j] = lane * 8 + j < n ? src[lane * 8 + j] : 0.f;
  quantize_block_warp_vals(v, n, o);
}

}  // namespace tg
