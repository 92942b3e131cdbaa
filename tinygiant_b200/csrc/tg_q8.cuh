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

}  // namespace tg
