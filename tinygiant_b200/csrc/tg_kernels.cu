// tg_kernels.cu — matvec, quantizer and utility kernels (sm_100a); the MoE
// expert phases are in tg_moe.cu and the fused router in tg_route.cu.
//
//   quantize_rows_kernel   fp32 rows -> Q8 blocks      (csrc/libtinygiant.c:169-208)
//   matvec_kernel          one matrix . one input      (mm_task / gmm_task, 345-364, 906-931)
//   f16/f32 matvec, rms_norm, repack
//
// Each output element is produced by the same sequence of rounded float
// operations as the reference (see tg_dots.cuh); the order-free parts
// (integer sub-block sums, max|x|) run in parallel.
#include <cuda_fp16.h>

#include <algorithm>

#include "tg_dots.cuh"
#include "tg_kernels.h"
#include "tg_plan.cuh"
#include "tg_q8.cuh"
#include "tg_warpdot.cuh"

namespace tg {

// ---------------------------------------------------------------------
// Q8 quantizer: one CTA of 256 threads per 256-block.

__global__ void __launch_bounds__(256) quantize_rows_kernel(const float* __restrict__ x, int ncols, long ldx,
                                                            Q8Dev* __restrict__ out, int nb) {
  __shared__ Q8Scratch sh;
  const int b = blockIdx.x, row = blockIdx.y, t = threadIdx.x;
  const int n = min(QK, ncols - b * QK);
  const bool valid = t < n;
  const float v = valid ? x[(size_t)row * ldx + (size_t)b * QK + t] : 0.f;
  quantize_block_cta(v, valid, out + (size_t)row * nb + b, sh);
}

// ---------------------------------------------------------------------
// One matrix against one input: out[r] = dot (+ (bias ? bias[r] : 0.f)).

// Rows r0 .. r0 + R - 1 of W (one CTA; smem: R x terms-per-row floats).
template <int R>
__device__ __forceinline__ void matvec_rows(const WDesc& W, int r0, const Q8Dev* __restrict__ xq8,
                                            const float* __restrict__ x, const float* __restrict__ bias,
                                            int bias_term, float* __restrict__ out, DevStatus* st, float* smem) {
  if (r0 >= W.rows) return;
  const int nr = min(R, W.rows - r0);
  if (W.fmt == FMT_F16) {
    for (int rho = threadIdx.x; rho < nr; rho += blockDim.x) {
      const int r = r0 + rho;
      float v = dot_f16_row(reinterpret_cast<const uint16_t*>(W.main + (size_t)r * W.rs), x, W.cols);
      out[r] = bias_term ? fadd(v, bias ? bias[r] : 0.f) : v;
    }
    return;
  }
  const int P = terms_per_row(W.fmt, W.cols);
  const Q8Dev* xrow[1] = {xq8};
  for (int u = threadIdx.x; u < nr * P; u += blockDim.x) {
    const int rho = u / P, p = u - rho * P;
    float o[1];
    if (!row_terms(W, r0 + rho, p, xrow, 1, false, o)) {
      set_error(st, ERR_BAD_FORMAT, 3, W.fmt, 0);
      o[0] = 0.f;
    }
    smem[rho * P + p] = o[0];
  }
  __syncthreads();
  for (int rho = threadIdx.x; rho < nr; rho += blockDim.x) {
    const int r = r0 + rho;
    float v = 0.f;
    for (int p = 0; p < P; p++) v = fadd(v, smem[rho * P + p]);
    out[r] = bias_term ? fadd(v, bias ? bias[r] : 0.f) : v;
  }
}

template <int R>
__global__ void __launch_bounds__(256) matvec_kernel(WDesc W, const Q8Dev* __restrict__ xq8, const float* __restrict__ x,
                                                     const float* __restrict__ bias, int bias_term,
                                                     float* __restrict__ out, DevStatus* st) {
  extern __shared__ float smem[];
  matvec_rows<R>(W, blockIdx.x * R, xq8, x, bias, bias_term, out, st, smem);
}

// Three matrices against one input in one launch: blocks [0, nb0) take W0's
// rows, the next nb1 W1's, the rest W2's.
struct Matvec3 {
  WDesc W[3];
  const float* bias[3];
  float* out[3];
  int nb[3];
};

template <int R>
__global__ void __launch_bounds__(256) matvec3_kernel(Matvec3 a, const Q8Dev* __restrict__ xq8,
                                                      const float* __restrict__ x, int bias_term, DevStatus* st) {
  extern __shared__ float smem[];
  int b = blockIdx.x, m = 0;
  while (m < 2 && b >= a.nb[m]) b -= a.nb[m++];
  matvec_rows<R>(a.W[m], b * R, xq8, x, a.bias[m], bias_term, a.out[m], st, smem);
}

__global__ void f32_matvec_kernel(const float* __restrict__ A, const float* __restrict__ x, float* __restrict__ out,
                                  int nrows, int ncols) {
  const int r = blockIdx.x * blockDim.x + threadIdx.x;
  if (r >= nrows) return;
  const float* row = A + (size_t)r * ncols;
  float a0[4] = {0.f, 0.f, 0.f, 0.f}, a1[4] = {0.f, 0.f, 0.f, 0.f};
  int i = 0;
  for (; i + 7 < ncols; i += 8) {
#pragma unroll
    for (int l = 0; l < 4; l++) {
      a0[l] = __fmaf_rn(row[i + l], x[i + l], a0[l]);
      a1[l] = __fmaf_rn(row[i + 4 + l], x[i + 4 + l], a1[l]);
    }
  }
  float s[4];
#pragma unroll
  for (int l = 0; l < 4; l++) s[l] = fadd(a0[l], a1[l]);
  float sum = fadd(fadd(s[0], s[1]), fadd(s[2], s[3]));
  for (; i < ncols; i++) sum = fadd(sum, fmul(row[i], x[i]));
  out[r] = sum;
}

__global__ void f16_matvec_kernel(const uint16_t* __restrict__ A, const float* __restrict__ x, float* __restrict__ out,
                                  int nrows, int ncols) {
  const int r = blockIdx.x * blockDim.x + threadIdx.x;
  if (r >= nrows) return;
  out[r] = dot_f16_row(A + (size_t)r * ncols, x, ncols);
}

// RMSNorm (680-698): 4 fused lane chains over i % 4, pairwise sum, scalar
// tail; scale = 1/sqrtf(ss/dim + eps); out = (x * scale) * w.
__global__ void rms_norm_kernel(const float* __restrict__ x, const float* __restrict__ w, float* __restrict__ out,
                                int dim, float eps) {
  __shared__ float lanes[4];
  __shared__ float scale_s;
  const int t = threadIdx.x;
  const int dim4 = dim & ~3;
  if (t < 4) {
    float a = 0.f;
    for (int i = t; i < dim4; i += 4) a = __fmaf_rn(x[i], x[i], a);
    lanes[t] = a;
  }
  __syncthreads();
  if (t == 0) {
    float ss = fadd(fadd(lanes[0], lanes[1]), fadd(lanes[2], lanes[3]));
    for (int i = dim4; i < dim; i++) ss = fadd(ss, fmul(x[i], x[i]));
    scale_s = __fdiv_rn(1.f, __fsqrt_rn(fadd(__fdiv_rn(ss, (float)dim), eps)));
  }
  __syncthreads();
  const float sc = scale_s;
  for (int i = t; i < dim; i += blockDim.x) out[i] = fmul(fmul(x[i], sc), w[i]);
}

__global__ void add_kernel(const float* __restrict__ a, const float* __restrict__ b, float* out, size_t n) {
  const size_t i = (size_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (i < n) out[i] = fadd(a[i], b[i]);
}

// Raw blocks (rows x nb of the reference's layout) -> the row layout of
// WDesc; one thread per block, the row's first block also zeroes its padding.
__global__ void repack_kernel(const uint8_t* __restrict__ raw, int fmt, int rows, int cols, uint8_t* __restrict__ dst) {
  const RowLayout L = row_layout(fmt, cols);
  const int nb = (fmt == FMT_Q6K) ? cols / QK : cols / 32;
  const long i = (long)blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= (long)rows * nb) return;
  const long row = i / nb;
  const int b = (int)(i - row * nb);
  uint8_t* d = dst + row * L.rs;
  int used = 0;
  if (fmt == FMT_Q6K) {
    const uint8_t* s = raw + i * Q6K_BYTES;
    for (int j = 0; j < 192; j++) d[b * 192 + j] = s[j];
    for (int j = 0; j < 16; j++) d[L.a1 + b * 16 + j] = s[192 + j];
    d[L.a2 + b * 2] = s[208];
    d[L.a2 + b * 2 + 1] = s[209];
    used = nb * Q6K_BYTES;
  } else if (fmt == FMT_MXFP4) {
    const uint8_t* s = raw + i * MXFP4_BYTES;
    d[L.a1 + b] = s[0];
    for (int j = 0; j < 16; j++) d[b * 16 + j] = s[1 + j];
    used = nb * MXFP4_BYTES;
  } else if (fmt == FMT_Q80) {
    const uint8_t* s = raw + i * Q80_BYTES;
    d[L.a2 + b * 2] = s[0];
    d[L.a2 + b * 2 + 1] = s[1];
    for (int j = 0; j < 32; j++) d[b * 32 + j] = s[2 + j];
    used = nb * Q80_BYTES;
  }
  if (b == 0)
    for (int j = used; j < L.rs; j++) d[j] = 0;
}

// Test hook: the exact int32 sub-block sums of every row of W against one
// Q8 input, in the reference's order (per row: Q4_K 8 per block, Q6_K 16 per
// block, MXFP4/Q8_0 1 per 32 values).  One thread per (row, block).
__global__ void debug_isums_kernel(WDesc W, const Q8Dev* __restrict__ xq, int32_t* __restrict__ out) {
  const int units = terms_per_row(W.fmt, W.cols);
  const long i = (long)blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= (long)W.rows * units) return;
  const int r = (int)(i / units), p = (int)(i % units);
  if (W.fmt == FMT_Q4K) {
    uint32_t w[36];
    load_words(W.main + (size_t)r * W.rs + (size_t)p * Q4K_BYTES, w, 9);
    int is[8];
    q4k_isums(w, reinterpret_cast<const int*>(xq[p].qs), is);
    for (int j = 0; j < 8; j++) out[i * 8 + j] = is[j];
  } else if (W.fmt == FMT_Q6K) {
    uint32_t w[48];
    load_words(W.main + (size_t)r * W.rs + (size_t)p * 192, w, 12);
    int is[16];
    q6k_isums(w, reinterpret_cast<const int*>(xq[p].qs), is);
    for (int j = 0; j < 16; j++) out[i * 16 + j] = is[j];
  } else if (W.fmt == FMT_MXFP4) {
    uint4 cv = ldg16(W.main + (size_t)r * W.rs + (size_t)p * 16);
    uint32_t cw[4] = {cv.x, cv.y, cv.z, cv.w};
    out[i] = mxfp4_isum(cw, reinterpret_cast<const int*>(xq[p >> 3].qs) + (p & 7) * 8);
  } else if (W.fmt == FMT_Q80) {
    const uint8_t* q = W.main + (size_t)r * W.rs + (size_t)p * 32;
    uint4 a = ldg16(q), b = ldg16(q + 16);
    int qw[8] = {(int)a.x, (int)a.y, (int)a.z, (int)a.w, (int)b.x, (int)b.y, (int)b.z, (int)b.w};
    out[i] = q80_isum(qw, reinterpret_cast<const int*>(xq[p >> 3].qs) + (p & 7) * 8);
  }
}

// ---------------------------------------------------------------------
// Launchers.

static constexpr int MV_R = 32;

void launch_quantize_rows(const float* x, int nrows, int ncols, long ldx, Q8Dev* out, cudaStream_t s) {
  const int nb = (ncols + QK - 1) / QK;
  if (nrows <= 0 || nb <= 0) return;
  quantize_rows_kernel<<<dim3(nb, nrows), 256, 0, s>>>(x, ncols, ldx, out, nb);
}

cudaError_t launch_matvec(const WDesc& W, const Q8Dev* xq8, const float* x, const float* bias, int bias_term,
                          float* out, DevStatus* st, cudaStream_t s) {
  const int P = W.fmt == FMT_F16 ? 1 : terms_per_row(W.fmt, W.cols);
  const size_t smem = sizeof(float) * (size_t)MV_R * P;
  auto k = matvec_kernel<MV_R>;
  cudaError_t e = ensure_smem(reinterpret_cast<const void*>(k), smem);
  if (e != cudaSuccess) return e;
  k<<<(W.rows + MV_R - 1) / MV_R, 256, smem, s>>>(W, xq8, x, bias, bias_term, out, st);
  return cudaGetLastError();
}

cudaError_t launch_matvec3(const WDesc* W, const float* const* bias, float* const* out, const Q8Dev* xq8,
                           const float* x, int bias_term, DevStatus* st, cudaStream_t s) {
  Matvec3 a{};
  size_t smem = 0;
  int blocks = 0;
  for (int m = 0; m < 3; m++) {
    a.W[m] = W[m];
    a.bias[m] = bias[m];
    a.out[m] = out[m];
    a.nb[m] = (W[m].rows + MV_R - 1) / MV_R;
    blocks += a.nb[m];
    const int P = W[m].fmt == FMT_F16 ? 1 : terms_per_row(W[m].fmt, W[m].cols);
    smem = std::max(smem, sizeof(float) * (size_t)MV_R * P);
  }
  auto k = matvec3_kernel<MV_R>;
  cudaError_t e = ensure_smem(reinterpret_cast<const void*>(k), smem);
  if (e != cudaSuccess) return e;
  k<<<blocks, 256, smem, s>>>(a, xq8, x, bias_term, st);
  return cudaGetLastError();
}

void launch_f32_matvec(const float* A, const float* x, float* out, int nrows, int ncols, cudaStream_t s) {
  f32_matvec_kernel<<<(nrows + 127) / 128, 128, 0, s>>>(A, x, out, nrows, ncols);
}

void launch_f16_matvec(const uint16_t* A, const float* x, float* out, int nrows, int ncols, cudaStream_t s) {
  f16_matvec_kernel<<<(nrows + 127) / 128, 128, 0, s>>>(A, x, out, nrows, ncols);
}

void launch_add(const float* a, const float* b, float* out, size_t n, cudaStream_t s) {
  if (n) add_kernel<<<(unsigned)((n + 255) / 256), 256, 0, s>>>(a, b, out, n);
}

void launch_rms_norm(const float* x, const float* w, float* out, int dim, float eps, cudaStream_t s) {
  rms_norm_kernel<<<1, 256, 0, s>>>(x, w, out, dim, eps);
}

int debug_isums_per_row(int fmt, int cols) {
  const int u = terms_per_row(fmt, cols);
  return fmt == FMT_Q4K ? 8 * u : fmt == FMT_Q6K ? 16 * u : u;
}

void launch_debug_isums(const WDesc& W, const Q8Dev* xq, int32_t* out, cudaStream_t s) {
  const long n = (long)W.rows * terms_per_row(W.fmt, W.cols);
  debug_isums_kernel<<<(unsigned)((n + 127) / 128), 128, 0, s>>>(W, xq, out);
}

void launch_repack(const uint8_t* raw, int fmt, int rows, int cols, uint8_t* dst, cudaStream_t s) {
  const long nblocks = (long)rows * ((fmt == FMT_Q6K) ? cols / QK : cols / 32);
  if (nblocks <= 0) return;
  repack_kernel<<<(unsigned)((nblocks + 255) / 256), 256, 0, s>>>(raw, fmt, rows, cols, dst);
}

// Test hook: div_rn_d (the double-assisted exact division of the fused step)
// against __fdiv_rn on n pseudo-random operand pairs; counts mismatches.
// Half the dividends and divisors have exponents in 2^-30 .. 2^30, the rest
// any bit pattern (divisors positive).
__device__ __forceinline__ uint32_t mix32(uint32_t x) {
  x ^= x >> 16;
  x *= 0x7feb352du;
  x ^= x >> 15;
  x *= 0x846ca68bu;
  x ^= x >> 16;
  return x;
}

__global__ void debug_div_kernel(long long n, uint32_t seed, unsigned long long* bad) {
  unsigned long long nb = 0;
  for (long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x; i < n; i += (long long)gridDim.x * blockDim.x) {
    const uint32_t h1 = mix32((uint32_t)i * 2654435761u ^ seed), h2 = mix32(h1 ^ 0x9e3779b9u), h3 = mix32(h2 ^ seed);
    uint32_t xb = h1, db = h2 & 0x7fffffffu;
    if (h3 & 1u) db = (db & 0x007fffffu) | ((97u + (h3 >> 8) % 61u) << 23);
    if (h3 & 2u) xb = (xb & 0x807fffffu) | ((97u + (h3 >> 16) % 61u) << 23);
    const float x = __uint_as_float(xb), d = __uint_as_float(db);
    if (!(d > 0.f)) continue;
    const float got = div_rn_d(x, d, 1.0 / (double)d), want = __fdiv_rn(x, d);
    if (__float_as_uint(got) != __float_as_uint(want) && !(got != got && want != want)) nb++;
  }
  if (nb) atomicAdd(bad, nb);
}

void launch_debug_div(long long n, uint32_t seed, unsigned long long* bad, cudaStream_t s) {
  debug_div_kernel<<<148 * 4, 256, 0, s>>>(n, seed, bad);
}

}  // namespace tg
