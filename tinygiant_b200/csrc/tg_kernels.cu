// tg_kernels.cu — CUDA kernels of the fused quantized expert path (sm_100a).
//
//   quantize_rows_kernel   fp32 rows -> Q8 blocks      (csrc/libtinygiant.c:169-208)
//   moe_gateup_kernel      gate.x, up.x, act -> hidden (moe_phase_a, 1279-1327)
//   moe_down_kernel        down.h * w (+bias), combine (moe_phase_b + 1428-1434)
//   matvec_kernel          one matrix . one input      (mm_task / gmm_task, 345-364, 906-931)
//   f16/f32 matvec, rms_norm, repack
//
// Each output element is produced by the same sequence of rounded float
// operations as the reference (see tg_dots.cuh); the order-free parts
// (integer sub-block sums, max|x|) run in parallel.
#include <cuda_fp16.h>

#include "tg_dots.cuh"
#include "tg_kernels.h"
#include "tg_plan.cuh"

namespace tg {

// ---------------------------------------------------------------------
// Q8 quantizer: one CTA of 256 threads per 256-block.

__device__ __forceinline__ float max_nan(float a, float b) {
  if (a != a) return a;
  if (b != b) return b;
  return a > b ? a : b;
}

__global__ void __launch_bounds__(256) quantize_rows_kernel(const float* __restrict__ x, int ncols, long ldx,
                                                            Q8Dev* __restrict__ out, int nb) {
  __shared__ float wmax[8];
  __shared__ int wsum[8];
  const int b = blockIdx.x, row = blockIdx.y, t = threadIdx.x, lane = t & 31, w = t >> 5;
  const int n = min(QK, ncols - b * QK);
  const float v = t < n ? x[(size_t)row * ldx + (size_t)b * QK + t] : 0.f;
  float a = t < n ? fabsf(v) : 0.f;
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) a = max_nan(a, __shfl_xor_sync(0xffffffffu, a, o));
  if (lane == 0) wmax[w] = a;
  __syncthreads();
  float amax = wmax[0];
#pragma unroll
  for (int i = 1; i < 8; i++) amax = max_nan(amax, wmax[i]);
  const float sc = __fdiv_rn(amax, 127.f);
  const float inv = amax > 0.f ? __fdiv_rn(127.f, amax) : 0.f;
  int q = 0;
  if (t < n) {
    float s = __fmul_rn(v, inv);
    q = (s != s) ? 0 : __float2int_rn(s);
  }
  int bs = q;
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) bs += __shfl_xor_sync(0xffffffffu, bs, o);
  Q8Dev* o = out + (size_t)row * nb + b;
  o->qs[t] = (int8_t)q;
  if (lane == 0) {
    wsum[w] = bs;
    o->bsums[w] = bs;
  }
  __syncthreads();
  if (t == 0) {
    int total = 0;
#pragma unroll
    for (int i = 0; i < 8; i++) total += wsum[i];
    o->scale = sc;
    o->sum = total;
  }
}

// ---------------------------------------------------------------------
// Phase A: CTA = (tile of R rows of I, slot).  For each group of <= 4 active
// rows: every (matrix, row, term) unit computes its outer terms, one thread
// per (matrix, row, token) folds them in order, then gate/up biases and the
// activation produce hidden[active row][r].

template <int R>
__global__ void __launch_bounds__(256) moe_gateup_kernel(MoePlan plan, const Q8Dev* __restrict__ xq8, int gbpr,
                                                         float* __restrict__ hidden, DevStatus* st) {
  extern __shared__ float smem[];
  const int s = blockIdx.y;
  const SlotDesc S = plan.slots[s];
  const int I = plan.inter_dim, D = plan.embed_dim;
  const int r0 = blockIdx.x * R;
  if (r0 >= I || S.n_rows == 0) return;
  const int nr = min(R, I - r0);
  const int fmt = S.gate.fmt;
  if (fmt == FMT_F16 || fmt < 0 || fmt > FMT_Q80 || S.up.fmt != fmt) {
    if (threadIdx.x == 0) set_error(st, ERR_BAD_FORMAT, 1, fmt, s);
    return;
  }
  const int P = terms_per_row(fmt, D);
  float* terms = smem;                 // [2][R][4][P]
  float* tot = terms + 2 * R * 4 * P;  // [2][R][4]
  for (int g0 = 0; g0 < S.n_rows; g0 += 4) {
    const int ng = min(4, S.n_rows - g0);
    const bool x4 = use_x4(plan.assoc_rule, g0, S.n_rows, plan.k);
    const Q8Dev* xrow[4];
    for (int j = 0; j < 4; j++) xrow[j] = xq8 + (size_t)plan.rows[S.row_off + g0 + min(j, ng - 1)] * gbpr;
    const int nunits = 2 * nr * P;
    for (int u = threadIdx.x; u < nunits; u += blockDim.x) {
      const int m = u / (nr * P), rem = u - m * nr * P, rho = rem / P, p = rem - rho * P;
      float o[4];
      row_terms(m ? S.up : S.gate, r0 + rho, p, xrow, ng, x4, o);
      for (int j = 0; j < ng; j++) terms[((m * R + rho) * 4 + j) * P + p] = o[j];
    }
    __syncthreads();
    for (int f = threadIdx.x; f < 2 * nr * ng; f += blockDim.x) {
      const int m = f / (nr * ng), rem = f - m * nr * ng, rho = rem / ng, j = rem - rho * ng;
      const float* tp = terms + ((m * R + rho) * 4 + j) * P;
      float acc = 0.f;
      for (int p = 0; p < P; p++) acc = fadd(acc, tp[p]);
      tot[(m * R + rho) * 4 + j] = acc;
    }
    __syncthreads();
    for (int f = threadIdx.x; f < nr * ng; f += blockDim.x) {
      const int rho = f / ng, j = f - rho * ng, r = r0 + rho;
      float gv = tot[(0 * R + rho) * 4 + j], uv = tot[(1 * R + rho) * 4 + j];
      if (S.gb) {
        gv = fadd(gv, S.gb[r]);
        uv = fadd(uv, S.ub[r]);
      }
      hidden[(size_t)(S.row_off + g0 + j) * I + r] = act_fn(plan.act, gv, uv);
    }
    __syncthreads();
  }
}

// ---------------------------------------------------------------------
// Phase B: CTA = R consecutive output rows of D, all active (slot, row)
// pairs.  Chunks of CH active rows: unit terms, per-(active row, row) fold,
// part = w * (v + bias), then the combine adds parts into the output in the
// flat active-row order, which is the reference's expert order.

template <int R, int CH>
__global__ void __launch_bounds__(256) moe_down_kernel(MoePlan plan, const int* __restrict__ row_slot,
                                                       const Q8Dev* __restrict__ hq8, int dbpr,
                                                       const float* __restrict__ hidden, float* __restrict__ out,
                                                       DevStatus* st) {
  extern __shared__ float smem[];
  const int D = plan.embed_dim, I = plan.inter_dim;
  const int r0 = blockIdx.x * R;
  if (r0 >= D) return;
  const int nr = min(R, D - r0);
  const int Pmax = I / 32;
  float* terms = smem;                // [CH][R][Pmax]
  float* parts = terms + CH * R * Pmax;  // [CH][R]
  for (int c0 = 0; c0 < plan.total_rows; c0 += CH) {
    const int nch = min(CH, plan.total_rows - c0);
    const int nunits = nch * nr * Pmax;
    for (int u = threadIdx.x; u < nunits; u += blockDim.x) {
      const int i = u / (nr * Pmax), rem = u - i * nr * Pmax, rho = rem / Pmax, p = rem - rho * Pmax;
      const int sr = c0 + i;
      const SlotDesc& S = plan.slots[row_slot[sr]];
      const int fmt = S.down.fmt;
      if (fmt == FMT_F16 || p >= terms_per_row(fmt, I)) continue;
      const bool x4 = use_x4(plan.assoc_rule, sr - S.row_off, S.n_rows, plan.k);
      const Q8Dev* xrow[1] = {hq8 + (size_t)sr * dbpr};
      float o[1];
      if (!row_terms(S.down, r0 + rho, p, xrow, 1, x4, o)) {
        set_error(st, ERR_BAD_FORMAT, 2, fmt, row_slot[sr]);
        o[0] = 0.f;
      }
      terms[(i * R + rho) * Pmax + p] = o[0];
    }
    __syncthreads();
    for (int f = threadIdx.x; f < nch * nr; f += blockDim.x) {
      const int i = f / nr, rho = f - i * nr, sr = c0 + i, r = r0 + rho;
      const SlotDesc& S = plan.slots[row_slot[sr]];
      float v;
      if (S.down.fmt == FMT_F16) {
        v = dot_f16_row(reinterpret_cast<const uint16_t*>(S.down.main) + (size_t)r * I, hidden + (size_t)sr * I, I);
      } else {
        const int P = terms_per_row(S.down.fmt, I);
        const float* tp = terms + (i * R + rho) * Pmax;
        v = 0.f;
        for (int p = 0; p < P; p++) v = fadd(v, tp[p]);
      }
      const float w = plan.wts[sr];
      float part;
      if (plan.bias_term) part = fmul(w, fadd(v, S.db ? S.db[r] : 0.f));
      else part = fmul(w, v);
      parts[i * R + rho] = part;
    }
    __syncthreads();
    for (int rho = threadIdx.x; rho < nr; rho += blockDim.x) {
      for (int i = 0; i < nch; i++) {
        float* o = out + (size_t)plan.rows[c0 + i] * D + r0 + rho;
        *o = fadd(*o, parts[i * R + rho]);
      }
    }
    __syncthreads();
  }
}

// ---------------------------------------------------------------------
// One matrix against one input: out[r] = dot (+ (bias ? bias[r] : 0.f)).

template <int R>
__global__ void __launch_bounds__(256) matvec_kernel(WDesc W, const Q8Dev* __restrict__ xq8, const float* __restrict__ x,
                                                     const float* __restrict__ bias, int bias_term,
                                                     float* __restrict__ out, DevStatus* st) {
  extern __shared__ float smem[];
  const int r0 = blockIdx.x * R;
  if (r0 >= W.rows) return;
  const int nr = min(R, W.rows - r0);
  if (W.fmt == FMT_F16) {
    for (int rho = threadIdx.x; rho < nr; rho += blockDim.x) {
      const int r = r0 + rho;
      float v = dot_f16_row(reinterpret_cast<const uint16_t*>(W.main) + (size_t)r * W.cols, x, W.cols);
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

// f32 rows with the reference's lane structure (662-676).
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

// Raw reference blocks -> HBM layout (tg_common.cuh WDesc).
__global__ void repack_kernel(const uint8_t* __restrict__ raw, int fmt, long nblocks, uint8_t* __restrict__ mainp,
                              uint8_t* __restrict__ aux1, uint8_t* __restrict__ aux2) {
  const long i = (long)blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= nblocks) return;
  if (fmt == FMT_Q6K) {
    const uint8_t* b = raw + i * Q6K_BYTES;
    for (int j = 0; j < 192; j++) mainp[i * 192 + j] = b[j];
    for (int j = 0; j < 16; j++) aux1[i * 16 + j] = b[192 + j];
    aux2[i * 2] = b[208];
    aux2[i * 2 + 1] = b[209];
  } else if (fmt == FMT_MXFP4) {
    const uint8_t* b = raw + i * MXFP4_BYTES;
    aux1[i] = b[0];
    for (int j = 0; j < 16; j++) mainp[i * 16 + j] = b[1 + j];
  } else if (fmt == FMT_Q80) {
    const uint8_t* b = raw + i * Q80_BYTES;
    aux2[i * 2] = b[0];
    aux2[i * 2 + 1] = b[1];
    for (int j = 0; j < 32; j++) mainp[i * 32 + j] = b[2 + j];
  }
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
    load_words(W.main + ((size_t)r * units + p) * Q4K_BYTES, w, 9);
    int is[8];
    q4k_isums(w, reinterpret_cast<const int*>(xq[p].qs), is);
    for (int j = 0; j < 8; j++) out[i * 8 + j] = is[j];
  } else if (W.fmt == FMT_Q6K) {
    uint32_t w[48];
    load_words(W.main + ((size_t)r * units + p) * 192, w, 12);
    int is[16];
    q6k_isums(w, reinterpret_cast<const int*>(xq[p].qs), is);
    for (int j = 0; j < 16; j++) out[i * 16 + j] = is[j];
  } else if (W.fmt == FMT_MXFP4) {
    uint4 cv = ldg16(W.main + ((size_t)r * units + p) * 16);
    uint32_t cw[4] = {cv.x, cv.y, cv.z, cv.w};
    out[i] = mxfp4_isum(cw, reinterpret_cast<const int*>(xq[p >> 3].qs) + (p & 7) * 8);
  } else if (W.fmt == FMT_Q80) {
    const uint8_t* q = W.main + ((size_t)r * units + p) * 32;
    uint4 a = ldg16(q), b = ldg16(q + 16);
    int qw[8] = {(int)a.x, (int)a.y, (int)a.z, (int)a.w, (int)b.x, (int)b.y, (int)b.z, (int)b.w};
    out[i] = q80_isum(qw, reinterpret_cast<const int*>(xq[p >> 3].qs) + (p & 7) * 8);
  }
}

// ---------------------------------------------------------------------
// Launchers.

static constexpr int GU_R = 16;
static constexpr int DN_R = 16;
static constexpr int DN_CH = 8;
static constexpr int MV_R = 32;

void launch_quantize_rows(const float* x, int nrows, int ncols, long ldx, Q8Dev* out, cudaStream_t s) {
  const int nb = (ncols + QK - 1) / QK;
  if (nrows <= 0 || nb <= 0) return;
  quantize_rows_kernel<<<dim3(nb, nrows), 256, 0, s>>>(x, ncols, ldx, out, nb);
}

size_t gateup_smem_bytes(int gate_fmt, int D) {
  const int P = terms_per_row(gate_fmt, D);
  return sizeof(float) * (size_t)(2 * GU_R * 4 * P + 2 * GU_R * 4);
}

cudaError_t launch_moe_gateup(const MoePlan& plan, int gate_fmt, const Q8Dev* xq8, int gbpr, float* hidden,
                              DevStatus* st, cudaStream_t s) {
  if (plan.n_slots == 0) return cudaSuccess;
  const size_t smem = gateup_smem_bytes(gate_fmt, plan.embed_dim);
  auto k = moe_gateup_kernel<GU_R>;
  cudaError_t e = cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
  if (e != cudaSuccess) return e;
  dim3 grid((plan.inter_dim + GU_R - 1) / GU_R, plan.n_slots);
  k<<<grid, 256, smem, s>>>(plan, xq8, gbpr, hidden, st);
  return cudaGetLastError();
}

cudaError_t launch_moe_down(const MoePlan& plan, const int* row_slot, const Q8Dev* hq8, int dbpr, const float* hidden,
                            float* out, DevStatus* st, cudaStream_t s) {
  if (plan.total_rows == 0) return cudaSuccess;
  const int Pmax = plan.inter_dim / 32;
  const size_t smem = sizeof(float) * (size_t)(DN_CH * DN_R * Pmax + DN_CH * DN_R);
  auto k = moe_down_kernel<DN_R, DN_CH>;
  cudaError_t e = cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
  if (e != cudaSuccess) return e;
  k<<<(plan.embed_dim + DN_R - 1) / DN_R, 256, smem, s>>>(plan, row_slot, hq8, dbpr, hidden, out, st);
  return cudaGetLastError();
}

cudaError_t launch_matvec(const WDesc& W, const Q8Dev* xq8, const float* x, const float* bias, int bias_term,
                          float* out, DevStatus* st, cudaStream_t s) {
  const int P = W.fmt == FMT_F16 ? 1 : terms_per_row(W.fmt, W.cols);
  const size_t smem = sizeof(float) * (size_t)MV_R * P;
  auto k = matvec_kernel<MV_R>;
  cudaError_t e = cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
  if (e != cudaSuccess) return e;
  k<<<(W.rows + MV_R - 1) / MV_R, 256, smem, s>>>(W, xq8, x, bias, bias_term, out, st);
  return cudaGetLastError();
}

void launch_f32_matvec(const float* A, const float* x, float* out, int nrows, int ncols, cudaStream_t s) {
  f32_matvec_kernel<<<(nrows + 127) / 128, 128, 0, s>>>(A, x, out, nrows, ncols);
}

void launch_f16_matvec(const uint16_t* A, const float* x, float* out, int nrows, int ncols, cudaStream_t s) {
  f16_matvec_kernel<<<(nrows + 127) / 128, 128, 0, s>>>(A, x, out, nrows, ncols);
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

void launch_repack(const uint8_t* raw, int fmt, long nblocks, uint8_t* mainp, uint8_t* aux1, uint8_t* aux2,
                   cudaStream_t s) {
  if (nblocks <= 0) return;
  repack_kernel<<<(unsigned)((nblocks + 255) / 256), 256, 0, s>>>(raw, fmt, nblocks, mainp, aux1, aux2);
}

}  // namespace tg
