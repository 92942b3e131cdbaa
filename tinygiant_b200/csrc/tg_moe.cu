// tg_moe.cu — the two expert phases of one MoE call (sm_100a).
//
//   moe_gateup_kernel : gate.x, up.x (+ biases), activation -> hidden, and the
//                       Q8 re-quantization of hidden   (moe_phase_a, csrc/libtinygiant.c:1279-1327,
//                                                       plus the quantize in moe_phase_b 1356-1360)
//   moe_down_kernel   : down.hidden, part = w * (v + bias), ordered combine
//                                                      (moe_phase_b 1329-1384, combine 1428-1434)
//
// Float results follow the reference's association exactly (tg_dots.cuh);
// the combine adds each expert's part into an output element in the call's
// expert order, as the reference's serial loop does.
#include "tg_dots.cuh"
#include "tg_moe.h"
#include "tg_q8.cuh"

namespace tg {

constexpr int GU_R = 16;   // rows of I per gate/up tile (divides 256)
constexpr int DN_R = 16;   // rows of D per down CTA
constexpr int DN_CH = 8;   // active rows per down chunk

// ---------------------------------------------------------------------
// Phase A: CTA = (tile of GU_R rows of I, slot).  For each group of <= 4
// active rows: every (matrix, row, term) unit computes its outer terms, one
// thread per (matrix, row, token) folds them in order, then the biases and
// the activation produce hidden[active row][r].  The last CTA to finish a
// 256-row block of a slot's hidden rows quantizes that block (Q8) for phase B.

__global__ void __launch_bounds__(256) moe_gateup_kernel(const PlanHdr* __restrict__ ph,
                                                         const Q8Dev* __restrict__ xq8, int gbpr,
                                                         float* __restrict__ hidden, Q8Dev* __restrict__ hq8,
                                                         int dbpr, int* __restrict__ counters, DevStatus* st) {
  extern __shared__ float smem[];
  __shared__ Q8Scratch qsh;
  __shared__ int last_flag;
  const int s = blockIdx.y;
  if (s >= ph->n_slots) return;
  const SlotDesc S = ph->slots[s];
  const int I = ph->inter_dim, D = ph->embed_dim, k = ph->k, rule = ph->assoc_rule, act = ph->act;
  const int r0 = blockIdx.x * GU_R;
  if (r0 >= I || S.n_rows == 0) return;
  const int nr = min(GU_R, I - r0);
  const int fmt = S.gate.fmt;
  if (fmt == FMT_F16 || fmt < 0 || fmt > FMT_Q80 || S.up.fmt != fmt) {
    if (threadIdx.x == 0) set_error(st, ERR_BAD_FORMAT, 1, fmt, s);
    return;
  }
  const int P = terms_per_row(fmt, D);
  float* terms = smem;                    // [2][R][4][P]
  float* tot = terms + 2 * GU_R * 4 * P;  // [2][R][4]
  for (int g0 = 0; g0 < S.n_rows; g0 += 4) {
    const int ng = min(4, S.n_rows - g0);
    const bool x4 = use_x4(rule, g0, S.n_rows, k);
    const Q8Dev* xrow[4];
    for (int j = 0; j < 4; j++) xrow[j] = xq8 + (size_t)ph->rows[S.row_off + g0 + min(j, ng - 1)] * gbpr;
    const int nunits = 2 * nr * P;
    for (int u = threadIdx.x; u < nunits; u += blockDim.x) {
      const int m = u / (nr * P), rem = u - m * nr * P, rho = rem / P, p = rem - rho * P;
      float o[4];
      row_terms(m ? S.up : S.gate, r0 + rho, p, xrow, ng, x4, o);
      for (int j = 0; j < ng; j++) terms[((m * GU_R + rho) * 4 + j) * P + p] = o[j];
    }
    __syncthreads();
    for (int f = threadIdx.x; f < 2 * nr * ng; f += blockDim.x) {
      const int m = f / (nr * ng), rem = f - m * nr * ng, rho = rem / ng, j = rem - rho * ng;
      const float* tp = terms + ((m * GU_R + rho) * 4 + j) * P;
      float acc = 0.f;
      for (int p = 0; p < P; p++) acc = fadd(acc, tp[p]);
      tot[(m * GU_R + rho) * 4 + j] = acc;
    }
    __syncthreads();
    for (int f = threadIdx.x; f < nr * ng; f += blockDim.x) {
      const int rho = f / ng, j = f - rho * ng, r = r0 + rho;
      float gv = tot[(0 * GU_R + rho) * 4 + j], uv = tot[(1 * GU_R + rho) * 4 + j];
      if (S.gb) {
        gv = fadd(gv, S.gb[r]);
        uv = fadd(uv, S.ub[r]);
      }
      hidden[(size_t)(S.row_off + g0 + j) * I + r] = act_fn(act, gv, uv);
    }
    __syncthreads();
  }

  // Last-arriver quantization of the 256-row block of hidden this tile is in.
  const int kb = r0 / QK;
  const int blk_rows = min(QK, I - kb * QK);
  const int tiles_in_blk = (blk_rows + GU_R - 1) / GU_R;
  if (threadIdx.x == 0) {
    __threadfence();
    int* c = counters + (size_t)s * dbpr + kb;
    const int prev = atomicAdd(c, 1);
    last_flag = prev == tiles_in_blk - 1;
    if (last_flag) *c = 0;   // every tile of this block has arrived: reset for the next call
  }
  __syncthreads();
  if (!last_flag) return;
  __threadfence();
  const int t = threadIdx.x;
  for (int j = 0; j < S.n_rows; j++) {
    const size_t row = (size_t)(S.row_off + j);
    const bool valid = t < blk_rows;
    const float v = valid ? __ldcg(hidden + row * I + (size_t)kb * QK + t) : 0.f;
    quantize_block_cta(v, valid, hq8 + row * dbpr + kb, qsh);
  }
}

// ---------------------------------------------------------------------
// Phase B: CTA = DN_R consecutive output rows of D, all active (slot, row)
// pairs, in chunks of DN_CH: unit terms, per-(active row, row) fold,
// part = w * (v + bias), then the combine adds parts into the output in the
// flat active-row order, which is the reference's expert order.

__global__ void __launch_bounds__(256) moe_down_kernel(const PlanHdr* __restrict__ ph,
                                                       const Q8Dev* __restrict__ hq8, int dbpr,
                                                       const float* __restrict__ hidden, float* __restrict__ out,
                                                       DevStatus* st) {
  extern __shared__ float smem[];
  const int D = ph->embed_dim, I = ph->inter_dim, total = ph->total_rows, k = ph->k, rule = ph->assoc_rule;
  const int bias_term = ph->bias_term;
  const SlotDesc* slots = ph->slots;
  const int* rows = ph->rows;
  const int* row_slot = ph->row_slot;
  const float* wts = ph->wts;
  const int r0 = blockIdx.x * DN_R;
  if (r0 >= D) return;
  const int nr = min(DN_R, D - r0);
  const int Pmax = max(1, I / 32);
  float* terms = smem;                         // [CH][R][Pmax]
  float* parts = terms + DN_CH * DN_R * Pmax;  // [CH][R]
  for (int c0 = 0; c0 < total; c0 += DN_CH) {
    const int nch = min(DN_CH, total - c0);
    const int nunits = nch * nr * Pmax;
    for (int u = threadIdx.x; u < nunits; u += blockDim.x) {
      const int i = u / (nr * Pmax), rem = u - i * nr * Pmax, rho = rem / Pmax, p = rem - rho * Pmax;
      const int sr = c0 + i;
      const SlotDesc& S = slots[row_slot[sr]];
      const int fmt = S.down.fmt;
      if (fmt == FMT_F16 || p >= terms_per_row(fmt, I)) continue;
      const bool x4 = use_x4(rule, sr - S.row_off, S.n_rows, k);
      const Q8Dev* xrow[1] = {hq8 + (size_t)sr * dbpr};
      float o[1];
      if (!row_terms(S.down, r0 + rho, p, xrow, 1, x4, o)) {
        set_error(st, ERR_BAD_FORMAT, 2, fmt, row_slot[sr]);
        o[0] = 0.f;
      }
      terms[(i * DN_R + rho) * Pmax + p] = o[0];
    }
    __syncthreads();
    for (int f = threadIdx.x; f < nch * nr; f += blockDim.x) {
      const int i = f / nr, rho = f - i * nr, sr = c0 + i, r = r0 + rho;
      const SlotDesc& S = slots[row_slot[sr]];
      float v;
      if (S.down.fmt == FMT_F16) {
        v = dot_f16_row(reinterpret_cast<const uint16_t*>(S.down.main) + (size_t)r * I, hidden + (size_t)sr * I, I);
      } else {
        const int P = terms_per_row(S.down.fmt, I);
        const float* tp = terms + (i * DN_R + rho) * Pmax;
        v = 0.f;
        for (int p = 0; p < P; p++) v = fadd(v, tp[p]);
      }
      const float w = wts[sr];
      parts[i * DN_R + rho] = bias_term ? fmul(w, fadd(v, S.db ? S.db[r] : 0.f)) : fmul(w, v);
    }
    __syncthreads();
    for (int rho = threadIdx.x; rho < nr; rho += blockDim.x) {
      for (int i = 0; i < nch; i++) {
        float* o = out + (size_t)rows[c0 + i] * D + r0 + rho;
        *o = fadd(*o, parts[i * DN_R + rho]);
      }
    }
    __syncthreads();
  }
}

// ---------------------------------------------------------------------
// Launchers.

cudaError_t launch_moe_gateup(const PlanHdr* ph, int max_slots, int gate_fmt, int D, int I, const Q8Dev* xq8,
                              float* hidden, Q8Dev* hq8, int* counters, DevStatus* st, cudaStream_t s) {
  if (max_slots <= 0) return cudaSuccess;
  const int P = terms_per_row(gate_fmt, D);
  const size_t smem = sizeof(float) * (size_t)(2 * GU_R * 4 * P + 2 * GU_R * 4);
  cudaError_t e = ensure_smem(reinterpret_cast<const void*>(moe_gateup_kernel), smem);
  if (e != cudaSuccess) return e;
  const int gbpr = (D + QK - 1) / QK, dbpr = (I + QK - 1) / QK;
  dim3 grid((I + GU_R - 1) / GU_R, max_slots);
  moe_gateup_kernel<<<grid, 256, smem, s>>>(ph, xq8, gbpr, hidden, hq8, dbpr, counters, st);
  return cudaGetLastError();
}

cudaError_t launch_moe_down(const PlanHdr* ph, int D, int I, const Q8Dev* hq8, const float* hidden, float* out,
                            DevStatus* st, cudaStream_t s) {
  const int Pmax = I / 32 > 1 ? I / 32 : 1;
  const size_t smem = sizeof(float) * (size_t)(DN_CH * DN_R * Pmax + DN_CH * DN_R);
  cudaError_t e = ensure_smem(reinterpret_cast<const void*>(moe_down_kernel), smem);
  if (e != cudaSuccess) return e;
  const int dbpr = (I + QK - 1) / QK;
  moe_down_kernel<<<(D + DN_R - 1) / DN_R, 256, smem, s>>>(ph, hq8, dbpr, hidden, out, st);
  return cudaGetLastError();
}

size_t moe_counter_ints(int max_slots, int I) { return (size_t)max_slots * ((I + QK - 1) / QK); }

}  // namespace tg
