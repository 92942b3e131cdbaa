// tg_route.cu — one layer's routing on the GPU, fused into a single kernel.
//
// For T rows of the residual stream x:
//   x' = x + add (the previous layer's MoE output, when given)       engine.py:341
//   N  = x' / sqrt(mean(x'^2) + eps) * w                             engine.py:281-282
//   logits = W_r N (+ b)                                             router.py:29-33
//   top-k by descending logit, softmax over the selected logits      router.py:35-42
//   union of selected experts ascending by id, active rows in token
//   order with their weights (a zero weight is inactive)             engine.py:297-318,
//                                                                    libtinygiant.c:1411-1423
// and the Q8 blocks of N (libtinygiant.c:1408-1410).  CTAs split the experts
// (one warp per expert); the last CTA to finish selects and builds the plan
// that the expert kernels read, so no host round trip is needed.
//
// Float order: the norm and the logit dots reduce in a fixed order (warp
// trees), which differs from numpy's; routing agrees with the reference
// except where two logits tie to within rounding.
#include "tg_moe.h"
#include "tg_q8.cuh"

namespace tg {

constexpr int RT_WARPS = 8;   // experts per CTA
constexpr int RT_TC = 8;      // token rows per smem chunk

__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}

__global__ void __launch_bounds__(256) layer_route_kernel(RouteArgs a) {
  extern __shared__ float sm[];
  __shared__ Q8Scratch qsh;
  __shared__ float red[RT_WARPS];
  __shared__ int last_flag;
  const int T = a.T, D = a.D, E = a.E, t = threadIdx.x, lane = t & 31, w = t >> 5;
  const int gbpr = (D + QK - 1) / QK;
  float* xs = sm;   // [RT_TC][D]
  const int e = blockIdx.x * RT_WARPS + w;
  for (int t0 = 0; t0 < T; t0 += RT_TC) {
    const int nt = min(RT_TC, T - t0);
    for (int i = t; i < nt * D; i += blockDim.x) {
      const size_t gi = (size_t)t0 * D + i;
      float v = a.x_in[gi];
      if (a.add_in) v = fadd(v, a.add_in[gi]);
      xs[i] = v;
      if (blockIdx.x == 0 && a.x_out) a.x_out[gi] = v;
    }
    __syncthreads();
    if (a.normalize) {
      for (int tt = 0; tt < nt; tt++) {
        float ss = 0.f;
        for (int i = t; i < D; i += blockDim.x) ss = __fmaf_rn(xs[tt * D + i], xs[tt * D + i], ss);
        ss = warp_sum(ss);
        if (lane == 0) red[w] = ss;
        __syncthreads();
        float tot = 0.f;
#pragma unroll
        for (int j = 0; j < RT_WARPS; j++) tot = fadd(tot, red[j]);
        const float rr = __fsqrt_rn(fadd(__fdiv_rn(tot, (float)D), a.eps));
        for (int i = t; i < D; i += blockDim.x) {
          float v = __fdiv_rn(xs[tt * D + i], rr);
          if (a.norm_w) v = fmul(v, a.norm_w[i]);
          xs[tt * D + i] = v;
        }
        __syncthreads();
      }
    }
    // Q8 blocks of the normalized rows (CTA 0).
    if (blockIdx.x == 0) {
      for (int tt = 0; tt < nt; tt++)
        for (int b = 0; b < gbpr; b++) {
          const int n = min(QK, D - b * QK);
          const bool valid = t < n;
          quantize_block_cta(valid ? xs[tt * D + b * QK + t] : 0.f, valid, a.xq8 + (size_t)(t0 + tt) * gbpr + b, qsh);
        }
    }
    // Logits: one warp per expert.
    if (e < E) {
      const float* wr = a.router_w + (size_t)e * D;
      for (int tt = 0; tt < nt; tt++) {
        float acc = 0.f;
        for (int i = lane; i < D; i += 32) acc = __fmaf_rn(__ldg(wr + i), xs[tt * D + i], acc);
        acc = warp_sum(acc);
        if (lane == 0) a.logits[(size_t)(t0 + tt) * E + e] = a.router_b ? fadd(acc, a.router_b[e]) : acc;
      }
    }
    __syncthreads();
  }
  if (blockIdx.x == 0 && a.zero_out)
    for (size_t i = t; i < (size_t)T * D; i += blockDim.x) a.zero_out[i] = 0.f;

  // The last CTA to finish selects experts and builds the plan.
  if (t == 0) {
    __threadfence();
    const int prev = atomicAdd(a.counter, 1);
    last_flag = prev == (int)gridDim.x - 1;
    if (last_flag) *a.counter = 0;
  }
  __syncthreads();
  if (!last_flag) return;
  __threadfence();

  const int K = a.top_k;
  int* cnt = reinterpret_cast<int*>(sm);   // [E]
  int* off = cnt + E;                      // [E]
  int* slot_of = off + E;                  // [E]
  for (int i = t; i < E; i += blockDim.x) cnt[i] = 0;
  __syncthreads();
  // Selection: one warp per token.
  for (int tok = w; tok < T; tok += RT_WARPS) {
    const float* lg = a.logits + (size_t)tok * E;
    float best_v[8];
    int best_i[8];
    float m0 = 0.f, sum = 0.f;
    for (int j = 0; j < K; j++) {
      float bv = -INFINITY;
      int bi = 0x7fffffff;
      for (int i = lane; i < E; i += 32) {
        bool taken = false;
        for (int q = 0; q < j; q++) taken |= (best_i[q] == i);
        const float v = __ldcg(lg + i);
        if (!taken && (v > bv || (v == bv && i < bi))) {
          bv = v;
          bi = i;
        }
      }
#pragma unroll
      for (int o = 16; o > 0; o >>= 1) {
        const float ov = __shfl_xor_sync(0xffffffffu, bv, o);
        const int oi = __shfl_xor_sync(0xffffffffu, bi, o);
        if (ov > bv || (ov == bv && oi < bi)) {
          bv = ov;
          bi = oi;
        }
      }
      if (bi >= E) {
        // no candidate compared greater (NaN logits): take the lowest
        // untaken index with weight 0, so every index stays in range
        bv = -INFINITY;
        bi = 0;
        for (bool hit = true; hit && bi < E;) {
          hit = false;
          for (int q = 0; q < j; q++) hit |= (best_i[q] == bi);
          if (hit) bi++;
        }
      }
      best_v[j] = bv;
      best_i[j] = bi;
    }
    m0 = best_v[0];
    float ex[8];
    for (int j = 0; j < K; j++) {
      ex[j] = expf(fsub(best_v[j], m0));
      sum = fadd(sum, ex[j]);
    }
    if (lane == 0) {
      for (int j = 0; j < K; j++) {
        const float wt = __fdiv_rn(ex[j], sum);
        a.sel_idx[(size_t)tok * K + j] = best_i[j];
        a.sel_w[(size_t)tok * K + j] = wt;
        // experts held by another GPU (no local weights) are skipped here;
        // their contribution arrives through the cross-GPU sum
        if (wt != 0.f && a.experts[best_i[j]].gate.main) atomicAdd(&cnt[best_i[j]], 1);
      }
    }
  }
  __syncthreads();
  if (t == 0) {
    int ns = 0, o = 0;
    for (int i = 0; i < E; i++) {
      off[i] = o;
      slot_of[i] = cnt[i] ? ns : -1;
      if (cnt[i]) ns++;
      o += cnt[i];
    }
    PlanHdr* h = a.plan;
    h->n_slots = ns;
    h->total_rows = o;
    h->k = T;
    h->embed_dim = D;
    h->inter_dim = a.I;
    h->act = a.act;
    h->assoc_rule = a.assoc_rule;
    h->bias_term = a.bias_term;
    h->slots = a.slots;
    h->rows = a.rows;
    h->wts = a.wts;
    h->row_slot = a.row_slot;
  }
  __syncthreads();
  for (int ex_i = t; ex_i < E; ex_i += blockDim.x) {
    const int c = cnt[ex_i];
    if (!c) continue;
    int o = off[ex_i];
    const int sl = slot_of[ex_i];
    for (int tok = 0; tok < T; tok++)
      for (int j = 0; j < K; j++) {
        const float wt = a.sel_w[(size_t)tok * K + j];
        if (a.sel_idx[(size_t)tok * K + j] == ex_i && wt != 0.f) {  // cnt > 0 implies the expert is local
          a.rows[o] = tok;
          a.wts[o] = wt;
          a.row_slot[o] = sl;
          o++;
        }
      }
    const ExpertDesc& X = a.experts[ex_i];
    SlotDesc d;
    d.gate = X.gate;
    d.up = X.up;
    d.down = X.down;
    d.gb = X.gb;
    d.ub = X.ub;
    d.db = X.db;
    d.n_rows = c;
    d.row_off = off[ex_i];
    d.pad[0] = ex_i;
    d.pad[1] = 0;
    a.slots[sl] = d;
  }
}

size_t route_smem_bytes(int D, int E) {
  const size_t xs = sizeof(float) * (size_t)RT_TC * D, sel = sizeof(int) * 3 * (size_t)E;
  return xs > sel ? xs : sel;
}

cudaError_t launch_layer_route(const RouteArgs& a, cudaStream_t s) {
  if (a.top_k < 1 || a.top_k > 8 || a.top_k > a.E) return cudaErrorInvalidValue;
  const size_t smem = route_smem_bytes(a.D, a.E);
  cudaError_t e = ensure_smem(reinterpret_cast<const void*>(layer_route_kernel), smem);
  if (e != cudaSuccess) return e;
  layer_route_kernel<<<(a.E + RT_WARPS - 1) / RT_WARPS, 256, smem, s>>>(a);
  return cudaGetLastError();
}

}  // namespace tg
