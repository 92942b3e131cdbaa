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
// and the Q8 blocks of N (libtinygiant.c:1408-1410).  One CTA per expert
// computes that expert's logits (its 8 KB router row is read once); the last
// CTA to finish selects the experts and writes the plan the expert kernels
// read, so the step needs no host round trip.
//
// Float order: the norm and the logit dots reduce in a fixed order (warp
// trees), not numpy's; routing agrees with the reference except where two
// logits tie to within rounding.
#include "tg_moe.h"
#include "tg_ptx.cuh"
#include "tg_q8.cuh"

namespace tg {

constexpr int RT_TC = 8;      // token rows per shared-memory chunk
constexpr int RT_THREADS = 256;

__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}

__global__ void __launch_bounds__(RT_THREADS) layer_route_kernel(RouteArgs a) {
  extern __shared__ __align__(16) float sm[];
  __shared__ float red[RT_THREADS / 32][RT_TC];
  __shared__ float rr_s[RT_TC];
  __shared__ int last_flag;
  __shared__ uint64_t bar;
  const int T = a.T, D = a.D, E = a.E, t = threadIdx.x, lane = t & 31, w = t >> 5;
  const int nw = RT_THREADS / 32;
  const int gbpr = (D + QK - 1) / QK;
  const int e = blockIdx.x;                 // this CTA's expert
  float* xs = sm;                           // [RT_TC][D]
  float* wrow = sm + RT_TC * D;             // [D] this expert's router row
  // Router weights do not depend on the preceding kernel: start the copy of
  // this expert's row before waiting for it.
  const float* wsrc = a.router_w + (size_t)e * D;
  const bool bulk = ((uintptr_t)wsrc & 15) == 0 && (D * 4) % 16 == 0;
  if (t == 0 && bulk) {
    mbar_init(&bar, 1);
    fence_mbar_init();
    mbar_arrive_expect_tx(&bar, (uint32_t)D * 4);
    bulk_g2s(wrow, wsrc, (uint32_t)D * 4, &bar);
  }
  pdl_wait();
  pdl_trigger();
  const float* wr = bulk ? wrow : wsrc;
  bool have_w = !bulk;
  for (int t0 = 0; t0 < T; t0 += RT_TC) {
    const int nt = min(RT_TC, T - t0);
    if ((D & 3) == 0) {
      // float4 loads, all issued before any use
      const float4* xi = reinterpret_cast<const float4*>(a.x_in + (size_t)t0 * D);
      const float4* ai = a.add_in ? reinterpret_cast<const float4*>(a.add_in + (size_t)t0 * D) : nullptr;
      float4* xo = a.x_out && e == 0 ? reinterpret_cast<float4*>(a.x_out + (size_t)t0 * D) : nullptr;
      for (int i = t; i < nt * D / 4; i += RT_THREADS) {
        float4 v = xi[i];
        if (ai) {
          const float4 d = ai[i];
          v = make_float4(fadd(v.x, d.x), fadd(v.y, d.y), fadd(v.z, d.z), fadd(v.w, d.w));
        }
        reinterpret_cast<float4*>(xs)[i] = v;
        if (xo) xo[i] = v;
      }
    } else {
      for (int i = t; i < nt * D; i += RT_THREADS) {
        const size_t gi = (size_t)t0 * D + i;
        float v = a.x_in[gi];
        if (a.add_in) v = fadd(v, a.add_in[gi]);
        xs[i] = v;
        if (e == 0 && a.x_out) a.x_out[gi] = v;
      }
    }
    __syncthreads();
    if (a.normalize) {
      float ss[RT_TC];
#pragma unroll
      for (int tt = 0; tt < RT_TC; tt++) ss[tt] = 0.f;
#pragma unroll
      for (int tt = 0; tt < RT_TC; tt++)
        if (tt < nt)
          for (int i = t; i < D; i += RT_THREADS) ss[tt] = __fmaf_rn(xs[tt * D + i], xs[tt * D + i], ss[tt]);
#pragma unroll
      for (int tt = 0; tt < RT_TC; tt++)
        if (tt < nt) {
          const float v = warp_sum(ss[tt]);
          if (lane == 0) red[w][tt] = v;
        }
      __syncthreads();
      if (t < nt) {
        float tot = 0.f;
        for (int j = 0; j < nw; j++) tot = fadd(tot, red[j][t]);
        rr_s[t] = __fsqrt_rn(fadd(__fdiv_rn(tot, (float)D), a.eps));
      }
      __syncthreads();
      for (int i = t; i < nt * D; i += RT_THREADS) {
        const int tt = i / D;
        float v = __fdiv_rn(xs[i], rr_s[tt]);
        if (a.norm_w) v = fmul(v, a.norm_w[i - tt * D]);
        xs[i] = v;
      }
      __syncthreads();
    }
    // Q8 blocks of the (normalized) rows: CTA 0, one warp per block.
    if (e == 0)
      for (int q = w; q < nt * gbpr; q += nw) {
        const int tt = q / gbpr, b = q - tt * gbpr;
        quantize_block_warp(xs + tt * D + b * QK, min(QK, D - b * QK), a.xq8 + (size_t)(t0 + tt) * gbpr + b);
      }
    // This expert's logits for the chunk.
    if (!have_w) {
      if (!mbar_wait(&bar, 0)) {
        if (t == 0) set_error(a.st, ERR_WAIT_TIMEOUT, 20, e, 0);
        return;
      }
      have_w = true;
    }
    float part[RT_TC];
#pragma unroll
    for (int tt = 0; tt < RT_TC; tt++) part[tt] = 0.f;
    for (int i = t; i < D; i += RT_THREADS) {
      const float wv = wr[i];
#pragma unroll
      for (int tt = 0; tt < RT_TC; tt++)
        if (tt < nt) part[tt] = __fmaf_rn(wv, xs[tt * D + i], part[tt]);
    }
#pragma unroll
    for (int tt = 0; tt < RT_TC; tt++)
      if (tt < nt) {
        const float v = warp_sum(part[tt]);
        if (lane == 0) red[w][tt] = v;
      }
    __syncthreads();
    if (t < nt) {
      float acc = 0.f;
      for (int j = 0; j < nw; j++) acc = fadd(acc, red[j][t]);
      a.logits[(size_t)(t0 + t) * E + e] = a.router_b ? fadd(acc, a.router_b[e]) : acc;
    }
    __syncthreads();
  }
  if (e == 0 && a.zero_out)
    for (size_t i = t; i < (size_t)T * D; i += RT_THREADS) a.zero_out[i] = 0.f;

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
  int* off = cnt + E;                      // [E] row offset of each expert
  int* slot_of = off + E;                  // [E]
  int* wsum = slot_of + E;                 // [2][nw] scan scratch
  int* sidx = wsum + 2 * nw;               // [T][K] selected experts
  float* sw = reinterpret_cast<float*>(sidx + T * K);   // [T][K] their weights
  for (int i = t; i < E; i += RT_THREADS) cnt[i] = 0;
  __syncthreads();
  // Selection: one warp per token; lane l holds logits l, l+32, ... (E <= 256).
  for (int tok = w; tok < T; tok += nw) {
    const float* lg = a.logits + (size_t)tok * E;
    float v[8];
#pragma unroll
    for (int q = 0; q < 8; q++) v[q] = lane + 32 * q < E ? __ldcg(lg + lane + 32 * q) : -INFINITY;
    unsigned taken = 0;
    float bvs[8], ex[8];
    int bis[8];
#pragma unroll
    for (int j = 0; j < 8; j++) {
      if (j >= K) break;
      float bv = -INFINITY;
      int bi = 0x7fffffff;
#pragma unroll
      for (int q = 0; q < 8; q++) {
        const int i = lane + 32 * q;
        if (i < E && !(taken >> q & 1u) && (v[q] > bv || (v[q] == bv && i < bi))) {
          bv = v[q];
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
        // nothing compared greater (NaN logits): the lowest untaken index, weight 0
        bi = E;
        for (int q = 0; q < 8; q++) {
          const int i = lane + 32 * q;
          if (i < E && !(taken >> q & 1u) && i < bi) bi = i;
        }
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) bi = min(bi, __shfl_xor_sync(0xffffffffu, bi, o));
        bv = -INFINITY;
      }
      if ((bi & 31) == lane) taken |= 1u << (bi >> 5);
      bvs[j] = bv;
      bis[j] = bi;
    }
    float sum = 0.f;
#pragma unroll
    for (int j = 0; j < 8; j++)
      if (j < K) {
        ex[j] = expf(fsub(bvs[j], bvs[0]));
        sum = fadd(sum, ex[j]);
      }
    if (lane < K) {
      // lane j publishes selection j
      float wt = 0.f;
      int bi = 0;
#pragma unroll
      for (int j = 0; j < 8; j++)
        if (j == lane) {
          wt = __fdiv_rn(ex[j], sum);
          bi = bis[j];
        }
      sidx[tok * K + lane] = bi;
      sw[tok * K + lane] = wt;
      a.sel_idx[(size_t)tok * K + lane] = bi;
      a.sel_w[(size_t)tok * K + lane] = wt;
      // experts held by another GPU (no local weights) are skipped; their
      // contribution arrives through the cross-GPU sum
      if (wt != 0.f && a.experts[bi].gate.main) atomicAdd(&cnt[bi], 1);
    }
  }
  __syncthreads();
  // Exclusive scans of row counts and of non-empty experts (E <= 256).
  {
    const int c = t < E ? cnt[t] : 0, nz = c > 0;
    int sc = c, sz = nz;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      const int a1 = __shfl_up_sync(0xffffffffu, sc, o), a2 = __shfl_up_sync(0xffffffffu, sz, o);
      if (lane >= o) {
        sc += a1;
        sz += a2;
      }
    }
    if (lane == 31) {
      wsum[w] = sc;
      wsum[nw + w] = sz;
    }
    __syncthreads();
    int bc = 0, bz = 0;
    for (int j = 0; j < w; j++) {
      bc += wsum[j];
      bz += wsum[nw + j];
    }
    if (t < E) {
      off[t] = bc + sc - c;
      slot_of[t] = nz ? bz + sz - 1 : -1;
    }
    if (t == RT_THREADS - 1) {
      PlanHdr* h = a.plan;
      h->n_slots = bz + sz;
      h->total_rows = bc + sc;
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
  }
  __syncthreads();
  for (int ex_i = t; ex_i < E; ex_i += RT_THREADS) {
    const int c = cnt[ex_i];
    if (!c) continue;
    int o = off[ex_i];
    const int sl = slot_of[ex_i];
    const ExpertDesc& X = a.experts[ex_i];
    SlotDesc d;
    d.gate = X.gate;
    d.up = X.up;
    d.down = X.down;
    d.gb = X.gb;
    d.ub = X.ub;
    d.db = X.db;
    d.n_rows = c;
    d.row_off = o;
    d.pad[0] = ex_i;
    d.pad[1] = 0;
    for (int q = 0; q < T * K; q++)
      if (sidx[q] == ex_i && sw[q] != 0.f) {
        a.rows[o] = q / K;
        a.wts[o] = sw[q];
        a.row_slot[o] = sl;
        o++;
      }
    a.slots[sl] = d;
  }
}

size_t route_smem_bytes(int D, int E, int T, int K) {
  const size_t xs = sizeof(float) * (size_t)(RT_TC + 1) * D;
  const size_t sel = sizeof(int) * (3 * (size_t)E + 2 * (RT_THREADS / 32) + 2 * (size_t)T * K);
  return xs > sel ? xs : sel;
}

cudaError_t launch_layer_route(const RouteArgs& a, cudaStream_t s) {
  if (a.top_k < 1 || a.top_k > 8 || a.top_k > a.E || a.E > RT_THREADS) return cudaErrorInvalidValue;
  const size_t smem = route_smem_bytes(a.D, a.E, a.T, a.top_k);
  if (smem > 227 * 1024) return cudaErrorInvalidValue;
  cudaError_t e = ensure_smem(reinterpret_cast<const void*>(layer_route_kernel), smem);
  if (e != cudaSuccess) return e;
  cudaLaunchConfig_t cfg{};
  cfg.gridDim = dim3(a.E);
  cfg.blockDim = dim3(RT_THREADS);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = s;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  RouteArgs args = a;
  void* kargs[] = {(void*)&args};
  return cudaLaunchKernelExC(&cfg, reinterpret_cast<const void*>(layer_route_kernel), kargs);
}

}  // namespace tg
