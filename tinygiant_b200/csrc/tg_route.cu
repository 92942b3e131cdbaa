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
#include "tg_warpdot.cuh"

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
    d.expert = ex_i;
    d.pad = 0;
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

// ---------------------------------------------------------------------
// Routing for batched steps (many rows): the same results as
// layer_route_kernel's, in four kernels that each use the whole GPU.
//   norm_q8_kernel   one CTA per row: x' = x + add (x_out), N = x' / rr * w,
//                    N's Q8 blocks; the row's MoE output zeroed
//   logits_kernel    W_r N for tiles of 16 rows x 32 experts, a fixed order over D
//   select_kernel    one warp per row: top-k (larger logit first, NaN last, ties
//                    to the lower id), softmax over the selected, membership
//                    (stored expert-major, so each expert's rows are contiguous)
//   plan_kernel      one CTA per expert: its active rows in row order, slots in
//                    expert order, the plan header (engine.py:297-318)

__global__ void __launch_bounds__(256) norm_q8_kernel(BatchRouteArgs a) {
  __shared__ float red[8];
  __shared__ float rr_s;
  pdl_wait();
  pdl_trigger();
  const int t = blockIdx.x, tid = threadIdx.x, lane = tid & 31, w = tid >> 5;
  const int D = a.D, gbpr = (D + QK - 1) / QK;
  if (t == 0)
    for (int e = tid; e < a.E; e += 256) a.ecnt[e] = 0;   // select_kernel counts each expert's rows
  const float* x = a.x_in + (size_t)t * D;
  const float* ad = a.add_in ? a.add_in + (size_t)t * D : nullptr;
  float* n = a.nbuf + (size_t)t * D;
  float ss = 0.f;
  for (int i = tid; i < D; i += 256) {
    float v = x[i];
    if (ad) v = fadd(v, ad[i]);
    if (a.x_out) a.x_out[(size_t)t * D + i] = v;
    if (a.zero_out) a.zero_out[(size_t)t * D + i] = 0.f;
    n[i] = v;
    ss = __fmaf_rn(v, v, ss);
  }
  if (a.normalize) {
    ss = warp_sum(ss);
    if (lane == 0) red[w] = ss;
    __syncthreads();
    if (tid == 0) {
      float tot = 0.f;
      for (int j = 0; j < 8; j++) tot = fadd(tot, red[j]);
      rr_s = __fsqrt_rn(fadd(__fdiv_rn(tot, (float)D), a.eps));
    }
    __syncthreads();
    const float rr = rr_s;
    const double yd = 1.0 / (double)rr;
    for (int i = tid; i < D; i += 256) {
      float v = div_rn_d(n[i], rr, yd);
      if (a.norm_w) v = fmul(v, a.norm_w[i]);
      n[i] = v;
    }
  }
  __syncthreads();
  for (int b = w; b < gbpr; b += 8) quantize_block_warp(n + b * QK, min(QK, D - b * QK), a.xq8 + (size_t)t * gbpr + b);
}

// Tile: 16 rows x 32 experts per CTA; lane = expert, warp w = rows 2w and
// 2w + 1.  Per 128-value chunk of D the router rows and the normalized rows
// are staged in shared memory (router rows padded to 132 floats, so a
// quarter warp's 16-byte loads hit distinct banks); each lane keeps its two
// rows' dots in four chains each (value d in chain d % 4) and adds the chains
// in a fixed order per chunk.
constexpr int LG_T = 16, LG_E = 32, LG_D = 128, LG_WP = 132;
__global__ void __launch_bounds__(256) logits_kernel(BatchRouteArgs a) {
  __shared__ __align__(16) float Ws[LG_E][LG_WP];
  __shared__ __align__(16) float Ns[LG_T][LG_D];
  pdl_wait();
  pdl_trigger();
  const int tid = threadIdx.x, lane = tid & 31, w = tid >> 5;
  const int D = a.D, E = a.E, T = a.T;
  const int t0 = blockIdx.x * LG_T, e0 = blockIdx.y * LG_E;
  const int e = e0 + lane, ta = t0 + 2 * w, tb = ta + 1;
  float acc_a = 0.f, acc_b = 0.f;
  // this thread's share of a chunk: router values i = tid + 256 q, row values
  // likewise; the next chunk's are loaded into registers while this one is
  // computed from shared memory
  constexpr int NWQ = LG_E * LG_D / 256, NNQ = LG_T * LG_D / 256;
  float wr[NWQ], nr[NNQ];
  auto fetch = [&](int d0) {
#pragma unroll
    for (int q = 0; q < NWQ; q++) {
      const int i = tid + 256 * q, er = i / LG_D, dc = i % LG_D;
      wr[q] = e0 + er < E && d0 + dc < D ? __ldg(a.router_w + (size_t)(e0 + er) * D + d0 + dc) : 0.f;
    }
#pragma unroll
    for (int q = 0; q < NNQ; q++) {
      const int i = tid + 256 * q, tr = i / LG_D, dc = i % LG_D;
      nr[q] = t0 + tr < T && d0 + dc < D ? __ldcg(a.nbuf + (size_t)(t0 + tr) * D + d0 + dc) : 0.f;
    }
  };
  fetch(0);
  for (int d0 = 0; d0 < D; d0 += LG_D) {
#pragma unroll
    for (int q = 0; q < NWQ; q++) {
      const int i = tid + 256 * q;
      Ws[i / LG_D][i % LG_D] = wr[q];
    }
#pragma unroll
    for (int q = 0; q < NNQ; q++) {
      const int i = tid + 256 * q;
      Ns[i / LG_D][i % LG_D] = nr[q];
    }
    __syncthreads();
    if (d0 + LG_D < D) fetch(d0 + LG_D);
    float ca[4] = {0.f, 0.f, 0.f, 0.f}, cb[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll 8
    for (int dc = 0; dc < LG_D; dc += 4) {
      const float4 wv = *reinterpret_cast<const float4*>(&Ws[lane][dc]);
      const float4 na = *reinterpret_cast<const float4*>(&Ns[2 * w][dc]);
      const float4 nb = *reinterpret_cast<const float4*>(&Ns[2 * w + 1][dc]);
      ca[0] = __fmaf_rn(wv.x, na.x, ca[0]);
      ca[1] = __fmaf_rn(wv.y, na.y, ca[1]);
      ca[2] = __fmaf_rn(wv.z, na.z, ca[2]);
      ca[3] = __fmaf_rn(wv.w, na.w, ca[3]);
      cb[0] = __fmaf_rn(wv.x, nb.x, cb[0]);
      cb[1] = __fmaf_rn(wv.y, nb.y, cb[1]);
      cb[2] = __fmaf_rn(wv.z, nb.z, cb[2]);
      cb[3] = __fmaf_rn(wv.w, nb.w, cb[3]);
    }
    acc_a = fadd(acc_a, fadd(fadd(ca[0], ca[1]), fadd(ca[2], ca[3])));
    acc_b = fadd(acc_b, fadd(fadd(cb[0], cb[1]), fadd(cb[2], cb[3])));
    __syncthreads();
  }
  if (e < E) {
    const float b = a.router_b ? a.router_b[e] : 0.f;
    if (ta < T) a.logits[(size_t)ta * E + e] = a.router_b ? fadd(acc_a, b) : acc_a;
    if (tb < T) a.logits[(size_t)tb * E + e] = a.router_b ? fadd(acc_b, b) : acc_b;
  }
}

__global__ void __launch_bounds__(256) select_kernel(BatchRouteArgs a) {
  pdl_wait();
  pdl_trigger();
  const int lane = threadIdx.x & 31;
  const int t = (int)(((long)blockIdx.x * blockDim.x + threadIdx.x) >> 5);
  const int E = a.E, K = a.top_k;
  if (t >= a.T) return;
  float v[8], bvs[8];
  uint32_t key[8];
  int id[8], bis[8];
#pragma unroll
  for (int i = 0; i < 8; i++) {
    const int e = lane + 32 * i;
    v[i] = e < E ? __ldcg(a.logits + (size_t)t * E + e) : 0.f;
    uint32_t u = __float_as_uint(v[i]);
    if (u == 0x80000000u) u = 0u;
    id[i] = e;
    key[i] = e >= E ? 0u : v[i] != v[i] ? 1u : (u >> 31) ? ~u : (u | 0x80000000u);
    if (e < E) a.member[(size_t)e * a.T + t] = 0;
  }
  // K rounds: the warp's largest key, the lowest id among equal keys
#pragma unroll 1
  for (int j = 0; j < K; j++) {
    uint32_t best = 0u;
    int bi = 0;
    float bv = 0.f;
#pragma unroll
    for (int i = 0; i < 8; i++)
      if (key[i] > best) {
        best = key[i];
        bi = i;
        bv = v[i];
      }
    const uint32_t M = __reduce_max_sync(0xffffffffu, best);
    const uint32_t I = __reduce_min_sync(0xffffffffu, best == M ? (uint32_t)(lane + 32 * bi) : 0xffffffffu);
    float sel_v = 0.f;
    if (I == (uint32_t)(lane + 32 * bi)) {
#pragma unroll
      for (int i = 0; i < 8; i++)
        if (i == bi) key[i] = 0u;
      sel_v = bv != bv ? -INFINITY : bv;
    }
    bvs[j] = __shfl_sync(0xffffffffu, sel_v, (int)(I & 31));
    bis[j] = (int)I;
  }
  float sum = 0.f, ex[8];
#pragma unroll
  for (int j = 0; j < 8; j++)
    if (j < K) {
      ex[j] = expf(fsub(bvs[j], bvs[0]));
      sum = fadd(sum, ex[j]);
    }
  __syncwarp();
  if (lane < K) {
    float wt = 0.f;
    int bi = 0;
#pragma unroll
    for (int j = 0; j < 8; j++)
      if (j == lane) {
        wt = __fdiv_rn(ex[j], sum);
        bi = bis[j];
      }
    a.sel_idx[(size_t)t * K + lane] = bi;
    a.sel_w[(size_t)t * K + lane] = wt;
  }
  // experts held by another GPU (no local weights) are skipped; a valid
  // selection's place among the row's valid selections in expert order is
  // where the plan puts its active row in tok_rows
  int bi = 0;
  float wt = 0.f;
  if (lane < K) {
    bi = a.sel_idx[(size_t)t * K + lane];
    wt = a.sel_w[(size_t)t * K + lane];
  }
  const bool valid = lane < K && wt != 0.f && a.experts[bi].gate.main != nullptr;
  const unsigned vm = __ballot_sync(0xffffffffu, valid);
  int p = 0;
  for (int q = 0; q < K; q++) p += ((vm >> q) & 1u) && __shfl_sync(0xffffffffu, bi, q) < bi;
  if (valid) {
    a.member[(size_t)bi * a.T + t] = (uint8_t)(lane + 1);
    a.tpos[(size_t)t * K + lane] = p;
    atomicAdd(a.ecnt + bi, 1);
  }
  if (lane < K && lane >= __popc(vm)) a.tok_rows[(size_t)t * K + lane] = -1;
}

// One CTA per expert e (blockIdx.x).  Every CTA scans the experts' row
// counts (select_kernel's) into row offsets and slot numbers; CTA e then
// lists its expert's active rows in row order: each warp counts the members
// of its 32-row chunks of the expert's membership column, the chunks' counts
// are scanned, and each member row is written at the expert's offset plus
// the members before it.  CTA 0 writes the plan header.
constexpr int PLAN_THREADS = 512, PLAN_MAX_CHUNKS = 256;   // rows up to 8192
__global__ void __launch_bounds__(PLAN_THREADS) plan_kernel(BatchRouteArgs a) {
  __shared__ int off[256], slot_of[256], chunk[PLAN_MAX_CHUNKS];
  __shared__ int wsum[2][PLAN_THREADS / 32];
  pdl_wait();
  pdl_trigger();
  const int tid = threadIdx.x, lane = tid & 31, w = tid >> 5;
  constexpr int NW = PLAN_THREADS / 32;
  const int E = a.E, T = a.T, K = a.top_k, e = blockIdx.x;
  {   // exclusive scans of the counts and of the non-empty experts (E <= 256 <= threads)
    const int c = tid < E ? __ldcg(a.ecnt + tid) : 0, nz = c > 0;
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
      wsum[0][w] = sc;
      wsum[1][w] = sz;
    }
    __syncthreads();
    int bc = 0, bz = 0;
    for (int j = 0; j < w; j++) {
      bc += wsum[0][j];
      bz += wsum[1][j];
    }
    if (tid < E) {
      off[tid] = bc + sc - c;
      slot_of[tid] = nz ? bz + sz - 1 : -1;
    }
    if (e == 0 && tid == PLAN_THREADS - 1) {
      PlanHdr* h = a.plan;
      h->n_slots = bz + sz;
      h->total_rows = bc + sc;
      h->k = T;
      h->embed_dim = a.D;
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
  }
  const int sl = slot_of[e];
  if (sl < 0) return;   // uniform over the CTA
  const uint8_t* col = a.member + (size_t)e * T;
  const int nch = (T + 31) / 32;
  for (int c = w; c < nch; c += NW) {
    const int t = 32 * c + lane;
    const unsigned bal = __ballot_sync(0xffffffffu, t < T && __ldcg(col + t) != 0);
    if (lane == 0) chunk[c] = __popc(bal);
  }
  __syncthreads();
  if (w == 0) {   // exclusive scan over the chunks
    int run = 0;
    for (int c0 = 0; c0 < nch; c0 += 32) {
      const int c = c0 + lane;
      const int v = c < nch ? chunk[c] : 0;
      int sc = v;
#pragma unroll
      for (int o = 1; o < 32; o <<= 1) {
        const int a1 = __shfl_up_sync(0xffffffffu, sc, o);
        if (lane >= o) sc += a1;
      }
      if (c < nch) chunk[c] = run + sc - v;
      run += __shfl_sync(0xffffffffu, sc, 31);
    }
  }
  __syncthreads();
  for (int c = w; c < nch; c += NW) {
    const int t = 32 * c + lane;
    const int m = t < T ? __ldcg(col + t) : 0;
    const unsigned bal = __ballot_sync(0xffffffffu, m != 0);
    if (m) {
      const int pos = off[e] + chunk[c] + __popc(bal & ((1u << lane) - 1u));
      a.rows[pos] = t;
      a.wts[pos] = a.sel_w[(size_t)t * K + (m - 1)];
      a.row_slot[pos] = sl;
      a.tok_rows[(size_t)t * K + a.tpos[(size_t)t * K + (m - 1)]] = pos;
    }
  }
  if (tid == 0) {
    const ExpertDesc& X = a.experts[e];
    SlotDesc d;
    d.gate = X.gate;
    d.up = X.up;
    d.down = X.down;
    d.gb = X.gb;
    d.ub = X.ub;
    d.db = X.db;
    d.n_rows = __ldcg(a.ecnt + e);
    d.row_off = off[e];
    d.expert = e;
    d.pad = 0;
    a.slots[sl] = d;
  }
}

static cudaError_t launch_cfg(const void* fn, dim3 grid, dim3 block, cudaStream_t s, BatchRouteArgs* a) {
  cudaLaunchConfig_t cfg{};
  cfg.gridDim = grid;
  cfg.blockDim = block;
  cfg.stream = s;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  void* kargs[] = {(void*)a};
  return cudaLaunchKernelExC(&cfg, fn, kargs);
}

cudaError_t launch_batch_route(const BatchRouteArgs& args, cudaStream_t s) {
  if (args.top_k < 1 || args.top_k > 8 || args.top_k > args.E || args.E > 256 || args.T < 1 ||
      args.T > 32 * PLAN_MAX_CHUNKS || !args.ecnt)
    return cudaErrorInvalidValue;
  BatchRouteArgs a = args;
  cudaError_t e = launch_cfg(reinterpret_cast<const void*>(norm_q8_kernel), dim3(a.T), dim3(256), s, &a);
  if (e == cudaSuccess)
    e = launch_cfg(reinterpret_cast<const void*>(logits_kernel), dim3((a.T + LG_T - 1) / LG_T, (a.E + LG_E - 1) / LG_E),
                   dim3(256), s, &a);
  if (e == cudaSuccess)
    e = launch_cfg(reinterpret_cast<const void*>(select_kernel), dim3((a.T * 32 + 255) / 256), dim3(256), s, &a);
  if (e == cudaSuccess) e = launch_cfg(reinterpret_cast<const void*>(plan_kernel), dim3(a.E), dim3(PLAN_THREADS), s, &a);
  return e;
}

}  // namespace tg
