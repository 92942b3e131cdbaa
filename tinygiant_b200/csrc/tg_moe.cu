// tg_moe.cu — the two expert phases of one MoE call (sm_100a).
//
//   moe_gateup_kernel : gate.x, up.x (+ biases), activation -> hidden
//                                        (moe_phase_a, csrc/libtinygiant.c:1279-1327)
//   moe_down_kernel   : Q8 of hidden, down.hidden, part = w * (v + bias),
//                       ordered combine  (moe_phase_b 1329-1384, combine 1428-1434)
//
// Both kernels are warp-autonomous: a warp owns a stream of work items (one
// (expert, row) of gate and up; one output row across the experts for down)
// and stages each item's weight rows into its own ring of shared-memory
// stages with bulk asynchronous copies (cp.async.bulk, mbarrier completion,
// no multicast), several items ahead of the one it computes.  No CTA-wide
// barrier sits on the streaming path.
//
// A row dot is spread over the lanes (Q4_K: 4 lanes per 256-block, one per
// 64-value group; Q6_K: 8 lanes per block; MXFP4 / Q8_0: one lane per
// 32-value block).  Integer sums are exact (dp4a); the float terms are formed
// and folded in the reference's association and order (tg_dots.cuh), so each
// fp32 row result equals the reference's bit for bit.  The combine adds each
// expert's part into an output element in the call's expert order.
//
// The gate/up kernel also starts L2 prefetches of the selected experts' down
// matrices, so they stream from HBM while phase A runs; the down kernel
// stages its first rows before waiting for phase A (programmatic dependent
// launch).
#include <algorithm>

#include "tg_kernels.h"
#include "tg_moe.h"
#include "tg_q8.cuh"
#include "tg_warpdot.cuh"

namespace tg {

constexpr int NWARP = 8;      // warps per CTA
constexpr int MAX_NST = 8;    // ring stages per warp

// ---------------------------------------------------------------------
// L2 prefetch of the plan's down matrices, spread over every lane of the
// grid: lane gl takes piece gl / n of slot gl % n's matrix.

__device__ __forceinline__ void prefetch_down_l2(const PlanHdr* ph, int n_slots, long gl, long GL) {
  if (n_slots == 0) return;
  const long maxp = GL / n_slots;
  const long sl = gl % n_slots, piece = gl / n_slots;
  if (piece >= maxp) return;
  const WDesc W = ph->slots[sl].down;
  const uint8_t* ptr = W.main;
  const size_t len = (size_t)W.rows * W.rs;
  if (!ptr || len < 16 || ((uintptr_t)ptr & 15)) return;
  const long np = min(maxp, (long)((len + 8191) / 8192));
  if (piece >= np) return;
  const size_t lo = (len * piece / np) & ~(size_t)15;
  const size_t hi = piece + 1 == np ? (len & ~(size_t)15) : ((len * (piece + 1) / np) & ~(size_t)15);
  if (hi > lo) prefetch_l2(ptr + lo, (uint32_t)(hi - lo));
}

// ---------------------------------------------------------------------
// Phase A.  Items are (slot s, row r of I), warp gw takes gw, gw + NW, ...
// A stage holds gate row r then up row r (stage_bytes = 2 * row stage);
// stage_bytes == 0 reads the rows from global memory.

template <int FMT>
__global__ void __launch_bounds__(NWARP * 32, 2)
    moe_gateup_kernel(const PlanHdr* __restrict__ ph, const Q8Dev* __restrict__ xq8, int gbpr,
                      float* __restrict__ hidden, uint32_t stage_bytes, int nst, DevStatus* st) {
  extern __shared__ __align__(128) uint8_t sm[];
  __shared__ uint64_t bars[NWARP][MAX_NST];
  const int lane = threadIdx.x & 31, wid = threadIdx.x >> 5;
  uint64_t* bar = bars[wid];
  uint8_t* ring = sm + (size_t)wid * nst * stage_bytes;
  const bool staged = stage_bytes != 0;
  if (staged && lane == 0) {
    for (int i = 0; i < nst; i++) mbar_init(&bar[i], 1);
    fence_mbar_init();
  }
  __syncwarp();
  pdl_wait();   // the plan and the inputs' Q8 blocks are written by the preceding kernel
  pdl_trigger();
  const int n_slots = ph->n_slots, I = ph->inter_dim, D = ph->embed_dim, k = ph->k;
  const int rule = ph->assoc_rule, act = ph->act;
  const SlotDesc* slots = ph->slots;
  const int* prow = ph->rows;
  const uint32_t half = stage_bytes / 2;
  const long n_items = (long)n_slots * I;
  const long gw = (long)blockIdx.x * NWARP + wid, NW = (long)gridDim.x * NWARP;

  auto issue = [&](long item, int stg) {   // lane 0
    const int s = (int)(item / I), r = (int)(item - (long)s * I);
    const WDesc G = slots[s].gate, U = slots[s].up;
    uint8_t* dst = ring + (size_t)stg * stage_bytes;
    mbar_arrive_expect_tx(&bar[stg], row_tx(G, r) + row_tx(U, r));
    stage_row(G, r, dst, &bar[stg]);
    stage_row(U, r, dst + half, &bar[stg]);
  };
  if (staged && lane == 0)
    for (int i = 0; i < nst; i++) {
      const long it = gw + i * NW;
      if (it < n_items) issue(it, i);
    }
  prefetch_down_l2(ph, n_slots, gw * 32 + lane, NW * 32);

  int j = 0;
  for (long item = gw; item < n_items; item += NW, j++) {
    const int stg = j % nst;
    const int s = (int)(item / I), r = (int)(item - (long)s * I);
    const SlotDesc& S = slots[s];
    const WDesc G = S.gate, U = S.up;
    const uint8_t* dst = staged ? ring + (size_t)stg * stage_bytes : nullptr;
    if (staged && !mbar_wait(&bar[stg], (uint32_t)(j / nst) & 1u)) {
      if (lane == 0) set_error(st, ERR_WAIT_TIMEOUT, 10, s, r);
      for (int i = 1; i < nst; i++)   // bounded waits for the other stages' copies in flight
        if (item + i * NW < n_items) mbar_wait(&bar[(j + i) % nst], (uint32_t)((j + i) / nst) & 1u);
      return;
    }
    const RowPtrs pg = row_ptrs(G, r, dst), pu = row_ptrs(U, r, dst ? dst + half : nullptr);
    const int n = S.n_rows, off = S.row_off;
    for (int g0 = 0; g0 < n; g0 += 4) {
      const int ng = min(4, n - g0);
      const bool x4 = use_x4(rule, g0, n, k);
      const Q8Dev* xp[4];
#pragma unroll
      for (int t = 0; t < 4; t++) xp[t] = xq8 + (size_t)prow[off + g0 + min(t, ng - 1)] * gbpr;
      float gv[4], uv[4];
      warp_dot<FMT>(pg, D, xp, ng, x4, gv);
      warp_dot<FMT>(pu, D, xp, ng, x4, uv);
      float gt = 0.f, ut = 0.f;
#pragma unroll
      for (int t = 0; t < 4; t++) {
        const float a = shfl(gv[t], 0), b = shfl(uv[t], 0);
        if (lane == t) {
          gt = a;
          ut = b;
        }
      }
      if (lane < ng) {
        if (S.gb) {
          gt = fadd(gt, S.gb[r]);
          ut = fadd(ut, S.ub[r]);
        }
        hidden[(size_t)(off + g0 + lane) * I + r] = act_fn(act, gt, ut);
      }
    }
    __syncwarp();
    if (staged && lane == 0 && item + nst * NW < n_items) issue(item + nst * NW, stg);
  }
}

// ---------------------------------------------------------------------
// Phase B.  Warp gw owns output rows gw, gw + NW, ... of D; for each it takes
// the slots in the call's order (with parts_out: only slots of format FMT),
// one ring stage per (row, slot).  Hidden rows are quantized into shared
// memory by each CTA (xcap > 0) or read from hq8 (quantized beforehand).

// The warp's position in its (row, slot) sequence.
struct DnCursor {
  long r;
  int s;
};

template <int FMT>
__device__ __forceinline__ bool dn_next(DnCursor& c, const SlotDesc* slots, int n_slots, int D, long NW,
                                        bool all) {
  for (;;) {
    if (++c.s >= n_slots) {
      c.s = 0;
      c.r += NW;
    }
    if (c.r >= D) return false;
    if (n_slots == 0) continue;
    if (all || slots[c.s].down.fmt == FMT) return true;
  }
}

template <int FMT>
__global__ void __launch_bounds__(NWARP * 32, 2)
    moe_down_kernel(const PlanHdr* __restrict__ ph, const Q8Dev* __restrict__ hq8, int dbpr,
                    const float* __restrict__ hidden, float* __restrict__ out, float* __restrict__ parts_out,
                    uint32_t stage_bytes, int nst, int xcap, int T, DevStatus* st) {
  extern __shared__ __align__(128) uint8_t sm[];
  __shared__ uint64_t bars[NWARP][MAX_NST];
  const int lane = threadIdx.x & 31, wid = threadIdx.x >> 5;
  uint64_t* bar = bars[wid];
  const bool staged = stage_bytes != 0;
  uint8_t* ring = sm + (size_t)wid * nst * stage_bytes;
  float* accw = reinterpret_cast<float*>(sm + (size_t)NWARP * nst * stage_bytes) + (size_t)wid * T;
  Q8Dev* xs = reinterpret_cast<Q8Dev*>(sm + (size_t)NWARP * nst * stage_bytes + round16((size_t)NWARP * T * 4));
  if (staged && lane == 0) {
    for (int i = 0; i < nst; i++) mbar_init(&bar[i], 1);
    fence_mbar_init();
  }
  __syncwarp();
  // The plan was written before the preceding kernel passed its own wait, so
  // it is readable here; hidden is not (pdl_wait below).
  const int D = ph->embed_dim, I = ph->inter_dim, n_slots = ph->n_slots, k = ph->k, rule = ph->assoc_rule;
  const int bias_term = ph->bias_term, total = ph->total_rows;
  const SlotDesc* slots = ph->slots;
  const int* rows = ph->rows;
  const float* wts = ph->wts;
  const long gw = (long)blockIdx.x * NWARP + wid, NW = (long)gridDim.x * NWARP;
  const bool all = parts_out == nullptr;

  DnCursor ic{gw, -1};   // issue cursor (all lanes keep it)
  int issued = 0;
  auto issue_next = [&](int stg) {
    if (!dn_next<FMT>(ic, slots, n_slots, D, NW, all)) return false;
    if (lane == 0) {
      const WDesc W = slots[ic.s].down;
      uint8_t* dst = ring + (size_t)stg * stage_bytes;
      mbar_arrive_expect_tx(&bar[stg], row_tx(W, (int)ic.r));
      stage_row(W, (int)ic.r, dst, &bar[stg]);
    }
    issued++;
    return true;
  };
  if (staged)
    for (int i = 0; i < nst; i++)
      if (!issue_next(i)) break;

  pdl_wait();   // hidden is complete
  pdl_trigger();
  bool bad = false;
  if (xcap > 0) {
    if (total > xcap) {
      bad = true;
    } else {
      for (int b = wid; b < total * dbpr; b += NWARP) {
        const int row = b / dbpr, blk = b - row * dbpr;
        quantize_block_warp(hidden + (size_t)row * I + (size_t)blk * QK, min(QK, I - blk * QK), xs + b);
      }
    }
    __syncthreads();
  }
  const Q8Dev* xq = xcap > 0 ? xs : hq8;
  int j = 0;
  auto drain = [&]() {   // bounded waits for this warp's copies in flight
    for (int i = j; i < issued; i++) mbar_wait(&bar[i % nst], (uint32_t)(i / nst) & 1u);
  };
  if (bad) {
    if (threadIdx.x == 0) set_error(st, ERR_BAD_PLAN, 13, total, xcap);
    if (staged) drain();
    return;
  }
  // Rows of this warp, slots in the same order as issued.
  for (long r = gw; r < D; r += NW) {
    if (all)
      for (int t = lane; t < T; t += 32) accw[t] = out[(size_t)t * D + r];
    __syncwarp();
    for (int s = 0; s < n_slots; s++) {
      const SlotDesc& S = slots[s];
      if (!all && S.down.fmt != FMT) continue;
      const int stg = j % nst;
      const uint8_t* dst = staged ? ring + (size_t)stg * stage_bytes : nullptr;
      if (staged && !mbar_wait(&bar[stg], (uint32_t)(j / nst) & 1u)) {
        if (lane == 0) set_error(st, ERR_WAIT_TIMEOUT, 11, (int)r, s);
        j++;
        drain();
        return;
      }
      const RowPtrs rp = row_ptrs(S.down, (int)r, dst);
      const int n = S.n_rows, off = S.row_off;
      const float* db = S.db;
      for (int g0 = 0; g0 < n; g0 += 4) {
        const int ng = min(4, n - g0);
        float v[4];
        if constexpr (FMT == FMT_F16) {
          if (lane == 0)
            for (int t = 0; t < ng; t++)
              v[t] = dot_f16_lane(reinterpret_cast<const uint16_t*>(rp.m), hidden + (size_t)(off + g0 + t) * I, I);
        } else {
          const bool x4 = use_x4(rule, g0, n, k);
          const Q8Dev* xp[4];
#pragma unroll
          for (int t = 0; t < 4; t++) xp[t] = xq + (size_t)(off + g0 + min(t, ng - 1)) * dbpr;
          warp_dot<FMT>(rp, I, xp, ng, x4, v);
        }
        if (lane == 0)
          for (int t = 0; t < ng; t++) {
            const int sr = off + g0 + t;
            const float w = wts[sr];
            const float part = bias_term ? fmul(w, fadd(v[t], db ? db[r] : 0.f)) : fmul(w, v[t]);
            if (all) accw[rows[sr]] = fadd(accw[rows[sr]], part);
            else parts_out[(size_t)sr * D + r] = part;
          }
      }
      __syncwarp();
      j++;
      if (staged) issue_next(stg);
    }
    __syncwarp();
    if (all)
      for (int t = lane; t < T; t += 32) out[(size_t)t * D + r] = accw[t];
    __syncwarp();
  }
}

// Calls whose experts mix down formats: out[t][r] += each stored part in
// the call's order (one thread per output element).
__global__ void combine_parts_kernel(const PlanHdr* __restrict__ ph, const float* __restrict__ parts,
                                     float* __restrict__ out) {
  const int D = ph->embed_dim, k = ph->k, total = ph->total_rows;
  const size_t i = (size_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= (size_t)k * D) return;
  const int t = (int)(i / D), r = (int)(i - (size_t)t * D);
  float v = out[i];
  for (int sr = 0; sr < total; sr++)
    if (ph->rows[sr] == t) v = fadd(v, parts[(size_t)sr * D + r]);
  out[i] = v;
}

// ---------------------------------------------------------------------
// Launchers.

static cudaError_t launch_pdl(const void* fn, dim3 grid, size_t smem, cudaStream_t s, void** args) {
  cudaLaunchConfig_t cfg{};
  cfg.gridDim = grid;
  cfg.blockDim = dim3(NWARP * 32);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = s;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  return cudaLaunchKernelExC(&cfg, fn, args);
}

static int sm_count() {
  static int sms = 0;
  if (!sms) {
    int dev = 0;
    cudaGetDevice(&dev);
    cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
    if (sms < 1) sms = 1;
  }
  return sms;
}

// CTAs of `fn` resident at once with `smem` bytes (all SMs).
static int resident_ctas(const void* fn, size_t smem) {
  int per = 0;
  if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per, fn, NWARP * 32, smem) != cudaSuccess || per < 1) per = 1;
  return per * sm_count();
}

// Ring depth for a per-CTA budget, or 0 stages (global reads) when even two
// stages per warp do not fit.
static void ring_shape(uint32_t stage, uint32_t budget, uint32_t fixed, uint32_t& stage_bytes, int& nst) {
  nst = (int)std::min<uint32_t>(MAX_NST, budget / std::max<uint32_t>(1, NWARP * stage));
  nst = std::max(nst, 2);
  stage_bytes = stage;
  if ((size_t)NWARP * nst * stage + fixed > 200 * 1024) {
    stage_bytes = 0;
    nst = 1;
  }
}

template <int FMT>
static cudaError_t gateup_fmt(const PlanHdr* ph, int max_slots, int D, int I, const Q8Dev* xq8, float* hidden,
                              DevStatus* st, cudaStream_t s) {
  uint32_t stage;
  int nst;
  ring_shape(2 * rows_stage_bytes(row_layout(FMT, D).rs, 1), 48 * 1024, 0, stage, nst);
  const size_t smem = (size_t)NWARP * nst * stage;
  const void* fn = reinterpret_cast<const void*>(moe_gateup_kernel<FMT>);
  cudaError_t e = ensure_smem(fn, smem);
  if (e != cudaSuccess) return e;
  static int cap[5] = {0, 0, 0, 0, 0};
  static size_t cap_smem[5] = {0, 0, 0, 0, 0};
  if (!cap[FMT] || cap_smem[FMT] != smem) {
    cap[FMT] = resident_ctas(fn, smem);
    cap_smem[FMT] = smem;
  }
  const long max_items = (long)max_slots * I;
  const int grid = (int)std::max<long>(1, std::min<long>((max_items + NWARP - 1) / NWARP, cap[FMT]));
  int gbpr = (D + QK - 1) / QK;
  void* args[] = {(void*)&ph, (void*)&xq8, (void*)&gbpr, (void*)&hidden, (void*)&stage, (void*)&nst, (void*)&st};
  return launch_pdl(fn, dim3(grid), smem, s, args);
}

cudaError_t launch_moe_gateup(const PlanHdr* ph, int max_slots, int gate_fmt, int D, int I, const Q8Dev* xq8,
                              float* hidden, Q8Dev* /*hq8*/, int* /*counters*/, DevStatus* st, cudaStream_t s) {
  if (max_slots <= 0) return cudaSuccess;
  switch (gate_fmt) {
    case FMT_Q4K: return gateup_fmt<FMT_Q4K>(ph, max_slots, D, I, xq8, hidden, st, s);
    case FMT_Q6K: return gateup_fmt<FMT_Q6K>(ph, max_slots, D, I, xq8, hidden, st, s);
    case FMT_MXFP4: return gateup_fmt<FMT_MXFP4>(ph, max_slots, D, I, xq8, hidden, st, s);
    case FMT_Q80: return gateup_fmt<FMT_Q80>(ph, max_slots, D, I, xq8, hidden, st, s);
    default: return cudaErrorInvalidValue;
  }
}

// Staged Q8 rows of hidden per down CTA are capped at this many bytes; larger
// plans quantize hidden once into hq8 first.
constexpr uint32_t DN_XS_MAX = 64 * 1024;

template <int FMT>
static cudaError_t down_fmt(const PlanHdr* ph, int max_slots, int max_rows, int D, int I, int T, Q8Dev* hq8,
                            const float* hidden, float* out, float* parts_out, DevStatus* st, cudaStream_t s) {
  const int dbpr = (I + QK - 1) / QK;
  int xcap = 0;
  if (FMT != FMT_F16 && (size_t)max_rows * dbpr * sizeof(Q8Dev) <= DN_XS_MAX) xcap = std::max(max_rows, 1);
  const uint32_t fixed = round16((size_t)NWARP * T * 4) + (uint32_t)((size_t)xcap * dbpr * sizeof(Q8Dev));
  uint32_t stage;
  int nst;
  ring_shape(rows_stage_bytes(row_layout(FMT, I).rs, 1), 40 * 1024, fixed, stage, nst);
  const size_t smem = (size_t)NWARP * nst * stage + fixed;
  if (smem > 227 * 1024) return cudaErrorInvalidValue;
  if (FMT != FMT_F16 && xcap == 0) {
    launch_quantize_rows(hidden, max_rows, I, I, hq8, s);
    cudaError_t e = cudaGetLastError();
    if (e != cudaSuccess) return e;
  }
  const void* fn = reinterpret_cast<const void*>(moe_down_kernel<FMT>);
  cudaError_t e = ensure_smem(fn, smem);
  if (e != cudaSuccess) return e;
  const int grid = std::max(1, std::min((D + NWARP - 1) / NWARP, resident_ctas(fn, smem)));
  const Q8Dev* hq = hq8;
  void* args[] = {(void*)&ph,     (void*)&hq,    (void*)&dbpr, (void*)&hidden, (void*)&out, (void*)&parts_out,
                  (void*)&stage, (void*)&nst, (void*)&xcap, (void*)&T,      (void*)&st};
  return launch_pdl(fn, dim3(grid), smem, s, args);
}

cudaError_t launch_moe_down(const PlanHdr* ph, int max_slots, int max_rows, int down_fmt_all, int D, int I, int T,
                            Q8Dev* hq8, const float* hidden, float* out, float* parts_out, DevStatus* st,
                            cudaStream_t s) {
  switch (down_fmt_all) {
    case FMT_Q4K: return down_fmt<FMT_Q4K>(ph, max_slots, max_rows, D, I, T, hq8, hidden, out, parts_out, st, s);
    case FMT_Q6K: return down_fmt<FMT_Q6K>(ph, max_slots, max_rows, D, I, T, hq8, hidden, out, parts_out, st, s);
    case FMT_MXFP4: return down_fmt<FMT_MXFP4>(ph, max_slots, max_rows, D, I, T, hq8, hidden, out, parts_out, st, s);
    case FMT_Q80: return down_fmt<FMT_Q80>(ph, max_slots, max_rows, D, I, T, hq8, hidden, out, parts_out, st, s);
    case FMT_F16: return down_fmt<FMT_F16>(ph, max_slots, max_rows, D, I, T, hq8, hidden, out, parts_out, st, s);
    default: return cudaErrorInvalidValue;
  }
}

cudaError_t launch_combine_parts(const PlanHdr* ph, int D, int T, const float* parts, float* out, cudaStream_t s) {
  const size_t n = (size_t)T * D;
  combine_parts_kernel<<<(unsigned)((n + 255) / 256), 256, 0, s>>>(ph, parts, out);
  return cudaGetLastError();
}

size_t moe_counter_ints(int /*max_slots*/, int /*I*/) { return 1; }

}  // namespace tg
