// tg_step.cu — one MoE layer step for decode-sized batches (T <= 8) as a
// single persistent kernel.
//
// The step is the engine's MoE block (tinygiant/engine.py:281-342) followed by
// tg_moe_forward_rows_v2 (csrc/libtinygiant.c:1386-1437):
//   R  x' = x + add; N = x' / sqrt(mean(x'^2) + eps) * w; logits = W_r N (+ b);
//      Q8 blocks of N                                  (router.py:29-33, 169-208)
//   S  top-k by descending logit, softmax over the selected, union of the
//      selected experts ascending by id, active rows in token order
//                                                      (router.py:35-42, engine.py:297-318)
//   A  gate.x, up.x (+ biases), activation -> hidden   (moe_phase_a, 1279-1327)
//   B  Q8 of hidden, down.hidden, part = w * (v + b), combine in expert order
//                                                      (moe_phase_b 1329-1384, 1428-1434)
// One CTA per SM.  R runs one warp per expert (its router row); every CTA
// quantizes N itself and repeats S on its own (both are tiny) instead of
// waiting for one CTA to publish them.  A and B stream their weight rows
// through a per-warp ring of shared-memory stages filled by bulk
// asynchronous copies (cp.async.bulk, no multicast): the ring runs straight
// from a warp's gate/up items into its down items, so the down weights are
// in flight while phase A computes.
//
// There is no grid-wide barrier.  The two values CTAs exchange — router
// logits and hidden activations — are written as 64-bit words holding the
// launch's epoch in the high half and the fp32 value in the low half; one
// aligned 64-bit store is seen whole, so a consumer that reads a word tagged
// with this launch's epoch has its value, and consumers poll the words
// themselves (one L2 round trip per poll, no separate flag).  The epoch is the
// launch count: each CTA adds one to a 64-bit counter as it starts (before
// it lets the next kernel launch), so the G CTAs of launch n read counts
// n*G .. n*G + G - 1.  Words a launch does not rewrite are never read by it.
// Every wait (poll, mbarrier) gives up after about a second and records an
// error instead of hanging; the grid never exceeds the CTAs the GPU holds at
// once, so every producer runs.
#include <algorithm>

#include "tg_moe.h"
#include "tg_q8.cuh"
#include "tg_warpdot.cuh"

namespace tg {

constexpr int SW_MAX = 20;         // warps per CTA: 20 for MXFP4 steps (their phase A decodes on the
                                   // integer pipes and gains from more warps), 16 otherwise
constexpr int ST_MAX_NST = 8;      // ring stages per warp
constexpr int STEP_T_MAX = 8;
constexpr int STEP_K_MAX = 8;
constexpr int STEP_R_MAX = STEP_T_MAX * STEP_K_MAX;   // active rows
constexpr int STEP_E_MAX = 256;
constexpr int STEP_GB_MAX = 16;    // 256-value blocks per token row (D <= 4096)
constexpr int STEP_RW_MAX = 2;     // router rows per CTA
constexpr int STEP_POLLS = 1 << 23;   // polls of another CTA's words before giving up (~1 s with the sleeps)

struct StepShared {
  int sel_e[STEP_T_MAX][STEP_K_MAX];
  float sel_v[STEP_T_MAX][STEP_K_MAX];
  float sel_w[STEP_T_MAX][STEP_K_MAX];
  int cnt[STEP_E_MAX];
  int slot_of[STEP_E_MAX];
  union {
    int off[STEP_E_MAX];     // the plan (T > 1): each expert's first active row
    int slot_a[STEP_R_MAX];  // after it: phase A's slot order, most active rows first
  };
  int wsum[2][SW_MAX];
  int n_slots, total, ok;
  uint32_t epoch;
  int slot_e[STEP_R_MAX], slot_n[STEP_R_MAX], slot_off[STEP_R_MAX];
  int row_t[STEP_R_MAX];   // active row -> token
  int row_s[STEP_R_MAX];   // active row -> slot
  float row_w[STEP_R_MAX];
  float part_ss[STEP_T_MAX][STEP_GB_MAX];
  float part_dot[STEP_RW_MAX][STEP_T_MAX][STEP_GB_MAX];
  float rrt[STEP_T_MAX];
  double yd[STEP_T_MAX];
  uint64_t rbar[SW_MAX];
  uint64_t xbar, ebar;
  unsigned long long tw[SW_MAX][8];
  uint64_t bars[SW_MAX][ST_MAX_NST];
};

// ---------------------------------------------------------------------
// Epoch-tagged words.

__device__ __forceinline__ void st_tagged(unsigned long long* p, uint32_t ep, float v) {
  const unsigned long long w = ((unsigned long long)ep << 32) | __float_as_uint(v);
  asm volatile("st.relaxed.gpu.global.u64 [%0], %1;" ::"l"(p), "l"(w) : "memory");
}
__device__ __forceinline__ unsigned long long ld_tagged(const unsigned long long* p) {
  unsigned long long w;
  asm volatile("ld.relaxed.gpu.global.u64 %0, [%1];" : "=l"(w) : "l"(p) : "memory");
  return w;
}
__device__ __forceinline__ ulonglong2 ld_tagged2(const unsigned long long* p) {
  ulonglong2 w;
  asm volatile("ld.relaxed.gpu.global.v2.u64 {%0, %1}, [%2];" : "=l"(w.x), "=l"(w.y) : "l"(p) : "memory");
  return w;
}
__device__ __forceinline__ bool tag_is(unsigned long long w, uint32_t ep) { return (uint32_t)(w >> 32) == ep; }
// A flag that publishes other data: released by its writer (after the data,
// which the warp's other lanes wrote before a __syncwarp), acquired by its
// readers.  (A full fence instead would also wait, on the lane that issues
// the ring's bulk copies, for those copies.)
__device__ __forceinline__ void st_flag_release(unsigned long long* p, uint32_t ep) {
  const unsigned long long w = (unsigned long long)ep << 32;
  asm volatile("st.release.gpu.global.u64 [%0], %1;" ::"l"(p), "l"(w) : "memory");
}
__device__ __forceinline__ unsigned long long ld_flag_acquire(const unsigned long long* p) {
  unsigned long long w;
  asm volatile("ld.acquire.gpu.global.u64 %0, [%1];" : "=l"(w) : "l"(p) : "memory");
  return w;
}
__device__ __forceinline__ float tag_val(unsigned long long w) { return __uint_as_float((uint32_t)w); }

// System-scope forms, for words another GPU writes over NVLink.
__device__ __forceinline__ void st_tagged_sys(unsigned long long* p, uint32_t ep, float v) {
  const unsigned long long w = ((unsigned long long)ep << 32) | __float_as_uint(v);
  asm volatile("st.relaxed.sys.global.u64 [%0], %1;" ::"l"(p), "l"(w) : "memory");
}
__device__ __forceinline__ unsigned long long ld_tagged_sys(const unsigned long long* p) {
  unsigned long long w;
  asm volatile("ld.relaxed.sys.global.u64 %0, [%1];" : "=l"(w) : "l"(p) : "memory");
  return w;
}

// Word of hidden value r (0 .. I-1) of active row o: each 256-value block is
// stored so that lane l's values 8l .. 8l+7 are four 16-byte pairs at
// 64-word strides (value p = 8l + j at word 64 (j / 2) + 2l + j % 2), which
// makes each of a warp's four pair loads one contiguous 512-byte line set.
__device__ __forceinline__ size_t hid_word(int o, int r, int dbpr) {
  const int b = r >> 8, p = r & 255;
  return ((size_t)o * dbpr + b) * 256 + ((p & 7) >> 1) * 64 + 2 * (p >> 3) + (p & 1);
}

// The expert-parallel combine of output row r (one warp; lane t < T holds
// token t's part): stores the part as a tagged word into slot rank of every
// shard's receive block over NVLink, then polls this shard's block until all
// world parts of row r carry this launch's epoch, and writes their sum in
// shard order (the same on every shard).  Not inlined, so the step's other
// paths keep its registers.  False after the poll limit.
static __device__ __noinline__ bool ep_combine_row(unsigned long long* const* peers, const unsigned long long* recv,
                                                   int rank, int world, int T, int D, int r, float v, uint32_t ep,
                                                   float* out, int poll_limit) {
  const int lane = threadIdx.x & 31;
  constexpr int EPW = 8;
  if (lane < T)
    for (int p = 0; p < world; p++) st_tagged_sys(peers[p] + ((size_t)rank * T + lane) * D + r, ep, v);
  float part[EPW];
  for (int it = 0;; it++) {
    bool ok = true;
    if (lane < T)
#pragma unroll
      for (int p = 0; p < EPW; p++) {
        part[p] = 0.f;
        if (p < world) {
          const unsigned long long w = ld_tagged_sys(recv + ((size_t)p * T + lane) * D + r);
          ok &= tag_is(w, ep);
          part[p] = tag_val(w);
        }
      }
    if (__all_sync(FULL, ok)) break;
    if (it >= poll_limit) return false;
    __nanosleep(64);
  }
  float sum = 0.f;
#pragma unroll
  for (int p = 0; p < EPW; p++)
    if (p < world) sum = fadd(sum, part[p]);
  if (lane < T) out[(size_t)lane * D + r] = sum;
  return true;
}

// Matrix descriptor of format F with `rows` rows of `cols` values at m (row
// layout of tg_common.cuh).
template <int F>
__device__ __forceinline__ WDesc wdesc(const uint8_t* m, int rows, int cols) {
  const RowLayout L = row_layout(F, cols);
  WDesc w;
  w.main = m;
  w.aux1 = L.a1 >= 0 ? m + L.a1 : nullptr;
  w.aux2 = L.a2 >= 0 ? m + L.a2 : nullptr;
  w.fmt = F;
  w.rows = rows;
  w.cols = cols;
  w.rs = L.rs;
  return w;
}

struct StepArgs {
  const float* x_in;      // [T][D]
  const float* add_in;    // [T][D] or null
  float* x_out;           // [T][D] x_in + add_in, or null
  const float* norm_w;    // [D] or null
  float eps;
  int normalize;
  const float* router_w;  // [E][D]
  const float* router_b;  // [E] or null
  int T, D, E, top_k, I, act, assoc_rule, bias_term;
  const StepExpert* etab; // [E]
  float* logits;          // [T][E]
  float* out;             // [T][D], overwritten with the step's MoE output
  int* sel_idx;           // [T][top_k]
  float* sel_w;           // [T][top_k]
  unsigned long long* sync;   // launch counter
  unsigned long long* lgt;    // [T][E] tagged logits
  unsigned long long* hidt;   // [T*top_k][dbpr][256] tagged hidden
  unsigned long long* hflag;  // [T*top_k*dbpr] tagged: block q of hq is this epoch's
  XQ* hq;                     // [T*top_k*dbpr] Q8 of hidden, each block quantized once in the grid
  int ep_rank, ep_world;      // expert-parallel combine in the kernel (ep_world 1: off)
  unsigned long long* const* ep_peers;   // [ep_world] every shard's receive block
  const unsigned long long* ep_recv;     // this shard's receive block [ep_world][T][D]
  uint32_t stage_bytes;   // ring stage size
  int nst;                // ring stages per warp
  int xcap;               // active rows whose Q8 hidden blocks fit each CTA's shared memory
  int xq_n;               // XQ blocks in shared memory: T gbpr + xcap dbpr, or the larger if alias_x
  int alias_x;            // the Q8 of hidden overlays the Q8 of the inputs (written after phase A)
  int rwc;                // router rows staged per CTA
  int pa;                 // row pairs per phase-A item
  int sb;                 // slots per phase-B item
  DevStatus* st;
  unsigned long long* trace;   // [gridDim.x][16] phase timestamps, or null
  int poll_limit;         // polls of another CTA's (or GPU's) words before giving up
  int skip_logit_cta;     // fault injection (tests): this CTA publishes no logits; -1: none
};

// Phase timestamps for the diagnostics hook tg_cuda_step_trace: slot i of
// this CTA's 32 gets clock64(), slots 12/13 the global timer at start / end,
// slot 19 the logits poll count; then 8 words per warp.
__device__ __forceinline__ unsigned long long gtimer() {
  unsigned long long t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}
#define TG_MARK(i)                                                                         \
  do {                                                                                     \
    if (trace && (threadIdx.x & 31) == 0)                                                  \
      trace[blockIdx.x * 32 + (i)] = (unsigned long long)clock64();                         \
  } while (0)

// A warp's position in its stream of items: phase 0 = gate/up item a (slot
// a / I, row a % I); phase 1 = output row r, slots s .. s + SB - 1.
struct SCur {
  int ph;
  int a, r;
  int s;
};

__device__ __forceinline__ bool scur_next(SCur& c, int gw, int NW, int nA, int D, int n_slots, int SB) {
  if (c.ph == 0) {
    c.a += NW;
    if (c.a < nA) return true;
    c.ph = 1;
    c.r = gw;
    c.s = 0;
    return n_slots > 0 && c.r < D;
  }
  c.s += SB;
  if (c.s < n_slots) return true;
  c.s = 0;
  c.r += NW;
  return c.r < D;
}

// The whole warp: the bulk copies of item c into stage dst (completing on
// bar): lane 0 sets the stage's byte count, then each copy comes from its own
// lane.  Phase 0: rows r0 .. r0 + nr - 1 of slot aord[c.a / nrb]'s gate (lane 0, at dst)
// and up (lane 1, at dst + ghalf); phase 1: row c.r of the down matrices of
// slots c.s .. c.s + SB - 1 (lane j: slot c.s + j, dr bytes apart; SB <= 32).
// Not inlined: the ring calls it from two places.
template <int GF, int DF>
static __device__ __noinline__ void step_issue(const StepExpert* sx, const int* aord, SCur c, uint8_t* dst,
                                               uint64_t* bar, int nrb, int pa, int I, int D, uint32_t ghalf,
                                               uint32_t dr, int n_slots, int SB) {
  const int lane = threadIdx.x & 31;
  if (c.ph == 0) {
    const int sq = c.a / nrb, s = aord[sq], r0 = (c.a - sq * nrb) * pa, nr = min(pa, I - r0);
    const WDesc Gw = wdesc<GF>(sx[s].g, I, D), Uw = wdesc<GF>(sx[s].u, I, D);
    if (lane == 0) mbar_arrive_expect_tx(bar, row_tx(Gw, r0, nr) + row_tx(Uw, r0, nr));
    __syncwarp();
    if (lane == 0) stage_row(Gw, r0, dst, bar, nr);
    else if (lane == 1) stage_row(Uw, r0, dst + ghalf, bar, nr);
  } else {
    const int s = c.s + lane;
    const bool on = s < min(n_slots, c.s + SB);
    const WDesc Dw = wdesc<DF>(sx[on ? s : c.s].d, D, I);
    uint32_t tx = on ? row_tx(Dw, (int)c.r) : 0u;
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) tx += __shfl_xor_sync(FULL, tx, o);
    if (lane == 0) mbar_arrive_expect_tx(bar, tx);
    __syncwarp();
    if (on) stage_row(Dw, (int)c.r, dst + lane * dr, bar);
  }
}

// TRACE: the diagnostics hook (a.trace) is on; the kernel without it keeps
// fewer values live.  T1: a one-token step (a.T == 1), the common decode
// case, compiled with T a constant.  EP: the expert-parallel combine may be
// on (a.ep_world > 1); without it the kernel has no combine code.
template <int GF, int DF, int SW, bool TRACE, bool T1, bool EP>
__global__ void __launch_bounds__(SW * 32, 1) layer_step_kernel(StepArgs a) {
  unsigned long long* const trace = TRACE ? a.trace : nullptr;
  extern __shared__ __align__(128) uint8_t dsm[];
  __shared__ StepShared sh;
  const int lane = threadIdx.x & 31, wid = threadIdx.x >> 5, tid = threadIdx.x;
  const int T = T1 ? 1 : a.T, D = a.D, E = a.E, K = a.top_k, I = a.I;
  const int G = gridDim.x;
  // work items go to warps CTA-interleaved, so every SM gets an even share
  const int gw = wid * G + blockIdx.x, NW = G * SW;
  const int gbpr = (D + QK - 1) / QK, dbpr = (I + QK - 1) / QK;
  uint8_t* ring = dsm + (size_t)wid * a.nst * a.stage_bytes;
  // phase R borrows the rings' bytes: x (and add) at their start, this CTA's
  // router rows at their end; no ring item is issued before R has read them
  const size_t rings = (size_t)SW * a.nst * a.stage_bytes, rrow_bytes = round16((size_t)a.rwc * D * 4);
  float* rrow = reinterpret_cast<float*>(dsm + rings - rrow_bytes);   // [rwc][D]
  XQ* xa = reinterpret_cast<XQ*>(dsm + rings);           // [T][gbpr]
  XQ* xs = a.alias_x ? xa : xa + (size_t)T * gbpr;         // [xcap][dbpr]
  StepExpert* sx = reinterpret_cast<StepExpert*>(xa + a.xq_n);   // [xcap] the slots' experts
  StepExpert* etab = sx + a.xcap;                                                 // [E]
  uint64_t* bar = sh.bars[wid];
  if (trace && tid == 0) trace[blockIdx.x * 32 + 12] = gtimer();
  if (wid == 0) TG_MARK(0);

  // ---- Before the preceding kernel completes: the epoch, this warp's router
  // row and the expert table (none of them written by a preceding kernel).
  // router rows staged here: experts blockIdx.x + r G < E, r < rwc
  const int nrw = min(a.rwc, (E - (int)blockIdx.x + G - 1) / G);
  const bool wbulk = wid < nrw;
  const float* wsrc = a.router_w + (size_t)(blockIdx.x + wid * G) * D;
  if (lane == 0) {
    for (int i = 0; i < a.nst; i++) mbar_init(&bar[i], 1);
    mbar_init(&sh.rbar[wid], 1);
    if (wid == 0) {
      mbar_init(&sh.xbar, 1);
      mbar_init(&sh.ebar, 1);
      sh.ok = 1;
    }
    fence_mbar_init();
    if (wbulk) {
      mbar_arrive_expect_tx(&sh.rbar[wid], (uint32_t)D * 4);
      bulk_g2s(rrow + (size_t)wid * D, wsrc, (uint32_t)D * 4, &sh.rbar[wid]);
    }
    if (wid == 0) {
      mbar_arrive_expect_tx(&sh.ebar, (uint32_t)E * sizeof(StepExpert));
      bulk_g2s(etab, a.etab, (uint32_t)E * sizeof(StepExpert), &sh.ebar);
      unsigned long long prev;
      asm volatile("atom.add.relaxed.gpu.u64 %0, [%1], 1;" : "=l"(prev) : "l"(a.sync) : "memory");
      sh.epoch = (uint32_t)(prev / (unsigned long long)G) + 1u;
    }
  }
  __syncthreads();
  pdl_trigger();   // this CTA holds its epoch count: the next launch may take its own
  const uint32_t ep = sh.epoch;
  pdl_wait();      // x (and add) are written by the preceding kernel
  const uint32_t xbytes = (uint32_t)T * D * 4;
  const bool xstaged = (size_t)xbytes * (a.add_in ? 2 : 1) + rrow_bytes <= rings;
  const float* xsm = reinterpret_cast<const float*>(dsm);
  const float* asm_ = a.add_in ? xsm + (size_t)T * D : nullptr;
  if (tid == 0 && xstaged) {
    mbar_arrive_expect_tx(&sh.xbar, xbytes * (a.add_in ? 2 : 1));
    bulk_g2s(dsm, a.x_in, xbytes, &sh.xbar);
    if (a.add_in) bulk_g2s(dsm + xbytes, a.add_in, xbytes, &sh.xbar);
  }
  if (wid == 0) TG_MARK(1);

  // ---- R, in three passes over the 256-value blocks q of the token rows
  // (token q / gbpr, block q % gbpr), spread over all warps:
  //  1  x' = x + add (written to x_out by CTA 0), each block's sum of squares
  //     and, per router row staged here, its partial logit W_r[e] . (x' * w):
  //     lane chains over the lane's 8 values, then warp trees;
  //  2  per token ss = its blocks' sums in block order, rr = sqrt(ss / D +
  //     eps); per (router row, token) the logit = (the blocks' partial dots
  //     in block order) / rr (+ b), published tagged;
  //  3  N = x' / rr * w, quantized into shared memory (XQ).
  bool dead = false;   // this warp stopped on an error
  const int nq = T * gbpr;
  if (xstaged && !mbar_wait(&sh.xbar, 0)) {
    if (lane == 0) set_error(a.st, ERR_WAIT_TIMEOUT, 36, blockIdx.x, wid);
    dead = true;
  }
  for (int r = 0; r < nrw; r++)
    if (!mbar_wait(&sh.rbar[r], 0)) {
      if (lane == 0) set_error(a.st, ERR_WAIT_TIMEOUT, 30, blockIdx.x + r * G, 0);
      dead = true;
    }
  if (wid == 0) TG_MARK(3);
  const bool nwt = a.normalize && a.norm_w;
  // lane l's values 8l .. 8l + 7 of block q (0 past the row end)
  auto load_block = [&](int q, float (&v)[8], bool store_x) {
    const int t = q / gbpr, i0 = (q - t * gbpr) * QK + 8 * lane;
    const size_t o = (size_t)t * D + i0;
    float4 h[2];
#pragma unroll
    for (int k = 0; k < 2; k++) {
      h[k] = make_float4(0.f, 0.f, 0.f, 0.f);
      if (i0 + 4 * k < D) {
        h[k] = xstaged ? *reinterpret_cast<const float4*>(xsm + o + 4 * k)
                       : __ldcg(reinterpret_cast<const float4*>(a.x_in + o + 4 * k));
        if (a.add_in) {
          const float4 d = xstaged ? *reinterpret_cast<const float4*>(asm_ + o + 4 * k)
                                   : __ldcg(reinterpret_cast<const float4*>(a.add_in + o + 4 * k));
          h[k] = make_float4(fadd(h[k].x, d.x), fadd(h[k].y, d.y), fadd(h[k].z, d.z), fadd(h[k].w, d.w));
        }
        if (store_x) *reinterpret_cast<float4*>(a.x_out + o + 4 * k) = h[k];
      }
    }
    v[0] = h[0].x; v[1] = h[0].y; v[2] = h[0].z; v[3] = h[0].w;
    v[4] = h[1].x; v[5] = h[1].y; v[6] = h[1].z; v[7] = h[1].w;
  };
  auto load8 = [&](const float* p, int i0, float (&w)[8]) {   // 8 floats at p + i0 (0 past D)
#pragma unroll
    for (int k = 0; k < 2; k++) {
      const float4 f = i0 + 4 * k < D ? *reinterpret_cast<const float4*>(p + i0 + 4 * k) : make_float4(0.f, 0.f, 0.f, 0.f);
      w[4 * k] = f.x; w[4 * k + 1] = f.y; w[4 * k + 2] = f.z; w[4 * k + 3] = f.w;
    }
  };
#pragma unroll 1
  for (int q = dead ? nq : wid; q < nq; q += SW) {
    const int t = q / gbpr, b = q - t * gbpr, i0 = b * QK + 8 * lane;
    float v[8];
    load_block(q, v, blockIdx.x == 0 && a.x_out);
    float ss = 0.f;
#pragma unroll
    for (int jj = 0; jj < 8; jj++) ss = __fmaf_rn(v[jj], v[jj], ss);
    float nw[8];
    if (nwt) load8(a.norm_w, i0, nw);
#pragma unroll 1
    for (int r = 0; r < nrw; r++) {
      float w[8];
      load8(rrow + (size_t)r * D, i0, w);
      float dot = 0.f;
#pragma unroll
      for (int jj = 0; jj < 8; jj++) dot = __fmaf_rn(w[jj], nwt ? fmul(v[jj], nw[jj]) : v[jj], dot);
#pragma unroll
      for (int o = 16; o > 0; o >>= 1) dot = fadd(dot, __shfl_xor_sync(FULL, dot, o));
      if (lane == 0) sh.part_dot[r][t][b] = dot;
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) ss = fadd(ss, __shfl_xor_sync(FULL, ss, o));
    if (lane == 0) sh.part_ss[t][b] = ss;
  }
  if (wid == 0) TG_MARK(16);
  if (__syncthreads_or(dead)) {   // wait for the expert table copy, the last one in flight
    if (tid == 0) mbar_wait(&sh.ebar, 0);
    return;
  }
  for (int i = tid; i < T * (1 + nrw); i += SW * 32) {
    const int t = i % T, r = i / T - 1;
    float ss = 0.f;
    for (int b = 0; b < gbpr; b++) ss = fadd(ss, sh.part_ss[t][b]);
    // ss / D: for D a power of two the product with 2^-k, which rounds the
    // same real number once, so it equals the division
    const float msq = (D & (D - 1)) == 0 ? fmul(ss, __int_as_float((128 - __ffs(D)) << 23))   // 2^-log2(D)
                                         : __fdiv_rn(ss, (float)D);
    const float rr = a.normalize ? __fsqrt_rn(fadd(msq, a.eps)) : 1.f;
    if (r < 0) {
      sh.rrt[t] = rr;
      sh.yd[t] = 1.0 / (double)rr;
    } else {
      const int e = blockIdx.x + r * G;
      float dot = 0.f;
      for (int b = 0; b < gbpr; b++) dot = fadd(dot, sh.part_dot[r][t][b]);
      if (a.normalize) dot = __fdiv_rn(dot, rr);
      const float lg = a.router_b ? fadd(dot, a.router_b[e]) : dot;
      a.logits[(size_t)t * E + e] = lg;
      if ((int)blockIdx.x != a.skip_logit_cta) st_tagged(a.lgt + (size_t)t * E + e, ep, lg);
    }
  }
  __syncthreads();
  if (wid == 0) TG_MARK(17);
  if (tid == 0 && !mbar_wait(&sh.ebar, 0)) {
    set_error(a.st, ERR_WAIT_TIMEOUT, 37, blockIdx.x, 0);
    sh.ok = 0;
  }
  if (wid == 0) TG_MARK(2);

  // ---- S: warp t < T polls token t's logits (tagged with this epoch) into
  // registers, takes its top K and their softmax weights (and, for one
  // token, plans); meanwhile the other warps quantize N (R3), and the
  // selecting warps join in when done.  Every CTA plans on its own.
  bool sfail = false;
  if (wid < T) {
    const int t = wid;
    constexpr int NV = STEP_E_MAX / 32;   // logits per lane: experts lane + 32 i
    float v[NV];
    for (int it = 0;; it++) {
      bool ok = true;
#pragma unroll
      for (int i = 0; i < NV; i++) {
        const int e = lane + 32 * i;
        v[i] = 0.f;
        if (e < E) {
          const unsigned long long w = ld_tagged(a.lgt + (size_t)t * E + e);
          ok &= tag_is(w, ep);
          v[i] = tag_val(w);
        }
      }
      if (__all_sync(FULL, ok)) {
        if (trace && t == 0 && lane == 0) trace[blockIdx.x * 32 + 19] = it + 1;
        break;
      }
      if (it >= a.poll_limit) {
        if (lane == 0) set_error(a.st, ERR_WAIT_TIMEOUT, 31, blockIdx.x, t);
        sfail = true;
        break;
      }
      __nanosleep(64);
    }
    if (t == 0) TG_MARK(9);
    // order keys: larger logit larger key, -0 as +0, NaN (1) below every
    // number, absent (0) below NaN; equal keys go to the lower expert id
    // (router.py:35-38, NaN last).  Composite c = key << 32 | (255 - id):
    // larger c first is that order, and the logit is recovered from the key.
    unsigned long long c[NV];
#pragma unroll
    for (int i = 0; i < NV; i++) {
      uint32_t u = __float_as_uint(v[i]);
      if (u == 0x80000000u) u = 0u;
      const int e = lane + 32 * i;   // < 256
      const uint32_t k = e >= E ? 0u : v[i] != v[i] ? 1u : (u >> 31) ? ~u : (u | 0x80000000u);
      c[i] = ((unsigned long long)k << 32) | (uint32_t)(255 - e);
    }
    // the lane's list in that order (a sorting network: 5 comparators when
    // E <= 128 leaves 4 entries per lane, else 19), then K rounds: the
    // warp's largest head wins and its lane steps to its next
    auto cas = [&](int x, int y) {
      const unsigned long long cx = c[x], cy = c[y];
      c[x] = cx > cy ? cx : cy;
      c[y] = cx > cy ? cy : cx;
    };
    const bool four = E <= 128;
    if (four) {
      cas(0, 1); cas(2, 3); cas(0, 2); cas(1, 3); cas(1, 2);
    } else {
      cas(0, 2); cas(1, 3); cas(4, 6); cas(5, 7);
      cas(0, 4); cas(1, 5); cas(2, 6); cas(3, 7);
      cas(0, 1); cas(2, 3); cas(4, 5); cas(6, 7);
      cas(2, 4); cas(3, 5);
      cas(1, 4); cas(3, 6);
      cas(1, 2); cas(3, 4); cas(5, 6);
    }
    if (t == 0) TG_MARK(22);
    // round jj's winner (key M, 255 - id L) is kept by lane jj; the rounds
    // run branch-free (the winner's lane shifts its list by selects)
    uint32_t myM = 0u, myL = 0u;
    const int kk = sfail ? 0 : K;
#pragma unroll
    for (int jj = 0; jj < STEP_K_MAX; jj++) {
      if (jj < kk) {
        const uint32_t hi = (uint32_t)(c[0] >> 32);
        const uint32_t M = __reduce_max_sync(FULL, hi);
        const uint32_t L = __reduce_max_sync(FULL, hi == M ? (uint32_t)c[0] : 0u);
        const bool win = hi == M && (uint32_t)c[0] == L;
        if (lane == jj) {
          myM = M;
          myL = L;
        }
        if (four) {
          c[0] = win ? c[1] : c[0];
          c[1] = win ? c[2] : c[1];
          c[2] = win ? c[3] : c[2];
          c[3] = win ? 0ull : c[3];
        } else {
#pragma unroll
          for (int i = 0; i < NV - 1; i++) c[i] = win ? c[i + 1] : c[i];
          c[NV - 1] = win ? 0ull : c[NV - 1];
        }
      }
    }
    // selection lane (lane < K): expert and logit (-0 comes back as +0,
    // which no softmax term tells apart)
    const int my_e = 255 - (int)myL;
    const float my_v = myM == 1u ? -INFINITY : __uint_as_float(myM >= 0x80000000u ? (myM & 0x7FFFFFFFu) : ~myM);
    if (lane < kk) {
      sh.sel_e[t][lane] = my_e;
      sh.sel_v[t][lane] = my_v;
    }
    __syncwarp();
    if (t == 0) TG_MARK(23);
    // softmax over the selected (lane j < K takes selection j; the sum runs
    // in j order)
    const float v0 = __shfl_sync(FULL, my_v, 0);   // every lane: a full-mask shuffle
    const float ex = lane < K ? expf(fsub(my_v, v0)) : 0.f;
    // the K shuffles are independent: issue them together, then the ordered sum
    float exs[STEP_K_MAX];
#pragma unroll
    for (int jj = 0; jj < STEP_K_MAX; jj++) exs[jj] = shfl(ex, jj);
    float sum = 0.f;
#pragma unroll
    for (int jj = 0; jj < STEP_K_MAX; jj++)
      if (jj < K) sum = fadd(sum, exs[jj]);
    const float w = lane < K ? __fdiv_rn(ex, sum) : 0.f;
    if (t == 0) TG_MARK(24);
    if (lane < kk) {   // (no selection after a failed poll: the step returns below)
      sh.sel_w[t][lane] = w;
      if (blockIdx.x == 0) {
        a.sel_idx[t * K + lane] = my_e;
        a.sel_w[t * K + lane] = w;
      }
    }
    if (T == 1) {
      // one token: its selected experts (nonzero weight, local) ascending by
      // id are the slots, one active row each
      const int e = lane < kk ? my_e : 0x7fffffff;
      const bool valid = lane < kk && w != 0.f && etab[lane < kk ? e : 0].g != nullptr;
      const unsigned vm = __ballot_sync(FULL, valid);
      int rank = 0;
#pragma unroll
      for (int q = 0; q < STEP_K_MAX; q++) {
        const int eq = __shfl_sync(FULL, e, q);
        rank += q < K && ((vm >> q) & 1u) && eq < e;
      }
      if (valid) {
        sh.slot_e[rank] = e;
        sh.slot_n[rank] = 1;
        sh.slot_off[rank] = rank;
        sh.row_t[rank] = 0;
        sh.row_s[rank] = rank;
        sh.slot_a[rank] = rank;
        sh.row_w[rank] = w;
        sx[rank] = etab[e];
      }
      if (lane == 0) {
        sh.n_slots = __popc(vm);
        sh.total = __popc(vm);
      }
    }
    if (t == 0) TG_MARK(14);
  }
  if (wid == T) TG_MARK(20);
  // R3, warps T.. first: N of block q, quantized
  auto r3_prep = [&](int q, float (&v)[8]) {
    const int t = q / gbpr, b = q - t * gbpr, i0 = b * QK + 8 * lane;
    load_block(q, v, false);
    if (a.normalize) {
      const float rr = sh.rrt[t];
      const double yd = sh.yd[t];
      float nw[8];
      if (a.norm_w) load8(a.norm_w, i0, nw);
#pragma unroll
      for (int jj = 0; jj < 8; jj++) {
        float x = div_rn_d(v[jj], rr, yd);
        if (a.norm_w) x = fmul(x, nw[jj]);
        v[jj] = i0 + jj < D ? x : 0.f;
      }
    }
  };
  auto r3_n = [&](int q) { return min(QK, D - (q % gbpr) * QK); };
  if (nq <= SW) {
#pragma unroll 1
    for (int q = (wid + SW - T) % SW; q < nq; q += SW) {
      float v[8];
      r3_prep(q, v);
      quantize_xq<GF == FMT_MXFP4, GF>(v, r3_n(q), xa + q);
    }
  } else {
    // two blocks per pass (independent chains; a missing second block
    // repeats the first, rewriting the same bytes)
#pragma unroll 1
    for (int q = (wid + SW - T) % SW; q < nq; q += 2 * SW) {
      const int q2 = q + SW < nq ? q + SW : q;
      float v[8], v2[8];
      r3_prep(q, v);
      r3_prep(q2, v2);
      quantize_xq<GF == FMT_MXFP4, GF>(v, r3_n(q), xa + q);
      quantize_xq<GF == FMT_MXFP4, GF>(v2, r3_n(q2), xa + q2);
    }
  }
  if (wid == T) TG_MARK(18);
  for (int i = tid; i < E; i += SW * 32) sh.cnt[i] = 0;
  if (__syncthreads_or(sfail || !sh.ok)) return;
  if (wid == 0) TG_MARK(21);
  if (T > 1) {
    // experts held by another GPU (no local weights) are skipped; their
    // contribution arrives through the cross-GPU sum
    // cnt[e]: the tokens that selected expert e, as a bit mask
    for (int i = tid; i < T * K; i += SW * 32) {
      const int t = i / K, j = i - t * K;
      const int e = sh.sel_e[t][j];
      if (sh.sel_w[t][j] != 0.f && etab[e].g) atomicOr(&sh.cnt[e], 1 << t);
    }
    __syncthreads();
    {   // exclusive scans of row counts and of non-empty experts over e < E <= 256
      const int c = tid < E ? __popc(sh.cnt[tid]) : 0, nz = c > 0;
      int sc = c, sz = nz;
#pragma unroll
      for (int o = 1; o < 32; o <<= 1) {
        const int a1 = __shfl_up_sync(FULL, sc, o), a2 = __shfl_up_sync(FULL, sz, o);
        if (lane >= o) {
          sc += a1;
          sz += a2;
        }
      }
      if (lane == 31) {
        sh.wsum[0][wid] = sc;
        sh.wsum[1][wid] = sz;
      }
      __syncthreads();
      int bc = 0, bz = 0;
      for (int j = 0; j < wid; j++) {
        bc += sh.wsum[0][j];
        bz += sh.wsum[1][j];
      }
      if (tid < E) {
        sh.off[tid] = bc + sc - c;
        sh.slot_of[tid] = nz ? bz + sz - 1 : -1;
      }
      if (tid == SW * 32 - 1) {
        sh.n_slots = bz + sz;
        sh.total = bc + sc;
      }
    }
    __syncthreads();
    for (int e = tid; e < E; e += SW * 32) {
      const int s = sh.slot_of[e];
      if (s < 0) continue;
      sh.slot_e[s] = e;
      sh.slot_n[s] = __popc(sh.cnt[e]);
      sh.slot_off[s] = sh.off[e];
      sx[s] = etab[e];
    }
    // a slot's rows in token order: (t, j) goes after the slot's earlier tokens
    for (int i = tid; i < T * K; i += SW * 32) {
      const int t = i / K, j = i - t * K;
      const int e = sh.sel_e[t][j];
      const int m = sh.cnt[e];
      if (!((m >> t) & 1) || sh.sel_w[t][j] == 0.f) continue;   // (a token selects an expert at most once)
      const int o = sh.off[e] + __popc(m & ((1 << t) - 1));
      sh.row_t[o] = t;
      sh.row_s[o] = sh.slot_of[e];
      sh.row_w[o] = sh.sel_w[t][j];
    }
    __syncthreads();
    // phase A takes the slots with the most rows first, so that their longer
    // items spread over the warps (ties in slot order)
    if (wid == 0)
      for (int q = lane; q < sh.n_slots; q += 32) {
        const int nq = sh.slot_n[q];
        int rk = 0;
        for (int t = 0; t < sh.n_slots; t++) {
          const int nt2 = sh.slot_n[t];
          rk += nt2 > nq || (nt2 == nq && t < q);
        }
        sh.slot_a[rk] = q;
      }
    __syncthreads();
  }

  if (wid == 0) TG_MARK(4);
  // ---- A and B: the per-warp ring
  // Phase A items are (slot, block of pa consecutive rows of gate and of up);
  // phase B items are (output row, group of sb consecutive slots).  With a
  // 256-block format, phase A lanes are (row, gate|up, block) and phase B
  // lanes (slot, block): each lane folds one block's term in the reference's
  // order and the row's lanes fold the terms in block order.  Other formats
  // split each row over half a warp (half_dot_sub32).
  const int n_slots = sh.n_slots, total = sh.total;
  const int grs = row_layout(GF, D).rs, drs = row_layout(DF, I).rs;
  constexpr bool GBLK = GF == FMT_Q4K || GF == FMT_Q6K;
  constexpr bool DBLK = DF == FMT_Q4K || DF == FMT_Q6K;
  const int pa = a.pa, SB = a.sb;
  const uint32_t ghalf = rows_stage_bytes(grs, pa), dr = rows_stage_bytes(drs, 1);
  const int nrb = (I + pa - 1) / pa;   // row blocks per slot
  const int nA = n_slots * nrb;
  const int k = T, rule = a.assoc_rule, act = a.act;
  const int gbb = GF == FMT_Q4K ? Q4K_BYTES : 192, dbb = DF == FMT_Q4K ? Q4K_BYTES : 192;   // main bytes per block

  auto issue = [&](const SCur& c, int stg) {   // the whole warp
    step_issue<GF, DF>(sx, sh.slot_a, c, ring + (size_t)stg * a.stage_bytes, &bar[stg], nrb, pa, I, D, ghalf, dr,
                       n_slots, SB);
  };
  SCur ic{0, gw - NW, 0, 0};
  int issued = 0;
  bool more = true;
  fence_proxy_async();   // the rings' bytes were read through the generic proxy in phase R (any lane may issue)
  for (int i = 0; i < a.nst && more; i++) {
    more = scur_next(ic, gw, NW, nA, D, n_slots, SB);
    if (more) {
      issue(ic, i);
      issued++;
    }
  }
  int j = 0;   // items consumed
  // Stops the warp: no further copies are issued, and those in flight
  // (items from .. issued-1) are waited for, each wait bounded.
  auto stop = [&](int from) {
    if (dead) return;
    dead = true;
    for (int i = from; i < issued; i++) mbar_wait(&bar[i % a.nst], (uint32_t)(i / a.nst) & 1u);
  };
  unsigned long long* tw = sh.tw[wid];   // trace: wait / compute / issue cycles, phases A and B
  if (lane == 0)
    for (int q = 0; q < 8; q++) tw[q] = 0;
  int tph = 0;
  long long tc = 0;
  auto wait_stage = [&](int stg, int item) -> bool {
    if (dead) return false;
    if (trace) tc = clock64();
    const bool okw = mbar_wait(&bar[stg], (uint32_t)(item / a.nst) & 1u);
    if (trace) {
      const long long t1 = clock64();
      if (lane == 0) tw[3 * tph] += t1 - tc;
      tc = t1;
    }
    if (!okw) {
      if (lane == 0) set_error(a.st, ERR_WAIT_TIMEOUT, 32, blockIdx.x, wid);
      stop(item + 1);
      return false;
    }
    return true;
  };
  auto refill = [&](int stg) {
    __syncwarp();
    long long t0 = 0;
    if (trace) {
      t0 = clock64();
      if (lane == 0) tw[3 * tph + 1] += t0 - tc;
    }
    if (dead || !more) return;
    more = scur_next(ic, gw, NW, nA, D, n_slots, SB);
    if (more) {
      issue(ic, stg);
      issued++;
    }
    if (trace && lane == 0) tw[3 * tph + 2] += clock64() - t0;
  };

  // phase A: items gw, gw + NW, ... < nA
  const int gbpr2 = GBLK ? gbpr : 1;                 // lanes per row
  const int a_pr = lane / (2 * gbpr2), a_m = (lane / gbpr2) & 1, a_b = lane - (lane / gbpr2) * gbpr2;
  for (int it = gw; it < nA; it += NW, j++) {
    const int stg = j % a.nst;
    if (!wait_stage(stg, j)) continue;
    const int sq = it / nrb, s = sh.slot_a[sq], r0 = (it - sq * nrb) * pa, nr = min(pa, I - r0);
    const StepExpert& X = sx[s];
    const WDesc Gw = wdesc<GF>(X.g, I, D), Uw = wdesc<GF>(X.u, I, D);
    const uint8_t* dst = ring + (size_t)stg * a.stage_bytes;
    const int n = sh.slot_n[s], off = sh.slot_off[s];
    if constexpr (GBLK) {
      const bool on = a_pr < nr;
      const RowPtrs rp = row_ptrs(a_m ? Uw : Gw, r0, dst + (a_m ? ghalf : 0));
      const uint8_t* mb = rp.m + (size_t)a_pr * grs + (size_t)a_b * gbb;
      const uint8_t* s1b = rp.a1 ? rp.a1 + (size_t)a_pr * grs + a_b * 16 : nullptr;
      const uint8_t* s2b = rp.a2 ? rp.a2 + (size_t)a_pr * grs + a_b * 2 : nullptr;
      const int r = r0 + a_pr;
#pragma unroll 1
      for (int jj = 0; jj < n; jj++) {
        const bool x4 = use_x4(rule, jj & ~3, n, k);
        float term = 0.f;
        if (on) {
          const XQ& xb = xa[(size_t)sh.row_t[off + jj] * gbpr + a_b];
          if constexpr (GF == FMT_Q4K) term = q4k_block_term(mb, xb, x4);
          else term = q6k_block_term(mb, s1b, s2b, xb);
        }
        const float tot = fold_row(term, lane - a_b, gbpr2);
        const float up = shfl(tot, min(lane + gbpr2, 31));
        if (on && a_m == 0 && a_b == 0) {
          float gt = tot, ut = up;
          if (X.gb) {
            gt = fadd(gt, X.gb[r]);
            ut = fadd(ut, X.ub[r]);
          }
          st_tagged(a.hidt + hid_word(off + jj, r, dbpr), ep, act_fn(act, gt, ut));
        }
      }
    } else {
      // one row: lanes 0-15 its gate row, lanes 16-31 its up row
      const RowPtrs rp = row_ptrs(lane < 16 ? Gw : Uw, r0, dst + (lane < 16 ? 0 : ghalf));
#pragma unroll 1
      for (int jj = 0; jj < n; jj++) {
        const float v = half_dot_sub32<GF>(rp, D / 32, xa + (size_t)sh.row_t[off + jj] * gbpr);
        const float up = shfl(v, 16);
        if (lane == 0) {
          float gt = v, ut = up;
          if (X.gb) {
            gt = fadd(gt, X.gb[r0]);
            ut = fadd(ut, X.ub[r0]);
          }
          st_tagged(a.hidt + hid_word(off + jj, r0, dbpr), ep, act_fn(act, gt, ut));
        }
      }
    }
    refill(stg);
  }

  if (wid == 0) TG_MARK(5);
  if (wid == SW - 1) TG_MARK(10);
  tph = 1;
  // ---- hidden: every CTA needs the Q8 of every active row's hidden blocks
  // (tagged with this epoch) in its shared memory.  A few blocks: each CTA
  // polls and quantizes them itself, two blocks per warp at a time.
  bool okh = !dead;
  if (total > a.xcap) {
    if (tid == 0) set_error(a.st, ERR_BAD_PLAN, 35, total, a.xcap);
    okh = false;
  }
  const int nh = okh ? total * dbpr : 0;   // hidden blocks
  const long long ta = trace ? clock64() : 0;
  if (a.alias_x) __syncthreads();   // xs overlays xa: every warp of this CTA is past phase A
  if (wid == 0) TG_MARK(25);
  if (nh > 4 * SW) {
    // Many blocks: each is quantized once in the grid (block q by warp q / G
    // of CTA q % G) into hq, published by its tagged flag; every CTA then
    // copies all of them, each warp's lanes polling 32 flags at a time.
    for (int q = (int)blockIdx.x + wid * G; q < nh && okh; q += NW) {
      const int nq = min(QK, I - (q % dbpr) * QK);
      const unsigned long long* src = a.hidt + (size_t)q * 256 + 2 * lane;
      float v[8];
      for (int it = 0;; it++) {
        bool ok = true;
#pragma unroll
        for (int p = 0; p < 4; p++) {
          const int i = 8 * lane + 2 * p;
          v[2 * p] = v[2 * p + 1] = 0.f;
          if (i < nq) {
            const ulonglong2 w = ld_tagged2(src + 64 * p);
            ok &= tag_is(w.x, ep);
            v[2 * p] = tag_val(w.x);
            if (i + 1 < nq) {
              ok &= tag_is(w.y, ep);
              v[2 * p + 1] = tag_val(w.y);
            }
          }
        }
        if (__all_sync(FULL, ok)) {
          if (wid == 0 && q == (int)blockIdx.x) TG_MARK(26);
          break;
        }
        if (it >= a.poll_limit) {
          if (lane == 0) set_error(a.st, ERR_WAIT_TIMEOUT, 33, blockIdx.x, wid);
          okh = false;
          break;
        }
        __nanosleep(64);
      }
      if (!okh) break;
      quantize_xq<DF == FMT_MXFP4, DF>(v, nq, a.hq + q);
      __syncwarp();   // the warp's stores of block q before its flag
      if (lane == 31) st_flag_release(a.hflag + q, ep);
    }
    if (wid == 0) TG_MARK(6);
    for (int q0 = wid; q0 < nh && okh; q0 += 32 * SW) {
      const int q = q0 + SW * lane;
      bool seen = q >= nh;
      for (int it = 0;; it++) {
        if (!seen) seen = tag_is(ld_flag_acquire(a.hflag + q), ep);
        if (__all_sync(FULL, seen)) {
          if (wid == 0 && q0 == 0) TG_MARK(27);
          if (trace && lane == 0) {
            tw[6] += it + 1;
            if (q0 == wid) tw[7] = clock64() - ta;
          }
          break;
        }
        if (it >= a.poll_limit) {
          if (lane == 0) set_error(a.st, ERR_WAIT_TIMEOUT, 34, blockIdx.x, wid);
          okh = false;
          break;
        }
        __nanosleep(64);
      }
      if (!okh) break;
      __syncwarp();   // each lane's acquired flag before the warp reads the blocks
      constexpr int QW = sizeof(XQ) / 16;
      const int nb = min(32, (nh - q0 + SW - 1) / SW);   // blocks q0 + SW i, i < nb
      for (int i = lane; i < nb * QW; i += 32) {
        const int bi = i / QW, c = i - bi * QW;
        reinterpret_cast<uint4*>(xs + q0 + SW * bi)[c] = __ldcg(reinterpret_cast<const uint4*>(a.hq + q0 + SW * bi) + c);
      }
    }
  } else {
    for (int q0 = wid; q0 < nh; q0 += 2 * SW) {
      float v[2][8];
      int nn[2];
#pragma unroll
      for (int h = 0; h < 2; h++) {
        const int q = q0 + h * SW;
        nn[h] = q < nh ? min(QK, I - (q % dbpr) * QK) : 0;
      }
      for (int it = 0;; it++) {
        bool ok = true;
#pragma unroll
        for (int h = 0; h < 2; h++) {
          const unsigned long long* src = a.hidt + (size_t)(q0 + h * SW) * 256 + 2 * lane;
#pragma unroll
          for (int p = 0; p < 4; p++) {
            const int i = 8 * lane + 2 * p;
            v[h][2 * p] = v[h][2 * p + 1] = 0.f;
            if (i < nn[h]) {
              const ulonglong2 w = ld_tagged2(src + 64 * p);
              ok &= tag_is(w.x, ep);
              v[h][2 * p] = tag_val(w.x);
              if (i + 1 < nn[h]) {
                ok &= tag_is(w.y, ep);
                v[h][2 * p + 1] = tag_val(w.y);
              }
            }
          }
        }
        if (__all_sync(FULL, ok)) {
          if (trace && lane == 0) {
            tw[6] += it + 1;
            if (q0 == wid) tw[7] = clock64() - ta;
          }
          break;
        }
        if (it >= a.poll_limit) {
          if (lane == 0) set_error(a.st, ERR_WAIT_TIMEOUT, 33, blockIdx.x, wid);
          okh = false;
          break;
        }
        __nanosleep(64);
      }
      if (!okh) break;
      if (wid == 0 && q0 == 0) TG_MARK(6);
#pragma unroll 1
      for (int h = 0; h < 2 && nn[h] > 0; h++) {
        XQ& xb = xs[q0 + h * SW];
        float vv[8];
#pragma unroll
        for (int jj = 0; jj < 8; jj++) vv[jj] = h ? v[1][jj] : v[0][jj];
        quantize_xq<DF == FMT_MXFP4, DF>(vv, nn[h], &xb);
      }
    }
  }
  if (wid == 0) TG_MARK(15);
  if (!__syncthreads_and(okh)) stop(j);
  if (wid == 0) TG_MARK(7);

  // phase B: rows r = gw, gw + NW, ... < D; slots in groups of SB (one ring
  // stage), the group's active rows in rounds of rpr: lane = block * rpr +
  // row, so the 8 lanes of a quarter warp read 8 different rows (distinct
  // slots' bytes, or one slot's bytes broadcast)
  const int dbpr2 = DBLK ? dbpr : 1, rpr = 32 / dbpr2;
  const int b_b = lane / rpr, b_r = lane - b_b * rpr;
  // Output row r (lane t < T holds token t's value); expert parallel: this
  // shard's part, combined across shards by ep_combine_row.
  auto emit_row = [&](int r, float v) {
    if (dead) return;
    if (!EP || a.ep_world == 1) {
      if (lane < T) a.out[(size_t)lane * D + r] = v;
    } else if (!ep_combine_row(a.ep_peers, a.ep_recv, a.ep_rank, a.ep_world, T, D, r, v, ep, a.out,
                                       a.poll_limit)) {
      if (lane == 0) set_error(a.st, ERR_WAIT_TIMEOUT, 38, blockIdx.x, r);
      dead = true;
    }
  };
  if (n_slots > 0)
    for (int r = gw; r < D; r += NW) {
      float acc = 0.f;   // lane t < T: token t's output, parts added in slot order
      for (int s0 = 0; s0 < n_slots; s0 += SB, j++) {
        const int stg = j % a.nst;
        if (!wait_stage(stg, j)) continue;
        const uint8_t* dst = ring + (size_t)stg * a.stage_bytes;
        const int s1 = min(n_slots, s0 + SB);
        // the group's active rows ra .. rb - 1 (slot-major, each slot's in token order)
        const int ra = sh.slot_off[s0], rb = sh.slot_off[s1 - 1] + sh.slot_n[s1 - 1];
        if constexpr (DBLK) {
          // rounds of rpr rows: lane = block * rpr + row, each lane one block term
          for (int q0 = ra; q0 < rb; q0 += rpr) {
            const int rho = q0 + b_r, rc = rho < rb ? rho : q0;
            const bool on = b_b < dbpr2 && rho < rb;
            const int sc = sh.row_s[rc];
            const StepExpert& X = sx[sc];
            const RowPtrs rp = row_ptrs(wdesc<DF>(X.d, D, I), (int)r, dst + (sc - s0) * dr);
            const int bb = min(b_b, dbpr2 - 1);
            float term = 0.f;
            if (on) {
              const XQ& xb = xs[(size_t)rc * dbpr + bb];
              const uint8_t* mb = rp.m + (size_t)bb * dbb;
              if constexpr (DF == FMT_Q4K) {
                term = q4k_block_term(mb, xb, use_x4(rule, (rc - sh.slot_off[sc]) & ~3, sh.slot_n[sc], k));
              } else {
                term = q6k_block_term(mb, rp.a1 ? rp.a1 + bb * 16 : nullptr, rp.a2 ? rp.a2 + bb * 2 : nullptr, xb);
              }
            }
            const float tot = fold_row(term, b_r, dbpr2, rpr);
            float part = 0.f;
            if (rho < rb) {
              const float w = sh.row_w[rc];
              part = a.bias_term ? fmul(w, fadd(tot, X.db ? X.db[r] : 0.f)) : fmul(w, tot);
            }
            // row q0 + i's part on lane i: token t's lane adds the round's rows in order
            const int nr = min(rpr, rb - q0);
            for (int i = 0; i < nr; i++) {
              const float v = shfl(part, i);
              if (lane == sh.row_t[q0 + i]) acc = fadd(acc, v);
            }
          }
        } else {
          // two rows per pass: lanes 0-15 row q0, lanes 16-31 row q0 + 1
#pragma unroll 1
          for (int q0 = ra; q0 < rb; q0 += 2) {
            const int rho = q0 + (lane >> 4), rc = rho < rb ? rho : q0;
            const int sc = sh.row_s[rc];
            const StepExpert& X = sx[sc];
            const RowPtrs rp = row_ptrs(wdesc<DF>(X.d, D, I), r, dst + (sc - s0) * dr);
            const float v = half_dot_sub32<DF>(rp, I / 32, xs + (size_t)rc * dbpr);
            const float w = sh.row_w[rc], db = X.db ? X.db[r] : 0.f;
            const float part = a.bias_term ? fmul(w, fadd(v, db)) : fmul(w, v);
            const float p0 = shfl(part, 0), p1 = shfl(part, 16);
            if (lane == sh.row_t[q0]) acc = fadd(acc, p0);
            if (q0 + 1 < rb && lane == sh.row_t[q0 + 1]) acc = fadd(acc, p1);
          }
        }
        refill(stg);
      }
      emit_row(r, lane < T ? acc : 0.f);
      __syncwarp();
    }
  else
    for (int r = gw; r < D; r += NW) emit_row(r, 0.f);

  if (wid == 0) TG_MARK(8);
  if (wid == SW - 1) TG_MARK(11);
  if (trace && tid == 0) trace[blockIdx.x * 32 + 13] = gtimer();
  if (trace && lane == 0)
    for (int q = 0; q < 8; q++) trace[(size_t)gridDim.x * 32 + ((size_t)blockIdx.x * SW_MAX + wid) * 8 + q] = tw[q];
  // bounded waits for any copies still in flight before the CTA exits
  if (!dead)
    for (int i = j; i < issued; i++) mbar_wait(&bar[i % a.nst], (uint32_t)(i / a.nst) & 1u);
}

// ---------------------------------------------------------------------
// Launcher.

// The exchange block: launch counter (32 words), tagged logits [t][E], tagged
// hidden [t top_k][dbpr][256], hidden blocks' flags [t top_k dbpr] and their
// Q8 [t top_k dbpr] (XQ), each region from a 256-byte boundary.
static size_t round32(size_t n) { return (n + 31) & ~(size_t)31; }
size_t step_sync_words(int T, int E, int top_k, int I) {
  const int t = std::min(T, STEP_T_MAX), dbpr = (I + QK - 1) / QK;
  const size_t nh = (size_t)t * top_k * dbpr;
  return 32 + round32((size_t)t * E) + nh * 256 + round32(nh) + round32(nh * sizeof(XQ) / 8);
}

// Shared-memory shape of one launch, or false when the step does not fit.
struct StepShape {
  uint32_t stage;
  int nst, rwc, xcap, pa, sb, alias, xq_n;
  size_t smem;
};

#define TG_STEP_PAIRS(X)       \
  X(FMT_Q4K, FMT_Q6K)          \
  X(FMT_Q4K, FMT_Q4K)          \
  X(FMT_MXFP4, FMT_MXFP4)      \
  X(FMT_Q6K, FMT_Q6K)          \
  X(FMT_Q80, FMT_Q80)

template <int GF, int DF>
static const void* step_fn(bool trace, bool t1, bool ep) {
  constexpr int SW = GF == FMT_MXFP4 ? SW_MAX : 16;
  if (trace) return reinterpret_cast<const void*>(layer_step_kernel<GF, DF, SW, true, false, true>);
  if (ep)
    return t1 ? reinterpret_cast<const void*>(layer_step_kernel<GF, DF, SW, false, true, true>)
              : reinterpret_cast<const void*>(layer_step_kernel<GF, DF, SW, false, false, true>);
  return t1 ? reinterpret_cast<const void*>(layer_step_kernel<GF, DF, SW, false, true, false>)
            : reinterpret_cast<const void*>(layer_step_kernel<GF, DF, SW, false, false, false>);
}

// The step kernel's static shared memory for a format pair (StepShared and
// whatever the compiler adds to it), cached; 0 if it cannot be read.
static size_t step_static_smem(int gf, int df) {
  static size_t cache[16][16] = {};
  if (gf < 0 || gf >= 16 || df < 0 || df >= 16) return 0;
  if (!cache[gf][df]) {
    const void* fn = nullptr;
#define TG_STEP_FN(GFV, DFV) \
  if (gf == GFV && df == DFV) fn = step_fn<GFV, DFV>(false, false, true);
    TG_STEP_PAIRS(TG_STEP_FN)
#undef TG_STEP_FN
    cudaFuncAttributes at{};
    if (!fn || cudaFuncGetAttributes(&at, fn) != cudaSuccess) return 0;
    cache[gf][df] = at.sharedSizeBytes;
  }
  return cache[gf][df];
}

static size_t step_smem_optin() {
  static int v = 0;
  if (!v) {
    int dev = 0;
    cudaGetDevice(&dev);
    cudaDeviceGetAttribute(&v, cudaDevAttrMaxSharedMemoryPerBlockOptin, dev);
    if (v < 48 * 1024) v = 48 * 1024;
  }
  return (size_t)v;
}

static int step_sms() {
  static int sms = 0;
  if (!sms) {
    int dev = 0;
    cudaGetDevice(&dev);
    cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
    if (sms < 1) sms = 1;
  }
  return sms;
}

// Warps per CTA of a step with this gate format.
static int step_warps_for(int gate_fmt) { return gate_fmt == FMT_MXFP4 ? SW_MAX : 16; }

static bool step_shape(const StepLaunch& l, StepShape& sh) {
  const int SW = step_warps_for(l.gate_fmt);
  const bool gf = l.gate_fmt == FMT_Q4K || l.gate_fmt == FMT_Q6K || l.gate_fmt == FMT_MXFP4 || l.gate_fmt == FMT_Q80;
  const bool df = l.down_fmt == FMT_Q4K || l.down_fmt == FMT_Q6K || l.down_fmt == FMT_MXFP4 || l.down_fmt == FMT_Q80;
  if (!gf || !df || l.T < 1 || l.T > STEP_T_MAX || l.E < 1 || l.E > STEP_E_MAX || l.top_k < 1 ||
      l.top_k > STEP_K_MAX || l.top_k > l.E || (l.D & 3))
    return false;
  // rows are read and written as float4; the expert table and the exchange
  // block are copied / addressed in 16-byte units
  const void* ptrs[] = {l.x_in, l.add_in, l.x_out, l.norm_w, l.router_w, l.out, l.etab, l.sync};
  for (const void* q : ptrs)
    if (reinterpret_cast<uintptr_t>(q) & 15) return false;
  if (!l.etab || !l.sync || l.ep_world < 1 || l.ep_world > 8 || (l.ep_world > 1 && (!l.ep_peers || !l.ep_recv)))
    return false;
  // 256-block formats put a row's blocks on consecutive lanes: at most 16
  // blocks per gate / up row (a row pair fills the warp), 32 per down row
  const bool gblk = l.gate_fmt == FMT_Q4K || l.gate_fmt == FMT_Q6K;
  const bool dblk = l.down_fmt == FMT_Q4K || l.down_fmt == FMT_Q6K;
  const int bg = l.D / QK, bd = l.I / QK;
  if ((gblk && (bg < 1 || bg > 16)) || (dblk && (bd < 1 || bd > 32))) return false;
  const int G = step_sms();
  sh.pa = gblk ? std::max(1, 16 / bg) : 1;
  sh.rwc = (l.E + G - 1) / G;
  if (sh.rwc > STEP_RW_MAX || (l.D + QK - 1) / QK > STEP_GB_MAX) return false;
  const int gbpr = (l.D + QK - 1) / QK, dbpr = (l.I + QK - 1) / QK;
  sh.xcap = l.T * l.top_k;
  // the router rows live at the end of the rings' bytes during phase R
  const size_t rrow = round16((size_t)sh.rwc * l.D * 4);
  const size_t nxa = (size_t)l.T * gbpr, nxh = (size_t)sh.xcap * dbpr;
  const size_t tabs = (size_t)sh.xcap * sizeof(StepExpert) + (size_t)l.E * sizeof(StepExpert);
  const size_t optin = step_smem_optin();
  const size_t stat = std::max(sizeof(StepShared), step_static_smem(l.gate_fmt, l.down_fmt));
  const size_t budget = optin - 256 - stat;
  const uint32_t dr = rows_stage_bytes(row_layout(l.down_fmt, l.I).rs, 1);
  const uint32_t sa = 2 * rows_stage_bytes(row_layout(l.gate_fmt, l.D).rs, sh.pa);
  // phase-B slots per item (one stage): as many as fit; 32-value formats at
  // most what the phase-A stage holds
  const int max_slots = std::min(l.E, l.T * l.top_k);
  const int sb_cap = std::max(1, std::min(max_slots, dblk ? 32 : std::max(2, (int)(sa / dr))));
  // the Q8 of the inputs and of hidden side by side, else (larger steps)
  // overlaid: hidden is quantized after phase A
  for (int alias = 0; alias < 2; alias++) {
    const size_t nxq = alias ? std::max(nxa, nxh) : nxa + nxh;
    const size_t fixed = nxq * sizeof(XQ) + tabs;
    if (optin < stat + fixed + rrow + 4096) continue;
    int sb = sb_cap;
    for (;;) {
      sh.stage = std::max(sa, (uint32_t)sb * dr);
      if (fixed + (size_t)SW * 2 * sh.stage <= budget || sb == 1) break;
      sb--;
    }
    sh.sb = sb;
    if (fixed + (size_t)SW * 2 * sh.stage > budget || (size_t)SW * 2 * sh.stage < rrow) continue;
    sh.nst = (int)std::min<size_t>(ST_MAX_NST, (budget - fixed) / ((size_t)SW * sh.stage));
    sh.smem = (size_t)SW * sh.nst * sh.stage + fixed;
    sh.alias = alias;
    sh.xq_n = (int)nxq;
    return true;
  }
  return false;
}

template <int GF, int DF>
static cudaError_t step_launch(StepArgs a, const StepShape& sh, cudaStream_t s) {
  constexpr int SW = GF == FMT_MXFP4 ? SW_MAX : 16;
  a.stage_bytes = sh.stage;
  a.nst = sh.nst;
  a.rwc = sh.rwc;
  a.xcap = sh.xcap;
  a.pa = sh.pa;
  a.sb = sh.sb;
  a.alias_x = sh.alias;
  a.xq_n = sh.xq_n;
  const void* fn = step_fn<GF, DF>(a.trace != nullptr, a.T == 1, a.ep_world > 1);
  cudaError_t e = ensure_smem(fn, sh.smem);
  if (e != cudaSuccess) return e;
  static size_t fits = 0;   // largest shared-memory size known to fit one CTA per SM
  if (sh.smem > fits) {
    int per = 0;
    e = cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per, fn, SW * 32, sh.smem);
    if (e != cudaSuccess) return e;
    if (per < 1) return cudaErrorInvalidConfiguration;
    fits = sh.smem;
  }
  cudaLaunchConfig_t cfg{};
  cfg.gridDim = dim3(step_sms());
  cfg.blockDim = dim3(SW * 32);
  cfg.dynamicSmemBytes = sh.smem;
  cfg.stream = s;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  void* args[] = {(void*)&a};
  return cudaLaunchKernelExC(&cfg, fn, args);
}

// Gate / down format pairs with a fused step kernel.
bool step_eligible(const StepLaunch& l) {
  StepShape sh;
  if (!step_shape(l, sh)) return false;
#define TG_STEP_HAS(GFV, DFV) \
  if (l.gate_fmt == GFV && l.down_fmt == DFV) return true;
  TG_STEP_PAIRS(TG_STEP_HAS)
#undef TG_STEP_HAS
  return false;
}

static unsigned long long* g_step_trace = nullptr;
void set_step_trace(void* p) { g_step_trace = static_cast<unsigned long long*>(p); }
int step_warps() { return SW_MAX; }
static int g_poll_limit = STEP_POLLS, g_skip_logit_cta = -1;
void set_step_fault(int skip_logit_cta, int poll_limit) {
  g_skip_logit_cta = skip_logit_cta;
  g_poll_limit = poll_limit > 0 ? poll_limit : STEP_POLLS;
}

cudaError_t launch_layer_step(const StepLaunch& l, cudaStream_t s) {
  StepShape sh;
  if (!step_shape(l, sh)) return cudaErrorInvalidValue;
  StepArgs a{};
  a.x_in = l.x_in;
  a.add_in = l.add_in;
  a.x_out = l.x_out;
  a.norm_w = l.norm_w;
  a.eps = l.eps;
  a.normalize = l.normalize;
  a.router_w = l.router_w;
  a.router_b = l.router_b;
  a.T = l.T;
  a.D = l.D;
  a.E = l.E;
  a.top_k = l.top_k;
  a.I = l.I;
  a.act = l.act;
  a.assoc_rule = l.assoc_rule;
  a.bias_term = l.bias_term;
  a.etab = l.etab;
  a.logits = l.logits;
  a.out = l.out;
  a.sel_idx = l.sel_idx;
  a.sel_w = l.sel_w;
  a.sync = l.sync;
  // the tagged regions are placed for this launch's T (inside the block the
  // layer sized for its largest T); words left there by earlier launches
  // carry older epochs and are never taken
  a.lgt = l.sync + 32;
  a.hidt = a.lgt + round32((size_t)std::min(l.T, STEP_T_MAX) * l.E);
  {
    const size_t nh = (size_t)std::min(l.T, STEP_T_MAX) * l.top_k * ((l.I + QK - 1) / QK);
    a.hflag = a.hidt + nh * 256;
    a.hq = reinterpret_cast<XQ*>(a.hflag + round32(nh));
  }
  a.st = l.st;
  a.trace = g_step_trace;
  a.poll_limit = g_poll_limit;
  a.skip_logit_cta = g_skip_logit_cta;
  a.ep_rank = l.ep_rank;
  a.ep_world = l.ep_world;
  a.ep_peers = l.ep_peers;
  a.ep_recv = l.ep_recv;
#define TG_STEP_CASE(GFV, DFV) \
  if (l.gate_fmt == GFV && l.down_fmt == DFV) return step_launch<GFV, DFV>(a, sh, s);
  TG_STEP_PAIRS(TG_STEP_CASE)
#undef TG_STEP_CASE
  return cudaErrorInvalidValue;
}

}  // namespace tg
