// tg_gemm.cu — the MoE expert path for batched steps (T > 8 rows) as grouped
// GEMMs on the 5th-generation tensor cores (tcgen05, kind::i8, accumulators
// in tensor memory).
//
// The arithmetic is the reference's (csrc/libtinygiant.c): per expert, per
// weight row and active input row, per 256-value block the int32 sum of each
// sub-block (Q4_K: 32 values, dot_q4k_q8 223-337; Q6_K: 16 values,
// dot_q6k_q8 403-487) and the block's fp32 fold in the reference's
// association, blocks folded in order.  The tensor cores produce exactly
// those integer sums: each tcgen05.mma covers one sub-block (K = 32 bytes),
// starts from zero and writes its own tensor-memory columns, so no sum mixes
// two sub-blocks; the epilogue reads the sums back (tcgen05.ld) and folds them
// in fp32 as the matvec kernels do.  Outputs equal tg_moe_forward_rows_v2's.
//
// Work unit: (slot, matrix, 128 weight rows, 32 active rows of the slot).
// Persistent CTAs (one per SM) walk the units.  Per unit the 128 rows' whole
// weight window is one bulk copy (cp.async.bulk, no multicast); per 256-value
// block the CTA unpacks the rows into int8 tiles in the canonical K-major
// no-swizzle layout (8-row x 16-byte core matrices), stages the active rows'
// Q8 blocks the same way, issues the MMAs from one thread and commits them to
// an mbarrier.  Sixteen warps read the accumulators: warp w takes TMEM lanes
// 32 (w % 4) .. (its rows) and active rows 8 (w / 4) .. + 7.
//
//   gate/up pass:  gu[row][m I + r] = dot(matrix m of the slot's expert, row r; x of the active row)
//   act + Q8 pass: hq8[row] = Q8(act(gu gate + gb, gu up + ub))
//   down pass:     parts[row][r] = w (dot(down row r, hidden row) + db[r])
//   combine:       out[t][r] += parts of token t's active rows in slot order (1428-1434)
#include <algorithm>

#include "tg_moe.h"
#include "tg_q8.cuh"
#include "tg_warpdot.cuh"

namespace tg {

constexpr int TC_M = 128;     // weight rows per unit (MMA M)
constexpr int TC_N = 32;      // active rows per unit (MMA N)
constexpr int TC_WARPS = 16;
constexpr int TC_MAX_SLOTS = 256;

__device__ __forceinline__ uint64_t umma_desc(uint32_t saddr) {
  // canonical K-major, no swizzle: core matrices of 8 rows x 16 bytes,
  // the two 16-byte halves of K 128 bytes apart, 8-row groups 256 bytes apart
  return (uint64_t)((saddr >> 4) & 0x3FFFu) | ((uint64_t)(128u >> 4) << 16) | ((uint64_t)(256u >> 4) << 32) |
         (1ull << 46);
}
// Byte offset of (row, k) in a 32-byte-K tile of that layout.
__device__ __forceinline__ int kmaj(int row, int k) { return (row >> 3) * 256 + (k >> 4) * 128 + (row & 7) * 16 + (k & 15); }

// kind::i8 instruction descriptor: int32 accumulators, A signed or not,
// B signed, both K-major, M = 128, N = TC_N.
__host__ __device__ constexpr uint32_t umma_idesc(bool a_signed) {
  return (2u << 4) | ((a_signed ? 1u : 0u) << 7) | (1u << 10) | ((uint32_t)(TC_N >> 3) << 17) |
         ((uint32_t)(TC_M >> 4) << 24);
}

__device__ __forceinline__ void tc_fence_before() { asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory"); }
__device__ __forceinline__ void tc_fence_after() { asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory"); }

__device__ __forceinline__ void tc_ld8(uint32_t taddr, uint32_t (&r)[8]) {
  asm volatile("tcgen05.ld.sync.aligned.32x32b.x8.b32 {%0,%1,%2,%3,%4,%5,%6,%7}, [%8];"
               : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7])
               : "r"(taddr));
}
__device__ __forceinline__ void tc_wait_ld() { asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory"); }

struct TcArgs {
  const PlanHdr* ph;
  const Q8Dev* xsrc;   // gate/up: Q8 inputs [k][K/256]; down: Q8 hidden [total_rows][K/256]
  float* out;          // gate/up: gu [total_rows][2 I]; down: parts [total_rows][D]
  int K, R;            // input values per row (D or I), output rows per matrix (I or D)
  int mats;            // matrices per slot in this pass (2: gate, up; 1: down)
  DevStatus* st;
};

constexpr int TC_MAX_BPR = 16;    // 256-value blocks per input row (K <= 4096)

struct TcShared {
  uint64_t wbar, mbar;
  uint32_t tmem;
  int n_units;
  int unit_end[TC_MAX_SLOTS];   // inclusive prefix of units per slot
  int src[TC_N];                // the chunk's active rows' Q8 source rows
  int x4[TC_N];
  float xscale[TC_N][TC_MAX_BPR];
  float xbsf[TC_N][TC_MAX_BPR][8];
};

// A step is 8 MMAs (256 tensor-memory columns): Q4_K one 256-value block
// (its 8 sub-blocks), Q6_K half a block (its 8 16-value groups of half h).
// Steps alternate between the two 256-column buffers, so the MMAs of step
// s + 1 run while the epilogue reads step s.
template <int WF>
struct TcFmt;
template <>
struct TcFmt<FMT_Q4K> {
  static constexpr int SPB = 1;            // steps per block
  static constexpr bool A_SIGNED = false;  // nibbles 0..15
};
template <>
struct TcFmt<FMT_Q6K> {
  static constexpr int SPB = 2;
  static constexpr bool A_SIGNED = true;   // q - 32
};

template <int WF, int MODE>   // MODE 0: gate/up; 1: down
__global__ void __launch_bounds__(TC_WARPS * 32, 1) tc_gemm_kernel(TcArgs a) {
  using F = TcFmt<WF>;
  extern __shared__ __align__(1024) uint8_t dsm[];
  __shared__ TcShared sh;
  const int tid = threadIdx.x, lane = tid & 31, wid = tid >> 5;
  const PlanHdr* ph = a.ph;
  const int bpr = a.K / QK;
  const RowLayout lay = row_layout(WF, a.K);
  const int tiles = (a.R + TC_M - 1) / TC_M;
  // shared memory: A tiles [8][4 KB], B tiles [8][TC_N x 32 B], raw weight window
  uint8_t* At = dsm;
  uint8_t* Bt = At + 8 * 4096;
  uint8_t* raw = Bt + 8 * TC_N * 32;

  if (wid == 0) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(&sh.tmem)),
                 "r"(512));
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;");
  }
  if (tid == 0) {
    mbar_init(&sh.wbar, 1);
    mbar_init(&sh.mbar, 1);
    fence_mbar_init();
  }
  pdl_wait();   // the plan and the inputs come from the preceding kernels
  const int n_slots = ph->n_slots;
  // units per slot: mats x tiles x chunks of TC_N active rows
  if (wid == 0) {
    int run = 0;
    for (int s0 = 0; s0 < n_slots; s0 += 32) {
      const int s = s0 + lane;
      const int u = s < n_slots ? a.mats * tiles * ((ph->slots[s].n_rows + TC_N - 1) / TC_N) : 0;
      int inc = u;
#pragma unroll
      for (int o = 1; o < 32; o <<= 1) {
        const int v = __shfl_up_sync(FULL, inc, o);
        if (lane >= o) inc += v;
      }
      if (s < n_slots) sh.unit_end[s] = run + inc;
      run += __shfl_sync(FULL, inc, 31);
    }
    if (lane == 0) sh.n_units = run;
  }
  // Q6_K's A tile m holds its group's 16 values in K-half m % 2 and zeros in
  // the other half, which never change
  if (WF == FMT_Q6K)
    for (int i = tid; i < 8 * 4096 / 16; i += TC_WARPS * 32) reinterpret_cast<uint4*>(At)[i] = make_uint4(0, 0, 0, 0);
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = sh.tmem;
  const int n_units = sh.n_units;
  const int nsteps = bpr * F::SPB;
  uint32_t wphase = 0, mphase = 0;
  bool ok = true;
  // epilogue coordinates: TMEM lane quarter q (rows 32 q ..), active rows 8 tg ..
  const int q = wid & 3, tg = wid >> 2, r = 32 * q + lane;

  for (int u = blockIdx.x; u < n_units && ok; u += gridDim.x) {
    int s = 0;
    while (sh.unit_end[s] <= u) s++;
    const int ub = s ? sh.unit_end[s - 1] : 0, rel = u - ub;
    const SlotDesc& S = ph->slots[s];
    const int nch = (S.n_rows + TC_N - 1) / TC_N;
    const int mat = rel / (tiles * nch), tile = (rel / nch) % tiles, ch = rel % nch;
    const WDesc W = MODE == 0 ? (mat ? S.up : S.gate) : S.down;
    const int r0 = tile * TC_M, nr = min(TC_M, a.R - r0);
    const int j0 = ch * TC_N, nt = min(TC_N, S.n_rows - j0), off = S.row_off;
    // the tile's weight window: rows r0 .. r0 + nr - 1, one bulk copy
    if (tid == 0) {
      const uint8_t* src = W.main + (size_t)r0 * lay.rs;
      mbar_arrive_expect_tx(&sh.wbar, (uint32_t)nr * lay.rs);
      bulk_g2s(raw, src, (uint32_t)nr * lay.rs, &sh.wbar);
    }
    // the chunk's active rows: Q8 source rows, association, and every
    // block's scale and 32-value sums (one round trip for the unit)
    if (tid < TC_N) {
      const int j = j0 + tid;
      sh.src[tid] = tid < nt ? (MODE == 0 ? ph->rows[off + j] : off + j) : -1;
      sh.x4[tid] = tid < nt && use_x4(ph->assoc_rule, j & ~3, S.n_rows, ph->k);
    }
    __syncthreads();
    for (int i = tid; i < TC_N * bpr; i += TC_WARPS * 32) {
      const int jj = i / bpr, b = i - jj * bpr, src = sh.src[jj];
      float sc = 0.f;
      float bs[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
      if (src >= 0) {
        const Q8Dev& xb = a.xsrc[(size_t)src * bpr + b];
        sc = __ldcg(&xb.scale);
        // bsums sit at byte 264 of the 320-byte block: 8-byte aligned
#pragma unroll
        for (int c = 0; c < 4; c++) {
          const int2 v = __ldcg(reinterpret_cast<const int2*>(xb.bsums) + c);
          bs[2 * c] = (float)v.x;
          bs[2 * c + 1] = (float)v.y;
        }
      }
      sh.xscale[jj][b] = sc;
#pragma unroll
      for (int c = 0; c < 8; c++) sh.xbsf[jj][b][c] = bs[c];
    }
    // B prefetch: thread (active row jj, 16-byte piece p) of a block's 256 values
    const int bj = tid >> 4, bp = tid & 15;
    auto load_b = [&](int b) -> uint4 {
      const int src = sh.src[bj];
      return src >= 0 ? __ldcg(reinterpret_cast<const uint4*>(a.xsrc[(size_t)src * bpr + b].qs) + bp)
                      : make_uint4(0, 0, 0, 0);
    };
    uint4 bnext = load_b(0);
    bool wok = mbar_wait(&sh.wbar, wphase);
    if (!wok && tid == 0) set_error(a.st, ERR_WAIT_TIMEOUT, 60, blockIdx.x, u);
    wphase ^= 1u;

    // stage step st: A tiles from the weight window, and at a block's first
    // step its B tiles (the prefetched values) and the next block's prefetch
    auto stage = [&](int st) {
      const int b = st / F::SPB, h = st - b * F::SPB;
      if constexpr (WF == FMT_Q4K) {
        // thread: row rr, 16-byte piece p of the 128 nibble bytes -> 32 values
        for (int i = tid; i < TC_M * 8; i += TC_WARPS * 32) {
          const int rr = i >> 3, p = i & 7;
          uint4 w = make_uint4(0, 0, 0, 0);
          if (rr < nr) w = *reinterpret_cast<const uint4*>(raw + (size_t)rr * lay.rs + b * Q4K_BYTES + 16 + 16 * p);
          // bytes 32g .. 32g + 31: low nibbles -> sub-block 2g, high -> 2g + 1
          const int g = p >> 1, kb = 16 * (p & 1);
          const uint4 lo = make_uint4(w.x & 0x0F0F0F0Fu, w.y & 0x0F0F0F0Fu, w.z & 0x0F0F0F0Fu, w.w & 0x0F0F0F0Fu);
          const uint4 hi = make_uint4((w.x >> 4) & 0x0F0F0F0Fu, (w.y >> 4) & 0x0F0F0F0Fu, (w.z >> 4) & 0x0F0F0F0Fu,
                                      (w.w >> 4) & 0x0F0F0F0Fu);
          *reinterpret_cast<uint4*>(At + (2 * g) * 4096 + kmaj(rr, kb)) = lo;
          *reinterpret_cast<uint4*>(At + (2 * g + 1) * 4096 + kmaj(rr, kb)) = hi;
        }
      } else {
        // thread: row rr, group (lq, k4) of half h: tile m = 2 k4 + lq, values in K-half lq
        for (int i = tid; i < TC_M * 8; i += TC_WARPS * 32) {
          const int rr = i >> 3, m = i & 7, k4 = m >> 1, lq = m & 1;
          uint4 v = make_uint4(0, 0, 0, 0);
          if (rr < nr) {
            const uint8_t* mb = raw + (size_t)rr * lay.rs + b * 192;
            const uint4 va = *reinterpret_cast<const uint4*>(mb + 64 * h + 16 * lq + 32 * (k4 & 1));
            const uint4 vh = *reinterpret_cast<const uint4*>(mb + 128 + 32 * h + 16 * lq);
            const uint32_t qa[4] = {va.x, va.y, va.z, va.w}, qh[4] = {vh.x, vh.y, vh.z, vh.w};
            uint32_t o[4];
#pragma unroll
            for (int c = 0; c < 4; c++) {
              uint32_t t;
              if (k4 == 0) t = (qa[c] & 0x0F0F0F0Fu) | ((qh[c] & 0x03030303u) << 4);
              else if (k4 == 1) t = (qa[c] & 0x0F0F0F0Fu) | ((qh[c] & 0x0C0C0C0Cu) << 2);
              else if (k4 == 2) t = ((qa[c] >> 4) & 0x0F0F0F0Fu) | (qh[c] & 0x30303030u);
              else t = ((qa[c] >> 4) & 0x0F0F0F0Fu) | ((qh[c] >> 2) & 0x30303030u);
              o[c] = __vsub4(t, 0x20202020u);   // q - 32 as int8 (bytes 0..63 -> -32..31)
            }
            v = make_uint4(o[0], o[1], o[2], o[3]);
          }
          *reinterpret_cast<uint4*>(At + m * 4096 + kmaj(rr, 16 * lq)) = v;
        }
      }
      if (h == 0) {
        // 16 bytes bp = values 16 bp ..: sub-block bp / 2, K-half bp % 2
        if (bj < TC_N) *reinterpret_cast<uint4*>(Bt + (bp >> 1) * (TC_N * 32) + kmaj(bj, 16 * (bp & 1))) = bnext;
        if (b + 1 < bpr) bnext = load_b(b + 1);
      }
    };
    auto issue = [&](int st) {   // one thread
      const int h = st % F::SPB;
      constexpr uint32_t idesc = umma_idesc(F::A_SIGNED);
      const uint32_t tb = tmem + (uint32_t)(st & 1) * 256;
#pragma unroll
      for (int m = 0; m < 8; m++) {
        // Q4_K: sub-block m; Q6_K: group (h, lq = m % 2, k4 = m / 2) of chunk 4 h + m / 2
        const int bt = WF == FMT_Q4K ? m : 4 * h + (m >> 1);
        const uint64_t da = umma_desc(smem_u32(At + m * 4096)), db = umma_desc(smem_u32(Bt + bt * (TC_N * 32)));
        asm volatile("{\n\t.reg .pred p;\n\tsetp.ne.b32 p, %4, 0;\n\t"
                     "tcgen05.mma.cta_group::1.kind::i8 [%0], %1, %2, %3, p;\n\t}" ::"r"(tb + m * TC_N),
                     "l"(da), "l"(db), "r"(idesc), "r"(0));
      }
      asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(
          smem_u32(&sh.mbar)));
    };

    float acc[8], fold[8];
#pragma unroll
    for (int c = 0; c < 8; c++) acc[c] = fold[c] = 0.f;
    if (wok) stage(0);
    fence_proxy_async();
    tc_fence_before();
    ok = __syncthreads_and(wok) != 0;   // uniform: every thread leaves together
    tc_fence_after();
    if (ok && tid == 0) issue(0);
    for (int st = 0; st < nsteps && ok; st++) {
      const bool mok = mbar_wait(&sh.mbar, mphase);
      if (!mok && tid == 0) set_error(a.st, ERR_WAIT_TIMEOUT, 61, blockIdx.x, u);
      mphase ^= 1u;
      tc_fence_after();
      // MMAs of step st are done: A / B are free for step st + 1
      if (mok && st + 1 < nsteps) stage(st + 1);
      fence_proxy_async();
      tc_fence_before();
      ok = __syncthreads_and(mok) != 0;
      tc_fence_after();
      if (!ok) break;
      if (tid == 0 && st + 1 < nsteps) issue(st + 1);
      // epilogue of step st (row r, active rows 8 tg .. 8 tg + 7; warps past
      // the chunk's rows idle)
      const int b = st / F::SPB, h = st - b * F::SPB;
      const uint32_t tl = tmem + (uint32_t)(st & 1) * 256 + ((uint32_t)(32 * q) << 16) + 8 * tg;
      if (8 * tg >= nt) {
      } else if constexpr (WF == FMT_Q4K) {
        const uint4 hd = *reinterpret_cast<const uint4*>(raw + (size_t)min(r, nr - 1) * lay.rs + b * Q4K_BYTES);
        const float d = f16_fast(hd.x & 0xFFFFu), dmin = f16_fast(hd.x >> 16);
        float bsum[8];
#pragma unroll
        for (int c = 0; c < 8; c++) bsum[c] = 0.f;
#pragma unroll
        for (int g = 0; g < 4; g++) {
          uint32_t il[8], ih[8];
          tc_ld8(tl + (2 * g) * TC_N, il);
          tc_ld8(tl + (2 * g + 1) * TC_N, ih);
          tc_wait_ld();
          int sl, ml, shh, mh;
          q4k_pair_scales(g, hd.y, hd.z, hd.w, sl, ml, shh, mh);
          const float dsl = fmul(d, (float)sl), dml = fmul(dmin, (float)ml);
          const float dsh = fmul(d, (float)shh), dmh = fmul(dmin, (float)mh);
#pragma unroll
          for (int c = 0; c < 8; c++) {
            const int jj = 8 * tg + c;
            const float flo = i2f_small((int)il[c]), fhi = i2f_small((int)ih[c]);
            const float blo = sh.xbsf[jj][b][2 * g], bhi = sh.xbsf[jj][b][2 * g + 1];
            if (sh.x4[jj]) {
              bsum[c] = fadd(bsum[c], fsub(fadd(fsub(fmul(dsl, flo), fmul(dml, blo)), fmul(dsh, fhi)), fmul(dmh, bhi)));
            } else {
              bsum[c] = fadd(bsum[c], fsub(fmul(dsl, flo), fmul(dml, blo)));
              bsum[c] = fadd(bsum[c], fsub(fmul(dsh, fhi), fmul(dmh, bhi)));
            }
          }
        }
#pragma unroll
        for (int c = 0; c < 8; c++) acc[c] = fadd(acc[c], fmul(sh.xscale[8 * tg + c][b], bsum[c]));
      } else {
        // the reference's fp32 fold of the block's 16 products sc * isum16,
        // in its order (half h, l-half lq, quarter k4); each product is an
        // exact integer in fp32
        const uint8_t* rowp = raw + (size_t)min(r, nr - 1) * lay.rs;
        const uint4 sv = *reinterpret_cast<const uint4*>(rowp + lay.a1 + b * 16);
        const uint32_t sw[4] = {sv.x, sv.y, sv.z, sv.w};
#pragma unroll
        for (int lq = 0; lq < 2; lq++)
#pragma unroll
          for (int k4 = 0; k4 < 4; k4++) {
            uint32_t is[8];
            tc_ld8(tl + (2 * k4 + lq) * TC_N, is);
            tc_wait_ld();
            const int si = 8 * h + lq + 2 * k4;
            const int sc = sbyte(sw[si >> 2], si & 3);
#pragma unroll
            for (int c = 0; c < 8; c++) fold[c] = fadd(fold[c], (float)(sc * (int)is[c]));
          }
        if (h == 1) {
          const float d = f16_fast((uint32_t)rowp[lay.a2 + 2 * b] | ((uint32_t)rowp[lay.a2 + 2 * b + 1] << 8));
#pragma unroll
          for (int c = 0; c < 8; c++) {
            acc[c] = fadd(acc[c], fmul(fmul(d, sh.xscale[8 * tg + c][b]), fold[c]));
            fold[c] = 0.f;
          }
        }
      }
      tc_fence_before();
    }
    // outputs of this unit
    if (ok && r < nr) {
#pragma unroll
      for (int c = 0; c < 8; c++) {
        const int jj = 8 * tg + c;
        if (jj >= nt) continue;
        const int row = off + j0 + jj;
        if (MODE == 0) {
          a.out[(size_t)row * (2 * a.R) + (size_t)mat * a.R + r0 + r] = acc[c];
        } else {
          const float w = ph->wts[row];
          const float v = acc[c];
          a.out[(size_t)row * a.R + r0 + r] =
              ph->bias_term ? fmul(w, fadd(v, S.db ? S.db[r0 + r] : 0.f)) : fmul(w, v);
        }
      }
    }
    tc_fence_before();
    __syncthreads();   // the weight window and tensor memory are reused by the next unit
    tc_fence_after();
  }
  pdl_trigger();
  tc_fence_before();
  __syncthreads();
  if (wid == 0) asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(512));
}

// hq8[row] = Q8 of act(gate + gb, up + ub) over the slot's bias vectors: one
// warp per (active row, 256-block).
__global__ void act_quant_kernel(const PlanHdr* __restrict__ ph, const float* __restrict__ gu, int I,
                                 Q8Dev* __restrict__ hq8) {
  pdl_wait();
  pdl_trigger();
  const int lane = threadIdx.x & 31;
  const int dbpr = (I + QK - 1) / QK;
  const long wq = ((long)blockIdx.x * blockDim.x + threadIdx.x) >> 5;
  if (wq >= (long)ph->total_rows * dbpr) return;
  const int row = (int)(wq / dbpr), b = (int)(wq - (long)row * dbpr);
  const SlotDesc& S = ph->slots[ph->row_slot[row]];
  const int n = min(QK, I - b * QK);
  float v[8];
#pragma unroll
  for (int j = 0; j < 8; j++) {
    const int i = b * QK + 8 * lane + j;
    v[j] = 0.f;
    if (8 * lane + j < n) {
      float g = gu[(size_t)row * 2 * I + i], u = gu[(size_t)row * 2 * I + I + i];
      if (S.gb) {
        g = fadd(g, S.gb[i]);
        u = fadd(u, S.ub[i]);
      }
      v[j] = act_fn(ph->act, g, u);
    }
  }
  quantize_block_warp_vals(v, n, hq8 + (size_t)row * dbpr + b);
}

// out[t][r] += the parts of token t's active rows, in slot order.
__global__ void combine_rows_kernel(const PlanHdr* __restrict__ ph, const int* __restrict__ tok_rows, int K,
                                    const float* __restrict__ parts, float* __restrict__ out) {
  pdl_wait();
  pdl_trigger();
  const int D = ph->embed_dim;
  const size_t i = (size_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= (size_t)ph->k * D) return;
  const int t = (int)(i / D), r = (int)(i - (size_t)t * D);
  float v = out[i];
  for (int c = 0; c < K; c++) {
    const int sr = tok_rows[(size_t)t * K + c];
    if (sr < 0) break;
    v = fadd(v, parts[(size_t)sr * D + r]);
  }
  out[i] = v;
}

// ---------------------------------------------------------------------
// Host side.

static int tc_sms() {
  static int sms = 0;
  if (!sms) {
    int dev = 0;
    cudaGetDevice(&dev);
    cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
    if (sms < 1) sms = 1;
  }
  return sms;
}

static cudaError_t pdl_launch(const void* fn, dim3 grid, dim3 block, size_t smem, cudaStream_t s, void** args) {
  cudaLaunchConfig_t cfg{};
  cfg.gridDim = grid;
  cfg.blockDim = block;
  cfg.dynamicSmemBytes = smem;
  cfg.stream = s;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  return cudaLaunchKernelExC(&cfg, fn, args);
}

static size_t tc_smem(int wf, int K) {
  return (size_t)8 * 4096 + 8 * TC_N * 32 + (size_t)TC_M * row_layout(wf, K).rs + 64;
}

bool tc_moe_eligible(int gate_fmt, int down_fmt, int D, int I) {
  if (gate_fmt != FMT_Q4K || (down_fmt != FMT_Q4K && down_fmt != FMT_Q6K)) return false;
  if (D % QK || I % QK || D / QK > TC_MAX_BPR || I / QK > TC_MAX_BPR) return false;
  return tc_smem(gate_fmt, D) <= 220 * 1024 && tc_smem(down_fmt, I) <= 220 * 1024;
}

size_t tc_moe_scratch_bytes(int max_rows, int T, int K, int D, int I) {
  (void)T;
  (void)K;
  const int dbpr = I / QK;
  return (size_t)max_rows * 2 * I * 4 + (size_t)max_rows * dbpr * sizeof(Q8Dev) + (size_t)max_rows * D * 4 + 3 * 256;
}

template <int WF, int MODE>
static cudaError_t tc_launch(const TcArgs& a, cudaStream_t s) {
  const void* fn = reinterpret_cast<const void*>(tc_gemm_kernel<WF, MODE>);
  const size_t smem = tc_smem(WF, a.K);
  cudaError_t e = ensure_smem(fn, smem);
  if (e != cudaSuccess) return e;
  TcArgs args = a;
  void* p[] = {(void*)&args};
  return pdl_launch(fn, dim3(tc_sms()), dim3(TC_WARPS * 32), smem, s, p);
}

cudaError_t launch_tc_moe(const PlanHdr* ph, int gate_fmt, int down_fmt, int T, int K, int D, int I, int max_rows,
                          const Q8Dev* xq8, const int* tok_rows, void* scratch, float* out, DevStatus* st,
                          cudaStream_t s) {
  uint8_t* p = static_cast<uint8_t*>(scratch);
  auto take = [&](size_t n) {
    uint8_t* q = p;
    p += (n + 255) & ~(size_t)255;
    return q;
  };
  float* gu = reinterpret_cast<float*>(take((size_t)max_rows * 2 * I * 4));
  Q8Dev* hq8 = reinterpret_cast<Q8Dev*>(take((size_t)max_rows * (I / QK) * sizeof(Q8Dev)));
  float* parts = reinterpret_cast<float*>(take((size_t)max_rows * D * 4));
  TcArgs g{ph, xq8, gu, D, I, 2, st};
  cudaError_t e = tc_launch<FMT_Q4K, 0>(g, s);
  if (e != cudaSuccess) return e;
  {
    const long warps = (long)max_rows * (I / QK);
    const PlanHdr* php = ph;
    const float* gup = gu;
    int Iv = I;
    Q8Dev* hp = hq8;
    void* a2[] = {(void*)&php, (void*)&gup, (void*)&Iv, (void*)&hp};
    e = pdl_launch(reinterpret_cast<const void*>(act_quant_kernel), dim3((unsigned)((warps * 32 + 255) / 256)),
                   dim3(256), 0, s, a2);
    if (e != cudaSuccess) return e;
  }
  TcArgs dn{ph, hq8, parts, I, D, 1, st};
  e = down_fmt == FMT_Q6K ? tc_launch<FMT_Q6K, 1>(dn, s) : tc_launch<FMT_Q4K, 1>(dn, s);
  if (e != cudaSuccess) return e;
  {
    const PlanHdr* php = ph;
    int Kv = K;
    const int* trc = tok_rows;
    const float* pp = parts;
    float* op = out;
    void* a4[] = {(void*)&php, (void*)&trc, (void*)&Kv, (void*)&pp, (void*)&op};
    e = pdl_launch(reinterpret_cast<const void*>(combine_rows_kernel), dim3((unsigned)(((size_t)T * D + 255) / 256)),
                   dim3(256), 0, s, a4);
  }
  return e;
}

}  // namespace tg
