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
#include <cuda.h>   // CUtensorMap and its encoder's signature (resolved through the runtime)

#include <algorithm>
#include <type_traits>
#include <vector>

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

// One 2-D tile (box) of a tensor map into shared memory, completing on bar
// (no multicast).  x, the innermost coordinate, is a byte offset and must be
// a multiple of 16; the parts of the box outside the tensor read as zeros.
__device__ __forceinline__ void tma_load_2d(void* dst, const CUtensorMap* map, int x, int y, uint64_t* bar) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.tile.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3}], [%4];" ::
          "r"(smem_u32(dst)),
      "l"(map), "r"(x), "r"(y), "r"(smem_u32(bar))
      : "memory");
}

struct TcArgs {
  const PlanHdr* ph;
  const Q8Dev* xsrc;   // gate/up: Q8 inputs [k][K/256]; down: Q8 hidden [total_rows][K/256]
  float* out;          // gate/up: gu [total_rows][2 I]; down: parts [total_rows][D]
  int K, R;            // input values per row (D or I), output rows per matrix (I or D)
  int mats;            // matrices per slot in this pass (2: gate, up; 1: down)
  DevStatus* st;
  const CUtensorMap* tmaps;   // MXFP4: [E][3] (gate, up, down) tensor maps
  float negz;                 // -0.0f (the packed epilogue's product addend)
  int* dbg;                   // test hook: every int32 sub-block sum, or null (tc_debug_isum_index)
};

// Test hook layout: the int32 sum of sub-block sb (the oracle's order: Q4_K
// and MXFP4 32-value sub-blocks in value order, Q6_K the 16-value groups
// (h, l-half, quarter) as (2 h + l-half) 4 + quarter) of weight row wr of
// matrix mat (gate/up pass: 0 gate, 1 up) against plan row prow.
__host__ __device__ __forceinline__ size_t tc_debug_isum_index(int prow, int mats, int mat, int R, int wr, int nsb,
                                                              int sb) {
  return (((size_t)prow * mats + mat) * R + wr) * nsb + sb;
}

constexpr int TC_MAX_BPR = 16;    // 256-value blocks per input row (K <= 4096)
constexpr int TC_NS = 4;          // MXFP4 code ring: stages of 128 rows x 128 bytes
constexpr int TC_STAGE = TC_M * 128;
// The thread that issues the MMAs and the TMA copies: lane 0 of the last
// warp, whose epilogue share is the last to be used as chunks shrink.
constexpr int TC_ISSUER = (TC_WARPS - 1) * 32;

struct TcShared {
  uint64_t wbar, mbar;
  uint64_t cbar[TC_NS];
  uint32_t tmem;
  int n_units;
  int unit_end[TC_MAX_SLOTS];   // inclusive prefix of units per slot
  int src[TC_N];                // the chunk's active rows' Q8 source rows
  int x4[TC_N];
  float xscale[TC_N][TC_MAX_BPR];
  float xbsf[TC_N][TC_MAX_BPR][8];
  // per weight row, double-buffered by block parity: Q4_K the block's
  // 16-byte header, Q6_K its 16 scales and d (copied by the stage step, so
  // the epilogue's lanes read consecutive rows without bank conflicts)
  uint4 hdr[2][TC_M];
  float dq[2][TC_M];
};

// A step is 8 MMAs (256 tensor-memory columns): Q4_K one 256-value block
// (its 8 sub-blocks), Q6_K half a block (its 8 16-value groups of half h),
// MXFP4 the 8 32-value sub-blocks that pair with one Q8 block.  Steps
// alternate between the two 256-column buffers, so the MMAs of step s + 1
// run while the epilogue reads step s.  Q4_K and Q6_K stage A from a
// shared-memory window of the unit's weight rows (one bulk copy); MXFP4 rows
// (1536 bytes at K = 2880) would not fit, so their code bytes stream through
// a ring of TC_NS step stages, each one 2-D TMA box (128 rows x 128 bytes)
// issued TC_NS steps ahead, the last 128 bytes of every row (the e8m0
// scales) sit in a per-unit box, and the next unit's rows are prefetched
// into L2.
template <int WF>
struct TcFmt;
template <>
struct TcFmt<FMT_Q4K> {
  static constexpr int SPB = 1;            // steps per block
  static constexpr bool A_SIGNED = false;  // nibbles 0..15
  static constexpr bool RAW = true;        // weight window in shared memory
};
template <>
struct TcFmt<FMT_Q6K> {
  static constexpr int SPB = 2;
  static constexpr bool A_SIGNED = true;   // q - 32
  static constexpr bool RAW = true;
};
template <>
struct TcFmt<FMT_MXFP4> {
  static constexpr int SPB = 1;
  static constexpr bool A_SIGNED = true;   // doubled e2m1 values -12..12
  static constexpr bool RAW = false;
};

// Four MXFP4 codes (the selector nibbles of sel; seln = sel with its sign
// bits flipped) -> their doubled e2m1 values as int8 (csrc/libtinygiant.c:
// 514).  prmt looks the magnitude {0,1,2,3,4,6,8,12}[code & 7] up for a code
// whose sign bit is clear and emits 0 (the entry's sign) for one whose sign
// bit is set, so p holds the positive codes' values and n the negative
// codes' magnitudes, each byte nonzero in at most one; 0x80 - n per byte,
// xor 0x80, is -n as int8.
__device__ __forceinline__ uint32_t mx_unpack4(uint32_t sel, uint32_t seln) {
  constexpr uint32_t T0 = 0x03020100u, T1 = 0x0C080604u;
  const uint32_t p = prmt(T0, T1, sel), n = prmt(T0, T1, seln);
  return p | ((0x80808080u - n) ^ 0x80808080u);
}

// tcgen05.ld of N consecutive 32-bit columns (32x32b shape).
template <int N>
__device__ __forceinline__ void tc_ld(uint32_t taddr, uint32_t (&r)[N]);
template <>
__device__ __forceinline__ void tc_ld<1>(uint32_t taddr, uint32_t (&r)[1]) {
  asm volatile("tcgen05.ld.sync.aligned.32x32b.x1.b32 {%0}, [%1];" : "=r"(r[0]) : "r"(taddr));
}
template <>
__device__ __forceinline__ void tc_ld<2>(uint32_t taddr, uint32_t (&r)[2]) {
  asm volatile("tcgen05.ld.sync.aligned.32x32b.x2.b32 {%0,%1}, [%2];" : "=r"(r[0]), "=r"(r[1]) : "r"(taddr));
}
template <>
__device__ __forceinline__ void tc_ld<4>(uint32_t taddr, uint32_t (&r)[4]) {
  asm volatile("tcgen05.ld.sync.aligned.32x32b.x4.b32 {%0,%1,%2,%3}, [%4];"
               : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3])
               : "r"(taddr));
}
template <>
__device__ __forceinline__ void tc_ld<8>(uint32_t taddr, uint32_t (&r)[8]) {
  tc_ld8(taddr, r);
}

template <int V>
using IC = std::integral_constant<int, V>;

// Packed pairs of fp32 operations (sm_100 f32x2): each half rounds as the
// scalar operation does, so pairs of independent accumulators keep their
// exact values.  a - b is a + (-b).  A packed multiply feeding a packed add
// is fused into one fma by the assembler even with .rn, so products are
// formed as fma(a, b, z) with z = -0 from a kernel argument (not a constant
// the assembler could fold): exactly the rounded product, and an fma is not
// fused again.
__device__ __forceinline__ float2 fadd2(float2 a, float2 b) {
  float2 d;
  asm("{\n\t.reg .b64 ra, rb, rd;\n\tmov.b64 ra, {%2, %3};\n\tmov.b64 rb, {%4, %5};\n\t"
      "add.rn.f32x2 rd, ra, rb;\n\tmov.b64 {%0, %1}, rd;\n\t}"
      : "=f"(d.x), "=f"(d.y)
      : "f"(a.x), "f"(a.y), "f"(b.x), "f"(b.y));
  return d;
}
__device__ __forceinline__ float2 fmul2z(float2 a, float2 b, float2 z) {
  float2 d;
  asm("{\n\t.reg .b64 ra, rb, rc, rd;\n\tmov.b64 ra, {%2, %3};\n\tmov.b64 rb, {%4, %5};\n\t"
      "mov.b64 rc, {%6, %7};\n\tfma.rn.f32x2 rd, ra, rb, rc;\n\tmov.b64 {%0, %1}, rd;\n\t}"
      : "=f"(d.x), "=f"(d.y)
      : "f"(a.x), "f"(a.y), "f"(b.x), "f"(b.y), "f"(z.x), "f"(z.y));
  return d;
}
__device__ __forceinline__ float2 splat2(float v) { return make_float2(v, v); }
// i2f_small of two integers (|v| < 2^22): exact.
__device__ __forceinline__ float2 i2f_small2(int a, int b) {
  return fadd2(make_float2(__int_as_float(0x4B400000 + a), __int_as_float(0x4B400000 + b)), splat2(-12582912.0f));
}

template <int WF, int MODE>   // MODE 0: gate/up; 1: down
__global__ void __launch_bounds__(TC_WARPS * 32, 1) tc_gemm_kernel(TcArgs a) {
  using F = TcFmt<WF>;
  extern __shared__ __align__(1024) uint8_t dsm[];
  __shared__ TcShared sh;
  const int tid = threadIdx.x, lane = tid & 31, wid = tid >> 5;
  const PlanHdr* ph = a.ph;
  const int bpr = (a.K + QK - 1) / QK, nsub = a.K / 32;
  const RowLayout lay = row_layout(WF, a.K);
  const int tiles = (a.R + TC_M - 1) / TC_M;
  // shared memory (from a 1024-byte boundary: the MXFP4 ring's 128-byte
  // swizzle): A tiles [8][4 KB], B tiles [8][TC_N x 32 B], raw weight window
  uint8_t* At = dsm + ((1024u - (smem_u32(dsm) & 1023u)) & 1023u);
  uint8_t* Bt = At + 8 * 4096;
  uint8_t* raw = Bt + 8 * TC_N * 32;
  uint8_t* ring = raw;                            // MXFP4: TC_NS x TC_STAGE code bytes
  uint8_t* tail = ring + TC_NS * TC_STAGE;        // MXFP4: rows' last 128 bytes [128][128]
  const int tx = lay.rs - 128;                    // MXFP4: the tail box's x (rs >= 144)
  // byte (row, o) of a 128-byte-row box written with the 128-byte swizzle
  auto swz = [](int row, int o) { return row * 128 + ((((o >> 4) ^ row) & 7) << 4) + (o & 15); };

  if (wid == 0) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(&sh.tmem)),
                 "r"(512));
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;");
  }
  if (tid == 0) {
    mbar_init(&sh.wbar, 1);
    mbar_init(&sh.mbar, 1);
    for (int k = 0; k < TC_NS; k++) mbar_init(&sh.cbar[k], 1);
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
  uint32_t wphase = 0, mphase = 0, cph = 0;
  bool ok = true;
  // epilogue coordinates: TMEM lane quarter q (weight rows 32 q ..); the
  // four warps of a quarter split the chunk's active rows
  const int q = wid & 3, tg = wid >> 2, r = 32 * q + lane;
  const float2 nz2 = splat2(a.negz);

  // unit u -> (slot, matrix, 128-row tile, chunk of TC_N active rows)
  auto coords = [&](int u, int& s, int& mat, int& tile, int& ch) {
    int lo = 0, hi = n_slots - 1;   // the first slot whose units end past u
    while (lo < hi) {
      const int mid = (lo + hi) >> 1;
      if (sh.unit_end[mid] > u) hi = mid;
      else lo = mid + 1;
    }
    s = lo;
    const int rel = u - (s ? sh.unit_end[s - 1] : 0);
    const int nch = (ph->slots[s].n_rows + TC_N - 1) / TC_N;
    mat = rel / (tiles * nch);
    tile = (rel / nch) % tiles;
    ch = rel % nch;
  };

  for (int u = blockIdx.x; u < n_units && ok; u += gridDim.x) {
    int s, mat, tile, ch;
    coords(u, s, mat, tile, ch);
    const SlotDesc& S = ph->slots[s];
    const WDesc W = MODE == 0 ? (mat ? S.up : S.gate) : S.down;
    const int r0 = tile * TC_M, nr = min(TC_M, a.R - r0);
    const int j0 = ch * TC_N, nt = min(TC_N, S.n_rows - j0), off = S.row_off;
    // active rows per epilogue warp: the chunk's nt rows over a quarter's 4 warps
    const int ew = nt <= 4 ? 1 : nt <= 8 ? 2 : nt <= 16 ? 4 : 8, c0 = tg * ew;
    if constexpr (F::RAW) {
      // the tile's weight window: rows r0 .. r0 + nr - 1, one bulk copy
      if (tid == TC_ISSUER) {
        const uint8_t* src = W.main + (size_t)r0 * lay.rs;
        mbar_arrive_expect_tx(&sh.wbar, (uint32_t)nr * lay.rs);
        bulk_g2s(raw, src, (uint32_t)nr * lay.rs, &sh.wbar);
      }
    } else {
      // the next unit's weight rows into L2 while this one runs
      const int un = u + gridDim.x;
      if (un < n_units) {
        int s2, m2, t2, c2;
        coords(un, s2, m2, t2, c2);
        const SlotDesc& S2 = ph->slots[s2];
        const WDesc W2 = MODE == 0 ? (m2 ? S2.up : S2.gate) : S2.down;
        const int r2 = t2 * TC_M;
        if (tid < min(TC_M, a.R - r2))
          asm volatile("cp.async.bulk.prefetch.L2.global [%0], %1;" ::"l"(W2.main + (size_t)(r2 + tid) * lay.rs),
                       "r"((uint32_t)lay.rs)
                       : "memory");
      }
    }
    // MXFP4 step st's code bytes (and at step 0 the rows' tails) into ring
    // stage st % TC_NS: one thread, one TMA box each; a box counts in full
    // (rows past the matrix read as zeros)
    const CUtensorMap* tmap = F::RAW ? nullptr : a.tmaps + 3 * S.expert + (MODE == 0 ? mat : 2);
    auto issue_codes = [&](int st) {
      const int k = st % TC_NS;
      mbar_arrive_expect_tx(&sh.cbar[k], (uint32_t)(TC_STAGE * (st == 0 ? 2 : 1)));
      tma_load_2d(ring + k * TC_STAGE, tmap, 128 * st, r0, &sh.cbar[k]);
      if (st == 0) tma_load_2d(tail, tmap, tx, r0, &sh.cbar[k]);
    };
    if constexpr (!F::RAW) {
      if (tid == TC_ISSUER)
        for (int st = 0; st < min(TC_NS, nsteps); st++) issue_codes(st);
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
        if constexpr (WF == FMT_Q4K) {
          // bsums sit at byte 264 of the 320-byte block: 8-byte aligned
#pragma unroll
          for (int c = 0; c < 4; c++) {
            const int2 v = __ldcg(reinterpret_cast<const int2*>(xb.bsums) + c);
            bs[2 * c] = (float)v.x;
            bs[2 * c + 1] = (float)v.y;
          }
        }
      }
      sh.xscale[jj][b] = sc;
      if constexpr (WF == FMT_Q4K) {
#pragma unroll
        for (int c = 0; c < 8; c++) sh.xbsf[jj][b][c] = bs[c];
      }
    }
    // B prefetch: thread (active row jj, 16-byte piece p) of a block's 256 values
    const int bj = tid >> 4, bp = tid & 15;
    auto load_b = [&](int b) -> uint4 {
      const int src = sh.src[bj];
      return src >= 0 ? __ldcg(reinterpret_cast<const uint4*>(a.xsrc[(size_t)src * bpr + b].qs) + bp)
                      : make_uint4(0, 0, 0, 0);
    };
    uint4 bnext = load_b(0);
    bool wok = true;
    if constexpr (F::RAW) {
      wok = mbar_wait(&sh.wbar, wphase);
      if (!wok && tid == 0) set_error(a.st, ERR_WAIT_TIMEOUT, 60, blockIdx.x, u);
      wphase ^= 1u;
    }

    // stage step st: A tiles (from the weight window or the code ring), and
    // at a block's first step its B tiles (the prefetched values) and the
    // next block's prefetch.  False if the code ring's wait gave up.
    auto stage = [&](int st) -> bool {
      const int b = st / F::SPB, h = st - b * F::SPB;
      bool sok = true;
      // item i = 8 j + l (l: the lane's place in its quarter-warp phase) ->
      // row rr = 8 (j / 8) + l: a phase's 8 stores go to 8 distinct rows of a
      // core matrix, and its 8 window reads to 8 distinct 16-byte columns
      if constexpr (WF == FMT_Q4K) {
        // thread: row rr, 16-byte piece p of the 128 nibble bytes -> 32 values
        for (int i = tid; i < TC_M * 8; i += TC_WARPS * 32) {
          const int l = i & 7, j = i >> 3, rr = 8 * (j >> 3) + l, p = (l + j) & 7;
          uint4 w = make_uint4(0, 0, 0, 0);
          if (rr < nr) w = *reinterpret_cast<const uint4*>(raw + (size_t)rr * lay.rs + b * Q4K_BYTES + 16 + 16 * p);
          if (p == 0)
            sh.hdr[b & 1][rr] = rr < nr ? *reinterpret_cast<const uint4*>(raw + (size_t)rr * lay.rs + b * Q4K_BYTES)
                                        : make_uint4(0, 0, 0, 0);
          // bytes 32g .. 32g + 31: low nibbles -> sub-block 2g, high -> 2g + 1
          const int g = p >> 1, kb = 16 * (p & 1);
          const uint4 lo = make_uint4(w.x & 0x0F0F0F0Fu, w.y & 0x0F0F0F0Fu, w.z & 0x0F0F0F0Fu, w.w & 0x0F0F0F0Fu);
          const uint4 hi = make_uint4((w.x >> 4) & 0x0F0F0F0Fu, (w.y >> 4) & 0x0F0F0F0Fu, (w.z >> 4) & 0x0F0F0F0Fu,
                                      (w.w >> 4) & 0x0F0F0F0Fu);
          *reinterpret_cast<uint4*>(At + (2 * g) * 4096 + kmaj(rr, kb)) = lo;
          *reinterpret_cast<uint4*>(At + (2 * g + 1) * 4096 + kmaj(rr, kb)) = hi;
        }
      } else if constexpr (WF == FMT_Q6K) {
        // thread: row rr, group (lq, k4) of half h: tile m = 2 k4 + lq, values in K-half lq
        for (int i = tid; i < TC_M * 8; i += TC_WARPS * 32) {
          const int l = i & 7, j = i >> 3, rr = 8 * (j >> 3) + l, m = (l + j) & 7, k4 = m >> 1, lq = m & 1;
          if (h == 0 && m == 0) {
            const uint8_t* rowp = raw + (size_t)min(rr, nr - 1) * lay.rs;
            sh.hdr[b & 1][rr] = *reinterpret_cast<const uint4*>(rowp + lay.a1 + b * 16);
            sh.dq[b & 1][rr] = f16_fast((uint32_t)rowp[lay.a2 + 2 * b] | ((uint32_t)rowp[lay.a2 + 2 * b + 1] << 8));
          }
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
      } else {
        // thread item k: row rr, sub-block m; code word c (bytes 4c .. 4c + 3:
        // values 4c .. 4c + 3 low, 16 + 4c .. high) -> K positions 8c .. 8c + 7
        // holding values 4c, 16 + 4c, 4c + 1, 17 + 4c, ...; B is staged in the
        // same order.  Rows past nr and sub-blocks past the row end hold stale
        // bytes: their products land in unread accumulator lanes / columns.
        const int ks = st % TC_NS;
        sok = mbar_wait(&sh.cbar[ks], (cph >> ks) & 1u);
        cph ^= 1u << ks;
        if (!sok && tid == 0) set_error(a.st, ERR_WAIT_TIMEOUT, 62, blockIdx.x, u);
        // (ring rows are 128-byte swizzled: sub-block m of row rr sits in
        // column m ^ (rr % 8), so m = j % 8 keeps a phase's reads distinct)
#pragma unroll
        for (int k = 0; k < 2; k++) {
          const int i = tid + k * TC_WARPS * 32, l = i & 7, j = i >> 3, rr = 8 * (j >> 3) + l, m = j & 7;
          const uint4 cv = *reinterpret_cast<const uint4*>(ring + ks * TC_STAGE + swz(rr, 16 * m));
          const uint32_t cw[4] = {cv.x, cv.y, cv.z, cv.w};
          uint32_t o[8];
#pragma unroll
          for (int c = 0; c < 4; c++) {
            const uint32_t cn = cw[c] ^ 0x88888888u;
            o[2 * c] = mx_unpack4(cw[c], cn);
            o[2 * c + 1] = mx_unpack4(cw[c] >> 16, cn >> 16);
          }
          *reinterpret_cast<uint4*>(At + m * 4096 + kmaj(rr, 0)) = make_uint4(o[0], o[1], o[2], o[3]);
          *reinterpret_cast<uint4*>(At + m * 4096 + kmaj(rr, 16)) = make_uint4(o[4], o[5], o[6], o[7]);
        }
      }
      if (h == 0) {
        // 16 bytes bp = values 16 bp ..: sub-block bp / 2, K-half bp % 2
        uint4 bv = bnext;
        if constexpr (WF == FMT_MXFP4) {
          // K-half 0 of sub-block m interleaves values 0..7 with 16..23, K-half 1
          // values 8..15 with 24..31: pieces 2m and 2m + 1 swap the halves they lack
          const bool ev = (bp & 1) == 0;
          const uint32_t r0s = __shfl_xor_sync(FULL, ev ? bv.z : bv.x, 1);
          const uint32_t r1s = __shfl_xor_sync(FULL, ev ? bv.w : bv.y, 1);
          const uint32_t x0 = ev ? bv.x : r0s, x1 = ev ? bv.y : r1s;
          const uint32_t y0 = ev ? r0s : bv.z, y1 = ev ? r1s : bv.w;
          bv = make_uint4(__byte_perm(x0, y0, 0x5140), __byte_perm(x0, y0, 0x7362), __byte_perm(x1, y1, 0x5140),
                          __byte_perm(x1, y1, 0x7362));
        }
        *reinterpret_cast<uint4*>(Bt + (bp >> 1) * (TC_N * 32) + kmaj(bj, 16 * (bp & 1))) = bv;
        if (b + 1 < bpr) bnext = load_b(b + 1);
      }
      return sok;
    };
    auto issue = [&](int st) {   // the issuer thread
      const int h = st % F::SPB;
      constexpr uint32_t idesc = umma_idesc(F::A_SIGNED);
      const uint32_t tb = tmem + (uint32_t)(st & 1) * 256;
#pragma unroll
      for (int m = 0; m < 8; m++) {
        // Q4_K, MXFP4: sub-block m; Q6_K: group (h, lq = m % 2, k4 = m / 2) of chunk 4 h + m / 2
        const int bt = WF == FMT_Q6K ? 4 * h + (m >> 1) : m;
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

    // test hook: this thread's sums (weight row r0 + r, active row c0 + c)
    const int nsb_dbg = WF == FMT_Q6K ? a.K / 16 : a.K / 32;
    auto dbg_put1 = [&](int c, int sb, int v) {
      if (r < nr && c0 + c < nt)
        a.dbg[tc_debug_isum_index(off + j0 + c0 + c, a.mats, MODE == 0 ? mat : 0, a.R, r0 + r, nsb_dbg, sb)] = v;
    };
    auto dbg_put = [&](int c, int sb, int lo, int hi) {
      dbg_put1(c, sb, lo);
      dbg_put1(c, sb + 1, hi);
    };
    // epilogue of step st for this warp's EW active rows c0 .. c0 + EW - 1
    // (weight row r): the reference's fp32 fold of the integer sums
    auto epilogue = [&](auto ewc, int st) {
      constexpr int EW = decltype(ewc)::value;
      const int b = st / F::SPB, h = st - b * F::SPB;
      (void)h;
      const uint32_t tl = tmem + (uint32_t)(st & 1) * 256 + ((uint32_t)(32 * q) << 16) + c0;
      if constexpr (WF == FMT_Q4K) {
        const uint4 hd = sh.hdr[b & 1][r];
        const float d = f16_fast(hd.x & 0xFFFFu), dmin = f16_fast(hd.x >> 16);
        if constexpr (EW >= 2) {
          // active rows in pairs (c, c + 1) on f32x2: a pair shares its x4
          // group (c0 + c even, chunks start at multiples of 4)
          constexpr int P = EW / 2;
          float2 bs2[P];
#pragma unroll
          for (int pp = 0; pp < P; pp++) bs2[pp] = splat2(0.f);
          // two sub-block pairs' sums in flight per wait
#pragma unroll
          for (int g2 = 0; g2 < 4; g2 += 2) {
          uint32_t il2[2][EW], ih2[2][EW];
#pragma unroll
          for (int gg = 0; gg < 2; gg++) {
            tc_ld<EW>(tl + (2 * (g2 + gg)) * TC_N, il2[gg]);
            tc_ld<EW>(tl + (2 * (g2 + gg) + 1) * TC_N, ih2[gg]);
          }
          tc_wait_ld();
          if (a.dbg) {
#pragma unroll
            for (int gg = 0; gg < 2; gg++)
#pragma unroll
              for (int c = 0; c < EW; c++) dbg_put(c, 8 * b + 2 * (g2 + gg), (int)il2[gg][c], (int)ih2[gg][c]);
          }
#pragma unroll
          for (int gg = 0; gg < 2; gg++) {
            const int g = g2 + gg;
            const uint32_t (&il)[EW] = il2[gg];
            const uint32_t (&ih)[EW] = ih2[gg];
            int sl, ml, shh, mh;
            q4k_pair_scales(g, hd.y, hd.z, hd.w, sl, ml, shh, mh);
            const float2 dsl = splat2(fmul(d, (float)sl)), ndml = splat2(-fmul(dmin, (float)ml));
            const float2 dsh = splat2(fmul(d, (float)shh)), ndmh = splat2(-fmul(dmin, (float)mh));
#pragma unroll
            for (int pp = 0; pp < P; pp++) {
              const int jj = c0 + 2 * pp;
              const float2 flo = i2f_small2((int)il[2 * pp], (int)il[2 * pp + 1]);
              const float2 fhi = i2f_small2((int)ih[2 * pp], (int)ih[2 * pp + 1]);
              const float2 ba = *reinterpret_cast<const float2*>(&sh.xbsf[jj][b][2 * g]);
              const float2 bb = *reinterpret_cast<const float2*>(&sh.xbsf[jj + 1][b][2 * g]);
              const float2 blo = make_float2(ba.x, bb.x), bhi = make_float2(ba.y, bb.y);
              if (sh.x4[jj]) {
                float2 t = fadd2(fmul2z(dsl, flo, nz2), fmul2z(ndml, blo, nz2));
                t = fadd2(t, fmul2z(dsh, fhi, nz2));
                t = fadd2(t, fmul2z(ndmh, bhi, nz2));
                bs2[pp] = fadd2(bs2[pp], t);
              } else {
                bs2[pp] = fadd2(bs2[pp], fadd2(fmul2z(dsl, flo, nz2), fmul2z(ndml, blo, nz2)));
                bs2[pp] = fadd2(bs2[pp], fadd2(fmul2z(dsh, fhi, nz2), fmul2z(ndmh, bhi, nz2)));
              }
            }
          }
          }
#pragma unroll
          for (int pp = 0; pp < P; pp++) {
            const float2 xs = make_float2(sh.xscale[c0 + 2 * pp][b], sh.xscale[c0 + 2 * pp + 1][b]);
            const float2 v = fadd2(make_float2(acc[2 * pp], acc[2 * pp + 1]), fmul2z(xs, bs2[pp], nz2));
            acc[2 * pp] = v.x;
            acc[2 * pp + 1] = v.y;
          }
        } else {
          float bsum[EW];
#pragma unroll
          for (int c = 0; c < EW; c++) bsum[c] = 0.f;
#pragma unroll
          for (int g = 0; g < 4; g++) {
            uint32_t il[EW], ih[EW];
            tc_ld<EW>(tl + (2 * g) * TC_N, il);
            tc_ld<EW>(tl + (2 * g + 1) * TC_N, ih);
            tc_wait_ld();
            if (a.dbg)
#pragma unroll
              for (int c = 0; c < EW; c++) dbg_put(c, 8 * b + 2 * g, (int)il[c], (int)ih[c]);
            int sl, ml, shh, mh;
            q4k_pair_scales(g, hd.y, hd.z, hd.w, sl, ml, shh, mh);
            const float dsl = fmul(d, (float)sl), dml = fmul(dmin, (float)ml);
            const float dsh = fmul(d, (float)shh), dmh = fmul(dmin, (float)mh);
#pragma unroll
            for (int c = 0; c < EW; c++) {
              const int jj = c0 + c;
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
          for (int c = 0; c < EW; c++) acc[c] = fadd(acc[c], fmul(sh.xscale[c0 + c][b], bsum[c]));
        }
      } else if constexpr (WF == FMT_Q6K) {
        // the reference's fp32 fold of the block's 16 products sc * isum16,
        // in its order (half h, l-half lq, quarter k4); each product is an
        // exact integer in fp32
        const uint4 sv = sh.hdr[b & 1][r];
        const uint32_t sw[2] = {h ? sv.z : sv.x, h ? sv.w : sv.y};   // scales 8 h .. 8 h + 7
#pragma unroll
        for (int lq = 0; lq < 2; lq++)
#pragma unroll
          for (int k4 = 0; k4 < 4; k4++) {
            uint32_t is[EW];
            tc_ld<EW>(tl + (2 * k4 + lq) * TC_N, is);
            tc_wait_ld();
            if (a.dbg)
#pragma unroll
              for (int c = 0; c < EW; c++) dbg_put1(c, 16 * b + (2 * h + lq) * 4 + k4, (int)is[c]);
            const int si = lq + 2 * k4;
            const int sc = sbyte(sw[si >> 2], si & 3);
#pragma unroll
            for (int c = 0; c < EW; c++) fold[c] = fadd(fold[c], (float)(sc * (int)is[c]));
          }
        if (h == 1) {
          const float d = sh.dq[b & 1][r];
#pragma unroll
          for (int c = 0; c < EW; c++) {
            acc[c] = fadd(acc[c], fmul(fmul(d, sh.xscale[c0 + c][b]), fold[c]));
            fold[c] = 0.f;
          }
        }
      } else {
        // MXFP4 (dot_mxfp4_q8 533-547): total += (x.scale * e8m0_half(e)) * isum,
        // sub-blocks in order; the block's live sub-blocks nm (the last Q8
        // block of a row may hold fewer than 8)
        const int nm = min(8, nsub - 8 * b);
        const int eo = lay.a1 - tx + 8 * b;   // the block's scales in the row's tail (8-byte aligned)
        const uint8_t* ep = tail + swz(r, eo);
        uint32_t e8[8];
        if (nm == 8) {
          const uint2 v = *reinterpret_cast<const uint2*>(ep);
#pragma unroll
          for (int m = 0; m < 8; m++) e8[m] = ((m < 4 ? v.x : v.y) >> (8 * (m & 3))) & 0xFFu;
        } else {
#pragma unroll
          for (int m = 0; m < 8; m++) e8[m] = m < nm ? (uint32_t)tail[swz(r, eo + m)] : 0u;
        }
        float xs[EW];
#pragma unroll
        for (int c = 0; c < EW; c++) xs[c] = sh.xscale[c0 + c][b];
        constexpr int MB = EW <= 2 ? 8 : 4;   // accumulator loads in flight per wait
#pragma unroll
        for (int m0 = 0; m0 < 8; m0 += MB) {
          if (m0 >= nm) break;
          uint32_t is[MB][EW];
#pragma unroll
          for (int m = 0; m < MB; m++)
            if (m0 + m < nm) tc_ld<EW>(tl + (m0 + m) * TC_N, is[m]);
          tc_wait_ld();
          if (a.dbg)
#pragma unroll
            for (int m = 0; m < MB; m++)
              if (m0 + m < nm)
#pragma unroll
                for (int c = 0; c < EW; c++) dbg_put1(c, 8 * b + m0 + m, (int)is[m][c]);
#pragma unroll
          for (int m = 0; m < MB; m++) {
            if (m0 + m >= nm) break;
            const float es = e8m0_half(e8[m0 + m]);
            if constexpr (EW >= 2) {
#pragma unroll
              for (int pp = 0; pp < EW / 2; pp++) {
                const float2 t = fmul2z(fmul2z(make_float2(xs[2 * pp], xs[2 * pp + 1]), splat2(es), nz2),
                                       i2f_small2((int)is[m][2 * pp], (int)is[m][2 * pp + 1]), nz2);
                const float2 v = fadd2(make_float2(acc[2 * pp], acc[2 * pp + 1]), t);
                acc[2 * pp] = v.x;
                acc[2 * pp + 1] = v.y;
              }
            } else {
              acc[0] = fadd(acc[0], fmul(fmul(xs[0], es), i2f_small((int)is[m][0])));
            }
          }
        }
      }
    };

    if (wok) wok = stage(0);
    fence_proxy_async();
    tc_fence_before();
    ok = __syncthreads_and(wok) != 0;   // uniform: every thread leaves together
    tc_fence_after();
    if (ok && tid == TC_ISSUER) issue(0);
    // every thread has read ring stage 0: refill it (stage k refills follow stage(k))
    if constexpr (!F::RAW) {
      if (ok && tid == TC_ISSUER && TC_NS < nsteps) issue_codes(TC_NS);
    }
    for (int st = 0; st < nsteps && ok; st++) {
      const bool mok = mbar_wait(&sh.mbar, mphase);
      if (!mok && tid == 0) set_error(a.st, ERR_WAIT_TIMEOUT, 61, blockIdx.x, u);
      mphase ^= 1u;
      tc_fence_after();
      // MMAs of step st are done: A / B are free for step st + 1
      bool sok = true;
      if (mok && st + 1 < nsteps) sok = stage(st + 1);
      fence_proxy_async();
      tc_fence_before();
      ok = __syncthreads_and(mok && sok) != 0;
      tc_fence_after();
      if (!ok) break;
      if (tid == TC_ISSUER && st + 1 < nsteps) issue(st + 1);
      // every thread has read ring stage (st + 1) % TC_NS: refill it
      if constexpr (!F::RAW) {
        if (tid == TC_ISSUER && st + 1 + TC_NS < nsteps) issue_codes(st + 1 + TC_NS);
      }
      // warps past the chunk's rows idle
      if (c0 < nt) {
        switch (ew) {
          case 1: epilogue(IC<1>{}, st); break;
          case 2: epilogue(IC<2>{}, st); break;
          case 4: epilogue(IC<4>{}, st); break;
          default: epilogue(IC<8>{}, st); break;
        }
      }
      tc_fence_before();
    }
    // outputs of this unit
    if (ok && r < nr) {
#pragma unroll
      for (int c = 0; c < 8; c++) {
        const int jj = c0 + c;
        if (c >= ew || jj >= nt) continue;
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
  const size_t tiles = (size_t)8 * 4096 + 8 * TC_N * 32 + 64;
  const RowLayout lay = row_layout(wf, K);
  return 1024 + (wf == FMT_MXFP4 ? tiles + (size_t)(TC_NS + 1) * TC_STAGE : tiles + (size_t)TC_M * lay.rs);
}

// K input values per row in format f: whole 256-value blocks for Q4_K / Q6_K,
// 32-value sub-blocks for MXFP4, at most TC_MAX_BPR Q8 blocks.
static bool tc_fmt_ok(int f, int K) {
  if (f == FMT_Q4K || f == FMT_Q6K) return K > 0 && K % QK == 0 && K / QK <= TC_MAX_BPR;
  if (f == FMT_MXFP4) return K >= QK && K % 32 == 0 && (K + QK - 1) / QK <= TC_MAX_BPR;
  return false;
}

bool tc_moe_eligible(int gate_fmt, int down_fmt, int D, int I) {
  if ((gate_fmt != FMT_Q4K && gate_fmt != FMT_MXFP4) || !tc_fmt_ok(gate_fmt, D) || !tc_fmt_ok(down_fmt, I))
    return false;
  // dynamic + static shared memory within the 227 KB a CTA may use
  constexpr size_t cap = 227 * 1024 - sizeof(TcShared) - 256;
  return tc_smem(gate_fmt, D) <= cap && tc_smem(down_fmt, I) <= cap;
}

size_t tc_moe_scratch_bytes(int max_rows, int T, int K, int D, int I) {
  (void)T;
  (void)K;
  const int dbpr = (I + QK - 1) / QK;
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

size_t tc_tmap_bytes(int E) { return (size_t)E * 3 * sizeof(CUtensorMap); }

// The tensor map of an MXFP4 matrix: bytes as a [rows][rs] 2-D tensor, boxes
// of 128 rows x 128 bytes written with the 128-byte swizzle (16-byte column c
// of box row y lands in column c ^ (y % 8)), out-of-range elements read as
// zeros.
cudaError_t tc_build_tmaps(const ExpertDesc* experts, int E, void* d_tmaps) {
  using Encode = CUresult (*)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*, const cuuint64_t*,
                              const cuuint64_t*, const cuuint32_t*, const cuuint32_t*, CUtensorMapInterleave,
                              CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);
  static Encode encode = nullptr;
  if (!encode) {
    void* fn = nullptr;
    cudaDriverEntryPointQueryResult q{};
    const cudaError_t e = cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &fn, cudaEnableDefault, &q);
    if (e != cudaSuccess || q != cudaDriverEntryPointSuccess || !fn) return e != cudaSuccess ? e : cudaErrorNotSupported;
    encode = reinterpret_cast<Encode>(fn);
  }
  std::vector<CUtensorMap> maps((size_t)E * 3);
  memset(maps.data(), 0, maps.size() * sizeof(CUtensorMap));
  for (int e = 0; e < E; e++) {
    const WDesc* m3[3] = {&experts[e].gate, &experts[e].up, &experts[e].down};
    for (int m = 0; m < 3; m++) {
      const WDesc& W = *m3[m];
      if (!W.main || W.fmt != FMT_MXFP4 || W.rs < 128 || W.rs % 16) continue;
      const cuuint64_t dims[2] = {(cuuint64_t)W.rs, (cuuint64_t)W.rows};
      const cuuint64_t strides[1] = {(cuuint64_t)W.rs};
      const cuuint32_t box[2] = {128, (cuuint32_t)TC_M};
      const cuuint32_t estr[2] = {1, 1};
      const CUresult r = encode(&maps[(size_t)e * 3 + m], CU_TENSOR_MAP_DATA_TYPE_UINT8, 2,
                                const_cast<uint8_t*>(W.main), dims, strides, box, estr,
                                CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                                CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
      if (r != CUDA_SUCCESS) return cudaErrorInvalidValue;
    }
  }
  return cudaMemcpy(d_tmaps, maps.data(), maps.size() * sizeof(CUtensorMap), cudaMemcpyHostToDevice);
}

static int* g_tc_dbg_gu = nullptr;
static int* g_tc_dbg_dn = nullptr;
void set_tc_debug(int* gate_up, int* down) {
  g_tc_dbg_gu = gate_up;
  g_tc_dbg_dn = down;
}

cudaError_t launch_tc_moe(const PlanHdr* ph, int gate_fmt, int down_fmt, int T, int K, int D, int I, int max_rows,
                          const Q8Dev* xq8, const int* tok_rows, const void* tmaps, void* scratch, float* out,
                          DevStatus* st, cudaStream_t s) {
  const CUtensorMap* tm = static_cast<const CUtensorMap*>(tmaps);
  if ((gate_fmt == FMT_MXFP4 || down_fmt == FMT_MXFP4) && !tm) return cudaErrorInvalidValue;
  uint8_t* p = static_cast<uint8_t*>(scratch);
  auto take = [&](size_t n) {
    uint8_t* q = p;
    p += (n + 255) & ~(size_t)255;
    return q;
  };
  const int dbpr = (I + QK - 1) / QK;
  float* gu = reinterpret_cast<float*>(take((size_t)max_rows * 2 * I * 4));
  Q8Dev* hq8 = reinterpret_cast<Q8Dev*>(take((size_t)max_rows * dbpr * sizeof(Q8Dev)));
  float* parts = reinterpret_cast<float*>(take((size_t)max_rows * D * 4));
  TcArgs g{ph, xq8, gu, D, I, 2, st, tm, -0.0f, g_tc_dbg_gu};
  cudaError_t e = gate_fmt == FMT_MXFP4 ? tc_launch<FMT_MXFP4, 0>(g, s) : tc_launch<FMT_Q4K, 0>(g, s);
  if (e != cudaSuccess) return e;
  {
    const long warps = (long)max_rows * dbpr;
    const PlanHdr* php = ph;
    const float* gup = gu;
    int Iv = I;
    Q8Dev* hp = hq8;
    void* a2[] = {(void*)&php, (void*)&gup, (void*)&Iv, (void*)&hp};
    e = pdl_launch(reinterpret_cast<const void*>(act_quant_kernel), dim3((unsigned)((warps * 32 + 255) / 256)),
                   dim3(256), 0, s, a2);
    if (e != cudaSuccess) return e;
  }
  TcArgs dn{ph, hq8, parts, I, D, 1, st, tm, -0.0f, g_tc_dbg_dn};
  e = down_fmt == FMT_Q6K     ? tc_launch<FMT_Q6K, 1>(dn, s)
      : down_fmt == FMT_MXFP4 ? tc_launch<FMT_MXFP4, 1>(dn, s)
                              : tc_launch<FMT_Q4K, 1>(dn, s);
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
