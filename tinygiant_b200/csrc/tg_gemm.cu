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
// Persistent CTAs (one per SM) walk the units with specialised warps joined
// by mbarrier rings, so that loading, unpacking, the MMAs and the epilogue of
// different steps overlap, across unit boundaries too:
//   producer (warp 0): per 256-value block one 2-D TMA box of the unit's 128
//     weight rows (no multicast) and, one lane per active row, a bulk copy of
//     that row's Q8 block; per unit the rows' scale tails (Q6_K, MXFP4);
//   unpack warps: the weight box into int8 A tiles in the canonical K-major
//     no-swizzle layout (8-row x 16-byte core matrices), the Q8 blocks into
//     the B tiles, and the epilogue's per-step scales;
//   MMA (warp 1, one thread): one tcgen05.mma per sub-block into one of two
//     256-column accumulator buffers, committed to mbarriers;
//   epilogue warps: warp w reads TMEM lanes 32 (w % 4) .. (its weight rows)
//     for its share of the active rows and folds them in fp32.
// Every wait is bounded; a role that gives up records the error and the
// others stop waiting.
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
constexpr int TC_MAX_SLOTS = 256;
// Warp roles.  The four pipelines between them are mbarrier rings: weight
// stages (producer -> unpack), A/B operand stages (unpack -> MMA), the two
// tensor-memory accumulator buffers (MMA -> epilogue) and the epilogue's
// per-step data (unpack -> epilogue).
constexpr int TW_PROD = 0;    // lane 0 (and lanes < nt for the Q8 blocks): TMA loads of the weight stages
constexpr int TW_MMA = 1;     // lane 0: the MMAs
constexpr int TW_UNP = 2;     // warps 2 ..: unpack A, stage B, the epilogue's per-step data
constexpr int TC_NA = 2;      // A/B operand stages
constexpr int TC_NE = 2;      // epilogue data stages
// Per format the epilogue warp count: Q4_K and Q6_K steps are bound by the
// epilogue's fp32 fold (16 warps, 4 per lane quarter, up to 8 active rows
// each); MXFP4 steps by decoding the codes (8 epilogue warps, up to 16 active
// rows each).  Six unpack warps for every format.  The epilogue warps follow
// the unpack warps: warp wid reads TMEM lane quarter wid % 4, and each
// quarter gets one warp of each group tg = (wid - EPI) / 4.
template <int WF>
struct TcRoles {
  static constexpr int NUNP = 6;
  static constexpr int NEPI = WF == FMT_MXFP4 ? 8 : 16;
  static constexpr int EPI = TW_UNP + NUNP;
  static constexpr int WARPS = EPI + NEPI;
  static constexpr int UT = NUNP * 32;           // unpack threads
  static constexpr int NQ = NEPI / 4;            // epilogue warps per lane quarter
  static constexpr int EWMAX = TC_N / NQ;        // active rows per epilogue warp, at most
  static_assert(NEPI % 4 == 0 && TC_N % NQ == 0, "warp roles");
};

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
  int tailb;                  // Q6_K, MXFP4: bytes per row of the row-tail box (tc_tail_box)
  unsigned long long* trace;  // diagnostics: [gridDim.x][16] cycle counters of the roles (TC_TR_*), or null
};

// Trace counters per CTA (lane 0 of the producer, the MMA warp, the first
// unpack warp and the first epilogue warp): cycles spent waiting on each
// ring, and each role's whole span.
enum {
  TC_TR_PROD_WAIT = 0, TC_TR_PROD_SPAN,
  TC_TR_MMA_WAIT_AB, TC_TR_MMA_WAIT_TM, TC_TR_MMA_SPAN,
  TC_TR_UNP_WAIT_RAW, TC_TR_UNP_WAIT_AB, TC_TR_UNP_WAIT_EM, TC_TR_UNP_WAIT_TAIL, TC_TR_UNP_SPAN,
  TC_TR_EPI_WAIT_EM, TC_TR_EPI_WAIT_TM, TC_TR_EPI_SPAN,
  TC_TR_UNITS, TC_TR_STEPS, TC_TR_N = 16
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
constexpr int TC_XB = 304;        // bytes of an active row's Q8 block staged per step: qs, scale, sum, bsums
static_assert(TC_XB % 16 == 0 && TC_XB >= 296 && TC_XB <= (int)sizeof(Q8Dev), "staged Q8 block");

// The epilogue's data for one step, written by the unpack warps: per weight
// row the block's scales, per active row its Q8 scale and (Q4_K) 32-value
// sums, in the layouts the epilogue reads.
template <int WF>
struct TcEMeta;
template <>
struct TcEMeta<FMT_Q4K> {
  // per weight row and sub-block pair g the block's fp32 scale products
  // (d sc_2g, -(dmin m_2g), d sc_2g+1, -(dmin m_2g+1))
  float4 sc4[TC_M][4];
  float xscale[TC_N];      // active rows' Q8 scales
  float4 xb4[TC_N / 2][4]; // rows (2p, 2p + 1)'s 32-value sums of sub-blocks 2g (x, y) and 2g + 1 (z, w)
};
template <>
struct TcEMeta<FMT_Q6K> {
  uint4 sc16[TC_M];        // the block's 16 int8 scales
  float dq[TC_M];          // its d
  float xscale[TC_N];
};
template <>
struct TcEMeta<FMT_MXFP4> {
  uint2 e8[TC_M];          // the step's 8 e8m0 scales
  float xscale[TC_N];
};

template <int WF>
struct TcShared {
  uint64_t raw_full[4], raw_empty[4];     // weight stages
  uint64_t tail_full[2], tail_empty[2];   // the unit's row tails (Q6_K scales and d, MXFP4 e8m0)
  uint64_t ab_full[TC_NA], ab_empty[TC_NA];
  uint64_t tm_full[2], tm_empty[2];       // accumulator buffers
  uint64_t em_full[TC_NE], em_empty[TC_NE];
  uint32_t tmem;
  int n_units;
  int abort;                              // a role gave up: the others stop waiting
  unsigned long long tr[TC_TR_N];         // trace counters
  int unit_end[TC_MAX_SLOTS];             // inclusive prefix of units per slot
  TcEMeta<WF> em[TC_NE];
};

// A step is 8 MMAs (256 tensor-memory columns): Q4_K one 256-value block
// (its 8 sub-blocks), Q6_K half a block (its 8 16-value groups of half h),
// MXFP4 the 8 32-value sub-blocks that pair with one Q8 block.  Steps
// alternate between the two 256-column buffers, so the MMAs of step s + 1
// run while the epilogue reads step s.  Weight stages are 2-D TMA boxes of
// the unit's 128 rows: a Q4_K block (144 bytes a row), a Q6_K block's
// quants (192 bytes; its scales and d come with the unit's row-tail box), or
// 128 bytes of MXFP4 codes (128-byte swizzle; the e8m0 scales in the tail
// box).  The producer streams them across unit boundaries.
template <int WF>
struct TcFmt;
template <>
struct TcFmt<FMT_Q4K> {
  static constexpr int SPB = 1;            // steps per block
  static constexpr bool A_SIGNED = false;  // nibbles 0..15
  static constexpr int RAWB = Q4K_BYTES;   // weight stage bytes per row (one block)
  static constexpr int NR = 4;             // weight stages
  static constexpr bool TAIL = false;
};
template <>
struct TcFmt<FMT_Q6K> {
  static constexpr int SPB = 2;
  static constexpr bool A_SIGNED = true;   // q - 32
  static constexpr int RAWB = 192;         // a block's ql and qh
  static constexpr int NR = 3;
  static constexpr bool TAIL = true;
};
template <>
struct TcFmt<FMT_MXFP4> {
  static constexpr int SPB = 1;
  static constexpr bool A_SIGNED = true;   // doubled e2m1 values -12..12
  static constexpr int RAWB = 128;         // 8 sub-blocks' codes
  static constexpr int NR = 4;
  static constexpr bool TAIL = true;
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
template <>
__device__ __forceinline__ void tc_ld<16>(uint32_t taddr, uint32_t (&r)[16]) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x16.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15}, [%16];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]), "=r"(r[8]),
        "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15])
      : "r"(taddr));
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

// Bounded wait for phase `parity` of `bar` that also gives up once another
// role has set *abort.
__device__ __forceinline__ bool tc_wait(uint64_t* bar, uint32_t parity, const volatile int* abort) {
  if (mbar_try_wait(bar, parity)) return true;
  const long long t0 = clock64();
  while (!mbar_try_wait(bar, parity))
    if (*abort || clock64() - t0 > (1ll << 31)) return false;
  return true;
}

// DIAG: a diagnostics hook is on (the int32 sums of a.dbg, the role counters
// of a.trace); the kernel without them keeps fewer values live.
template <int WF, int MODE, bool DIAG>   // MODE 0: gate/up; 1: down
__global__ void __launch_bounds__(TcRoles<WF>::WARPS * 32, 1) tc_gemm_kernel(TcArgs a) {
  using F = TcFmt<WF>;
  using RL = TcRoles<WF>;
  constexpr int TC_UT = RL::UT, TW_NUNP = RL::NUNP, TW_EPI = RL::EPI, TW_NEPI = RL::NEPI;
  extern __shared__ __align__(1024) uint8_t dsm[];
  __shared__ TcShared<WF> sh;
  const int tid = threadIdx.x, lane = tid & 31, wid = tid >> 5;
  const PlanHdr* ph = a.ph;
  const int bpr = (a.K + QK - 1) / QK, nsub = a.K / 32;
  const RowLayout lay = row_layout(WF, a.K);
  const int tiles = (a.R + TC_M - 1) / TC_M;
  const int nsteps = bpr * F::SPB;
  const int tb = a.tailb;
  // shared memory from a 1024-byte boundary (the MXFP4 boxes' 128-byte
  // swizzle): A stages [TC_NA][8][4 KB], B stages [TC_NA][8][TC_N x 32 B],
  // weight stages [NR][128][RAWB], row tails [2][128][tb], the weight
  // stages' Q8 blocks [NR][TC_N][TC_XB]
  uint8_t* At = dsm + ((1024u - (smem_u32(dsm) & 1023u)) & 1023u);
  uint8_t* Bt = At + TC_NA * 8 * 4096;
  uint8_t* raw = Bt + TC_NA * 8 * TC_N * 32;
  uint8_t* tailb = raw + F::NR * TC_M * F::RAWB;
  uint8_t* xraw = tailb + 2 * TC_M * tb;   // [NR][TC_N][TC_XB]: the stages' Q8 blocks
  volatile int* abort = &sh.abort;
  // byte (row, o) of a 128-byte-row box written with the 128-byte swizzle
  auto swz = [](int row, int o) { return row * 128 + ((((o >> 4) ^ row) & 7) << 4) + (o & 15); };

  if (wid == 0) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(&sh.tmem)),
                 "r"(512));
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;");
  }
  if (tid == 32) {
    for (int k = 0; k < 4; k++) {
      mbar_init(&sh.raw_full[k], 1);
      mbar_init(&sh.raw_empty[k], TW_NUNP);
    }
    for (int k = 0; k < 2; k++) {
      mbar_init(&sh.tail_full[k], 1);
      mbar_init(&sh.tail_empty[k], TW_NUNP);
      mbar_init(&sh.tm_full[k], 1);
      mbar_init(&sh.tm_empty[k], TW_NEPI);
    }
    for (int k = 0; k < TC_NA; k++) {
      mbar_init(&sh.ab_full[k], TW_NUNP);
      mbar_init(&sh.ab_empty[k], 1);
    }
    for (int k = 0; k < TC_NE; k++) {
      mbar_init(&sh.em_full[k], TW_NUNP);
      mbar_init(&sh.em_empty[k], TW_NEPI);
    }
    sh.abort = 0;
    for (int k = 0; k < TC_TR_N; k++) sh.tr[k] = 0;
    fence_mbar_init();
  }
  // Q6_K's A tile m holds its group's 16 values in K-half m % 2 and zeros in
  // the other half, which never change
  if (WF == FMT_Q6K)
    for (int i = tid; i < TC_NA * 8 * 4096 / 16; i += RL::WARPS * 32)
      reinterpret_cast<uint4*>(At)[i] = make_uint4(0, 0, 0, 0);
  pdl_wait();   // the plan and the inputs come from the preceding kernels
  const int n_slots = ph->n_slots;
  // units per slot: mats x tiles x chunks of TC_N active rows
  if (wid == 1) {
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
  fence_proxy_async();   // the zeroed A tiles, before the tensor cores read them
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = sh.tmem;
  const int n_units = sh.n_units;

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
  auto fail = [&](int site, int u) {
    if (!*abort) set_error(a.st, ERR_WAIT_TIMEOUT, site, blockIdx.x, u);
    *abort = 1;
  };
  int issued = 0, tails = 0, mmas = 0;   // producer / MMA thread: for the waits at exit
  // the traced threads: lane 0 of the producer, MMA, first unpack and first epilogue warps
  const bool trt = DIAG && a.trace && lane == 0 && (wid == TW_PROD || wid == TW_MMA || wid == TW_UNP || wid == TW_EPI);
  auto twait = [&](uint64_t* bar, uint32_t parity, int slot) -> bool {
    if (!trt) return tc_wait(bar, parity, abort);
    const long long t0 = clock64();
    const bool r = tc_wait(bar, parity, abort);
    sh.tr[slot] += (unsigned long long)(clock64() - t0);
    return r;
  };
  const long long tstart = DIAG ? clock64() : 0;

  if (wid == TW_PROD) {
    // ---- producer warp: per unit its row tails (lane 0, once); per block
    // one weight box (lane 0) and the active rows' Q8 blocks (lane j: row j,
    // its qs, scale and sums: TC_XB bytes), all completing on the stage's
    // barrier
    bool ok = true;
    for (int u = blockIdx.x; u < n_units && ok; u += gridDim.x) {
      int s, mat, tile, ch;
      coords(u, s, mat, tile, ch);
      const SlotDesc& S = ph->slots[s];
      const CUtensorMap* mm = a.tmaps + 6 * S.expert + 2 * (MODE == 0 ? mat : 2);
      const int r0 = tile * TC_M, j0 = ch * TC_N, nt = min(TC_N, S.n_rows - j0);
      const int src = lane < nt ? (MODE == 0 ? ph->rows[S.row_off + j0 + lane] : S.row_off + j0 + lane) : 0;
      if constexpr (F::TAIL) {
        const int k = tails & 1;
        bool w = true;
        if (lane == 0 && tails >= 2) w = twait(&sh.tail_empty[k], ((tails >> 1) - 1) & 1, TC_TR_PROD_WAIT);
        if (!__shfl_sync(FULL, (int)w, 0)) {
          if (lane == 0) fail(67, u);
          break;
        }
        if (lane == 0) {
          mbar_arrive_expect_tx(&sh.tail_full[k], (uint32_t)(TC_M * tb));
          tma_load_2d(tailb + k * TC_M * tb, mm + 1, WF == FMT_Q6K ? lay.a1 : lay.rs - 128, r0, &sh.tail_full[k]);
        }
        tails++;
      }
      for (int b = 0; b < bpr; b++) {
        const int k = issued % F::NR;
        bool w = true;
        if (lane == 0 && issued >= F::NR) w = twait(&sh.raw_empty[k], ((issued / F::NR) - 1) & 1, TC_TR_PROD_WAIT);
        if (!__shfl_sync(FULL, (int)w, 0)) {
          if (lane == 0) fail(66, u);
          ok = false;
          break;
        }
        if (lane == 0) {
          mbar_arrive_expect_tx(&sh.raw_full[k], (uint32_t)(TC_M * F::RAWB + nt * TC_XB));
          tma_load_2d(raw + k * TC_M * F::RAWB, mm, F::RAWB * b, r0, &sh.raw_full[k]);
        }
        __syncwarp();   // the stage's byte count is set before any of its copies lands
        if (lane < nt) bulk_g2s(xraw + (k * TC_N + lane) * TC_XB, a.xsrc + (size_t)src * bpr + b, TC_XB, &sh.raw_full[k]);
        issued++;
      }
    }
    if (trt) sh.tr[TC_TR_PROD_SPAN] = clock64() - tstart;
  } else if (wid == TW_MMA) {
    // ---- MMA issuer: one MMA per sub-block, each from zero into its own columns
    if (lane == 0) {
      constexpr uint32_t idesc = umma_idesc(F::A_SIGNED);
      const int my_units = n_units > (int)blockIdx.x ? (n_units - 1 - (int)blockIdx.x) / (int)gridDim.x + 1 : 0;
      const int total = my_units * nsteps;
      for (int gs = 0; gs < total; gs++) {
        const int ka = gs % TC_NA, kt = gs & 1;
        if (!twait(&sh.ab_full[ka], (gs / TC_NA) & 1, TC_TR_MMA_WAIT_AB)) {
          fail(64, gs);
          break;
        }
        if (gs >= 2 && !twait(&sh.tm_empty[kt], ((gs >> 1) - 1) & 1, TC_TR_MMA_WAIT_TM)) {
          fail(65, gs);
          break;
        }
        tc_fence_after();
        const uint32_t tbuf = tmem + (uint32_t)kt * 256;
        const uint8_t* A = At + ka * 8 * 4096;
        const uint8_t* B = Bt + ka * 8 * TC_N * 32;
#pragma unroll
        for (int m = 0; m < 8; m++) {
          // Q4_K, MXFP4: sub-block m; Q6_K: group (lq = m % 2, k4 = m / 2) of the half, B chunk m / 2
          const int bt = WF == FMT_Q6K ? (m >> 1) : m;
          const uint64_t da = umma_desc(smem_u32(A + m * 4096)), db = umma_desc(smem_u32(B + bt * (TC_N * 32)));
          asm volatile("{\n\t.reg .pred p;\n\tsetp.ne.b32 p, %4, 0;\n\t"
                       "tcgen05.mma.cta_group::1.kind::i8 [%0], %1, %2, %3, p;\n\t}" ::"r"(tbuf + m * TC_N),
                       "l"(da), "l"(db), "r"(idesc), "r"(0));
        }
        asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(
            smem_u32(&sh.ab_empty[ka])));
        asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(
            smem_u32(&sh.tm_full[kt])));
        mmas = gs + 1;
      }
    }
    if (trt) {
      sh.tr[TC_TR_MMA_SPAN] = clock64() - tstart;
      sh.tr[TC_TR_STEPS] = mmas;
    }
  } else if (wid < TW_EPI) {
    // ---- unpack warps: per step A from the weight stage, B from the stage's
    // Q8 blocks, and the epilogue's data
    const int ut = tid - TW_UNP * 32;
    // B pieces per step: Q4_K and MXFP4: active row i / 16, 16-byte piece
    // i % 16 of the block; Q6_K: row i / 8, piece 8 h + i % 8 (half h's values)
    constexpr int NPC = WF == FMT_Q6K ? 8 : 16;
    int ur = 0, gs = 0, ui = 0;   // weight stages consumed, steps, units
    bool ok = true;
    for (int u = blockIdx.x; u < n_units && ok; u += gridDim.x, ui++) {
      int s, mat, tile, ch;
      coords(u, s, mat, tile, ch);
      const SlotDesc& S = ph->slots[s];
      const int j0 = ch * TC_N, nt = min(TC_N, S.n_rows - j0);
      const uint8_t* tl = tailb + (ui & 1) * TC_M * tb;
      if constexpr (F::TAIL) {
        if (!twait(&sh.tail_full[ui & 1], (ui >> 1) & 1, TC_TR_UNP_WAIT_TAIL)) {
          fail(67, u);
          break;
        }
      }
      for (int st = 0; st < nsteps; st++, gs++) {
        const int b = st / F::SPB, h = st - b * F::SPB;
        const int kr = ur % F::NR, ka = gs % TC_NA, ke = gs % TC_NE;
        if (h == 0 && !twait(&sh.raw_full[kr], (ur / F::NR) & 1, TC_TR_UNP_WAIT_RAW)) {
          fail(60, u);
          ok = false;
          break;
        }
        if (gs >= TC_NA && !twait(&sh.ab_empty[ka], ((gs / TC_NA) - 1) & 1, TC_TR_UNP_WAIT_AB)) {
          fail(62, u);
          ok = false;
          break;
        }
        if (gs >= TC_NE && !twait(&sh.em_empty[ke], ((gs / TC_NE) - 1) & 1, TC_TR_UNP_WAIT_EM)) {
          fail(63, u);
          ok = false;
          break;
        }
        const uint8_t* rw = raw + kr * TC_M * F::RAWB;
        uint8_t* A = At + ka * 8 * 4096;
        uint8_t* B = Bt + ka * 8 * TC_N * 32;
        TcEMeta<WF>& E = sh.em[ke];
        // item i = 8 j + l (l: the lane's place in its quarter-warp phase) ->
        // row rr = 8 (j / 8) + l: a phase's 8 stores go to 8 distinct rows of a
        // core matrix
        if constexpr (WF == FMT_Q4K) {
          // thread: row rr, 16-byte piece p of the 128 nibble bytes -> 32 values
          // (rows 144 bytes apart: a phase's 8 reads hit 8 distinct 16-byte columns)
#pragma unroll 1
          for (int i = ut; i < TC_M * 8; i += TC_UT) {
            const int l = i & 7, j = i >> 3, rr = 8 * (j >> 3) + l, p = j & 7;
            const uint8_t* row = rw + rr * Q4K_BYTES;
            const uint4 w = *reinterpret_cast<const uint4*>(row + 16 + 16 * p);
            // bytes 32g .. 32g + 31: low nibbles -> sub-block 2g, high -> 2g + 1
            const int g = p >> 1, kb = 16 * (p & 1);
            const uint4 lo = make_uint4(w.x & 0x0F0F0F0Fu, w.y & 0x0F0F0F0Fu, w.z & 0x0F0F0F0Fu, w.w & 0x0F0F0F0Fu);
            const uint4 hi = make_uint4((w.x >> 4) & 0x0F0F0F0Fu, (w.y >> 4) & 0x0F0F0F0Fu, (w.z >> 4) & 0x0F0F0F0Fu,
                                        (w.w >> 4) & 0x0F0F0F0Fu);
            *reinterpret_cast<uint4*>(A + (2 * g) * 4096 + kmaj(rr, kb)) = lo;
            *reinterpret_cast<uint4*>(A + (2 * g + 1) * 4096 + kmaj(rr, kb)) = hi;
          }
          // each row's scale products from its block header (as dot_q4k_q8_x4 forms them)
          for (int rr = ut; rr < TC_M; rr += TC_UT) {
            const uint4 hd = *reinterpret_cast<const uint4*>(rw + rr * Q4K_BYTES);
            const float d = f16_fast(hd.x & 0xFFFFu), dmin = f16_fast(hd.x >> 16);
#pragma unroll
            for (int g = 0; g < 4; g++) {
              int sl, ml, shh, mh;
              q4k_pair_scales(g, hd.y, hd.z, hd.w, sl, ml, shh, mh);
              E.sc4[rr][g] = make_float4(fmul(d, (float)sl), -fmul(dmin, (float)ml), fmul(d, (float)shh),
                                         -fmul(dmin, (float)mh));
            }
          }
        } else if constexpr (WF == FMT_Q6K) {
          // thread: row rr, group (lq, k4) of half h: tile m = 2 k4 + lq, values in K-half lq
#pragma unroll 1
          for (int i = ut; i < TC_M * 8; i += TC_UT) {
            const int l = i & 7, j = i >> 3, rr = 8 * (j >> 3) + l, m = (l + j) & 7, k4 = m >> 1,
                      lq = m & 1;
            const uint8_t* mb = rw + rr * 192;
            const uint4 va = *reinterpret_cast<const uint4*>(mb + 64 * h + 16 * lq + 32 * (k4 & 1));
            const uint4 vh = *reinterpret_cast<const uint4*>(mb + 128 + 32 * h + 16 * lq);
            const uint32_t qa[4] = {va.x, va.y, va.z, va.w}, qh[4] = {vh.x, vh.y, vh.z, vh.w};
            // quarter k4: low (k4 < 2) or high nibbles of ql, bits 2 k4 .. of qh as bits 4..5
            const int ls = 4 * (k4 >> 1), hs = 2 * k4;
            uint32_t o[4];
#pragma unroll
            for (int c = 0; c < 4; c++) {
              const uint32_t t = ((qa[c] >> ls) & 0x0F0F0F0Fu) | (((qh[c] >> hs) & 0x03030303u) << 4);
              // q - 32 as int8 per byte (q = 0..63): q + 96 without carries (bit 7 set
              // first), then bit 7 flipped back
              o[c] = ((t | 0x80808080u) - 0x20202020u) ^ 0x80808080u;
            }
            *reinterpret_cast<uint4*>(A + m * 4096 + kmaj(rr, 16 * lq)) = make_uint4(o[0], o[1], o[2], o[3]);
          }
          // the block's 16 scales and d from the row tail (scales at 16 b, d at 16 bpr + 2 b)
          for (int rr = ut; rr < TC_M; rr += TC_UT) {
            const uint8_t* t = tl + rr * tb;
            E.sc16[rr] = *reinterpret_cast<const uint4*>(t + 16 * b);
            E.dq[rr] = f16_fast((uint32_t)t[16 * bpr + 2 * b] | ((uint32_t)t[16 * bpr + 2 * b + 1] << 8));
          }
        } else {
          // thread: row rr, sub-block m; code word c (bytes 4c .. 4c + 3: values
          // 4c .. 4c + 3 low, 16 + 4c .. high) -> K positions 8c .. 8c + 7
          // holding values 4c, 16 + 4c, 4c + 1, 17 + 4c, ...; B is staged in the
          // same order.  Sub-blocks past the row end hold other bytes of the
          // row (or zeros): their products land in columns the epilogue skips.
          // (Rows are 128-byte swizzled: sub-block m of row rr sits in column
          // m ^ (rr % 8), so m = j % 8 keeps a phase's reads distinct.)
#pragma unroll 1
          for (int i = ut; i < TC_M * 8; i += TC_UT) {
            const int l = i & 7, j = i >> 3, rr = 8 * (j >> 3) + l, m = j & 7;
            const uint4 cv = *reinterpret_cast<const uint4*>(rw + swz(rr, 16 * m));
            const uint32_t cw[4] = {cv.x, cv.y, cv.z, cv.w};
            uint32_t o[8];
#pragma unroll
            for (int c = 0; c < 4; c++) {
              const uint32_t cn = cw[c] ^ 0x88888888u;
              o[2 * c] = mx_unpack4(cw[c], cn);
              o[2 * c + 1] = mx_unpack4(cw[c] >> 16, cn >> 16);
            }
            *reinterpret_cast<uint4*>(A + m * 4096 + kmaj(rr, 0)) = make_uint4(o[0], o[1], o[2], o[3]);
            *reinterpret_cast<uint4*>(A + m * 4096 + kmaj(rr, 16)) = make_uint4(o[4], o[5], o[6], o[7]);
          }
          // the step's live e8m0 scales (the last Q8 block of a row may pair
          // with fewer than 8 sub-blocks), 8-byte aligned in the swizzled tail
          const int nm = min(8, nsub - 8 * b), eo = lay.a1 - (lay.rs - 128) + 8 * b;
          for (int rr = ut; rr < TC_M; rr += TC_UT) {
            uint2 e = make_uint2(0, 0);
            if (nm == 8) {
              e = *reinterpret_cast<const uint2*>(tl + swz(rr, eo));
            } else {
              for (int m = 0; m < nm; m++) {
                const uint32_t v = (uint32_t)tl[swz(rr, eo + m)] << (8 * (m & 3));
                if (m < 4) e.x |= v;
                else e.y |= v;
              }
            }
            E.e8[rr] = e;
          }
        }
        // B: the stage's Q8 blocks into the K-major tiles (16 bytes bp = values
        // 16 bp ..: 32-value chunk bp / 2, K-half bp % 2); rows past the
        // chunk's nt are zeros
        const uint8_t* xr = xraw + kr * TC_N * TC_XB;
#pragma unroll
        for (int it = 0; it < (TC_N * NPC + TC_UT - 1) / TC_UT; it++) {   // (uniform per warp: multiples of 32)
          const int i = ut + it * TC_UT;
          if (TC_N * NPC % TC_UT && i >= TC_N * NPC) break;
          const int bj = i / NPC, pl = i % NPC, bp = WF == FMT_Q6K ? 8 * h + pl : pl;
          uint4 v = bj < nt ? *reinterpret_cast<const uint4*>(xr + bj * TC_XB + 16 * bp) : make_uint4(0, 0, 0, 0);
          if constexpr (WF == FMT_MXFP4) {
            // K-half 0 of sub-block m interleaves values 0..7 with 16..23, K-half 1
            // values 8..15 with 24..31: pieces 2m and 2m + 1 swap the halves they lack
            const bool ev = (pl & 1) == 0;
            const uint32_t r0s = __shfl_xor_sync(FULL, ev ? v.z : v.x, 1);
            const uint32_t r1s = __shfl_xor_sync(FULL, ev ? v.w : v.y, 1);
            const uint32_t x0 = ev ? v.x : r0s, x1 = ev ? v.y : r1s;
            const uint32_t y0 = ev ? r0s : v.z, y1 = ev ? r1s : v.w;
            v = make_uint4(__byte_perm(x0, y0, 0x5140), __byte_perm(x0, y0, 0x7362), __byte_perm(x1, y1, 0x5140),
                           __byte_perm(x1, y1, 0x7362));
          }
          *reinterpret_cast<uint4*>(B + (pl >> 1) * (TC_N * 32) + kmaj(bj, 16 * (pl & 1))) = v;
        }
        for (int jj = ut; jj < TC_N; jj += TC_UT)
          E.xscale[jj] = jj < nt ? *reinterpret_cast<const float*>(xr + jj * TC_XB + 256) : 0.f;
        if constexpr (WF == FMT_Q4K) {
          // thread (pair p, sub-block pair g): the bsums of rows 2p, 2p + 1 (at byte 264)
          for (int i = ut; i < TC_N / 2 * 4; i += TC_UT) {
            const int pr = i >> 2, g = i & 3, j0r = 2 * pr;
            int2 v0 = make_int2(0, 0), v1 = make_int2(0, 0);
            if (j0r < nt) v0 = *reinterpret_cast<const int2*>(xr + j0r * TC_XB + 264 + 8 * g);
            if (j0r + 1 < nt) v1 = *reinterpret_cast<const int2*>(xr + (j0r + 1) * TC_XB + 264 + 8 * g);
            E.xb4[pr][g] = make_float4((float)v0.x, (float)v1.x, (float)v0.y, (float)v1.y);
          }
        }
        fence_proxy_async();   // A and B, before the tensor cores read them
        __syncwarp();
        if (lane == 0) {
          mbar_arrive(&sh.ab_full[ka]);
          mbar_arrive(&sh.em_full[ke]);
          if (h == F::SPB - 1) mbar_arrive(&sh.raw_empty[kr]);
        }
        if (h == F::SPB - 1) ur++;
      }
      if constexpr (F::TAIL) {
        if (ok) {
          __syncwarp();
          if (lane == 0) mbar_arrive(&sh.tail_empty[ui & 1]);
        }
      }
    }
    if (trt) {
      sh.tr[TC_TR_UNP_SPAN] = clock64() - tstart;
      sh.tr[TC_TR_UNITS] = ui;
    }
  } else {
    // ---- epilogue: TMEM lane quarter q = wid % 4 (weight rows 32 q ..), the
    // chunk's active rows split over the quarter's four warps; the
    // reference's fp32 fold of the integer sums
    const int q = wid & 3, tg = (wid - TW_EPI) >> 2, r = 32 * q + lane;
    const float2 nz2 = splat2(a.negz);
    const int nsb_dbg = WF == FMT_Q6K ? a.K / 16 : a.K / 32;
    int gs = 0;
    bool ok = true;
    for (int u = blockIdx.x; u < n_units && ok; u += gridDim.x) {
      int s, mat, tile, ch;
      coords(u, s, mat, tile, ch);
      const SlotDesc& S = ph->slots[s];
      const int r0 = tile * TC_M, nr = min(TC_M, a.R - r0);
      const int j0 = ch * TC_N, nt = min(TC_N, S.n_rows - j0), off = S.row_off;
      // active rows per epilogue warp: the chunk's nt rows over a quarter's NQ
      // warps, a power of two
      int ew = 1;
      while (ew * RL::NQ < nt) ew *= 2;
      const int c0 = tg * ew;
      uint32_t x4m = 0;   // bit c: active row c0 + c takes the x4 association
      for (int c = 0; c < ew; c++)
        if (c0 + c < nt && use_x4(ph->assoc_rule, (j0 + c0 + c) & ~3, S.n_rows, ph->k)) x4m |= 1u << c;
      float acc[RL::EWMAX], fold[RL::EWMAX];
#pragma unroll
      for (int c = 0; c < RL::EWMAX; c++) acc[c] = fold[c] = 0.f;
      // test hook: this thread's sums (weight row r0 + r, active row c0 + c)
      auto dbg_put1 = [&](int c, int sb, int v) {
        if (r < nr && c0 + c < nt)
          a.dbg[tc_debug_isum_index(off + j0 + c0 + c, a.mats, MODE == 0 ? mat : 0, a.R, r0 + r, nsb_dbg, sb)] = v;
      };
      auto dbg_put = [&](int c, int sb, int lo, int hi) {
        dbg_put1(c, sb, lo);
        dbg_put1(c, sb + 1, hi);
      };
      // epilogue of step st for this warp's EW active rows c0 .. c0 + EW - 1
      // (weight row r), from accumulator columns tl
      auto epilogue = [&](auto ewc, int st, const TcEMeta<WF>& E, uint32_t tl) {
        constexpr int EW = decltype(ewc)::value;
        const int b = st / F::SPB, h = st - b * F::SPB;
        (void)h;
        if constexpr (WF == FMT_Q4K) {
          const float4* sc = E.sc4[r];
          if constexpr (EW >= 2) {
            // active rows in pairs (c, c + 1) on f32x2: a pair shares its x4
            // group (c0 + c even, chunks start at multiples of 4)
            constexpr int P = EW / 2;
            constexpr int GW = EW >= 8 ? 1 : 2;   // sub-block pairs per accumulator wait
            float2 bs2[P];
#pragma unroll
            for (int pp = 0; pp < P; pp++) bs2[pp] = splat2(0.f);
#pragma unroll
            for (int g2 = 0; g2 < 4; g2 += GW) {
              uint32_t il2[GW][EW], ih2[GW][EW];
#pragma unroll
              for (int gg = 0; gg < GW; gg++) {
                tc_ld<EW>(tl + (2 * (g2 + gg)) * TC_N, il2[gg]);
                tc_ld<EW>(tl + (2 * (g2 + gg) + 1) * TC_N, ih2[gg]);
              }
              tc_wait_ld();
              if (DIAG && a.dbg) {
#pragma unroll
                for (int gg = 0; gg < GW; gg++)
#pragma unroll
                  for (int c = 0; c < EW; c++) dbg_put(c, 8 * b + 2 * (g2 + gg), (int)il2[gg][c], (int)ih2[gg][c]);
              }
#pragma unroll
              for (int gg = 0; gg < GW; gg++) {
                const int g = g2 + gg;
                const float4 s4 = sc[g];
                const float2 dsl = splat2(s4.x), ndml = splat2(s4.y), dsh = splat2(s4.z), ndmh = splat2(s4.w);
#pragma unroll
                for (int pp = 0; pp < P; pp++) {
                  const float2 flo = i2f_small2((int)il2[gg][2 * pp], (int)il2[gg][2 * pp + 1]);
                  const float2 fhi = i2f_small2((int)ih2[gg][2 * pp], (int)ih2[gg][2 * pp + 1]);
                  const float4 b4 = E.xb4[(c0 >> 1) + pp][g];
                  const float2 blo = make_float2(b4.x, b4.y), bhi = make_float2(b4.z, b4.w);
                  if ((x4m >> (2 * pp)) & 1u) {
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
              const float2 xs = make_float2(E.xscale[c0 + 2 * pp], E.xscale[c0 + 2 * pp + 1]);
              const float2 v = fadd2(make_float2(acc[2 * pp], acc[2 * pp + 1]), fmul2z(xs, bs2[pp], nz2));
              acc[2 * pp] = v.x;
              acc[2 * pp + 1] = v.y;
            }
          } else {
            // (x - y = x + (-y) exactly: the negated products are the reference's subtrahends)
            float bsum = 0.f;
            const int hi1 = c0 & 1;
#pragma unroll
            for (int g = 0; g < 4; g++) {
              uint32_t il[1], ih[1];
              tc_ld<1>(tl + (2 * g) * TC_N, il);
              tc_ld<1>(tl + (2 * g + 1) * TC_N, ih);
              tc_wait_ld();
              if (DIAG && a.dbg) dbg_put(0, 8 * b + 2 * g, (int)il[0], (int)ih[0]);
              const float4 s4 = sc[g];
              const float flo = i2f_small((int)il[0]), fhi = i2f_small((int)ih[0]);
              const float4 b4 = E.xb4[c0 >> 1][g];
              const float blo = hi1 ? b4.y : b4.x, bhi = hi1 ? b4.w : b4.z;
              if (x4m & 1u) {
                bsum = fadd(bsum, fadd(fadd(fadd(fmul(s4.x, flo), fmul(s4.y, blo)), fmul(s4.z, fhi)), fmul(s4.w, bhi)));
              } else {
                bsum = fadd(bsum, fadd(fmul(s4.x, flo), fmul(s4.y, blo)));
                bsum = fadd(bsum, fadd(fmul(s4.z, fhi), fmul(s4.w, bhi)));
              }
            }
            acc[0] = fadd(acc[0], fmul(E.xscale[c0], bsum));
          }
        } else if constexpr (WF == FMT_Q6K) {
          // the reference's fp32 fold of the block's 16 products sc * isum16,
          // in its order (half h, l-half lq, quarter k4); each product is an
          // exact integer in fp32
          const uint4 sv = E.sc16[r];
          const uint32_t sw[2] = {h ? sv.z : sv.x, h ? sv.w : sv.y};   // scales 8 h .. 8 h + 7
          // (float)(sc * isum) as float(sc) * float(isum): both exact, |isum| < 2^22 and |product| < 2^24
#pragma unroll
          for (int lq = 0; lq < 2; lq++)
#pragma unroll
            for (int k2 = 0; k2 < 4; k2 += 2) {
              uint32_t is2[2][EW];
              tc_ld<EW>(tl + (2 * k2 + lq) * TC_N, is2[0]);
              tc_ld<EW>(tl + (2 * (k2 + 1) + lq) * TC_N, is2[1]);
              tc_wait_ld();
#pragma unroll
              for (int kk = 0; kk < 2; kk++) {
                const int k4 = k2 + kk;
                const uint32_t (&is)[EW] = is2[kk];
                if (DIAG && a.dbg)
#pragma unroll
                  for (int c = 0; c < EW; c++) dbg_put1(c, 16 * b + (2 * h + lq) * 4 + k4, (int)is[c]);
                const int si = lq + 2 * k4;
                const float scf = (float)sbyte(sw[si >> 2], si & 3);
                if constexpr (EW >= 2) {
#pragma unroll
                  for (int pp = 0; pp < EW / 2; pp++) {
                    const float2 v = fadd2(make_float2(fold[2 * pp], fold[2 * pp + 1]),
                                           fmul2z(splat2(scf), i2f_small2((int)is[2 * pp], (int)is[2 * pp + 1]), nz2));
                    fold[2 * pp] = v.x;
                    fold[2 * pp + 1] = v.y;
                  }
                } else {
                  fold[0] = fadd(fold[0], fmul(scf, i2f_small((int)is[0])));
                }
              }
            }
          if (h == 1) {
            const float d = E.dq[r];
#pragma unroll
            for (int c = 0; c < EW; c++) {
              acc[c] = fadd(acc[c], fmul(fmul(d, E.xscale[c0 + c]), fold[c]));
              fold[c] = 0.f;
            }
          }
        } else {
          // MXFP4 (dot_mxfp4_q8 533-547): total += (x.scale * e8m0_half(e)) * isum,
          // sub-blocks in order; the block's live sub-blocks nm
          const int nm = min(8, nsub - 8 * b);
          const uint2 eh = E.e8[r];
          float xs[EW];
#pragma unroll
          for (int c = 0; c < EW; c++) xs[c] = E.xscale[c0 + c];
          constexpr int MB = EW >= 8 ? 2 : EW >= 4 ? 4 : 8;   // accumulator loads in flight per wait
#pragma unroll
          for (int m0 = 0; m0 < 8; m0 += MB) {
            if (m0 >= nm) break;
            uint32_t is[MB][EW];
#pragma unroll
            for (int m = 0; m < MB; m++)
              if (m0 + m < nm) tc_ld<EW>(tl + (m0 + m) * TC_N, is[m]);
            tc_wait_ld();
            if (DIAG && a.dbg)
#pragma unroll
              for (int m = 0; m < MB; m++)
                if (m0 + m < nm)
#pragma unroll
                  for (int c = 0; c < EW; c++) dbg_put1(c, 8 * b + m0 + m, (int)is[m][c]);
#pragma unroll
            for (int m = 0; m < MB; m++) {
              if (m0 + m >= nm) break;
              const int mi = m0 + m;
              const float es = e8m0_half(((mi < 4 ? eh.x : eh.y) >> (8 * (mi & 3))) & 0xFFu);
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

      for (int st = 0; st < nsteps; st++, gs++) {
        const int ke = gs % TC_NE, kt = gs & 1;
        if (!twait(&sh.em_full[ke], (gs / TC_NE) & 1, TC_TR_EPI_WAIT_EM)) {
          fail(68, u);
          ok = false;
          break;
        }
        if (!twait(&sh.tm_full[kt], (gs >> 1) & 1, TC_TR_EPI_WAIT_TM)) {
          fail(61, u);
          ok = false;
          break;
        }
        tc_fence_after();
        if (c0 < nt) {   // warps past the chunk's rows idle
          const uint32_t tl = tmem + (uint32_t)kt * 256 + ((uint32_t)(32 * q) << 16) + c0;
          const TcEMeta<WF>& E = sh.em[ke];
          switch (ew) {
            case 1: epilogue(IC<1>{}, st, E, tl); break;
            case 2: epilogue(IC<2>{}, st, E, tl); break;
            case 4: epilogue(IC<4>{}, st, E, tl); break;
            case 8: epilogue(IC<8>{}, st, E, tl); break;
            default:
              if constexpr (RL::EWMAX >= 16) epilogue(IC<16>{}, st, E, tl);
              break;
          }
        }
        tc_fence_before();
        __syncwarp();
        if (lane == 0) {
          mbar_arrive(&sh.tm_empty[kt]);
          mbar_arrive(&sh.em_empty[ke]);
        }
      }
      // outputs of this unit
      if (ok && r < nr) {
#pragma unroll
        for (int c = 0; c < RL::EWMAX; c++) {
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
    }
  }

  if (trt && wid == TW_EPI) sh.tr[TC_TR_EPI_SPAN] = clock64() - tstart;
  // Exit: no copy or MMA of this CTA may still be in flight (after a role
  // gave up, stages issued before it may not have been waited for).
  if (wid == TW_PROD && lane == 0) {
    for (int i = max(0, issued - F::NR); i < issued; i++) mbar_wait(&sh.raw_full[i % F::NR], (i / F::NR) & 1);
    for (int i = max(0, tails - 2); i < tails; i++) mbar_wait(&sh.tail_full[i & 1], (i >> 1) & 1);
  }
  if (wid == TW_MMA && lane == 0 && mmas > 0) mbar_wait(&sh.ab_empty[(mmas - 1) % TC_NA], ((mmas - 1) / TC_NA) & 1);
  pdl_trigger();
  tc_fence_before();
  __syncthreads();
  if (wid == 0) asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(512));
  if (DIAG && a.trace && tid < TC_TR_N) a.trace[(size_t)blockIdx.x * TC_TR_N + tid] = sh.tr[tid];
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

// Weight stage bytes per row and weight stages, as TcFmt<f>.
static int tc_rawb(int f) { return f == FMT_Q4K ? TcFmt<FMT_Q4K>::RAWB : f == FMT_Q6K ? TcFmt<FMT_Q6K>::RAWB : TcFmt<FMT_MXFP4>::RAWB; }
static int tc_nr(int f) { return f == FMT_Q4K ? TcFmt<FMT_Q4K>::NR : f == FMT_Q6K ? TcFmt<FMT_Q6K>::NR : TcFmt<FMT_MXFP4>::NR; }

// Bytes per row of the row-tail box: MXFP4 the last 128 bytes of the row
// (its e8m0 scales); Q6_K its scales and d from offset a1, rounded up to an
// odd number of 16-byte units (rows that many bytes apart fall in distinct
// shared-memory banks); 0 for Q4_K or a tail that does not fit one box.
static int tc_tail_box(int f, int K) {
  const RowLayout lay = row_layout(f, K);
  if (f == FMT_MXFP4) return 128;
  if (f != FMT_Q6K) return 0;
  int u = (lay.rs - lay.a1 + 15) / 16;
  if (!(u & 1)) u++;
  return 16 * u <= 256 ? 16 * u : 0;
}

static size_t tc_smem(int wf, int K) {
  const size_t ab = (size_t)TC_NA * (8 * 4096 + 8 * TC_N * 32);
  return 1024 + ab + (size_t)tc_nr(wf) * (TC_M * tc_rawb(wf) + TC_N * TC_XB) + (size_t)2 * TC_M * tc_tail_box(wf, K);
}

// K input values per row in format f: whole 256-value blocks for Q4_K / Q6_K,
// 32-value sub-blocks for MXFP4, at most TC_MAX_BPR Q8 blocks; the row tail
// one box (Q6_K) or inside the row's last 128 bytes (MXFP4).
static bool tc_fmt_ok(int f, int K) {
  const RowLayout lay = row_layout(f, K);
  if (f == FMT_Q4K) return K > 0 && K % QK == 0 && K / QK <= TC_MAX_BPR;
  if (f == FMT_Q6K) return K > 0 && K % QK == 0 && K / QK <= TC_MAX_BPR && tc_tail_box(f, K) > 0;
  if (f == FMT_MXFP4)
    return K >= QK && K % 32 == 0 && (K + QK - 1) / QK <= TC_MAX_BPR && lay.rs >= 144 && lay.a1 >= lay.rs - 128;
  return false;
}

bool tc_moe_eligible(int gate_fmt, int down_fmt, int D, int I) {
  if ((gate_fmt != FMT_Q4K && gate_fmt != FMT_MXFP4) || !tc_fmt_ok(gate_fmt, D) || !tc_fmt_ok(down_fmt, I))
    return false;
  // dynamic + static shared memory within the 227 KB a CTA may use
  auto fits = [](int f, int K) {
    const size_t st = f == FMT_Q4K ? sizeof(TcShared<FMT_Q4K>) : f == FMT_Q6K ? sizeof(TcShared<FMT_Q6K>)
                                                                           : sizeof(TcShared<FMT_MXFP4>);
    return tc_smem(f, K) + st + 256 <= 227 * 1024;
  };
  return fits(gate_fmt, D) && fits(down_fmt, I);
}

size_t tc_moe_scratch_bytes(int max_rows, int T, int K, int D, int I) {
  (void)T;
  (void)K;
  const int dbpr = (I + QK - 1) / QK;
  return (size_t)max_rows * 2 * I * 4 + (size_t)max_rows * dbpr * sizeof(Q8Dev) + (size_t)max_rows * D * 4 + 3 * 256;
}

template <int WF, int MODE>
static cudaError_t tc_launch(const TcArgs& a, cudaStream_t s) {
  const void* fn = a.dbg || a.trace ? reinterpret_cast<const void*>(tc_gemm_kernel<WF, MODE, true>)
                                     : reinterpret_cast<const void*>(tc_gemm_kernel<WF, MODE, false>);
  const size_t smem = tc_smem(WF, a.K);
  cudaError_t e = ensure_smem(fn, smem);
  if (e != cudaSuccess) return e;
  TcArgs args = a;
  void* p[] = {(void*)&args};
  return pdl_launch(fn, dim3(tc_sms()), dim3(TcRoles<WF>::WARPS * 32), smem, s, p);
}

size_t tc_tmap_bytes(int E) { return (size_t)E * 6 * sizeof(CUtensorMap); }

// Two tensor maps per expert matrix (gate, up, down), each the matrix's bytes
// as a [rows][rs] 2-D tensor read in boxes of 128 rows, out-of-range elements
// as zeros: the weight stages (Q4_K 144-byte blocks, Q6_K 192-byte quants,
// MXFP4 128 bytes of codes written with the 128-byte swizzle: 16-byte column
// c of box row y lands in column c ^ (y % 8)) and the row tails (Q6_K
// tc_tail_box bytes from offset a1; MXFP4 the same map as the codes).
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
  std::vector<CUtensorMap> maps((size_t)E * 6);
  memset(maps.data(), 0, maps.size() * sizeof(CUtensorMap));
  for (int e = 0; e < E; e++) {
    const WDesc* m3[3] = {&experts[e].gate, &experts[e].up, &experts[e].down};
    for (int m = 0; m < 3; m++) {
      const WDesc& W = *m3[m];
      if (!W.main || !tc_fmt_ok(W.fmt, W.cols) || W.rs % 16) continue;
      const bool mx = W.fmt == FMT_MXFP4;
      const cuuint64_t dims[2] = {(cuuint64_t)W.rs, (cuuint64_t)W.rows};
      const cuuint64_t strides[1] = {(cuuint64_t)W.rs};
      const cuuint32_t estr[2] = {1, 1};
      const int tb = tc_tail_box(W.fmt, W.cols);
      const cuuint32_t boxes[2][2] = {{(cuuint32_t)tc_rawb(W.fmt), (cuuint32_t)TC_M},
                                      {(cuuint32_t)(mx ? 128 : tb), (cuuint32_t)TC_M}};
      for (int t = 0; t < 2; t++) {
        if (boxes[t][0] == 0) continue;   // Q4_K: no tail
        const CUresult r = encode(&maps[(size_t)e * 6 + 2 * m + t], CU_TENSOR_MAP_DATA_TYPE_UINT8, 2,
                                  const_cast<uint8_t*>(W.main), dims, strides, boxes[t], estr,
                                  CU_TENSOR_MAP_INTERLEAVE_NONE,
                                  mx ? CU_TENSOR_MAP_SWIZZLE_128B : CU_TENSOR_MAP_SWIZZLE_NONE,
                                  CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
        if (r != CUDA_SUCCESS) return cudaErrorInvalidValue;
      }
    }
  }
  return cudaMemcpy(d_tmaps, maps.data(), maps.size() * sizeof(CUtensorMap), cudaMemcpyHostToDevice);
}

static int* g_tc_dbg_gu = nullptr;
static int* g_tc_dbg_dn = nullptr;
static unsigned long long* g_tc_trace = nullptr;
void set_tc_trace(void* p) { g_tc_trace = static_cast<unsigned long long*>(p); }
int tc_trace_ctas() { return tc_sms(); }
void set_tc_debug(int* gate_up, int* down) {
  g_tc_dbg_gu = gate_up;
  g_tc_dbg_dn = down;
}

cudaError_t launch_tc_moe(const PlanHdr* ph, int gate_fmt, int down_fmt, int T, int K, int D, int I, int max_rows,
                          const Q8Dev* xq8, const int* tok_rows, const void* tmaps, void* scratch, float* out,
                          DevStatus* st, cudaStream_t s) {
  const CUtensorMap* tm = static_cast<const CUtensorMap*>(tmaps);
  if (!tm) return cudaErrorInvalidValue;
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
  TcArgs g{ph, xq8, gu, D, I, 2, st, tm, -0.0f, g_tc_dbg_gu, tc_tail_box(gate_fmt, D), g_tc_trace};
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
  TcArgs dn{ph, hq8, parts, I, D, 1, st, tm, -0.0f, g_tc_dbg_dn, tc_tail_box(down_fmt, I),
            g_tc_trace ? g_tc_trace + (size_t)tc_sms() * TC_TR_N : nullptr};
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
