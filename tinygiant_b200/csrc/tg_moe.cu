// tg_moe.cu — the two expert phases of one MoE call (sm_100a).
//
//   moe_gateup_kernel : gate.x, up.x (+ biases), activation -> hidden, then the
//                       Q8 re-quantization of hidden   (moe_phase_a, csrc/libtinygiant.c:1279-1327,
//                                                       and the quantize of moe_phase_b 1356-1360)
//   moe_down_kernel   : down.hidden, part = w * (v + bias), ordered combine
//                                                      (moe_phase_b 1329-1384, combine 1428-1434)
//
// Memory: each CTA's weight tile (16 gate + 16 up rows, or 8 down rows of
// every selected expert) is requested with bulk asynchronous copies (TMA,
// cp.async.bulk, no multicast) the moment the plan is readable, so a step's
// whole expert working set is in flight at once; compute reads the tiles from
// shared memory.  The down kernel issues its copies before waiting for the
// gate/up kernel (programmatic dependent launch), overlapping its weight
// stream with phase A.
//
// Compute: the lanes of a warp take a row's column units (Q4_K: a 64-value
// group of a block; Q6_K: 32 values of a block; MXFP4 / Q8_0: one 32-value
// block), exact int32 sums by dp4a, float terms in the reference's
// association, then a fold in the reference's order (tg_dots.cuh): every fp32
// row result equals the reference's bit for bit.  The combine adds each
// expert's part into an output element in the call's expert order.
#include <algorithm>

#include "tg_dots.cuh"
#include "tg_moe.h"
#include "tg_ptx.cuh"
#include "tg_q8.cuh"

namespace tg {

constexpr int A_ROWS = 16;    // gate/up rows per CTA; divides 256
constexpr int B_ROWS = 8;     // output rows per down CTA
constexpr int NWARP = 8;
constexpr int Q8_WORDS = sizeof(Q8Dev) / 16;   // uint4 per Q8 block

// ---------------------------------------------------------------------
// Tiles: the arrays of `rows` consecutive rows of a matrix in the HBM layout
// (tg_common.cuh WDesc), each rounded up to 16 bytes in shared memory.

struct TileMap {
  uint32_t n_main, n_aux1, n_aux2;   // bytes of each array
  uint32_t o_aux1, o_aux2, bytes;    // offsets in the tile; total
};

__host__ __device__ __forceinline__ TileMap tile_map(int fmt, int rows, int cols) {
  TileMap t{};
  const uint32_t bpr = cols / QK, nsub = cols / 32;
  switch (fmt) {
    case FMT_Q4K: t.n_main = rows * bpr * Q4K_BYTES; break;
    case FMT_Q6K: t.n_main = rows * bpr * 192; t.n_aux1 = rows * bpr * 16; t.n_aux2 = rows * bpr * 2; break;
    case FMT_MXFP4: t.n_main = rows * nsub * 16; t.n_aux1 = rows * nsub; break;
    case FMT_Q80: t.n_main = rows * nsub * 32; t.n_aux2 = rows * nsub * 2; break;
    default: t.n_main = rows * cols * 2; break;
  }
  t.o_aux1 = round16(t.n_main);
  t.o_aux2 = t.o_aux1 + round16(t.n_aux1);
  t.bytes = t.o_aux2 + round16(t.n_aux2);
  return t;
}

// Row r0's byte offset of each array in global memory.
__device__ __forceinline__ void tile_src(const WDesc& W, int r0, const uint8_t** m, const uint8_t** a1,
                                         const uint8_t** a2) {
  const TileMap t = tile_map(W.fmt, r0, W.cols);   // sizes of r0 rows = offsets of row r0
  *m = W.main + t.n_main;
  *a1 = W.aux1 ? W.aux1 + t.n_aux1 : nullptr;
  *a2 = W.aux2 ? W.aux2 + t.n_aux2 : nullptr;
}

// Thread 0: starts the bulk copies of rows [r0, r0+n) of W into `dst` and
// returns the bytes they will complete on `bar`; arrays whose source is not
// 16-byte aligned are left for copy_unaligned (all threads).
__device__ __forceinline__ uint32_t issue_tile(const WDesc& W, int r0, int n, uint8_t* dst, uint64_t* bar) {
  const TileMap t = tile_map(W.fmt, n, W.cols);
  const uint8_t *m, *a1, *a2;
  tile_src(W, r0, &m, &a1, &a2);
  uint32_t tx = 0;
  const uint8_t* src[3] = {m, a1, a2};
  const uint32_t len[3] = {t.n_main, t.n_aux1, t.n_aux2}, off[3] = {0, t.o_aux1, t.o_aux2};
  for (int i = 0; i < 3; i++)
    if (len[i] && ((uintptr_t)src[i] & 15) == 0) {
      bulk_g2s(dst + off[i], src[i], round16(len[i]), bar);
      tx += round16(len[i]);
    }
  return tx;
}

__device__ __forceinline__ uint32_t tile_tx_bytes(const WDesc& W, int r0, int n) {
  const TileMap t = tile_map(W.fmt, n, W.cols);
  const uint8_t *m, *a1, *a2;
  tile_src(W, r0, &m, &a1, &a2);
  uint32_t tx = 0;
  if (t.n_main && ((uintptr_t)m & 15) == 0) tx += round16(t.n_main);
  if (t.n_aux1 && ((uintptr_t)a1 & 15) == 0) tx += round16(t.n_aux1);
  if (t.n_aux2 && ((uintptr_t)a2 & 15) == 0) tx += round16(t.n_aux2);
  return tx;
}

// All threads: byte copies of the arrays issue_tile skipped.
__device__ __forceinline__ void copy_unaligned(const WDesc& W, int r0, int n, uint8_t* dst) {
  const TileMap t = tile_map(W.fmt, n, W.cols);
  const uint8_t *m, *a1, *a2;
  tile_src(W, r0, &m, &a1, &a2);
  const uint8_t* src[3] = {m, a1, a2};
  const uint32_t len[3] = {t.n_main, t.n_aux1, t.n_aux2}, off[3] = {0, t.o_aux1, t.o_aux2};
  for (int i = 0; i < 3; i++)
    if (len[i] && ((uintptr_t)src[i] & 15) != 0)
      for (uint32_t j = threadIdx.x; j < len[i]; j += blockDim.x) dst[off[i] + j] = src[i][j];
}

// ---------------------------------------------------------------------
// Staged Q8 inputs.  XBlk holds one 256-value Q8 block in shared memory with
// the exact int32 sums of each 16 values (for Q6_K's bias correction); its
// 368-byte stride puts the 8 blocks of a row on distinct banks.  For MXFP4
// each 4-byte group of qs is stored in the order [x0, x2, x1, x3], matching
// the order mxfp4_decode produces values in.

struct __align__(16) XBlk {
  int8_t qs[QK];
  float scale;
  int32_t sum;
  int32_t bsums[8];
  int32_t xs16[16];
  int32_t pad[2];
};
static_assert(sizeof(XBlk) == 368, "XBlk layout");

// Stages nrows Q8 rows (nb blocks each) from src (row pointers) into xs
// (row-major, nb blocks per row).  All threads; ends with __syncthreads.
template <int FMT>
__device__ __forceinline__ void stage_x(XBlk* xs, const Q8Dev* const* src, int nrows, int nb) {
  const int n = nrows * nb;
  // qs: 16 x 16 bytes per block
  for (int i = threadIdx.x; i < n * 16; i += blockDim.x) {
    const int blk = i >> 4, w = i & 15;
    const int row = blk / nb, b = blk - row * nb;
    uint4 v = reinterpret_cast<const uint4*>(src[row][b].qs)[w];
    if constexpr (FMT == FMT_MXFP4) {
      v.x = __byte_perm(v.x, 0, 0x3120);
      v.y = __byte_perm(v.y, 0, 0x3120);
      v.z = __byte_perm(v.z, 0, 0x3120);
      v.w = __byte_perm(v.w, 0, 0x3120);
    }
    reinterpret_cast<uint4*>(xs[blk].qs)[w] = v;
  }
  // scale, sum, bsums
  for (int i = threadIdx.x; i < n * 10; i += blockDim.x) {
    const int blk = i / 10, f = i - blk * 10;
    const int row = blk / nb, b = blk - row * nb;
    const Q8Dev& q = src[row][b];
    if (f == 0) xs[blk].scale = q.scale;
    else if (f == 1) xs[blk].sum = q.sum;
    else xs[blk].bsums[f - 2] = q.bsums[f - 2];
  }
  if constexpr (FMT == FMT_Q6K) {
    for (int i = threadIdx.x; i < n * 16; i += blockDim.x) {
      const int blk = i >> 4, j = i & 15;
      const int row = blk / nb, b = blk - row * nb;
      const int4 v = reinterpret_cast<const int4*>(src[row][b].qs)[j];
      int acc = dp4a(v.x, 0x01010101, 0);
      acc = dp4a(v.y, 0x01010101, acc);
      acc = dp4a(v.z, 0x01010101, acc);
      acc = dp4a(v.w, 0x01010101, acc);
      xs[blk].xs16[j] = acc;
    }
  }
  __syncthreads();
}

__device__ __forceinline__ uint4 lds16(const uint8_t* p) { return *reinterpret_cast<const uint4*>(p); }

// 4 e2m1 codes (one per byte, 0..15) -> 4 signed doubled values, in the byte
// order [v0, v2, v1, v3] (selector trick: c | c >> 12 packs the nibbles).
__device__ __forceinline__ int mxfp4_decode(uint32_t c) {
  const uint32_t sel = c | (c >> 12);
  const uint32_t pos = __byte_perm(0x03020100u, 0x0C080604u, sel & 0x7777u);   // 0,1,2,3 | 4,6,8,12
  const uint32_t neg = __byte_perm(0xFDFEFF00u, 0xF4F8FAFCu, sel & 0x7777u);   // 0,-1,-2,-3 | -4,-6,-8,-12
  return (int)__byte_perm(pos, neg, ((sel & 0x8888u) >> 1) | 0x3210u);
}

// Units of a row: one 256-value block (Q4_K, Q6_K) or one 32-value block
// (MXFP4, Q8_0); a unit produces one term of the row fold per token.
template <int FMT>
__host__ __device__ __forceinline__ int units_per_row(int cols) {
  return (FMT == FMT_Q4K || FMT == FMT_Q6K) ? cols / QK : cols / 32;
}

// The term of unit u of tile row rr for n tokens (x rows xr[t], staged).
// Q4_K / Q6_K: the block's sum folded in the reference's order times sx
// (and d); MXFP4 / Q8_0: (sx * scale) * isum.
template <int FMT>
__device__ __forceinline__ void unit_terms(const uint8_t* tile, const TileMap& tm, int cols, int rr, int u,
                                           const XBlk* const* xr, int n, bool x4, float* out) {
  if constexpr (FMT == FMT_Q4K) {
    const int bpr = cols / QK;
    const uint8_t* bl = tile + (rr * bpr + u) * Q4K_BYTES;
    const uint4 h = lds16(bl);
    const float d = f16_bits_to_f32(h.x & 0xFFFFu), dmin = f16_bits_to_f32(h.x >> 16);
    for (int t = 0; t < n; t++) {
      const XBlk& x = xr[t][u];
      const int4* xv = reinterpret_cast<const int4*>(x.qs);
      float bs = 0.f;
#pragma unroll
      for (int g = 0; g < 4; g++) {
        const uint4 q0 = lds16(bl + 16 + 32 * g), q1 = lds16(bl + 32 + 32 * g);
        const uint32_t q[8] = {q0.x, q0.y, q0.z, q0.w, q1.x, q1.y, q1.z, q1.w};
        const int4 a0 = xv[4 * g], a1 = xv[4 * g + 1], a2 = xv[4 * g + 2], a3 = xv[4 * g + 3];
        const int xl[8] = {a0.x, a0.y, a0.z, a0.w, a1.x, a1.y, a1.z, a1.w};
        const int xh[8] = {a2.x, a2.y, a2.z, a2.w, a3.x, a3.y, a3.z, a3.w};
        int ilo = 0, ihi = 0;
#pragma unroll
        for (int j = 0; j < 8; j++) {
          ilo = dp4a((int)(q[j] & 0x0F0F0F0Fu), xl[j], ilo);
          ihi = dp4a((int)((q[j] >> 4) & 0x0F0F0F0Fu), xh[j], ihi);
        }
        int sl, ml, sh, mh;
        q4k_scale_min(2 * g, h.y, h.z, h.w, sl, ml);
        q4k_scale_min(2 * g + 1, h.y, h.z, h.w, sh, mh);
        const float dsl = fmul(d, (float)sl), dml = fmul(dmin, (float)ml);
        const float dsh = fmul(d, (float)sh), dmh = fmul(dmin, (float)mh);
        const float blo = (float)x.bsums[2 * g], bhi = (float)x.bsums[2 * g + 1];
        if (x4) {
          bs = fadd(bs, fsub(fadd(fsub(fmul(dsl, (float)ilo), fmul(dml, blo)), fmul(dsh, (float)ihi)), fmul(dmh, bhi)));
        } else {
          bs = fadd(bs, fsub(fmul(dsl, (float)ilo), fmul(dml, blo)));
          bs = fadd(bs, fsub(fmul(dsh, (float)ihi), fmul(dmh, bhi)));
        }
      }
      out[t] = fmul(x.scale, bs);
    }
  } else if constexpr (FMT == FMT_Q6K) {
    const int bpr = cols / QK, bi = rr * bpr + u;
    const uint8_t* mp = tile + bi * 192;
    const uint4 sv = lds16(tile + tm.o_aux1 + bi * 16);
    const uint32_t sw[4] = {sv.x, sv.y, sv.z, sv.w};
    const uint16_t dbits = *reinterpret_cast<const uint16_t*>(tile + tm.o_aux2 + bi * 2);
    const float d = f16_bits_to_f32(dbits);
    for (int t = 0; t < n; t++) {
      const XBlk& x = xr[t][u];
      const int* xw = reinterpret_cast<const int*>(x.qs);
      float bs = 0.f;
#pragma unroll
      for (int h = 0; h < 2; h++)
#pragma unroll
        for (int c = 0; c < 2; c++) {
          // 16-byte chunks: ql[64h + 16c], ql[64h + 32 + 16c], qh[32h + 16c]
          const uint4 va = lds16(mp + 64 * h + 16 * c), vb = lds16(mp + 64 * h + 32 + 16 * c),
                      vh = lds16(mp + 128 + 32 * h + 16 * c);
          const uint32_t qa[4] = {va.x, va.y, va.z, va.w}, qb[4] = {vb.x, vb.y, vb.z, vb.w},
                         qh[4] = {vh.x, vh.y, vh.z, vh.w};
          int is[4] = {0, 0, 0, 0};
#pragma unroll
          for (int q = 0; q < 4; q++) {
            const int v0 = (int)((qa[q] & 0x0F0F0F0Fu) | ((qh[q] & 0x03030303u) << 4));
            const int v1 = (int)((qb[q] & 0x0F0F0F0Fu) | ((qh[q] & 0x0C0C0C0Cu) << 2));
            const int v2 = (int)(((qa[q] >> 4) & 0x0F0F0F0Fu) | (qh[q] & 0x30303030u));
            const int v3 = (int)(((qb[q] >> 4) & 0x0F0F0F0Fu) | ((qh[q] >> 2) & 0x30303030u));
            const int base = 32 * h + 4 * c + q;
            is[0] = dp4a(v0, xw[base], is[0]);
            is[1] = dp4a(v1, xw[base + 8], is[1]);
            is[2] = dp4a(v2, xw[base + 16], is[2]);
            is[3] = dp4a(v3, xw[base + 24], is[3]);
          }
#pragma unroll
          for (int kq = 0; kq < 4; kq++) {
            // (q - 32) . x = q . x - 32 * sum(x) over the 16 values
            const int isk = is[kq] - 32 * x.xs16[8 * h + 2 * kq + c];
            const int si = 8 * h + c + 2 * kq;
            const float sc = (float)(int8_t)((sw[si >> 2] >> (8 * (si & 3))) & 0xFFu);
            bs = fadd(bs, fmul(sc, (float)isk));
          }
        }
      out[t] = fmul(fmul(d, x.scale), bs);
    }
  } else if constexpr (FMT == FMT_MXFP4) {
    const int nsub = cols / 32, bi = rr * nsub + u;
    const uint4 cv = lds16(tile + bi * 16);
    const uint32_t cw[4] = {cv.x, cv.y, cv.z, cv.w};
    int lo[4], hi[4];
#pragma unroll
    for (int i = 0; i < 4; i++) {
      lo[i] = mxfp4_decode(cw[i] & 0x0F0F0F0Fu);
      hi[i] = mxfp4_decode((cw[i] >> 4) & 0x0F0F0F0Fu);
    }
    const float dh = e8m0_half(tile[tm.o_aux1 + bi]);
    for (int t = 0; t < n; t++) {
      const XBlk& x = xr[t][u >> 3];
      const int4* xv = reinterpret_cast<const int4*>(x.qs) + (u & 7) * 2;
      const int4 xa = xv[0], xc = xv[1];
      int acc = dp4a(lo[0], xa.x, 0);
      acc = dp4a(lo[1], xa.y, acc);
      acc = dp4a(lo[2], xa.z, acc);
      acc = dp4a(lo[3], xa.w, acc);
      acc = dp4a(hi[0], xc.x, acc);
      acc = dp4a(hi[1], xc.y, acc);
      acc = dp4a(hi[2], xc.z, acc);
      acc = dp4a(hi[3], xc.w, acc);
      out[t] = fmul(fmul(x.scale, dh), (float)acc);
    }
  } else {  // FMT_Q80
    const int nsub = cols / 32, bi = rr * nsub + u;
    const uint4 qa = lds16(tile + bi * 32), qb = lds16(tile + bi * 32 + 16);
    const int qw[8] = {(int)qa.x, (int)qa.y, (int)qa.z, (int)qa.w, (int)qb.x, (int)qb.y, (int)qb.z, (int)qb.w};
    const uint16_t dbits = *reinterpret_cast<const uint16_t*>(tile + tm.o_aux2 + bi * 2);
    const float d = f16_bits_to_f32(dbits);
    for (int t = 0; t < n; t++) {
      const XBlk& x = xr[t][u >> 3];
      const int4* xv = reinterpret_cast<const int4*>(x.qs) + (u & 7) * 2;
      const int4 xa = xv[0], xc = xv[1];
      const int xw[8] = {xa.x, xa.y, xa.z, xa.w, xc.x, xc.y, xc.z, xc.w};
      int acc = 0;
#pragma unroll
      for (int i = 0; i < 8; i++) acc = dp4a(qw[i], xw[i], acc);
      out[t] = fmul(fmul(x.scale, d), (float)acc);
    }
  }
}

// ---------------------------------------------------------------------
// Phase A.

// Dynamic shared memory of the gate/up kernel: two stages of (gate tile, up
// tile), up to 4 staged Q8 input rows, the term buffer [2][R][4][upr+1].
struct GuLayout {
  TileMap tm;
  uint32_t tile_bytes, stage_bytes, xs_off, p_off, total;
  int gbpr, upr, pstride;
};

template <int FMT>
__host__ __device__ __forceinline__ GuLayout gu_layout(int D) {
  GuLayout L;
  L.tm = tile_map(FMT, A_ROWS, D);
  L.tile_bytes = L.tm.bytes;
  L.stage_bytes = 2 * L.tile_bytes;
  L.gbpr = (D + QK - 1) / QK;
  L.upr = units_per_row<FMT>(D);
  L.pstride = L.upr + 1;   // odd stride: the row fold reads without bank conflicts
  L.xs_off = 2 * L.stage_bytes;
  L.p_off = L.xs_off + (uint32_t)sizeof(XBlk) * 4 * L.gbpr;
  L.total = L.p_off + (uint32_t)sizeof(float) * 2 * A_ROWS * 4 * L.pstride + 2 * A_ROWS * 4 * sizeof(float);
  return L;
}

// Persistent: CTA b takes tiles b, b + grid, ... of (slot, 16-row block of I);
// two stages, so the next tile's weights are in flight while one is computed.
// Per tile and group of <= 4 active rows: every thread computes whole units
// (one block of one row of gate or up), one thread per (matrix, row, token)
// folds the row, 16 threads apply the biases and the activation.
template <int FMT>
__global__ void __launch_bounds__(256, 2) moe_gateup_kernel(const PlanHdr* __restrict__ ph,
                                                         const Q8Dev* __restrict__ xq8, int gbpr,
                                                         float* __restrict__ hidden, Q8Dev* __restrict__ hq8,
                                                         int dbpr, int* __restrict__ counters, DevStatus* st) {
  extern __shared__ __align__(128) uint8_t sm[];
  __shared__ uint64_t bar[2];
  __shared__ __align__(16) SlotDesc sd[2];
  __shared__ const Q8Dev* xsrc[4];
  __shared__ Q8Scratch qsh;
  __shared__ int last_flag;
  pdl_wait();   // the plan and the inputs' Q8 blocks are written by the preceding kernel
  const int n_slots = ph->n_slots;
  const int I = ph->inter_dim, D = ph->embed_dim, k = ph->k, rule = ph->assoc_rule, act = ph->act;
  const SlotDesc* slots = ph->slots;
  const int* prow = ph->rows;
  const int tps = (I + A_ROWS - 1) / A_ROWS;   // tiles per slot
  const int n_tiles = n_slots * tps;
  if ((int)blockIdx.x >= n_tiles) {
    pdl_trigger();
    return;
  }
  const GuLayout L = gu_layout<FMT>(D);
  auto load_sd = [&](int stage, int tau) {
    if (threadIdx.x < (int)(sizeof(SlotDesc) / 16))
      reinterpret_cast<uint4*>(&sd[stage])[threadIdx.x] =
          reinterpret_cast<const uint4*>(slots + tau / tps)[threadIdx.x];
  };
  auto issue = [&](int stage, int tau) {   // thread 0
    const SlotDesc& S = sd[stage];
    const int r0 = (tau % tps) * A_ROWS, nr = min(A_ROWS, I - r0);
    uint8_t* base = sm + stage * L.stage_bytes;
    mbar_arrive_expect_tx(&bar[stage], tile_tx_bytes(S.gate, r0, nr) + tile_tx_bytes(S.up, r0, nr));
    issue_tile(S.gate, r0, nr, base, &bar[stage]);
    issue_tile(S.up, r0, nr, base + L.tile_bytes, &bar[stage]);
  };
  auto unaligned = [&](int stage, int tau) {   // all threads
    const SlotDesc& S = sd[stage];
    const int r0 = (tau % tps) * A_ROWS, nr = min(A_ROWS, I - r0);
    uint8_t* base = sm + stage * L.stage_bytes;
    copy_unaligned(S.gate, r0, nr, base);
    copy_unaligned(S.up, r0, nr, base + L.tile_bytes);
  };
  const int tau0 = blockIdx.x, tau1 = blockIdx.x + gridDim.x;
  load_sd(0, tau0);
  if (tau1 < n_tiles) load_sd(1, tau1);
  if (threadIdx.x == 0) {
    mbar_init(&bar[0], 1);
    mbar_init(&bar[1], 1);
    fence_mbar_init();
  }
  __syncthreads();
  if (threadIdx.x == 0) {
    issue(0, tau0);
    if (tau1 < n_tiles) issue(1, tau1);
  }
  pdl_trigger();
  unaligned(0, tau0);
  if (tau1 < n_tiles) unaligned(1, tau1);
  XBlk* xs = reinterpret_cast<XBlk*>(sm + L.xs_off);
  float* P = reinterpret_cast<float*>(sm + L.p_off);                     // [2][R][4][pstride]
  float* tot = P + 2 * A_ROWS * 4 * L.pstride;                           // [2][R][4]
  const int upr = L.upr;
  int it = 0;
  for (int tau = tau0; tau < n_tiles; tau += gridDim.x, it++) {
    const int stage = it & 1;
    const uint32_t parity = (it >> 1) & 1;
    const int s = tau / tps, r0 = (tau % tps) * A_ROWS, nr = min(A_ROWS, I - r0);
    const SlotDesc& S = sd[stage];
    const uint8_t* tile_g = sm + stage * L.stage_bytes;
    const uint8_t* tile_u = tile_g + L.tile_bytes;
    bool ready = false;
    for (int g0 = 0; g0 < S.n_rows; g0 += 4) {
      const int ng = min(4, S.n_rows - g0);
      const bool x4 = use_x4(rule, g0, S.n_rows, k);
      if (threadIdx.x < ng) xsrc[threadIdx.x] = xq8 + (size_t)prow[S.row_off + g0 + threadIdx.x] * gbpr;
      __syncthreads();
      stage_x<FMT>(xs, xsrc, ng, gbpr);
      if (!ready) {
        if (!mbar_wait(&bar[stage], parity)) {
          if (threadIdx.x == 0) set_error(st, ERR_WAIT_TIMEOUT, 10, s, r0);
          mbar_wait(&bar[stage ^ 1], parity);   // a bounded wait for the other stage's copies
          return;
        }
        ready = true;
      }
      const XBlk* xr[4] = {xs, xs + gbpr, xs + 2 * gbpr, xs + 3 * gbpr};
      // units: (matrix m, row rho, unit p)
      for (int uu = threadIdx.x; uu < 2 * nr * upr; uu += blockDim.x) {
        const int m = uu / (nr * upr), rem = uu - m * nr * upr, rho = rem / upr, p = rem - rho * upr;
        float o[4];
        unit_terms<FMT>(m ? tile_u : tile_g, L.tm, D, rho, p, xr, ng, x4, o);
        for (int t = 0; t < ng; t++) P[((m * A_ROWS + rho) * 4 + t) * L.pstride + p] = o[t];
      }
      __syncthreads();
      // row folds in order: one thread per (matrix, row, token)
      for (int f = threadIdx.x; f < 2 * nr * ng; f += blockDim.x) {
        const int m = f / (nr * ng), rem = f - m * nr * ng, rho = rem / ng, t = rem - rho * ng;
        const float* pp = P + ((m * A_ROWS + rho) * 4 + t) * L.pstride;
        float acc = 0.f;
        for (int q = 0; q < upr; q++) acc = fadd(acc, pp[q]);
        tot[(m * A_ROWS + rho) * 4 + t] = acc;
      }
      __syncthreads();
      for (int f = threadIdx.x; f < nr * ng; f += blockDim.x) {
        const int rho = f / ng, t = f - rho * ng, r = r0 + rho;
        float gv = tot[rho * 4 + t], uv = tot[(A_ROWS + rho) * 4 + t];
        if (S.gb) {
          gv = fadd(gv, S.gb[r]);
          uv = fadd(uv, S.ub[r]);
        }
        hidden[(size_t)(S.row_off + g0 + t) * I + r] = act_fn(act, gv, uv);
      }
      __syncthreads();
    }
    if (!ready && !mbar_wait(&bar[stage], parity)) {   // a slot without rows still drains its stage
      if (threadIdx.x == 0) set_error(st, ERR_WAIT_TIMEOUT, 12, s, r0);
      return;
    }
    // The last CTA to finish a 256-row block of this slot's hidden rows
    // quantizes that block for phase B.
    const int kb = r0 / QK;
    const int blk_rows = min(QK, I - kb * QK);
    const int tiles_in_blk = (blk_rows + A_ROWS - 1) / A_ROWS;
    if (threadIdx.x == 0) {
      __threadfence();
      int* c = counters + (size_t)s * dbpr + kb;
      const int prev = atomicAdd(c, 1);
      last_flag = prev == tiles_in_blk - 1;
      if (last_flag) *c = 0;   // every tile of the block has arrived: reset for the next call
    }
    __syncthreads();
    if (last_flag) {
      __threadfence();
      const int t = threadIdx.x;
      for (int j = 0; j < S.n_rows; j++) {
        const size_t row = (size_t)(S.row_off + j);
        const bool valid = t < blk_rows;
        const float v = valid ? __ldcg(hidden + row * I + (size_t)kb * QK + t) : 0.f;
        quantize_block_cta(v, valid, hq8 + row * dbpr + kb, qsh);
      }
    }
    __syncthreads();
    // this stage is free: fetch the tile after next into it
    const int tn = tau + 2 * (int)gridDim.x;
    if (tn < n_tiles) {
      load_sd(stage, tn);
      __syncthreads();
      if (threadIdx.x == 0) issue(stage, tn);
      unaligned(stage, tn);
    }
  }
}

// ---------------------------------------------------------------------
// Phase B.

// The fields of a slot the down kernel reads, staged in shared memory.
struct __align__(16) DnSlot {
  WDesc down;
  const float* db;
  int n_rows, row_off;
  int pad[2];
};

// Active rows per combine batch: bounded by the term buffer
// [items][B_ROWS][upr+1] and the staged inputs [items][dbpr].
template <int FMT>
__host__ __device__ __forceinline__ int dn_batch(int I) {
  const int upr = units_per_row<FMT>(I);
  return upr <= 8 ? 32 : 8;
}

// Dynamic shared memory: [tile buffers][terms][parts][running output]
// [staged inputs][slot table]; nb = active rows per batch.
template <int FMT>
__host__ __device__ __forceinline__ uint32_t dn_fixed_bytes(int I, int T, int max_slots, int nb) {
  const int upr = units_per_row<FMT>(I), dbpr = (I + QK - 1) / QK;
  return (uint32_t)sizeof(float) * (nb * B_ROWS * (upr + 1) + nb * B_ROWS + T * B_ROWS) +
         (uint32_t)sizeof(XBlk) * nb * dbpr + (uint32_t)sizeof(DnSlot) * max_slots;
}

// CTA = B_ROWS output rows.  The selected experts' down tiles (B_ROWS rows
// each) stream through two shared-memory buffers in windows of consecutive
// slots.  Per batch of active rows (the call's order): units (active row,
// output row, block) on all threads, one thread per (active row, output row)
// folds the row and forms w * (v + bias), one thread per output row adds the
// parts in order into the running output.  With parts_out set (calls whose
// experts mix down formats) only slots of format FMT are computed and the
// parts are stored for combine_parts_kernel.
template <int FMT>
__global__ void __launch_bounds__(256, 2) moe_down_kernel(const PlanHdr* __restrict__ ph,
                                                       const Q8Dev* __restrict__ hq8, int dbpr,
                                                       const float* __restrict__ hidden, float* __restrict__ out,
                                                       float* __restrict__ parts_out, uint32_t buf_bytes,
                                                       uint32_t tile_region, int max_slots, int nbmax,
                                                       DevStatus* st) {
  extern __shared__ __align__(128) uint8_t sm[];
  __shared__ uint64_t bar[2];
  constexpr int NBMAX = 32;
  __shared__ int b_sr[NBMAX], b_slot[NBMAX];
  __shared__ const Q8Dev* b_x[NBMAX];
  __shared__ int cur_s, cur_j, n_batch;
  // The plan was written before the preceding kernel passed its own wait, so
  // it is readable here; hidden and its Q8 blocks are not (pdl_wait below).
  const int D = ph->embed_dim, I = ph->inter_dim, n_slots = ph->n_slots, k = ph->k, rule = ph->assoc_rule;
  const int bias_term = ph->bias_term;
  const SlotDesc* gslots = ph->slots;
  const int* rows = ph->rows;
  const float* wts = ph->wts;
  const int r0 = blockIdx.x * B_ROWS;
  const int nr = min(B_ROWS, D - r0);
  const TileMap tm = tile_map(FMT, B_ROWS, I);
  if (n_slots > max_slots) {
    if (threadIdx.x == 0) set_error(st, ERR_BAD_PLAN, 13, n_slots, max_slots);
    pdl_wait();
    pdl_trigger();
    return;
  }
  const int upr = units_per_row<FMT>(I), ps = upr + 1;
  float* P = reinterpret_cast<float*>(sm + tile_region);          // [nbmax][B_ROWS][ps]
  float* parts = P + nbmax * B_ROWS * ps;                          // [nbmax][B_ROWS]
  float* acc = parts + nbmax * B_ROWS;                             // [k][B_ROWS]
  XBlk* xs = reinterpret_cast<XBlk*>(acc + k * B_ROWS);            // [nbmax][dbpr]
  DnSlot* slots = reinterpret_cast<DnSlot*>(xs + nbmax * dbpr);    // [max_slots]
  for (int i = threadIdx.x; i < n_slots; i += blockDim.x) {
    DnSlot d;
    d.down = gslots[i].down;
    d.db = gslots[i].db;
    d.n_rows = gslots[i].n_rows;
    d.row_off = gslots[i].row_off;
    slots[i] = d;
  }
  const uint32_t half = buf_bytes;
  const int per_buf = (int)(half / tm.bytes);                      // slot tiles per buffer
  auto mine = [&](int s) { return parts_out == nullptr || slots[s].down.fmt == FMT; };
  auto issue_window = [&](int buf, int lo, int hi) {
    if (threadIdx.x == 0) {
      uint32_t tx = 0;
      for (int s = lo; s < hi; s++)
        if (mine(s)) tx += tile_tx_bytes(slots[s].down, r0, nr);
      mbar_arrive_expect_tx(&bar[buf], tx);
      for (int s = lo; s < hi; s++)
        if (mine(s)) issue_tile(slots[s].down, r0, nr, sm + buf * half + (s - lo) * tm.bytes, &bar[buf]);
    }
  };
  if (threadIdx.x == 0) {
    mbar_init(&bar[0], 1);
    mbar_init(&bar[1], 1);
    fence_mbar_init();
  }
  __syncthreads();   // slot table and barriers ready
  issue_window(0, 0, min(n_slots, per_buf));
  if (per_buf < n_slots) issue_window(1, per_buf, min(n_slots, 2 * per_buf));
  pdl_wait();   // hidden and its Q8 blocks are complete
  pdl_trigger();
  if (!parts_out)
    for (int i = threadIdx.x; i < k * B_ROWS; i += blockDim.x) {
      const int t = i / B_ROWS, rho = i - t * B_ROWS;
      acc[i] = rho < nr ? out[(size_t)t * D + r0 + rho] : 0.f;
    }
  uint32_t phase[2] = {0, 0};
  int buf = 0;
  for (int lo = 0; lo < n_slots; lo += per_buf) {
    const int hi = min(n_slots, lo + per_buf);
    uint8_t* base = sm + buf * half;
    for (int s = lo; s < hi; s++)
      if (mine(s)) copy_unaligned(slots[s].down, r0, nr, base + (s - lo) * tm.bytes);
    if (threadIdx.x == 0) {
      cur_s = lo;
      cur_j = 0;
    }
    __syncthreads();
    if (!mbar_wait(&bar[buf], phase[buf])) {
      if (threadIdx.x == 0) set_error(st, ERR_WAIT_TIMEOUT, 11, blockIdx.x, lo);
      mbar_wait(&bar[buf ^ 1], phase[buf ^ 1]);
      return;
    }
    phase[buf] ^= 1;
    for (;;) {
      // next batch of active rows of the window, in the call's order
      if (threadIdx.x == 0) {
        int s = cur_s, j = cur_j, nb = 0;
        while (s < hi && nb < nbmax) {
          if (!mine(s) || j >= slots[s].n_rows) {
            s++;
            j = 0;
            continue;
          }
          const int sr = slots[s].row_off + j;
          b_sr[nb] = sr;
          b_slot[nb] = s;
          b_x[nb] = hq8 + (size_t)sr * dbpr;
          nb++;
          j++;
        }
        cur_s = s;
        cur_j = j;
        n_batch = nb;
      }
      __syncthreads();
      const int ni = n_batch;
      if (ni == 0) break;
      stage_x<FMT>(xs, b_x, ni, dbpr);
      // units: (active row it, output row rho, unit p)
      for (int uu = threadIdx.x; uu < ni * nr * upr; uu += blockDim.x) {
        const int it = uu / (nr * upr), rem = uu - it * nr * upr, rho = rem / upr, p = rem - rho * upr;
        const int s = b_slot[it], sr = b_sr[it];
        const bool x4 = use_x4(rule, sr - slots[s].row_off, slots[s].n_rows, k);
        const XBlk* xr[1] = {xs + it * dbpr};
        float o[1];
        unit_terms<FMT>(base + (s - lo) * tm.bytes, tm, I, rho, p, xr, 1, x4, o);
        P[(it * B_ROWS + rho) * ps + p] = o[0];
      }
      __syncthreads();
      // row folds and parts: one thread per (active row, output row)
      for (int f = threadIdx.x; f < ni * nr; f += blockDim.x) {
        const int it = f / nr, rho = f - it * nr;
        const int s = b_slot[it], sr = b_sr[it];
        float v;
        if constexpr (FMT == FMT_F16) {
          // the reference's 8 fused lane chains, pairwise lane sum, then the tail
          const uint16_t* row = reinterpret_cast<const uint16_t*>(base + (s - lo) * tm.bytes) + (size_t)rho * I;
          const float* x = hidden + (size_t)sr * I;
          float a0[4] = {0.f, 0.f, 0.f, 0.f}, a1[4] = {0.f, 0.f, 0.f, 0.f};
          int q = 0;
          for (; q + 7 < I; q += 8)
#pragma unroll
            for (int l = 0; l < 4; l++) {
              a0[l] = __fmaf_rn(half_ieee(row[q + l]), x[q + l], a0[l]);
              a1[l] = __fmaf_rn(half_ieee(row[q + 4 + l]), x[q + 4 + l], a1[l]);
            }
          v = fadd(fadd(fadd(a0[0], a1[0]), fadd(a0[1], a1[1])), fadd(fadd(a0[2], a1[2]), fadd(a0[3], a1[3])));
          for (; q < I; q++) v = fadd(v, fmul(f16_bits_to_f32(row[q]), x[q]));
        } else {
          const float* pp = P + (it * B_ROWS + rho) * ps;
          v = 0.f;
          for (int q = 0; q < upr; q++) v = fadd(v, pp[q]);
        }
        const float* db = slots[s].db;
        const float w = wts[sr];
        const float part = bias_term ? fmul(w, fadd(v, db ? db[r0 + rho] : 0.f)) : fmul(w, v);
        if (parts_out) parts_out[(size_t)sr * D + r0 + rho] = part;
        else parts[it * B_ROWS + rho] = part;
      }
      __syncthreads();
      if (!parts_out && threadIdx.x < nr)
        for (int it = 0; it < ni; it++) {
          const int t = rows[b_sr[it]];
          acc[t * B_ROWS + threadIdx.x] = fadd(acc[t * B_ROWS + threadIdx.x], parts[it * B_ROWS + threadIdx.x]);
        }
      __syncthreads();
    }
    // this buffer is free: start the window after next
    const int nlo = lo + 2 * per_buf;
    if (nlo < n_slots) issue_window(buf, nlo, min(n_slots, nlo + per_buf));
    buf ^= 1;
  }
  if (!parts_out)
    for (int i = threadIdx.x; i < k * B_ROWS; i += blockDim.x) {
      const int t = i / B_ROWS, rho = i - t * B_ROWS;
      if (rho < nr) out[(size_t)t * D + r0 + rho] = acc[i];
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
  cfg.blockDim = dim3(256);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = s;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  return cudaLaunchKernelExC(&cfg, fn, args);
}

// CTAs of `fn` resident at once with `smem` bytes (all SMs).
static int resident_ctas(const void* fn, size_t smem) {
  static int sms = 0;
  if (!sms) {
    int dev = 0;
    cudaGetDevice(&dev);
    cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
  }
  int per = 0;
  if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per, fn, 256, smem) != cudaSuccess || per < 1) per = 1;
  return per * sms;
}

template <int FMT>
static cudaError_t gateup_fmt(const PlanHdr* ph, int max_slots, int D, int I, const Q8Dev* xq8, float* hidden,
                              Q8Dev* hq8, int* counters, DevStatus* st, cudaStream_t s) {
  const GuLayout L = gu_layout<FMT>(D);
  const void* fn = reinterpret_cast<const void*>(moe_gateup_kernel<FMT>);
  cudaError_t e = ensure_smem(fn, L.total);
  if (e != cudaSuccess) return e;
  static int cap[5] = {0, 0, 0, 0, 0};
  if (!cap[FMT]) cap[FMT] = resident_ctas(fn, L.total);
  const int max_tiles = ((I + A_ROWS - 1) / A_ROWS) * max_slots;
  int gbpr = (D + QK - 1) / QK, dbpr = (I + QK - 1) / QK;
  void* args[] = {(void*)&ph, (void*)&xq8, (void*)&gbpr, (void*)&hidden, (void*)&hq8, (void*)&dbpr,
                  (void*)&counters, (void*)&st};
  return launch_pdl(fn, dim3(std::min(max_tiles, cap[FMT])), L.total, s, args);
}

cudaError_t launch_moe_gateup(const PlanHdr* ph, int max_slots, int gate_fmt, int D, int I, const Q8Dev* xq8,
                              float* hidden, Q8Dev* hq8, int* counters, DevStatus* st, cudaStream_t s) {
  if (max_slots <= 0) return cudaSuccess;
  switch (gate_fmt) {
    case FMT_Q4K: return gateup_fmt<FMT_Q4K>(ph, max_slots, D, I, xq8, hidden, hq8, counters, st, s);
    case FMT_Q6K: return gateup_fmt<FMT_Q6K>(ph, max_slots, D, I, xq8, hidden, hq8, counters, st, s);
    case FMT_MXFP4: return gateup_fmt<FMT_MXFP4>(ph, max_slots, D, I, xq8, hidden, hq8, counters, st, s);
    case FMT_Q80: return gateup_fmt<FMT_Q80>(ph, max_slots, D, I, xq8, hidden, hq8, counters, st, s);
    default: return cudaErrorInvalidValue;
  }
}

template <int FMT>
static cudaError_t down_fmt(const PlanHdr* ph, int max_slots, int max_rows, int D, int I, int T, const Q8Dev* hq8,
                            const float* hidden, float* out, float* parts_out, DevStatus* st, cudaStream_t s) {
  const TileMap tm = tile_map(FMT, B_ROWS, I);
  // One buffer holding every slot's tile when that is small; otherwise two
  // buffers of up to 48 KB streaming windows of slots.
  const uint32_t all = (uint32_t)max_slots * tm.bytes;
  uint32_t buf = all <= 48 * 1024 ? all : std::max<uint32_t>(48 * 1024 / tm.bytes, 1) * tm.bytes;
  const uint32_t region = all <= 48 * 1024 ? buf : 2 * buf;
  int nb = std::min(dn_batch<FMT>(I), std::max(1, max_rows));
  const uint32_t total = region + dn_fixed_bytes<FMT>(I, T, max_slots, nb);
  if (total > 227 * 1024) return cudaErrorInvalidValue;
  const void* fn = reinterpret_cast<const void*>(moe_down_kernel<FMT>);
  cudaError_t e = ensure_smem(fn, total);
  if (e != cudaSuccess) return e;
  int dbpr = (I + QK - 1) / QK;
  uint32_t bufb = buf, reg = region;
  void* args[] = {(void*)&ph,   (void*)&hq8, (void*)&dbpr,      (void*)&hidden, (void*)&out, (void*)&parts_out,
                  (void*)&bufb, (void*)&reg, (void*)&max_slots, (void*)&nb,     (void*)&st};
  return launch_pdl(fn, dim3((D + B_ROWS - 1) / B_ROWS), total, s, args);
}

cudaError_t launch_moe_down(const PlanHdr* ph, int max_slots, int max_rows, int down_fmt_all, int D, int I, int T,
                            const Q8Dev* hq8, const float* hidden, float* out, float* parts_out, DevStatus* st,
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

size_t moe_counter_ints(int max_slots, int I) { return (size_t)max_slots * ((I + QK - 1) / QK); }

}  // namespace tg
