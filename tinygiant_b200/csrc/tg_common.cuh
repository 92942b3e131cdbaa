// tg_common.cuh — shared device definitions for the B200 MoE expert path.
//
// Block formats are TinyGiant's (csrc/libtinygiant.c:22-24, 159-166, 511-514,
// 574, 594): Q4_K 144 B / 256 values, Q6_K 210 B / 256, MXFP4 17 B / 32,
// Q8_0 34 B / 32, F16 2 B / value.  In HBM every quantized matrix is stored
// re-laid out so each row is one 16-byte-aligned window (WDesc below); the
// values are unchanged.
#pragma once
#include <mutex>
#include <cstdint>
#include <cuda_runtime.h>

namespace tg {

constexpr int QK = 256;
constexpr int Q4K_BYTES = 144;
constexpr int Q6K_BYTES = 210;
constexpr int MXFP4_BYTES = 17;
constexpr int Q80_BYTES = 34;

enum Fmt : int { FMT_Q4K = 0, FMT_F16 = 1, FMT_Q6K = 2, FMT_MXFP4 = 3, FMT_Q80 = 4 };
enum Act : int { ACT_SILU = 0, ACT_GPTOSS = 1 };

// How a Q4_K row dot associates its float terms (csrc/libtinygiant.c):
//   X1  : dot_q4k_q8     (223-272) — block_sum += T_lo; block_sum += T_hi;
//   X4  : dot_q4k_q8_x4  (276-337) — block_sum += ((T_lo + dsh*ih) - dmh*bh)
// Q6_K, MXFP4 and Q8_0 associate identically in both kernels.
enum AssocRule : int {
  ASSOC_MOE = 0,   // moe_phase_a/b: a group of 4 active rows uses x4 unless it holds 1 row (1298-1316, 1362-1378)
  ASSOC_ROWS = 1,  // q4k_rows/q6k_rows: x4 for every group whenever k > 1 (1136-1180)
  ASSOC_X1 = 2,    // tg_expert_forward*, matmul: x1 always
};

// Q8 activation block in HBM: the reference's q8_block fields (scale, sum,
// bsums[8], qs[256]; 159-164), reordered so qs starts 16-byte aligned.
struct __align__(16) Q8Dev {
  int8_t qs[QK];
  float scale;
  int32_t sum;
  int32_t bsums[8];
  int32_t pad[6];
};
static_assert(sizeof(Q8Dev) == 320, "Q8Dev layout");

// A weight matrix resident in HBM.  Rows are stored one after the other,
// rs bytes apart, each row holding all of its own data (one contiguous
// window per row, so a row moves in one bulk copy):
//   Q4_K : the raw 144-byte blocks                          rs = 144 bpr
//   Q6_K : ql|qh 192 B/block, then int8 scales 16 B/block, then fp16 d
//          2 B/block, zero-padded to 16 bytes                rs = round16(210 bpr)
//   MXFP4: codes 16 B/block, then e8m0 1 B/block, padded     rs = round16(17 nsub)
//   Q8_0 : int8 32 B/block, then fp16 d 2 B/block, padded    rs = round16(34 nsub)
//   F16  : raw fp16 values                                   rs = 2 cols
// main, aux1 and aux2 point at row 0's blocks, scales (Q6_K int8 scales,
// MXFP4 e8m0) and fp16 d values (Q6_K, Q8_0); row r's are rs * r further on.
struct WDesc {
  const uint8_t* main;
  const uint8_t* aux1;
  const uint8_t* aux2;
  int fmt;
  int rows;
  int cols;
  int rs;
};

// Row stride and the offsets of aux1 / aux2 inside a row (-1: none).
struct RowLayout {
  int rs, a1, a2;
};

__host__ __device__ __forceinline__ RowLayout row_layout(int fmt, int cols) {
  const int bpr = cols / QK, nsub = cols / 32;
  switch (fmt) {
    case FMT_Q4K: return {bpr * Q4K_BYTES, -1, -1};
    case FMT_Q6K: return {(bpr * Q6K_BYTES + 15) & ~15, bpr * 192, bpr * 208};
    case FMT_MXFP4: return {(nsub * MXFP4_BYTES + 15) & ~15, nsub * 16, -1};
    case FMT_Q80: return {(nsub * Q80_BYTES + 15) & ~15, -1, nsub * 32};
    default: return {cols * 2, -1, -1};
  }
}

// ---------------------------------------------------------------------
// Exact scalar decoders.

// IEEE half -> float exactly as the reference's f16_to_f32 (128-137),
// including its exponent-31 path, which wraps (255 + 112) << 23 in uint32.
__device__ __forceinline__ float f16_bits_to_f32(uint32_t h) {
  uint32_t s = (h & 0x8000u) << 16, e = (h >> 10) & 0x1Fu, m = h & 0x3FFu;
  if (e == 0) {
    if (m == 0) return __uint_as_float(s);
    int lz = __clz(m) - 21;  // leading zeros within the 11-bit field (m < 0x400)
    m = (m << lz) & 0x3FFu;
    e = 1u - (uint32_t)lz;   // wraps like the reference's uint32 e--
  } else if (e == 31) {
    e = 255;
  }
  return __uint_as_float(s | ((e + 112u) << 23) | (m << 13));
}

// e8m0 -> 2^(e-128) (516-519).
__device__ __forceinline__ float e8m0_half(uint32_t e) {
  uint32_t bits = e < 2 ? (0x00200000u << e) : ((e - 1u) << 23);
  return __uint_as_float(bits);
}

// 6-bit scale/min pair j of a Q4_K block (146-155).  s0/s1/s2 are the 12
// scale bytes as three little-endian words.
__device__ __forceinline__ void q4k_scale_min(int j, uint32_t s0, uint32_t s1, uint32_t s2, int& sc, int& m) {
  auto byte = [&](int i) -> int {
    uint32_t w = i < 4 ? s0 : (i < 8 ? s1 : s2);
    return (int)((w >> (8 * (i & 3))) & 0xFFu);
  };
  if (j < 4) {
    sc = byte(j) & 63;
    m = byte(j + 4) & 63;
  } else {
    sc = (byte(j + 4) & 0xF) | ((byte(j - 4) >> 6) << 4);
    m = (byte(j + 4) >> 4) | ((byte(j) >> 6) << 4);
  }
}

// Round-to-nearest-even float ops that nvcc never contracts into an FMA.
__device__ __forceinline__ float fmul(float a, float b) { return __fmul_rn(a, b); }
__device__ __forceinline__ float fadd(float a, float b) { return __fadd_rn(a, b); }
__device__ __forceinline__ float fsub(float a, float b) { return __fsub_rn(a, b); }

// Activation (1248-1257).
__device__ __forceinline__ float act_fn(int act, float g, float u) {
  if (act == ACT_GPTOSS) {
    if (g > 7.f) g = 7.f;
    if (u > 7.f) u = 7.f;
    else if (u < -7.f) u = -7.f;
    float den = fadd(1.f, expf(fmul(-1.702f, g)));
    return fmul(__fdiv_rn(g, den), fadd(u, 1.f));
  }
  float den = fadd(1.f, expf(-g));
  return fmul(__fdiv_rn(g, den), u);
}

// Raises a kernel's dynamic shared-memory limit only when a launch needs more
// than was set before, so launches during CUDA-graph capture make no
// attribute calls after the first (uncaptured) use.
inline cudaError_t ensure_smem(const void* fn, size_t bytes) {
  struct Entry { const void* fn; size_t bytes; };
  static Entry table[32];
  static int n = 0;
  static std::mutex mu;   // entry points that run without the runtime lock reach this too
  std::lock_guard<std::mutex> lk(mu);
  for (int i = 0; i < n; i++)
    if (table[i].fn == fn) {
      if (table[i].bytes >= bytes) return cudaSuccess;
      cudaError_t e = cudaFuncSetAttribute(fn, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)bytes);
      if (e == cudaSuccess) table[i].bytes = bytes;
      return e;
    }
  cudaError_t e = cudaFuncSetAttribute(fn, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)bytes);
  if (e == cudaSuccess && n < 32) table[n++] = Entry{fn, bytes};
  return e;
}

// ---------------------------------------------------------------------
// Device error status.  Kernels never trap: on a bad descriptor or a wait
// that runs out they record a code here and return; the host reads it after
// the stream synchronises.
enum ErrCode : int {
  ERR_NONE = 0,
  ERR_BAD_FORMAT = 1,
  ERR_WAIT_TIMEOUT = 2,
  ERR_BAD_PLAN = 3,
};

struct DevStatus {
  int code;
  int where;
  int a, b;
};

__device__ __forceinline__ void set_error(DevStatus* st, int code, int where, int a = 0, int b = 0) {
  if (st && atomicCAS(&st->code, 0, code) == 0) {
    st->where = where;
    st->a = a;
    st->b = b;
  }
}

}  // namespace tg
