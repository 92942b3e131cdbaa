// tg_pack.cpp — host packers that turn fp32 weights into Q4_K / Q6_K rows.
//
// The reference only consumes blocks that llama.cpp produced; it has no
// quantizer.  These packers fill the same block layouts that the reference
// decodes (Q4_K: csrc/libtinygiant.c:139-155, 210-222; Q6_K: 382-401) with a
// plain per-sub-block fit:
//   Q4_K : value ~= d*sc_j*q - dmin*m_j, q in [0,15]; per 32-value sub-block
//          lo = min(min(x), 0), scale_j = (max(x) - lo)/15, min_j = -lo; the
//          block's d = max(scale_j)/63 and dmin = max(min_j)/63 are stored as
//          fp16, and sc_j, m_j are 6-bit roundings against them.
//   Q6_K : value ~= d*sc_j*(q - 32), q-32 in [-32,31]; per 16-value
//          sub-block scale_j = v/-32 with v its largest-magnitude value;
//          d = max|scale_j|/127 (fp16), sc_j an int8 rounding.
// Rounding is to nearest even throughout, so the output is deterministic.
#include <cmath>
#include <cstdint>
#include <cstring>
#include <thread>
#include <vector>

#include "../../include/tinygiant.h"

namespace {

uint16_t f32_to_f16(float f) {
  uint32_t x;
  memcpy(&x, &f, 4);
  const uint32_t sign = (x >> 16) & 0x8000u, exp = (x >> 23) & 0xFFu;
  uint32_t man = x & 0x7FFFFFu;
  if (exp == 0xFF) return (uint16_t)(sign | 0x7C00u | (man ? 0x200u : 0u));
  const int e = (int)exp - 127 + 15;
  if (e >= 31) return (uint16_t)(sign | 0x7C00u);
  if (e <= 0) {
    if (e < -10) return (uint16_t)sign;
    man |= 0x800000u;
    const int shift = 14 - e;
    uint32_t h = man >> shift;
    const uint32_t rem = man & ((1u << shift) - 1), half = 1u << (shift - 1);
    if (rem > half || (rem == half && (h & 1u))) h++;
    return (uint16_t)(sign | h);
  }
  uint32_t h = ((uint32_t)e << 10) | (man >> 13);
  const uint32_t rem = man & 0x1FFFu;
  if (rem > 0x1000u || (rem == 0x1000u && (h & 1u))) h++;
  return (uint16_t)(sign | h);
}

float f16_to_f32(uint16_t h) {
  uint32_t s = (uint32_t)(h & 0x8000u) << 16, e = (h >> 10) & 0x1Fu, m = h & 0x3FFu, bits;
  if (e == 0) {
    if (m == 0) {
      bits = s;
    } else {
      int k = -1;
      do {
        m <<= 1;
        k++;
      } while (!(m & 0x400u));
      bits = s | ((uint32_t)(112 - k) << 23) | ((m & 0x3FFu) << 13);
    }
  } else if (e == 31) {
    bits = s | 0x7F800000u | (m << 13);
  } else {
    bits = s | ((e + 112u) << 23) | (m << 13);
  }
  float f;
  memcpy(&f, &bits, 4);
  return f;
}

int clampi(int v, int lo, int hi) { return v < lo ? lo : (v > hi ? hi : v); }

void pack_q4k_block(const float* x, uint8_t* out) {
  float scale[8], minv[8], max_scale = 0.f, max_min = 0.f;
  for (int j = 0; j < 8; j++) {
    float lo = x[32 * j], hi = x[32 * j];
    for (int i = 1; i < 32; i++) {
      lo = std::fmin(lo, x[32 * j + i]);
      hi = std::fmax(hi, x[32 * j + i]);
    }
    if (lo > 0.f) lo = 0.f;
    scale[j] = (hi - lo) / 15.f;
    minv[j] = -lo;
    max_scale = std::fmax(max_scale, scale[j]);
    max_min = std::fmax(max_min, minv[j]);
  }
  const uint16_t dh = f32_to_f16(max_scale / 63.f), mh = f32_to_f16(max_min / 63.f);
  const float d = f16_to_f32(dh), dmin = f16_to_f32(mh);
  int sc[8], mn[8];
  for (int j = 0; j < 8; j++) {
    sc[j] = d > 0.f ? clampi((int)std::nearbyint(scale[j] / d), 0, 63) : 0;
    mn[j] = dmin > 0.f ? clampi((int)std::nearbyint(minv[j] / dmin), 0, 63) : 0;
  }
  memset(out, 0, 144);
  memcpy(out, &dh, 2);
  memcpy(out + 2, &mh, 2);
  uint8_t* s = out + 4;
  for (int j = 0; j < 4; j++) {
    s[j] = (uint8_t)(sc[j] & 63);
    s[j + 4] = (uint8_t)(mn[j] & 63);
  }
  for (int j = 4; j < 8; j++) {
    s[j + 4] = (uint8_t)((sc[j] & 0xF) | ((mn[j] & 0xF) << 4));
    s[j - 4] |= (uint8_t)((sc[j] >> 4) << 6);
    s[j] |= (uint8_t)((mn[j] >> 4) << 6);
  }
  uint8_t q[256];
  for (int j = 0; j < 8; j++) {
    const float step = d * (float)sc[j], off = dmin * (float)mn[j];
    for (int i = 0; i < 32; i++) {
      const float v = x[32 * j + i];
      q[32 * j + i] = step > 0.f ? (uint8_t)clampi((int)std::nearbyint((v + off) / step), 0, 15) : 0;
    }
  }
  uint8_t* qs = out + 16;
  for (int g = 0; g < 4; g++)
    for (int i = 0; i < 32; i++) qs[32 * g + i] = (uint8_t)(q[64 * g + i] | (q[64 * g + 32 + i] << 4));
}

void pack_q6k_block(const float* x, uint8_t* out) {
  float scale[16], max_abs = 0.f;
  for (int j = 0; j < 16; j++) {
    float v = 0.f;
    for (int i = 0; i < 16; i++)
      if (std::fabs(x[16 * j + i]) > std::fabs(v)) v = x[16 * j + i];
    scale[j] = v / -32.f;
    max_abs = std::fmax(max_abs, std::fabs(scale[j]));
  }
  const uint16_t dh = f32_to_f16(max_abs / 127.f);
  const float d = f16_to_f32(dh);
  int sc[16];
  for (int j = 0; j < 16; j++) sc[j] = d > 0.f ? clampi((int)std::nearbyint(scale[j] / d), -127, 127) : 0;
  uint8_t q[256];
  for (int j = 0; j < 16; j++) {
    const float step = d * (float)sc[j];
    for (int i = 0; i < 16; i++) {
      const int l = step != 0.f ? clampi((int)std::nearbyint(x[16 * j + i] / step), -32, 31) : 0;
      q[16 * j + i] = (uint8_t)(l + 32);
    }
  }
  uint8_t* ql = out;
  uint8_t* qh = out + 128;
  for (int h = 0; h < 2; h++)
    for (int l = 0; l < 32; l++) {
      const int q1 = q[128 * h + l], q2 = q[128 * h + l + 32], q3 = q[128 * h + l + 64], q4 = q[128 * h + l + 96];
      ql[64 * h + l] = (uint8_t)((q1 & 15) | ((q3 & 15) << 4));
      ql[64 * h + l + 32] = (uint8_t)((q2 & 15) | ((q4 & 15) << 4));
      qh[32 * h + l] = (uint8_t)((q1 >> 4) | ((q2 >> 4) << 2) | ((q3 >> 4) << 4) | ((q4 >> 4) << 6));
    }
  for (int j = 0; j < 16; j++) out[192 + j] = (uint8_t)(int8_t)sc[j];
  memcpy(out + 208, &dh, 2);
}

template <typename F>
void pack_rows(const float* w, int rows, int cols, uint8_t* out, int block_bytes, F fn) {
  const int bpr = cols / 256;
  const long nblk = (long)rows * bpr;
  unsigned nt = std::thread::hardware_concurrency();
  if (nt == 0) nt = 1;
  if (nblk < 4096) nt = 1;
  std::vector<std::thread> th;
  for (unsigned t = 0; t < nt; t++)
    th.emplace_back([=] {
      for (long b = t; b < nblk; b += nt) fn(w + b * 256, out + b * block_bytes);
    });
  for (auto& t : th) t.join();
}

}  // namespace

extern "C" {

void tg_pack_q4k(const float* w, int rows, int cols, uint8_t* out) {
  if (rows <= 0 || cols <= 0 || cols % 256) return;
  pack_rows(w, rows, cols, out, 144, pack_q4k_block);
}

void tg_pack_q6k(const float* w, int rows, int cols, uint8_t* out) {
  if (rows <= 0 || cols <= 0 || cols % 256) return;
  pack_rows(w, rows, cols, out, 210, pack_q6k_block);
}

}  // extern "C"
