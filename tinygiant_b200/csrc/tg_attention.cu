// tg_attention.cu — the reference ABI's attention decode steps on the GPU
// (csrc/libtinygiant.c:723-815 tg_attention_decode, 939-983 tg_attention_v2,
// 985-1036 tg_attention_decode_q4), and the whole-layer entry built on them
// (1467-1507 tg_transformer_layer).
//
// One decode step for one token:
//   q, k, v = Wq x (+bq), Wk x (+bk), Wv x (+bv)   weights in any format, the
//             quantized ones against one Q8 copy of x, as tg_matmul;
//   per head, optionally, x <- rms_norm(x) * w (q with q_norm_w, k with
//             k_norm_w); then RoPE on q and k with row `pos` of the tables;
//   k, v appended to the KV cache at position kv_len;
//   per query head (KV head h / (n_heads / n_kv_heads)): scores over the
//             positions [start, kv_len] (start from the sliding window),
//             softmax with an optional per-head sink logit, weighted sum of v;
//   out = Wo attn (+bo).
//
// The caller's KV cache is host memory ([n_kv_heads][kv_max][head_dim]
// floats each for k and v).  The GPU keeps a mirror per cache pointer: the
// positions below kv_len that the mirror has not seen are uploaded, the new
// row is written on the device and back into the caller's arrays.  The
// mirror assumes the host cache changes only through these calls;
// tg_cuda_unregister(kv_ptr) or tg_cuda_registry_clear() drops it.
//
// Floating point: the reference's NEON lane sums and fused / unfused
// multiply-adds are not reproduced; results agree within the fp32 tolerance.
#include <algorithm>
#include <cmath>
#include <cstring>
#include <map>
#include <vector>

#include "../../include/tinygiant.h"
#include "tg_kernels.h"
#include "tg_runtime.h"

namespace tg {

constexpr int ATT_THREADS = 256;
constexpr int ATT_MAX_HD = 256;   // head_dim limit (one thread per element)

__device__ __forceinline__ float block_sum(float v, float* red) {
  const int lane = threadIdx.x & 31, w = threadIdx.x >> 5, nw = blockDim.x >> 5;
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  __syncthreads();
  if (lane == 0) red[w] = v;
  __syncthreads();
  float t = 0.f;
  for (int i = 0; i < nw; i++) t += red[i];
  return t;
}

__device__ __forceinline__ float block_max(float v, float* red) {
  const int lane = threadIdx.x & 31, w = threadIdx.x >> 5, nw = blockDim.x >> 5;
  for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
  __syncthreads();
  if (lane == 0) red[w] = v;
  __syncthreads();
  float t = -INFINITY;
  for (int i = 0; i < nw; i++) t = fmaxf(t, red[i]);
  return t;
}

// Block h: query head h < H, key head H + j, value head H + KH + j.  Norm and
// RoPE for q and k heads; k and v rows into the mirror at position kv_len and
// into knew / vnew (returned to the host).
__global__ void __launch_bounds__(ATT_THREADS) attn_prep_kernel(float* q, float* k, const float* v, const float* qnw,
                                                                const float* knw, float eps, const float* cosr,
                                                                const float* sinr, int H, int KH, int hd,
                                                                float* kv_k, float* kv_v, int kv_len, int kv_max,
                                                                float* knew, float* vnew) {
  __shared__ float xs[ATT_MAX_HD];
  __shared__ float red[ATT_THREADS / 32];
  const int h = blockIdx.x, t = threadIdx.x, half = hd / 2;
  if (h >= H + KH) {   // value head: copy only
    const int j = h - H - KH;
    for (int d = t; d < hd; d += blockDim.x) {
      const float x = v[j * hd + d];
      kv_v[((size_t)j * kv_max + kv_len) * hd + d] = x;
      vnew[j * hd + d] = x;
    }
    return;
  }
  const bool isq = h < H;
  float* x = isq ? q + (size_t)h * hd : k + (size_t)(h - H) * hd;
  const float* nw = isq ? qnw : knw;
  for (int d = t; d < hd; d += blockDim.x) xs[d] = x[d];
  __syncthreads();
  if (nw) {
    float ss = 0.f;
    for (int d = t; d < hd; d += blockDim.x) ss += xs[d] * xs[d];
    ss = block_sum(ss, red);
    const float scale = 1.f / sqrtf(ss / (float)hd + eps);
    __syncthreads();
    for (int d = t; d < hd; d += blockDim.x) xs[d] = xs[d] * scale * nw[d];
    __syncthreads();
  }
  for (int i = t; i < half; i += blockDim.x) {
    const float x1 = xs[i], x2 = xs[half + i], c = cosr[i], s = sinr[i];
    const float y1 = x1 * c - x2 * s, y2 = x2 * c + x1 * s;
    xs[i] = y1;
    xs[half + i] = y2;
  }
  __syncthreads();
  for (int d = t; d < hd; d += blockDim.x) {
    x[d] = xs[d];
    if (!isq) {
      const int j = h - H;
      kv_k[((size_t)j * kv_max + kv_len) * hd + d] = xs[d];
      knew[j * hd + d] = xs[d];
    }
  }
}

// Block (h, sp): query head h against KV head h / gqa over its share of the
// positions [start, seq_len) (split sp of nsp, `chunk` positions each):
// scores, their local maximum pm, the sum ps of exp(score - pm) and the
// unnormalised sum pacc[d] of exp(score - pm) v[d].  A thread per score
// (float4 rows when head_dim % 4 == 0; scores in sc[h][.], global scratch of
// kv_max per head); for the weighted sum, warp w takes positions w, w + nw,
// ..., its lanes the dimensions, and the warps' partial sums add up in
// shared memory.
__global__ void __launch_bounds__(ATT_THREADS) attn_split_kernel(const float* q, const float* kv_k, const float* kv_v,
                                                                 int kv_max, int hd, int gqa, int start, int seq_len,
                                                                 int chunk, float inv_sqrt, float* sc, float* pm,
                                                                 float* ps, float* pacc) {
  __shared__ __align__(16) float qs[ATT_MAX_HD];
  __shared__ float red[ATT_THREADS / 32];
  __shared__ float part[ATT_THREADS / 32][ATT_MAX_HD];
  const int h = blockIdx.x, sp = blockIdx.y, nsp = gridDim.y;
  const int t = threadIdx.x, lane = t & 31, w = t >> 5, nw = blockDim.x >> 5;
  const int kvh = h / gqa, p0 = start + sp * chunk, n = min(chunk, seq_len - p0);
  const float* kc = kv_k + ((size_t)kvh * kv_max + p0) * hd;
  const float* vc = kv_v + ((size_t)kvh * kv_max + p0) * hd;
  float* s = sc + (size_t)h * kv_max + (p0 - start);
  for (int d = t; d < hd; d += blockDim.x) qs[d] = q[(size_t)h * hd + d];
  __syncthreads();
  float m = -INFINITY;
  if ((hd & 3) == 0) {
    const float4* q4 = reinterpret_cast<const float4*>(qs);
    for (int i = t; i < n; i += blockDim.x) {
      const float4* kt = reinterpret_cast<const float4*>(kc + (size_t)i * hd);
      float d0 = 0.f, d1 = 0.f, d2 = 0.f, d3 = 0.f;   // independent chains: loads stay in flight
#pragma unroll 8
      for (int d4 = 0; d4 < hd / 4; d4++) {
        const float4 kv = __ldg(kt + d4), qv = q4[d4];
        d0 += qv.x * kv.x;
        d1 += qv.y * kv.y;
        d2 += qv.z * kv.z;
        d3 += qv.w * kv.w;
      }
      const float v = ((d0 + d1) + (d2 + d3)) * inv_sqrt;
      s[i] = v;
      m = fmaxf(m, v);
    }
  } else {
    for (int i = t; i < n; i += blockDim.x) {
      const float* kt = kc + (size_t)i * hd;
      float dot = 0.f;
      for (int d = 0; d < hd; d++) dot += qs[d] * kt[d];
      const float v = dot * inv_sqrt;
      s[i] = v;
      m = fmaxf(m, v);
    }
  }
  m = block_max(m, red);
  __syncthreads();   // every score is written
  float sp_sum = 0.f;
  for (int i = t; i < n; i += blockDim.x) {
    const float e = expf(s[i] - m);
    s[i] = e;
    sp_sum += e;
  }
  const float sum = block_sum(sp_sum, red);
  __syncthreads();   // every exponential is written
  constexpr int DJ = ATT_MAX_HD / 32;
  float acc[DJ];
#pragma unroll
  for (int jj = 0; jj < DJ; jj++) acc[jj] = 0.f;
#pragma unroll 4
  for (int i = w; i < n; i += nw) {
    const float e = s[i];
    const float* vt = vc + (size_t)i * hd;
#pragma unroll
    for (int jj = 0; jj < DJ; jj++) {
      const int d = lane + 32 * jj;
      if (d < hd) acc[jj] += e * __ldg(vt + d);
    }
  }
#pragma unroll
  for (int jj = 0; jj < DJ; jj++) {
    const int d = lane + 32 * jj;
    if (d < hd) part[w][d] = acc[jj];
  }
  __syncthreads();
  const size_t o = (size_t)h * nsp + sp;
  for (int d = t; d < hd; d += blockDim.x) {
    float v = 0.f;
    for (int ww = 0; ww < nw; ww++) v += part[ww][d];
    pacc[o * hd + d] = v;
  }
  if (t == 0) {
    pm[o] = m;
    ps[o] = sum;
  }
}

// Block h: the splits of head h merged, with the sink logit:
// out[d] = sum_s pacc_s[d] e^(pm_s - M) / (sum_s ps_s e^(pm_s - M) + e^(sink - M)),
// M the largest of the split maxima and the sink.
__global__ void attn_combine_kernel(const float* pm, const float* ps, const float* pacc, int nsp, int hd,
                                    const float* sinks, float* out) {
  const int h = blockIdx.x;
  float M = sinks ? sinks[h] : -INFINITY;
  for (int k = 0; k < nsp; k++) M = fmaxf(M, pm[(size_t)h * nsp + k]);
  float tot = sinks ? expf(sinks[h] - M) : 0.f;
  for (int k = 0; k < nsp; k++) tot += ps[(size_t)h * nsp + k] * expf(pm[(size_t)h * nsp + k] - M);
  const float inv = 1.f / tot;
  for (int d = threadIdx.x; d < hd; d += blockDim.x) {
    float v = 0.f;
    for (int k = 0; k < nsp; k++)
      v += pacc[((size_t)h * nsp + k) * hd + d] * expf(pm[(size_t)h * nsp + k] - M);
    out[(size_t)h * hd + d] = v * inv;
  }
}

// ---------------------------------------------------------------------
// KV-cache mirrors.

struct KvMirror {
  float* d = nullptr;
  size_t floats = 0;
  int valid = 0;   // positions [0, valid) of every head match the host
};
static std::map<const float*, KvMirror> g_kv;

static KvMirror* kv_mirror(const float* host, int KH, int kv_max, int hd, const char* what) {
  const size_t n = (size_t)KH * kv_max * hd;
  KvMirror& m = g_kv[host];
  if (m.d && m.floats != n) {
    cudaStreamSynchronize(stream());
    cudaFree(m.d);
    m = KvMirror{};
  }
  if (!m.d) {
    if (cudaMalloc(&m.d, n * sizeof(float)) != cudaSuccess) {
      g_kv.erase(host);
      set_host_error(100, "%s: cudaMalloc(KV mirror of %zu floats) failed", what, n);
      return nullptr;
    }
    m.floats = n;
    m.valid = 0;
  }
  return &m;
}

// Uploads host positions [m.valid, kv_len) of every head.
static bool kv_sync(KvMirror& m, const float* host, int KH, int kv_max, int hd, int kv_len, cudaStream_t s) {
  if (kv_len <= m.valid) return true;
  for (int h = 0; h < KH; h++) {
    const size_t o = ((size_t)h * kv_max + m.valid) * hd;
    if (cudaMemcpyAsync(m.d + o, host + o, sizeof(float) * (size_t)(kv_len - m.valid) * hd, cudaMemcpyHostToDevice,
                        s) != cudaSuccess)
      return false;
  }
  return true;
}

void kv_mirror_forget(const void* host) {
  auto it = g_kv.find(static_cast<const float*>(host));
  if (it == g_kv.end()) return;
  cudaStreamSynchronize(stream());
  cudaFree(it->second.d);
  g_kv.erase(it);
}

void kv_mirror_clear() {
  if (g_kv.empty()) return;
  cudaStreamSynchronize(stream());
  for (auto& kv : g_kv) cudaFree(kv.second.d);
  g_kv.clear();
}

// ---------------------------------------------------------------------
// The step.  Formats: FMT_* for quantized / F16 matrices, -1 for fp32.

// Device scratch of the step, grown on demand.
static struct {
  void* p = nullptr;
  size_t n = 0;
  bool reserve(size_t need, const char* what) {
    if (need <= n) return true;
    const size_t cap = (std::max(need, 2 * n) + 4095) & ~(size_t)4095;
    if (p) {
      cudaStreamSynchronize(stream());
      cudaFree(p);
    }
    p = nullptr;
    n = 0;
    if (cudaMalloc(&p, cap) != cudaSuccess) {
      set_host_error(100, "%s: cudaMalloc(%zu) failed", what, cap);
      return false;
    }
    n = cap;
    return true;
  }
} g_att;

static bool attention_step(const char* what, int fq, int fk, int fv, int fo, const void* wq, const void* wk,
                           const void* wv, const void* wo, const float* bq, const float* bk, const float* bv,
                           const float* bo, const float* qnw, const float* knw, const float* sinks, float* kv_k,
                           float* kv_v, int kv_len, int kv_max, int window, const float* rope_cos,
                           const float* rope_sin, const float* input, float* output, int D, int H, int KH, int hd,
                           int pos, float eps) {
  if (!input || !output || !wq || !wk || !wv || !wo || !kv_k || !kv_v || !rope_cos || !rope_sin) {
    set_host_error(3, "%s: null pointer argument", what);
    return false;
  }
  if (D <= 0 || H <= 0 || KH <= 0 || hd <= 0 || H % KH || hd % 2 || hd > ATT_MAX_HD || kv_max <= 0 || kv_len < 0 ||
      kv_len >= kv_max || pos < 0 || window < 0) {
    set_host_error(3, "%s: bad shape (embed %d, heads %d / %d, head_dim %d (even, <= %d), kv_len %d, kv_max %d, "
                      "pos %d, window %d)",
                   what, D, H, KH, hd, ATT_MAX_HD, kv_len, kv_max, pos, window);
    return false;
  }
  const int qd = H * hd, kd = KH * hd, half = hd / 2;
  auto cols_ok = [&](int f, int cols) {
    if (f == FMT_Q4K || f == FMT_Q6K) return cols % QK == 0;
    if (f == FMT_MXFP4 || f == FMT_Q80) return cols % 32 == 0;
    return true;
  };
  if (!cols_ok(fq, D) || !cols_ok(fk, D) || !cols_ok(fv, D) || !cols_ok(fo, qd)) {
    set_host_error(3, "%s: a projection's input width does not fit its format's block", what);
    return false;
  }
  if (!ensure_init()) return false;
  WDesc Wq, Wk, Wv, Wo;
  if (!lookup_matrix(wq, fq, qd, D, &Wq) || !lookup_matrix(wk, fk, kd, D, &Wk) || !lookup_matrix(wv, fv, kd, D, &Wv) ||
      !lookup_matrix(wo, fo, D, qd, &Wo))
    return false;
  const float *dbq = nullptr, *dbk = nullptr, *dbv = nullptr, *dbo = nullptr, *dqn = nullptr, *dkn = nullptr,
              *dsk = nullptr;
  if ((bq && !(dbq = lookup_vector(bq, qd))) || (bk && !(dbk = lookup_vector(bk, kd))) ||
      (bv && !(dbv = lookup_vector(bv, kd))) || (bo && !(dbo = lookup_vector(bo, D))))
    return false;
  if (qnw && (!(dqn = lookup_vector(qnw, hd)) || !knw || !(dkn = lookup_vector(knw, hd)))) {
    if (!knw) set_host_error(3, "%s: q_norm_w given without k_norm_w", what);
    return false;
  }
  if (sinks && !(dsk = lookup_vector(sinks, H))) return false;

  cudaStream_t s = stream();
  KvMirror* mk = kv_mirror(kv_k, KH, kv_max, hd, what);
  KvMirror* mv = mk ? kv_mirror(kv_v, KH, kv_max, hd, what) : nullptr;
  if (!mk || !mv) return false;
  if (!kv_sync(*mk, kv_k, KH, kv_max, hd, kv_len, s) || !kv_sync(*mv, kv_v, KH, kv_max, hd, kv_len, s)) {
    set_host_error(100, "%s: KV upload failed", what);
    return false;
  }

  // device scratch: x | rope rows | q | k | v | attn | out, knew, vnew | scores | Q8 of x / of attn
  const size_t fx = D, fr = 2 * (size_t)half, fq_ = qd, fk_ = kd, fa = qd, fo_ = D + 2 * (size_t)kd;
  const size_t fsc = (size_t)H * kv_max;
  constexpr int ATT_MAX_SPLIT = 8;   // position splits per head
  const size_t fpm = (size_t)H * ATT_MAX_SPLIT, fpa = fpm * hd;
  const int nbx = (D + QK - 1) / QK, nba = (qd + QK - 1) / QK;
  size_t off = 0;
  auto take = [&](size_t bytes) {
    const size_t o = off;
    off = (off + bytes + 255) & ~(size_t)255;
    return o;
  };
  // x and the two RoPE rows share one region (one upload)
  const size_t o_x = take(4 * (fx + fr)), o_q = take(4 * fq_), o_k = take(4 * fk_), o_v = take(4 * fk_),
               o_a = take(4 * fa), o_o = take(4 * fo_), o_s = take(4 * fsc), o_xq = take(sizeof(Q8Dev) * nbx),
               o_aq = take(sizeof(Q8Dev) * nba), o_pm = take(4 * fpm), o_ps = take(4 * fpm), o_pa = take(4 * fpa);
  float* hin = (float*)pinned_up(4 * (fx + fr));
  const float* hout = deliver_reserve(fo_);   // mapped: output and the new K / V rows
  if (!hin || !hout || !g_att.reserve(off, what)) return false;
  uint8_t* b = (uint8_t*)g_att.p;
  float *x = (float*)(b + o_x), *rr = x + fx, *q = (float*)(b + o_q), *k = (float*)(b + o_k), *v = (float*)(b + o_v),
        *att = (float*)(b + o_a), *ob = (float*)(b + o_o), *sc = (float*)(b + o_s);
  Q8Dev *xq = (Q8Dev*)(b + o_xq), *aq = (Q8Dev*)(b + o_aq);
  float *pm = (float*)(b + o_pm), *ps = (float*)(b + o_ps), *pa = (float*)(b + o_pa);

  memcpy(hin, input, 4 * fx);
  memcpy(hin + fx, rope_cos + (size_t)pos * half, 4 * (size_t)half);
  memcpy(hin + fx + half, rope_sin + (size_t)pos * half, 4 * (size_t)half);
  if (cudaMemcpyAsync(x, hin, 4 * (fx + fr), cudaMemcpyHostToDevice, s) != cudaSuccess) {
    set_host_error(100, "%s: input upload failed", what);
    return false;
  }

  auto proj = [&](const WDesc& W, int f, const Q8Dev* xq8, const float* xin, const float* bias, float* o) -> bool {
    if (f == -1) {
      launch_f32_matvec((const float*)W.main, xin, o, W.rows, W.cols, s);
      count_launches(1);
      return cudaGetLastError() == cudaSuccess;
    }
    count_launches(1);
    return launch_matvec(W, xq8, xin, bias, 1, o, status_ptr(), s) == cudaSuccess;
  };
  auto quantized = [](int f) { return f != -1 && f != FMT_F16; };
  const bool quant_in = quantized(fq) || quantized(fk) || quantized(fv);
  if (quant_in) {
    launch_quantize_rows(x, 1, D, D, xq, s);
    count_launches(1);
  }
  bool ok;
  if (fq != -1 && fk != -1 && fv != -1) {   // q, k, v in one launch
    const WDesc W3[3] = {Wq, Wk, Wv};
    const float* b3[3] = {dbq, dbk, dbv};
    float* o3[3] = {q, k, v};
    count_launches(1);
    ok = launch_matvec3(W3, b3, o3, xq, x, 1, status_ptr(), s) == cudaSuccess;
  } else {
    ok = proj(Wq, fq, xq, x, dbq, q) && proj(Wk, fk, xq, x, dbk, k) && proj(Wv, fv, xq, x, dbv, v);
  }
  if (ok) {
    attn_prep_kernel<<<H + 2 * KH, ATT_THREADS, 0, s>>>(q, k, v, dqn, dkn, eps, rr, rr + half, H, KH, hd, mk->d,
                                                         mv->d, kv_len, kv_max, ob + D, ob + D + kd);
    const int seq_len = kv_len + 1, start = (window > 0 && seq_len > window) ? seq_len - window : 0;
    // positions split over up to ATT_MAX_SPLIT CTAs per head, >= 128 each
    const int npos = seq_len - start;
    const int nsp = std::max(1, std::min(ATT_MAX_SPLIT, npos / 128));
    const int chunk = (npos + nsp - 1) / nsp;
    attn_split_kernel<<<dim3(H, nsp), ATT_THREADS, 0, s>>>(q, mk->d, mv->d, kv_max, hd, H / KH, start, seq_len,
                                                           chunk, 1.f / sqrtf((float)hd), sc, pm, ps, pa);
    attn_combine_kernel<<<H, 128, 0, s>>>(pm, ps, pa, nsp, hd, dsk, att);
    count_launches(3);
    ok = cudaGetLastError() == cudaSuccess;
  }
  if (ok && quantized(fo)) {
    launch_quantize_rows(att, 1, qd, qd, aq, s);
    count_launches(1);
  }
  ok = ok && proj(Wo, fo, aq, att, dbo, ob);
  if (ok) {
    deliver_begin();
    ok = deliver_async(ob, fo_, s, what);
  }
  if (!ok) {
    set_host_error(100, "%s: launch failed (%s)", what, cudaGetErrorString(cudaGetLastError()));
    cudaStreamSynchronize(s);
    return false;
  }
  if (!finish_delivered(what)) return false;
  mk->valid = mv->valid = std::max(mk->valid, kv_len + 1);
  memcpy(output, hout, 4 * (size_t)D);
  for (int h = 0; h < KH; h++) {
    memcpy(kv_k + ((size_t)h * kv_max + kv_len) * hd, hout + D + (size_t)h * hd, 4 * (size_t)hd);
    memcpy(kv_v + ((size_t)h * kv_max + kv_len) * hd, hout + D + kd + (size_t)h * hd, 4 * (size_t)hd);
  }
  return true;
}

}  // namespace tg

using namespace tg;

extern "C" {

void tg_attention_decode(const float* wq, const float* wk, const float* wv, const float* wo, const float* q_norm_w,
                         const float* k_norm_w, float* kv_k, float* kv_v, int kv_len, int kv_max,
                         const float* rope_cos, const float* rope_sin, const float* input, float* output,
                         int embed_dim, int n_heads, int n_kv_heads, int head_dim, int pos) {
  std::lock_guard<std::recursive_mutex> lk(ctx_mutex());
  if (!q_norm_w || !k_norm_w) {
    set_host_error(3, "tg_attention_decode: q_norm_w and k_norm_w are required");
    return;
  }
  attention_step("tg_attention_decode", -1, -1, -1, -1, wq, wk, wv, wo, nullptr, nullptr, nullptr, nullptr, q_norm_w,
                 k_norm_w, nullptr, kv_k, kv_v, kv_len, kv_max, 0, rope_cos, rope_sin, input, output, embed_dim,
                 n_heads, n_kv_heads, head_dim, pos, 1e-6f);
}

void tg_attention_decode_q4(const uint8_t* wq_q4, const uint8_t* wk_q4, const uint16_t* wv_f16, const uint8_t* wo_q4,
                            const float* q_norm_w, const float* k_norm_w, float* kv_k, float* kv_v, int kv_len,
                            int kv_max, const float* rope_cos, const float* rope_sin, const float* input,
                            float* output, int embed_dim, int n_heads, int n_kv_heads, int head_dim, int pos) {
  std::lock_guard<std::recursive_mutex> lk(ctx_mutex());
  if (!q_norm_w || !k_norm_w) {
    set_host_error(3, "tg_attention_decode_q4: q_norm_w and k_norm_w are required");
    return;
  }
  attention_step("tg_attention_decode_q4", FMT_Q4K, FMT_Q4K, FMT_F16, FMT_Q4K, wq_q4, wk_q4, wv_f16, wo_q4, nullptr,
                 nullptr, nullptr, nullptr, q_norm_w, k_norm_w, nullptr, kv_k, kv_v, kv_len, kv_max, 0, rope_cos,
                 rope_sin, input, output, embed_dim, n_heads, n_kv_heads, head_dim, pos, 1e-6f);
}

// Format codes other than Q4_K / Q6_K / MXFP4 / Q8_0 decode as F16, as the
// reference's dispatch does (libtinygiant.c:611-620).
void tg_attention_v2(int fmt_q, int fmt_k, int fmt_v, int fmt_o, const void* wq, const void* wk, const void* wv,
                     const void* wo, const float* bq, const float* bk, const float* bv, const float* bo,
                     const float* q_norm_w, const float* k_norm_w, const float* sinks, float* kv_k, float* kv_v,
                     int kv_len, int kv_max, int window, const float* rope_cos, const float* rope_sin,
                     const float* input, float* output, int embed_dim, int n_heads, int n_kv_heads, int head_dim,
                     int pos, float eps) {
  std::lock_guard<std::recursive_mutex> lk(ctx_mutex());
  auto f = [](int c) { return c == FMT_Q4K || c == FMT_Q6K || c == FMT_MXFP4 || c == FMT_Q80 ? c : FMT_F16; };
  attention_step("tg_attention_v2", f(fmt_q), f(fmt_k), f(fmt_v), f(fmt_o), wq, wk, wv, wo, bq, bk, bv, bo, q_norm_w,
                 k_norm_w, sinks, kv_k, kv_v, kv_len, kv_max, window, rope_cos, rope_sin, input, output, embed_dim,
                 n_heads, n_kv_heads, head_dim, pos, eps);
}

// One decoder layer for one token (libtinygiant.c:1467-1507): x += attention
// (rms_norm(x)), then x += the pre-routed experts' weighted outputs on
// rms_norm(x), through the GPU entries above and tg_expert_forward_mixed.
// x changes only if every step succeeded.
void tg_transformer_layer(const float* wq, const float* wk, const float* wv, const float* wo,
                          const float* attn_norm_w, const float* q_norm_w, const float* k_norm_w,
                          const float* ffn_norm_w, float* kv_k, float* kv_v, int kv_len, int kv_max,
                          const float* rope_cos, const float* rope_sin, const uint8_t** gate_ptrs,
                          const uint8_t** up_ptrs, const void** down_ptrs, const int* down_is_f16,
                          const float* expert_weights, int n_active, float* x, int embed_dim, int inter_dim,
                          int n_heads, int n_kv_heads, int head_dim, int pos) {
  std::lock_guard<std::recursive_mutex> lk(ctx_mutex());
  const char* what = "tg_transformer_layer";
  if (!x || embed_dim <= 0 || n_active < 0 || (n_active > 0 && (!gate_ptrs || !up_ptrs || !down_ptrs ||
                                                                 !down_is_f16 || !expert_weights))) {
    set_host_error(3, "%s: bad arguments", what);
    return;
  }
  const unsigned seq0 = host_error_seq();
  std::vector<float> xl(x, x + embed_dim), normed(embed_dim), part(embed_dim), moe(embed_dim, 0.f);
  tg_rms_norm(xl.data(), attn_norm_w, normed.data(), embed_dim, 1e-6f);
  if (host_error_seq() != seq0) return;
  tg_attention_decode(wq, wk, wv, wo, q_norm_w, k_norm_w, kv_k, kv_v, kv_len, kv_max, rope_cos, rope_sin,
                      normed.data(), part.data(), embed_dim, n_heads, n_kv_heads, head_dim, pos);
  if (host_error_seq() != seq0) return;
  for (int i = 0; i < embed_dim; i++) xl[i] += part[i];
  tg_rms_norm(xl.data(), ffn_norm_w, normed.data(), embed_dim, 1e-6f);
  if (host_error_seq() != seq0) return;
  for (int e = 0; e < n_active; e++) {
    tg_expert_forward_mixed(gate_ptrs[e], up_ptrs[e], down_ptrs[e], down_is_f16[e], normed.data(), moe.data(),
                            expert_weights[e], embed_dim, inter_dim);
    if (host_error_seq() != seq0) return;
  }
  for (int i = 0; i < embed_dim; i++) x[i] = xl[i] + moe[i];
}

}  // extern "C"
