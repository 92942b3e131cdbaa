// tg_runtime.cu — host side of libtinygiant.so: device context, the
// host-pointer -> HBM weight registry, per-call staging, and the C ABI.
//
// The reference engine passes host pointers (numpy arrays, mmap views of the
// expert files) to every call and reads the results right after.  Here each
// weight matrix is uploaded once, repacked into the aligned HBM layout, and
// found again by its host address; per call only activations cross PCIe:
// one host->device copy of [plan | inputs | output], the kernels, one
// device->host copy of the output.
#include <sys/mman.h>
#include <unistd.h>

#include <algorithm>
#include <atomic>
#include <climits>
#include <chrono>
#include <cstdarg>
#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <map>
#include <mutex>
#include <string>
#include <tuple>
#include <vector>

#include "../../include/tinygiant.h"
#include "tg_kernels.h"
#include "tg_moe.h"
#include "tg_runtime.h"

namespace tg {

// ---------------------------------------------------------------------
// Errors.

static std::mutex g_err_mu;
static int g_err_code = 0;
static unsigned g_err_seq = 0;   // errors recorded so far
static std::string g_err_msg;

unsigned host_error_seq() {
  std::lock_guard<std::mutex> lk(g_err_mu);
  return g_err_seq;
}

void set_host_error(int code, const char* fmt, ...) {
  char buf[512];
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(buf, sizeof buf, fmt, ap);
  va_end(ap);
  {
    std::lock_guard<std::mutex> lk(g_err_mu);
    g_err_code = code;
    g_err_msg = buf;
    g_err_seq++;
  }
  fprintf(stderr, "libtinygiant(cuda): %s\n", buf);
  if (getenv("TG_CUDA_ABORT_ON_ERROR")) abort();
}

static bool cuda_ok(cudaError_t e, const char* what) {
  if (e == cudaSuccess) return true;
  set_host_error(100 + (int)e, "%s: %s", what, cudaGetErrorString(e));
  return false;
}

std::atomic<uint64_t> g_launches{0};

// ---------------------------------------------------------------------
// Growable device / pinned buffers.

struct DevBuf {
  void* p = nullptr;
  size_t n = 0;
  bool reserve(size_t need) {
    if (need <= n) return true;
    size_t cap = std::max(need, n * 2);
    cap = (cap + 4095) & ~(size_t)4095;
    if (p) cudaFree(p);
    p = nullptr;
    n = 0;
    if (!cuda_ok(cudaMalloc(&p, cap), "cudaMalloc(scratch)")) return false;
    n = cap;
    return true;
  }
};

struct PinBuf {
  void* p = nullptr;
  size_t n = 0;
  bool reserve(size_t need) {
    if (need <= n) return true;
    size_t cap = std::max(need, n * 2);
    cap = (cap + 4095) & ~(size_t)4095;
    if (p) cudaFreeHost(p);
    p = nullptr;
    n = 0;
    if (!cuda_ok(cudaMallocHost(&p, cap), "cudaMallocHost(staging)")) return false;
    n = cap;
    return true;
  }
};

// Pinned host memory mapped into the device's address space.
struct MapBuf {
  void* h = nullptr;
  void* d = nullptr;
  size_t n = 0;
  bool reserve(size_t need) {
    if (need <= n) return true;
    size_t cap = std::max(need, n * 2);
    cap = (cap + 4095) & ~(size_t)4095;
    if (h) cudaFreeHost(h);
    h = d = nullptr;
    n = 0;
    if (!cuda_ok(cudaHostAlloc(&h, cap, cudaHostAllocMapped | cudaHostAllocPortable), "cudaHostAlloc(result)") ||
        !cuda_ok(cudaHostGetDevicePointer(&d, h, 0), "cudaHostGetDevicePointer(result)"))
      return false;
    memset(h, 0, cap);
    n = cap;
    return true;
  }
};

// The head of the mapped result block: the request number the host set
// before launching, echoed by the device after the result and the status
// record are written.
struct RetHdr {
  unsigned int req;
  unsigned int done;
  unsigned int pad[2];
  DevStatus st;
};
constexpr size_t RET_DATA = 64;   // the floats start here (16-byte aligned)

// ---------------------------------------------------------------------
// Context.

struct Ctx {
  std::recursive_mutex mu;
  bool inited = false;
  bool init_failed = false;
  int device = -1;
  cudaStream_t own_stream = nullptr;
  cudaStream_t user_stream = nullptr;
  bool user_stream_set = false;
  DevStatus* d_status = nullptr;
  DevStatus* h_status = nullptr;  // pinned
  unsigned int* d_arrived = nullptr;   // deliver_kernel's CTA count (zero between launches)
  DevBuf d_stage, d_xq8, d_hidden, d_hq8, d_tmp, d_counters, d_parts;
  PinBuf h_up, h_down;
  MapBuf h_ret;                   // deliver_async's result block
  MapBuf h_in;                    // fetch_async's input block
  unsigned int ret_seq = 0;
  int threads = 1;
};

static Ctx g;

cudaStream_t stream() { return g.user_stream_set ? g.user_stream : g.own_stream; }

std::recursive_mutex& ctx_mutex() { return g.mu; }

// Arrival counters owned by resident layers, cleared with the library's own
// after a device-side error.
static std::vector<std::pair<void*, size_t>> g_counter_bufs;
void register_counters(void* p, size_t n) { g_counter_bufs.push_back({p, n}); }
void unregister_counters(void* p) {
  for (size_t i = 0; i < g_counter_bufs.size(); i++)
    if (g_counter_bufs[i].first == p) {
      g_counter_bufs.erase(g_counter_bufs.begin() + i);
      return;
    }
}
DevStatus* status_ptr() { return g.d_status; }
void count_launches(int n) { g_launches += n; }
void* pinned_up(size_t n) { return g.h_up.reserve(n) ? g.h_up.p : nullptr; }
void* pinned_down(size_t n) { return g.h_down.reserve(n) ? g.h_down.p : nullptr; }

// The gate/up kernel's per-(slot, 256-block) arrival counters must start at
// zero; they reset themselves, and are cleared again after a device error.
bool reserve_counters(size_t n_ints) {
  const size_t old = g.d_counters.n;
  if (!g.d_counters.reserve(sizeof(int) * n_ints)) return false;
  if (g.d_counters.n != old) return cuda_ok(cudaMemset(g.d_counters.p, 0, g.d_counters.n), "cudaMemset(counters)");
  return true;
}

bool ensure_init() {
  if (g.inited) return true;
  if (g.init_failed) {
    set_host_error(1, "no usable CUDA device (initialisation failed earlier)");
    return false;
  }
  int n = 0;
  cudaError_t e = cudaGetDeviceCount(&n);
  if (e != cudaSuccess || n == 0) {
    g.init_failed = true;
    set_host_error(1, "no CUDA device available (%s); this library has no CPU path",
                   e == cudaSuccess ? "0 devices" : cudaGetErrorString(e));
    return false;
  }
  if (g.device < 0) {
    int cur = 0;
    if (cudaGetDevice(&cur) != cudaSuccess) cur = 0;
    g.device = cur;
  }
  if (!cuda_ok(cudaSetDevice(g.device), "cudaSetDevice")) {
    g.init_failed = true;
    return false;
  }
  if (!cuda_ok(cudaStreamCreateWithFlags(&g.own_stream, cudaStreamNonBlocking), "cudaStreamCreate") ||
      !cuda_ok(cudaMalloc(&g.d_status, sizeof(DevStatus)), "cudaMalloc(status)") ||
      !cuda_ok(cudaMallocHost(&g.h_status, sizeof(DevStatus)), "cudaMallocHost(status)") ||
      !cuda_ok(cudaMemset(g.d_status, 0, sizeof(DevStatus)), "cudaMemset(status)") ||
      !cuda_ok(cudaMalloc(&g.d_arrived, sizeof(unsigned int)), "cudaMalloc(arrivals)") ||
      !cuda_ok(cudaMemset(g.d_arrived, 0, sizeof(unsigned int)), "cudaMemset(arrivals)")) {
    g.init_failed = true;
    return false;
  }
  register_counters(g.d_arrived, sizeof(unsigned int));   // cleared again after a device error
  g.inited = true;
  return true;
}

// Enqueues the copy of the device status record to its pinned host copy.
bool status_copy_async(cudaStream_t s, const char* what) {
  return cuda_ok(cudaMemcpyAsync(g.h_status, g.d_status, sizeof(DevStatus), cudaMemcpyDeviceToHost, s), what);
}

// Synchronises the stream, whose work ends with status_copy_async, and turns
// a device-side error record into a host error (resetting the record and
// every arrival counter).
bool finish_copied(const char* what) {
  cudaStream_t s = stream();
  if (!cuda_ok(cudaStreamSynchronize(s), what)) return false;
  if (g.h_status->code != 0) {
    DevStatus st = *g.h_status;
    cudaMemsetAsync(g.d_status, 0, sizeof(DevStatus), s);
    if (g.d_counters.p) cudaMemsetAsync(g.d_counters.p, 0, g.d_counters.n, s);
    for (auto& c : g_counter_bufs) cudaMemsetAsync(c.first, 0, c.second, s);
    cudaStreamSynchronize(s);
    g.h_status->code = 0;
    set_host_error(200 + st.code, "%s: device error %d at site %d (%d, %d)", what, st.code, st.where, st.a, st.b);
    return false;
  }
  return true;
}

// Synchronises the stream and turns a device-side error record into a host error.
bool finish(const char* what) {
  return status_copy_async(stream(), what) && finish_copied(what);
}

// ---------------------------------------------------------------------
// Results without a stream synchronisation: one CTA copies n floats and the
// status record into the mapped result block, then, after a system-scope
// fence, echoes the host's request number; the host spins on that word.

__global__ void deliver_kernel(const float* __restrict__ src, size_t n, const DevStatus* __restrict__ st,
                               RetHdr* hdr, float* out, unsigned int* arrived) {
  __shared__ unsigned int req;
  __shared__ bool last;
  if (threadIdx.x == 0) req = *reinterpret_cast<volatile unsigned int*>(&hdr->req);
  asm volatile("griddepcontrol.wait;" ::: "memory");   // src and st come from the preceding kernel
  const size_t n4 = n / 4, step = (size_t)gridDim.x * blockDim.x, i0 = (size_t)blockIdx.x * blockDim.x + threadIdx.x;
  for (size_t i = i0; i < n4; i += step)
    reinterpret_cast<float4*>(out)[i] = __ldcg(reinterpret_cast<const float4*>(src) + i);
  for (size_t i = n4 * 4 + i0; i < n; i += step) out[i] = __ldcg(src + i);
  // the last CTA to finish its share writes the status and the echo (one
  // CTA: no count)
  __syncthreads();
  if (threadIdx.x == 0) {
    if (gridDim.x == 1) {
      last = true;
    } else {
      __threadfence_system();
      last = atomicAdd(arrived, 1u) == gridDim.x - 1;
      if (last) *arrived = 0;
      __threadfence();
    }
  }
  __syncthreads();
  if (last && threadIdx.x == 0) {
    volatile DevStatus* hs = &hdr->st;
    hs->code = st->code;
    hs->where = st->where;
    hs->a = st->a;
    hs->b = st->b;
    __threadfence_system();
    *reinterpret_cast<volatile unsigned int*>(&hdr->done) = req;
  }
}

// Copies n floats from mapped pinned host memory, which the host wrote
// before the launch, into device memory (one CTA for a decode step's rows,
// more for large batches).  The loads skip any cached copy of the host lines
// (ld.global.cv).  It lets the next kernel launch at once; that kernel waits
// for this grid (griddepcontrol.wait) before it reads dst.
// Reads of mapped host memory cross PCIe (about a microsecond each): each
// thread keeps four in flight before it stores them.
__global__ void fetch_kernel(const float* __restrict__ src, size_t n, float* __restrict__ dst) {
  asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
  const size_t n4 = n / 4, step = (size_t)gridDim.x * blockDim.x, i0 = (size_t)blockIdx.x * blockDim.x + threadIdx.x;
  const float4* s4 = reinterpret_cast<const float4*>(src);
  float4* d4 = reinterpret_cast<float4*>(dst);
  for (size_t i = i0; i < n4; i += 4 * step) {
    float4 v[4];
#pragma unroll
    for (int k = 0; k < 4; k++)
      if (i + k * step < n4) v[k] = __ldcv(s4 + i + k * step);
#pragma unroll
    for (int k = 0; k < 4; k++)
      if (i + k * step < n4) d4[i + k * step] = v[k];
  }
  for (size_t i = n4 * 4 + i0; i < n; i += step) dst[i] = __ldcv(src + i);
}

// CTAs of the delivery copy: one up to 64 K floats (a decode step's rows),
// then one per 64 K floats, at most 32.
static unsigned copy_ctas(size_t n_floats) {
  return (unsigned)std::min<size_t>(32, std::max<size_t>(1, (n_floats + 65535) / 65536));
}
// CTAs of the fetch: one per 8 K floats (each thread then reads at most four
// float4 at once), at most 64.
static unsigned fetch_ctas(size_t n_floats) {
  return (unsigned)std::min<size_t>(64, std::max<size_t>(1, (n_floats + 8191) / 8192));
}

float* fetch_reserve(size_t n_floats) {
  return g.h_in.reserve(sizeof(float) * n_floats) ? static_cast<float*>(g.h_in.h) : nullptr;
}

bool fetch_async(float* d_dst, size_t n_floats, cudaStream_t s, const char* what) {
  if (!g.h_in.reserve(sizeof(float) * n_floats)) return false;
  fetch_kernel<<<fetch_ctas(n_floats), 512, 0, s>>>(static_cast<const float*>(g.h_in.d), n_floats, d_dst);
  count_launches(1);
  return cuda_ok(cudaGetLastError(), what);
}

float* deliver_reserve(size_t n_floats) {
  if (!g.h_ret.reserve(RET_DATA + sizeof(float) * n_floats)) return nullptr;
  return reinterpret_cast<float*>(static_cast<uint8_t*>(g.h_ret.h) + RET_DATA);
}

bool deliver_async(const float* d_src, size_t n_floats, cudaStream_t s, const char* what) {
  if (!g.h_ret.reserve(RET_DATA + sizeof(float) * n_floats)) return false;
  RetHdr* hdr = static_cast<RetHdr*>(g.h_ret.d);
  float* out = reinterpret_cast<float*>(static_cast<uint8_t*>(g.h_ret.d) + RET_DATA);
  // launched as a programmatic dependent: it is scheduled while the
  // preceding kernel runs and waits for that grid before reading its output
  const DevStatus* st = g.d_status;
  unsigned int* arrived = g.d_arrived;
  void* args[] = {(void*)&d_src, (void*)&n_floats, (void*)&st, (void*)&hdr, (void*)&out, (void*)&arrived};
  cudaLaunchConfig_t cfg{};
  cfg.gridDim = dim3(copy_ctas(n_floats));
  cfg.blockDim = dim3(512);
  cfg.stream = s;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  const cudaError_t e = cudaLaunchKernelExC(&cfg, (const void*)deliver_kernel, args);
  count_launches(1);
  return cuda_ok(e, what);
}

// Sets the next request number; call before launching the work that ends
// with deliver_async.
void deliver_begin() {
  RetHdr* hdr = static_cast<RetHdr*>(g.h_ret.h);
  __atomic_store_n(&hdr->req, ++g.ret_seq, __ATOMIC_RELEASE);
}

// Waits (spinning, bounded) until the device has echoed the request, then
// turns a device-side error record into a host error as finish_copied does.
// If the echo does not come (a failed launch or kernel), the stream is
// synchronised to report the CUDA error.
bool finish_delivered(const char* what) {
  RetHdr* hdr = static_cast<RetHdr*>(g.h_ret.h);
  const unsigned int want = g.ret_seq;
  const auto t0 = std::chrono::steady_clock::now();
  int spins = 0;
  while (__atomic_load_n(&hdr->done, __ATOMIC_ACQUIRE) != want) {
    if (++spins % 4096 == 0 && std::chrono::steady_clock::now() - t0 > std::chrono::seconds(10)) {
      cudaStreamSynchronize(stream());
      if (__atomic_load_n(&hdr->done, __ATOMIC_ACQUIRE) == want) break;
      const cudaError_t e = cudaGetLastError();
      set_host_error(100 + (int)e, "%s: the result was not delivered (%s)", what, cudaGetErrorString(e));
      return false;
    }
  }
  if (hdr->st.code != 0) {
    const DevStatus st{hdr->st.code, hdr->st.where, hdr->st.a, hdr->st.b};
    cudaStream_t s = stream();
    cudaMemsetAsync(g.d_status, 0, sizeof(DevStatus), s);
    if (g.d_counters.p) cudaMemsetAsync(g.d_counters.p, 0, g.d_counters.n, s);
    for (auto& c : g_counter_bufs) cudaMemsetAsync(c.first, 0, c.second, s);
    cudaStreamSynchronize(s);
    hdr->st.code = 0;
    set_host_error(200 + st.code, "%s: device error %d at site %d (%d, %d)", what, st.code, st.where, st.a, st.b);
    return false;
  }
  return true;
}

// ---------------------------------------------------------------------
// Weight registry.

static size_t align_up(size_t x, size_t a) { return (x + a - 1) / a * a; }

size_t host_row_bytes(int fmt, int ncols) {
  switch (fmt) {
    case FMT_Q4K: return (size_t)(ncols / QK) * Q4K_BYTES;
    case FMT_Q6K: return (size_t)(ncols / QK) * Q6K_BYTES;
    case FMT_MXFP4: return (size_t)(ncols / 32) * MXFP4_BYTES;
    case FMT_Q80: return (size_t)(ncols / 32) * Q80_BYTES;
    default: return (size_t)ncols * 2;
  }
}

// Bump allocator over large cudaMalloc chunks; every sub-allocation is
// 256-byte aligned and padded so bulk copies may round a tile up to 16 bytes.
struct Slab {
  std::vector<std::pair<uint8_t*, size_t>> chunks;
  size_t used = 0, cap = 0, total = 0;
  uint8_t* cur = nullptr;
  uint8_t* alloc(size_t n) {
    n = align_up(n + 64, 256);
    if (!cur || used + n > cap) {
      size_t sz = std::max(n, (size_t)256 << 20);
      uint8_t* p = nullptr;
      if (!cuda_ok(cudaMalloc(&p, sz), "cudaMalloc(weights)")) return nullptr;
      chunks.push_back({p, sz});
      cur = p;
      used = 0;
      cap = sz;
      total += sz;
    }
    uint8_t* r = cur + used;
    used += n;
    return r;
  }
  void clear() {
    for (auto& c : chunks) cudaFree(c.first);
    chunks.clear();
    cur = nullptr;
    used = cap = total = 0;
  }
};

// Content fingerprint of an unregistered host matrix: four lanes of 64-bit
// xor-rotate-multiply over 32-byte strides, then the tail.  Each lane's step
// is a bijection of the lane state for a fixed input word, so a change to any
// one word always changes the result; the reference reuses host buffers for
// different experts (a pread buffer refilled with another expert's bytes), so
// every byte counts, not a sample of them.  ~14 GB/s on one host core.
static inline uint64_t rotl64(uint64_t x, int r) { return (x << r) | (x >> (64 - r)); }
static uint64_t content_hash(const uint8_t* p, size_t n) {
  constexpr uint64_t K = 0x9E3779B97F4A7C15ull;
  uint64_t h0 = n, h1 = n ^ 0x243F6A8885A308D3ull, h2 = n ^ 0x13198A2E03707344ull, h3 = n ^ 0xA4093822299F31D0ull;
  size_t i = 0;
  for (; i + 32 <= n; i += 32) {
    uint64_t w[4];
    memcpy(w, p + i, 32);
    h0 = rotl64(h0 ^ w[0], 29) * K;
    h1 = rotl64(h1 ^ w[1], 29) * K;
    h2 = rotl64(h2 ^ w[2], 29) * K;
    h3 = rotl64(h3 ^ w[3], 29) * K;
  }
  for (; i < n; i++) h0 = rotl64(h0 ^ p[i], 29) * K;
  return rotl64(h0, 1) ^ rotl64(h1, 17) ^ rotl64(h2, 33) ^ rotl64(h3, 49);
}

// The check policy for unregistered host matrices (tg_cuda_set_weight_check):
// 2 every byte fingerprinted per call (default), 1 a 96-byte sample (first,
// middle and last 32 bytes), 0 none.
static int g_check = 2;

static uint64_t sample_hash(const uint8_t* h, size_t n) {
  uint8_t buf[96] = {};
  const size_t offs[3] = {0, n / 2, n > 32 ? n - 32 : 0};
  for (int i = 0; i < 3; i++) memcpy(buf + 32 * i, h + offs[i], std::min<size_t>(32, n - std::min(n, offs[i])));
  return content_hash(buf, sizeof buf) ^ n;
}

static uint64_t check_hash(const uint8_t* h, size_t n) {
  return g_check == 2 ? content_hash(h, n) : g_check == 1 ? sample_hash(h, n) : 0;
}

struct Entry {
  WDesc w;
  size_t raw_bytes;
  size_t dev_bytes;   // the device allocation's size
  uint64_t hash;      // check_hash of the host bytes last uploaded
  int check;          // the policy that hash was taken under
};

// A registered raw byte range (tg_cuda_register): matrices inside it are
// found by address and are not re-checked.
struct Range {
  size_t nbytes;
};

static Slab g_slab;
static std::atomic<uint64_t> g_reuploads{0}, g_evictions{0};
static std::map<std::tuple<uintptr_t, int, int, int>, Entry> g_mats;
static std::map<uintptr_t, Range> g_ranges;

static bool in_registered_range(uintptr_t p, size_t n) {
  auto it = g_ranges.upper_bound(p);
  if (it == g_ranges.begin()) return false;
  --it;
  return p >= it->first && p + n <= it->first + it->second.nbytes;
}

// Copies raw host bytes to HBM in the layout of WDesc w (already allocated).
// Host bytes (any memory: pageable, mapped files) to the device through two
// pinned 4 MiB staging buffers, so the host copy of one chunk overlaps the
// DMA of the previous one; an event guards each buffer's reuse.
static bool upload_bytes(void* dst, const uint8_t* h, size_t n, cudaStream_t s) {
  constexpr size_t CH = (size_t)4 << 20;
  static void* pin[2] = {nullptr, nullptr};
  static cudaEvent_t ev[2];
  if (!pin[0]) {
    for (int i = 0; i < 2; i++)
      if (!cuda_ok(cudaMallocHost(&pin[i], CH), "cudaMallocHost(upload staging)") ||
          !cuda_ok(cudaEventCreateWithFlags(&ev[i], cudaEventDisableTiming), "cudaEventCreate(upload)")) {
        pin[0] = pin[1] = nullptr;
        return false;
      }
  }
  for (size_t off = 0, k = 0; off < n; off += CH, k++) {
    const int b = (int)(k & 1);
    const size_t len = std::min(CH, n - off);
    if (!cuda_ok(cudaEventSynchronize(ev[b]), "upload weights")) return false;
    memcpy(pin[b], h + off, len);
    if (!cuda_ok(cudaMemcpyAsync(static_cast<uint8_t*>(dst) + off, pin[b], len, cudaMemcpyHostToDevice, s),
                 "upload weights") ||
        !cuda_ok(cudaEventRecord(ev[b], s), "upload weights"))
      return false;
  }
  return true;
}

static bool upload_into(const uint8_t* h, size_t raw, const WDesc& w) {
  cudaStream_t s = stream();
  if (!(w.fmt == FMT_Q6K || w.fmt == FMT_MXFP4 || w.fmt == FMT_Q80)) {
    if (!upload_bytes((void*)w.main, h, raw, s)) return false;
  } else {
    if (!g.d_tmp.reserve(raw)) return false;
    if (!upload_bytes(g.d_tmp.p, h, raw, s)) return false;
    launch_repack((const uint8_t*)g.d_tmp.p, w.fmt, w.rows, w.cols, (uint8_t*)w.main, s);
    g_launches++;
  }
  return cuda_ok(cudaStreamSynchronize(s), "upload weights");
}

// Device descriptor of a rows x cols matrix in format fmt at host address h
// (fmt -1: fp32 values, fmt -2: fp32 vector of `rows` values).
bool lookup_matrix(const void* hp, int fmt, int rows, int cols, WDesc* out) {
  const uint8_t* h = (const uint8_t*)hp;
  if (!h) {
    set_host_error(2, "NULL weight pointer");
    return false;
  }
  size_t raw = fmt == -1 ? (size_t)rows * cols * 4 : fmt == -2 ? (size_t)rows * 4 : (size_t)rows * host_row_bytes(fmt, cols);
  auto key = std::make_tuple((uintptr_t)h, fmt, rows, cols);
  const bool trusted = in_registered_range((uintptr_t)h, raw);
  auto it = g_mats.find(key);
  if (it != g_mats.end()) {
    if (!trusted && g_check) {
      const uint64_t hv = check_hash(h, raw);
      if (hv != it->second.hash || it->second.check != g_check) {
        if (!upload_into(h, raw, it->second.w)) return false;
        it->second.hash = hv;
        it->second.check = g_check;
        g_reuploads++;
      }
    }
    *out = it->second.w;
    return true;
  }
  // The same host address seen before with another shape or format: the
  // caller has reused the buffer, so the old entries go, and their device
  // allocation is reused when it is large enough.
  const size_t need = (fmt == FMT_Q4K || fmt == FMT_Q6K || fmt == FMT_MXFP4 || fmt == FMT_Q80 || fmt == FMT_F16)
                          ? (size_t)rows * row_layout(fmt, cols).rs
                          : raw;
  uint8_t* reuse = nullptr;
  size_t reuse_bytes = 0;
  for (auto jt = g_mats.lower_bound(std::make_tuple((uintptr_t)h, INT_MIN, INT_MIN, INT_MIN));
       jt != g_mats.end() && std::get<0>(jt->first) == (uintptr_t)h;) {
    if (!reuse && jt->second.dev_bytes >= need) {
      reuse = const_cast<uint8_t*>(jt->second.w.main);
      reuse_bytes = jt->second.dev_bytes;
    }
    jt = g_mats.erase(jt);
    g_evictions++;
  }
  Entry e{};
  e.raw_bytes = raw;
  e.w.fmt = fmt;
  e.w.rows = rows;
  e.w.cols = cols;
  uint8_t* m = reuse ? reuse : g_slab.alloc(need);
  if (!m) return false;
  e.dev_bytes = reuse ? reuse_bytes : need;
  e.w.main = m;
  if (fmt == FMT_Q4K || fmt == FMT_Q6K || fmt == FMT_MXFP4 || fmt == FMT_Q80 || fmt == FMT_F16) {
    const RowLayout L = row_layout(fmt, cols);
    e.w.aux1 = L.a1 >= 0 ? m + L.a1 : nullptr;
    e.w.aux2 = L.a2 >= 0 ? m + L.a2 : nullptr;
    e.w.rs = L.rs;
  } else {
    e.w.rs = fmt == -1 ? cols * 4 : 4;
  }
  e.hash = trusted ? 0 : check_hash(h, raw);
  e.check = trusted ? 0 : g_check;
  if (!upload_into(h, raw, e.w)) return false;
  g_mats[key] = e;
  *out = e.w;
  return true;
}

const float* lookup_vector(const float* h, int n) {
  if (!h) return nullptr;
  WDesc w;
  if (!lookup_matrix(h, -2, n, 1, &w)) return nullptr;
  return (const float*)w.main;
}

// ---------------------------------------------------------------------
// Per-call staging.

struct Stage {
  size_t off = 0;
  size_t take(size_t n) {
    size_t o = off;
    off = align_up(off + n, 256);
    return o;
  }
};

// ---------------------------------------------------------------------
// The MoE driver shared by every expert entry point.

struct HostSlot {
  WDesc gate, up, down;
  const float *gb = nullptr, *ub = nullptr, *db = nullptr;
  std::vector<int> rows;
  std::vector<float> wts;
};

// Runs the plan: output[k][D] (host) accumulates.  `zero_output` clears it first.
bool run_moe(std::vector<HostSlot>& slots, int gate_fmt, int act, int rule, int bias_term, const float* inputs,
             float* output, int k, int D, int I, bool zero_output) {
  const char* what = "tg_moe_forward";
  if (zero_output) memset(output, 0, sizeof(float) * (size_t)k * D);
  // Drop experts with no active rows: the reference skips them entirely.
  std::vector<HostSlot*> act_slots;
  int total = 0;
  for (auto& s : slots)
    if (!s.rows.empty()) {
      act_slots.push_back(&s);
      total += (int)s.rows.size();
    }
  if (act_slots.empty() || k == 0) return true;
  const int n = (int)act_slots.size();
  const int gbpr = (D + QK - 1) / QK, dbpr = (I + QK - 1) / QK;

  Stage st;
  size_t o_hdr = st.take(sizeof(PlanHdr));
  size_t o_slots = st.take(sizeof(SlotDesc) * n);
  size_t o_rows = st.take(sizeof(int) * total);
  size_t o_wts = st.take(sizeof(float) * total);
  size_t o_rslot = st.take(sizeof(int) * total);
  size_t o_in = st.take(sizeof(float) * (size_t)k * D);
  size_t o_out = st.take(sizeof(float) * (size_t)k * D);
  size_t bytes = st.off;
  if (!g.h_up.reserve(bytes) || !g.d_stage.reserve(bytes) || !g.h_down.reserve(sizeof(float) * (size_t)k * D) ||
      !g.d_xq8.reserve(sizeof(Q8Dev) * (size_t)k * gbpr) || !g.d_hidden.reserve(sizeof(float) * (size_t)total * I) ||
      !g.d_hq8.reserve(sizeof(Q8Dev) * (size_t)total * dbpr) || !reserve_counters(moe_counter_ints(n, I)))
    return false;
  uint8_t* hb = (uint8_t*)g.h_up.p;
  uint8_t* db = (uint8_t*)g.d_stage.p;
  SlotDesc* hs = (SlotDesc*)(hb + o_slots);
  int* hrows = (int*)(hb + o_rows);
  float* hwts = (float*)(hb + o_wts);
  int* hrs = (int*)(hb + o_rslot);
  int off = 0;
  for (int i = 0; i < n; i++) {
    HostSlot& s = *act_slots[i];
    SlotDesc d{};
    d.gate = s.gate;
    d.up = s.up;
    d.down = s.down;
    d.gb = s.gb;
    d.ub = s.ub;
    d.db = s.db;
    d.n_rows = (int)s.rows.size();
    d.row_off = off;
    hs[i] = d;
    for (size_t j = 0; j < s.rows.size(); j++) {
      hrows[off] = s.rows[j];
      hwts[off] = s.wts[j];
      hrs[off] = i;
      off++;
    }
  }
  PlanHdr* hh = (PlanHdr*)(hb + o_hdr);
  hh->n_slots = n;
  hh->total_rows = total;
  hh->k = k;
  hh->embed_dim = D;
  hh->inter_dim = I;
  hh->act = act;
  hh->assoc_rule = rule;
  hh->bias_term = bias_term;
  hh->slots = (const SlotDesc*)(db + o_slots);
  hh->rows = (const int*)(db + o_rows);
  hh->wts = (const float*)(db + o_wts);
  hh->row_slot = (const int*)(db + o_rslot);
  memcpy(hb + o_in, inputs, sizeof(float) * (size_t)k * D);
  memcpy(hb + o_out, output, sizeof(float) * (size_t)k * D);

  cudaStream_t s = stream();
  if (!cuda_ok(cudaMemcpyAsync(db, hb, bytes, cudaMemcpyHostToDevice, s), what)) return false;
  const PlanHdr* dph = (const PlanHdr*)(db + o_hdr);
  const float* d_in = (const float*)(db + o_in);
  float* d_out = (float*)(db + o_out);
  Q8Dev* xq8 = (Q8Dev*)g.d_xq8.p;
  float* hidden = (float*)g.d_hidden.p;
  Q8Dev* hq8 = (Q8Dev*)g.d_hq8.p;

  // down formats of the call: one pass if uniform, else one pass per format
  // writing parts, then the ordered combine
  std::vector<int> dfmts;
  for (HostSlot* hsl : act_slots)
    if (std::find(dfmts.begin(), dfmts.end(), hsl->down.fmt) == dfmts.end()) dfmts.push_back(hsl->down.fmt);
  float* parts = nullptr;
  if (dfmts.size() > 1) {
    if (!g.d_parts.reserve(sizeof(float) * (size_t)total * D)) return false;
    parts = (float*)g.d_parts.p;
  }
  launch_quantize_rows(d_in, k, D, D, xq8, s);
  if (!cuda_ok(launch_moe_gateup(dph, n, gate_fmt, D, I, xq8, hidden, hq8, (int*)g.d_counters.p, g.d_status, s),
               what))
    return false;
  for (int f : dfmts)
    if (!cuda_ok(launch_moe_down(dph, n, total, f, D, I, k, hq8, hidden, d_out, parts, g.d_status, s), what))
      return false;
  if (parts && !cuda_ok(launch_combine_parts(dph, D, k, parts, d_out, s), what)) return false;
  g_launches += 2 + (int)dfmts.size() + (parts ? 1 : 0);
  // the output and the status record come back through the mapped result
  // block; the host waits on its echo instead of synchronising the stream
  const float* ho = deliver_reserve((size_t)k * D);
  if (!ho) return false;
  deliver_begin();
  if (!deliver_async(d_out, (size_t)k * D, s, what) || !finish_delivered(what)) return false;
  memcpy(output, ho, sizeof(float) * (size_t)k * D);
  return true;
}

bool fmt_quantized(int f) { return f == FMT_Q4K || f == FMT_Q6K || f == FMT_MXFP4 || f == FMT_Q80; }

// Validates a quantized matrix shape: ncols a multiple of the format's block.
bool check_cols(int fmt, int ncols, const char* what) {
  int blk = (fmt == FMT_Q4K || fmt == FMT_Q6K) ? QK : (fmt == FMT_MXFP4 || fmt == FMT_Q80) ? 32 : 1;
  if (ncols <= 0 || ncols % blk != 0) {
    set_host_error(3, "%s: %d columns is not a positive multiple of %d for format %d", what, ncols, blk, fmt);
    return false;
  }
  return true;
}

}  // namespace tg

using namespace tg;

// ---------------------------------------------------------------------
// C ABI.

extern "C" {

int tg_cuda_last_error(char* buf, size_t len) {
  std::lock_guard<std::mutex> lk(g_err_mu);
  int c = g_err_code;
  if (buf && len) {
    snprintf(buf, len, "%s", g_err_msg.c_str());
  }
  g_err_code = 0;
  g_err_msg.clear();
  return c;
}

int tg_cuda_set_device(int device) {
  std::lock_guard<std::recursive_mutex> lk(g.mu);
  if (g.inited) return device == g.device ? 0 : -1;
  g.device = device;
  return 0;
}

void tg_cuda_set_stream(void* s) {
  std::lock_guard<std::recursive_mutex> lk(g.mu);
  g.user_stream = (cudaStream_t)s;
  g.user_stream_set = s != nullptr;
}

int tg_cuda_register(const void* host_ptr, size_t nbytes) {
  std::lock_guard<std::recursive_mutex> lk(g.mu);
  if (!ensure_init()) return -1;
  if (!host_ptr || nbytes == 0) {
    set_host_error(2, "tg_cuda_register: empty range");
    return -1;
  }
  g_ranges[(uintptr_t)host_ptr] = Range{nbytes};
  return 0;
}

int tg_cuda_unregister(const void* host_ptr) {
  std::lock_guard<std::recursive_mutex> lk(g.mu);
  kv_mirror_forget(host_ptr);
  int n = (int)g_ranges.erase((uintptr_t)host_ptr);
  for (auto it = g_mats.begin(); it != g_mats.end();) {
    if (std::get<0>(it->first) == (uintptr_t)host_ptr) {
      it = g_mats.erase(it);
      n++;
    } else {
      ++it;
    }
  }
  return n > 0 ? 0 : -1;
}

void tg_cuda_registry_clear(void) {
  std::lock_guard<std::recursive_mutex> lk(g.mu);
  if (g.inited) cudaStreamSynchronize(stream());
  kv_mirror_clear();
  g_mats.clear();
  g_ranges.clear();
  g_slab.clear();
}

size_t tg_cuda_registry_bytes(void) {
  std::lock_guard<std::recursive_mutex> lk(g.mu);
  return g_slab.total;
}

uint64_t tg_cuda_launch_count(void) { return g_launches.load(); }

int tg_cuda_set_weight_check(int mode) {
  std::lock_guard<std::recursive_mutex> lk(g.mu);
  const int prev = g_check;
  if (mode >= 0 && mode <= 2) g_check = mode;
  return prev;
}

void tg_cuda_registry_stats(uint64_t* reuploads, uint64_t* evictions, size_t* entries) {
  std::lock_guard<std::recursive_mutex> lk(g.mu);
  if (reuploads) *reuploads = g_reuploads.load();
  if (evictions) *evictions = g_evictions.load();
  if (entries) *entries = g_mats.size();
}

size_t tg_row_bytes(int fmt, int ncols) { return host_row_bytes(fmt, ncols); }

void tg_set_threads(int n) {
  std::lock_guard<std::recursive_mutex> lk(g.mu);
  g.threads = n < 1 ? 1 : n;
}

int tg_get_threads(void) {
  std::lock_guard<std::recursive_mutex> lk(g.mu);
  return g.threads;
}

void tg_moe_forward_rows_v2(const uint8_t* const* gate_ptrs, const uint8_t* const* up_ptrs,
                            const void* const* down_ptrs, int gate_fmt, const int* down_fmts,
                            const float* const* gate_bias, const float* const* up_bias,
                            const float* const* down_bias, int act, int n_experts, const float* row_weights,
                            const float* inputs, float* output, int k, int embed_dim, int inter_dim) {
  std::lock_guard<std::recursive_mutex> lk(g.mu);
  const char* what = "tg_moe_forward_rows_v2";
  if (n_experts <= 0 || k <= 0) return;
  if (!fmt_quantized(gate_fmt)) {
    set_host_error(4, "%s: gate format %d is not supported (0 Q4_K, 2 Q6_K, 3 MXFP4, 4 Q8_0)", what, gate_fmt);
    return;
  }
  if (!check_cols(gate_fmt, embed_dim, what) || inter_dim <= 0 || inter_dim % 32 != 0) {
    if (inter_dim % 32 != 0) set_host_error(3, "%s: inter_dim %d is not a multiple of 32", what, inter_dim);
    return;
  }
  if (gate_bias && !up_bias) {
    set_host_error(4, "%s: gate_bias given without up_bias", what);
    return;
  }
  if (!ensure_init()) return;
  std::vector<HostSlot> slots(n_experts);
  for (int e = 0; e < n_experts; e++) {
    HostSlot& s = slots[e];
    for (int r = 0; r < k; r++) {
      float w = row_weights[(size_t)e * k + r];
      if (w == 0.f) continue;
      s.rows.push_back(r);
      s.wts.push_back(w);
    }
    if (s.rows.empty()) continue;
    int dfmt = down_fmts[e];
    if (!(fmt_quantized(dfmt) || dfmt == FMT_F16)) {
      set_host_error(4, "%s: down format %d of expert %d is not supported", what, dfmt, e);
      return;
    }
    if (dfmt != FMT_F16 && !check_cols(dfmt, inter_dim, what)) return;
    if (!lookup_matrix(gate_ptrs[e], gate_fmt, inter_dim, embed_dim, &s.gate) ||
        !lookup_matrix(up_ptrs[e], gate_fmt, inter_dim, embed_dim, &s.up) ||
        !lookup_matrix(down_ptrs[e], dfmt, embed_dim, inter_dim, &s.down))
      return;
    if (gate_bias) {
      s.gb = lookup_vector(gate_bias[e], inter_dim);
      s.ub = lookup_vector(up_bias[e], inter_dim);
      if (!s.gb || !s.ub) return;
    }
    if (down_bias) {
      s.db = lookup_vector(down_bias[e], embed_dim);
      if (!s.db) return;
    }
  }
  run_moe(slots, gate_fmt, act == ACT_GPTOSS ? ACT_GPTOSS : ACT_SILU, ASSOC_MOE, 1, inputs, output, k, embed_dim,
          inter_dim, false);
}

void tg_moe_forward_rows(const uint8_t* const* gate_ptrs, const uint8_t* const* up_ptrs, const void* const* down_ptrs,
                         const int* down_fmts, int n_experts, const float* row_weights, const float* inputs,
                         float* output, int k, int embed_dim, int inter_dim) {
  tg_moe_forward_rows_v2(gate_ptrs, up_ptrs, down_ptrs, FMT_Q4K, down_fmts, nullptr, nullptr, nullptr, ACT_SILU,
                         n_experts, row_weights, inputs, output, k, embed_dim, inter_dim);
}

// Down format codes of the single-expert entries: 1 F16, 2 Q6_K, else Q4_K.
static int single_down_fmt(int f) { return f == 1 ? FMT_F16 : f == 2 ? FMT_Q6K : FMT_Q4K; }

static void expert_rows(const char* what, const uint8_t* gate, const uint8_t* up, const void* down, int down_format,
                        const float* inputs, float* output, const float* weights, int k, int D, int I, int rule,
                        bool zero) {
  if (k <= 0) return;
  if (!check_cols(FMT_Q4K, D, what)) return;
  int dfmt = single_down_fmt(down_format);
  if (dfmt != FMT_F16 && !check_cols(dfmt, I, what)) return;
  if (!ensure_init()) return;
  std::vector<HostSlot> slots(1);
  HostSlot& s = slots[0];
  for (int r = 0; r < k; r++) {
    s.rows.push_back(r);
    s.wts.push_back(weights[r]);
  }
  if (!lookup_matrix(gate, FMT_Q4K, I, D, &s.gate) || !lookup_matrix(up, FMT_Q4K, I, D, &s.up) ||
      !lookup_matrix(down, dfmt, D, I, &s.down))
    return;
  run_moe(slots, FMT_Q4K, ACT_SILU, rule, 0, inputs, output, k, D, I, zero);
}

void tg_expert_forward(const uint8_t* q4_data, const float* input, float* output, float weight, int embed_dim,
                       int inter_dim) {
  std::lock_guard<std::recursive_mutex> lk(g.mu);
  size_t gate_bytes = (size_t)inter_dim * host_row_bytes(FMT_Q4K, embed_dim);
  expert_rows("tg_expert_forward", q4_data, q4_data + gate_bytes, q4_data + 2 * gate_bytes, 0, input, output,
              &weight, 1, embed_dim, inter_dim, ASSOC_X1, false);
}

void tg_expert_forward_mixed(const uint8_t* gate_q4, const uint8_t* up_q4, const void* down_data, int down_format,
                             const float* input, float* output, float weight, int embed_dim, int inter_dim) {
  std::lock_guard<std::recursive_mutex> lk(g.mu);
  expert_rows("tg_expert_forward_mixed", gate_q4, up_q4, down_data, down_format, input, output, &weight, 1,
              embed_dim, inter_dim, ASSOC_X1, false);
}

void tg_expert_forward_rows(const uint8_t* gate_q4, const uint8_t* up_q4, const void* down_data, int down_format,
                            const float* inputs, float* output, const float* weights, int k, int embed_dim,
                            int inter_dim) {
  std::lock_guard<std::recursive_mutex> lk(g.mu);
  expert_rows("tg_expert_forward_rows", gate_q4, up_q4, down_data, down_format, inputs, output, weights, k,
              embed_dim, inter_dim, ASSOC_ROWS, false);
}

void tg_moe_forward(const uint8_t** expert_ptrs, const float* weights, int n_experts, const float* input,
                    float* output, int embed_dim, int inter_dim) {
  std::lock_guard<std::recursive_mutex> lk(g.mu);
  const char* what = "tg_moe_forward";
  memset(output, 0, sizeof(float) * (size_t)embed_dim);
  if (n_experts <= 0) return;
  if (!check_cols(FMT_Q4K, embed_dim, what) || !check_cols(FMT_Q4K, inter_dim, what)) return;
  if (!ensure_init()) return;
  size_t gate_bytes = (size_t)inter_dim * host_row_bytes(FMT_Q4K, embed_dim);
  std::vector<HostSlot> slots(n_experts);
  for (int e = 0; e < n_experts; e++) {
    HostSlot& s = slots[e];
    s.rows.push_back(0);
    s.wts.push_back(weights[e]);
    const uint8_t* b = expert_ptrs[e];
    if (!lookup_matrix(b, FMT_Q4K, inter_dim, embed_dim, &s.gate) ||
        !lookup_matrix(b + gate_bytes, FMT_Q4K, inter_dim, embed_dim, &s.up) ||
        !lookup_matrix(b + 2 * gate_bytes, FMT_Q4K, embed_dim, inter_dim, &s.down))
      return;
  }
  run_moe(slots, FMT_Q4K, ACT_SILU, ASSOC_X1, 0, input, output, 1, embed_dim, inter_dim, false);
}

// Matvec entries.

static void matvec_entry(const char* what, int fmt, const void* mat, const float* bias, int bias_term,
                         const float* input, float* output, int nrows, int ncols) {
  if (nrows <= 0) return;
  if (fmt != FMT_F16 && !check_cols(fmt, ncols, what)) return;
  if (!ensure_init()) return;
  WDesc w;
  if (!lookup_matrix(mat, fmt, nrows, ncols, &w)) return;
  const float* dbias = nullptr;
  if (bias && !(dbias = lookup_vector(bias, nrows))) return;
  const int nb = (ncols + QK - 1) / QK;
  cudaStream_t s = stream();
  if (!g.h_up.reserve(sizeof(float) * ncols) || !g.d_stage.reserve(sizeof(float) * ncols + 256 + sizeof(float) * nrows) ||
      !g.d_xq8.reserve(sizeof(Q8Dev) * nb) || !g.h_down.reserve(sizeof(float) * nrows))
    return;
  float* d_x = (float*)g.d_stage.p;
  float* d_out = (float*)((uint8_t*)g.d_stage.p + align_up(sizeof(float) * ncols, 256));
  memcpy(g.h_up.p, input, sizeof(float) * ncols);
  if (!cuda_ok(cudaMemcpyAsync(d_x, g.h_up.p, sizeof(float) * ncols, cudaMemcpyHostToDevice, s), what)) return;
  if (fmt != FMT_F16) {
    launch_quantize_rows(d_x, 1, ncols, ncols, (Q8Dev*)g.d_xq8.p, s);
    g_launches++;
  }
  if (!cuda_ok(launch_matvec(w, (const Q8Dev*)g.d_xq8.p, d_x, dbias, bias_term, d_out, g.d_status, s), what)) return;
  g_launches++;
  if (!cuda_ok(cudaMemcpyAsync(g.h_down.p, d_out, sizeof(float) * nrows, cudaMemcpyDeviceToHost, s), what)) return;
  if (!finish(what)) return;
  memcpy(output, g.h_down.p, sizeof(float) * nrows);
}

void tg_matmul_q4k(const uint8_t* q4_matrix, const float* input, float* output, int nrows, int ncols) {
  std::lock_guard<std::recursive_mutex> lk(g.mu);
  matvec_entry("tg_matmul_q4k", FMT_Q4K, q4_matrix, nullptr, 0, input, output, nrows, ncols);
}

void tg_matmul_q6k(const uint8_t* q6_matrix, const float* input, float* output, int nrows, int ncols) {
  std::lock_guard<std::recursive_mutex> lk(g.mu);
  matvec_entry("tg_matmul_q6k", FMT_Q6K, q6_matrix, nullptr, 0, input, output, nrows, ncols);
}

// Any format code other than Q4_K/Q6_K/MXFP4/Q8_0 decodes as F16, as the
// reference's dispatch default does (libtinygiant.c:596-620).
void tg_matmul(int fmt, const void* mat, const float* bias, const float* input, float* output, int nrows, int ncols) {
  std::lock_guard<std::recursive_mutex> lk(g.mu);
  matvec_entry("tg_matmul", fmt_quantized(fmt) ? fmt : FMT_F16, mat, bias, 1, input, output, nrows, ncols);
}

static void plain_matvec(const char* what, bool f16, const void* A, const float* x, float* out, int nrows,
                         int ncols) {
  if (nrows <= 0) return;
  if (!ensure_init()) return;
  WDesc w;
  if (!lookup_matrix(A, f16 ? FMT_F16 : -1, nrows, ncols, &w)) return;
  cudaStream_t s = stream();
  if (!g.h_up.reserve(sizeof(float) * ncols) || !g.d_stage.reserve(align_up(sizeof(float) * ncols, 256) + sizeof(float) * nrows) ||
      !g.h_down.reserve(sizeof(float) * nrows))
    return;
  float* d_x = (float*)g.d_stage.p;
  float* d_out = (float*)((uint8_t*)g.d_stage.p + align_up(sizeof(float) * ncols, 256));
  memcpy(g.h_up.p, x, sizeof(float) * ncols);
  if (!cuda_ok(cudaMemcpyAsync(d_x, g.h_up.p, sizeof(float) * ncols, cudaMemcpyHostToDevice, s), what)) return;
  if (f16) launch_f16_matvec((const uint16_t*)w.main, d_x, d_out, nrows, ncols, s);
  else launch_f32_matvec((const float*)w.main, d_x, d_out, nrows, ncols, s);
  g_launches++;
  if (!cuda_ok(cudaGetLastError(), what)) return;
  if (!cuda_ok(cudaMemcpyAsync(g.h_down.p, d_out, sizeof(float) * nrows, cudaMemcpyDeviceToHost, s), what)) return;
  if (!finish(what)) return;
  memcpy(out, g.h_down.p, sizeof(float) * nrows);
}

void tg_f16_matvec(const uint16_t* A, const float* x, float* out, int nrows, int ncols) {
  std::lock_guard<std::recursive_mutex> lk(g.mu);
  plain_matvec("tg_f16_matvec", true, A, x, out, nrows, ncols);
}

void tg_f32_matvec(const float* A, const float* x, float* out, int nrows, int ncols) {
  std::lock_guard<std::recursive_mutex> lk(g.mu);
  plain_matvec("tg_f32_matvec", false, A, x, out, nrows, ncols);
}

void tg_rms_norm(const float* x, const float* weight, float* out, int dim, float eps) {
  std::lock_guard<std::recursive_mutex> lk(g.mu);
  const char* what = "tg_rms_norm";
  if (dim <= 0) return;
  if (!ensure_init()) return;
  const float* dw = lookup_vector(weight, dim);
  if (!dw) return;
  cudaStream_t s = stream();
  size_t xb = align_up(sizeof(float) * dim, 256);
  if (!g.h_up.reserve(xb) || !g.d_stage.reserve(2 * xb) || !g.h_down.reserve(xb)) return;
  float* d_x = (float*)g.d_stage.p;
  float* d_out = (float*)((uint8_t*)g.d_stage.p + xb);
  memcpy(g.h_up.p, x, sizeof(float) * dim);
  if (!cuda_ok(cudaMemcpyAsync(d_x, g.h_up.p, sizeof(float) * dim, cudaMemcpyHostToDevice, s), what)) return;
  launch_rms_norm(d_x, dw, d_out, dim, eps, s);
  g_launches++;
  if (!cuda_ok(cudaGetLastError(), what)) return;
  if (!cuda_ok(cudaMemcpyAsync(g.h_down.p, d_out, sizeof(float) * dim, cudaMemcpyDeviceToHost, s), what)) return;
  if (!finish(what)) return;
  memcpy(out, g.h_down.p, sizeof(float) * dim);
}

// ---- Test hooks --------------------------------------------------------

int tg_cuda_device_count(void) {
  int n = 0;
  if (cudaGetDeviceCount(&n) != cudaSuccess) {
    cudaGetLastError();
    return 0;
  }
  return n;
}

// The reference's 296-byte q8_block: scale, sum, bsums[8], qs[256].
struct RefQ8 {
  float scale;
  int32_t sum;
  int32_t bsums[8];
  int8_t qs[256];
};
static_assert(sizeof(RefQ8) == 296, "q8_block");

int tg_cuda_debug_quantize_q8(const float* x, int nrows, int ncols, void* out_blocks) {
  std::lock_guard<std::recursive_mutex> lk(g.mu);
  const char* what = "tg_cuda_debug_quantize_q8";
  if (nrows <= 0 || ncols <= 0) return 0;
  if (!ensure_init()) return -1;
  const int nb = (ncols + QK - 1) / QK;
  const size_t xb = align_up(sizeof(float) * (size_t)nrows * ncols, 256);
  const size_t qb = sizeof(Q8Dev) * (size_t)nrows * nb;
  if (!g.h_up.reserve(xb) || !g.d_stage.reserve(xb + qb) || !g.h_down.reserve(qb)) return -1;
  memcpy(g.h_up.p, x, sizeof(float) * (size_t)nrows * ncols);
  cudaStream_t s = stream();
  float* dx = (float*)g.d_stage.p;
  Q8Dev* dq = (Q8Dev*)((uint8_t*)g.d_stage.p + xb);
  if (!cuda_ok(cudaMemcpyAsync(dx, g.h_up.p, sizeof(float) * (size_t)nrows * ncols, cudaMemcpyHostToDevice, s), what))
    return -1;
  launch_quantize_rows(dx, nrows, ncols, ncols, dq, s);
  g_launches++;
  if (!cuda_ok(cudaMemcpyAsync(g.h_down.p, dq, qb, cudaMemcpyDeviceToHost, s), what) || !finish(what)) return -1;
  const Q8Dev* hq = (const Q8Dev*)g.h_down.p;
  RefQ8* o = (RefQ8*)out_blocks;
  for (size_t i = 0; i < (size_t)nrows * nb; i++) {
    o[i].scale = hq[i].scale;
    o[i].sum = hq[i].sum;
    memcpy(o[i].bsums, hq[i].bsums, sizeof o[i].bsums);
    memcpy(o[i].qs, hq[i].qs, sizeof o[i].qs);
  }
  return 0;
}

int tg_cuda_debug_row_isums(int fmt, const void* mat, int nrows, int ncols, const void* xq_blocks, int32_t* out) {
  std::lock_guard<std::recursive_mutex> lk(g.mu);
  const char* what = "tg_cuda_debug_row_isums";
  if (!fmt_quantized(fmt)) {
    set_host_error(4, "%s: format %d has no integer sums", what, fmt);
    return -1;
  }
  if (nrows <= 0 || !check_cols(fmt, ncols, what)) return -1;
  if (!ensure_init()) return -1;
  WDesc w;
  if (!lookup_matrix(mat, fmt, nrows, ncols, &w)) return -1;
  const int nb = (ncols + QK - 1) / QK;
  const int per_row = debug_isums_per_row(fmt, ncols);
  const size_t qb = align_up(sizeof(Q8Dev) * nb, 256), ob = sizeof(int32_t) * (size_t)nrows * per_row;
  if (!g.h_up.reserve(qb) || !g.d_stage.reserve(qb + ob) || !g.h_down.reserve(ob)) return -1;
  Q8Dev* hq = (Q8Dev*)g.h_up.p;
  const RefQ8* in = (const RefQ8*)xq_blocks;
  memset(hq, 0, qb);
  for (int b = 0; b < nb; b++) {
    memcpy(hq[b].qs, in[b].qs, 256);
    hq[b].scale = in[b].scale;
    hq[b].sum = in[b].sum;
    memcpy(hq[b].bsums, in[b].bsums, sizeof hq[b].bsums);
  }
  cudaStream_t s = stream();
  Q8Dev* dq = (Q8Dev*)g.d_stage.p;
  int32_t* dout = (int32_t*)((uint8_t*)g.d_stage.p + qb);
  if (!cuda_ok(cudaMemcpyAsync(dq, hq, qb, cudaMemcpyHostToDevice, s), what)) return -1;
  launch_debug_isums(w, dq, dout, s);
  g_launches++;
  if (!cuda_ok(cudaGetLastError(), what)) return -1;
  if (!cuda_ok(cudaMemcpyAsync(g.h_down.p, dout, ob, cudaMemcpyDeviceToHost, s), what) || !finish(what)) return -1;
  memcpy(out, g.h_down.p, ob);
  return per_row;
}

int tg_cuda_debug_div_check(long long n, unsigned seed, unsigned long long* mismatches) {
  std::lock_guard<std::recursive_mutex> lk(g.mu);
  const char* what = "tg_cuda_debug_div_check";
  if (n < 0 || !mismatches || !ensure_init()) return -1;
  if (!g.d_stage.reserve(256) || !g.h_down.reserve(256)) return -1;
  cudaStream_t s = stream();
  unsigned long long* d = (unsigned long long*)g.d_stage.p;
  if (!cuda_ok(cudaMemsetAsync(d, 0, sizeof(*d), s), what)) return -1;
  launch_debug_div(n, seed, d, s);
  g_launches++;
  if (!cuda_ok(cudaGetLastError(), what)) return -1;
  if (!cuda_ok(cudaMemcpyAsync(g.h_down.p, d, sizeof(*d), cudaMemcpyDeviceToHost, s), what) || !finish(what)) return -1;
  *mismatches = *(unsigned long long*)g.h_down.p;
  return 0;
}

// Host page-cache hints on the caller's (host) memory, as the reference
// issues them; they do not touch the GPU.
static void page_range(const void* addr, size_t len, void** a, size_t* n) {
  uintptr_t pg = (uintptr_t)sysconf(_SC_PAGESIZE);
  uintptr_t p = (uintptr_t)addr & ~(pg - 1);
  *a = (void*)p;
  *n = len + ((uintptr_t)addr - p);
}

void tg_prefetch(const void* addr, size_t len) {
  void* a;
  size_t n;
  page_range(addr, len, &a, &n);
  posix_madvise(a, n, POSIX_MADV_WILLNEED);
}

void tg_prefetch_batch(const void** addrs, const size_t* lens, int count) {
  for (int i = 0; i < count; i++) tg_prefetch(addrs[i], lens[i]);
}

int tg_mlock(const void* addr, size_t len) {
  void* a;
  size_t n;
  page_range(addr, len, &a, &n);
  return mlock(a, n);
}

}  // extern "C"
