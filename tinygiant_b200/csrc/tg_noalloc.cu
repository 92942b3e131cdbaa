// tg_noalloc.cu — tg_cuda_matmul_q4k_noalloc: the Q4_K matvec of
// tg_matmul_q4k (csrc/libtinygiant.c:345-364, 906-931) on caller-owned device
// memory, for callers that cannot allocate device memory.
//
// The only scratch is the Q8 copy of the input vector, held in a file-scope
// __device__ array of fixed size.  Every GPU that loads this library holds
// that array until the process exits.  Per call the path launches the same
// two kernels as tg_matmul_q4k (quantize_rows_kernel, matvec_kernel) with the
// same arguments apart from the scratch pointer, so the outputs are
// bit-identical to it.
//
// Nothing in the scratch has to start at zero: the quantizer writes every
// field of every Q8 block (qs, scale, sum, bsums) that the matvec reads,
// before the matvec reads it.
#include <mutex>

#include "tg_kernels.h"
#include "tg_runtime.h"

namespace tg {

// Columns are limited to 65,536, i.e. 256 Q8 blocks of 320 bytes: 80 KiB.
constexpr int NOALLOC_MAX_COLS = 65536;
constexpr int NOALLOC_MAX_BLOCKS = NOALLOC_MAX_COLS / QK;
constexpr int NOALLOC_MAX_DEVICES = 64;

static __device__ __align__(256) Q8Dev g_noalloc_xq8[NOALLOC_MAX_BLOCKS];

static std::mutex g_noalloc_mu;
static Q8Dev* g_noalloc_ptr[NOALLOC_MAX_DEVICES];

// Device address of the scratch on the current device, looked up once per
// device (the first call on a device must therefore run outside stream
// capture).  The address is kept for the life of the process: after a
// cudaDeviceReset it would be stale, so a process that resets a device must
// not call this entry point on that device again.  Returns 0 with *out set,
// or the error code it recorded.
static int noalloc_scratch(int dev, Q8Dev** out) {
  std::lock_guard<std::mutex> lk(g_noalloc_mu);
  if (!g_noalloc_ptr[dev]) {
    Q8Dev* ptr = nullptr;
    cudaError_t e = cudaGetSymbolAddress((void**)&ptr, g_noalloc_xq8);
    if (e != cudaSuccess || !ptr) {
      const int code = 100 + (int)(e != cudaSuccess ? e : cudaErrorInvalidSymbol);
      set_host_error(code, "tg_cuda_matmul_q4k_noalloc: cudaGetSymbolAddress on device %d: %s", dev,
                     cudaGetErrorString(e));
      return code;
    }
    g_noalloc_ptr[dev] = ptr;
  }
  *out = g_noalloc_ptr[dev];
  return 0;
}

static bool device_pointer(const void* p, int dev) {
  cudaPointerAttributes a;
  if (cudaPointerGetAttributes(&a, p) != cudaSuccess) {
    cudaGetLastError();
    return false;
  }
  return (a.type == cudaMemoryTypeDevice || a.type == cudaMemoryTypeManaged) && a.device == dev;
}

}  // namespace tg

using namespace tg;

extern "C" int tg_cuda_matmul_q4k_noalloc(const uint8_t* q4_matrix, const float* input, float* output, int nrows,
                                          int ncols, void* stream) {
  const char* what = "tg_cuda_matmul_q4k_noalloc";
  if (nrows <= 0 || ncols <= 0 || ncols % QK != 0) {
    set_host_error(3, "%s: need nrows > 0 and ncols a positive multiple of %d (got %d x %d)", what, QK, nrows, ncols);
    return 3;
  }
  if (ncols > NOALLOC_MAX_COLS) {
    set_host_error(3, "%s: ncols %d exceeds the fixed scratch maximum of %d columns", what, ncols, NOALLOC_MAX_COLS);
    return 3;
  }
  int dev = -1;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess || dev < 0 || dev >= NOALLOC_MAX_DEVICES) {
    set_host_error(2, "%s: no usable CUDA device (%s)", what, cudaGetErrorString(e));
    return 2;
  }
  if (((uintptr_t)q4_matrix & 15) || ((uintptr_t)input & 3) || ((uintptr_t)output & 3)) {
    set_host_error(3, "%s: the matrix must be 16-byte aligned and the vectors 4-byte aligned", what);
    return 3;
  }
  if (!device_pointer(q4_matrix, dev) || !device_pointer(input, dev) || !device_pointer(output, dev)) {
    set_host_error(3, "%s: matrix, input and output must be device memory on the current device %d", what, dev);
    return 3;
  }
  Q8Dev* xq8 = nullptr;
  if (const int rc = noalloc_scratch(dev, &xq8)) return rc;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  WDesc w{q4_matrix, nullptr, nullptr, FMT_Q4K, nrows, ncols, (ncols / QK) * Q4K_BYTES};
  launch_quantize_rows(input, 1, ncols, ncols, xq8, s);
  e = cudaGetLastError();
  if (e == cudaSuccess) e = launch_matvec(w, xq8, input, nullptr, 0, output, nullptr, s);
  if (e != cudaSuccess) {
    set_host_error(100 + (int)e, "%s: launch failed: %s", what, cudaGetErrorString(e));
    return 100 + (int)e;
  }
  count_launches(2);
  return 0;
}
