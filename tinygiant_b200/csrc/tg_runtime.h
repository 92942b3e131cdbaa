// tg_runtime.h — host runtime internals shared by the C-ABI translation units.
#pragma once
#include <cuda_runtime.h>

#include <mutex>

#include "tg_common.cuh"

namespace tg {

void set_host_error(int code, const char* fmt, ...);
bool ensure_init();
cudaStream_t stream();
bool finish(const char* what);
bool status_copy_async(cudaStream_t s, const char* what);
bool finish_copied(const char* what);
size_t host_row_bytes(int fmt, int ncols);
bool lookup_matrix(const void* h, int fmt, int rows, int cols, WDesc* out);
const float* lookup_vector(const float* h, int n);
std::recursive_mutex& ctx_mutex();
DevStatus* status_ptr();
void count_launches(int n);
void* pinned_up(size_t n);
void* pinned_down(size_t n);
void register_counters(void* p, size_t n);
void unregister_counters(void* p);

}  // namespace tg
