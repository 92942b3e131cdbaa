// tg_runtime.h — host runtime internals shared by the C-ABI translation units.
#pragma once
#include <cuda_runtime.h>

#include <mutex>

#include "tg_common.cuh"

namespace tg {

void set_host_error(int code, const char* fmt, ...);
// Count of errors recorded so far (a call failed if it changed).
unsigned host_error_seq();
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
// Small results to the host without a stream synchronisation (mapped pinned
// memory and a request number echoed by the device): deliver_reserve sizes
// the block and returns the host copy of the floats; deliver_async enqueues
// the copy (capturable); deliver_begin sets the request before a launch;
// finish_delivered waits for it and checks the device status.
float* deliver_reserve(size_t n_floats);
bool deliver_async(const float* d_src, size_t n_floats, cudaStream_t s, const char* what);
void deliver_begin();
bool finish_delivered(const char* what);
// Small inputs the other way: fetch_reserve sizes a mapped pinned block and
// returns its host pointer; fetch_async enqueues a one-CTA kernel that copies
// it into device memory (capturable) and lets a dependent kernel launched
// with programmatic stream serialization start at once.
float* fetch_reserve(size_t n_floats);
bool fetch_async(float* d_dst, size_t n_floats, cudaStream_t s, const char* what);
void unregister_counters(void* p);
// Attention decode's KV-cache mirrors (tg_attention.cu), dropped with the registry.
void kv_mirror_forget(const void* host);
void kv_mirror_clear();

}  // namespace tg
