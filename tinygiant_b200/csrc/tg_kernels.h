// tg_kernels.h — host-side launchers for the kernels in tg_kernels.cu.
#pragma once
#include <cuda_runtime.h>

#include "tg_plan.cuh"

namespace tg {

void launch_quantize_rows(const float* x, int nrows, int ncols, long ldx, Q8Dev* out, cudaStream_t s);
cudaError_t launch_matvec(const WDesc& W, const Q8Dev* xq8, const float* x, const float* bias, int bias_term,
                          float* out, DevStatus* st, cudaStream_t s);
// Three matrices (quantized or F16) against one input in one launch.
cudaError_t launch_matvec3(const WDesc* W, const float* const* bias, float* const* out, const Q8Dev* xq8,
                           const float* x, int bias_term, DevStatus* st, cudaStream_t s);
void launch_f32_matvec(const float* A, const float* x, float* out, int nrows, int ncols, cudaStream_t s);
void launch_f16_matvec(const uint16_t* A, const float* x, float* out, int nrows, int ncols, cudaStream_t s);
void launch_add(const float* a, const float* b, float* out, size_t n, cudaStream_t s);
void launch_rms_norm(const float* x, const float* w, float* out, int dim, float eps, cudaStream_t s);
int debug_isums_per_row(int fmt, int cols);
void launch_debug_isums(const WDesc& W, const Q8Dev* xq, int32_t* out, cudaStream_t s);
void launch_debug_div(long long n, uint32_t seed, unsigned long long* bad, cudaStream_t s);
// Raw reference blocks of a rows x cols matrix -> the WDesc row layout at dst.
void launch_repack(const uint8_t* raw, int fmt, int rows, int cols, uint8_t* dst, cudaStream_t s);

}  // namespace tg
