// tg_attention.cu — attention and whole-layer entries of the reference ABI.
//
// These sit outside the MoE expert path this library accelerates
// (csrc/libtinygiant.c:723-1036, 1467-1507).  They are exported so the
// reference loader binds every symbol; a call records an error and leaves
// its outputs untouched (there is no CPU fallback).
#include "../../include/tinygiant.h"
#include "tg_runtime.h"

extern "C" {

void tg_attention_decode(const float*, const float*, const float*, const float*, const float*, const float*, float*,
                         float*, int, int, const float*, const float*, const float*, float*, int, int, int, int, int) {
  tg::set_host_error(5, "tg_attention_decode is not implemented on the GPU in this build");
}

void tg_attention_decode_q4(const uint8_t*, const uint8_t*, const uint16_t*, const uint8_t*, const float*,
                            const float*, float*, float*, int, int, const float*, const float*, const float*, float*,
                            int, int, int, int, int) {
  tg::set_host_error(5, "tg_attention_decode_q4 is not implemented on the GPU in this build");
}

void tg_attention_v2(int, int, int, int, const void*, const void*, const void*, const void*, const float*, const float*,
                     const float*, const float*, const float*, const float*, const float*, float*, float*, int, int,
                     int, const float*, const float*, const float*, float*, int, int, int, int, int, float) {
  tg::set_host_error(5, "tg_attention_v2 is not implemented on the GPU in this build");
}

void tg_transformer_layer(const float*, const float*, const float*, const float*, const float*, const float*,
                          const float*, const float*, float*, float*, int, int, const float*, const float*,
                          const uint8_t**, const uint8_t**, const void**, const int*, const float*, int, float*, int,
                          int, int, int, int, int) {
  tg::set_host_error(5, "tg_transformer_layer is not implemented on the GPU in this build");
}

}  // extern "C"
