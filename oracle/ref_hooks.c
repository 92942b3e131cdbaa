/*
 * ref_hooks.c — exports the reference's static kernels for golden vectors.
 *
 * TEST INFRASTRUCTURE ONLY.  Compiled by oracle/Makefile with the reference's
 * csrc/ on the include path, exactly as the reference's own
 * csrc/test_libtinygiant.c pulls in "libtinygiant.c" to reach its static
 * functions; x86 builds get NEON from oracle/neon_shim/arm_neon.h.  The
 * resulting oracle/_ref/libtinygiant_ref_hooks.so is what
 * tests/golden/make_golden.py runs to record reference outputs.
 */
#include "libtinygiant.c"

size_t refh_q8_block_bytes(void) { return sizeof(q8_block); }

void refh_quantize_q8(const float *x, void *out, int ncols) { quantize_q8(x, (q8_block *)out, ncols); }

/* One row against one Q8 input: the x1 kernels (dot_fmt). */
float refh_dot(int fmt, const uint8_t *row, const void *xq, int ncols) {
    return dot_fmt(fmt, row, (const q8_block *)xq, NULL, ncols);
}

/* One row against four Q8 inputs: the x4 kernels (dot_fmt_x4). */
void refh_dot_x4(int fmt, const uint8_t *row, const void *xq0, const void *xq1, const void *xq2, const void *xq3,
                 int ncols, float *out) {
    const q8_block *p[4] = { xq0, xq1, xq2, xq3 };
    dot_fmt_x4(fmt, row, p, NULL, ncols, out);
}

float refh_act(int act, float g, float u) { return act_fn(act, g, u); }
