/*
 * tinygiant.h — C ABI of the B200 drop-in libtinygiant.so.
 *
 * The first block is the reference's ABI: the 21 symbols that the reference
 * loader tinygiant/_lib.py:39-93 registers with ctypes, with the same names,
 * argument lists, return types and accumulate (+=) semantics as
 * csrc/libtinygiant.c.  Every pointer is a HOST pointer, exactly as the
 * reference engine passes numpy arrays and mmap views; weight bytes are
 * uploaded to HBM on first use and stay resident (see tg_cuda_register).
 * All calls are synchronous: results are in the caller's buffers on return.
 *
 * Errors: the reference functions return void and validate nothing.  Here a
 * call that cannot run (no GPU, an unsupported format, a bad shape, a CUDA
 * failure) leaves its outputs untouched, prints one line to stderr and
 * records the error for tg_cuda_last_error(); there is no CPU fallback.
 *
 * Format codes (libtinygiant.c:594): 0 Q4_K, 1 F16, 2 Q6_K, 3 MXFP4, 4 Q8_0.
 * Activation codes (libtinygiant.c:1248): 0 SiLU, 1 gpt-oss.
 */
#ifndef TINYGIANT_H
#define TINYGIANT_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* ---- Reference ABI ------------------------------------------------------ */

/* out[D] += w * down(silu(gate.x) * up.x) for one all-Q4_K expert stored
 * contiguously as [gate | up | down] (libtinygiant.c:1040-1080). */
void tg_expert_forward(const uint8_t *q4_data, const float *input, float *output, float weight,
                       int embed_dim, int inter_dim);

/* As tg_expert_forward with separate Q4_K gate/up and a down matrix in
 * format 1 (F16), 2 (Q6_K) or anything else (Q4_K) (libtinygiant.c:1084-1128). */
void tg_expert_forward_mixed(const uint8_t *gate_q4, const uint8_t *up_q4, const void *down_data,
                             int down_format, const float *input, float *output, float weight,
                             int embed_dim, int inter_dim);

/* out[nrows] = Q4_K matrix . Q8(x) (libtinygiant.c:375-378). */
void tg_matmul_q4k(const uint8_t *q4_matrix, const float *input, float *output, int nrows, int ncols);

/* out[nrows] = Q6_K matrix . Q8(x) (libtinygiant.c:498-501). */
void tg_matmul_q6k(const uint8_t *q6_matrix, const float *input, float *output, int nrows, int ncols);

/* out = x / sqrt(mean(x^2) + eps) * w (libtinygiant.c:680-698). */
void tg_rms_norm(const float *x, const float *weight, float *out, int dim, float eps);

/* out[nrows] = A (fp32, row-major) . x (libtinygiant.c:662-676). */
void tg_f32_matvec(const float *A, const float *x, float *out, int nrows, int ncols);

/* out[nrows] = A (fp16, row-major) . x (libtinygiant.c:655-658). */
void tg_f16_matvec(const uint16_t *A, const float *x, float *out, int nrows, int ncols);

/* Single-row GQA attention decode step, fp32 weights (libtinygiant.c:723-814). */
void tg_attention_decode(const float *wq, const float *wk, const float *wv, const float *wo,
                         const float *q_norm_w, const float *k_norm_w, float *kv_k, float *kv_v,
                         int kv_len, int kv_max, const float *rope_cos, const float *rope_sin,
                         const float *input, float *output, int embed_dim, int n_heads, int n_kv_heads,
                         int head_dim, int pos);

/* Same with Q4_K q/k/o and fp16 v projections (libtinygiant.c:985-1036). */
void tg_attention_decode_q4(const uint8_t *wq_q4, const uint8_t *wk_q4, const uint16_t *wv_f16,
                            const uint8_t *wo_q4, const float *q_norm_w, const float *k_norm_w,
                            float *kv_k, float *kv_v, int kv_len, int kv_max, const float *rope_cos,
                            const float *rope_sin, const float *input, float *output, int embed_dim,
                            int n_heads, int n_kv_heads, int head_dim, int pos);

/* Host page-cache hints (libtinygiant.c:1550-1571). */
void tg_prefetch(const void *addr, size_t len);
void tg_prefetch_batch(const void **addrs, const size_t *lens, int count);
int tg_mlock(const void *addr, size_t len);

/* Generic attention decode step: any weight format per projection,
 * optional biases, QK norm, sinks and sliding window (libtinygiant.c:939-983).
 * These three run on the GPU.  kv_k / kv_v ([n_kv_heads][kv_max][head_dim]
 * host floats) get a device mirror per pointer: positions below kv_len it
 * has not seen are uploaded, and the new row is written to both.  A caller
 * that writes a cache itself (or frees one and reuses its address) calls
 * tg_cuda_unregister(kv_ptr) first.  head_dim even and <= 256;
 * n_heads a multiple of n_kv_heads; kv_len < kv_max. */
void tg_attention_v2(int fmt_q, int fmt_k, int fmt_v, int fmt_o, const void *wq, const void *wk,
                     const void *wv, const void *wo, const float *bq, const float *bk, const float *bv,
                     const float *bo, const float *q_norm_w, const float *k_norm_w, const float *sinks,
                     float *kv_k, float *kv_v, int kv_len, int kv_max, int window, const float *rope_cos,
                     const float *rope_sin, const float *input, float *output, int embed_dim, int n_heads,
                     int n_kv_heads, int head_dim, int pos, float eps);

/* The MoE layer the engine calls (libtinygiant.c:1386-1437, engine.py:336-340):
 * for each of n_experts experts, the rows r with row_weights[e*k + r] != 0
 * run gate/up (gate_fmt), the activation, down (down_fmts[e]) and
 * output[r] += w * (down.h + down_bias); experts combine in the given order.
 * Bias arrays are per-expert pointer arrays or NULL (gate_bias implies up_bias). */
void tg_moe_forward_rows_v2(const uint8_t *const *gate_ptrs, const uint8_t *const *up_ptrs,
                            const void *const *down_ptrs, int gate_fmt, const int *down_fmts,
                            const float *const *gate_bias, const float *const *up_bias,
                            const float *const *down_bias, int act, int n_experts, const float *row_weights,
                            const float *inputs, float *output, int k, int embed_dim, int inter_dim);

/* out[nrows] = mat(fmt) . x + (bias ? bias : 0) (libtinygiant.c:925-931). */
void tg_matmul(int fmt, const void *mat, const float *bias, const float *input, float *output, int nrows,
               int ncols);

/* Bytes of one row of ncols values in format fmt (libtinygiant.c:596-606). */
size_t tg_row_bytes(int fmt, int ncols);

/* CPU thread-pool size of the reference (libtinygiant.c:85-104).  Recorded
 * and reported back; the GPU path does not use host threads. */
void tg_set_threads(int n);
int tg_get_threads(void);

/* k rows through one expert with Q4_K gate/up (libtinygiant.c:1182-1231). */
void tg_expert_forward_rows(const uint8_t *gate_q4, const uint8_t *up_q4, const void *down_data,
                            int down_format, const float *inputs, float *output, const float *weights,
                            int k, int embed_dim, int inter_dim);

/* tg_moe_forward_rows_v2 with Q4_K gate, SiLU and no biases (libtinygiant.c:1439-1448). */
void tg_moe_forward_rows(const uint8_t *const *gate_ptrs, const uint8_t *const *up_ptrs,
                         const void *const *down_ptrs, const int *down_fmts, int n_experts,
                         const float *row_weights, const float *inputs, float *output, int k, int embed_dim,
                         int inter_dim);

/* Zeroes output, then adds weights[e] * expert_e(x) for all-Q4_K experts
 * (libtinygiant.c:1452-1460). */
void tg_moe_forward(const uint8_t **expert_ptrs, const float *weights, int n_experts, const float *input,
                    float *output, int embed_dim, int inter_dim);

/* Whole decoder layer with fp32 attention and pre-routed experts
 * (libtinygiant.c:1467-1507), built on the GPU entries above; x changes only
 * if every step succeeded. */
void tg_transformer_layer(const float *wq, const float *wk, const float *wv, const float *wo,
                          const float *attn_norm_w, const float *q_norm_w, const float *k_norm_w,
                          const float *ffn_norm_w, float *kv_k, float *kv_v, int kv_len, int kv_max,
                          const float *rope_cos, const float *rope_sin, const uint8_t **gate_ptrs,
                          const uint8_t **up_ptrs, const void **down_ptrs, const int *down_is_f16,
                          const float *expert_weights, int n_active, float *x, int embed_dim, int inter_dim,
                          int n_heads, int n_kv_heads, int head_dim, int pos);

/* ---- Extensions (no counterpart in the reference) ----------------------- */

/* Error of the most recent failed call (0 = none) with its message copied
 * into buf (NUL-terminated, truncated to len); reading clears it. */
int tg_cuda_last_error(char *buf, size_t len);

/* CUDA device used by this process (default: the current device, else 0).
 * Must be called before the first compute call to take effect. */
int tg_cuda_set_device(int device);

/* Runs all later work on the given cudaStream_t (NULL: the library's own
 * stream).  Host-pointer calls still synchronise that stream before return. */
void tg_cuda_set_stream(void *stream);

/* Declares [host_ptr, host_ptr + nbytes) as immutable weight bytes (e.g. a
 * whole mmap'd expert file): matrices inside it are uploaded to HBM on first
 * use and never re-checked.  Matrices outside any declared range are
 * uploaded on first use too, and every later call checks their host bytes
 * against what was uploaded and re-uploads on a change (the policy is
 * tg_cuda_set_weight_check's).  Register only bytes that stay fixed while
 * registered (a mapped expert file); a buffer that is refilled (a pread
 * buffer reused for another expert) must be unregistered before it is
 * refilled, or left unregistered.  0 on success. */
int tg_cuda_register(const void *host_ptr, size_t nbytes);
int tg_cuda_unregister(const void *host_ptr);
void tg_cuda_registry_clear(void);
/* Bytes of HBM the registry holds. */
size_t tg_cuda_registry_bytes(void);
/* Registry counters: matrices uploaded again because their host bytes changed
 * (an unregistered matrix's whole content is fingerprinted on every call that
 * uses it), entries dropped because their host address came back with another
 * shape or format, and the entries held now.  Any pointer may be NULL. */
/* Policy for unregistered host matrices; returns the previous one.
 *   2 (default)  every byte is fingerprinted on every call that uses the
 *                matrix: any change is seen; costs one host pass over the
 *                weights per call (~14 GB/s), about what the reference's CPU
 *                path reads per call;
 *   1            a 96-byte sample (first, middle, last 32 bytes): sees a
 *                buffer refilled with another expert's bytes, not an edit
 *                elsewhere; a few microseconds;
 *   0            no check: host weights never change after first use (the
 *                reference's own assumption for its hot path).
 * Registered ranges (tg_cuda_register) are never checked. */
int tg_cuda_set_weight_check(int mode);
void tg_cuda_registry_stats(uint64_t *reuploads, uint64_t *evictions, size_t *entries);

/* Number of kernels this library has launched since load. */
uint64_t tg_cuda_launch_count(void);

/* ---- Resident layers routed on the GPU ---------------------------------- *
 * A layer holds all n_experts experts (uploaded through the registry), an
 * fp32 router W_r [n_experts][embed_dim] (+ optional bias) and scratch for up
 * to max_tokens rows.  One step = rmsnorm -> router -> top_k softmax ->
 * plan -> experts (engine.py:281-342 + tg_moe_forward_rows_v2), all on the
 * GPU.  Returns NULL on failure. */
void *tg_layer_create(int n_experts, const uint8_t *const *gate_ptrs, const uint8_t *const *up_ptrs,
                      const void *const *down_ptrs, int gate_fmt, const int *down_fmts,
                      const float *const *gate_bias, const float *const *up_bias,
                      const float *const *down_bias, int act, int embed_dim, int inter_dim,
                      const float *router_w, const float *router_b, int top_k, int max_tokens);
/* Expert-parallel shard of a layer: this GPU uploads only experts e with
 * e % n_shards == shard (the router is replicated); its steps produce the
 * local experts' part of the output, to be summed across GPUs. */
void *tg_layer_create_shard(int n_experts, const uint8_t *const *gate_ptrs, const uint8_t *const *up_ptrs,
                            const void *const *down_ptrs, int gate_fmt, const int *down_fmts,
                            const float *const *gate_bias, const float *const *up_bias,
                            const float *const *down_bias, int act, int embed_dim, int inter_dim,
                            const float *router_w, const float *router_b, int top_k, int max_tokens, int shard,
                            int n_shards);
/* A second HBM copy of a layer's weights (for working sets beyond L2). */
void *tg_layer_clone(void *layer);
void tg_layer_destroy(void *layer);
size_t tg_layer_expert_bytes(void *layer, int expert);
/* Enqueue one step on device buffers: x' = x + add (add may be NULL);
 * N = normalize ? rmsnorm(x') * norm_w (NULL: 1) : x'; moe_out = experts(N);
 * x_out = x' (may be NULL).  Asynchronous on the library stream. */
int tg_layer_forward_dev(void *layer, const float *x, const float *add, float *x_out, float *moe_out, int T,
                         int normalize, const float *norm_w);
/* 1 (default): a step runs as one persistent kernel when the batch is
 * decode-sized (T <= 8) and the formats have one; 0: three kernels (router,
 * gate/up, down).  Same results either way.  Returns the previous setting. */
int tg_layer_set_fused(void *layer, int on);
/* Expert parallel with the combine inside the step kernel: each shard
 * stores its part of the output into every shard's receive block over
 * NVLink and sums the parts of its own block in shard order, so no separate
 * all-reduce follows the step.  tg_layer_ep_handle writes the CUDA IPC handle
 * (64 bytes) of this shard's block; tg_layer_ep_connect takes all shards'
 * handles in shard order.  Decode-sized steps of a connected shard return
 * the whole layer's output.  Return 0, or -1 on error. */
int tg_layer_ep_handle(void *layer, void *handle_out);
int tg_layer_ep_connect(void *layer, const void *handles);
/* Restarts the layer's step epochs at 1 (clears its exchange block, arrival
 * counters and, for a shard, its receive block; synchronises).  After any
 * shard of a layer saw an error, every shard calls it, with none of their
 * steps in flight (between two barriers), so that all shards tag and expect
 * the same epochs again.  0 on success. */
int tg_layer_ep_reset(void *layer);
/* 1 (default): batched steps (T > 8) run the expert GEMMs on the tensor
 * cores (tcgen05); 0: the matvec kernels.  Same results either way.  Returns
 * the previous setting. */
int tg_layer_set_tc(void *layer, int on);
/* Replaces a layer's fp32 router [E][D] (and bias [E], or NULL: a layer made
 * with a bias gets zeros, one made without keeps none) from host arrays;
 * stacks give each layer its own.  Returns 0, or -1 on error. */
int tg_layer_set_router(void *layer, const float *router_w, const float *router_b);
/* Diagnostics: fused steps launched after this call write per-CTA phase
 * timestamps into dev_buf (32 uint64 per CTA: SM clocks, the global timer in
 * slots 12/13, the logits poll count in slot 19; then 8 uint64 per warp of
 * ring and poll counters, tg_cuda_step_trace_warps() warps per CTA); NULL
 * stops it.  Returns the step's grid size. */
int tg_cuda_step_trace(void *dev_buf);
/* Warps per CTA of the fused step, i.e. the per-warp trace records per CTA. */
int tg_cuda_step_trace_warps(void);
/* Diagnostics: batched steps' tensor-core GEMM launches after this call write
 * per-CTA role counters into dev_buf ([2][grid][16] uint64: the gate/up pass,
 * then the down pass; cycles the producer, MMA, unpack and epilogue roles
 * waited on each ring, each role's span, units and steps); NULL stops it.
 * Returns the GEMMs' grid size. */
int tg_cuda_tc_trace(void *dev_buf);
/* Tests of the fused step's bounded waits (no device fault is involved):
 * steps launched after this call give up on a poll of another CTA's or GPU's
 * words after poll_limit polls (<= 0: the default, about a second) and
 * record a timeout in the device status; CTA skip_logit_cta (-1: none)
 * publishes no router logits, so every CTA's logits poll runs out.  Steps
 * already captured in a CUDA graph keep the settings they were captured
 * with.  Returns 0. */
int tg_cuda_debug_step_fault(int skip_logit_cta, int poll_limit);
/* Test hook: batched steps on the tensor cores launched after this call write
 * every int32 sub-block sum of their gate/up GEMM into gate_up and of their
 * down GEMM into down (device buffers; NULL: off), at
 * ((plan_row * mats + matrix) * rows + weight_row) * nsb + sub_block with
 * mats 2 (gate, up) or 1 (down), rows the matrix's rows, nsb its row's
 * sub-blocks (Q4_K, MXFP4: values / 32; Q6_K: values / 16 in the order
 * (2 h + l-half) * 4 + quarter per block).  Plan rows are the step's active
 * (expert, token) rows: experts ascending, tokens ascending within each.
 * Layer graphs keep the pointers they were captured with.  Returns 0. */
int tg_cuda_debug_tc_isums(void *gate_up, void *down);
/* Host buffers, synchronous: out[T][D] += experts(normalize ? rmsnorm(x) : x). */
int tg_layer_forward(void *layer, const float *x_host, float *out_host, int T, int normalize);
/* Selected experts and weights [T][top_k] of the layer's last step. */
int tg_layer_last_routing(void *layer, int T, int *idx, float *w);
/* x [T][D] (device) += experts_l(rmsnorm(x) * norm_w[l]) for l = 0..n_layers-1,
 * in place, asynchronous. */
int tg_stack_forward_dev(void *const *layers, int n_layers, float *x, int T, const float *const *norm_w);

/* CUDA graphs over the library stream (capture the enqueued work between
 * begin and end; launch replays it). */
int tg_cuda_graph_begin(void);
void *tg_cuda_graph_end(void);
int tg_cuda_graph_launch(void *graph);
void tg_cuda_graph_destroy(void *graph);
/* The cudaStream_t the library enqueues on; synchronise it and report
 * device-side errors. */
void *tg_cuda_stream(void);
int tg_cuda_synchronize(void);

/* Number of CUDA devices visible to this process (0 without a GPU). */
int tg_cuda_device_count(void);

/* Test hooks exposing the intermediates that must match the reference bit
 * for bit.  tg_cuda_debug_quantize_q8 writes nrows x ceil(ncols/256) blocks
 * in the reference's 296-byte q8_block layout (libtinygiant.c:159-164).
 * tg_cuda_debug_row_isums writes every row's int32 sub-block sums of a
 * quantized matrix against one input given as such blocks (per row: Q4_K 8
 * per block, Q6_K 16 per block, MXFP4 / Q8_0 1 per 32 values) and returns
 * the count per row, or -1. */
int tg_cuda_debug_quantize_q8(const float *x, int nrows, int ncols, void *out_blocks);
int tg_cuda_debug_row_isums(int fmt, const void *mat, int nrows, int ncols, const void *xq_blocks, int32_t *out);
/* Test hook: the fused step's double-assisted exact fp32 division against
 * the IEEE division on n pseudo-random operand pairs; writes the number of
 * results that differ (0 expected).  Returns 0, or -1 on error. */
int tg_cuda_debug_div_check(long long n, unsigned seed, unsigned long long *mismatches);

/* ---- Allocation-free matvec -------------------------------------------- *
 * No counterpart in the reference: an extension for callers that cannot
 * allocate device memory.  out[r] = row r of a Q4_K matrix . input, the
 * arithmetic of tg_matmul_q4k (bit-identical to it), with every pointer
 * caller-owned device memory on the current device: q4_matrix (16-byte
 * aligned, nrows x ncols/256 blocks of 144 bytes, the reference layout),
 * input[ncols], output[nrows].  Enqueued on `stream` (a cudaStream_t; NULL is
 * the default stream) and asynchronous: the caller synchronises.
 * Allocates nothing: the Q8 copy of the input lives in a fixed 80 KiB
 * __device__ array that each GPU loading the library holds until exit, so
 * ncols is limited to 65536 (larger sizes are rejected with error 3).
 * Calls that overlap on one device (several streams or host threads in
 * flight at once) race on that scratch: order them on one stream.  The first
 * call on each device looks up the scratch address; make it outside any
 * stream capture.  The address is kept until exit, so a device that the
 * process resets (cudaDeviceReset) must not be used with this entry point
 * afterwards.  Returns 0 when enqueued, else the error code that
 * tg_cuda_last_error reports. */
int tg_cuda_matmul_q4k_noalloc(const uint8_t *q4_matrix, const float *input, float *output, int nrows, int ncols,
                               void *stream);

#ifdef __cplusplus
}
#endif

#endif /* TINYGIANT_H */
