// tg_moe.h — launchers of the MoE expert kernels (tg_moe.cu) and of the
// fused routing kernel (tg_route.cu).
#pragma once
#include <cuda_runtime.h>

#include "tg_plan.cuh"

namespace tg {

cudaError_t launch_moe_gateup(const PlanHdr* ph, int max_slots, int gate_fmt, int D, int I, const Q8Dev* xq8,
                              float* hidden, Q8Dev* hq8, int* counters, DevStatus* st, cudaStream_t s);
// Down phase for a plan whose experts all use down format down_fmt_all, or,
// with parts_out ([total_rows][D]), the slots of that format only, storing
// their parts for launch_combine_parts.  T: the call's input rows;
// max_slots / max_rows: upper bounds of the plan's slots and active rows.
// hq8 ([max_rows][ceil(I/256)]) receives the Q8 blocks of hidden when
// max_rows is too large for the down kernel to quantize them itself.
cudaError_t launch_moe_down(const PlanHdr* ph, int max_slots, int max_rows, int down_fmt_all, int D, int I, int T,
                            Q8Dev* hq8, const float* hidden, float* out, float* parts_out, DevStatus* st,
                            cudaStream_t s);
cudaError_t launch_combine_parts(const PlanHdr* ph, int D, int T, const float* parts, float* out, cudaStream_t s);
// Ints of zero-initialised counter space the expert kernels need.
size_t moe_counter_ints(int max_slots, int I);

struct RouteArgs {
  const float* x_in;      // [T][D] residual stream before this layer
  const float* add_in;    // [T][D] previous MoE output to add first, or null
  float* x_out;           // [T][D] x_in + add_in (written by CTA 0), or null
  float* zero_out;        // [T][D] buffer to clear for this layer's MoE output, or null
  const float* norm_w;    // [D] RMSNorm weight, or null for 1
  float eps;
  int normalize;          // 1: N = rmsnorm(x'); 0: N = x'
  const float* router_w;  // [E][D] fp32
  const float* router_b;  // [E] or null
  int T, D, E, top_k, I, act, assoc_rule, bias_term;
  const ExpertDesc* experts;  // [E]
  Q8Dev* xq8;             // [T][ceil(D/256)]
  float* logits;          // [T][E]
  int* counter;           // one int, zero between launches
  PlanHdr* plan;
  SlotDesc* slots;        // [min(E, T*top_k)]
  int* rows;              // [T*top_k]
  float* wts;             // [T*top_k]
  int* row_slot;          // [T*top_k]
  int* sel_idx;           // [T][top_k]
  float* sel_w;           // [T][top_k]
  DevStatus* st;          // device error record
};

size_t route_smem_bytes(int D, int E, int T, int K);

// Routing for batched steps (tg_route.cu): the RouteArgs fields plus the
// normalized rows and an expert x row membership matrix.
struct BatchRouteArgs {
  const float* x_in;
  const float* add_in;
  float* x_out;
  float* zero_out;
  const float* norm_w;
  float eps;
  int normalize;
  const float* router_w;
  const float* router_b;
  int T, D, E, top_k, I, act, assoc_rule, bias_term;
  const ExpertDesc* experts;
  Q8Dev* xq8;
  float* nbuf;            // [T][D] normalized rows
  uint8_t* member;        // [E][T] selection rank + 1 of each active (expert, row), else 0
  int* ecnt;              // [E] active rows per expert (zeroed by the norm kernel, counted by select)
  int* tpos;              // [T][top_k] each valid selection's place among its row's, in expert order
  int* tok_rows;          // [T][top_k] each row's active rows (plan indices) in slot order, then -1
  float* logits;
  PlanHdr* plan;
  SlotDesc* slots;
  int* rows;
  float* wts;
  int* row_slot;
  int* sel_idx;
  float* sel_w;
};
cudaError_t launch_batch_route(const BatchRouteArgs& a, cudaStream_t s);

// One expert's weight pointers for the fused step kernel; the row layouts
// follow from the layer's formats and shape.  A null gate marks an expert
// held by another GPU.
struct StepExpert {
  const uint8_t* g;
  const uint8_t* u;
  const uint8_t* d;
  const float* gb;
  const float* ub;
  const float* db;
};
static_assert(sizeof(StepExpert) == 48, "StepExpert is copied in 16-byte units");

// Words of the fused step's exchange block for a layer of E experts, top_k,
// intermediate I and up to T rows per step: the launch counter, the tagged
// logits [T][E] and the tagged hidden activations [T*top_k][ceil(I/256)][256].
// All zero at creation (and after an error reset).
size_t step_sync_words(int T, int E, int top_k, int I);

// One layer step (routing + experts) as a single persistent kernel, for
// decode-sized batches (tg_step.cu).  `out` is overwritten with the MoE
// output.
struct StepLaunch {
  const float* x_in;
  const float* add_in;
  float* x_out;
  const float* norm_w;
  float eps;
  int normalize;
  const float* router_w;
  const float* router_b;
  int T, D, E, top_k, I, act, assoc_rule, bias_term, gate_fmt, down_fmt;
  const StepExpert* etab;     // [E]
  float* logits;              // [T][E]
  float* out;                 // [T][D]
  int* sel_idx;               // [T][top_k]
  float* sel_w;               // [T][top_k]
  unsigned long long* sync;   // the exchange block (step_sync_words), 256-byte aligned
  DevStatus* st;
  // expert parallel, combined inside the kernel: every GPU stores its part of
  // the output as tagged words into slot ep_rank of every GPU's receive block
  // [ep_world][T][D] (ep_peers: those blocks, mapped into this process) and
  // sums the ep_world parts of its own block in rank order.  ep_world 1: off.
  int ep_rank = 0, ep_world = 1;
  unsigned long long* const* ep_peers = nullptr;   // device array [ep_world]
  const unsigned long long* ep_recv = nullptr;     // this GPU's receive block
};
bool step_eligible(const StepLaunch& l);
cudaError_t launch_layer_step(const StepLaunch& l, cudaStream_t s);
// Diagnostics: later step launches write [grid][16] phase timestamps to p
// (device memory; null turns it off).
void set_step_trace(void* p);
// Warps per CTA of the fused step kernel (the trace's per-warp records).
int step_warps();
// Tests of the bounded waits: later step launches give up after poll_limit
// polls of another CTA's or GPU's words (<= 0: the default, about a second),
// and CTA skip_logit_cta (-1: none) publishes no logits, so every CTA's
// logits poll runs out and the step reports a timeout.
void set_step_fault(int skip_logit_cta, int poll_limit);
cudaError_t launch_layer_route(const RouteArgs& a, cudaStream_t s);
// Batched steps on the tensor cores (tg_gemm.cu): for a plan written by the
// route kernel, the gate/up and down grouped GEMMs (tcgen05, exact per
// sub-block int32 sums), the activation and Q8 of hidden, and the ordered
// combine into out (which the route kernel zeroed).  K: top_k; max_rows:
// T * top_k; scratch: tc_moe_scratch_bytes of device memory.
// MXFP4 matrices are read through TMA tensor maps, [E][3] (gate, up, down)
// in device memory: tc_tmap_bytes(E) of them, written by tc_build_tmaps
// from the layer's expert table (entries of absent or other-format
// matrices are zero).
bool tc_moe_eligible(int gate_fmt, int down_fmt, int D, int I);
size_t tc_moe_scratch_bytes(int max_rows, int T, int K, int D, int I);
size_t tc_tmap_bytes(int E);
cudaError_t tc_build_tmaps(const ExpertDesc* experts, int E, void* d_tmaps);
// Test hook: later grouped-GEMM passes write every int32 sub-block sum of the
// gate/up pass into gate_up and of the down pass into down (device memory,
// [plan row][matrix][weight row][sub-block], tc_debug_isum_index); null: off.
void set_tc_debug(int* gate_up, int* down);
// Diagnostics: per-CTA role counters of later grouped-GEMM launches into p
// ([2][tc_trace_ctas()][16]: gate/up pass, then down), or off (null).
void set_tc_trace(void* p);
int tc_trace_ctas();
cudaError_t launch_tc_moe(const PlanHdr* ph, int gate_fmt, int down_fmt, int T, int K, int D, int I, int max_rows,
                          const Q8Dev* xq8, const int* tok_rows, const void* tmaps, void* scratch, float* out,
                          DevStatus* st, cudaStream_t s);

}  // namespace tg
