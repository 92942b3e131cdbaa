// tg_layer.cu — HBM-resident MoE layers and stacks, routed on the GPU.
//
// The reference engine keeps experts on disk / in the page cache and routes
// in numpy before every MoE call (tinygiant/engine.py:281-342).  Here a
// layer's experts, router and scratch live in HBM; one layer step is three
// kernels on one stream (fused norm + router + plan build, gate/up +
// activation + Q8, down + combine) with no host round trip, so steps and
// whole stacks can be captured in a CUDA graph.  Expert weights come from the
// same registry as the reference-ABI calls (uploaded once, repacked).
#include <cstring>
#include <vector>

#include "../../include/tinygiant.h"
#include "tg_kernels.h"
#include "tg_moe.h"
#include "tg_runtime.h"

namespace tg {

struct Layer {
  int E = 0, D = 0, I = 0, gate_fmt = 0, down_fmt = 0, act = 0, top_k = 0, max_tokens = 0;
  int max_slots = 0, max_rows = 0;
  std::vector<ExpertDesc> experts;  // host copy of the device table
  std::vector<void*> owned;         // device allocations to free
  ExpertDesc* d_experts = nullptr;
  StepExpert* d_step = nullptr;     // [E] weight pointers for the fused step kernel
  float* router_w = nullptr;
  float* router_b = nullptr;
  // scratch
  Q8Dev* xq8 = nullptr;
  float* logits = nullptr;
  int* counter = nullptr;
  PlanHdr* plan = nullptr;
  SlotDesc* slots = nullptr;
  int* rows = nullptr;
  float* wts = nullptr;
  int* row_slot = nullptr;
  int* sel_idx = nullptr;
  float* sel_w = nullptr;
  float* hidden = nullptr;
  Q8Dev* hq8 = nullptr;
  int* counters = nullptr;
  unsigned long long* step_sync = nullptr;   // the fused step kernel's exchange block (step_sync_words)
  bool fused = true;               // use the fused step kernel when the shape allows
  bool tc = true;                  // batched steps (T > 8) on the tensor-core grouped GEMMs
  void* tc_scratch = nullptr;      // their intermediates (tc_moe_scratch_bytes)
  void* tc_tmaps = nullptr;        // batched layers: TMA tensor maps [E][6] of the expert matrices (tc_build_tmaps)
  float* nbuf = nullptr;           // batched routing: normalized rows [max_tokens][D]
  uint8_t* member = nullptr;       // batched routing: [E][rows of the step] selection membership
  int* ecnt = nullptr;             // batched routing: [E] active rows per expert
  int* tpos = nullptr;             // batched routing: [max_tokens][top_k]
  int* tok_rows = nullptr;         // batched routing: [max_tokens][top_k] active rows per token
  // tg_layer_forward's CUDA graph (copy in, step, copies out) for one
  // (rows, normalize, host staging buffers, stream)
  cudaGraphExec_t fwd_exec = nullptr;
  int fwd_T = 0, fwd_norm = -1;
  const void* fwd_hx = nullptr;
  const void* fwd_ho = nullptr;
  cudaStream_t fwd_s = nullptr;
  // expert-parallel combine inside the step kernel: this GPU's receive block
  // [n_shards][max_tokens][D] of tagged words, and the blocks of every shard
  // mapped into this process (tg_layer_ep_connect)
  int shard = 0, n_shards = 1;
  unsigned long long* ep_recv = nullptr;
  unsigned long long** ep_peers_d = nullptr;   // device array [n_shards]
  std::vector<void*> ep_opened;                // peer mappings to close
  bool ep_connected = false;
  float* moe_out = nullptr;  // [2][max_tokens][D] for stacks and the host entry
  float* xbuf = nullptr;     // [max_tokens][D]
};

static bool dmalloc(Layer* L, void** p, size_t n) {
  n = (n + 255) & ~(size_t)255;
  if (cudaMalloc(p, n) != cudaSuccess) {
    cudaGetLastError();
    set_host_error(101, "cudaMalloc(%zu bytes) failed for a layer", n);
    return false;
  }
  L->owned.push_back(*p);
  return cudaMemset(*p, 0, n) == cudaSuccess;
}

// Receive block of the in-kernel expert-parallel combine: [n_shards][T][D]
// tagged words for up to the fused step's 8 rows.
static size_t ep_recv_bytes(const Layer* L) {
  return sizeof(unsigned long long) * (size_t)L->n_shards * std::min(L->max_tokens, 8) * L->D;
}

static bool alloc_scratch(Layer* L) {
  const int T = L->max_tokens, D = L->D, I = L->I, E = L->E;
  const int gbpr = (D + QK - 1) / QK, dbpr = (I + QK - 1) / QK;
  L->max_rows = T * L->top_k;
  L->max_slots = std::min(E, L->max_rows);
  return dmalloc(L, (void**)&L->xq8, sizeof(Q8Dev) * (size_t)T * gbpr) &&
         dmalloc(L, (void**)&L->logits, sizeof(float) * (size_t)T * E) &&
         dmalloc(L, (void**)&L->counter, sizeof(int)) && dmalloc(L, (void**)&L->plan, sizeof(PlanHdr)) &&
         dmalloc(L, (void**)&L->slots, sizeof(SlotDesc) * (size_t)L->max_slots) &&
         dmalloc(L, (void**)&L->rows, sizeof(int) * (size_t)L->max_rows) &&
         dmalloc(L, (void**)&L->wts, sizeof(float) * (size_t)L->max_rows) &&
         dmalloc(L, (void**)&L->row_slot, sizeof(int) * (size_t)L->max_rows) &&
         dmalloc(L, (void**)&L->sel_idx, sizeof(int) * (size_t)L->max_rows) &&
         dmalloc(L, (void**)&L->sel_w, sizeof(float) * (size_t)L->max_rows) &&
         dmalloc(L, (void**)&L->hidden, sizeof(float) * (size_t)L->max_rows * I) &&
         dmalloc(L, (void**)&L->hq8, sizeof(Q8Dev) * (size_t)L->max_rows * dbpr) &&
         dmalloc(L, (void**)&L->counters, sizeof(int) * moe_counter_ints(L->max_slots, I)) &&
         (register_counters(L->counters, sizeof(int) * moe_counter_ints(L->max_slots, I)), true) &&
         dmalloc(L, (void**)&L->step_sync, sizeof(unsigned long long) * step_sync_words(T, E, L->top_k, I)) &&
         (register_counters(L->step_sync, sizeof(unsigned long long) * step_sync_words(T, E, L->top_k, I)), true) &&
         (T <= 8 || (dmalloc(L, (void**)&L->nbuf, sizeof(float) * (size_t)T * D) &&
                     dmalloc(L, (void**)&L->member, (size_t)T * E) &&
                     dmalloc(L, (void**)&L->ecnt, sizeof(int) * 256) &&
                     dmalloc(L, (void**)&L->tpos, sizeof(int) * (size_t)L->max_rows) &&
                     dmalloc(L, (void**)&L->tok_rows, sizeof(int) * (size_t)L->max_rows))) &&
         (!(T > 8 && tc_moe_eligible(L->gate_fmt, L->down_fmt, D, I)) ||
          (dmalloc(L, &L->tc_scratch, tc_moe_scratch_bytes(L->max_rows, T, L->top_k, D, I)) &&
           dmalloc(L, &L->tc_tmaps, tc_tmap_bytes(E)) &&
           tc_build_tmaps(L->experts.data(), E, L->tc_tmaps) == cudaSuccess)) &&
         (L->n_shards == 1 ||
          (dmalloc(L, (void**)&L->ep_recv, ep_recv_bytes(L)) &&
           (register_counters(L->ep_recv, ep_recv_bytes(L)), true) &&
           dmalloc(L, (void**)&L->ep_peers_d, sizeof(void*) * (size_t)L->n_shards))) &&
         dmalloc(L, (void**)&L->moe_out, sizeof(float) * 2 * (size_t)T * D) &&
         dmalloc(L, (void**)&L->xbuf, sizeof(float) * (size_t)T * D);
}

// Device copies of the expert table and of the step kernel's pointer table.
static bool upload_tables(Layer* L) {
  std::vector<StepExpert> st(L->E);
  for (int e = 0; e < L->E; e++) {
    const ExpertDesc& X = L->experts[e];
    st[e] = StepExpert{X.gate.main, X.up.main, X.down.main, X.gb, X.ub, X.db};
  }
  if (!dmalloc(L, (void**)&L->d_experts, sizeof(ExpertDesc) * L->E) ||
      !dmalloc(L, (void**)&L->d_step, sizeof(StepExpert) * L->E))
    return false;
  return cudaMemcpy(L->d_experts, L->experts.data(), sizeof(ExpertDesc) * L->E, cudaMemcpyHostToDevice) ==
             cudaSuccess &&
         cudaMemcpy(L->d_step, st.data(), sizeof(StepExpert) * L->E, cudaMemcpyHostToDevice) == cudaSuccess;
}

static void free_layer(Layer* L) {
  if (L->fwd_exec) cudaGraphExecDestroy(L->fwd_exec);
  for (void* p : L->ep_opened) cudaIpcCloseMemHandle(p);
  if (L->ep_recv) unregister_counters(L->ep_recv);
  if (L->counters) unregister_counters(L->counters);
  if (L->step_sync) unregister_counters(L->step_sync);
  for (void* p : L->owned) cudaFree(p);
  delete L;
}

// Enqueues one layer step: x' = x + add (if add), N = rmsnorm(x') or x',
// moe_out = 0, moe_out += experts(N); x_out = x' (if x_out).
static bool layer_enqueue(Layer* L, const float* x, const float* add, float* x_out, float* moe_out, int T,
                          int normalize, const float* norm_w, cudaStream_t s, const char* what) {
  if (T < 1 || T > L->max_tokens) {
    set_host_error(3, "%s: %d rows exceed the layer's max_tokens %d", what, T, L->max_tokens);
    return false;
  }
  StepLaunch sl{};
  sl.x_in = x;
  sl.add_in = add;
  sl.x_out = x_out;
  sl.norm_w = norm_w;
  sl.eps = 1e-6f;
  sl.normalize = normalize;
  sl.router_w = L->router_w;
  sl.router_b = L->router_b;
  sl.T = T;
  sl.D = L->D;
  sl.E = L->E;
  sl.top_k = L->top_k;
  sl.I = L->I;
  sl.act = L->act;
  sl.assoc_rule = ASSOC_MOE;
  sl.bias_term = 1;
  sl.gate_fmt = L->gate_fmt;
  sl.down_fmt = L->down_fmt;
  sl.etab = L->d_step;
  sl.logits = L->logits;
  sl.out = moe_out;
  sl.sel_idx = L->sel_idx;
  sl.sel_w = L->sel_w;
  sl.sync = L->step_sync;
  sl.st = status_ptr();
  if (L->ep_connected) {
    sl.ep_rank = L->shard;
    sl.ep_world = L->n_shards;
    sl.ep_peers = L->ep_peers_d;
    sl.ep_recv = L->ep_recv;
  }
  if (L->fused && step_eligible(sl)) {
    const cudaError_t e = launch_layer_step(sl, s);
    count_launches(1);
    if (e != cudaSuccess) {
      set_host_error(100 + (int)e, "%s: %s", what, cudaGetErrorString(e));
      return false;
    }
    return true;
  }
  RouteArgs a{};
  a.x_in = x;
  a.add_in = add;
  a.x_out = x_out;
  a.zero_out = moe_out;
  a.norm_w = norm_w;
  a.eps = 1e-6f;
  a.normalize = normalize;
  a.router_w = L->router_w;
  a.router_b = L->router_b;
  a.T = T;
  a.D = L->D;
  a.E = L->E;
  a.top_k = L->top_k;
  a.I = L->I;
  a.act = L->act;
  a.assoc_rule = ASSOC_MOE;
  a.bias_term = 1;
  a.experts = L->d_experts;
  a.xq8 = L->xq8;
  a.logits = L->logits;
  a.counter = L->counter;
  a.plan = L->plan;
  a.slots = L->slots;
  a.rows = L->rows;
  a.wts = L->wts;
  a.row_slot = L->row_slot;
  a.sel_idx = L->sel_idx;
  a.sel_w = L->sel_w;
  a.st = status_ptr();
  cudaError_t e;
  if (T > 8 && L->nbuf) {
    BatchRouteArgs b{};
    b.x_in = x;
    b.add_in = add;
    b.x_out = x_out;
    b.zero_out = moe_out;
    b.norm_w = norm_w;
    b.eps = 1e-6f;
    b.normalize = normalize;
    b.router_w = L->router_w;
    b.router_b = L->router_b;
    b.T = T;
    b.D = L->D;
    b.E = L->E;
    b.top_k = L->top_k;
    b.I = L->I;
    b.act = L->act;
    b.assoc_rule = ASSOC_MOE;
    b.bias_term = 1;
    b.experts = L->d_experts;
    b.xq8 = L->xq8;
    b.nbuf = L->nbuf;
    b.member = L->member;
    b.ecnt = L->ecnt;
    b.tpos = L->tpos;
    b.tok_rows = L->tok_rows;
    b.logits = L->logits;
    b.plan = L->plan;
    b.slots = L->slots;
    b.rows = L->rows;
    b.wts = L->wts;
    b.row_slot = L->row_slot;
    b.sel_idx = L->sel_idx;
    b.sel_w = L->sel_w;
    e = launch_batch_route(b, s);
    count_launches(4);
  } else {
    e = launch_layer_route(a, s);
    count_launches(1);
  }
  if (L->tc && L->tc_scratch && T > 8) {
    if (e == cudaSuccess)
      e = launch_tc_moe(L->plan, L->gate_fmt, L->down_fmt, T, L->top_k, L->D, L->I, T * L->top_k, L->xq8,
                        L->tok_rows, L->tc_tmaps, L->tc_scratch, moe_out, status_ptr(), s);
    count_launches(4);
    if (e != cudaSuccess) {
      set_host_error(100 + (int)e, "%s: %s", what, cudaGetErrorString(e));
      return false;
    }
    return true;
  }
  if (e == cudaSuccess)
    e = launch_moe_gateup(L->plan, std::min(L->max_slots, T * L->top_k), L->gate_fmt, L->D, L->I, L->xq8, L->hidden,
                          L->hq8, L->counters, status_ptr(), s);
  if (e == cudaSuccess)
    e = launch_moe_down(L->plan, std::min(L->max_slots, T * L->top_k), T * L->top_k, L->down_fmt, L->D, L->I, T, L->hq8,
                        L->hidden,
                        moe_out, nullptr, status_ptr(), s);
  count_launches(2);
  if (e != cudaSuccess) {
    set_host_error(100 + (int)e, "%s: %s", what, cudaGetErrorString(e));
    return false;
  }
  return true;
}

}  // namespace tg

using namespace tg;

extern "C" {

// Expert-parallel shard: this GPU holds experts e with e % n_shards == shard
// (the router is replicated); a step computes only the local experts' part.
void* tg_layer_create_shard(int n_experts, const uint8_t* const* gate_ptrs, const uint8_t* const* up_ptrs,
                            const void* const* down_ptrs, int gate_fmt, const int* down_fmts,
                            const float* const* gate_bias, const float* const* up_bias, const float* const* down_bias,
                            int act, int embed_dim, int inter_dim, const float* router_w, const float* router_b,
                            int top_k, int max_tokens, int shard, int n_shards) {
  std::lock_guard<std::recursive_mutex> lk(ctx_mutex());
  const char* what = "tg_layer_create";
  if (n_shards < 1 || shard < 0 || shard >= n_shards) {
    set_host_error(3, "%s: shard %d of %d", what, shard, n_shards);
    return nullptr;
  }
  if (n_experts < 1 || top_k < 1 || top_k > 8 || top_k > n_experts || max_tokens < 1 || !router_w) {
    set_host_error(3, "%s: bad arguments (n_experts %d, top_k %d in 1..8, max_tokens %d, router %p)", what, n_experts,
                   top_k, max_tokens, (const void*)router_w);
    return nullptr;
  }
  if (!(gate_fmt == FMT_Q4K || gate_fmt == FMT_Q6K || gate_fmt == FMT_MXFP4 || gate_fmt == FMT_Q80)) {
    set_host_error(4, "%s: gate format %d is not supported", what, gate_fmt);
    return nullptr;
  }
  if (gate_bias && !up_bias) {
    set_host_error(4, "%s: gate_bias given without up_bias", what);
    return nullptr;
  }
  for (int e = 1; e < n_experts; e++)
    if (down_fmts[e] != down_fmts[0]) {
      set_host_error(4, "%s: experts of a resident layer share one down format (expert %d: %d, expert 0: %d)", what,
                     e, down_fmts[e], down_fmts[0]);
      return nullptr;
    }
  if (!ensure_init()) return nullptr;
  Layer* L = new Layer;
  L->E = n_experts;
  L->D = embed_dim;
  L->I = inter_dim;
  L->gate_fmt = gate_fmt;
  L->down_fmt = down_fmts[0];
  L->act = act == ACT_GPTOSS ? ACT_GPTOSS : ACT_SILU;
  L->top_k = top_k;
  L->max_tokens = max_tokens;
  L->shard = shard;
  L->n_shards = n_shards;
  L->experts.resize(n_experts);
  for (int e = 0; e < n_experts; e++) {
    ExpertDesc& X = L->experts[e];
    memset(&X, 0, sizeof X);
    if (e % n_shards != shard) continue;   // held by another GPU
    if (!lookup_matrix(gate_ptrs[e], gate_fmt, inter_dim, embed_dim, &X.gate) ||
        !lookup_matrix(up_ptrs[e], gate_fmt, inter_dim, embed_dim, &X.up) ||
        !lookup_matrix(down_ptrs[e], down_fmts[e], embed_dim, inter_dim, &X.down)) {
      free_layer(L);
      return nullptr;
    }
    if (gate_bias) {
      X.gb = lookup_vector(gate_bias[e], inter_dim);
      X.ub = lookup_vector(up_bias[e], inter_dim);
    }
    if (down_bias) X.db = lookup_vector(down_bias[e], embed_dim);
  }
  const size_t rw = sizeof(float) * (size_t)n_experts * embed_dim;
  if (!upload_tables(L) || !dmalloc(L, (void**)&L->router_w, rw) ||
      (router_b && !dmalloc(L, (void**)&L->router_b, sizeof(float) * n_experts)) || !alloc_scratch(L)) {
    free_layer(L);
    return nullptr;
  }
  cudaMemcpy(L->router_w, router_w, rw, cudaMemcpyHostToDevice);
  if (router_b) cudaMemcpy(L->router_b, router_b, sizeof(float) * n_experts, cudaMemcpyHostToDevice);
  if (cudaGetLastError() != cudaSuccess) {
    set_host_error(100, "%s: upload failed", what);
    free_layer(L);
    return nullptr;
  }
  return L;
}

void* tg_layer_create(int n_experts, const uint8_t* const* gate_ptrs, const uint8_t* const* up_ptrs,
                      const void* const* down_ptrs, int gate_fmt, const int* down_fmts, const float* const* gate_bias,
                      const float* const* up_bias, const float* const* down_bias, int act, int embed_dim,
                      int inter_dim, const float* router_w, const float* router_b, int top_k, int max_tokens) {
  return tg_layer_create_shard(n_experts, gate_ptrs, up_ptrs, down_ptrs, gate_fmt, down_fmts, gate_bias, up_bias,
                               down_bias, act, embed_dim, inter_dim, router_w, router_b, top_k, max_tokens, 0, 1);
}

// A second resident copy of a layer: every expert weight byte and the router
// are copied to fresh HBM (used to measure with working sets beyond L2).
void* tg_layer_clone(void* handle) {
  std::lock_guard<std::recursive_mutex> lk(ctx_mutex());
  Layer* src = (Layer*)handle;
  if (!src) return nullptr;
  Layer* L = new Layer;
  L->E = src->E;
  L->D = src->D;
  L->I = src->I;
  L->gate_fmt = src->gate_fmt;
  L->down_fmt = src->down_fmt;
  L->act = src->act;
  L->top_k = src->top_k;
  L->max_tokens = src->max_tokens;
  L->fused = src->fused;
  L->tc = src->tc;
  L->shard = src->shard;
  L->n_shards = src->n_shards;
  L->experts = src->experts;
  auto copy_w = [&](WDesc& w) -> bool {
    if (!w.main) return true;   // expert held by another GPU
    const size_t bytes = (size_t)w.rows * w.rs;
    void* p = nullptr;
    if (!dmalloc(L, &p, bytes + 64)) return false;
    if (cudaMemcpy(p, w.main, bytes, cudaMemcpyDeviceToDevice) != cudaSuccess) return false;
    const uint8_t* m = (const uint8_t*)p;
    if (w.aux1) w.aux1 = m + (w.aux1 - w.main);
    if (w.aux2) w.aux2 = m + (w.aux2 - w.main);
    w.main = m;
    return true;
  };
  for (auto& X : L->experts)
    if (!copy_w(X.gate) || !copy_w(X.up) || !copy_w(X.down)) {
      free_layer(L);
      return nullptr;
    }
  const size_t rw = sizeof(float) * (size_t)L->E * L->D;
  if (!upload_tables(L) || !dmalloc(L, (void**)&L->router_w, rw) ||
      (src->router_b && !dmalloc(L, (void**)&L->router_b, sizeof(float) * L->E)) || !alloc_scratch(L)) {
    free_layer(L);
    return nullptr;
  }
  cudaMemcpy(L->router_w, src->router_w, rw, cudaMemcpyDeviceToDevice);
  if (src->router_b) cudaMemcpy(L->router_b, src->router_b, sizeof(float) * L->E, cudaMemcpyDeviceToDevice);
  return L;
}

void tg_layer_destroy(void* handle) {
  std::lock_guard<std::recursive_mutex> lk(ctx_mutex());
  if (!handle) return;
  cudaStreamSynchronize(stream());
  free_layer((Layer*)handle);
}

// Bytes of expert weights of one expert of the layer (gate + up + down, HBM layout).
size_t tg_layer_expert_bytes(void* handle, int e) {
  Layer* L = (Layer*)handle;
  if (!L || e < 0 || e >= L->E) return 0;
  const ExpertDesc& X = L->experts[e];
  if (!X.gate.main) return 0;
  return (size_t)X.gate.rows * host_row_bytes(X.gate.fmt, X.gate.cols) +
         (size_t)X.up.rows * host_row_bytes(X.up.fmt, X.up.cols) +
         (size_t)X.down.rows * host_row_bytes(X.down.fmt, X.down.cols);
}

// Device-resident step, enqueued on the library stream (no synchronisation):
// x' = x + add (add may be NULL), N = normalize ? rmsnorm(x') * norm_w : x',
// moe_out = sum over the selected experts (cleared first), x_out = x' (may be NULL).
// Diagnostics: fused steps launched after this call record per-CTA phase
// timestamps into dev_buf ([grid][16] uint64, device memory); NULL stops it.
// Returns the grid size a fused step uses.
// Restarts the layer's step epochs at 1: clears its exchange block (launch
// counter, tagged logits and hidden words), its arrival counters and, for an
// expert-parallel shard, its receive block, then synchronises.  The shards of
// one layer call it together, with no step of theirs in flight (between a
// barrier after their last step and one before their next), after any of
// them saw an error: a shard that reset alone would tag its words with
// epochs its peers no longer wait for.
int tg_layer_ep_reset(void* handle) {
  std::lock_guard<std::recursive_mutex> lk(ctx_mutex());
  Layer* L = (Layer*)handle;
  if (!L || !ensure_init()) return -1;
  cudaStream_t s = stream();
  bool ok = cudaMemsetAsync(L->step_sync, 0, sizeof(unsigned long long) * step_sync_words(L->max_tokens, L->E,
                                                                                          L->top_k, L->I), s) ==
            cudaSuccess;
  ok = ok && cudaMemsetAsync(L->counters, 0, sizeof(int) * moe_counter_ints(L->max_slots, L->I), s) == cudaSuccess;
  if (L->ep_recv) ok = ok && cudaMemsetAsync(L->ep_recv, 0, ep_recv_bytes(L), s) == cudaSuccess;
  ok = ok && cudaStreamSynchronize(s) == cudaSuccess;
  if (!ok) {
    const cudaError_t e = cudaGetLastError();
    set_host_error(100 + (int)e, "tg_layer_ep_reset: %s", cudaGetErrorString(e));
    return -1;
  }
  return 0;
}

int tg_cuda_debug_tc_isums(void* gate_up, void* down) {
  set_tc_debug(static_cast<int*>(gate_up), static_cast<int*>(down));
  return 0;
}

int tg_cuda_tc_trace(void* dev_buf) {
  std::lock_guard<std::recursive_mutex> lk(ctx_mutex());
  set_tc_trace(dev_buf);
  return tc_trace_ctas();
}

int tg_cuda_debug_step_fault(int skip_logit_cta, int poll_limit) {
  set_step_fault(skip_logit_cta, poll_limit);
  return 0;
}

int tg_cuda_step_trace(void* dev_buf) {
  set_step_trace(dev_buf);
  int dev = 0, sms = 0;
  cudaGetDevice(&dev);
  cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
  return sms;
}

int tg_cuda_step_trace_warps(void) { return step_warps(); }

// Selects the fused single-kernel step (on = 1, the default) or the
// three-kernel step (on = 0) for this layer.  Returns the previous setting.
// Replaces a layer's router with host arrays router_w [E][D] and router_b
// [E] (or NULL for none; a layer created without a bias keeps none).
int tg_layer_set_router(void* handle, const float* router_w, const float* router_b) {
  std::lock_guard<std::recursive_mutex> lk(ctx_mutex());
  const char* what = "tg_layer_set_router";
  Layer* L = static_cast<Layer*>(handle);
  if (!L || !router_w) {
    set_host_error(3, "%s: null layer or router", what);
    return -1;
  }
  if (router_b && !L->router_b) {
    set_host_error(3, "%s: the layer was created without a router bias", what);
    return -1;
  }
  cudaStream_t s = stream();
  bool ok = cudaStreamSynchronize(s) == cudaSuccess &&
            cudaMemcpy(L->router_w, router_w, sizeof(float) * (size_t)L->E * L->D, cudaMemcpyHostToDevice) == cudaSuccess;
  if (ok && L->router_b)
    ok = router_b ? cudaMemcpy(L->router_b, router_b, sizeof(float) * L->E, cudaMemcpyHostToDevice) == cudaSuccess
                  : cudaMemset(L->router_b, 0, sizeof(float) * L->E) == cudaSuccess;
  if (!ok) {
    set_host_error(100, "%s: upload failed", what);
    return -1;
  }
  return 0;
}

// Selects the tensor-core grouped GEMMs (on = 1, the default) or the matvec
// kernels (on = 0) for batched steps (T > 8).  Returns the previous setting.
int tg_layer_set_tc(void* handle, int on) {
  Layer* L = static_cast<Layer*>(handle);
  if (!L) return -1;
  const int prev = L->tc ? 1 : 0;
  L->tc = on != 0;
  return prev;
}

// Expert-parallel combine inside the step kernel.  tg_layer_ep_handle writes
// the CUDA IPC handle of this shard's receive block (64 bytes);
// tg_layer_ep_connect takes every shard's handle, in shard order, and maps
// the other shards' blocks into this process.
int tg_layer_ep_handle(void* handle, void* out) {
  std::lock_guard<std::recursive_mutex> lk(ctx_mutex());
  Layer* L = static_cast<Layer*>(handle);
  if (!L || !out || !L->ep_recv) {
    set_host_error(3, "tg_layer_ep_handle: not an expert-parallel shard");
    return -1;
  }
  cudaIpcMemHandle_t h;
  if (cudaIpcGetMemHandle(&h, L->ep_recv) != cudaSuccess) {
    set_host_error(100, "tg_layer_ep_handle: %s", cudaGetErrorString(cudaGetLastError()));
    return -1;
  }
  memcpy(out, &h, sizeof(h));
  return 0;
}

int tg_layer_ep_connect(void* handle, const void* handles) {
  std::lock_guard<std::recursive_mutex> lk(ctx_mutex());
  const char* what = "tg_layer_ep_connect";
  Layer* L = static_cast<Layer*>(handle);
  if (!L || !handles || !L->ep_recv || L->ep_connected) {
    set_host_error(3, "%s: not an unconnected expert-parallel shard", what);
    return -1;
  }
  std::vector<unsigned long long*> ptrs(L->n_shards);
  for (int p = 0; p < L->n_shards; p++) {
    if (p == L->shard) {
      ptrs[p] = L->ep_recv;
      continue;
    }
    cudaIpcMemHandle_t h;
    memcpy(&h, static_cast<const uint8_t*>(handles) + (size_t)p * sizeof(h), sizeof(h));
    void* dp = nullptr;
    if (cudaIpcOpenMemHandle(&dp, h, cudaIpcMemLazyEnablePeerAccess) != cudaSuccess) {
      set_host_error(100, "%s: shard %d: %s", what, p, cudaGetErrorString(cudaGetLastError()));
      return -1;
    }
    L->ep_opened.push_back(dp);
    ptrs[p] = static_cast<unsigned long long*>(dp);
  }
  if (cudaMemcpy(L->ep_peers_d, ptrs.data(), sizeof(void*) * ptrs.size(), cudaMemcpyHostToDevice) != cudaSuccess) {
    set_host_error(100, "%s: upload failed", what);
    return -1;
  }
  L->ep_connected = true;
  return 0;
}

int tg_layer_set_fused(void* handle, int on) {
  Layer* L = static_cast<Layer*>(handle);
  if (!L) return -1;
  const int prev = L->fused ? 1 : 0;
  L->fused = on != 0;
  return prev;
}

int tg_layer_forward_dev(void* handle, const float* x, const float* add, float* x_out, float* moe_out, int T,
                         int normalize, const float* norm_w) {
  std::lock_guard<std::recursive_mutex> lk(ctx_mutex());
  if (!handle || !ensure_init()) return -1;
  return layer_enqueue((Layer*)handle, x, add, x_out, moe_out, T, normalize, norm_w, stream(),
                       "tg_layer_forward_dev")
             ? 0
             : -1;
}

// Host buffers, synchronous: out[T][D] += experts(rmsnorm(x)) (normalize=1)
// or experts(x) (normalize=0).
int tg_layer_forward(void* handle, const float* x_host, float* out_host, int T, int normalize) {
  std::lock_guard<std::recursive_mutex> lk(ctx_mutex());
  const char* what = "tg_layer_forward";
  Layer* L = (Layer*)handle;
  if (!L || !ensure_init()) return -1;
  if (T < 1 || T > L->max_tokens) {
    set_host_error(3, "%s: %d rows exceed max_tokens %d", what, T, L->max_tokens);
    return -1;
  }
  const size_t n = sizeof(float) * (size_t)T * L->D;
  float* hx = fetch_reserve((size_t)T * L->D);     // mapped: the device reads it
  float* ho = deliver_reserve((size_t)T * L->D);   // mapped: the device writes it
  if (!hx || !ho) return -1;
  cudaStream_t s = stream();
  memcpy(hx, x_host, n);
  float* moe = L->moe_out;
  // The step's device work — the fetch of x from mapped host memory, the
  // step, and the delivery of its output and of the device status into
  // mapped host memory — is one CUDA graph per (rows, normalize, staging
  // buffers, stream), captured on first use and replayed; the host then
  // waits on the delivery's echo instead of synchronising the stream.
  const bool same = L->fwd_exec && L->fwd_T == T && L->fwd_norm == normalize && L->fwd_hx == hx &&
                    L->fwd_ho == ho && L->fwd_s == s;
  if (!same && s != nullptr && s != cudaStreamLegacy && s != cudaStreamPerThread) {
    if (L->fwd_exec) cudaGraphExecDestroy(L->fwd_exec);
    L->fwd_exec = nullptr;
    cudaGraph_t graph = nullptr;
    bool ok = cudaStreamBeginCapture(s, cudaStreamCaptureModeThreadLocal) == cudaSuccess;
    if (ok) {
      ok = fetch_async(L->xbuf, (size_t)T * L->D, s, what) &&
           layer_enqueue(L, L->xbuf, nullptr, nullptr, moe, T, normalize, nullptr, s, what) &&
           deliver_async(moe, (size_t)T * L->D, s, what);
      ok = cudaStreamEndCapture(s, &graph) == cudaSuccess && ok;
    }
    if (ok) ok = cudaGraphInstantiate(&L->fwd_exec, graph, 0) == cudaSuccess;
    if (graph) cudaGraphDestroy(graph);
    if (!ok) {
      if (L->fwd_exec) cudaGraphExecDestroy(L->fwd_exec);
      L->fwd_exec = nullptr;
      cudaGetLastError();
    } else {
      L->fwd_T = T;
      L->fwd_norm = normalize;
      L->fwd_hx = hx;
      L->fwd_ho = ho;
      L->fwd_s = s;
    }
  }
  if (L->fwd_exec && L->fwd_T == T && L->fwd_norm == normalize && L->fwd_hx == hx && L->fwd_ho == ho &&
      L->fwd_s == s) {
    deliver_begin();
    if (cudaGraphLaunch(L->fwd_exec, s) != cudaSuccess) {
      set_host_error(100, "%s: graph launch failed", what);
      return -1;
    }
    count_launches(1);
    if (!finish_delivered(what)) return -1;
  } else {
    deliver_begin();
    if (cudaMemcpyAsync(L->xbuf, hx, n, cudaMemcpyHostToDevice, s) != cudaSuccess) return -1;
    if (!layer_enqueue(L, L->xbuf, nullptr, nullptr, moe, T, normalize, nullptr, s, what)) return -1;
    if (!deliver_async(moe, (size_t)T * L->D, s, what)) return -1;
    if (!finish_delivered(what)) return -1;
  }
  for (size_t i = 0; i < (size_t)T * L->D; i++) out_host[i] += ho[i];
  return 0;
}

// The routing of the last step of a layer: idx/w [T][top_k] (host).
int tg_layer_last_routing(void* handle, int T, int* idx, float* w) {
  std::lock_guard<std::recursive_mutex> lk(ctx_mutex());
  Layer* L = (Layer*)handle;
  if (!L || T < 1 || T > L->max_tokens) return -1;
  cudaStreamSynchronize(stream());
  cudaMemcpy(idx, L->sel_idx, sizeof(int) * (size_t)T * L->top_k, cudaMemcpyDeviceToHost);
  cudaMemcpy(w, L->sel_w, sizeof(float) * (size_t)T * L->top_k, cudaMemcpyDeviceToHost);
  return cudaGetLastError() == cudaSuccess ? 0 : -1;
}

// A residual stack on the device: for each layer, x += experts(rmsnorm(x) *
// norm_w[l]) (norm_w may be NULL: weight 1).  x [T][D] is updated in place;
// enqueued on the library stream.
int tg_stack_forward_dev(void* const* layers, int n_layers, float* x, int T, const float* const* norm_w) {
  std::lock_guard<std::recursive_mutex> lk(ctx_mutex());
  const char* what = "tg_stack_forward_dev";
  if (n_layers < 1 || !layers || !ensure_init()) return -1;
  Layer* L0 = (Layer*)layers[0];
  float* bufs[2] = {x, L0->xbuf};   // residual ping-pong
  float* moe[2] = {L0->moe_out, L0->moe_out + (size_t)L0->max_tokens * L0->D};
  cudaStream_t s = stream();
  int cur = 0;
  for (int l = 0; l < n_layers; l++) {
    Layer* L = (Layer*)layers[l];
    if (L->D != L0->D || T > L0->max_tokens) {
      set_host_error(3, "%s: layer %d does not match layer 0", what, l);
      return -1;
    }
    const float* add = l ? moe[(l - 1) & 1] : nullptr;
    float* x_out = l ? bufs[cur ^ 1] : nullptr;
    if (!layer_enqueue(L, bufs[cur], add, x_out, moe[l & 1], T, 1, norm_w ? norm_w[l] : nullptr, s, what))
      return -1;
    if (l) cur ^= 1;
  }
  // x = x_last' + moe_last, written back into the caller's buffer.
  launch_add(bufs[cur], moe[(n_layers - 1) & 1], x, (size_t)T * L0->D, s);
  count_launches(1);
  return cudaGetLastError() == cudaSuccess ? 0 : -1;
}

// ---- CUDA graphs over the library stream --------------------------------

int tg_cuda_graph_begin(void) {
  std::lock_guard<std::recursive_mutex> lk(ctx_mutex());
  if (!ensure_init()) return -1;
  return cudaStreamBeginCapture(stream(), cudaStreamCaptureModeThreadLocal) == cudaSuccess ? 0 : -1;
}

void* tg_cuda_graph_end(void) {
  std::lock_guard<std::recursive_mutex> lk(ctx_mutex());
  cudaGraph_t graph = nullptr;
  if (cudaStreamEndCapture(stream(), &graph) != cudaSuccess || !graph) {
    set_host_error(102, "tg_cuda_graph_end: capture failed (%s)", cudaGetErrorString(cudaGetLastError()));
    return nullptr;
  }
  cudaGraphExec_t exec = nullptr;
  cudaError_t e = cudaGraphInstantiate(&exec, graph, 0);
  cudaGraphDestroy(graph);
  if (e != cudaSuccess) {
    set_host_error(102, "tg_cuda_graph_end: instantiate failed (%s)", cudaGetErrorString(e));
    return nullptr;
  }
  return exec;
}

int tg_cuda_graph_launch(void* exec) {
  std::lock_guard<std::recursive_mutex> lk(ctx_mutex());
  return cudaGraphLaunch((cudaGraphExec_t)exec, stream()) == cudaSuccess ? 0 : -1;
}

void tg_cuda_graph_destroy(void* exec) {
  if (exec) cudaGraphExecDestroy((cudaGraphExec_t)exec);
}

void* tg_cuda_stream(void) {
  std::lock_guard<std::recursive_mutex> lk(ctx_mutex());
  if (!ensure_init()) return nullptr;
  return (void*)stream();
}

int tg_cuda_synchronize(void) {
  std::lock_guard<std::recursive_mutex> lk(ctx_mutex());
  if (!ensure_init()) return -1;
  return finish("tg_cuda_synchronize") ? 0 : -1;
}

}  // extern "C"
