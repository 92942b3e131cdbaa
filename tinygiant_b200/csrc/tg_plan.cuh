// tg_plan.cuh — the device-side description of one MoE call.
//
// A call (tg_moe_forward_rows_v2 and the entries built on it, or one layer
// step routed on the GPU) selects n_slots experts, in order.  Slot s uses
// rows[row_off .. row_off + n_rows) of the k input rows with weights
// wts[...]; this is the reference's per-expert gather of active rows
// (csrc/libtinygiant.c:1411-1423), laid out flat.  The header lives in device
// memory so a plan built on the GPU (by the router kernel) and one staged
// from the host drive the same kernels; grids are sized by host-side upper
// bounds and surplus CTAs exit.
#pragma once
#include "tg_common.cuh"

namespace tg {

struct SlotDesc {
  WDesc gate, up, down;
  const float* gb;   // gate bias [inter] or null
  const float* ub;   // up bias [inter] or null
  const float* db;   // down bias [embed] or null
  int n_rows;        // active input rows of this expert
  int row_off;       // offset of this slot's rows in the flat arrays
  int expert;        // GPU-routed plans: the expert's index in the layer's table
  int pad;
};

// One expert of a resident layer (the GPU router selects among these).
struct ExpertDesc {
  WDesc gate, up, down;
  const float* gb;
  const float* ub;
  const float* db;
};

struct PlanHdr {
  int n_slots;
  int total_rows;
  int k;                  // input rows of the call
  int embed_dim;          // D
  int inter_dim;          // I
  int act;                // Act
  int assoc_rule;         // AssocRule
  int bias_term;          // 1: part = w * (v + (db ? db[r] : 0.f)); 0: part = w * v
  const SlotDesc* slots;  // [n_slots]
  const int* rows;        // [total_rows] input row of each active (slot, j)
  const float* wts;       // [total_rows] combine weight of each active (slot, j)
  const int* row_slot;    // [total_rows] slot of each active (slot, j)
};

// Whether active row j (0-based within its slot of n rows) is computed with
// the x4 association.
__host__ __device__ __forceinline__ bool use_x4(int rule, int j, int n, int k) {
  if (rule == ASSOC_X1) return false;
  if (rule == ASSOC_ROWS) return k > 1;
  int g0 = j & ~3;
  int m = n - g0 < 4 ? n - g0 : 4;
  return m > 1;
}

}  // namespace tg
