// The IQ2_XXS GEMV launcher shared by the dense, grouped and decode-layer entry points.
#pragma once
#include "common.cuh"

namespace b200q {

// One launch covers `nslots` slots (CTAs along grid.y).  Slot s < nslot_routed is expert s of the slab; slot
// nslot_routed (when extra_w is set) is the extra matrix (the shared expert).  A slot's ids are
// order[offsets[s] .. offsets[s] + counts[s]); counts == nullptr means one dense slot with ids 0 .. dense_rows-1.
// An id reads activation row  id < act_split ? id / act_div : id - act_split + act_base  and writes output row id.
struct GemvArgs {
    const uint8_t* slab;
    size_t expert_bytes;
    const uint8_t* extra_w;
    int nslot_routed;
    int n, k;
    const int* counts;
    const int* offsets;
    const int* order;
    int dense_rows;
    int act_div;
    int act_split, act_base;
    const int8_t* xq;   // [rows][k] int8
    const float* xs;    // [rows][k/32]
    float* y;           // [ids][ldy] fp32 (epi 0, 1)
    int ldy;
    int8_t* aq;         // epi 2: relu^2 rows quantised, [ids][n] int8 and as [ids][n/32]
    float* as;
    int32_t* dots;      // epi 3: [ids][n][k/32] int32 chunk dots
    int ctr;            // the launch slot of the unit counter (set by launch_iq2_gemv)
};

// epi: 0 store, 1 relu^2, 2 relu^2 + int8 per 32, 3 chunk dots.  maxcnt bounds a slot's ids (the staging size).
cudaError_t launch_iq2_gemv(const GemvArgs& a, int nslots, int maxcnt, int epi, cudaStream_t s);
bool iq2_shape_ok(int64_t n, int k);

}  // namespace b200q
