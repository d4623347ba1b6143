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
    float* y;           // [ids][ldy] fp32 (epi 0, 1); bf16 elements when y_bf16
    int y_bf16;
    // The split form of the layout (libbolt's allocation: qs and d planes, iq2_pack_split): slab / extra_w hold the
    // units' 2048 chunk bytes (expert_bytes apart), dplane / dplane_extra their 64 bytes of d (dplane_stride apart).
    const uint8_t* dplane;
    const uint8_t* dplane_extra;
    size_t dplane_stride;
    int ldy;
    int8_t* aq;         // epi 2: relu^2 rows quantised, [ids][n] int8 and as [ids][n/32]
    float* as;
    int32_t* dots;      // epi 3: [ids][n][k/32] int32 chunk dots
    int ctr;            // the launch slot of the unit counter (set by launch_iq2_gemv)
    // Optional schedule (iq2_schedule_slots): sched[0 .. nslots) the slots by token count, largest first,
    // sched[nslots .. 2 nslots] the exclusive prefix of their batch counts.  nullptr: the kernel derives it.
    const int* sched;
    // 1: counts, offsets, order and sched were written by an earlier launch on the stream than the one this launch
    // follows, so the kernel takes its schedule and first unit before waiting for that launch
    int sched_early;
    // Optional (the expert-parallel exchange over peer memory): once every CTA is done, the last one stores
    // *done_epoch into done_n flags, flag j at done_base[j] + done_off bytes (other GPUs' memory), after one
    // system-scope fence, so that those ranks may read this launch's outputs.
    unsigned char* const* done_base;
    size_t done_off;
    int done_n;
    const int* done_epoch;
    // Optional (the fused launch's down args): output row id at address y_rows[id] (bf16 or fp32 as y_bf16; another
    // GPU's memory allowed) instead of y + id * ldy
    const unsigned long long* y_rows;
};

constexpr int kIq2UnitTok = 3;   // tokens a GEMV work unit dots at most (a slot's tokens come in batches of this many)

// The GEMVs' slot schedule, computed by one CTA (all its threads call it; counts readable by all of them):
// order[0 .. nslots) the slots by token count, largest first (ties to the lower index), and bpre[0 .. nslots] the
// exclusive prefix of their batch counts ceil(count / kIq2UnitTok) in that order.  rank_tmp: nslots ints of shared
// memory (it may be order itself when order is in shared memory).
__device__ inline void iq2_schedule_slots(const int* counts, int nslots, int* order, int* bpre, int* rank_tmp) {
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5, nw = blockDim.x >> 5;
    // a slot's rank is counted by a warp, 32 other slots a ballot
    for (int s = warp; s < nslots; s += nw) {
        const int c = counts[s];
        int rank = 0;
        for (int o0 = 0; o0 < nslots; o0 += 32) {
            const int o = o0 + lane;
            const int co = o < nslots ? counts[o] : -1;
            rank += __popc(__ballot_sync(0xffffffffu, co > c || (co == c && o < s)));
        }
        if (lane == 0) rank_tmp[rank] = s;
    }
    __syncthreads();
    if (warp == 0) {
        // warp-wide exclusive scan of the ordered slots' batch counts
        int carry = 0;
        for (int i0 = 0; i0 < nslots; i0 += 32) {
            const int i = i0 + lane;
            const int s = i < nslots ? rank_tmp[i] : 0;
            const int v = i < nslots ? (counts[s] + kIq2UnitTok - 1) / kIq2UnitTok : 0;
            int incl = v;
#pragma unroll
            for (int o = 1; o < 32; o <<= 1) {
                const int y = __shfl_up_sync(0xffffffffu, incl, o);
                if (lane >= o) incl += y;
            }
            if (i < nslots) {
                order[i] = s;
                bpre[i] = carry + incl - v;
            }
            carry += __shfl_sync(0xffffffffu, incl, 31);
        }
        if (lane == 0) bpre[nslots] = carry;
    }
}

// The slot position holding batch bidx: the last i with bpre[i] <= bidx (slots without batches share their bpre with
// the next slot, so the last such i is the slot that holds the batch).
__device__ inline int iq2_batch_slot(const int* bpre, int nslots, int bidx) {
    int lo = 0, hi = nslots;
    while (hi - lo > 1) {
        const int mid = (lo + hi) >> 1;
        if (bpre[mid] <= bidx) lo = mid;
        else hi = mid;
    }
    return lo;
}

// The fused launch's order of the down phase's batches (launch_iq2_updown).  A batch's down units can start once all
// its up units are done, and batches are ordered by when that is expected: first those whose up units all fall in the
// launch's first wave (unit number < W: every warp starts on one unit), then the rest, each group by token count,
// fewest (the shortest up units) first, ties by batch index.  Batch bidx's up units are bidx * G .. bidx * G + G - 1.
// All threads of the CTA call it; cnt (by slot), order and bpre must be readable by all of them (shared memory);
// tmp: 8 * ceil(batches / 32) ints of shared memory.  Writes dorder[0 .. batches).
__device__ inline void iq2_schedule_batches(const int* cnt, const int* order, const int* bpre, int nslots, int G, int W,
                                            int* dorder, int* tmp) {
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5, nw = blockDim.x >> 5;
    const int nb = bpre[nslots], nch = (nb + 31) >> 5;
    auto key_of = [&](int bidx) {
        if (bidx >= nb) return 8;
        const int i = iq2_batch_slot(bpre, nslots, bidx);
        const int nt = min(kIq2UnitTok, cnt[order[i]] - kIq2UnitTok * (bidx - bpre[i]));
        return ((bidx + 1) * G - 1 >= W ? 4 : 0) + nt;
    };
    // per chunk of 32 batches, the number of each key
    for (int c = warp; c < nch; c += nw) {
        const int key = key_of(32 * c + lane);
#pragma unroll
        for (int k = 0; k < 8; k++) {
            const int m = __popc(__ballot_sync(0xffffffffu, key == k));
            if (lane == k) tmp[c * 8 + k] = m;
        }
    }
    __syncthreads();
    // each key's start in the order, and each chunk's start within its key
    if (warp == 0) {
        int run = 0;
        if (lane < 8)
            for (int c = 0; c < nch; c++) {
                const int v = tmp[c * 8 + lane];
                tmp[c * 8 + lane] = run;
                run += v;
            }
        int incl = lane < 8 ? run : 0;
#pragma unroll
        for (int o = 1; o < 8; o <<= 1) {
            const int y = __shfl_up_sync(0xffffffffu, incl, o);
            if (lane >= o) incl += y;
        }
        const int base = incl - (lane < 8 ? run : 0);
        if (lane < 8)
            for (int c = 0; c < nch; c++) tmp[c * 8 + lane] += base;
    }
    __syncthreads();
    for (int c = warp; c < nch; c += nw) {
        const int bidx = 32 * c + lane, key = key_of(bidx);
        const unsigned m = __match_any_sync(0xffffffffu, key);
        if (key < 8) dorder[tmp[c * 8 + key] + __popc(m & ((1u << lane) - 1u))] = bidx;
    }
}

// sum of a[0 .. n) (shared memory, 16-byte aligned): four words a load, several loads in flight
__device__ __forceinline__ int smem_sum(const int* a, int n) {
    const int4* v = reinterpret_cast<const int4*>(a);
    int s0 = 0, s1 = 0;
    int j = 0;
#pragma unroll 4
    for (; j + 8 <= n; j += 8) {
        const int4 x = v[j >> 2], y = v[(j >> 2) + 1];
        s0 += (x.x + x.y) + (x.z + x.w);
        s1 += (y.x + y.y) + (y.z + y.w);
    }
    for (; j < n; j++) s0 += a[j];
    return s0 + s1;
}

// #{j < n : a[j] > c, or a[j] == c and j < self} (ties to the lower index): the rank of element `self` of value c in
// an order by value, largest first (desc) or smallest first (!desc)
template <bool DESC>
__device__ __forceinline__ int smem_rank(const int* a, int n, int c, int self) {
    const int4* v = reinterpret_cast<const int4*>(a);
    int r = 0;
    int j = 0;
    auto before = [&](int x, int idx) { return (DESC ? x > c : x < c) | ((x == c) & (idx < self)); };
#pragma unroll 4
    for (; j + 4 <= n; j += 4) {
        const int4 x = v[j >> 2];
        r += before(x.x, j) + before(x.y, j + 1) + before(x.z, j + 2) + before(x.w, j + 3);
    }
    for (; j < n; j++) r += before(a[j], j);
    return r;
}

// The layer's grouping and GEMV schedule from the routing in shared memory, every thread of the CTA, each output by
// a direct count (the arrays are small): counts by expert (slot E: the shared expert's `extra` rows); offsets; the
// ids of each slot in increasing pair order (group_pairs' order); the slots by count, largest first, ties to the lower
// index (iq2_schedule_slots' order) with the exclusive prefix of their batches; and the down phase's batch order of
// iq2_schedule_batches.  An id whose expert is outside 0 .. E - 1 is left out.  tmp: an int a batch (kLayerIds in
// the one-launch layer).  s_cnt, s_bpre and tmp 16-byte aligned shared memory; s_ord and s_dord may be global.
// The ids in slot order come from one warp's walk over the ids, 32 at a time (linear in the ids: the expert-parallel
// prologue sees world x T x topk of them, most of them padding): match_any groups the lanes of one expert, a lane's
// place is the expert's running count plus its rank among them, and the group's lowest lane adds the group's size.
__device__ inline void layer_schedule(const int* ridx_s, int pairs, int E, int extra, int G, int W, int* s_cnt, int* s_offs,
                               int* s_ord, int* s_order, int* s_bpre, int* s_dord, int* tmp) {
    const int tid = threadIdx.x, nth = blockDim.x;
    const int nslots = E + (extra ? 1 : 0);
    for (int i = tid; i < E; i += nth) s_cnt[i] = 0;
    __syncthreads();
    for (int p = tid; p < pairs; p += nth) {   // an expert outside 0 .. E - 1 marks an id to leave out
        const int e = ridx_s[p];
        if ((unsigned)e < (unsigned)E) atomicAdd(&s_cnt[e], 1);
    }
    if (tid == 0 && extra) s_cnt[E] = extra;
    __syncthreads();
    for (int e = tid; e <= nslots; e += nth) s_offs[e] = smem_sum(s_cnt, e);
    for (int s = tid; s < nslots; s += nth) s_order[smem_rank<true>(s_cnt, nslots, s_cnt[s], s)] = s;
    __syncthreads();
    if (tid < 32) {   // s_bpre is free until its prefix below: the running counts
        for (int e = tid; e < E; e += 32) s_bpre[e] = s_offs[e];
        __syncwarp();
        for (int p0 = 0; p0 < pairs; p0 += 32) {
            const int p = p0 + tid;
            const int e = p < pairs ? ridx_s[p] : -1;
            const bool in = (unsigned)e < (unsigned)E;
            const unsigned m = __match_any_sync(0xffffffffu, in ? e : -1);
            const int before = __popc(m & ((1u << tid) - 1u));
            const int at = in ? s_bpre[e] : 0;
            __syncwarp();
            if (in) {
                s_ord[at + before] = p;
                if (before == 0) s_bpre[e] = at + __popc(m);
            }
            __syncwarp();
        }
    }
    for (int i = tid; i < extra; i += nth) s_ord[pairs + i] = pairs + i;
    for (int i = tid; i < nslots; i += nth) tmp[i] = (s_cnt[s_order[i]] + kIq2UnitTok - 1) / kIq2UnitTok;
    __syncthreads();
    for (int i = tid; i <= nslots; i += nth) s_bpre[i] = smem_sum(tmp, i);
    __syncthreads();
    const int nb = s_bpre[nslots];
    // each batch's key: first-wave batches (all up units numbered below W) before the rest, fewer tokens first
    for (int i = tid; i < nslots; i += nth) {
        const int c = s_cnt[s_order[i]];
        for (int bidx = s_bpre[i]; bidx < s_bpre[i + 1]; bidx++) {
            const int ntok = min(kIq2UnitTok, c - kIq2UnitTok * (bidx - s_bpre[i]));
            tmp[bidx] = ((bidx + 1) * G - 1 >= W ? 4 : 0) + ntok;
        }
    }
    __syncthreads();
    for (int bidx = tid; bidx < nb; bidx += nth) s_dord[smem_rank<false>(tmp, nb, tmp[bidx], bidx)] = bidx;
    __syncthreads();
}

// epi: 0 store, 1 relu^2, 2 relu^2 + int8 per 32, 3 chunk dots.  maxcnt bounds a slot's ids (the staging size).
cudaError_t launch_iq2_gemv(const GemvArgs& a, int nslots, int maxcnt, int epi, cudaStream_t s);
// One launch of both expert projections over the same slots: up (a: relu^2 + int8 rows into a.aq / a.as, which must be
// down's xq / xs) then down (b).  a.sched is required; ready: one int per batch of the schedule (at least its
// pairs + extra), zero when the launch starts.
// The decode layer in one launch (b200q_moe_decode): its router, grouping and schedule (done by the first CTA to
// arrive), the int8 rows of x (every CTA a share), the fused expert projections, and the combine with the router
// weights and the shared expert (every CTA a share, once every CTA is done with its units).
struct LayerArgs {
    const void* x;           // [T][H] bf16
    const void* logits;      // [T][E] bf16
    const float* bias;
    float scale;
    int T, H, E, topk, route, extra;   // extra: T with a shared expert (slot E), else 0
    int* ridx;               // [T * topk] routing results
    float* rw;
    void* out;               // [T][H]
    int out_dtype;
};

// a.sched must hold, after its 2 nslots + 1 ints, the down phase's batch order (iq2_schedule_batches with
// W = iq2_first_wave()).
cudaError_t launch_iq2_updown(const GemvArgs& up, const GemvArgs& down, int* ready, int nslots, cudaStream_t s);
// the unit numbers a launch's warps start on (one a warp): the W of iq2_schedule_batches
int iq2_first_wave();
// The whole decode layer as one launch (see LayerArgs): up's xq / xs and down's y are written by the launch itself
// (its schedule stays in shared memory); only for layers that layer_fits.
bool layer_fits(int T, int E, int topk, bool shared);
cudaError_t launch_decode_layer(const GemvArgs& up, const GemvArgs& down, int* ready, int nslots, const LayerArgs& L,
                                cudaStream_t s);
// ggml blocks [n][k/256][66] -> the split rt32 layout: qs [units][2048], dq [units][64] (units = n/32 * k/256)
cudaError_t launch_iq2_pack_split(const uint8_t* raw, uint8_t* qs, uint8_t* dq, int64_t n, int k, cudaStream_t s);
bool iq2_shape_ok(int64_t n, int k);

}  // namespace b200q
