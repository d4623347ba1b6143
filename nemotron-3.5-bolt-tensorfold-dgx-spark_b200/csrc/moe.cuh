// Device pieces of the MoE layer shared by its kernels (moe.cu) and the one-launch decode layer (iq2.cu): activation
// loads, the int8-per-32 row quantiser, the router and the expert-sorted grouping.
#pragma once
#include "common.cuh"

namespace b200q {

__device__ __forceinline__ float load_act(const void* p, int dtype, size_t i) {
    return dtype == B200Q_BF16 ? __bfloat162float(reinterpret_cast<const __nv_bfloat16*>(p)[i]) : reinterpret_cast<const float*>(p)[i];
}

// ---------------------------------------------------------------------------------------------------------
// Flags between GPUs (the expert-parallel exchange over peer memory, ep_peer.cu): a sender publishes an epoch after
// its data stores and a system-scope fence; a receiver polls with system-scope acquire loads.  Every wait is bounded
// in time and in polls: on a timeout the waiter sets bit `bit` of *err and goes on (its results are then wrong, and the
// host reads the flag), so a rank that never arrives ends in an error, not a hang.  Measured on B200: a system-scope
// fence about 2 us (3.5 when a hundred CTAs issue one at once), a GPU-scope one 0.2 us, a relaxed system-scope store
// or an acquire load 0.1 us; so a flag set is one fence then relaxed stores.
// ---------------------------------------------------------------------------------------------------------
constexpr unsigned long long kPeerWaitNs = 4000000000ull;   // 4 s
constexpr unsigned kPeerMaxPolls = 1u << 26;

__device__ __forceinline__ unsigned long long peer_clock() {
    unsigned long long t;
    asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
    return t;
}
__device__ __forceinline__ int ld_acquire_sys(const int* p) {
    int v;
    asm volatile("ld.acquire.sys.global.b32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
    return v;
}
__device__ __forceinline__ void fence_acq_rel_sys() { asm volatile("fence.acq_rel.sys;" ::: "memory"); }
__device__ __forceinline__ void st_relaxed_sys(int* p, int v) {
    asm volatile("st.relaxed.sys.global.b32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}
// one thread: wait until flags[0 .. n) have all reached epoch (wrap-safe compare).  Once a waiter has given up (bit
// `bit` of *err set), later waits give up after a few polls too, so a missing rank costs one timeout, not one a CTA;
// the host clears the bits (b200q_ep_peer_error).
__device__ inline void wait_epochs(const int* flags, int n, int epoch, int* err, int bit) {
    const unsigned long long t0 = peer_clock();
    unsigned polls = 0;
    for (int i = 0; i < n; i++) {
        while ((int)(ld_acquire_sys(flags + i) - epoch) < 0) {
            if (++polls > kPeerMaxPolls || ((polls & 63) == 0 && (peer_clock() - t0 > kPeerWaitNs ||
                                                                  ((*(volatile int*)err >> bit) & 1)))) {
                atomicOr(err, 1 << bit);
                return;
            }
            __nanosleep(32);
        }
    }
}

// The expert-parallel exchange over peer memory (ep_peer.cu) around b200q_moe_experts_decode: the received rows
// arrive in int8 form (quantised by their senders, the same arithmetic), the prologue first waits for the senders'
// flags, and the GEMV launch's last CTA publishes the outputs in the senders' flags.
struct ExpertsPeer {
    const int8_t* xq;                 // [R][H] int8 rows, [R][H/32] their scales: read by the GEMVs as they are
    const float* xs;
    const int* wait_flags;            // wait_n flags that must reach *epoch before the rows are read
    int wait_n;
    const int* epoch;
    int* err;                         // bit 0 set when that wait gave up
    unsigned char* const* done_base;  // GemvArgs::done_* (the value published is *epoch)
    size_t done_off;
    int done_n;
    // optional: the down outputs written straight to their senders (GemvArgs::y_rows): row r < world * cap came from
    // sender r / cap as its pair srcp[r], whose output row is at peers[r / cap] + ret_off + srcp[r] * row_bytes; a
    // later row (this rank's own, the shared expert's) goes to yloc + r * row_bytes.  yptr: R entries, filled by the
    // prologue.
    const int* srcp;
    unsigned char* const* peers;
    size_t ret_off;
    int cap, world, row_bytes;
    unsigned char* yloc;
    unsigned long long* yptr;
};
// b200q_moe_experts_decode; with peer, rows may be NULL (the int8 rows are peer->xq / xs).  Defined in moe.cu.
int experts_decode(const void* rows, int rows_dtype, int ldr, int R, int H, int F, const int* lidx, int lidx_stride,
                   int n_local, const void* up, const void* down, void* y, int y_dtype, int ldy, void* workspace,
                   size_t workspace_bytes, void* stream, const ExpertsPeer* peer);

// ---------------------------------------------------------------------------------------------------------
// quant_rows_k's arithmetic (bolt_kernels.cu:347-360), a warp per 32-group: s = amax/127, q = rn(x * 127/amax)
// ---------------------------------------------------------------------------------------------------------
__device__ __forceinline__ void quant_group(float v, int lane, int8_t* q, float* s) {
    float am = fabsf(v);
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) am = fmaxf(am, __shfl_xor_sync(0xffffffffu, am, o));
    const float inv = am > 0.f ? 127.f / am : 0.f;
    q[lane] = (int8_t)__float2int_rn(v * inv);
    if (lane == 0) *s = am / 127.f;
}

// ---------------------------------------------------------------------------------------------------------
// router: a warp per token (route_k's shape, bolt_kernels.cu:1655-1712), E <= 512 so a lane holds 16 logits.
// Top-k by repeated warp argmax, ties to the lower index.
//   softmax: w_i = exp(z_i - max) / sum over the picked of exp(z_j - max)   (softmax, top-k, renormalised)
//   sigmoid: route_k's form: pick by sigmoid(z) + bias, w = sigmoid / (1e-20 + sum of picked) * scale
// ---------------------------------------------------------------------------------------------------------
template <int NJ>   // logits a lane holds: E <= 32 NJ
__device__ void route_token(const void* logits, int dtype, int ldl, const float* bias, int E, int topk, int mode,
                            float scale, int t, int lane, int* ridx, float* rw, int* ridx_s) {
    float val[NJ], key[NJ];
    float mx = -3.0e38f;
#pragma unroll
    for (int j = 0; j < NJ; j++) {
        const int i = lane + 32 * j;
        if (i < E) {
            const float z = load_act(logits, dtype, (size_t)t * ldl + i);
            if (mode == B200Q_ROUTE_SOFTMAX) {
                val[j] = z;
                key[j] = z;
            } else {
                val[j] = 1.f / (1.f + expf(-z));
                key[j] = val[j] + (bias ? bias[i] : 0.f);
            }
            mx = fmaxf(mx, z);
        } else {
            val[j] = 0.f;
            key[j] = -3.0e38f;
        }
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, o));
    float picked = 0.f, sum = mode == B200Q_ROUTE_SOFTMAX ? 0.f : 1e-20f;
    int pick_i = 0;
    for (int kk = 0; kk < topk; kk++) {
        float bv = -3.4e38f;
        int bi = 0x7fffffff;
#pragma unroll
        for (int j = 0; j < NJ; j++) {
            const int i = lane + 32 * j;
            if (i < E && key[j] > bv) { bv = key[j]; bi = i; }
        }
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) {
            const float ov = __shfl_xor_sync(0xffffffffu, bv, o);
            const int oi = __shfl_xor_sync(0xffffffffu, bi, o);
            if (ov > bv || (ov == bv && oi < bi)) { bv = ov; bi = oi; }
        }
        float pv = 0.f;
#pragma unroll
        for (int j = 0; j < NJ; j++)
            if (lane + 32 * j == bi) { pv = val[j]; key[j] = -3.4e38f; }
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) pv += __shfl_xor_sync(0xffffffffu, pv, o);   // only one lane is non-zero
        if (mode == B200Q_ROUTE_SOFTMAX) pv = expf(pv - mx);
        sum += pv;
        if (lane == kk) { picked = pv; pick_i = bi; }
    }
    if (lane < topk) {
        ridx[t * topk + lane] = pick_i;
        if (ridx_s) ridx_s[t * topk + lane] = pick_i;
        rw[t * topk + lane] = mode == B200Q_ROUTE_SOFTMAX ? picked / sum : picked / sum * scale;
    }
}

// Softmax top-k of one token over bf16 logits, E <= 128 (a lane holds logits lane + 32 j), by a warp: route_token's
// selection, weights and rounding (larger logit first, ties to the lower index; w = exp(z - max) / the sum over the
// picked, in pick order), with each pick one redux over packed keys: a bf16 logit maps to 16 bits that order as its
// value, above 16 bits that order as the reversed index.
__device__ __forceinline__ void route_softmax_bf16(const __nv_bfloat16* lg, int E, int topk, int t, int lane,
                                                   int* ridx, float* rw, int* ridx_s) {
    uint32_t key[4];
#pragma unroll
    for (int j = 0; j < 4; j++) {
        const int i = lane + 32 * j;
        uint32_t b = i < E ? (uint32_t)__bfloat16_as_ushort(lg[(size_t)t * E + i]) : 0u;
        if (b == 0x8000u) b = 0u;   // -0 ties with +0, as the float compare has it
        const uint32_t ord = (b & 0x8000u) ? (~b & 0xFFFFu) : (b | 0x8000u);
        key[j] = i < E ? (ord << 16) | (0xFFFFu - (uint32_t)i) : 0u;
    }
    float mx = 0.f, sum = 0.f, picked = 0.f;
    int pick_i = 0;
    for (int kk = 0; kk < topk; kk++) {
        const uint32_t best = __reduce_max_sync(0xffffffffu, max(max(key[0], key[1]), max(key[2], key[3])));
        const int bi = (int)(0xFFFFu - (best & 0xFFFFu));
        const uint32_t o = best >> 16;
        const uint32_t b = (o & 0x8000u) ? (o & 0x7FFFu) : (~o & 0xFFFFu);
        const float z = __uint_as_float(b << 16);
        if (kk == 0) mx = z;   // the first pick is the largest logit
        const float pv = expf(z - mx);
        sum += pv;
        if (lane == kk) { picked = pv; pick_i = bi; }
#pragma unroll
        for (int j = 0; j < 4; j++)
            if (lane + 32 * j == bi) key[j] = 0u;
    }
    if (lane < topk) {
        ridx[t * topk + lane] = pick_i;
        ridx_s[t * topk + lane] = pick_i;
        rw[t * topk + lane] = picked / sum;
    }
}

// ---------------------------------------------------------------------------------------------------------
// grouping (moe_group_k's counting sort, bolt_kernels.cu:275-325), deterministic: the pairs of expert e in
// increasing pair order.  One CTA of 512 threads, E <= 512, pairs <= 4096.  extra > 0 appends a slot E with ids
// pairs .. pairs + extra - 1 (the shared expert over every token).
//   1. warp 0 walks the pairs 32 at a time in order: match_any finds the lanes of the same expert, a pair's place in
//      its expert is that expert's running count plus its rank among those lanes, and the lowest such lane adds
//      their number to the running count;
//   2. an exclusive scan of the counts (warp shuffles, then the warps' totals) gives the offsets;
//   3. every pair writes its index to order[offset + place].
// Shared memory: ridx_s[pairs] (the routing), place_s[pairs], run_s[512], warp_s[16].
// ---------------------------------------------------------------------------------------------------------
__device__ inline void group_pairs(const int* ridx_s, int pairs, int E, int extra, int* counts, int* offsets, int* order,
                            int* place_s, int* run_s, int* warp_s, int* counts_s = nullptr) {
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    run_s[tid] = 0;
    __syncthreads();
    if (warp == 0) {
        for (int p0 = 0; p0 < pairs; p0 += 32) {
            const int p = p0 + lane;
            const bool valid = p < pairs;
            const unsigned vm = __ballot_sync(0xffffffffu, valid);
            if (valid) {
                const int e = ridx_s[p];
                const unsigned peers = __match_any_sync(vm, e);
                const unsigned below = peers & ((1u << lane) - 1u);
                place_s[p] = run_s[e] + __popc(below);
                __syncwarp(vm);
                if (below == 0) run_s[e] += __popc(peers);
            }
            __syncwarp();
        }
    }
    __syncthreads();
    // exclusive scan of run_s[0 .. 512) (zero past E)
    const int c = tid < E ? run_s[tid] : 0;
    int incl = c;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
        const int y = __shfl_up_sync(0xffffffffu, incl, o);
        if (lane >= o) incl += y;
    }
    if (lane == 31) warp_s[warp] = incl;
    __syncthreads();
    int before = 0;
    for (int w = 0; w < warp; w++) before += warp_s[w];
    const int start = before + incl - c;
    if (tid < E) {
        counts[tid] = c;
        offsets[tid] = start;
        if (counts_s) counts_s[tid] = c;   // a shared-memory copy for the caller (slot E: extra)
    }
    if (counts_s && tid == 0) counts_s[E] = extra;
    __syncthreads();
    run_s[tid] = start;   // reused: the offsets, for the scatter
    __syncthreads();
    for (int p = tid; p < pairs; p += blockDim.x) order[run_s[ridx_s[p]] + place_s[p]] = p;
    if (tid == 0) {
        offsets[E] = pairs;
        if (extra > 0) { counts[E] = extra; offsets[E + 1] = pairs + extra; }
    }
    for (int i = tid; i < extra; i += blockDim.x) order[pairs + i] = pairs + i;
}

}  // namespace b200q
