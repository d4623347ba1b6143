// The expert-parallel decode step with its exchange over NVLink peer memory: no collective library on the data path.
// libbolt runs every expert of a layer on one GPU (the MoE block of enqueue_block, bolt_host.cu:665-720); across the
// ranks of one box the same layer is, per step and per rank, four launches on the rank's stream:
//
//   1. ep_dispatch_k: route this rank's tokens (route_k's arithmetic), give every (token, expert) pair its owner rank
//      and local expert index there, and store the pair's token row straight into the owner's region (plain stores
//      through the owner's memory mapped into this process), already in the int8-per-32 form the GEMVs read
//      (quant_rows_k's arithmetic: the owner would compute the same bytes); this rank's own tokens also go to its own
//      region as the rows of the shared expert.  The last CTA to finish publishes the step's epoch in every owner's
//      dispatch flags (one system-scope fence, then the flags).
//   2. the local experts' prologue (b200q_moe_experts_decode's, the shared expert being the last local expert): wait
//      until every sender's dispatch flag holds the epoch, then group the received rows by local expert and schedule
//      the GEMVs.
//   3. the fused up/down GEMVs over those rows; the down GEMV stores each routed row's output straight into its
//      sender's return rows (peer stores through a row-address table the prologue fills, GemvArgs::y_rows; the shared
//      expert's rows stay here), and the launch's last CTA publishes the epoch in every sender's return flags
//      (GemvArgs::done_*).
//   4. ep_peer_combine_k: wait for every owner's return flag, then combine this rank's return rows (local loads) with
//      the router weights (combine_k's order, bolt_kernels.cu:1714-1727), plus the shared expert's row.
//
// Buffer reuse needs no second copy: a sender's next dispatch comes after its combine, which waits for every owner's
// step to be done with the rows it received; an owner's next outputs (into the senders' return rows) come after its
// next prologue, which waits for every sender's next dispatch, so after every sender's combine.  Every wait is bounded (moe.cuh wait_epochs): a rank
// that never arrives sets an error bit in the state and the step completes with wrong values instead of hanging.
//
// The region (one cudaMalloc a rank, exported by CUDA IPC, the same layout on every rank), R = world * cap + T rows
// (cap = T * topk: sender s's rows at s * cap, its unused ones marked with the discard index; this rank's own tokens
// after them):
//   xq    [R][H] int8, xs [R][H/32] fp32    the rows the GEMVs read
//   lidx  [R] int32                         each row's local expert
//   srcp  [R] int32                         each received row's pair index at its sender
//   y     [R][H] of the return type         the shared expert's outputs (its rows, the last T)
//   ret   [cap][H] of the return type       this rank's pairs' outputs, written by their owners
//   yptr  [R] u64                           each row's output address (filled by the owner's prologue)
//   flags [2][world] int32                  [0][s] the epoch of sender s's dispatch, [1][o] of owner o's outputs
#include <cstring>

#include "iq2.cuh"
#include "moe.cuh"

namespace b200q {

struct EpRegion {
    int cap, R, elt;                                        // rows from each sender, all rows, the return type's bytes
    size_t xq, xs, lidx, srcp, y, ret, yptr, flags, bytes;  // byte offsets in the region, its size
};
static size_t al256(size_t v) { return (v + 255) & ~(size_t)255; }
static EpRegion ep_region(int world, int T, int H, int topk, int elt) {
    EpRegion r;
    r.cap = T * topk;
    r.R = world * r.cap + T;
    r.elt = elt;
    size_t o = 0;
    r.xq = o; o += al256((size_t)r.R * H);
    r.xs = o; o += al256((size_t)r.R * (H / 32) * 4);
    r.lidx = o; o += al256((size_t)r.R * 4);
    r.srcp = o; o += al256((size_t)r.R * 4);
    r.y = o; o += al256((size_t)r.R * H * elt);
    r.ret = o; o += al256((size_t)r.cap * H * elt);
    r.yptr = o; o += al256((size_t)r.R * 8);
    r.flags = o; o += al256((size_t)2 * world * 4);
    r.bytes = o;
    return r;
}

// A rank's own state (not shared): [0] the epoch of the last step, [1] the dispatch CTAs' arrival count, [2] error
// bits (0: a wait for senders' rows ran out, 1: a wait for owners' outputs ran out, 2: a routed expert or an owner
// out of range), then slot [2 pairs] (each pair's owner and row there) and rw [pairs].
constexpr int kStateHead = 64;
static size_t ep_state_bytes(int pairs) { return (size_t)(kStateHead + 3 * pairs) * 4; }

constexpr int kEpThreads = 512, kEpMaxPairs = 1024, kEpMaxWorld = 64;

struct EpArgs {
    const void* x; int xdt;            // [T][H] this rank's tokens
    const void* logits; int ldt;       // [T][E] and their element type
    const float* bias; float scale;
    int T, H, E, topk, route;
    const int* dest; const int* lidx; const int* nrep; int max_rep;   // placement tables [E][max_rep], [E]
    unsigned char* const* peers;       // [world] every rank's region, mapped here (this rank's own at [rank])
    int world, rank, discard, shared_lidx;
    EpRegion reg;
    int* state;
    void* out; int odt;                // [T][H]
    int* ridx_out; float* rw_out;      // optional copies of the routing
};

__device__ __forceinline__ int* flags_of(const EpArgs& a, int r) {
    return reinterpret_cast<int*>(a.peers[r] + a.reg.flags);
}

// One CTA: token row t of x as an int8 row into region `dst` at row `row`: quant_rows_k's arithmetic (s = amax/127,
// q = rn(x * 127/amax) per 32-group; the bytes of quant_group), a group by 8 lanes of 4 values, so that a warp stores
// 128 contiguous bytes of q at once.
__device__ __forceinline__ void quant_row_to(const EpArgs& a, int t, unsigned char* dst, int row) {
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5, sub = lane & 7;
    const int groups = a.H >> 5;
    int8_t* q = reinterpret_cast<int8_t*>(dst + a.reg.xq) + (size_t)row * a.H;
    float* sc = reinterpret_cast<float*>(dst + a.reg.xs) + (size_t)row * groups;
    for (int g = warp * 4 + (lane >> 3); g < groups; g += (kEpThreads / 32) * 4) {
        const size_t i = (size_t)t * a.H + g * 32 + sub * 4;
        float v[4];
        if (a.xdt == B200Q_BF16) {
            const uint2 u = *reinterpret_cast<const uint2*>(reinterpret_cast<const __nv_bfloat16*>(a.x) + i);
            const float2 f0 = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(&u.x));
            const float2 f1 = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(&u.y));
            v[0] = f0.x; v[1] = f0.y; v[2] = f1.x; v[3] = f1.y;
        } else {
            const float4 f = *reinterpret_cast<const float4*>(reinterpret_cast<const float*>(a.x) + i);
            v[0] = f.x; v[1] = f.y; v[2] = f.z; v[3] = f.w;
        }
        float am = fmaxf(fmaxf(fabsf(v[0]), fabsf(v[1])), fmaxf(fabsf(v[2]), fabsf(v[3])));
#pragma unroll
        for (int o = 4; o > 0; o >>= 1) am = fmaxf(am, __shfl_xor_sync(0xffffffffu, am, o));
        const float inv = am > 0.f ? 127.f / am : 0.f;
        uint32_t packed = 0;
#pragma unroll
        for (int j = 0; j < 4; j++) packed |= (uint32_t)(uint8_t)(int8_t)__float2int_rn(v[j] * inv) << (8 * j);
        reinterpret_cast<uint32_t*>(q + g * 32)[sub] = packed;
        if (sub == 0) sc[g] = am / 127.f;
    }
}

// Launch 1.  Every CTA routes all T tokens (a warp a token) and places every pair, so no CTA waits on another; CTA c
// then writes rows c, c + G, ... of the pairs (to their owners) and of this rank's tokens (to its own shared-expert
// rows), and marks the unused rows of every owner's block with the discard index.  The last CTA to arrive publishes
// the epoch.
__global__ void __launch_bounds__(kEpThreads) ep_dispatch_k(const EpArgs a) {
    pdl_wait();
    __shared__ int ridx_s[kEpMaxPairs], dst_s[kEpMaxPairs], lid_s[kEpMaxPairs], pos_s[kEpMaxPairs];
    __shared__ float rw_s[kEpMaxPairs];
    __shared__ int cnt_s[kEpMaxWorld];
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    const int pairs = a.T * a.topk, cap = a.reg.cap;
    for (int t = warp; t < a.T; t += kEpThreads / 32) {   // a warp a token (16 warps: one each at decode sizes)
        if (a.route == B200Q_ROUTE_SOFTMAX && a.ldt == B200Q_BF16 && a.E <= 128)
            route_softmax_bf16(reinterpret_cast<const __nv_bfloat16*>(a.logits), a.E, a.topk, t, lane, ridx_s, rw_s,
                               ridx_s);
        else if (a.E <= 128)
            route_token<4>(a.logits, a.ldt, a.E, a.bias, a.E, a.topk, a.route, a.scale, t, lane, ridx_s, rw_s, nullptr);
        else
            route_token<16>(a.logits, a.ldt, a.E, a.bias, a.E, a.topk, a.route, a.scale, t, lane, ridx_s, rw_s,
                            nullptr);
    }
    for (int i = threadIdx.x; i < a.world; i += kEpThreads) cnt_s[i] = 0;
    __syncthreads();
    // each pair's owner (a replicated expert's pairs split between its copies by token) and local index there
    for (int p = threadIdx.x; p < pairs; p += kEpThreads) {
        const int e = ridx_s[p], t = p / a.topk;
        int d = -1, l = 0;
        const int nr = (unsigned)e < (unsigned)a.E ? a.nrep[e] : 0;
        if (nr > 0 && nr <= a.max_rep) {
            const int q = e * a.max_rep + t % nr;
            d = a.dest[q];
            l = a.lidx[q];
        }
        if ((unsigned)d >= (unsigned)a.world) {
            d = -1;
            if (blockIdx.x == 0) atomicOr(a.state + 2, 4);
        }
        dst_s[p] = d;
        lid_s[p] = l;
    }
    __syncthreads();
    // a pair's row in its owner's block from this rank: the pairs before it with the same owner, in pair order.
    // Warp 0 walks the pairs 32 at a time: match_any finds the lanes of the same owner, a pair's row is that owner's
    // running count plus its rank among them, and the lowest of them adds their number to the count.
    if (warp == 0) {
        for (int p0 = 0; p0 < pairs; p0 += 32) {
            const int p = p0 + lane;
            const int d = p < pairs ? dst_s[p] : -2;
            const unsigned m = __match_any_sync(0xffffffffu, d);
            const int before = __popc(m & ((1u << lane) - 1u));
            if (d >= 0) {
                pos_s[p] = cnt_s[d] + before;
                __syncwarp(m);
                if (before == 0) cnt_s[d] += __popc(m);
            }
            __syncwarp();
        }
    }
    __syncthreads();
    if (blockIdx.x == 0) {
        int* slot = a.state + kStateHead;
        float* rw = reinterpret_cast<float*>(slot + 2 * pairs);
        for (int p = threadIdx.x; p < pairs; p += kEpThreads) {
            slot[2 * p] = dst_s[p];
            slot[2 * p + 1] = a.rank * cap + pos_s[p];
            rw[p] = rw_s[p];
            if (a.ridx_out) a.ridx_out[p] = ridx_s[p];
            if (a.rw_out) a.rw_out[p] = rw_s[p];
        }
    }
    for (int i = blockIdx.x; i < pairs + a.T; i += gridDim.x) {
        int t, d, row, l;
        if (i < pairs) {
            t = i / a.topk; d = dst_s[i]; row = a.rank * cap + pos_s[i]; l = lid_s[i];
            if (d < 0) continue;
        } else {
            t = i - pairs; d = a.rank; row = a.world * cap + t; l = a.shared_lidx;
        }
        unsigned char* dst = a.peers[d];
        quant_row_to(a, t, dst, row);
        if (threadIdx.x == 0) {
            reinterpret_cast<int*>(dst + a.reg.lidx)[row] = l;
            reinterpret_cast<int*>(dst + a.reg.srcp)[row] = i < pairs ? i : -1;
        }
    }
    // the unused rows of this rank's block at every owner: the discard index (never computed there)
    for (int j = blockIdx.x * kEpThreads + threadIdx.x; j < a.world * cap; j += gridDim.x * kEpThreads) {
        const int d = j / cap, pos = j - d * cap;
        if (pos >= cnt_s[d]) reinterpret_cast<int*>(a.peers[d] + a.reg.lidx)[a.rank * cap + pos] = a.discard;
    }
    // publish: the barrier orders the CTA's stores before thread 0's fence and count (a grid-wide barrier's
    // pattern); the last CTA to arrive acquires the others' counts with a system-scope fence, whose cumulativity
    // carries every CTA's stores, and stores the epoch in every owner's flags.  Only that CTA pays for a system-scope
    // fence (moe.cuh has the costs).
    __syncthreads();
    if (threadIdx.x == 0) {
        __threadfence();
        const int prev = atomicAdd(a.state + 1, 1);
        if (prev == (int)gridDim.x - 1) {
            fence_acq_rel_sys();
            a.state[1] = 0;
            const int e = *reinterpret_cast<volatile int*>(a.state) + 1;
            a.state[0] = e;
            for (int d = 0; d < a.world; d++) st_relaxed_sys(flags_of(a, d) + a.rank, e);
        }
    }
    pdl_trigger();
}

// Launch 4 (the last): out[t][h] = sum over k in order of rw[t][k] * ret[pair (t, k)][h] (fma), + the shared expert's
// row.  A thread owns 8 consecutive h; the return rows were stored here by their owners (L1-bypassing loads), the
// loads of up to kBatch pairs issued before their fmas.
__device__ __forceinline__ void load8(const unsigned char* p, int elt, float* v) {
    if (elt == 2) {
        const uint4 u = __ldcg(reinterpret_cast<const uint4*>(p));
        const __nv_bfloat162* b = reinterpret_cast<const __nv_bfloat162*>(&u);
#pragma unroll
        for (int j = 0; j < 4; j++) {
            const float2 f = __bfloat1622float2(b[j]);
            v[2 * j] = f.x;
            v[2 * j + 1] = f.y;
        }
    } else {
        const float4 f0 = __ldcg(reinterpret_cast<const float4*>(p)), f1 = __ldcg(reinterpret_cast<const float4*>(p) + 1);
        v[0] = f0.x; v[1] = f0.y; v[2] = f0.z; v[3] = f0.w; v[4] = f1.x; v[5] = f1.y; v[6] = f1.z; v[7] = f1.w;
    }
}

__global__ void __launch_bounds__(128) ep_peer_combine_k(const EpArgs a) {
    pdl_wait();
    if (threadIdx.x == 0) wait_epochs(flags_of(a, a.rank) + a.world, a.world, *reinterpret_cast<volatile int*>(a.state),
                                      a.state + 2, 1);
    __syncthreads();
    const int t = blockIdx.y, h0 = (blockIdx.x * blockDim.x + threadIdx.x) * 8;
    if (h0 >= a.H) return;
    const int pairs = a.T * a.topk, elt = a.reg.elt;
    const int* slot = a.state + kStateHead;
    const float* rw = reinterpret_cast<const float*>(slot + 2 * pairs);
    constexpr int kBatch = 4;
    float acc[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f}, v[kBatch][8];
    for (int k0 = 0; k0 < a.topk; k0 += kBatch) {
        float w[kBatch];
        bool ok[kBatch];
#pragma unroll
        for (int b = 0; b < kBatch; b++) {
            const int kk = k0 + b, p = t * a.topk + kk;
            const int d = kk < a.topk ? slot[2 * p] : -1;
            ok[b] = (unsigned)d < (unsigned)a.world;   // an owner out of range was recorded by the dispatch
            w[b] = 0.f;
            if (ok[b]) {
                w[b] = rw[p];
                load8(a.peers[a.rank] + a.reg.ret + ((size_t)p * a.H + h0) * elt, elt, v[b]);
            }
        }
#pragma unroll
        for (int b = 0; b < kBatch; b++)
            if (ok[b]) {
#pragma unroll
                for (int j = 0; j < 8; j++) acc[j] = fmaf(w[b], v[b][j], acc[j]);
            }
    }
    load8(a.peers[a.rank] + a.reg.y + ((size_t)(a.world * a.reg.cap + t) * a.H + h0) * elt, elt, v[0]);
#pragma unroll
    for (int j = 0; j < 8; j++) acc[j] += v[0][j];
    if (a.odt == B200Q_BF16) {
        __nv_bfloat162* o = reinterpret_cast<__nv_bfloat162*>(reinterpret_cast<__nv_bfloat16*>(a.out) + (size_t)t * a.H + h0);
#pragma unroll
        for (int j = 0; j < 4; j++) o[j] = __floats2bfloat162_rn(acc[2 * j], acc[2 * j + 1]);
    } else {
        float4* o = reinterpret_cast<float4*>(reinterpret_cast<float*>(a.out) + (size_t)t * a.H + h0);
        o[0] = make_float4(acc[0], acc[1], acc[2], acc[3]);
        o[1] = make_float4(acc[4], acc[5], acc[6], acc[7]);
    }
}

}  // namespace b200q

using namespace b200q;

extern "C" {

size_t b200q_ep_peer_region_bytes(int world, int T, int H, int topk, int ret_dtype) {
    if (world <= 0 || T <= 0 || H <= 0 || H % 32 || topk <= 0 || (ret_dtype != B200Q_F32 && ret_dtype != B200Q_BF16))
        return 0;
    return ep_region(world, T, H, topk, ret_dtype == B200Q_BF16 ? 2 : 4).bytes;
}

size_t b200q_ep_peer_state_bytes(int T, int topk) {
    if (T <= 0 || topk <= 0) return 0;
    return al256(ep_state_bytes(T * topk));
}

size_t b200q_ep_peer_workspace_bytes(int world, int T, int H, int F, int topk, int n_local) {
    if (world <= 0 || T <= 0 || topk <= 0 || n_local < 0) return 0;
    return b200q_moe_experts_workspace_bytes(world * T * topk + T, H, F, n_local + 1);
}

int b200q_peer_alloc(size_t bytes, void** ptr) {
    if (!ptr || bytes == 0) return B200Q_EINVAL;
    *ptr = nullptr;
    int st = status_from(cudaMalloc(ptr, bytes));
    if (st != B200Q_OK) return st;
    st = status_from(cudaMemset(*ptr, 0, bytes));
    if (st != B200Q_OK) {
        cudaFree(*ptr);
        *ptr = nullptr;
    }
    return st;
}

int b200q_peer_free(void* ptr) { return ptr ? status_from(cudaFree(ptr)) : B200Q_OK; }

size_t b200q_peer_handle_bytes(void) { return sizeof(cudaIpcMemHandle_t); }

int b200q_peer_export(void* ptr, void* handle) {
    if (!ptr || !handle) return B200Q_EINVAL;
    cudaIpcMemHandle_t h;
    const int st = status_from(cudaIpcGetMemHandle(&h, ptr));
    if (st == B200Q_OK) memcpy(handle, &h, sizeof(h));
    return st;
}

int b200q_peer_open(const void* handle, void** ptr) {
    if (!handle || !ptr) return B200Q_EINVAL;
    cudaIpcMemHandle_t h;
    memcpy(&h, handle, sizeof(h));
    *ptr = nullptr;
    return status_from(cudaIpcOpenMemHandle(ptr, h, cudaIpcMemLazyEnablePeerAccess));
}

int b200q_peer_close(void* ptr) { return ptr ? status_from(cudaIpcCloseMemHandle(ptr)) : B200Q_OK; }

int b200q_ep_peer_error(void* state, int clear) {
    if (!state) return B200Q_EINVAL;
    int v = 0;
    if (cudaMemcpy(&v, (int*)state + 2, sizeof(int), cudaMemcpyDeviceToHost) != cudaSuccess) return -1;
    if (clear && v) {
        const int z = 0;
        if (cudaMemcpy((int*)state + 2, &z, sizeof(int), cudaMemcpyHostToDevice) != cudaSuccess) return -1;
    }
    return v;
}

int b200q_ep_peer_decode(const void* x, int x_dtype, const void* logits, int logits_dtype, int T, int H, int F, int E,
                         int topk, int route, const float* bias, float scale, const int* dest, const int* lidx,
                         const int* nrep, int max_rep, void* region, void* const* peers, int world, int rank,
                         int n_local, int discard, const void* up, const void* down, int ret_dtype, void* state,
                         void* workspace, size_t workspace_bytes, void* out, int out_dtype, int* ridx_out,
                         float* rw_out, int phases, void* stream) {
    const int pairs = T * topk;
    if (!x || !logits || !dest || !lidx || !nrep || !region || !peers || !up || !down || !state || !workspace || !out ||
        T <= 0 || topk <= 0 || E <= 0 || E > 512 || topk > E || topk > 32 || pairs > kEpMaxPairs || world <= 0 ||
        world > kEpMaxWorld || rank < 0 || rank >= world || n_local < 0 || n_local + 1 > 511 ||
        discard < n_local + 1 || max_rep <= 0 || (long long)world * pairs + T > 4096 ||
        !iq2_shape_ok(F, H) || !iq2_shape_ok(H, F) ||
        (x_dtype != B200Q_F32 && x_dtype != B200Q_BF16) || (logits_dtype != B200Q_F32 && logits_dtype != B200Q_BF16) ||
        (ret_dtype != B200Q_F32 && ret_dtype != B200Q_BF16) || (out_dtype != B200Q_F32 && out_dtype != B200Q_BF16) ||
        (route != B200Q_ROUTE_SOFTMAX && route != B200Q_ROUTE_SIGMOID) || ((uintptr_t)x & 15) ||
        ((uintptr_t)out & 15) || ((uintptr_t)state & 15) || ((uintptr_t)region & 255) || phases <= 0 || phases > 7)
        return B200Q_EINVAL;
    EpArgs a = {};
    a.x = x; a.xdt = x_dtype; a.logits = logits; a.ldt = logits_dtype; a.bias = bias; a.scale = scale;
    a.T = T; a.H = H; a.E = E; a.topk = topk; a.route = route;
    a.dest = dest; a.lidx = lidx; a.nrep = nrep; a.max_rep = max_rep;
    a.peers = reinterpret_cast<unsigned char* const*>(peers);
    a.world = world; a.rank = rank; a.discard = discard; a.shared_lidx = n_local;
    a.reg = ep_region(world, T, H, topk, ret_dtype == B200Q_BF16 ? 2 : 4);
    a.state = (int*)state; a.out = out; a.odt = out_dtype; a.ridx_out = ridx_out; a.rw_out = rw_out;
    cudaStream_t s = (cudaStream_t)stream;
    int st;
    if (phases & 1) {
        const int grid = pairs + T < 2 * 148 ? pairs + T : 2 * 148;
        launch(ep_dispatch_k, dim3(grid), dim3(kEpThreads), 0, s, a);
        if ((st = launched()) != B200Q_OK) return st;
    }
    if (phases & 2) {
        // the local experts over this rank's received rows (its own region), the shared expert being local index
        // n_local (the last expert of the up / down slabs): the prologue waits for every sender's dispatch flag; the
        // fused GEMV's last CTA publishes the outputs in every sender's return flags (flag `rank` of the second row)
        unsigned char* self = (unsigned char*)region;
        ExpertsPeer pe = {};
        pe.xq = reinterpret_cast<const int8_t*>(self + a.reg.xq);
        pe.xs = reinterpret_cast<const float*>(self + a.reg.xs);
        pe.wait_flags = reinterpret_cast<const int*>(self + a.reg.flags);
        pe.wait_n = world;
        pe.epoch = a.state;
        pe.err = a.state + 2;
        pe.done_base = a.peers;
        pe.done_off = a.reg.flags + (size_t)(world + rank) * 4;
        pe.done_n = world;
        pe.srcp = reinterpret_cast<const int*>(self + a.reg.srcp);
        pe.peers = a.peers;
        pe.ret_off = a.reg.ret;
        pe.cap = a.reg.cap;
        pe.world = world;
        pe.row_bytes = H * a.reg.elt;
        pe.yloc = self + a.reg.y;
        pe.yptr = reinterpret_cast<unsigned long long*>(self + a.reg.yptr);
        st = experts_decode(nullptr, B200Q_BF16, H, a.reg.R, H, F, reinterpret_cast<const int*>(self + a.reg.lidx), 1,
                            n_local + 1, up, down, self + a.reg.y, ret_dtype, H, workspace, workspace_bytes, stream,
                            &pe);
        if (st != B200Q_OK) return st;
    }
    if (phases & 4) {
        launch(ep_peer_combine_k, dim3((H / 8 + 127) / 128, T), dim3(128), 0, s, a);
        if ((st = launched()) != B200Q_OK) return st;
    }
    return B200Q_OK;
}

}  // extern "C"
