// The MoE layer around the expert GEMVs: int8 rows of the activations, the router, the expert-sorted grouping,
// the weighted combine, and the decode layer that chains them.
#include "iq2.cuh"
#include "moe.cuh"

#include <cstdlib>

namespace b200q {



// ---------------------------------------------------------------------------------------------------------
// status plumbing
// ---------------------------------------------------------------------------------------------------------
static thread_local int g_last_cuda = 0;
int status_from(cudaError_t e) {
    if (e == cudaSuccess) return B200Q_OK;
    g_last_cuda = (int)e;
    return B200Q_ECUDA;
}
bool pdl_enabled() {
    static const bool on = [] { const char* e = getenv("B200Q_PDL"); return !(e && atoi(e) == 0); }();
    return on;
}

__global__ void quant_rows_k(const void* __restrict__ x, int dtype, int ldx, int8_t* __restrict__ q, int ldq,
                             float* __restrict__ s, int lds, int rows, int k) {
    pdl_wait();
    const int groups = k >> 5;
    const int64_t gw = ((int64_t)blockIdx.x * blockDim.x + threadIdx.x) >> 5;
    const int lane = threadIdx.x & 31;
    if (gw < (int64_t)rows * groups) {
        const int r = (int)(gw / groups), g = (int)(gw - (int64_t)r * groups);
        const float v = load_act(x, dtype, (size_t)r * ldx + g * 32 + lane);
        quant_group(v, lane, q + (size_t)r * ldq + g * 32, s + (size_t)r * lds + g);
    }
    pdl_trigger();
}

__global__ void route_k(const void* __restrict__ logits, int dtype, int ldl, const float* __restrict__ bias, int T, int E,
                        int topk, int mode, float scale, int* __restrict__ ridx, float* __restrict__ rw) {
    pdl_wait();
    const int t = blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
    if (t < T) {
        if (E <= 128) route_token<4>(logits, dtype, ldl, bias, E, topk, mode, scale, t, threadIdx.x & 31, ridx, rw, nullptr);
        else route_token<16>(logits, dtype, ldl, bias, E, topk, mode, scale, t, threadIdx.x & 31, ridx, rw, nullptr);
    }
    pdl_trigger();
}

__global__ void __launch_bounds__(512) group_k(const int* __restrict__ ridx, int pairs, int E, int* __restrict__ counts,
                                               int* __restrict__ offsets, int* __restrict__ order) {
    pdl_wait();
    __shared__ int ridx_s[4096], place_s[4096], run_s[512], warp_s[16];
    for (int i = threadIdx.x; i < pairs; i += blockDim.x) ridx_s[i] = ridx[i];
    __syncthreads();
    group_pairs(ridx_s, pairs, E, 0, counts, offsets, order, place_s, run_s, warp_s);
    pdl_trigger();
}

// ---------------------------------------------------------------------------------------------------------
// grouping for prompt chunks (any number of pairs): histogram, scan, scatter.  Inside an expert's run the pairs are in
// arrival order; the prompt GEMMs compute every row on its own, so their results do not depend on that order.
// ---------------------------------------------------------------------------------------------------------
__global__ void group_zero_k(int* __restrict__ counts, int* __restrict__ fill, int E) {
    pdl_wait();
    for (int i = blockIdx.x * blockDim.x + threadIdx.x; i < E; i += gridDim.x * blockDim.x) { counts[i] = 0; fill[i] = 0; }
    pdl_trigger();
}
__global__ void group_hist_k(const int* __restrict__ ridx, int pairs, int* __restrict__ counts) {
    pdl_wait();
    for (int p = blockIdx.x * blockDim.x + threadIdx.x; p < pairs; p += gridDim.x * blockDim.x) atomicAdd(&counts[ridx[p]], 1);
    pdl_trigger();
}
__global__ void __launch_bounds__(512) group_scan_k(const int* __restrict__ counts, int E, int* __restrict__ offsets) {
    pdl_wait();
    __shared__ int s[512];
    const int tid = threadIdx.x;
    s[tid] = tid < E ? counts[tid] : 0;
    __syncthreads();
    for (int off = 1; off < 512; off <<= 1) {
        const int v = tid >= off ? s[tid - off] : 0;
        __syncthreads();
        s[tid] += v;
        __syncthreads();
    }
    if (tid < E) offsets[tid] = s[tid] - counts[tid];
    if (tid == 0) offsets[E] = s[511];
    pdl_trigger();
}
__global__ void group_scatter_k(const int* __restrict__ ridx, int pairs, const int* __restrict__ offsets, int* __restrict__ fill,
                                int* __restrict__ order) {
    pdl_wait();
    for (int p = blockIdx.x * blockDim.x + threadIdx.x; p < pairs; p += gridDim.x * blockDim.x) {
        const int e = ridx[p];
        order[offsets[e] + atomicAdd(&fill[e], 1)] = p;
    }
    pdl_trigger();
}

// ---------------------------------------------------------------------------------------------------------
// decode prologue, one launch: block 0 routes every token (a warp per token), groups the pairs and orders the
// expert GEMVs' slots (iq2_schedule_slots); the other blocks write the int8 rows of x (a warp per 32-group).
// ---------------------------------------------------------------------------------------------------------
__global__ void __launch_bounds__(512) moe_prep_k(const void* __restrict__ x, const void* __restrict__ logits, int T, int H,
                                                  int F, int E, int topk, int route, const float* __restrict__ bias, float scale,
                                                  int extra, int* __restrict__ ridx, float* __restrict__ rw,
                                                  int* __restrict__ counts, int* __restrict__ offsets, int* __restrict__ order,
                                                  int8_t* __restrict__ xq, float* __restrict__ xs, int* __restrict__ sched,
                                                  int* __restrict__ ready, int wave) {
    pdl_wait();
    __shared__ int ridx_s[1024], place_s[1024], run_s[512], warp_s[16], cnt_s[513];   // T * topk <= 64 * 16
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    if (blockIdx.x == 0) {
        for (int i = threadIdx.x; i < T * topk + (extra > 0 ? T : 0); i += blockDim.x) ready[i] = 0;
        for (int t = warp; t < T; t += 16) {
            if (E <= 128) route_token<4>(logits, B200Q_BF16, E, bias, E, topk, route, scale, t, lane, ridx, rw, ridx_s);
            else route_token<16>(logits, B200Q_BF16, E, bias, E, topk, route, scale, t, lane, ridx, rw, ridx_s);
        }
        __syncthreads();
        group_pairs(ridx_s, T * topk, E, extra, counts, offsets, order, place_s, run_s, warp_s, cnt_s);
        // the expert GEMVs' schedule, once for both, from the counts kept in shared memory
        const int nsl = E + (extra > 0 ? 1 : 0);
        __syncthreads();
        iq2_schedule_slots(cnt_s, nsl, sched, sched + nsl, ridx_s);
        __syncthreads();
        // the fused GEMV's down-phase order of batches (place_s is free after the grouping)
        iq2_schedule_batches(cnt_s, sched, sched + nsl, nsl, F >> 5, wave, sched + 2 * nsl + 1, place_s);
    } else {
        const int groups = H >> 5;
        const int gw = (blockIdx.x - 1) * 16 + warp;
        if (gw < T * groups) {
            const int r = gw / groups, g = gw - r * groups;
            const float v = load_act(x, B200Q_BF16, (size_t)r * H + g * 32 + lane);
            quant_group(v, lane, xq + (size_t)r * H + g * 32, xs + (size_t)r * (H >> 5) + g);
        }
    }
    pdl_trigger();
}

// ---------------------------------------------------------------------------------------------------------
// the expert-parallel prologue over a rank's received rows, one launch.  Block 0 groups the rows by their local expert
// (lidx; an index outside 0 .. n_local - 1 is padding, left out and never computed) and orders the GEMVs' slots and
// the down phase's batches, with the one-launch layer's direct counts (layer_schedule: the results of group_pairs,
// iq2_schedule_slots and iq2_schedule_batches); the other blocks (none when rows is NULL: the rows came in int8 form)
// write the int8 rows of the rows that are not padding.
// With peer rows (the exchange over peer memory, ep_peer.cu), every block first waits until the wait_n senders'
// flags in wait_flags have reached *wait_epoch (bounded; a timeout sets bit 0 of *wait_err).
// ---------------------------------------------------------------------------------------------------------
__global__ void __launch_bounds__(512) moe_local_prep_k(const void* __restrict__ rows, int dtype, int ldr, int R, int H,
                                                        const int* __restrict__ lidx, int lidx_stride, int n_local,
                                                        int* __restrict__ counts, int* __restrict__ offsets,
                                                        int* __restrict__ order, int8_t* __restrict__ xq,
                                                        float* __restrict__ xs, int* __restrict__ sched,
                                                        int* __restrict__ ready, int F, int wave, const int* wait_flags,
                                                        int wait_n, const int* wait_epoch, int* wait_err,
                                                        ExpertsPeer rt) {
    pdl_wait();
    if (wait_flags) {
        if (threadIdx.x == 0) {
            wait_epochs(wait_flags, wait_n, *wait_epoch, wait_err, 0);
            asm volatile("fence.proxy.async.global;" ::: "memory");   // the GEMVs read the rows by bulk copies
        }
        __syncthreads();
    }
    // R <= 4096, n_local <= 511
    __shared__ __align__(16) int ridx_s[4096], tmp_s[4096], cnt_s[516], offs_s[516], order_s[516], bpre_s[516];
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    if (blockIdx.x == 0) {
        for (int i = threadIdx.x; i < R; i += blockDim.x) ready[i] = 0;
        for (int i = threadIdx.x; i < R; i += blockDim.x) {
            const int l = lidx[(size_t)i * lidx_stride];
            ridx_s[i] = (l < 0 || l >= n_local) ? n_local : l;   // padding: left out of the schedule
            if (rt.yptr) {   // the row's output address (a padding row's is never used)
                unsigned char* dst;
                if (i < rt.world * rt.cap) {
                    const int pp = rt.srcp[i];
                    dst = rt.peers[i / rt.cap] + rt.ret_off + (size_t)(pp < 0 ? 0 : pp) * rt.row_bytes;
                } else {
                    dst = rt.yloc + (size_t)i * rt.row_bytes;
                }
                rt.yptr[i] = reinterpret_cast<unsigned long long>(dst);
            }
        }
        __syncthreads();
        // counts by local expert, offsets, the ids of each expert in increasing row order (straight to `order`), the
        // experts by count with their batch prefix, and the down phase's batch order (straight to `sched`)
        layer_schedule(ridx_s, R, n_local, 0, F >> 5, wave, cnt_s, offs_s, order, order_s, bpre_s,
                       sched + 2 * n_local + 1, tmp_s);
        for (int e = threadIdx.x; e <= n_local; e += blockDim.x) {
            if (e < n_local) {
                counts[e] = cnt_s[e];
                sched[e] = order_s[e];
            } else {
                counts[e] = R - offs_s[e];   // the padding rows
            }
            offsets[e] = offs_s[e];
            sched[n_local + e] = bpre_s[e];
        }
    } else if (rows) {
        // a warp a (row, 32-group), grid-stride; padding rows are skipped
        const int groups = H >> 5;
        for (int gw = (blockIdx.x - 1) * 16 + warp; gw < R * groups; gw += (gridDim.x - 1) * 16) {
            const int r = gw / groups, g = gw - r * groups;
            const int l = lidx[(size_t)r * lidx_stride];
            if (l < 0 || l >= n_local) continue;
            const float v = load_act(rows, dtype, (size_t)r * ldr + g * 32 + lane);
            quant_group(v, lane, xq + (size_t)r * H + g * 32, xs + (size_t)r * (H >> 5) + g);
        }
    }
    pdl_trigger();
}

// ---------------------------------------------------------------------------------------------------------
// combine (combine_k, bolt_kernels.cu:1714-1727): out[t][h] = sum_k rw[t][k] mo[t*topk+k][h] (+ shared[t][h])
// ---------------------------------------------------------------------------------------------------------
__global__ void combine_k(const float* __restrict__ mo, const float* __restrict__ rw, const float* __restrict__ shared, int T,
                          int topk, int H, void* __restrict__ out, int out_dtype) {
    pdl_wait();
    const int t = blockIdx.y;
    const int h4 = blockIdx.x * blockDim.x + threadIdx.x;
    if (h4 * 4 < H) {
        float4 acc = make_float4(0.f, 0.f, 0.f, 0.f);
        for (int kk = 0; kk < topk; kk++) {
            const float wk = rw[t * topk + kk];
            const float4 v = reinterpret_cast<const float4*>(mo + ((size_t)t * topk + kk) * H)[h4];
            acc.x = fmaf(wk, v.x, acc.x); acc.y = fmaf(wk, v.y, acc.y);
            acc.z = fmaf(wk, v.z, acc.z); acc.w = fmaf(wk, v.w, acc.w);
        }
        if (shared) {
            const float4 sv = reinterpret_cast<const float4*>(shared + (size_t)t * H)[h4];
            acc.x += sv.x; acc.y += sv.y; acc.z += sv.z; acc.w += sv.w;
        }
        if (out_dtype == B200Q_BF16) {
            __nv_bfloat162* o = reinterpret_cast<__nv_bfloat162*>(reinterpret_cast<__nv_bfloat16*>(out) + (size_t)t * H) + 2 * h4;
            o[0] = __floats2bfloat162_rn(acc.x, acc.y);
            o[1] = __floats2bfloat162_rn(acc.z, acc.w);
        } else {
            reinterpret_cast<float4*>(reinterpret_cast<float*>(out) + (size_t)t * H)[h4] = acc;
        }
    }
    pdl_trigger();
}

// ---------------------------------------------------------------------------------------------------------
// workspace of the decode layer (256-byte aligned pieces)
// ---------------------------------------------------------------------------------------------------------
struct DecodeWs {
    int* ridx; float* rw; int* counts; int* offsets; int* order;
    int8_t* xq; float* xs; int8_t* aq; float* as; float* mo;
    int* sched;   // the expert GEMVs' slot schedule (2 nslots + 1 ints)
    int* ready;   // the fused GEMV's readiness counter of each batch (pairs + T ints), zeroed by the prologue
    size_t bytes;
};
static size_t al(size_t v) { return (v + 255) & ~(size_t)255; }
static DecodeWs decode_ws(char* base, int T, int H, int F, int E, int topk) {
    const size_t pairs = (size_t)T * topk, ids = pairs + T;
    DecodeWs w;
    size_t o = 0;
    w.ridx = (int*)(base + o); o += al(pairs * 4);
    w.rw = (float*)(base + o); o += al(pairs * 4);
    w.counts = (int*)(base + o); o += al((size_t)(E + 1) * 4);
    w.offsets = (int*)(base + o); o += al((size_t)(E + 2) * 4);
    w.order = (int*)(base + o); o += al(ids * 4);
    w.xq = (int8_t*)(base + o); o += al((size_t)T * H);
    w.xs = (float*)(base + o); o += al((size_t)T * (H / 32) * 4);
    w.aq = (int8_t*)(base + o); o += al(ids * F);
    w.as = (float*)(base + o); o += al(ids * (F / 32) * 4);
    w.mo = (float*)(base + o); o += al(ids * H * 4);
    w.sched = (int*)(base + o); o += al(((size_t)(2 * (E + 1) + 1) + ids) * 4);   // + the down phase's batch order
    w.ready = (int*)(base + o); o += al(ids * 4);
    w.bytes = o;
    return w;
}

struct ExpertsWs {
    int* counts; int* offsets; int* order; int8_t* xq; float* xs; int8_t* aq; float* as; int* sched;
    int* ready;   // the fused GEMV's readiness counter of each batch (R ints), zeroed by the prologue
    size_t bytes;
};
static ExpertsWs experts_ws(char* base, int R, int H, int F, int n_local) {
    ExpertsWs w;
    size_t o = 0;
    w.counts = (int*)(base + o); o += al((size_t)(n_local + 1) * 4);
    w.offsets = (int*)(base + o); o += al((size_t)(n_local + 2) * 4);
    w.order = (int*)(base + o); o += al((size_t)R * 4);
    w.xq = (int8_t*)(base + o); o += al((size_t)R * H);
    w.xs = (float*)(base + o); o += al((size_t)R * (H / 32) * 4);
    w.aq = (int8_t*)(base + o); o += al((size_t)R * F);
    w.as = (float*)(base + o); o += al((size_t)R * (F / 32) * 4);
    w.sched = (int*)(base + o); o += al((size_t)(2 * n_local + 1 + R) * 4);   // + the down phase's batch order
    w.ready = (int*)(base + o); o += al((size_t)R * 4);
    w.bytes = o;
    return w;
}

}  // namespace b200q

using namespace b200q;

extern "C" {

int b200q_abi(void) { return B200Q_ABI; }
int b200q_last_cuda_error(void) { return g_last_cuda; }
const char* b200q_strerror(int status) {
    switch (status) {
        case B200Q_OK: return "ok";
        case B200Q_EINVAL: return "invalid argument (null pointer, shape or alignment)";
        case B200Q_ENOSPACE: return "workspace or capacity too small";
        case B200Q_ECUDA: return "CUDA launch error (see b200q_last_cuda_error)";
        default: return "unknown status";
    }
}

int b200q_quant_rows(const void* x, int x_dtype, int ldx, int8_t* q, int ldq, float* s, int lds, int rows, int k,
                     void* stream) {
    if (!x || !q || !s || rows < 0 || k <= 0 || k % 32 || ldx < k || ldq < k || lds < k / 32 ||
        (x_dtype != B200Q_F32 && x_dtype != B200Q_BF16))
        return B200Q_EINVAL;
    if (rows == 0) return B200Q_OK;
    const int64_t warps = (int64_t)rows * (k / 32);
    launch(quant_rows_k, dim3((unsigned)((warps + 7) / 8)), dim3(256), 0, (cudaStream_t)stream, x, x_dtype, ldx, q, ldq, s,
           lds, rows, k);
    return launched();
}

int b200q_route(const void* logits, int l_dtype, int ldl, const float* bias, int T, int E, int topk, int mode,
                float scale, int* ridx, float* rw, void* stream) {
    if (!logits || !ridx || !rw || T < 0 || E <= 0 || E > 512 || topk <= 0 || topk > 16 || topk > E || ldl < E ||
        (mode != B200Q_ROUTE_SOFTMAX && mode != B200Q_ROUTE_SIGMOID) || (l_dtype != B200Q_F32 && l_dtype != B200Q_BF16))
        return B200Q_EINVAL;
    if (T == 0) return B200Q_OK;
    launch(route_k, dim3((T + 7) / 8), dim3(256), 0, (cudaStream_t)stream, logits, l_dtype, ldl, bias, T, E, topk, mode,
           scale, ridx, rw);
    return launched();
}

int b200q_moe_group(const int* ridx, int pairs, int E, int* counts, int* offsets, int* order, void* stream) {
    if ((!ridx && pairs > 0) || !counts || !offsets || !order || pairs < 0 || pairs > 4096 || E <= 0 || E > 512)
        return B200Q_EINVAL;
    launch(group_k, dim3(1), dim3(512), 0, (cudaStream_t)stream, ridx, pairs, E, counts, offsets, order);
    return launched();
}

int b200q_moe_group_large(const int* ridx, int pairs, int E, int* counts, int* offsets, int* order, int* fill_scratch,
                          void* stream) {
    if ((!ridx && pairs > 0) || !counts || !offsets || !order || !fill_scratch || pairs < 0 || E <= 0 || E > 512)
        return B200Q_EINVAL;
    cudaStream_t s = (cudaStream_t)stream;
    const int blocks = pairs > 0 ? (pairs + 255) / 256 < 1024 ? (pairs + 255) / 256 : 1024 : 1;
    int st;
    launch(group_zero_k, dim3(1), dim3(512), 0, s, counts, fill_scratch, E);
    if ((st = launched()) != B200Q_OK) return st;
    launch(group_hist_k, dim3(blocks), dim3(256), 0, s, ridx, pairs, counts);
    if ((st = launched()) != B200Q_OK) return st;
    launch(group_scan_k, dim3(1), dim3(512), 0, s, (const int*)counts, E, offsets);
    if ((st = launched()) != B200Q_OK) return st;
    launch(group_scatter_k, dim3(blocks), dim3(256), 0, s, ridx, pairs, (const int*)offsets, fill_scratch, order);
    return launched();
}

int b200q_combine(const float* mo, const float* rw, const float* shared, int T, int topk, int H, void* out, int out_dtype,
                  void* stream) {
    if (!mo || !rw || !out || T < 0 || topk <= 0 || H <= 0 || H % 4 || (out_dtype != B200Q_F32 && out_dtype != B200Q_BF16))
        return B200Q_EINVAL;
    if (T == 0) return B200Q_OK;
    launch(combine_k, dim3((H / 4 + 255) / 256, T), dim3(256), 0, (cudaStream_t)stream, mo, rw, shared, T, topk, H, out,
           out_dtype);
    return launched();
}

size_t b200q_moe_experts_workspace_bytes(int R, int H, int F, int n_local) {
    if (R <= 0 || H <= 0 || F <= 0 || n_local <= 0) return 0;
    return experts_ws(nullptr, R, H, F, n_local).bytes;
}

int b200q_moe_experts_decode(const void* rows, int rows_dtype, int ldr, int R, int H, int F, const int* lidx,
                             int lidx_stride, int n_local, const void* up, const void* down, void* y, int y_dtype,
                             int ldy, void* workspace, size_t workspace_bytes, void* stream) {
    return b200q::experts_decode(rows, rows_dtype, ldr, R, H, F, lidx, lidx_stride, n_local, up, down, y, y_dtype, ldy,
                                 workspace, workspace_bytes, stream, nullptr);
}

}  // extern "C"

int b200q::experts_decode(const void* rows, int rows_dtype, int ldr, int R, int H, int F, const int* lidx,
                          int lidx_stride, int n_local, const void* up, const void* down, void* y, int y_dtype, int ldy,
                          void* workspace, size_t workspace_bytes, void* stream, const ExpertsPeer* peer) {
    const bool given = peer && peer->xq;   // the rows come in int8 form
    if (R < 0 || R > 4096 || n_local <= 0 || n_local > 511 || !iq2_shape_ok(F, H) || !iq2_shape_ok(H, F) ||
        (!given && rows_dtype != B200Q_F32 && rows_dtype != B200Q_BF16) ||
        (y_dtype != B200Q_F32 && y_dtype != B200Q_BF16))
        return B200Q_EINVAL;
    if (R == 0) return B200Q_OK;
    if ((!given && (!rows || ldr < H)) ||
        (given && (!peer->xs || ((uintptr_t)peer->xq & 15) || ((uintptr_t)peer->xs & 15))) || !lidx ||
        lidx_stride < 1 || !up || !down || !y || !workspace || ldy < H || ((uintptr_t)workspace & 255) ||
        ((uintptr_t)up & 15) || ((uintptr_t)down & 15))
        return B200Q_EINVAL;
    ExpertsWs w = experts_ws((char*)workspace, R, H, F, n_local);
    if (workspace_bytes < w.bytes) return B200Q_ENOSPACE;
    cudaStream_t s = (cudaStream_t)stream;
    int st;
    // 1. grouping by local expert, the slot schedule, the int8 rows (unless given): at most one wave of quantiser
    // blocks (148 SMs x 4 blocks of 512 threads), striding over the rows
    const int qwarps = R * (H / 32), qblocks = (qwarps + 15) / 16 < 4 * 148 ? (qwarps + 15) / 16 : 4 * 148;
    launch(moe_local_prep_k, dim3(given ? 1 : 1 + qblocks), dim3(512), 0, s, given ? nullptr : rows, rows_dtype, ldr,
           R, H, lidx, lidx_stride, n_local, w.counts, w.offsets, w.order, w.xq, w.xs, w.sched, w.ready, F,
           iq2_first_wave(), peer ? peer->wait_flags : nullptr, peer ? peer->wait_n : 0,
           peer ? peer->epoch : nullptr, peer ? peer->err : nullptr, peer ? *peer : ExpertsPeer{});
    if ((st = launched()) != B200Q_OK) return st;
    // 2. up with relu^2 and the int8 rows of the result (row id = received row), then down, in one launch
    GemvArgs a = {};
    a.slab = (const uint8_t*)up; a.expert_bytes = iq2_bytes(F, H); a.nslot_routed = n_local; a.n = F; a.k = H;
    a.counts = w.counts; a.offsets = w.offsets; a.order = w.order; a.act_div = 1; a.act_split = 1 << 30;
    a.xq = given ? peer->xq : w.xq; a.xs = given ? peer->xs : w.xs; a.aq = w.aq; a.as = w.as; a.sched = w.sched;
    GemvArgs b = {};
    b.slab = (const uint8_t*)down; b.expert_bytes = iq2_bytes(H, F); b.nslot_routed = n_local; b.n = H; b.k = F;
    b.counts = w.counts; b.offsets = w.offsets; b.order = w.order; b.act_div = 1; b.act_split = 1 << 30;
    b.xq = w.aq; b.xs = w.as; b.y = (float*)y; b.ldy = ldy; b.y_bf16 = y_dtype == B200Q_BF16;
    b.sched = w.sched;
    if (peer && peer->yptr) b.y_rows = peer->yptr;   // the outputs go straight to their rows' owners
    // the launch whose end publishes the outputs: the down launch, or the fused launch (whose args are up's)
#ifdef B200Q_X_NOFUSE
    if (peer) { b.done_base = peer->done_base; b.done_off = peer->done_off; b.done_n = peer->done_n; b.done_epoch = peer->epoch; }
    if ((st = status_from(launch_iq2_gemv(a, n_local, 16, 2, s))) != B200Q_OK) return st;
    b.sched_early = 1;
    return status_from(launch_iq2_gemv(b, n_local, 16, 0, s));
#else
    if (peer) { a.done_base = peer->done_base; a.done_off = peer->done_off; a.done_n = peer->done_n; a.done_epoch = peer->epoch; }
    return status_from(launch_iq2_updown(a, b, w.ready, n_local, s));
#endif
}

extern "C" {

size_t b200q_moe_decode_workspace_bytes(int T, int H, int F, int E, int topk) {
    if (T <= 0 || H <= 0 || F <= 0 || E <= 0 || topk <= 0) return 0;
    return decode_ws(nullptr, T, H, F, E, topk).bytes;
}

int b200q_moe_decode(const void* x, const void* logits, const void* up, const void* down, const void* shared_up,
                     const void* shared_down, int T, int H, int F, int E, int topk, int route, const float* bias,
                     float scale, void* out, int out_dtype, void* workspace, size_t workspace_bytes, int* ridx_out,
                     float* rw_out, void* const* stage_events, void* stream) {
    if (!x || !logits || !up || !down || !out || !workspace || T <= 0 || T > 64 || E <= 0 || E > 512 || topk <= 0 ||
        topk > 16 || topk > E || !iq2_shape_ok(F, H) || !iq2_shape_ok(H, F) || ((shared_up == nullptr) != (shared_down == nullptr)) ||
        (route != B200Q_ROUTE_SOFTMAX && route != B200Q_ROUTE_SIGMOID) || (out_dtype != B200Q_F32 && out_dtype != B200Q_BF16) ||
        ((uintptr_t)workspace & 255) || ((uintptr_t)up & 15) || ((uintptr_t)down & 15) || ((uintptr_t)shared_up & 15) ||
        ((uintptr_t)shared_down & 15))
        return B200Q_EINVAL;
    DecodeWs w = decode_ws((char*)workspace, T, H, F, E, topk);
    if (workspace_bytes < w.bytes) return B200Q_ENOSPACE;
    cudaStream_t s = (cudaStream_t)stream;
    const int pairs = T * topk;
    const int extra = shared_up ? T : 0;
    const int nslots = E + (extra ? 1 : 0);
    const int maxcnt = T;
    int st;
    auto mark = [&](int i) {
        return stage_events ? status_from(cudaEventRecord((cudaEvent_t)stage_events[i], s)) : B200Q_OK;
    };

    if ((st = mark(0)) != B200Q_OK) return st;
#ifndef B200Q_X_NOLAYER
    if (layer_fits(T, E, topk, extra > 0)) {
        // the whole layer as one launch: router, grouping and schedule, int8 rows of x, up (relu^2 + int8 rows) and
        // down over every expert slot and the shared expert, combine
        GemvArgs a = {};
        a.slab = (const uint8_t*)up; a.expert_bytes = iq2_bytes(F, H); a.extra_w = (const uint8_t*)shared_up;
        a.nslot_routed = E; a.n = F; a.k = H; a.counts = w.counts; a.offsets = w.offsets; a.order = w.order;
        a.act_div = topk; a.act_split = pairs; a.act_base = 0; a.xq = w.xq; a.xs = w.xs; a.aq = w.aq; a.as = w.as;
        a.sched = w.sched;
        GemvArgs b = {};
        b.slab = (const uint8_t*)down; b.expert_bytes = iq2_bytes(H, F); b.extra_w = (const uint8_t*)shared_down;
        b.nslot_routed = E; b.n = H; b.k = F; b.counts = w.counts; b.offsets = w.offsets; b.order = w.order;
        b.act_div = 1; b.act_split = 1 << 30; b.xq = w.aq; b.xs = w.as; b.y = w.mo; b.ldy = H; b.sched = w.sched;
        LayerArgs L = {};
        L.x = x; L.logits = logits; L.bias = bias; L.scale = scale; L.T = T; L.H = H; L.E = E; L.topk = topk;
        // the routing goes straight to the caller's buffers when given (no copies after the launch)
        L.route = route; L.extra = extra; L.ridx = ridx_out ? ridx_out : w.ridx; L.rw = rw_out ? rw_out : w.rw;
        L.out = out; L.out_dtype = out_dtype;
        (void)maxcnt;
        if ((st = status_from(launch_decode_layer(a, b, w.ready, nslots, L, s))) != B200Q_OK) return st;
        for (int i = 1; i <= 4; i++)
            if ((st = mark(i)) != B200Q_OK) return st;   // one launch: the stage marks all follow it
        return B200Q_OK;
    } else
#endif
    {
    // 1. router + grouping (block 0) and the int8 rows of x (the rest)
    const int qwarps = T * (H / 32);
    launch(moe_prep_k, dim3(1 + (qwarps + 15) / 16), dim3(512), 0, s, x, logits, T, H, F, E, topk, route, bias, scale, extra,
           w.ridx, w.rw, w.counts, w.offsets, w.order, w.xq, w.xs, w.sched, w.ready, iq2_first_wave());
    if ((st = launched()) != B200Q_OK) return st;
    if ((st = mark(1)) != B200Q_OK) return st;

    // 2. up, relu^2, int8 rows of the result: ids < pairs read token id / topk, the shared ids pairs + t read token t
    GemvArgs a = {};
    a.slab = (const uint8_t*)up; a.expert_bytes = iq2_bytes(F, H); a.extra_w = (const uint8_t*)shared_up;
    a.nslot_routed = E; a.n = F; a.k = H; a.counts = w.counts; a.offsets = w.offsets; a.order = w.order;
    a.act_div = topk; a.act_split = pairs; a.act_base = 0; a.xq = w.xq; a.xs = w.xs; a.aq = w.aq; a.as = w.as;
    a.sched = w.sched;   // written by the prologue, the launch this one follows: read after the wait

    // 3. down over the int8 rows of every id, in the same launch: a batch's down units start once its up rows are in
    GemvArgs b = {};
    b.slab = (const uint8_t*)down; b.expert_bytes = iq2_bytes(H, F); b.extra_w = (const uint8_t*)shared_down;
    b.nslot_routed = E; b.n = H; b.k = F; b.counts = w.counts; b.offsets = w.offsets; b.order = w.order;
    b.act_div = 1; b.act_split = 1 << 30; b.xq = w.aq; b.xs = w.as; b.y = w.mo; b.ldy = H;
    b.sched = w.sched;
#ifdef B200Q_X_NOFUSE
    (void)maxcnt;
    if ((st = status_from(launch_iq2_gemv(a, nslots, maxcnt, 2, s))) != B200Q_OK) return st;
    if ((st = mark(2)) != B200Q_OK) return st;
    b.sched_early = 1;   // the prologue's schedule is two launches back: taken while the up GEMV finishes
    if ((st = status_from(launch_iq2_gemv(b, nslots, maxcnt, 0, s))) != B200Q_OK) return st;
#else
    (void)maxcnt;
    if ((st = status_from(launch_iq2_updown(a, b, w.ready, nslots, s))) != B200Q_OK) return st;
    if ((st = mark(2)) != B200Q_OK) return st;   // (stage 2 is both projections; stage 3 is empty)
#endif
    if ((st = mark(3)) != B200Q_OK) return st;

    // 4. combine + the shared expert's rows
    launch(combine_k, dim3((H / 4 + 255) / 256, T), dim3(256), 0, s, (const float*)w.mo, (const float*)w.rw,
           extra ? (const float*)(w.mo + (size_t)pairs * H) : (const float*)nullptr, T, topk, H, out, out_dtype);
    if ((st = launched()) != B200Q_OK) return st;
    if ((st = mark(4)) != B200Q_OK) return st;
    }
    if (ridx_out) {
        if (cudaMemcpyAsync(ridx_out, w.ridx, sizeof(int) * pairs, cudaMemcpyDeviceToDevice, s) != cudaSuccess) return status_from(cudaGetLastError());
    }
    if (rw_out) {
        if (cudaMemcpyAsync(rw_out, w.rw, sizeof(float) * pairs, cudaMemcpyDeviceToDevice, s) != cudaSuccess) return status_from(cudaGetLastError());
    }
    return B200Q_OK;
}

}  // extern "C"

// ---------------------------------------------------------------------------------------------------------
// The decode MoE layer for callers that cannot allocate device memory.
//
// Some hosts of this library cannot call cudaMalloc: a framework whose caching allocator owns the GPU's memory and
// fixes its budget at start-up, a plugin boundary that hands the operator nothing but tensors, or a decode loop that
// must never take cudaMalloc's implicit device synchronisation.  They cannot provide b200q_moe_decode's workspace, so
// this entry point runs the same four launches on a scratch array that lives in the library itself: a file-scope
// __device__ array of kNoAllocScratchBytes, which every GPU that loads the library holds until the process exits.
// Host code cannot use the array's name as a device address (it is a host-side stand-in), so the first call on each
// device, with that device current, asks the runtime for the address (cudaGetSymbolAddress) and keeps it; that first
// call should therefore come before any stream capture.  The address is kept for the process's life: a
// cudaDeviceReset rebuilds the context and may move the array, so the entry point is not for devices that get reset.
// Every call shares the one array: the layer writes every
// byte of scratch it reads before reading it, so nothing has to start at zero, but calls that overlap on the GPU
// (two streams, two threads) race on it.  Shapes whose scratch would exceed the array are refused with
// B200Q_ENOSPACE.
// ---------------------------------------------------------------------------------------------------------
#include <mutex>

namespace b200q {
constexpr size_t kNoAllocScratchBytes = (size_t)3 << 20;   // covers T <= 16, H <= 4096, F <= 2048, E <= 128, topk <= 8
static __device__ __align__(256) unsigned char g_noalloc_scratch[kNoAllocScratchBytes];
static std::mutex g_noalloc_mu;
static void* g_noalloc_ptr[256];   // the array's device address, by device ordinal

static int noalloc_scratch(void** out) {
    int dev = 0;
    cudaError_t e = cudaGetDevice(&dev);
    if (e != cudaSuccess) return status_from(e);
    if (dev < 0 || dev >= 256) return B200Q_EINVAL;
    std::lock_guard<std::mutex> lock(g_noalloc_mu);
    if (!g_noalloc_ptr[dev]) {
        void* p = nullptr;
        e = cudaGetSymbolAddress(&p, g_noalloc_scratch);
        if (e != cudaSuccess) return status_from(e);
        g_noalloc_ptr[dev] = p;
    }
    *out = g_noalloc_ptr[dev];
    return B200Q_OK;
}
}  // namespace b200q

extern "C" size_t b200q_moe_decode_noalloc_max_bytes(void) { return b200q::kNoAllocScratchBytes; }

extern "C" int b200q_moe_decode_noalloc(const void* x, const void* logits, const void* up, const void* down,
                                        const void* shared_up, const void* shared_down, int T, int H, int F, int E, int topk,
                                        int route, const float* bias, float scale, void* out, int out_dtype, int* ridx_out,
                                        float* rw_out, void* stream) {
    const size_t need = b200q_moe_decode_workspace_bytes(T, H, F, E, topk);
    if (need == 0) return B200Q_EINVAL;
    if (need > b200q::kNoAllocScratchBytes) return B200Q_ENOSPACE;
    void* scratch = nullptr;
    const int st = b200q::noalloc_scratch(&scratch);
    if (st != B200Q_OK) return st;
    return b200q_moe_decode(x, logits, up, down, shared_up, shared_down, T, H, F, E, topk, route, bias, scale, out,
                            out_dtype, scratch, b200q::kNoAllocScratchBytes, ridx_out, rw_out, nullptr, stream);
}
