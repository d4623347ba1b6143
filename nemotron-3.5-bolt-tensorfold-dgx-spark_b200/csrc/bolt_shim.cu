// libbolt's operator launchers over this engine (include/b200q_bolt.h): the names, signatures and view structs of the
// reference's engine/bolt_common.h:77-161, so its host code links here for the routed-expert MoE block.  Each shim
// maps libbolt's arguments onto the engine's kernels; libbolt's model constants (latent 1024, TOPN 9) are the fixed
// shapes its launchers assume.
#include "iq2.cuh"
#include "../../include/b200q_bolt.h"

#include <cstdio>
#include <mutex>

namespace b200q {

// the split forms of the t16 decode layouts (gemv_tc.cu)
cudaError_t launch_nv4_pack_split(const uint8_t* q, const uint8_t* sc, uint8_t* qt, uint8_t* sct, int n, int k,
                                  cudaStream_t s);
cudaError_t launch_q8_pack_split(const uint8_t* raw, uint8_t* qt, uint8_t* dt, int n, int k, cudaStream_t s);
int tc_gemv_split(int fmt, const uint8_t* qt, const uint8_t* sct, float s2, int n, int k, const float* x, int ldx, int T,
                  float* y, int ldy, void* ws, size_t ws_bytes, cudaStream_t s);
size_t tc_split_ws(int fmt, int n, int k, int T);
constexpr int kTcNv4 = 0, kTcQ8 = 1;
constexpr int kTcRows = 16;   // rows a decode GEMV launch takes
// the NVFP4 prompt GEMM over libbolt's buffers (nv4_gemm.cu)
int nv4_planes_pack(const uint8_t* q, const uint8_t* sc, uint8_t* qw, uint8_t* sfw, int n, int k, cudaStream_t s);
int nv4_quant_plain(const float* x, int ldx, uint8_t* q4, uint8_t* sf, int T, int k, cudaStream_t s);
int nv4_gemm_planes(const uint8_t* qw, const uint8_t* sfw, int n, int k, float s2, const uint8_t* q4, const uint8_t* sf,
                    int T, uint8_t* rows_img, float* y, int ldy, cudaStream_t s);

constexpr int kBoltLatent = 1024;   // moe_up's k, moe_down's n, k_combine's width (bolt_kernels.cu:682-695, 1714-1727)
constexpr int kBoltTopN = 9;        // routed experts a token (bolt_common.h:25)
constexpr int kBoltSlots = 512;     // experts a router output can name (moe_group_k's 512 counters, bolt_kernels.cu:278)

static void report(const char* what, cudaError_t e) {
    if (e != cudaSuccess) fprintf(stderr, "b200q shim: %s failed: %s\n", what, cudaGetErrorString(e));
}
static void report(const char* what, int status) {
    if (status != B200Q_OK) fprintf(stderr, "b200q shim: %s failed: %s\n", what, b200q_strerror(status));
}

// the one-item-per-slot work list: expert[e] = e, n_work = kBoltSlots
__global__ void work_slots_k(int* __restrict__ work_exp, int* __restrict__ n_work, const int* __restrict__ counts,
                             int* __restrict__ stat) {
    pdl_wait();
    const int e = blockIdx.x * blockDim.x + threadIdx.x;
    if (e < kBoltSlots) {
        work_exp[e] = e;
        if (stat && counts[e] > 0) atomicAdd(stat, 1);   // libbolt's profile counters: active experts, items
    }
    if (e == 0) {
        *n_work = kBoltSlots;
        if (stat) atomicAdd(stat + 1, kBoltSlots);
    }
    pdl_trigger();
}

// a grouped launch over libbolt's slab (split rt32 planes) and this engine's one-item-per-slot MoeWork
static GemvArgs slab_args(const IQ2Slab& slab, const MoeWork& w, int n, int k, int act_div) {
    GemvArgs a = {};
    a.slab = slab.qs;
    a.expert_bytes = slab.qs_stride;
    a.dplane = (const uint8_t*)slab.d;
    a.dplane_stride = slab.d_stride * 2;   // halves -> bytes
    a.nslot_routed = kBoltSlots;
    a.n = n;
    a.k = k;
    a.counts = w.count;
    a.offsets = w.first;
    a.order = w.order;
    a.act_div = act_div;
    a.act_split = 1 << 30;
    return a;
}

// The shims' scratch, one buffer a (device, stream, use) as libbolt's mma_pack_buffer keeps its per-stream row
// scratch (bolt_mma.cu:1183-1187): launches on one stream are ordered, so they share it.  It grows only outside stream
// capture.  Uses: the K-slice partials of the decode GEMVs (a capture that needs more than the buffer holds runs the
// GEMV as one K slice, the same sums), and mma_iq2's int8 rows.
enum { kWsPartials = 0, kWsRows = 1, kWsFp4Rows = 2 };
struct ShimWs { int dev; cudaStream_t s; int use; void* p; size_t bytes; };
static ShimWs g_ws[32];
static std::mutex g_ws_mu;

static void* shim_ws(cudaStream_t s, size_t need, size_t* have, int use = kWsPartials) {
    *have = 0;
    if (need == 0) return nullptr;
    int dev = 0;
    cudaGetDevice(&dev);
    std::lock_guard<std::mutex> lock(g_ws_mu);
    ShimWs* slot = nullptr;
    for (auto& w : g_ws)
        if (w.p && w.dev == dev && w.s == s && w.use == use) { slot = &w; break; }
    if (!slot)
        for (auto& w : g_ws)
            if (!w.p) { slot = &w; break; }
    if (!slot) return nullptr;
    if (slot->p && slot->bytes >= need) {
        *have = slot->bytes;
        return slot->p;
    }
    cudaStreamCaptureStatus cap = cudaStreamCaptureStatusNone;
    if (cudaStreamIsCapturing(s, &cap) != cudaSuccess || cap != cudaStreamCaptureStatusNone) {
        *have = slot->p ? slot->bytes : 0;
        return slot->p;
    }
    const size_t bytes = need > (size_t(16) << 20) ? need : (size_t(16) << 20);
    void* p = nullptr;
    if (cudaMalloc(&p, bytes) != cudaSuccess) {
        cudaGetLastError();
        *have = slot->p ? slot->bytes : 0;
        return slot->p;
    }
    if (slot->p) {
        cudaStreamSynchronize(s);   // the old buffer's last readers
        cudaFree(slot->p);
    }
    *slot = {dev, s, use, p, bytes};
    *have = bytes;
    return p;
}

// W x for T rows in 16-row pieces, libbolt's mma_* over the split planes
static void tc_rows(const char* what, int fmt, const uint8_t* qt, const uint8_t* sct, float s2, int n, int k,
                    const float* x, int ldx, float* y, int ldy, int T, cudaStream_t s) {
    if (T <= 0) return;
    size_t have = 0;
    void* ws = shim_ws(s, tc_split_ws(fmt, n, k, T < kTcRows ? T : kTcRows), &have);
    for (int t0 = 0; t0 < T; t0 += kTcRows) {
        const int rows = T - t0 < kTcRows ? T - t0 : kTcRows;
        const int st = tc_gemv_split(fmt, qt, sct, s2, n, k, x + (size_t)t0 * ldx, ldx, rows, y + (size_t)t0 * ldy, ldy,
                                     ws, have, s);
        if (st != B200Q_OK) {
            report(what, st);
            return;
        }
    }
}

}  // namespace b200q

using namespace b200q;

// repack_iq2 (bolt_kernels.cu:1053-1068): the checkpoint's blocks into the qs / d buffers load_slab allocates
// (rows * k/256 * 64 and * 2 bytes), as this engine's split rt32 layout; rows % 32 == 0
void repack_iq2(cudaStream_t s, const uint8_t* src, uint8_t* qs, void* d, size_t rows, int k) {
    if (!src || !qs || !d || rows % kIq2Tile || k % 256 || k <= 0) {
        report("repack_iq2", B200Q_EINVAL);
        return;
    }
    report("repack_iq2", launch_iq2_pack_split(src, qs, (uint8_t*)d, (int64_t)rows, k, s));
}

// route_k (bolt_kernels.cu:1653-1712): sigmoid + bias top-9, weights normalised and scaled
void k_route(cudaStream_t s, const float* logits, int ldl, const float* bias, int* ridx, float* rw, int E, float scale, int T) {
    report("k_route", b200q_route(logits, B200Q_F32, ldl, bias, T, E, kBoltTopN, B200Q_ROUTE_SIGMOID, scale, ridx, rw, s));
}

// moe_group_k (bolt_kernels.cu:275-344): the pairs in expert order, and the work list as one item per expert slot
void k_moe_group(cudaStream_t s, const int* ridx, int pairs, int* order, int* work_first, int* work_n, int* work_exp,
                 int* n_work, int* stat) {
    // work_n / work_first take the slots' counts and offsets (libbolt sizes them TMAX * TOPN >= 513 entries);
    // work_exp is the large-count grouping's fill scratch before it becomes the slot list
    const int st = pairs <= 4096 ? b200q_moe_group(ridx, pairs, kBoltSlots, work_n, work_first, order, s)
                                 : b200q_moe_group_large(ridx, pairs, kBoltSlots, work_n, work_first, order, work_exp, s);
    report("k_moe_group", st);
    if (st == B200Q_OK)
        report("k_moe_group", launch(work_slots_k, dim3((kBoltSlots + 255) / 256), dim3(256), 0, s, work_exp, n_work,
                                     (const int*)work_n, stat));
}

// quant_rows_k (bolt_kernels.cu:347-363)
void k_quant_rows(cudaStream_t s, const float* x, int ldx, int8_t* q, int ldq, float* sc, int ldsc, int rows, int k) {
    report("k_quant_rows", b200q_quant_rows(x, B200Q_F32, ldx, q, ldq, sc, ldsc, rows, k, s));
}

// moe_up (bolt_kernels.cu:682-688): act[p][0 .. width) = relu(W_up[e] . x[p / 9])^2 over the latent (k 1024)
void moe_up(cudaStream_t s, const IQ2Slab& up, const MoeWork& w, const int8_t* xq, const float* xs, float* act, int width,
            int pairs) {
    if (pairs <= 0) return;
    GemvArgs a = slab_args(up, w, width, kBoltLatent, kBoltTopN);
    a.xq = xq;
    a.xs = xs;
    a.y = act;
    a.ldy = width;
    report("moe_up", launch_iq2_gemv(a, kBoltSlots, 16, 1, s));
}

// moe_down (bolt_kernels.cu:689-695): out[p][0 .. 1024) = W_down[e] . act[p] (k = width)
void moe_down(cudaStream_t s, const IQ2Slab& down, const MoeWork& w, const int8_t* xq, const float* xs, float* out,
              int width, int pairs) {
    if (pairs <= 0) return;
    GemvArgs a = slab_args(down, w, kBoltLatent, width, 1);
    a.xq = xq;
    a.xs = xs;
    a.y = out;
    a.ldy = kBoltLatent;
    report("moe_down", launch_iq2_gemv(a, kBoltSlots, 16, 0, s));
}

// moe_coop_dense (bolt_kernels.cu:881-887): one IQ2 matrix (n rows, a slab of one) over T rows, epi 1 relu^2
void moe_coop_dense(cudaStream_t s, const IQ2Slab& w, const MoeWork& mw, int T, const int8_t* xq, const float* xs, float* y,
                    int ldy, int n, int k, int epi) {
    (void)mw;   // libbolt's one-expert work list: the dense launch needs none
    if (T <= 0) return;
    GemvArgs a = {};
    a.slab = w.qs;
    a.dplane = (const uint8_t*)w.d;
    a.n = n;
    a.k = k;
    a.dense_rows = T;
    a.act_div = 1;
    a.act_split = 1 << 30;
    a.xq = xq;
    a.xs = xs;
    a.y = y;
    a.ldy = ldy;
    report("moe_coop_dense", launch_iq2_gemv(a, 1, T, epi ? 1 : 0, s));
}

// moe_tile_dense (bolt_kernels.cu:888-893): libbolt's shared expert at prompt row counts (enqueue_block picks it for
// T >= 256, bolt_host.cu:674), on the int8 rows like moe_coop_dense; here the same dense expert GEMV, which takes any T
void moe_tile_dense(cudaStream_t s, const IQ2Slab& w, const MoeWork& mw, int T, const int8_t* xq, const float* xs, float* y,
                    int ldy, int n, int k, int epi) {
    moe_coop_dense(s, w, mw, T, xq, xs, y, ldy, n, k, epi);
}

// moe_bf16 (bolt_kernels.cu:1040): whether enqueue_block takes libbolt's opt-in bf16 routed path (BOLT_MOE_BF=1,
// bolt_host.cu:702) instead of its default int8 one.  That path is not provided here, so the answer is always no, and
// moe_up_bf / moe_down_bf exist so that libbolt's host links; called anyway, they report and do nothing.
bool moe_bf16() { return false; }
void moe_up_bf(cudaStream_t, const IQ2Slab&, const MoeWork&, const float*, int, float*, int, int) {
    fprintf(stderr, "b200q shim: moe_up_bf failed: the bf16 routed path is not provided (moe_bf16() is false)\n");
}
void moe_down_bf(cudaStream_t, const IQ2Slab&, const MoeWork&, const float*, int, float*, int, int) {
    fprintf(stderr, "b200q shim: moe_down_bf failed: the bf16 routed path is not provided (moe_bf16() is false)\n");
}

// combine_k (bolt_kernels.cu:1714-1727): out[t][0 .. 1024) = sum over the 9 picks of rw * o[t * 9 + k]
void k_combine(cudaStream_t s, const float* o, const float* rw, float* out, int T) {
    report("k_combine", b200q_combine(o, rw, nullptr, T, kBoltTopN, kBoltLatent, out, B200Q_F32, s));
}

// tile_bytes_* (bolt_mma.cu:1221-1224): ceil(n/16) units of 16 rows a 64 (NVFP4) or 32 (Q8_0) k, 512 code bytes each,
// and 64 / 32 scale bytes each
size_t tile_bytes_nv4(int n, int k) { return (size_t)((n + 15) / 16) * (k / 64) * 512; }
size_t tile_scale_bytes_nv4(int n, int k) { return (size_t)((n + 15) / 16) * (k / 64) * 64; }
size_t tile_bytes_q8(int n, int k) { return (size_t)((n + 15) / 16) * (k / 32) * 512; }
size_t tile_scale_bytes_q8(int n, int k) { return (size_t)((n + 15) / 16) * (k / 32) * 32; }

// tile_nv4 / tile_q8 (bolt_mma.cu:1365-1366, via load_nv4 / load_q8 bolt_host.cu:198-264)
void tile_nv4(cudaStream_t s, const uint8_t* q, const uint8_t* sc, void* qt, void* sct, int n, int k) {
    if (!q || !sc || !qt || !sct || n <= 0 || n % 16 || k <= 0 || k % 256) {
        report("tile_nv4", B200Q_EINVAL);
        return;
    }
    report("tile_nv4", launch_nv4_pack_split(q, sc, (uint8_t*)qt, (uint8_t*)sct, n, k, s));
}
void tile_q8(cudaStream_t s, const uint8_t* raw, void* qt, void* dt, int n, int k) {
    if (!raw || !qt || !dt || n <= 0 || n % 16 || k <= 0 || k % 256) {
        report("tile_q8", B200Q_EINVAL);
        return;
    }
    report("tile_q8", launch_q8_pack_split(raw, (uint8_t*)qt, (uint8_t*)dt, n, k, s));
}

// mma_nv4 / mma_q8 (bolt_mma.cu:1190-1194): y = s2 * sum e2m1 * e4m3 * x, y = sum (q * d) * x, fp32 rows
void mma_nv4(cudaStream_t s, const TNV4& w, const float* x, int ldx, float* y, int ldy, int T) {
    tc_rows("mma_nv4", kTcNv4, (const uint8_t*)w.q, (const uint8_t*)w.sc, w.s2, w.n, w.k, x, ldx, y, ldy, T, s);
}
void mma_q8(cudaStream_t s, const TQ8& w, const float* x, int ldx, float* y, int ldy, int T) {
    tc_rows("mma_q8", kTcQ8, (const uint8_t*)w.q, (const uint8_t*)w.d, 1.f, w.n, w.k, x, ldx, y, ldy, T, s);
}
// mma_q8_multi (bolt_mma.cu:1204-1217): each matrix over the same rows
void mma_q8_multi(cudaStream_t s, const TQ8Multi& m, const float* x, int ldx, int T) {
    for (int i = 0; i < 3; i++)
        if (m.w[i].n > 0)
            tc_rows("mma_q8_multi", kTcQ8, (const uint8_t*)m.w[i].q, (const uint8_t*)m.w[i].d, 1.f, m.w[i].n,
                    m.w[i].k, x, ldx, m.y[i], m.ldy[i], T, s);
}

// tile_nv4w (bolt_mma.cu:892-923, via load_nv4w bolt_host.cu:218-238): the checkpoint's q [n][k/2] and sc [n][k/16]
// into the weight planes, in libbolt's two buffers (tile_bytes_nv4 / tile_scale_bytes_nv4 bytes)
void tile_nv4w(cudaStream_t s, const uint8_t* q, const uint8_t* sc, void* qw, void* sfw, int n, int k) {
    report("tile_nv4w", nv4_planes_pack(q, sc, (uint8_t*)qw, (uint8_t*)sfw, n, k, s));
}
// quant_nv4_rows (bolt_mma.cu:926-951): libbolt's plain rows, the same bytes
void quant_nv4_rows(cudaStream_t s, const float* x, int ldx, uint8_t* q4, uint8_t* sf, int T, int k) {
    report("quant_nv4_rows", nv4_quant_plain(x, ldx, q4, sf, T, k, s));
}
// mma_nv4_fp4 (bolt_mma.cu:961-1059): the tcgen05 block-scaled fp4 GEMM over the planes and the plain rows
void mma_nv4_fp4(cudaStream_t s, const TNV4W& w, const uint8_t* q4, const uint8_t* sf, float* y, int ldy, int T) {
    if (T <= 0) return;
    const size_t need = b200q_nv4_rows_bytes(T, w.k);
    if (need == 0) {
        report("mma_nv4_fp4", B200Q_EINVAL);
        return;
    }
    size_t have = 0;
    uint8_t* img = (uint8_t*)shim_ws(s, need, &have, kWsFp4Rows);
    if (!img || have < need) {
        report("mma_nv4_fp4", B200Q_ENOSPACE);   // first grown inside a stream capture
        return;
    }
    report("mma_nv4_fp4", nv4_gemm_planes((const uint8_t*)w.q, (const uint8_t*)w.sf, w.n, w.k, w.s2, q4, sf, T, img, y,
                                          ldy, s));
}

// tile_bytes_iq2 / tile_scale_bytes_iq2 (bolt_mma.cu:1226-1227): 64 code bytes and one fp16 scale a row and 256 k,
// the byte counts of this engine's split rt32 planes (2048 + 64 bytes a 32-row unit)
size_t tile_bytes_iq2(int n, int k) { return (size_t)((n + 15) / 16) * (k / 64) * 256; }
size_t tile_scale_bytes_iq2(int n, int k) { return (size_t)((n + 15) / 16) * (k / 256) * 32; }

// tile_iq2 (bolt_mma.cu:1336-1361, via load_iq2 bolt_host.cu:266-283): the checkpoint's blocks [n][k/256][66] into qt
// (codes) and dt (scales) as the split rt32 layout; n % 32 == 0
void tile_iq2(cudaStream_t s, const uint8_t* raw, void* qt, void* dt, int n, int k) {
    if (!raw || !qt || !dt || n <= 0 || n % kIq2Tile || k <= 0 || k % 256) {
        report("tile_iq2", B200Q_EINVAL);
        return;
    }
    report("tile_iq2", launch_iq2_pack_split(raw, (uint8_t*)qt, (uint8_t*)dt, n, k, s));
}

// mma_iq2 (bolt_mma.cu:1196-1203), the shared expert (bolt_host.cu:680-681): y[t] = W x[t], epi 1 = relu(.)^2.  The
// rows are quantised to int8 per 32 (quant_rows_k) into a per-stream scratch and the dense expert GEMV runs on them,
// the arithmetic libbolt's moe_coop_dense / moe_tile_dense use for the shared expert; libbolt's mma_iq2 rounds the
// rows to bf16 instead, and the two agree to the rows' rounding.
void mma_iq2(cudaStream_t s, const TIQ2& w, const float* x, int ldx, float* y, int ldy, int T, int epi) {
    if (T <= 0) return;
    if (!w.q || !w.d || !x || !y || w.n <= 0 || w.n % kIq2Tile || w.k <= 0 || w.k % 256 || ldx < w.k || ldy < w.n) {
        report("mma_iq2", B200Q_EINVAL);
        return;
    }
    const size_t qbytes = ((size_t)T * w.k + 255) / 256 * 256;
    size_t have = 0;
    uint8_t* rows = (uint8_t*)shim_ws(s, qbytes + (size_t)T * (w.k / 32) * sizeof(float), &have, kWsRows);
    if (!rows || have < qbytes + (size_t)T * (w.k / 32) * sizeof(float)) {
        report("mma_iq2", B200Q_ENOSPACE);   // first grown inside a stream capture
        return;
    }
    int8_t* xq = (int8_t*)rows;
    float* xs = (float*)(rows + qbytes);
    const int st = b200q_quant_rows(x, B200Q_F32, ldx, xq, w.k, xs, w.k / 32, T, w.k, s);
    if (st != B200Q_OK) {
        report("mma_iq2", st);
        return;
    }
    GemvArgs a = {};
    a.slab = (const uint8_t*)w.q;
    a.dplane = (const uint8_t*)w.d;
    a.n = w.n;
    a.k = w.k;
    a.dense_rows = T;
    a.act_div = 1;
    a.act_split = 1 << 30;
    a.xq = xq;
    a.xs = xs;
    a.y = y;
    a.ldy = ldy;
    report("mma_iq2", launch_iq2_gemv(a, 1, T, epi ? 1 : 0, s));
}
