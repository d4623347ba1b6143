// TEST INFRASTRUCTURE: C entry points that call libb200q's libbolt-signature shims (include/b200q_bolt.h) the way
// libbolt's host code does, building IQ2Slab / MoeWork from plain pointers, so tests/test_gpu_bolt_shim.py can drive
// them through ctypes.  Built by tests/build_harness.py into tests/_build/libbolt_shim_harness.so.
#include "b200q_bolt.h"

extern "C" {

void hs_repack_iq2(void* s, const void* src, void* qs, void* d, size_t rows, int k) {
    repack_iq2((cudaStream_t)s, (const uint8_t*)src, (uint8_t*)qs, d, rows, k);
}

void hs_k_route(void* s, const float* logits, int ldl, const float* bias, int* ridx, float* rw, int E, float scale, int T) {
    k_route((cudaStream_t)s, logits, ldl, bias, ridx, rw, E, scale, T);
}

void hs_k_moe_group(void* s, const int* ridx, int pairs, int* order, int* first, int* count, int* exp, int* nwork) {
    k_moe_group((cudaStream_t)s, ridx, pairs, order, first, count, exp, nwork, nullptr);
}

void hs_k_quant_rows(void* s, const float* x, int ldx, int8_t* q, int ldq, float* sc, int ldsc, int rows, int k) {
    k_quant_rows((cudaStream_t)s, x, ldx, q, ldq, sc, ldsc, rows, k);
}

// moe_up / moe_down with the slab and work list as enqueue_block builds them (bolt_host.cu:700-713)
void hs_moe_up(void* s, const void* qs, const void* d, size_t qs_stride, size_t d_stride, int* order, int* first,
               int* count, int* exp, int* nwork, const int8_t* xq, const float* xs, float* act, int width, int pairs) {
    const IQ2Slab up{(const uint8_t*)qs, d, qs_stride, d_stride};
    const MoeWork w{order, first, count, exp, nwork};
    moe_up((cudaStream_t)s, up, w, xq, xs, act, width, pairs);
}

void hs_moe_down(void* s, const void* qs, const void* d, size_t qs_stride, size_t d_stride, int* order, int* first,
                 int* count, int* exp, int* nwork, const int8_t* xq, const float* xs, float* out, int width, int pairs) {
    const IQ2Slab down{(const uint8_t*)qs, d, qs_stride, d_stride};
    const MoeWork w{order, first, count, exp, nwork};
    moe_down((cudaStream_t)s, down, w, xq, xs, out, width, pairs);
}

void hs_moe_coop_dense(void* s, const void* qs, const void* d, int T, const int8_t* xq, const float* xs, float* y, int ldy,
                       int n, int k, int epi) {
    const IQ2Slab w{(const uint8_t*)qs, d, 0, 0};
    const MoeWork mw{nullptr, nullptr, nullptr, nullptr, nullptr};
    moe_coop_dense((cudaStream_t)s, w, mw, T, xq, xs, y, ldy, n, k, epi);
}

void hs_moe_tile_dense(void* s, const void* qs, const void* d, int T, const int8_t* xq, const float* xs, float* y, int ldy,
                       int n, int k, int epi) {
    const IQ2Slab w{(const uint8_t*)qs, d, 0, 0};
    const MoeWork mw{nullptr, nullptr, nullptr, nullptr, nullptr};
    moe_tile_dense((cudaStream_t)s, w, mw, T, xq, xs, y, ldy, n, k, epi);
}

int hs_moe_bf16(void) { return moe_bf16() ? 1 : 0; }

void hs_moe_up_bf(void* s) {
    const IQ2Slab w{nullptr, nullptr, 0, 0};
    const MoeWork mw{nullptr, nullptr, nullptr, nullptr, nullptr};
    moe_up_bf((cudaStream_t)s, w, mw, nullptr, 0, nullptr, 0, 0);
    moe_down_bf((cudaStream_t)s, w, mw, nullptr, 0, nullptr, 0, 0);
}

void hs_k_combine(void* s, const float* o, const float* rw, float* out, int T) {
    k_combine((cudaStream_t)s, o, rw, out, T);
}

// fmt 0 NVFP4, 1 Q8_0, 2 IQ2_XXS
size_t hs_tile_bytes(int fmt, int scales, int n, int k) {
    if (fmt == 0) return scales ? tile_scale_bytes_nv4(n, k) : tile_bytes_nv4(n, k);
    if (fmt == 1) return scales ? tile_scale_bytes_q8(n, k) : tile_bytes_q8(n, k);
    return scales ? tile_scale_bytes_iq2(n, k) : tile_bytes_iq2(n, k);
}

void hs_tile_iq2(void* s, const uint8_t* raw, void* qt, void* dt, int n, int k) { tile_iq2((cudaStream_t)s, raw, qt, dt, n, k); }

// the shared expert's up (epi 1) and down as enqueue_block calls them (bolt_host.cu:680-681)
void hs_mma_iq2(void* s, const void* qt, const void* dt, int n, int k, const float* x, int ldx, float* y, int ldy, int T,
                int epi) {
    const TIQ2 w{(const uint4*)qt, (const uint16_t*)dt, n, k};
    mma_iq2((cudaStream_t)s, w, x, ldx, y, ldy, T, epi);
}

void hs_tile_nv4(void* s, const uint8_t* q, const uint8_t* sc, void* qt, void* sct, int n, int k) {
    tile_nv4((cudaStream_t)s, q, sc, qt, sct, n, k);
}

void hs_tile_q8(void* s, const uint8_t* raw, void* qt, void* dt, int n, int k) { tile_q8((cudaStream_t)s, raw, qt, dt, n, k); }

// mma_nv4 / mma_q8 with the views load_nv4 / load_q8 return (bolt_host.cu:198-264)
void hs_mma_nv4(void* s, const void* qt, const void* sct, float s2, int n, int k, const float* x, int ldx, float* y,
                int ldy, int T) {
    const TNV4 w{(const uint4*)qt, (const uint2*)sct, s2, n, k};
    mma_nv4((cudaStream_t)s, w, x, ldx, y, ldy, T);
}

void hs_mma_q8(void* s, const void* qt, const void* dt, int n, int k, const float* x, int ldx, float* y, int ldy, int T) {
    const TQ8 w{(const uint4*)qt, (const uint32_t*)dt, n, k};
    mma_q8((cudaStream_t)s, w, x, ldx, y, ldy, T);
}

// libbolt's BOLT_NV4_FP4 prompt path with the views load_nv4w returns (bolt_host.cu:218-238, 634, 644)
void hs_tile_nv4w(void* s, const uint8_t* q, const uint8_t* sc, void* qw, void* sfw, int n, int k) {
    tile_nv4w((cudaStream_t)s, q, sc, qw, sfw, n, k);
}
void hs_quant_nv4_rows(void* s, const float* x, int ldx, uint8_t* q4, uint8_t* sf, int T, int k) {
    quant_nv4_rows((cudaStream_t)s, x, ldx, q4, sf, T, k);
}
void hs_mma_nv4_fp4(void* s, const void* qw, const void* sfw, float s2, int n, int k, const uint8_t* q4,
                    const uint8_t* sf, float* y, int ldy, int T) {
    const TNV4W w{(const uint4*)qw, (const uint32_t*)sfw, s2, n, k};
    mma_nv4_fp4((cudaStream_t)s, w, q4, sf, y, ldy, T);
}

// three matrices: q* / d* / n* / y* / ldy* for each (n = 0 leaves one unused)
void hs_mma_q8_multi(void* s, const void* const* qt, const void* const* dt, const int* n, int k, const float* x, int ldx,
                     float* const* y, const int* ldy, int T) {
    TQ8Multi m{};
    for (int i = 0; i < 3; i++) {
        m.w[i] = TQ8{(const uint4*)qt[i], (const uint32_t*)dt[i], n[i], n[i] ? k : 0};
        m.y[i] = y[i];
        m.ldy[i] = ldy[i];
    }
    mma_q8_multi((cudaStream_t)s, m, x, ldx, T);
}

}  // extern "C"

// ---------------------------------------------------------------------------------------------------------
// Timed loops (bench.py's libbolt-shape measurement): `iters` launches of one shim on a stream of its own, timed with
// events on that stream; ms a launch (negative on a CUDA error).  The same loop as oracle/ref_shim.cu's for libbolt's
// own launchers, so the two are timed alike.
// ---------------------------------------------------------------------------------------------------------
template <class F>
static float hs_timed(int iters, F f) {
    cudaStream_t s;
    if (cudaStreamCreateWithFlags(&s, cudaStreamNonBlocking) != cudaSuccess) return -1.f;
    cudaEvent_t e0, e1;
    cudaEventCreate(&e0);
    cudaEventCreate(&e1);
    for (int i = 0; i < 3; i++) f(s, i);
    cudaEventRecord(e0, s);
    for (int i = 0; i < iters; i++) f(s, i);
    cudaEventRecord(e1, s);
    float ms = -1.f;
    if (cudaEventSynchronize(e1) == cudaSuccess) cudaEventElapsedTime(&ms, e0, e1);
    cudaEventDestroy(e0);
    cudaEventDestroy(e1);
    cudaStreamDestroy(s);
    return cudaGetLastError() == cudaSuccess ? ms / iters : -1.f;
}

extern "C" {

float hs_time_moe(int which, int iters, int copies, const void* const* qs, const void* const* d, size_t qs_stride,
                  size_t d_stride, int* order, int* first, int* count, int* exp, int* nwork, const int8_t* xq,
                  const float* xs, float* y, int width, int pairs) {
    const MoeWork w{order, first, count, exp, nwork};
    return hs_timed(iters, [&](cudaStream_t s, int i) {
        const IQ2Slab slab{(const uint8_t*)qs[i % copies], d[i % copies], qs_stride, d_stride};
        if (which == 0) moe_up(s, slab, w, xq, xs, y, width, pairs);
        else moe_down(s, slab, w, xq, xs, y, width, pairs);
    });
}

float hs_time_mma(int fmt, int iters, int copies, const void* const* qt, const void* const* st, float s2, int n, int k,
                  const float* x, float* y, int T) {
    return hs_timed(iters, [&](cudaStream_t s, int i) {
        const int c = i % copies;
        if (fmt == 0) mma_nv4(s, TNV4{(const uint4*)qt[c], (const uint2*)st[c], s2, n, k}, x, k, y, n, T);
        else if (fmt == 1) mma_q8(s, TQ8{(const uint4*)qt[c], (const uint32_t*)st[c], n, k}, x, k, y, n, T);
        else mma_iq2(s, TIQ2{(const uint4*)qt[c], (const uint16_t*)st[c], n, k}, x, k, y, n, T, 0);
    });
}

}  // extern "C"
