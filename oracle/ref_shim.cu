// ref_shim.cu -- TEST INFRASTRUCTURE ONLY.
//
// extern "C" entry points over libbolt's own kernels (the reference engine's bolt_kernels.cu, compiled from where it
// lies by oracle/build_oracle.py into oracle/_ref/libbolt_ref.so, never copied).  The GPU tests call them on the same
// seeded inputs as the CPU oracle to pin the oracle to the reference itself, and to write the golden fixtures under
// tests/golden/.  Every wrapper passes its arguments straight to the reference launcher (bolt_common.h:77-157) and
// synchronises, so a test reads finished results.
#include "bolt_common.h"

#include <cuda_runtime.h>

extern "C" {

int ref_topn(void) { return TOPN; }

// k_quant_rows (bolt_kernels.cu:361-363)
int ref_quant_rows(const float* x, int ldx, int8_t* q, int ldq, float* sc, int ldsc, int rows, int k) {
    k_quant_rows(0, x, ldx, q, ldq, sc, ldsc, rows, k);
    return (int)cudaDeviceSynchronize();
}

// k_route (bolt_kernels.cu:1710-1712): sigmoid + bias, top TOPN, scaled
int ref_route(const float* logits, int ldl, const float* bias, int* ridx, float* rw, int E, float scale, int T) {
    k_route(0, logits, ldl, bias, ridx, rw, E, scale, T);
    return (int)cudaDeviceSynchronize();
}

// k_moe_group (bolt_kernels.cu:342-344)
int ref_moe_group(const int* ridx, int pairs, int* order, int* first, int* n, int* exp, int* n_work) {
    k_moe_group(0, ridx, pairs, order, first, n, exp, n_work, nullptr);
    return (int)cudaDeviceSynchronize();
}

// repack_iq2 (bolt_kernels.cu:1064-1067): ggml blocks -> planar qs [rows][k/256][64], d [rows][k/256]
int ref_repack_iq2(const uint8_t* src, uint8_t* qs, void* d, size_t rows, int k) {
    repack_iq2(0, src, qs, d, rows, k);
    return (int)cudaDeviceSynchronize();
}

// moe_up / moe_down (bolt_kernels.cu:682-695): the routed experts at libbolt's own shapes (k 1024 up, n 1024 down)
int ref_moe_up(const uint8_t* qs, const void* d, size_t qs_stride, size_t d_stride, int* order, int* first, int* count,
               int* expert, int* n_work, const int8_t* xq, const float* xs, float* act, int width, int pairs) {
    IQ2Slab slab{qs, d, qs_stride, d_stride};
    MoeWork w{order, first, count, expert, n_work};
    moe_up(0, slab, w, xq, xs, act, width, pairs);
    return (int)cudaDeviceSynchronize();
}
int ref_moe_down(const uint8_t* qs, const void* d, size_t qs_stride, size_t d_stride, int* order, int* first, int* count,
                 int* expert, int* n_work, const int8_t* xq, const float* xs, float* out, int width, int pairs) {
    IQ2Slab slab{qs, d, qs_stride, d_stride};
    MoeWork w{order, first, count, expert, n_work};
    moe_down(0, slab, w, xq, xs, out, width, pairs);
    return (int)cudaDeviceSynchronize();
}

// moe_coop_dense (bolt_kernels.cu:881-887): one IQ2 matrix over T int8 rows at any n, k
int ref_moe_coop_dense(const uint8_t* qs, const void* d, int* order, int* first, int* count, int* expert, int* n_work, int T,
                       const int8_t* xq, const float* xs, float* y, int ldy, int n, int k, int epi) {
    IQ2Slab slab{qs, d, 0, 0};
    MoeWork w{order, first, count, expert, n_work};
    moe_coop_dense(0, slab, w, T, xq, xs, y, ldy, n, k, epi);
    return (int)cudaDeviceSynchronize();
}

// k_combine (bolt_kernels.cu:1727): 1024 wide, TOPN pairs a token
int ref_combine(const float* o, const float* rw, float* out, int T) {
    k_combine(0, o, rw, out, T);
    return (int)cudaDeviceSynchronize();
}

// the fp32 dequant GEMVs (bolt_kernels.cu:228-240), T <= 16
int ref_gemv_iq2(const uint8_t* qs, const void* d, int n, int k, const float* x, int ldx, float* y, int ldy, int T, int epi) {
    IQ2W w{qs, d, n, k};
    gemv_iq2(0, w, x, ldx, y, ldy, T, epi);
    return (int)cudaDeviceSynchronize();
}
int ref_gemv_nv4(const uint8_t* q, const uint8_t* sc, float s2, int n, int k, const float* x, int ldx, float* y, int ldy, int T) {
    NV4W w{q, sc, s2, n, k};
    gemv_nv4(0, w, x, ldx, y, ldy, T);
    return (int)cudaDeviceSynchronize();
}
int ref_gemv_q8(const int8_t* q, const void* d, int n, int k, const float* x, int ldx, float* y, int ldy, int T) {
    Q8W w{q, d, n, k};
    gemv_q8(0, w, x, ldx, y, ldy, T, 0);
    return (int)cudaDeviceSynchronize();
}

}  // extern "C"

// ---------------------------------------------------------------------------------------------------------
// The tensor-core GEMMs of engine/bolt_mma.cu (compiled from a copy whose one sm_12x-only instruction is guarded out;
// mma_nv4_fp4 is never called here): the tile packers, the decode/verify GEMMs mma_nv4 / mma_q8 / mma_iq2, and the
// NVFP4 row quantiser of the prompt path.
// ---------------------------------------------------------------------------------------------------------
extern "C" {

size_t ref_tile_bytes(int fmt, int n, int k) {   // fmt 0 nv4, 1 q8, 2 iq2: the code tile
    return fmt == 0 ? tile_bytes_nv4(n, k) : fmt == 1 ? tile_bytes_q8(n, k) : tile_bytes_iq2(n, k);
}
size_t ref_tile_scale_bytes(int fmt, int n, int k) {
    return fmt == 0 ? tile_scale_bytes_nv4(n, k) : fmt == 1 ? tile_scale_bytes_q8(n, k) : tile_scale_bytes_iq2(n, k);
}
int ref_tile_nv4(const uint8_t* q, const uint8_t* sc, void* qt, void* sct, int n, int k) {
    tile_nv4(0, q, sc, qt, sct, n, k);
    return (int)cudaDeviceSynchronize();
}
int ref_tile_q8(const uint8_t* raw, void* qt, void* dt, int n, int k) {
    tile_q8(0, raw, qt, dt, n, k);
    return (int)cudaDeviceSynchronize();
}
int ref_tile_iq2(const uint8_t* raw, void* qt, void* dt, int n, int k) {
    tile_iq2(0, raw, qt, dt, n, k);
    return (int)cudaDeviceSynchronize();
}
// y [T][n] fp32 = x [T][k] fp32 . W^T (bolt_mma.cu:1190-1203)
int ref_mma_nv4(const void* qt, const void* sct, float s2, int n, int k, const float* x, int ldx, float* y, int ldy, int T) {
    TNV4 w{(const uint4*)qt, (const uint2*)sct, s2, n, k};
    mma_nv4(0, w, x, ldx, y, ldy, T);
    return (int)cudaDeviceSynchronize();
}
int ref_mma_q8(const void* qt, const void* dt, int n, int k, const float* x, int ldx, float* y, int ldy, int T) {
    TQ8 w{(const uint4*)qt, (const uint32_t*)dt, n, k};
    mma_q8(0, w, x, ldx, y, ldy, T);
    return (int)cudaDeviceSynchronize();
}
int ref_mma_iq2(const void* qt, const void* dt, int n, int k, const float* x, int ldx, float* y, int ldy, int T, int epi) {
    TIQ2 w{(const uint4*)qt, (const uint16_t*)dt, n, k};
    mma_iq2(0, w, x, ldx, y, ldy, T, epi);
    return (int)cudaDeviceSynchronize();
}
// rows to NVFP4 (quant_nv4_rows_k, bolt_mma.cu:925-951): q4 [T][k/2], sf step-major [k/64][(T+3)&~3][4]
int ref_quant_nv4_rows(const float* x, int ldx, uint8_t* q4, uint8_t* sf, int T, int k) {
    quant_nv4_rows(0, x, ldx, q4, sf, T, k);
    return (int)cudaDeviceSynchronize();
}

}  // extern "C"

// ---------------------------------------------------------------------------------------------------------
// Timed loops for the benchmark's reference arm: `iters` launches of one launcher on a stream of its own, timed with
// events on that stream; returns ms a launch (negative on a CUDA error).  Arguments as the wrappers above.
// ---------------------------------------------------------------------------------------------------------
template <class F>
static float timed(int iters, F f) {
    cudaStream_t s;
    if (cudaStreamCreateWithFlags(&s, cudaStreamNonBlocking) != cudaSuccess) return -1.f;
    cudaEvent_t e0, e1;
    cudaEventCreate(&e0);
    cudaEventCreate(&e1);
    for (int i = 0; i < 3; i++) f(s, i);   // warm-up
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

// moe_up or moe_down (which: 0 / 1) over `copies` slabs (rotated, to defeat L2), libbolt's shapes (k 1024, TOPN 9)
float ref_time_moe(int which, int iters, int copies, const uint8_t* const* qs, const void* const* d, size_t qs_stride,
                   size_t d_stride, int* order, int* first, int* count, int* expert, int* n_work, const int8_t* xq,
                   const float* xs, float* y, int width, int pairs) {
    MoeWork w{order, first, count, expert, n_work};
    return timed(iters, [&](cudaStream_t s, int i) {
        IQ2Slab slab{qs[i % copies], d[i % copies], qs_stride, d_stride};
        if (which == 0) moe_up(s, slab, w, xq, xs, y, width, pairs);
        else moe_down(s, slab, w, xq, xs, y, width, pairs);
    });
}
// the tile GEMMs over `copies` weight copies: fmt 0 mma_nv4, 1 mma_q8, 2 mma_iq2
float ref_time_mma(int fmt, int iters, int copies, const void* const* qt, const void* const* st, float s2, int n, int k,
                   const float* x, float* y, int T) {
    return timed(iters, [&](cudaStream_t s, int i) {
        const int c = i % copies;
        if (fmt == 0) mma_nv4(s, TNV4{(const uint4*)qt[c], (const uint2*)st[c], s2, n, k}, x, k, y, n, T);
        else if (fmt == 1) mma_q8(s, TQ8{(const uint4*)qt[c], (const uint32_t*)st[c], n, k}, x, k, y, n, T);
        else mma_iq2(s, TIQ2{(const uint4*)qt[c], (const uint16_t*)st[c], n, k}, x, k, y, n, T, 0);
    });
}

}  // extern "C"
