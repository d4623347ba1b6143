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
