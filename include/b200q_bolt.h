/* libbolt's operator launchers (the reference engine's engine/bolt_common.h:77-161), declared with libbolt's own
 * names, signatures and view structs and backed by libb200q (csrc/bolt_shim.cu), so that libbolt's host code
 * (bolt_host.cu's enqueue_block and load_slab) links against this engine for the routed-expert MoE block:
 *   load time   repack_iq2 (into the same qs / d buffers load_slab allocates, in this engine's split rt32 layout);
 *   per block   k_route, k_moe_group, k_quant_rows, moe_up, moe_down, k_combine; moe_coop_dense for the shared
 *               expert.
 * The structs repeat libbolt's member order and types so the bytes match.  libbolt's fixed model shapes stay fixed
 * here: the latent width 1024 (moe_up's k, moe_down's n, k_combine's width) and TOPN = 9 routed experts a token.
 * As in libbolt the launchers are asynchronous on the given stream and return nothing; a launch error is printed
 * (prefix "b200q shim") and left for the caller's cudaGetLastError. */
#pragma once
#include <cuda_runtime.h>
#include <cstddef>
#include <cstdint>

/* all experts of one projection: expert e at qs + e * qs_stride bytes and d + e * d_stride halves; with this engine's
 * repack_iq2, qs holds each (32-row tile, 256-k) unit's 2048 chunk bytes and d its 32 rows' scales (64 bytes) */
struct IQ2Slab { const uint8_t* qs; const void* d; size_t qs_stride, d_stride; };
/* the grouping of a block's (token, expert) pairs; this engine's k_moe_group makes one item per expert slot
 * (512 of them): first = its offset in order, count = its pairs, expert = the slot, n_work = 512 */
struct MoeWork { int *order, *first, *count, *expert, *n_work; };

void repack_iq2(cudaStream_t s, const uint8_t* src, uint8_t* qs, void* d, size_t rows, int k);
void k_route(cudaStream_t s, const float* logits, int ldl, const float* bias, int* ridx, float* rw, int E, float scale, int T);
void k_moe_group(cudaStream_t s, const int* ridx, int pairs, int* order, int* work_first, int* work_n, int* work_exp,
                 int* n_work, int* stat);
void k_quant_rows(cudaStream_t s, const float* x, int ldx, int8_t* q, int ldq, float* sc, int ldsc, int rows, int k);
void moe_up(cudaStream_t s, const IQ2Slab& up, const MoeWork& w, const int8_t* xq, const float* xs, float* act, int width,
            int pairs);
void moe_down(cudaStream_t s, const IQ2Slab& down, const MoeWork& w, const int8_t* xq, const float* xs, float* out,
              int width, int pairs);
void moe_coop_dense(cudaStream_t s, const IQ2Slab& w, const MoeWork& mw, int T, const int8_t* xq, const float* xs, float* y,
                    int ldy, int n, int k, int epi);
void k_combine(cudaStream_t s, const float* o, const float* rw, float* out, int T);
