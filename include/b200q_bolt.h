/* libbolt's operator launchers (the reference engine's engine/bolt_common.h:77-161), declared with libbolt's own
 * names, signatures and view structs and backed by libb200q (csrc/bolt_shim.cu), so that libbolt's host code
 * (bolt_host.cu's enqueue_block and load_slab) links against this engine for the routed-expert MoE block:
 *   load time   repack_iq2 (into the same qs / d buffers load_slab allocates, in this engine's split rt32 layout);
 *   per block   k_route, k_moe_group, k_quant_rows, moe_up, moe_down, k_combine; moe_coop_dense / moe_tile_dense
 *               for the shared expert; moe_bf16 (false) and the reporting stubs moe_up_bf / moe_down_bf.
 * and for the Mamba and attention projections (load_nv4 / load_q8, bolt_host.cu:198-264, and their decode calls):
 *   load time   tile_bytes_nv4, tile_scale_bytes_nv4, tile_bytes_q8, tile_scale_bytes_q8, tile_nv4, tile_q8 (the same
 *               buffer sizes as libbolt's tiles, holding this engine's t16 units split into a code plane and a scale
 *               plane);
 *   per step    mma_nv4, mma_q8, mma_q8_multi;
 * and for the prompt chunks' NVFP4 projections on the fp4 tensor cores (BOLT_NV4_FP4): tile_nv4w at load time,
 *               quant_nv4_rows + mma_nv4_fp4 per chunk;
 * and for the shared expert (load_iq2, bolt_host.cu:266-283, and bolt_host.cu:680-681): tile_bytes_iq2,
 * tile_scale_bytes_iq2, tile_iq2, mma_iq2.
 * The structs repeat libbolt's member order and types so the bytes match.  libbolt's fixed model shapes stay fixed
 * here: the latent width 1024 (moe_up's k, moe_down's n, k_combine's width) and TOPN = 9 routed experts a token.
 * As in libbolt the launchers are asynchronous on the given stream and return nothing; a launch error is printed
 * (prefix "b200q shim") and left for the caller's cudaGetLastError.  mma_nv4, mma_q8, mma_q8_multi and mma_iq2
 * take no scratch argument (libbolt's keep a row scratch a stream, mma_pack_buffer): they keep one buffer a
 * (device, stream), allocated at the first call outside stream capture, so a captured sequence should be run once
 * before it is captured. */
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
/* the same for prompt row counts (enqueue_block's choice at T >= 256) */
void moe_tile_dense(cudaStream_t s, const IQ2Slab& w, const MoeWork& mw, int T, const int8_t* xq, const float* xs, float* y,
                    int ldy, int n, int k, int epi);
/* libbolt's opt-in bf16 routed path (BOLT_MOE_BF=1) is not provided: moe_bf16() is false, and moe_up_bf /
 * moe_down_bf only report (they exist so that libbolt's host links) */
bool moe_bf16();
void moe_up_bf(cudaStream_t s, const IQ2Slab& up, const MoeWork& w, const float* x, int ldx, float* act, int width, int pairs);
void moe_down_bf(cudaStream_t s, const IQ2Slab& down, const MoeWork& w, const float* act, int ldx, float* out, int width,
                 int pairs);
void k_combine(cudaStream_t s, const float* o, const float* rw, float* out, int T);

/* an NVFP4 matrix (n rows, k): q = the 512 code bytes of each 16-row x 64-k unit, sc = its 64 e4m3 scale bytes,
 * s2 = the tensor's second-level scale (bolt_common.h:43) */
struct TNV4 { const uint4* q; const uint2* sc; float s2; int n, k; };
/* a Q8_0 matrix: q = the 512 int8 bytes of each 16-row x 32-k unit, d = its 16 fp16 scales (bolt_common.h:47) */
struct TQ8 { const uint4* q; const uint32_t* d; int n, k; };
/* up to three Q8_0 matrices over the same rows (the attention q / k / v, bolt_common.h:125) */
struct TQ8Multi { TQ8 w[3]; float* y[3]; int ldy[3]; };

size_t tile_bytes_nv4(int n, int k);
size_t tile_scale_bytes_nv4(int n, int k);
size_t tile_bytes_q8(int n, int k);
size_t tile_scale_bytes_q8(int n, int k);
/* q [n][k/2] (low nibble first), sc [n][k/16] e4m3 -> qt, sct; raw = ggml Q8_0 blocks [n][k/32][34] -> qt, dt.
 * n % 16 == 0, k % 256 == 0 */
void tile_nv4(cudaStream_t s, const uint8_t* q, const uint8_t* sc, void* qt, void* sct, int n, int k);
void tile_q8(cudaStream_t s, const uint8_t* raw, void* qt, void* dt, int n, int k);
/* y[t][0 .. n) = W x[t] for t < T (fp32 rows; 16-row pieces at a time, each one decode GEMV) */
void mma_nv4(cudaStream_t s, const TNV4& w, const float* x, int ldx, float* y, int ldy, int T);
void mma_q8(cudaStream_t s, const TQ8& w, const float* x, int ldx, float* y, int ldy, int T);
/* each matrix with n > 0 (libbolt leaves an unused one zeroed) into its own y */
void mma_q8_multi(cudaStream_t s, const TQ8Multi& m, const float* x, int ldx, int T);

/* libbolt's BOLT_NV4_FP4 prompt path (bolt_common.h:115-121, load_nv4w bolt_host.cu:218-238, calls at
 * bolt_host.cu:634,644): an NVFP4 matrix for the block-scaled fp4 tensor cores (bolt_common.h:46).  With this engine's
 * tile_nv4w, q (libbolt's tile_bytes_nv4(n, k) buffer) and sf (its tile_scale_bytes_nv4 buffer) hold the code and
 * scale planes of the tcgen05 GEMM's weight image (256-row tiles; a last tile of 128 rows when n % 256 == 128,
 * in_proj's 18560), exactly libbolt's byte counts.  n % 128 == 0, k % 256 == 0. */
struct TNV4W { const uint4* q; const uint32_t* sf; float s2; int n, k; };
void tile_nv4w(cudaStream_t s, const uint8_t* q, const uint8_t* sc, void* qw, void* sfw, int n, int k);
/* x fp32 [T][ldx] -> q4 [T][k/2] (e2m1, low nibble first), sf [T][k/16] (e4m3 of amax/6 a block of 16): libbolt's
 * layout and bytes (quant_nv4_rows_k's steps) */
void quant_nv4_rows(cudaStream_t s, const float* x, int ldx, uint8_t* q4, uint8_t* sf, int T, int k);
/* y[t][0 .. n) = s2 * sum_k (q4, sf)[t] (w.q, w.sf)[row], fp32 sums on the tcgen05 block-scaled fp4 MMA
 * (kind::mxf4nvf4).  The rows are rearranged into the GEMM's rows image in a scratch of (device, stream), allocated at
 * the first call outside stream capture, as mma_nv4's is. */
void mma_nv4_fp4(cudaStream_t s, const TNV4W& w, const uint8_t* q4, const uint8_t* sf, float* y, int ldy, int T);

/* an IQ2_XXS matrix: q = 64 code bytes a row and 256 k, d = one fp16 scale a row and 256 k (bolt_common.h:49); with
 * this engine's tile_iq2 they hold the split rt32 planes (n % 32 == 0) */
struct TIQ2 { const uint4* q; const uint16_t* d; int n, k; };
size_t tile_bytes_iq2(int n, int k);
size_t tile_scale_bytes_iq2(int n, int k);
void tile_iq2(cudaStream_t s, const uint8_t* raw, void* qt, void* dt, int n, int k);
/* y[t][0 .. n) = W x[t] (epi 1: relu(.)^2) for fp32 rows, computed on the rows quantised to int8 per 32 */
void mma_iq2(cudaStream_t s, const TIQ2& w, const float* x, int ldx, float* y, int ldy, int T, int epi = 0);
