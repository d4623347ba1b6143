/*
 * b200q.h -- the C ABI of libb200q, a B200 (sm_100a) engine for the weight-bound quantized GEMMs of
 * Nemotron-3.5-Bolt: the IQ2_XXS routed-expert MoE, the NVFP4 Mamba-2 projections and the Q8_0 projections.
 *
 * It replaces the operator launchers of the reference engine libbolt (engine/bolt_common.h:77-157), which are
 * C++ functions returning void.  Here every entry point is extern "C", takes plain device pointers, sizes and
 * a stream (a cudaStream_t passed as void*), and returns a status:
 *     B200Q_OK (0)  enqueued;   B200Q_EINVAL (-1)  bad pointer or shape (libbolt's -1);
 *     B200Q_ECUDA (-3)  a CUDA launch error (libbolt's -3, run_blocks, bolt_host.cu:865-869);
 *     B200Q_ENOSPACE (-2)  a workspace or fixed capacity too small.
 * Every operator is asynchronous on its stream, allocates nothing, never synchronises and never reads device
 * data on the host, so a sequence of them can be captured in a CUDA graph (the reference captures
 * enqueue_block, bolt_host.cu:839-857).  The caller owns every buffer, scratch included; the *_workspace_bytes
 * queries give the scratch sizes.  Kernels use programmatic dependent launch like libbolt's (bolt_common.h:84-110);
 * B200Q_PDL=0 in the environment turns it off.
 *
 * Weight layouts.  The packers take the checkpoint's raw bytes (already on the device) and write this library's
 * layouts (same byte counts):
 *     IQ2_XXS  ggml blocks [rows][k/256][66]       -> b200q_iq2_pack      (n % 32 == 0, k % 256 == 0)
 *     Q8_0     ggml blocks [rows][k/32][34]        -> b200q_q8_pack       (n % 16 == 0, k % 256 == 0)
 *     NVFP4    q [rows][k/2], sc [rows][k/16] e4m3 -> b200q_nv4_pack      (n % 16 == 0, k % 256 == 0)
 * A slab of experts is packed as one matrix of experts*rows rows (every expert's rows are a multiple of 32), so
 * expert e starts at e * b200q_iq2_bytes(rows, k).
 */
#ifndef B200Q_H
#define B200Q_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define B200Q_ABI 1

#define B200Q_OK 0
#define B200Q_EINVAL (-1)
#define B200Q_ENOSPACE (-2)
#define B200Q_ECUDA (-3)

/* activation element types */
#define B200Q_F32 0
#define B200Q_BF16 1

/* router forms */
#define B200Q_ROUTE_SOFTMAX 0   /* softmax over the logits, top-k, renormalised to sum 1 */
#define B200Q_ROUTE_SIGMOID 1   /* sigmoid + bias, top-k, sigmoids normalised and scaled (route_k)           */

/* ABI version; libbolt's is bolt_abi() (bolt_host.cu:1139), checked by bolt_native.zig:516. */
int b200q_abi(void);
/* The CUDA error behind the last B200Q_ECUDA of this thread (cudaError_t as int), 0 if none. */
int b200q_last_cuda_error(void);
const char* b200q_strerror(int status);
/* Errors the kernels recorded on the current device (a bitmask, 0 if none; bit 0: a streaming GEMV's bounded wait for
 * its copies ran out, so its outputs are incomplete; bit 4: the same in an fp16 tensor-core GEMM; bit 8: in the NVFP4
 * tensor-core GEMM; bit 12: in the Q8_0 decode GEMV); synchronous.  clear != 0 resets it.  No counterpart in libbolt,
 * whose kernels do not wait on barriers. */
int b200q_device_error(int clear);

/* ---------------------------------------------------------------------------------------------------------
 * Load-time packers (raw checkpoint bytes on the device -> this library's layouts).
 * --------------------------------------------------------------------------------------------------------- */

/* Bytes of an IQ2_XXS matrix of n rows: n*k/256*66 (the checkpoint tensor [n][k/256][66], bolt_host.cu:269). */
size_t b200q_iq2_bytes(int64_t n, int k);
/* Replaces repack_iq2 (bolt_kernels.cu:1054-1068, via load_slab bolt_host.cu:306-328) and tile_iq2
 * (bolt_mma.cu:1336-1361): ggml blocks [n][k/256][66] -> the rt32 layout.  raw and packed must not overlap. */
int b200q_iq2_pack(const void* raw, void* packed, int64_t n, int k, void* stream);

/* Bytes of a Q8_0 matrix: n*k/32*34.  Replaces tile_q8 (bolt_mma.cu:1270-1311, via load_q8 bolt_host.cu:198-217):
 * ggml blocks [n][k/32][34] -> the t16 layout. */
size_t b200q_q8_bytes(int64_t n, int k);
int b200q_q8_pack(const void* raw, void* packed, int64_t n, int k, void* stream);

/* Bytes of an NVFP4 matrix: n*k/2 + n*k/16.  Replaces tile_nv4 / tile_nv4w (bolt_mma.cu:1231-1268, 892-923, via
 * load_nv4 bolt_host.cu:219-264): q [n][k/2] (low nibble first) and sc [n][k/16] e4m3 -> the t16 layout. */
size_t b200q_nv4_bytes(int64_t n, int k);
int b200q_nv4_pack(const void* q, const void* sc, void* packed, int64_t n, int k, void* stream);

/* ---------------------------------------------------------------------------------------------------------
 * NVFP4 and Q8_0 decode GEMVs: y[t][n] = W[n] . x[t] for T <= 16 rows, x fp32 or bf16 [T][ldx], y fp32 [T][ldy].
 * NVFP4: y = s2 * sum e2m1 * e4m3 * x (exact products, fp32 sums), replacing mma_nv4 (bolt_mma.cu:1190) at decode
 * and verify row counts.  Q8_0: y = sum (q * d) * x, replacing mma_q8 (bolt_mma.cu:1194) and gemv_q8
 * (bolt_kernels.cu:228-231).  K is split across CTAs; the fp32 partials go to `workspace`
 * (>= b200q_*_gemv_workspace_bytes, 0 when no split is needed) and are summed in a fixed order.  A NULL or small
 * workspace runs without the split (slower, same result order).  w must be 16-byte aligned (the packers' output in
 * any device allocation is); x on its element size (B200Q_EINVAL otherwise), any row pitch: rows on 4 elements are
 * read four values a load, rows on 2 elements by pairs, others one value at a time.
 * --------------------------------------------------------------------------------------------------------- */
size_t b200q_nv4_gemv_workspace_bytes(int n, int k, int T);
int b200q_nv4_gemv(const void* w, float s2, int n, int k, const void* x, int x_dtype, int ldx, int T, float* y, int ldy,
                   void* workspace, size_t workspace_bytes, void* stream);
size_t b200q_q8_gemv_workspace_bytes(int n, int k, int T);
int b200q_q8_gemv(const void* w, int n, int k, const void* x, int x_dtype, int ldx, int T, float* y, int ldy,
                  void* workspace, size_t workspace_bytes, void* stream);

/* ---------------------------------------------------------------------------------------------------------
 * Router, grouping, activation quantisation, combine.
 * --------------------------------------------------------------------------------------------------------- */

/* Replaces k_quant_rows (bolt_kernels.cu:347-363): int8 per 32, s = amax/127, q = rn(x*127/amax).
 * x [rows][ldx] (B200Q_F32 or B200Q_BF16) -> q [rows][ldq] int8, s [rows][lds] fp32.  k % 32 == 0. */
int b200q_quant_rows(const void* x, int x_dtype, int ldx, int8_t* q, int ldq, float* s, int lds, int rows, int k,
                     void* stream);

/* Replaces k_route (bolt_kernels.cu:1655-1712).  logits [T][ldl] (fp32 or bf16) -> ridx [T][topk] int,
 * rw [T][topk] fp32.  mode B200Q_ROUTE_SOFTMAX: softmax, top-k, renormalised (bias and scale unused);
 * B200Q_ROUTE_SIGMOID: route_k's form, bias [E] may be NULL.  Ties go to the lower expert.  E <= 512, topk <= 16. */
int b200q_route(const void* logits, int l_dtype, int ldl, const float* bias, int T, int E, int topk, int mode,
                float scale, int* ridx, float* rw, void* stream);

/* Replaces k_moe_group (bolt_kernels.cu:275-325): counting sort of the pairs by expert.
 * counts [E], offsets [E+1] (exclusive prefix), order [pairs]: the pairs of each expert in increasing order
 * (libbolt fills an expert's run with atomics; this order is deterministic).  pairs <= 4096, E <= 512. */
int b200q_moe_group(const int* ridx, int pairs, int E, int* counts, int* offsets, int* order, void* stream);

/* Replaces k_combine (bolt_kernels.cu:1714-1727), generalised from TOPN=9 and width 1024:
 * out[t][h] = sum_k rw[t][k] * mo[t*topk+k][h]  (+ shared[t][h] when shared is not NULL).
 * mo [T*topk][H] fp32, out [T][H] fp32 or bf16 (out_dtype).  H % 4 == 0. */
int b200q_combine(const float* mo, const float* rw, const float* shared, int T, int topk, int H, void* out,
                  int out_dtype, void* stream);

/* ---------------------------------------------------------------------------------------------------------
 * IQ2_XXS GEMVs on int8 activation rows (the routed-expert arithmetic of moe_mma_k / moe_coop_k,
 * bolt_kernels.cu:373-519, 542-667): per 32-weight chunk an exact int32 dot of the signed grid integers and the
 * int8 row, then acc += (d*(0.5+s4)*0.25 * s_row) * dot.
 * --------------------------------------------------------------------------------------------------------- */

/* Dense: y[t][n] = W[n] . x[t] for T rows.  Replaces mma_iq2 (bolt_mma.cu:1196-1203) and moe_coop_dense
 * (bolt_kernels.cu:881-887).  w packed rt32 [n][k]; xq [T][k] int8, xs [T][k/32]; y [T][ldy] fp32.
 * epi 0: store; epi 1: store relu(v)^2.  n % 32 == 0, k % 256 == 0, k <= 8192. */
int b200q_iq2_gemv(const void* w, int n, int k, const int8_t* xq, const float* xs, int T, float* y, int ldy,
                   int epi, void* stream);

/* Test hook for the bit-exactness contract: the int32 dot of every (row, 32-chunk, token), computed by the same
 * device code as the GEMVs.  dots [T][n][k/32] int32. */
int b200q_iq2_chunk_dots(const void* w, int n, int k, const int8_t* xq, int T, int32_t* dots, void* stream);

/* Routed experts, one launch over every (token, expert) pair.  Replace moe_up / moe_down
 * (bolt_kernels.cu:682-695), generalised from k=1024, n=1024 and TOPN=9.
 * slab: E experts, packed rt32, expert e at e*b200q_iq2_bytes(n, k).  counts/offsets/order from b200q_moe_group.
 * up:   act row of pair p is xq[p / topk]; out row p.  down: act row p; out row p.
 * y: epi 0 fp32 [pairs][ldy]; epi 1 relu^2 fp32.
 * b200q_moe_up_q8 writes relu(up)^2 quantised to int8 per 32 (aq [pairs][n], as [pairs][n/32]), the fused form of
 * moe_up + k_quant_rows (bolt_host.cu:709-712). */
int b200q_moe_up(const void* slab, int E, int n, int k, const int* counts, const int* offsets, const int* order,
                 int topk, const int8_t* xq, const float* xs, float* y, int ldy, int epi, void* stream);
int b200q_moe_up_q8(const void* slab, int E, int n, int k, const int* counts, const int* offsets, const int* order,
                    int topk, const int8_t* xq, const float* xs, int8_t* aq, float* as, void* stream);
int b200q_moe_down(const void* slab, int E, int n, int k, const int* counts, const int* offsets, const int* order,
                   const int8_t* aq, const float* as, float* y, int ldy, void* stream);

/* ---------------------------------------------------------------------------------------------------------
 * Prompt-length GEMMs on the tcgen05 tensor cores (kind::f16: fp16 operands, fp32 accumulation in TMEM).
 * --------------------------------------------------------------------------------------------------------- */

/* Grouping for prompt chunks, any number of pairs (moe_group_k's job at prompt sizes, bolt_kernels.cu:275-325, which
 * libbolt does in one CTA): counts [E], offsets [E+1], order [pairs] (an expert's pairs in arrival order),
 * fill_scratch [E] ints.  E <= 512. */
int b200q_moe_group_large(const int* ridx, int pairs, int E, int* counts, int* offsets, int* order, int* fill_scratch,
                          void* stream);

/* ---------------------------------------------------------------------------------------------------------
 * Prompt-length GEMMs on the tcgen05 tensor cores (kind::f16, fp32 accumulation): the weights are dequantised
 * inside the kernel to fp16 with their scale folded in and rounded once (libbolt's PQ8 / PIQ2 arithmetic,
 * bolt_mma.cu:234-254, 380-397, in fp16), the activations rounded to fp16 once.  A CTA computes 256 rows x 256
 * weight rows; the activations are first converted into an fp16 "rows image" in the workspace.
 * --------------------------------------------------------------------------------------------------------- */

/* One prompt MoE projection pair over the expert-sorted pairs (replaces moe_up_tile / moe_down_tile, moe_tile_k
 * bolt_kernels.cu:697-862, and the shared expert's moe_tile_dense, :881-893):
 *   act[p] = fp16(relu(W_up[e] . x[p / topk])^2),   mo[p][0..H) = W_down[e] . act[p]   (pair-indexed; fp32, or bf16
 *   rounded to nearest even when mo_dtype is B200Q_BF16, as the expert-parallel return exchange sends it)
 * for every pair p of expert e, given b200q_moe_group_large's counts / offsets / order of the pairs' experts.
 * up: slab of E experts [F][H], down: slab of E experts [H][F] (packed rt32); x [T][H] fp32 or bf16 (ldx = H).
 * act_rows: NULL, or [pairs][F] fp16 receiving act (inspection only; it costs one extra pass).
 * workspace >= b200q_moe_prompt_workspace_bytes(pairs, E, H, F) (about (pairs + 128 E) (H + F) 2 bytes), 256-byte
 * aligned.  H % 256 == 0, F % 256 == 0, E <= 512. */
size_t b200q_moe_prompt_workspace_bytes(int pairs, int E, int H, int F);
int b200q_moe_prompt(const void* up, const void* down, int E, int H, int F, const int* counts, const int* offsets,
                     const int* order, int topk, int pairs, const void* x, int x_dtype, void* mo, int mo_dtype,
                     void* act_rows, void* workspace, size_t workspace_bytes, void* stream);

/* Q8_0 prompt GEMM (replaces mma_q8 / mma_q8_multi at prompt row counts, mma_big_k bolt_mma.cu:611-696):
 * y[t][n] = sum_k fp16(q * d) x[t][k] for any T.  Weights in the "q8 tc" layout (b200q_q8_tc_pack: units of 32 rows x
 * 32 k, [32][32] int8 then [32] fp16 d, the checkpoint's byte count); fused q/k/v projections are one matrix of
 * their stacked rows.  workspace >= b200q_q8_gemm_workspace_bytes(T, k).  n % 32 == 0, k % 256 == 0. */
size_t b200q_q8_tc_bytes(int64_t n, int k);
int b200q_q8_tc_pack(const void* raw, void* packed, int64_t n, int k, void* stream);
size_t b200q_q8_gemm_workspace_bytes(int T, int k);
int b200q_q8_gemm(const void* w, int n, int k, const void* x, int x_dtype, int ldx, int T, float* y, int ldy,
                  void* workspace, size_t workspace_bytes, void* stream);

/* NVFP4 prompt GEMM on the block-scaled fp4 tensor cores (replaces quant_nv4_rows + mma_nv4_fp4, bolt_mma.cu:925-1059,
 * dispatched for T >= 256 at bolt_host.cu:634,644):
 *   y[t][n] = s2 * sum_k e2m1(x4[t][k]) e4m3(sx[t][k/16]) e2m1(q[n][k]) e4m3(sc[n][k/16])      (fp32, [T][ldy])
 * Weights: b200q_nv4_tc_pack turns the checkpoint's q [n][k/2] (low nibble first) and sc [n][k/16] e4m3 into the
 * tensor cores' tile image (tile_nv4w_k, bolt_mma.cu:892-923): b200q_nv4_tc_bytes(n, k) bytes, n rounded up to 256.
 * Rows: b200q_quant_nv4_rows quantises x [T][ldx] (fp32 or bf16) to NVFP4 exactly as quant_nv4_rows_k does (scale
 * e4m3_enc(amax / 6) per 16, values e2m1_enc(v / scale)) into b200q_nv4_rows_bytes(T, k) bytes (T rounded up to
 * 128).  k % 256 == 0; pointers 16-byte aligned. */
size_t b200q_nv4_tc_bytes(int64_t n, int k);
int b200q_nv4_tc_pack(const void* q, const void* sc, void* packed, int64_t n, int k, void* stream);
size_t b200q_nv4_rows_bytes(int T, int k);
int b200q_quant_nv4_rows(const void* x, int x_dtype, int ldx, int T, int k, void* rows, void* stream);
/* A launch with at most a quarter of the SMs' worth of 128 x 256 tiles cuts K into slices; their fp32 partial sums go to
 * `workspace` (>= b200q_nv4_gemm_workspace_bytes, 0 when no split is needed) and are added in slice order.  A NULL
 * or small workspace runs without the split. */
size_t b200q_nv4_gemm_workspace_bytes(int n, int k, int T);
int b200q_nv4_gemm(const void* w, int n, int k, float s2, const void* rows, int T, float* y, int ldy, void* workspace,
                   size_t workspace_bytes, void* stream);

/* ---------------------------------------------------------------------------------------------------------
 * One decode MoE layer, the sequence enqueue_block runs for a MoE block
 * (bolt_host.cu:665-720) fused into four launches: router + grouping + int8 rows of x; up with relu^2 and the
 * int8 rows of the result; down; weighted combine plus the shared expert.
 *   x [T][H] bf16, logits [T][E] bf16 (the gate GEMM's output), up slab [E] x [F][H], down slab [E] x [H][F]
 *   (packed rt32), shared_up [F][H] / shared_down [H][F] (NULL: none), out [T][H] fp32 or bf16.
 *   route: B200Q_ROUTE_SOFTMAX or B200Q_ROUTE_SIGMOID (bias, scale as b200q_route).
 *   T <= 64, E <= 512, topk <= 16, H and F multiples of 256, H, F <= 8192.
 * workspace: workspace_bytes >= b200q_moe_decode_workspace_bytes(T, H, F, E, topk), 256-byte aligned.
 * ridx_out / rw_out: optional copies of the routing ([T][topk]).
 * stage_events: NULL, or 5 cudaEvent_t recorded on the stream before the prologue and after each of the four
 * launches (router/grouping/quantisation, up, down, combine), for per-kernel timing; the events' record calls sit
 * between the launches, so leave it NULL outside of profiling. */
size_t b200q_moe_decode_workspace_bytes(int T, int H, int F, int E, int topk);
int b200q_moe_decode(const void* x, const void* logits, const void* up, const void* down, const void* shared_up,
                     const void* shared_down, int T, int H, int F, int E, int topk, int route, const float* bias,
                     float scale, void* out, int out_dtype, void* workspace, size_t workspace_bytes, int* ridx_out,
                     float* rw_out, void* const* stage_events, void* stream);

/* The routed experts of one rank of the expert-parallel decode layer over the rows it received (no counterpart in
 * libbolt, which is single-GPU; the operators are moe_up / moe_down of bolt_kernels.cu:682-695 with libbolt's grouping,
 * k_moe_group :275-344, fused as b200q_moe_decode fuses them): row r goes through local expert lidx[r] (up, relu^2,
 * int8 rows, down) into y[r]; an lidx outside 0 .. n_local - 1 marks a padding row, left unwritten.  Three launches:
 * grouping + slot schedule + int8 rows of the input, the up GEMV, the down GEMV.
 *   rows [R][ldr] fp32 or bf16, R <= 4096; lidx: R int32, lidx_stride ints apart (1: an array; b200q_ep_pack's send
 *   rows carry theirs after the row's values); up [n_local] x [F][H], down [n_local] x [H][F] packed rt32,
 *   n_local <= 511; y [R][ldy] fp32 or bf16 (y_dtype; bf16 rounded to nearest even).
 *   workspace >= b200q_moe_experts_workspace_bytes(R, H, F, n_local), 256-byte aligned. */
size_t b200q_moe_experts_workspace_bytes(int R, int H, int F, int n_local);
int b200q_moe_experts_decode(const void* rows, int rows_dtype, int ldr, int R, int H, int F, const int* lidx,
                             int lidx_stride, int n_local, const void* up, const void* down, void* y, int y_dtype,
                             int ldy, void* workspace, size_t workspace_bytes, void* stream);

/* The expert-parallel decode exchange in its fixed-capacity layout (no counterpart in libbolt), around
 * b200q_moe_experts_decode and one all-to-all each way:
 * b200q_ep_pack writes this rank's send buffer: pair p = (t, k) of expert e = ridx[p] goes to rank
 * d = dest[e * max_rep + t % nrep[e]] as local expert lidx[e * max_rep + t % nrep[e]], into send row d * cap + pos,
 * pos = its place among the pairs bound for d in pair order (pos < cap is the caller's guarantee: cap = T * topk).
 * A send row is ldsend elements of send_dtype: x[t]'s H values (converted, bf16 rounded to nearest even), then the
 * local index as an int32 at element H (2 elements of bf16, 1 of fp32; ldsend >= H + 16 bytes' worth); rows no pair
 * takes get the index `discard` (>= every rank's local expert count).  slot[p] = the pair's send row.
 *   x [T][H] fp32 or bf16; ridx [T][topk] int32; dest, lidx [E][max_rep], nrep [E] int32; world * cap send rows.
 * b200q_ep_combine: out[t] = sum over k in order of rw[t][k] * back[slot[t * topk + k]] (fma, combine_k's order)
 * (+ shared[t]); back rows ldb elements of back_dtype (the exchange's return buffer), out fp32 or bf16. */
int b200q_ep_pack(const void* x, int x_dtype, int T, int H, const int* ridx, int topk, const int* dest,
                  const int* lidx, const int* nrep, int max_rep, int world, int cap, int discard, void* send,
                  int send_dtype, int ldsend, int* slot, void* stream);
int b200q_ep_combine(const void* back, int back_dtype, int ldb, const int* slot, const float* rw, const float* shared,
                     int T, int topk, int H, void* out, int out_dtype, void* stream);

/* SMs the persistent prompt GEMMs (b200q_moe_prompt, b200q_q8_gemm) leave free on the current device, 0 .. 128 (0 at
 * load): a pipelined expert-parallel exchange sets it while its transfers run beside the GEMMs, so that the
 * collective's kernels find SMs (no counterpart in libbolt, which is single-GPU).  Host-side, per device. */
int b200q_set_sm_reserve(int sms);

/* The expert-parallel decode step with its exchange over NVLink peer memory (no counterpart in libbolt, which is
 * single-GPU; the layer is the MoE block of enqueue_block, bolt_host.cu:665-720).  Every rank holds one region of
 * b200q_ep_peer_region_bytes (allocated by b200q_peer_alloc, zeroed), exports it (b200q_peer_export), and maps every
 * other rank's (b200q_peer_open); `peers` is a DEVICE array of the world regions as mapped in this process (its own
 * at [rank], also passed as `region`).  Ranks must be on distinct GPUs of one box with peer access.
 * A step is four launches on `stream` (phases: bit 0 the first, bit 1 the second and third, bit 2 the fourth; 7 all):
 *   1. route x's tokens (logits [T][E], route_k's arithmetic), store each pair's token row into its owner's region as
 *      the int8-per-32 row the GEMVs read (b200q_quant_rows' bytes; owner d = dest[e * max_rep + t % nrep[e]], local
 *      expert lidx[...] there) and this rank's own rows for the shared expert, then publish the step in every owner's
 *      flags;
 *   2, 3. wait until every sender has published, then the local experts over the received rows
 *      (b200q_moe_experts_decode's two launches: up [n_local + 1] x [F][H], down [n_local + 1] x [H][F], packed rt32,
 *      the shared expert LAST), outputs in ret_dtype in this rank's region; the GEMV launch's last CTA publishes
 *      them in every sender's flags;
 *   4. wait for every owner, then out[t] = sum over k in order of rw[t][k] * (pair (t, k)'s output row, read from
 *      its owner) (fma), + the shared expert's row; out [T][H] fp32 or bf16.
 * With ret_dtype fp32 the result is b200q_moe_decode's to the bit (the same int8 rows, GEMVs and combine order).
 * discard >= every rank's n_local + 1.  T * topk <= 1024, world * T * topk + T <= 4096, world <= 64.
 * state: b200q_ep_peer_state_bytes, zeroed once (the step's epoch, error bits); workspace:
 * b200q_ep_peer_workspace_bytes, 256-byte aligned.  ridx_out / rw_out (optional) receive the routing.
 * Every wait is bounded (4 s): b200q_ep_peer_error returns the bits a step recorded (bit 0: senders did not arrive,
 * bit 1: owners did not arrive, bit 2: a routing table entry out of range); synchronous, clear != 0 resets them.
 * Once a bit is set, later waits give up after a few polls until it is cleared. */
size_t b200q_ep_peer_region_bytes(int world, int T, int H, int topk, int ret_dtype);
size_t b200q_ep_peer_state_bytes(int T, int topk);
size_t b200q_ep_peer_workspace_bytes(int world, int T, int H, int F, int topk, int n_local);
int b200q_peer_alloc(size_t bytes, void** ptr);
int b200q_peer_free(void* ptr);
size_t b200q_peer_handle_bytes(void);
int b200q_peer_export(void* ptr, void* handle);
int b200q_peer_open(const void* handle, void** ptr);
int b200q_peer_close(void* ptr);
int b200q_ep_peer_error(void* state, int clear);
int b200q_ep_peer_decode(const void* x, int x_dtype, const void* logits, int logits_dtype, int T, int H, int F, int E,
                         int topk, int route, const float* bias, float scale, const int* dest, const int* lidx,
                         const int* nrep, int max_rep, void* region, void* const* peers, int world, int rank,
                         int n_local, int discard, const void* up, const void* down, int ret_dtype, void* state,
                         void* workspace, size_t workspace_bytes, void* out, int out_dtype, int* ridx_out,
                         float* rw_out, int phases, void* stream);

/* The decode MoE layer without a caller-provided workspace, for callers that cannot allocate device memory (a host
 * whose allocator owns the GPU's memory, a plugin that receives only tensors, a loop that must not take cudaMalloc's
 * implicit synchronisation).  No counterpart in the reference: libbolt allocates its own scratch at bolt_open.
 * Arguments and results are those of b200q_moe_decode.  Scratch is a library-resident device array of
 * b200q_moe_decode_noalloc_max_bytes() bytes (3 MiB: enough for T <= 16, H <= 4096, F <= 2048, E <= 128,
 * topk <= 8), held by every GPU that loads the library until exit; larger shapes return B200Q_ENOSPACE.  The first
 * call on a device looks up the array's device address, so make it before any stream capture.  The address is kept
 * for the life of the process; after cudaDeviceReset the array may sit elsewhere, so a process that resets a device
 * must not call this entry point on it again.  All calls share the array: calls that overlap on the GPU race.  It
 * allocates nothing. */
size_t b200q_moe_decode_noalloc_max_bytes(void);
int b200q_moe_decode_noalloc(const void* x, const void* logits, const void* up, const void* down, const void* shared_up,
                             const void* shared_down, int T, int H, int F, int E, int topk, int route, const float* bias,
                             float scale, void* out, int out_dtype, int* ridx_out, float* rw_out, void* stream);

/* ---------------------------------------------------------------------------------------------------------
 * Synthetic inputs (BASELINE's generators), host and device producing the same bytes.
 * --------------------------------------------------------------------------------------------------------- */

/* IQ2_XXS ggml blocks [nblocks][66]: d fp16 ~ U[1e-3, 1e-2], grid indices U{0..255}, sign indices U{0..127},
 * sub-scales U{0..15}; block i depends on (seed, i) only. */
void b200q_synth_iq2_host(uint64_t seed, int64_t nblocks, void* out);

/* ---------------------------------------------------------------------------------------------------------
 * Checkpoint ingestion (replaces libbolt's Store / open_store / lookup and load_slab / load_nv4 / load_q8,
 * bolt_host.cu:61-345).  b200q_ckpt_open reads dir/model.safetensors.index.json ({"weight_map": {tensor: shard}})
 * or, without one, dir/model.safetensors; shards are memory-mapped on first use and their JSON headers checked (every
 * data offset inside the file, byte counts matching dtype and shape).  NULL when the directory holds neither or the
 * index does not parse.  A handle is used from one thread at a time or under the caller's lock (lookups lock
 * internally); b200q_ckpt_close unmaps.
 * b200q_ckpt_tensor: a tensor's host bytes inside the mapping (valid until close), shape (up to 8 dims), dtype
 * (safetensors' name, up to 15 characters); EINVAL if absent or malformed.
 * The packers copy raw checkpoint bytes into `staging` (device, 16-byte aligned, >= b200q_ckpt_staging_bytes: fmt 0
 * one expert's IQ2_XXS blocks of n rows, 1 NVFP4, 2 Q8_0) and pack from there on `stream` into this library's
 * layouts, exactly as b200q_iq2_pack / b200q_nv4_pack / b200q_q8_pack of the same bytes:
 *   _iq2_slab  names[e] = expert e's [rows][k/256][66] blocks -> packed expert e at e * b200q_iq2_bytes(rows, k)
 *              (load_slab);
 *   _nv4       prefix.weight [n][k/2], prefix.weight_scale [n][k/16] e4m3, prefix.weight_scale_2 (fp32) -> the t16
 *              layout, *s2 = the tensor scale (load_nv4);
 *   _q8        name [n][k/32][34] -> the t16 layout (load_q8).
 * Every name and byte count is checked before the first copy (EINVAL), the staging size too (ENOSPACE).  The
 * copies read pageable host memory, so each returns once its bytes are staged.
 * --------------------------------------------------------------------------------------------------------- */
typedef struct b200q_ckpt b200q_ckpt;
b200q_ckpt* b200q_ckpt_open(const char* dir);
void b200q_ckpt_close(b200q_ckpt* c);
int64_t b200q_ckpt_count(b200q_ckpt* c);
int b200q_ckpt_tensor(b200q_ckpt* c, const char* name, const void** data, size_t* bytes, int64_t* shape, int* ndim,
                      char* dtype);
size_t b200q_ckpt_staging_bytes(int fmt, int n, int k);
int b200q_ckpt_pack_iq2_slab(b200q_ckpt* c, const char* const* names, int experts, int rows, int k, void* packed,
                             void* staging, size_t staging_bytes, void* stream);
int b200q_ckpt_pack_nv4(b200q_ckpt* c, const char* prefix, int n, int k, void* packed, float* s2, void* staging,
                        size_t staging_bytes, void* stream);
int b200q_ckpt_pack_q8(b200q_ckpt* c, const char* name, int n, int k, void* packed, void* staging,
                       size_t staging_bytes, void* stream);
int b200q_synth_iq2(uint64_t seed, int64_t nblocks, void* out, void* stream);

#ifdef __cplusplus
}
#endif
#endif
