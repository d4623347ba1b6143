/*
 * oracle.c -- TEST INFRASTRUCTURE ONLY.
 *
 * A scalar CPU restatement of the arithmetic of libbolt's quantized-GEMM hot path (the reference engine,
 * engine/bolt_kernels.cu and engine/bolt_mma.cu).  It is the checker for the B200 kernels: only tests/,
 * __graft_entry__.smoke() and bench.py's CPU-baseline leg load it.  Nothing in the product path links or
 * calls it.
 *
 * The ggml IQ2_XXS tables are not re-typed here: the build includes the reference's own table file by path
 * (oracle/build_oracle.py passes -DB200Q_IQ2_TABLES=<path of engine/iq2_tables.inc>).
 *
 * Every function names the reference lines it restates.  Float arithmetic is written in the order the
 * reference kernels evaluate it.  The build uses -ffp-contract=off and spells out the fused multiply-adds that
 * nvcc forms from `acc += a * b` (fmaf), so scalar results reproduce the kernels' roundings wherever the
 * kernels themselves are order-deterministic.
 *
 * Layouts at this boundary are the checkpoint's own (the bytes libbolt's loaders read):
 *   IQ2_XXS  [rows][K/256][66]: fp16 d, then 8 chunks of 8 bytes (4 grid-index bytes; a u32 of four 7-bit
 *            sign indices and a 4-bit sub-scale in bits 28-31)            (bolt_host.cu:266-285)
 *   Q8_0     [rows][K/32][34]: fp16 d, then 32 int8                       (bolt_host.cu:198-217)
 *   NVFP4    q [rows][K/2] (low nibble first), sc [rows][K/16] e4m3, one fp32 tensor scale s2
 *                                                                          (bolt_common.h:30-31)
 */
#include <math.h>
#include <stdint.h>
#include <stdlib.h>
#include <string.h>

#define GGML_TABLE_BEGIN(type, name, size) static const type name[size] = {
#define GGML_TABLE_END() };
#include B200Q_IQ2_TABLES

#define EXPORT __attribute__((visibility("default")))

/* ------------------------------------------------------------------------------------------------------ */
/* scalar formats                                                                                          */
/* ------------------------------------------------------------------------------------------------------ */

static float u2f(uint32_t u) { float f; memcpy(&f, &u, 4); return f; }
static uint32_t f2u(float f) { uint32_t u; memcpy(&u, &f, 4); return u; }

/* IEEE binary16 -> binary32, exact (what __half2float does). */
EXPORT float or_h2f(uint16_t h) {
    const uint32_t s = (uint32_t)(h >> 15) << 31, e = (h >> 10) & 31, m = h & 1023;
    if (e == 0) {
        const float v = ldexpf((float)m, -24);
        return (h >> 15) ? -v : v;
    }
    if (e == 31) return u2f(s | 0x7f800000u | (m << 13));
    return u2f(s | ((e + 112) << 23) | (m << 13));
}

/* binary32 -> binary16, round to nearest even (what __float2half_rn does), saturating to inf. */
EXPORT uint16_t or_f2h(float f) {
    const uint32_t s = (f2u(f) >> 16) & 0x8000u;
    const float a = fabsf(f);
    int e;
    if (a != a) return (uint16_t)(s | 0x7e00u);
    if (a < ldexpf(1.f, -14)) return (uint16_t)(s | (uint32_t)nearbyintf(a * 16777216.f));
    frexpf(a, &e);                                   /* a = m 2^e, m in [0.5, 1) */
    {
        uint32_t mant = (uint32_t)nearbyintf(ldexpf(a, 11 - e));   /* 11 significant bits, in [1024, 2048] */
        int ee = e - 1;
        if (mant == 2048) { mant = 1024; ee++; }
        if (ee > 15) return (uint16_t)(s | 0x7c00u);
        return (uint16_t)(s | ((uint32_t)(ee + 15) << 10) | (mant - 1024));
    }
}

EXPORT float or_bf2f(uint16_t b) { return u2f((uint32_t)b << 16); }

/* binary32 -> bfloat16, round to nearest even (what __float2bfloat16_rn does for finite values). */
EXPORT uint16_t or_f2bf(float f) {
    const uint32_t u = f2u(f);
    if ((u & 0x7fffffffu) > 0x7f800000u) return (uint16_t)((u >> 16) | 0x40);
    return (uint16_t)((u + 0x7fffu + ((u >> 16) & 1)) >> 16);
}

/* e4m3 (fn: bias 7, no infinities, 0x7f / 0xff are NaN) -> float, sign included: the __nv_fp8_e4m3 conversion
 * FmtNV4::e4m3 uses (bolt_kernels.cu:66-70).  On the positive codes it equals e4m3_dec (bolt_mma.cu:882-885). */
EXPORT float or_e4m3_dec(uint32_t c) {
    const int ef = (int)((c >> 3) & 15), m = (int)(c & 7);
    float v;
    if ((c & 0x7f) == 0x7f) return NAN;
    v = ef == 0 ? (float)m * 0.001953125f : ldexpf(1.f + (float)m * 0.125f, ef - 7);
    return (c & 0x80) ? -v : v;
}

/* e4m3_enc (bolt_mma.cu:868-881): a positive scale to e4m3, nearest, saturating at 448. */
EXPORT uint32_t or_e4m3_enc(float v) {
    int e, mant;
    float m;
    if (!(v > 0.f)) return 0u;
    if (v >= 448.f) return 0x7Eu;
    m = frexpf(v, &e);
    e -= 1;
    if (e < -6) {
        const int q = (int)rintf(v * 512.f);
        return q >= 8 ? 0x08u : (uint32_t)q;
    }
    mant = (int)rintf((2.f * m - 1.f) * 8.f);
    if (mant == 8) { mant = 0; e++; if (e > 8) return 0x7Eu; }
    return ((uint32_t)(e + 7) << 3) | (uint32_t)mant;
}

/* e2m1_enc (bolt_mma.cu:886-890): nearest of 0, .5, 1, 1.5, 2, 3, 4, 6, sign in bit 3. */
EXPORT uint32_t or_e2m1_enc(float v) {
    const float u = fabsf(v);
    const uint32_t c = u < 0.25f ? 0u : u < 0.75f ? 1u : u < 1.25f ? 2u : u < 1.75f ? 3u : u < 2.5f ? 4u : u < 3.5f ? 5u : u < 5.f ? 6u : 7u;
    return c | (v < 0.f ? 8u : 0u);
}

/* e2m1 nibble -> float (FmtNV4::deq, bolt_kernels.cu:74-82). */
EXPORT float or_e2m1_dec(uint32_t nib) {
    static const float mag[8] = {0.f, 0.5f, 1.f, 1.5f, 2.f, 3.f, 4.f, 6.f};
    const float v = mag[nib & 7];
    return (nib & 8) ? -v : v;
}

/* ------------------------------------------------------------------------------------------------------ */
/* IQ2_XXS                                                                                                 */
/* ------------------------------------------------------------------------------------------------------ */

/* The ggml tables exactly as the reference carries them (engine/iq2_tables.inc:1-117). */
EXPORT void or_iq2_tables(uint64_t* grid_out, uint8_t* signs_out, uint64_t* signs64_out, uint8_t* mask_out) {
    if (grid_out) memcpy(grid_out, iq2xxs_grid, sizeof(iq2xxs_grid));
    if (signs_out) memcpy(signs_out, ksigns_iq2xs, sizeof(ksigns_iq2xs));
    if (signs64_out) memcpy(signs64_out, ksigns64, sizeof(ksigns64));
    if (mask_out) memcpy(mask_out, kmask_iq2xs, sizeof(kmask_iq2xs));
}

static uint32_t rd32(const uint8_t* p) { return (uint32_t)p[0] | (uint32_t)p[1] << 8 | (uint32_t)p[2] << 16 | (uint32_t)p[3] << 24; }
static uint16_t rd16(const uint8_t* p) { return (uint16_t)(p[0] | p[1] << 8); }

/* The 8 signed grid integers of group `sub` of a chunk: grid byte times the sign from ksigns (bit j of
 * si | parity << 7), the int8 form of moe_mma_k (bolt_kernels.cu:457-465: q = grid ^ mask - mask). */
static void iq2_group_ints(uint32_t qx, uint32_t qy, int sub, int* w) {
    const uint64_t g = iq2xxs_grid[(qx >> (8 * sub)) & 255];
    const uint32_t sg = ksigns_iq2xs[(qy >> (7 * sub)) & 127];
    int j;
    for (j = 0; j < 8; j++) {
        const int mag = (int)((g >> (8 * j)) & 255);
        w[j] = ((sg >> j) & 1) ? -mag : mag;
    }
}

/* The chunk scale db = d (0.5 + s4) 0.25 in fp32, left to right (FmtIQ2::load bolt_kernels.cu:117;
 * moe_mma_k :453-454; moe_coop_k :620-621). */
static float iq2_chunk_scale(float d, uint32_t qy) { return d * (0.5f + (float)(qy >> 28)) * 0.25f; }

/* fp32 dequantisation of IQ2_XXS rows (FmtIQ2::load/deq, bolt_kernels.cu:110-132):
 * w = float(grid byte) with the sign bit flipped, times db. */
EXPORT void or_iq2_dequant(const uint8_t* blocks, int64_t rows, int K, float* out) {
    const int nb = K / 256;
    int64_t r;
#pragma omp parallel for schedule(static)
    for (r = 0; r < rows; r++) {
        int b, c, sub, j;
        for (b = 0; b < nb; b++) {
            const uint8_t* blk = blocks + ((size_t)r * nb + b) * 66;
            const float d = or_h2f(rd16(blk));
            for (c = 0; c < 8; c++) {
                const uint32_t qx = rd32(blk + 2 + 8 * c), qy = rd32(blk + 6 + 8 * c);
                const float db = iq2_chunk_scale(d, qy);
                for (sub = 0; sub < 4; sub++) {
                    int w[8];
                    iq2_group_ints(qx, qy, sub, w);
                    for (j = 0; j < 8; j++) out[(size_t)r * K + b * 256 + c * 32 + sub * 8 + j] = (float)w[j] * db;
                }
            }
        }
    }
}

/* "exact" mode: y[t][n] = sum_k dequant(W)[n][k] x[t][k], fp32 dequantisation, fp64 accumulation.  The
 * truth the fp32 GEMVs approximate (gemv_iq2 / gemv_body, bolt_kernels.cu:139-226,237-240). */
EXPORT void or_iq2_gemm_exact(const uint8_t* blocks, int N, int K, const float* x, int T, float* y, int epi) {
    int n;
#pragma omp parallel for schedule(dynamic, 16)
    for (n = 0; n < N; n++) {
        float* w = (float*)malloc(sizeof(float) * (size_t)K);
        int t, k;
        or_iq2_dequant(blocks + (size_t)n * (K / 256) * 66, 1, K, w);
        for (t = 0; t < T; t++) {
            double acc = 0.0;
            float v;
            for (k = 0; k < K; k++) acc += (double)w[k] * (double)x[(size_t)t * K + k];
            v = (float)acc;
            if (epi == 1) v = v > 0.f ? v * v : 0.f;
            y[(size_t)t * N + n] = v;
        }
        free(w);
    }
}

/* quant_rows_k (bolt_kernels.cu:347-360): int8 per 32, s = amax / 127, q = rn(v * (127 / amax)) (round half to
 * even, __float2int_rn).  x [rows][K] fp32 -> q [rows][K] int8, s [rows][K/32] fp32. */
EXPORT void or_quant_rows(const float* x, int64_t rows, int K, int8_t* q, float* s) {
    int64_t r;
#pragma omp parallel for schedule(static)
    for (r = 0; r < rows; r++) {
        int b, j;
        for (b = 0; b < K / 32; b++) {
            const float* v = x + (size_t)r * K + b * 32;
            float am = 0.f, inv;
            for (j = 0; j < 32; j++) am = fmaxf(am, fabsf(v[j]));
            inv = am > 0.f ? 127.f / am : 0.f;
            for (j = 0; j < 32; j++) q[(size_t)r * K + b * 32 + j] = (int8_t)(int)nearbyintf(v[j] * inv);
            s[(size_t)r * (K / 32) + b] = am / 127.f;
        }
    }
}

/* The int32 dot of one 32-weight chunk with one int8 activation row segment: the integer the m16n8k32 s8 MMA
 * produces per chunk in moe_mma_k / moe_coop_k (bolt_kernels.cu:466-478, 630-636).  dots [T][N][K/32]. */
EXPORT void or_iq2_chunk_dots(const uint8_t* blocks, int N, int K, const int8_t* xq, int T, int32_t* dots) {
    const int nb = K / 256, nc = K / 32;
    int n;
#pragma omp parallel for schedule(static)
    for (n = 0; n < N; n++) {
        int b, c, sub, j, t;
        for (b = 0; b < nb; b++) {
            const uint8_t* blk = blocks + ((size_t)n * nb + b) * 66;
            for (c = 0; c < 8; c++) {
                const uint32_t qx = rd32(blk + 2 + 8 * c), qy = rd32(blk + 6 + 8 * c);
                int w[32];
                for (sub = 0; sub < 4; sub++) iq2_group_ints(qx, qy, sub, w + 8 * sub);
                for (t = 0; t < T; t++) {
                    const int8_t* xr = xq + (size_t)t * K + b * 256 + c * 32;
                    int32_t acc = 0;
                    for (j = 0; j < 32; j++) acc += w[j] * (int32_t)xr[j];
                    dots[((size_t)t * N + n) * nc + b * 8 + c] = acc;
                }
            }
        }
    }
}

/* "int8" mode, the routed-expert arithmetic of moe_mma_k / moe_coop_k (bolt_kernels.cu:445-483, 599-652):
 * per chunk c in order, acc += (dA * s) * (float)dot with dA = d (0.5 + s4) 0.25 and s the activation row's
 * scale of chunk c; epi 1 stores relu(acc)^2 (:493).  xq [T][K] int8, xs [T][K/32]. */
EXPORT void or_iq2_gemm_i8(const uint8_t* blocks, int N, int K, const int8_t* xq, const float* xs, int T, float* y, int epi) {
    const int nb = K / 256, nc = K / 32;
    int n;
#pragma omp parallel for schedule(static)
    for (n = 0; n < N; n++) {
        int t, b, c, sub, j;
        for (t = 0; t < T; t++) {
            float acc = 0.f;
            for (b = 0; b < nb; b++) {
                const uint8_t* blk = blocks + ((size_t)n * nb + b) * 66;
                const float d = or_h2f(rd16(blk));
                for (c = 0; c < 8; c++) {
                    const uint32_t qx = rd32(blk + 2 + 8 * c), qy = rd32(blk + 6 + 8 * c);
                    const float dA = iq2_chunk_scale(d, qy);
                    const int8_t* xr = xq + (size_t)t * K + b * 256 + c * 32;
                    int w[32];
                    int32_t dot = 0;
                    for (sub = 0; sub < 4; sub++) iq2_group_ints(qx, qy, sub, w + 8 * sub);
                    for (j = 0; j < 32; j++) dot += w[j] * (int32_t)xr[j];
                    acc = fmaf(dA * xs[(size_t)t * nc + b * 8 + c], (float)dot, acc);
                }
            }
            if (epi == 1) acc = acc > 0.f ? acc * acc : 0.f;
            y[(size_t)t * N + n] = acc;
        }
    }
}

/* ------------------------------------------------------------------------------------------------------ */
/* router, grouping, combine                                                                               */
/* ------------------------------------------------------------------------------------------------------ */

/* Pick the top `topk` of score[0..E) (ties to the lower index), as route_k's warp argmax does
 * (bolt_kernels.cu:1676-1692). */
static void topk_desc(const double* score, int E, int topk, int* out) {
    unsigned char taken[1024];
    int k, i;
    memset(taken, 0, (size_t)E);
    for (k = 0; k < topk; k++) {
        int bi = -1;
        for (i = 0; i < E; i++)
            if (!taken[i] && (bi < 0 || score[i] > score[bi])) bi = i;
        taken[bi] = 1;
        out[k] = bi;
    }
}

/* The BASELINE router: softmax over E logits, top-k, the k probabilities renormalised to sum 1.  Written in
 * fp64 (the kernel computes it in fp32).  The reference router is route_k's sigmoid form (below); the softmax
 * form is the parameterisation BASELINE config 2 asks for.  logits [T][E] fp32 -> ridx/rw [T][topk]. */
EXPORT void or_route_softmax(const float* logits, int T, int E, int topk, int* ridx, float* rw) {
    int t, i, k;
    for (t = 0; t < T; t++) {
        double z[1024], mx = -1e300, den = 0.0;
        int pick[64];
        for (i = 0; i < E; i++) { z[i] = logits[(size_t)t * E + i]; if (z[i] > mx) mx = z[i]; }
        topk_desc(z, E, topk, pick);
        for (k = 0; k < topk; k++) den += exp(z[pick[k]] - mx);
        for (k = 0; k < topk; k++) {
            ridx[t * topk + k] = pick[k];
            rw[t * topk + k] = (float)(exp(z[pick[k]] - mx) / den);
        }
    }
}

/* route_k (bolt_kernels.cu:1655-1712): sig = sigmoid(z), pick the top `topk` of sig + bias (ties to the lower
 * index), weights = sig / (1e-20 + sum of the picked sig) * scale.  Written in fp64 for sig (the kernel uses
 * __expf); the sum is taken in pick order like the kernel's. */
EXPORT void or_route_sigmoid(const float* logits, int ldl, const float* bias, int T, int E, int topk, float scale,
                             int* ridx, float* rw) {
    int t, i, k;
    for (t = 0; t < T; t++) {
        double sel[1024];
        float sig[1024], sum = 1e-20f;
        int pick[64];
        for (i = 0; i < E; i++) {
            sig[i] = (float)(1.0 / (1.0 + exp(-(double)logits[(size_t)t * ldl + i])));
            sel[i] = (double)(sig[i] + (bias ? bias[i] : 0.f));
        }
        topk_desc(sel, E, topk, pick);
        for (k = 0; k < topk; k++) sum += sig[pick[k]];
        for (k = 0; k < topk; k++) {
            ridx[t * topk + k] = pick[k];
            rw[t * topk + k] = sig[pick[k]] / sum * scale;
        }
    }
}

/* moe_group_k's semantics (bolt_kernels.cu:275-325): a counting sort of pairs by expert.  counts[E],
 * offsets[E+1] (exclusive prefix), order[pairs] = the pairs of expert 0, then expert 1, ...  The reference
 * fills each expert's run with atomics (its order inside a run is unspecified); this one keeps pair order. */
EXPORT void or_group(const int* ridx, int pairs, int E, int* counts, int* offsets, int* order) {
    int p, e;
    int* fill = (int*)calloc((size_t)E, sizeof(int));
    memset(counts, 0, sizeof(int) * (size_t)E);
    for (p = 0; p < pairs; p++) counts[ridx[p]]++;
    offsets[0] = 0;
    for (e = 0; e < E; e++) offsets[e + 1] = offsets[e] + counts[e];
    for (p = 0; p < pairs; p++) { e = ridx[p]; order[offsets[e] + fill[e]++] = p; }
    free(fill);
}

/* combine_k (bolt_kernels.cu:1714-1727): out[t][h] = sum_k rw[t][k] * mo[t*topk + k][h], k in order. */
EXPORT void or_combine(const float* mo, const float* rw, int T, int topk, int H, float* out) {
    int t, k, h;
    for (t = 0; t < T; t++)
        for (h = 0; h < H; h++) {
            float acc = 0.f;
            for (k = 0; k < topk; k++) acc = fmaf(rw[t * topk + k], mo[((size_t)t * topk + k) * H + h], acc);
            out[(size_t)t * H + h] = acc;
        }
}

/* One decode MoE layer as BASELINE config 2 defines it, in the order enqueue_block runs the stages
 * (bolt_host.cu:665-720): router; int8 rows of x (quant_rows); per pair the expert's up rows with relu^2
 * (moe_up); int8 rows of those (quant_rows); the expert's down rows (moe_down); the weighted combine
 * (combine_k); plus the shared expert on every token.
 *   x [T][H] bf16 bits, logits [T][E] bf16 bits, up slab [E][F][H/256][66], down slab [E][H][F/256][66],
 *   shared up [F][H/256][66] / down [H][F/256][66] (NULL: no shared expert).
 *   mode 0: the int8-per-32 arithmetic of the routed-expert kernels; mode 1: "exact" (no activation
 *   quantisation, fp32 dequantisation, fp64 dot products).
 *   route 0: softmax top-k renormalised; route 1: sigmoid + bias top-k times scale (route_k).
 *   Outputs: out [T][H] fp32; ridx/rw [T][topk] when not NULL. */
EXPORT void or_moe_layer(const uint16_t* x_bf, const uint16_t* logits_bf, const uint8_t* up, const uint8_t* down,
                         const uint8_t* sh_up, const uint8_t* sh_down, int T, int H, int F, int E, int topk,
                         int route, const float* bias, float scale, int mode, float* out, int* ridx_out,
                         float* rw_out) {
    const size_t up_bytes = (size_t)F * (H / 256) * 66, down_bytes = (size_t)H * (F / 256) * 66;
    const int pairs = T * topk;
    float* x = (float*)malloc(sizeof(float) * (size_t)T * H);
    float* lg = (float*)malloc(sizeof(float) * (size_t)T * E);
    int* ridx = (int*)malloc(sizeof(int) * (size_t)pairs);
    float* rw = (float*)malloc(sizeof(float) * (size_t)pairs);
    float* act = (float*)malloc(sizeof(float) * (size_t)(pairs > T ? pairs : T) * F);
    float* mo = (float*)malloc(sizeof(float) * (size_t)pairs * H);
    float* sh = (float*)malloc(sizeof(float) * (size_t)T * H);
    int8_t* xq = (int8_t*)malloc((size_t)T * H);
    float* xs = (float*)malloc(sizeof(float) * (size_t)T * (H / 32));
    int8_t* aq = (int8_t*)malloc((size_t)(pairs > T ? pairs : T) * F);
    float* as = (float*)malloc(sizeof(float) * (size_t)(pairs > T ? pairs : T) * (F / 32));
    int i, p, h, t;
    for (i = 0; i < T * H; i++) x[i] = or_bf2f(x_bf[i]);
    for (i = 0; i < T * E; i++) lg[i] = or_bf2f(logits_bf[i]);
    if (route == 0) or_route_softmax(lg, T, E, topk, ridx, rw);
    else or_route_sigmoid(lg, E, bias, T, E, topk, scale, ridx, rw);
    if (mode == 0) or_quant_rows(x, T, H, xq, xs);
    for (p = 0; p < pairs; p++) {
        const int e = ridx[p], tok = p / topk;
        if (mode == 0) or_iq2_gemm_i8(up + (size_t)e * up_bytes, F, H, xq + (size_t)tok * H, xs + (size_t)tok * (H / 32), 1, act + (size_t)p * F, 1);
        else or_iq2_gemm_exact(up + (size_t)e * up_bytes, F, H, x + (size_t)tok * H, 1, act + (size_t)p * F, 1);
    }
    if (mode == 0) or_quant_rows(act, pairs, F, aq, as);
    for (p = 0; p < pairs; p++) {
        const int e = ridx[p];
        if (mode == 0) or_iq2_gemm_i8(down + (size_t)e * down_bytes, H, F, aq + (size_t)p * F, as + (size_t)p * (F / 32), 1, mo + (size_t)p * H, 0);
        else or_iq2_gemm_exact(down + (size_t)e * down_bytes, H, F, act + (size_t)p * F, 1, mo + (size_t)p * H, 0);
    }
    or_combine(mo, rw, T, topk, H, out);
    if (sh_up && sh_down) {
        if (mode == 0) {
            or_iq2_gemm_i8(sh_up, F, H, xq, xs, T, act, 1);
            or_quant_rows(act, T, F, aq, as);
            or_iq2_gemm_i8(sh_down, H, F, aq, as, T, sh, 0);
        } else {
            or_iq2_gemm_exact(sh_up, F, H, x, T, act, 1);
            or_iq2_gemm_exact(sh_down, H, F, act, T, sh, 0);
        }
        for (t = 0; t < T; t++)
            for (h = 0; h < H; h++) out[(size_t)t * H + h] += sh[(size_t)t * H + h];
    }
    if (ridx_out) memcpy(ridx_out, ridx, sizeof(int) * (size_t)pairs);
    if (rw_out) memcpy(rw_out, rw, sizeof(float) * (size_t)pairs);
    free(x); free(lg); free(ridx); free(rw); free(act); free(mo); free(sh); free(xq); free(xs); free(aq); free(as);
}

/* ------------------------------------------------------------------------------------------------------ */
/* NVFP4                                                                                                   */
/* ------------------------------------------------------------------------------------------------------ */

/* "exact" NVFP4 GEMM: y[t][n] = s2 * sum_k e2m1(q[n][k]) e4m3(sc[n][k/16]) x[t][k], fp64 accumulation
 * (FmtNV4::deq bolt_kernels.cu:71-83 gives the weight; gemv_nv4 :232-234 the product).  epi as above. */
EXPORT void or_nv4_gemm_exact(const uint8_t* q, const uint8_t* sc, float s2, int N, int K, const float* x, int T,
                              float* y) {
    int n;
#pragma omp parallel for schedule(static)
    for (n = 0; n < N; n++) {
        float* w = (float*)malloc(sizeof(float) * (size_t)K);
        int k, t;
        for (k = 0; k < K; k++) {
            const uint8_t byte = q[(size_t)n * (K / 2) + k / 2];
            const uint32_t nib = (k & 1) ? (byte >> 4) : (byte & 15);
            w[k] = or_e2m1_dec(nib) * or_e4m3_dec(sc[(size_t)n * (K / 16) + k / 16]);
        }
        for (t = 0; t < T; t++) {
            double acc = 0.0;
            for (k = 0; k < K; k++) acc += (double)w[k] * (double)x[(size_t)t * K + k];
            y[(size_t)t * N + n] = (float)(acc * (double)s2);
        }
        free(w);
    }
}

/* quant_nv4_rows_k (bolt_mma.cu:925-951): per block of 16, scale code = e4m3_enc(amax / 6), values
 * e2m1_enc(v * (1 / e4m3_dec(code))).  Output row-major: q4 [T][K/2] (element 2j low nibble), sf [T][K/16]
 * (the reference stores sf step-major for its own MMA; the values are the same). */
EXPORT void or_quant_nv4_rows(const float* x, int T, int K, uint8_t* q4, uint8_t* sf) {
    int r;
#pragma omp parallel for schedule(static)
    for (r = 0; r < T; r++) {
        int blk, j;
        for (blk = 0; blk < K / 16; blk++) {
            const float* v = x + (size_t)r * K + blk * 16;
            float amax = 0.f, sq, inv;
            uint32_t code;
            for (j = 0; j < 16; j++) amax = fmaxf(amax, fabsf(v[j]));
            code = or_e4m3_enc(amax * (1.f / 6.f));
            sq = or_e4m3_dec(code);
            inv = sq > 0.f ? 1.f / sq : 0.f;
            for (j = 0; j < 8; j++)
                q4[(size_t)r * (K / 2) + blk * 8 + j] = (uint8_t)(or_e2m1_enc(v[2 * j] * inv) | (or_e2m1_enc(v[2 * j + 1] * inv) << 4));
            sf[(size_t)r * (K / 16) + blk] = (uint8_t)code;
        }
    }
}

/* NVFP4 x NVFP4 (the prefill arithmetic of mma_nv4_fp4_k, bolt_mma.cu:961-1059): both operands quantised,
 * y = s2 * sum over blocks of e4m3(sa) e4m3(sb) sum_j e2m1(a) e2m1(b); the products are exact, the sum is taken
 * in fp64.  Weights q/sc as above; rows q4 [T][K/2], sf [T][K/16]. */
EXPORT void or_nv4_gemm_q4(const uint8_t* q, const uint8_t* sc, float s2, int N, int K, const uint8_t* q4,
                           const uint8_t* sf, int T, float* y) {
    int n;
#pragma omp parallel for schedule(static)
    for (n = 0; n < N; n++) {
        int t, blk, j;
        for (t = 0; t < T; t++) {
            double acc = 0.0;
            for (blk = 0; blk < K / 16; blk++) {
                double part = 0.0;
                for (j = 0; j < 16; j++) {
                    const int k = blk * 16 + j;
                    const uint8_t wb = q[(size_t)n * (K / 2) + k / 2], xb = q4[(size_t)t * (K / 2) + k / 2];
                    part += (double)or_e2m1_dec((k & 1) ? wb >> 4 : wb & 15) * (double)or_e2m1_dec((k & 1) ? xb >> 4 : xb & 15);
                }
                acc += part * (double)or_e4m3_dec(sc[(size_t)n * (K / 16) + blk]) * (double)or_e4m3_dec(sf[(size_t)t * (K / 16) + blk]);
            }
            y[(size_t)t * N + n] = (float)(acc * (double)s2);
        }
    }
}

/* ------------------------------------------------------------------------------------------------------ */
/* Q8_0                                                                                                    */
/* ------------------------------------------------------------------------------------------------------ */

/* "exact" Q8_0 GEMM (FmtQ8::deq, bolt_kernels.cu:41-52: w = int8 * d): fp64 accumulation of the exact
 * products.  blocks [N][K/32][34]. */
EXPORT void or_q8_gemm_exact(const uint8_t* blocks, int N, int K, const float* x, int T, float* y) {
    int n;
#pragma omp parallel for schedule(static)
    for (n = 0; n < N; n++) {
        float* w = (float*)malloc(sizeof(float) * (size_t)K);
        int b, j, t, k;
        for (b = 0; b < K / 32; b++) {
            const uint8_t* blk = blocks + ((size_t)n * (K / 32) + b) * 34;
            const float d = or_h2f(rd16(blk));
            for (j = 0; j < 32; j++) w[b * 32 + j] = (float)(int8_t)blk[2 + j] * d;
        }
        for (t = 0; t < T; t++) {
            double acc = 0.0;
            for (k = 0; k < K; k++) acc += (double)w[k] * (double)x[(size_t)t * K + k];
            y[(size_t)t * N + n] = (float)acc;
        }
        free(w);
    }
}

/* Q8_0 with the scale folded into fp16 (PQ8, bolt_mma.cu:234-254: a = fp16(int8 * d), one rounding of
 * 2^-11, then an fp32-accumulated product with the fp32 activation).  Accumulated in fp64 here. */
EXPORT void or_q8_gemm_f16fold(const uint8_t* blocks, int N, int K, const float* x, int T, float* y) {
    int n;
#pragma omp parallel for schedule(static)
    for (n = 0; n < N; n++) {
        float* w = (float*)malloc(sizeof(float) * (size_t)K);
        int b, j, t, k;
        for (b = 0; b < K / 32; b++) {
            const uint8_t* blk = blocks + ((size_t)n * (K / 32) + b) * 34;
            const float d = or_h2f(rd16(blk));
            for (j = 0; j < 32; j++) w[b * 32 + j] = or_h2f(or_f2h((float)(int8_t)blk[2 + j] * d));
        }
        for (t = 0; t < T; t++) {
            double acc = 0.0;
            for (k = 0; k < K; k++) acc += (double)w[k] * (double)x[(size_t)t * K + k];
            y[(size_t)t * N + n] = (float)acc;
        }
        free(w);
    }
}

/* IQ2_XXS with the chunk scale folded into fp16 weights (the shared-expert form PIQ2, bolt_mma.cu:380-397,
 * which folds into bf16; fp16 here): w = fp16(db * signed grid), fp64 accumulation.  epi as above. */
EXPORT void or_iq2_gemm_f16fold(const uint8_t* blocks, int N, int K, const float* x, int T, float* y, int epi) {
    int n;
#pragma omp parallel for schedule(dynamic, 16)
    for (n = 0; n < N; n++) {
        float* w = (float*)malloc(sizeof(float) * (size_t)K);
        int t, k;
        or_iq2_dequant(blocks + (size_t)n * (K / 256) * 66, 1, K, w);
        for (k = 0; k < K; k++) w[k] = or_h2f(or_f2h(w[k]));
        for (t = 0; t < T; t++) {
            double acc = 0.0;
            float v;
            for (k = 0; k < K; k++) acc += (double)w[k] * (double)x[(size_t)t * K + k];
            v = (float)acc;
            if (epi == 1) v = v > 0.f ? v * v : 0.f;
            y[(size_t)t * N + n] = v;
        }
        free(w);
    }
}

/* ------------------------------------------------------------------------------------------------------ */
/* inputs and threads of the timed CPU arm                                                                 */
/* ------------------------------------------------------------------------------------------------------ */

/* BASELINE's seeded IQ2_XXS generator (d fp16 ~ U[1e-3, 1e-2], grid indices U{0..255}, sign indices U{0..127},
 * sub-scales U{0..15}; block i depends on (seed, i) only), stated here so that the CPU arm of the benchmark makes
 * the weights the GPU arm makes from the same seed without loading the product library.  A CPU test checks the bytes
 * against the library's host generator. */
static uint64_t or_splitmix64(uint64_t x) {
    x += 0x9E3779B97F4A7C15ull;
    x = (x ^ (x >> 30)) * 0xBF58476D1CE4E5B9ull;
    x = (x ^ (x >> 27)) * 0x94D049BB133111EBull;
    return x ^ (x >> 31);
}

EXPORT void or_synth_iq2(uint64_t seed, int64_t nblocks, uint8_t* out) {
    int64_t i;
#pragma omp parallel for schedule(static)
    for (i = 0; i < nblocks; i++) {
        uint8_t* b = out + i * 66;
        uint64_t h = or_splitmix64(seed ^ or_splitmix64((uint64_t)i * 0x100000001B3ull + 0x51ED27ull));
        const float u = (float)(h >> 40) * (1.f / 16777216.f);
        const uint16_t d = or_f2h(1e-3f + 9e-3f * u);
        int c;
        b[0] = (uint8_t)(d & 255);
        b[1] = (uint8_t)(d >> 8);
        for (c = 0; c < 8; c++) {
            uint32_t grid, aux, s4, hi;
            uint8_t* p = b + 2 + 8 * c;
            h = or_splitmix64(h + (uint64_t)c);
            grid = (uint32_t)h;
            aux = (uint32_t)(h >> 32);
            s4 = (uint32_t)(or_splitmix64(h ^ 0xA5A5ull) & 15u);
            hi = (aux & 0x0fffffffu) | (s4 << 28);
            p[0] = (uint8_t)grid; p[1] = (uint8_t)(grid >> 8); p[2] = (uint8_t)(grid >> 16); p[3] = (uint8_t)(grid >> 24);
            p[4] = (uint8_t)hi; p[5] = (uint8_t)(hi >> 8); p[6] = (uint8_t)(hi >> 16); p[7] = (uint8_t)(hi >> 24);
        }
    }
}

/* the OpenMP thread count of the oracle's parallel loops (1: the scalar single-thread baseline) */
#include <omp.h>
EXPORT void or_set_threads(int n) { omp_set_num_threads(n > 0 ? n : 1); }
EXPORT int or_max_threads(void) { return omp_get_max_threads(); }

/* IQ2_XXS with the chunk scale folded into bf16 weights: the shared-expert GEMM of libbolt's mma_iq2 (PIQ2::step,
 * bolt_mma.cu:372-397 over the tables of PIQ2::init, :310-324): dA = d * (0.5 + s4) * 0.25 rounded to bf16, each
 * weight the bf16 product of that and the signed grid magnitude (round to nearest even), fp64 accumulation here (the
 * kernel: fp32 on the tensor cores).  x is taken as given (the kernel rounds its rows to bf16; the caller does here).
 * epi 1: relu^2. */
EXPORT void or_iq2_gemm_bf16fold(const uint8_t* blocks, int N, int K, const float* x, int T, float* y, int epi) {
    int n;
#pragma omp parallel for schedule(dynamic, 16)
    for (n = 0; n < N; n++) {
        float* w = (float*)malloc(sizeof(float) * (size_t)K);
        int b, c, l, j, t, k;
        for (b = 0; b < K / 256; b++) {
            const uint8_t* blk = blocks + ((size_t)n * (K / 256) + b) * 66;
            const float d = or_h2f(rd16(blk));
            for (c = 0; c < 8; c++) {
                const uint32_t qx = rd32(blk + 2 + 8 * c), qy = rd32(blk + 2 + 8 * c + 4);
                const float sa = or_bf2f(or_f2bf(d * (0.5f + (float)(qy >> 28)) * 0.25f));
                for (l = 0; l < 4; l++) {
                    const uint64_t g = iq2xxs_grid[(qx >> (8 * l)) & 255];
                    const uint32_t sidx = (qy >> (7 * l)) & 127;
                    const uint32_t sg = ksigns_iq2xs[sidx];
                    for (j = 0; j < 8; j++) {
                        float v = (float)((g >> (8 * j)) & 255);
                        if ((sg >> j) & 1) v = -v;
                        w[b * 256 + c * 32 + l * 8 + j] = or_bf2f(or_f2bf(v * sa));
                    }
                }
            }
        }
        for (t = 0; t < T; t++) {
            double acc = 0.0;
            float v;
            for (k = 0; k < K; k++) acc += (double)w[k] * (double)x[(size_t)t * K + k];
            v = (float)acc;
            if (epi == 1) v = v > 0.f ? v * v : 0.f;
            y[(size_t)t * N + n] = v;
        }
        free(w);
    }
}
