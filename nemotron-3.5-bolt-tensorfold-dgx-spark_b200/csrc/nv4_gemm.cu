// The NVFP4 prompt GEMM on the sm_100a block-scaled tensor cores: tcgen05.mma.kind::mxf4nvf4.block16 (e2m1 A and B,
// one ue4m3 scale per 16 k on each side, fp32 accumulation in TMEM), the path libbolt takes for prompt row counts
// (quant_nv4_rows_k + mma_nv4_fp4_k, bolt_mma.cu:925-1059, dispatched at bolt_host.cu:634,644).
//
// y[t][n] = s2 * sum_k e2m1(x4[t][k]) e4m3(sx[t][k/16]) e2m1(w[n][k]) e4m3(sw[n][k/16])
//
// Both operands live in HBM as "tile images": the exact bytes a pipeline stage holds in shared memory, so one
// cp.async.bulk per operand fills a stage (no tensor map, one destination, no register staging):
//   weights  (b200q_nv4_tc_pack)      record (n-tile of 256 rows, 256 k): 32 KB of e2m1 then 4 KB of scales
//   rows     (b200q_quant_nv4_rows)   record (m-tile of 128 rows, 256 k): 16 KB of e2m1 then 2 KB of scales
// e2m1 part: row r's 128 bytes (k = 2b low nibble, 2b + 1 high nibble of byte b) at r * 128 with the 16-byte chunk c
// stored at position c ^ (r & 7): the 128-byte-swizzled K-major layout of the UMMA descriptors.
// scale part: per 64-k block kb and 128-row group h, a 512-byte atom, the scale of (row r, 16-k block s) at
// (r % 32) * 16 + (r / 32) * 4 + s; tcgen05.cp 32x128b.warpx4 copies an atom to 4 TMEM columns (all 128 lanes), the
// layout the block-scaled MMA reads (row r's four scales in lane r % 32 + 32 q, column r / 32, byte s).
// Records are ordered tile-major: (tile, ks) at (tile * k/256 + ks) * record bytes.
//
// A persistent CTA (one per SM) loops over 128 x 256 output tiles: warp 0 (one lane) issues the bulk copies of a
// 4-stage ring, warp 1 (one lane) copies each stage's scales to TMEM and issues its four m128n256k64 MMAs, and 8
// epilogue warps drain the 256-column accumulator (tcgen05.ld), release it to the MMA warp, scale by s2 and store.
// Numerics: the products of e2m1 values and e4m3 scales are exact; the sums are the tensor core's fp32 sums.  Every
// wait is bounded (%globaltimer); on a timeout the kernel records an error (b200q_device_error bit 8), waits for its
// own copies and MMAs, frees its TMEM and returns.
#include "tcgen05.cuh"

namespace b200q {

constexpr int kF4M = 128, kF4N = 256, kF4K = 256;        // tile rows, tile columns (weight rows), k per stage
constexpr int kF4AData = kF4M * 128, kF4ASf = 4 * 512;    // 16 KB + 2 KB
constexpr int kF4BData = kF4N * 128, kF4BSf = 8 * 512;    // 32 KB + 4 KB
constexpr int kF4ARec = kF4AData + kF4ASf;                // 18432
constexpr int kF4BRec = kF4BData + kF4BSf;                // 36864
constexpr int kF4Stage = kF4ARec + kF4BRec;               // 55296 (a multiple of 1024)
constexpr int kF4Stages = 4;
constexpr int kF4EpiWarps = 8;
constexpr int kF4Threads = (2 + kF4EpiWarps) * 32;
constexpr size_t kF4Smem = (size_t)kF4Stages * kF4Stage + 1024 /*align*/ + 256 /*barriers*/;
constexpr int kF4SfCols = 48;                             // TMEM columns of a stage's scales: 16 (A) + 32 (B)
constexpr uint32_t kF4TmemCols = 512;                     // 256 accumulator + 4 x 48 scale columns, rounded up

// instruction descriptor, kind::mxf4nvf4: e2m1 A and B (format 1), K-major, N = 256 (128 for a ragged last weight
// tile), ue4m3 scales, M = 128, scale-factor ids 0 (each 32-bit TMEM column holds the four 16-k scales of a 64-k block)
constexpr uint32_t f4_idesc(int n) {
    return (1u << 7) | (1u << 10) | ((uint32_t)(n >> 3) << 17) | ((uint32_t)(kF4M >> 4) << 24);
}
constexpr uint32_t kIdescF4 = f4_idesc(kF4N), kIdescF4Half = f4_idesc(kF4N / 2);

__device__ int g_nv4_error;   // bit 0: a barrier wait timed out

int nv4_error_read(int clear) {
    int v = 0;
    if (cudaMemcpyFromSymbol(&v, g_nv4_error, sizeof(int)) != cudaSuccess) return -1;
    if (clear) {
        const int z = 0;
        cudaMemcpyToSymbol(g_nv4_error, &z, sizeof(int));
    }
    return v;
}

__device__ __forceinline__ void umma_f4(uint32_t tmem_d, uint64_t a, uint64_t b, uint32_t accumulate, uint32_t sfa,
                                        uint32_t sfb, uint32_t idesc) {
    asm volatile(
        "{ .reg .pred p; setp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::1.kind::mxf4nvf4.block_scale.block16 [%0], %1, %2, %3, [%5], [%6], p; }"
        ::"r"(tmem_d), "l"(a), "l"(b), "r"(idesc), "r"(accumulate), "r"(sfa), "r"(sfb));
}
__device__ __forceinline__ void tmem_cp_sf(uint32_t taddr, uint64_t src) {
    asm volatile("tcgen05.cp.cta_group::1.32x128b.warpx4 [%0], %1;" ::"r"(taddr), "l"(src));
}

// position of the scale of (row r of the record's rows, 16-k block j of the stage) inside a record's scale part
__host__ __device__ __forceinline__ uint32_t f4_sf_off(int r, int j, int groups) {
    const int kb = j >> 2, s = j & 3, h = r >> 7, rr = r & 127;
    return (uint32_t)((kb * groups + h) * 512 + (rr & 31) * 16 + (rr >> 5) * 4 + s);
}

// ---------------------------------------------------------------------------------------------------------
// e4m3 / e2m1 encoders of the prompt quantiser (e4m3_enc / e4m3_dec / e2m1_enc, bolt_mma.cu:868-890): the same
// steps, so the codes are bit-identical to libbolt's.
// ---------------------------------------------------------------------------------------------------------
__device__ __forceinline__ uint32_t f4_e4m3_enc(float v) {
    if (!(v > 0.f)) return 0u;
    if (v >= 448.f) return 0x7Eu;
    int e;
    const float m = frexpf(v, &e);
    e -= 1;
    if (e < -6) {
        const int q = (int)rintf(v * 512.f);
        return q >= 8 ? 0x08u : (uint32_t)q;
    }
    int mant = (int)rintf((2.f * m - 1.f) * 8.f);
    if (mant == 8) { mant = 0; e++; if (e > 8) return 0x7Eu; }
    return ((uint32_t)(e + 7) << 3) | (uint32_t)mant;
}
__device__ __forceinline__ float f4_e4m3_dec(uint32_t c) {
    const int ef = (int)(c >> 3), m = (int)(c & 7);
    return ef == 0 ? (float)m * 0.001953125f : ldexpf(1.f + (float)m * 0.125f, ef - 7);
}
__device__ __forceinline__ uint32_t f4_e2m1_enc(float v) {
    const float u = fabsf(v);
    const uint32_t c = u < 0.25f ? 0u : u < 0.75f ? 1u : u < 1.25f ? 2u : u < 1.75f ? 3u : u < 2.5f ? 4u : u < 3.5f ? 5u : u < 5.f ? 6u : 7u;
    return c | (v < 0.f ? 8u : 0u);
}

// 32 k of one row (two 16-k blocks) -> one 16-byte chunk of e2m1 codes (k = 2b low nibble, 2b + 1 high nibble of
// byte b) and two e4m3 scales: quant_nv4_rows_k's steps (bolt_mma.cu:926-946), scale = e4m3(amax / 6)
__device__ __forceinline__ void f4_quant32(const float* v, uint32_t* w, uint32_t* sc) {
#pragma unroll
    for (int b = 0; b < 2; b++) {
        float amax = 0.f;
#pragma unroll
        for (int j = 0; j < 16; j++) amax = fmaxf(amax, fabsf(v[16 * b + j]));
        const uint32_t code = f4_e4m3_enc(amax * (1.f / 6.f));
        const float sq = f4_e4m3_dec(code);
        const float inv = sq > 0.f ? 1.f / sq : 0.f;
        uint32_t lo = 0, hi = 0;
#pragma unroll
        for (int j = 0; j < 8; j++) {
            lo |= f4_e2m1_enc(v[16 * b + j] * inv) << (4 * j);
            hi |= f4_e2m1_enc(v[16 * b + 8 + j] * inv) << (4 * j);
        }
        w[2 * b] = lo;
        w[2 * b + 1] = hi;
        sc[b] = code;
    }
}

// rows -> NVFP4 tile image.  A thread quantises 32 k of one row (two 16-k blocks: one 16-byte chunk, two scales);
// rows T..Mp-1 of the last m-tile are written as zeros.
__global__ void quant_nv4_rows_k(const void* __restrict__ x, int dtype, int ldx, int T, int k, int Mp,
                                 uint8_t* __restrict__ out) {
    pdl_wait();
    const int per = k >> 5;
    const size_t i = (size_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (i < (size_t)Mp * per) {
        const int row = (int)(i / per), c32 = (int)(i % per);
        const int ks = c32 >> 3, c = c32 & 7, mt = row >> 7, r = row & 127;
        uint8_t* rec = out + ((size_t)mt * (k / kF4K) + ks) * kF4ARec;
        uint32_t w[4] = {0u, 0u, 0u, 0u}, sc[2] = {0u, 0u};
        if (row < T) {
            float v[32];
            if (dtype == B200Q_BF16) {
                const uint4* p = reinterpret_cast<const uint4*>(reinterpret_cast<const __nv_bfloat16*>(x) + (size_t)row * ldx + c32 * 32);
#pragma unroll
                for (int j = 0; j < 4; j++) {
                    const uint4 u = __ldg(p + j);
                    const uint32_t uw[4] = {u.x, u.y, u.z, u.w};
#pragma unroll
                    for (int e = 0; e < 4; e++) { v[8 * j + 2 * e] = __uint_as_float(uw[e] << 16); v[8 * j + 2 * e + 1] = __uint_as_float(uw[e] & 0xffff0000u); }
                }
            } else {
                const float4* p = reinterpret_cast<const float4*>(reinterpret_cast<const float*>(x) + (size_t)row * ldx + c32 * 32);
#pragma unroll
                for (int j = 0; j < 8; j++) { const float4 f = __ldg(p + j); v[4 * j] = f.x; v[4 * j + 1] = f.y; v[4 * j + 2] = f.z; v[4 * j + 3] = f.w; }
            }
            f4_quant32(v, w, sc);
        }
        *reinterpret_cast<uint4*>(rec + sw128_off(r, c)) = make_uint4(w[0], w[1], w[2], w[3]);
        rec[kF4AData + f4_sf_off(r, 2 * c, 1)] = (uint8_t)sc[0];
        rec[kF4AData + f4_sf_off(r, 2 * c + 1, 1)] = (uint8_t)sc[1];
    }
    pdl_trigger();
}

// checkpoint NVFP4 (q [n][k/2], sc [n][k/16] e4m3) -> weight tile image; rows n..Np-1 zero.  A thread moves one
// 16-byte chunk (32 k) and its two scales.
__global__ void nv4_tc_pack_k(const uint8_t* __restrict__ q, const uint8_t* __restrict__ sc, int64_t n, int k, int64_t Np,
                              uint8_t* __restrict__ out) {
    pdl_wait();
    const int per = k >> 5;
    const size_t i = (size_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (i < (size_t)Np * per) {
        const int64_t row = (int64_t)(i / per);
        const int c32 = (int)(i % per), ks = c32 >> 3, c = c32 & 7, r = (int)(row & 255);
        uint8_t* rec = out + ((size_t)(row >> 8) * (k / kF4K) + ks) * kF4BRec;
        uint4 v = make_uint4(0, 0, 0, 0);
        uint8_t s0 = 0, s1 = 0;
        if (row < n) {
            v = __ldg(reinterpret_cast<const uint4*>(q + (size_t)row * (k / 2) + (size_t)c32 * 16));
            s0 = sc[(size_t)row * (k / 16) + 2 * c32];
            s1 = sc[(size_t)row * (k / 16) + 2 * c32 + 1];
        }
        *reinterpret_cast<uint4*>(rec + sw128_off(r, c)) = v;
        rec[kF4BData + f4_sf_off(r, 2 * c, 2)] = s0;
        rec[kF4BData + f4_sf_off(r, 2 * c + 1, 2)] = s1;
    }
    pdl_trigger();
}

// ---------------------------------------------------------------------------------------------------------
// libbolt's own buffers for its BOLT_NV4_FP4 prompt path (the shims tile_nv4w / quant_nv4_rows / mma_nv4_fp4):
//  * rows, plain: q4 [T][k/2] (low nibble first), sf [T][k/16] e4m3 -- libbolt's quant_nv4_rows layout, the same bytes;
//    the GEMM's rows image is made from them by f4_rows_from_plain_k;
//  * weights, "planes": the weight image split into a code plane (in libbolt's tile buffer, n*k/2 bytes) and a scale
//    plane (its scale buffer, n*k/16 bytes), record (n-tile, ks) at nt*KS*32 KB + ks*rows*128 in the code plane and
//    nt*KS*4 KB + ks*rows*16 in the scale plane, rows = 256 except a last tile of 128 (n % 256 == 128, in_proj's
//    18560), whose records are packed at half size so that both planes hold exactly libbolt's byte counts.
// ---------------------------------------------------------------------------------------------------------
__global__ void quant_nv4_plain_k(const float* __restrict__ x, int ldx, int T, int k, uint8_t* __restrict__ q4,
                                  uint8_t* __restrict__ sf) {
    pdl_wait();
    const int per = k >> 5;
    const size_t i = (size_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (i < (size_t)T * per) {
        const int row = (int)(i / per), c32 = (int)(i % per);
        float v[32];
        const float4* p = reinterpret_cast<const float4*>(x + (size_t)row * ldx + c32 * 32);
#pragma unroll
        for (int j = 0; j < 8; j++) { const float4 f = __ldg(p + j); v[4 * j] = f.x; v[4 * j + 1] = f.y; v[4 * j + 2] = f.z; v[4 * j + 3] = f.w; }
        uint32_t w[4], sc[2];
        f4_quant32(v, w, sc);
        *reinterpret_cast<uint4*>(q4 + (size_t)row * (k / 2) + (size_t)c32 * 16) = make_uint4(w[0], w[1], w[2], w[3]);
        sf[(size_t)row * (k / 16) + 2 * c32] = (uint8_t)sc[0];
        sf[(size_t)row * (k / 16) + 2 * c32 + 1] = (uint8_t)sc[1];
    }
    pdl_trigger();
}

// plain rows (q4, sf) -> the rows image; rows T..Mp-1 zero
__global__ void f4_rows_from_plain_k(const uint8_t* __restrict__ q4, const uint8_t* __restrict__ sf, int T, int k, int Mp,
                                     uint8_t* __restrict__ out) {
    pdl_wait();
    const int per = k >> 5;
    const size_t i = (size_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (i < (size_t)Mp * per) {
        const int row = (int)(i / per), c32 = (int)(i % per);
        const int ks = c32 >> 3, c = c32 & 7, mt = row >> 7, r = row & 127;
        uint8_t* rec = out + ((size_t)mt * (k / kF4K) + ks) * kF4ARec;
        uint4 v = make_uint4(0, 0, 0, 0);
        uint8_t s0 = 0, s1 = 0;
        if (row < T) {
            v = __ldg(reinterpret_cast<const uint4*>(q4 + (size_t)row * (k / 2) + (size_t)c32 * 16));
            s0 = sf[(size_t)row * (k / 16) + 2 * c32];
            s1 = sf[(size_t)row * (k / 16) + 2 * c32 + 1];
        }
        *reinterpret_cast<uint4*>(rec + sw128_off(r, c)) = v;
        rec[kF4AData + f4_sf_off(r, 2 * c, 1)] = s0;
        rec[kF4AData + f4_sf_off(r, 2 * c + 1, 1)] = s1;
    }
    pdl_trigger();
}

// checkpoint NVFP4 -> the weight planes; a thread moves one 16-byte chunk (32 k) and its two scales
__global__ void nv4_tc_pack_planes_k(const uint8_t* __restrict__ q, const uint8_t* __restrict__ sc, int n, int k,
                                     uint8_t* __restrict__ qw, uint8_t* __restrict__ sfw) {
    pdl_wait();
    const int per = k >> 5, KS = k / kF4K;
    const size_t i = (size_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (i < (size_t)n * per) {
        const int row = (int)(i / per), c32 = (int)(i % per);
        const int ks = c32 >> 3, c = c32 & 7, nt = row >> 8, r = row & 255;
        const int rows = n - nt * kF4N < kF4N ? kF4N / 2 : kF4N;
        uint8_t* code = qw + (size_t)nt * KS * kF4BData + (size_t)ks * rows * 128;
        uint8_t* scl = sfw + (size_t)nt * KS * kF4BSf + (size_t)ks * rows * 16;
        *reinterpret_cast<uint4*>(code + sw128_off(r, c)) =
            __ldg(reinterpret_cast<const uint4*>(q + (size_t)row * (k / 2) + (size_t)c32 * 16));
        scl[f4_sf_off(r, 2 * c, rows / 128)] = sc[(size_t)row * (k / 16) + 2 * c32];
        scl[f4_sf_off(r, 2 * c + 1, rows / 128)] = sc[(size_t)row * (k / 16) + 2 * c32 + 1];
    }
    pdl_trigger();
}

struct F4Args {
    const uint8_t* w;        // weight tile image; with wsf, the code plane of the weight planes
    const uint8_t* wsf;      // the scale plane of the weight planes (nullptr: w is the interleaved image)
    const uint8_t* a;        // rows tile image
    float* y;
    int n, k, T, ldy;
    float s2;
    int ksplit;              // K slices a tile's sum is cut into (1: none)
    float* part;             // ksplit > 1: unscaled partial sums [ksplit][T][n]
};

// PLANES: the weights are the planes form (a.wsf, a last tile of 128 rows allowed); a template parameter so that the
// image form's MMA lane carries no per-stage branch on it
template <bool PLANES>
__global__ void __launch_bounds__(kF4Threads, 1) nv4_gemm_k(F4Args a) {
    extern __shared__ __align__(1024) unsigned char f4_dyn[];
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const uint32_t raw = (uint32_t)__cvta_generic_to_shared(f4_dyn);
    const uint32_t sbase = (raw + 1023u) & ~1023u;
    const uint32_t bars = sbase + kF4Stages * kF4Stage;   // full[s], empty[s], acc_full, acc_empty, drain, tmem slot
    auto full = [&](int s) { return bars + 8u * s; };
    auto empty = [&](int s) { return bars + 8u * (kF4Stages + s); };
    const uint32_t acc_full = bars + 8u * (2 * kF4Stages), acc_empty = acc_full + 8u, drain = acc_full + 16u;
    const uint32_t tmem_slot = acc_full + 24u;
    unsigned char* tmem_slot_ptr = f4_dyn + (tmem_slot - raw);

    const int MT = (a.T + kF4M - 1) / kF4M, NT = (a.n + kF4N - 1) / kF4N, KS = a.k / kF4K;
    // weight rows of n-tile nt: 256, or 128 for the last tile of the planes form when n % 256 == 128
    auto tile_rows = [&](int nt) { return (PLANES && a.n - nt * kF4N < kF4N) ? kF4N / 2 : kF4N; };
    const int tiles = MT * NT * a.ksplit;   // work items: (tile, K slice)
    // item -> tile (m fastest within an n-tile), K slice; stage range [ks0, ks1)
    auto item = [&](int i, int& mt, int& nt, int& ks0, int& ks1) {
        const int t = i / a.ksplit, sl = i - t * a.ksplit;
        nt = t / MT;
        mt = t - nt * MT;
        ks0 = sl * KS / a.ksplit;
        ks1 = (sl + 1) * KS / a.ksplit;
    };

    if (tid == 0) {
        for (int s = 0; s < kF4Stages; s++) { tc_mbar_init(full(s), 1); tc_mbar_init(empty(s), 1); }
        tc_mbar_init(acc_full, 1);
        tc_mbar_init(acc_empty, kF4EpiWarps);
        tc_mbar_init(drain, 1);
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    }
    if (warp == 1) {
        asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(tmem_slot), "r"(kF4TmemCols));
        asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;");
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = *reinterpret_cast<volatile uint32_t*>(tmem_slot_ptr);
    pdl_wait();

    if (warp == 0) {
        // producer: one lane streams the stage records
        if (lane == 0) {
            bool healthy = true;
            int it = 0;
            for (int tile = blockIdx.x; tile < tiles && healthy; tile += gridDim.x) {
                int mt, nt, ks0, ks1;
                item(tile, mt, nt, ks0, ks1);
                const uint8_t* ap = a.a + (size_t)mt * KS * kF4ARec;
                const int rows = tile_rows(nt);
                for (int ks = ks0; ks < ks1; ks++, it++) {
                    const int s = it % kF4Stages, use = it / kF4Stages;
                    if (use > 0 && !tc_mbar_wait(empty(s), (uint32_t)((use - 1) & 1))) { healthy = false; break; }
                    const uint32_t st = sbase + (uint32_t)(s * kF4Stage);
                    tc_mbar_arrive_tx(full(s), (uint32_t)(kF4ARec + rows * 144));
                    tc_bulk_g2s(st, ap + (size_t)ks * kF4ARec, (uint32_t)kF4ARec, full(s));
                    if constexpr (PLANES) {   // the planes: codes then scales, at the stage's usual places
                        tc_bulk_g2s(st + kF4ARec, a.w + (size_t)nt * KS * kF4BData + (size_t)ks * rows * 128,
                                    (uint32_t)(rows * 128), full(s));
                        tc_bulk_g2s(st + kF4ARec + kF4BData, a.wsf + (size_t)nt * KS * kF4BSf + (size_t)ks * rows * 16,
                                    (uint32_t)(rows * 16), full(s));
                    } else {
                        tc_bulk_g2s(st + kF4ARec, a.w + ((size_t)nt * KS + ks) * kF4BRec, (uint32_t)kF4BRec, full(s));
                    }
                }
            }
            // the copies of the last uses of every stage have landed before the CTA may exit
            for (int i = it - kF4Stages > 0 ? it - kF4Stages : 0; i < it; i++)
                if (!tc_mbar_wait(full(i % kF4Stages), (uint32_t)((i / kF4Stages) & 1))) healthy = false;
            if (!healthy) atomicOr(&g_nv4_error, 1);
        }
        __syncwarp();
    } else if (warp == 1) {
        // MMA issuer
        if (lane == 0) {
            bool healthy = true;
            int it = 0, tl = 0;
            for (int tile = blockIdx.x; tile < tiles && healthy; tile += gridDim.x, tl++) {
                int mt, nt, ks0, ks1;
                item(tile, mt, nt, ks0, ks1);
                if (tl > 0 && !tc_mbar_wait(acc_empty, (uint32_t)((tl - 1) & 1))) { healthy = false; break; }
                tc_fence_after();
                const bool half_n = PLANES && tile_rows(nt) < kF4N;   // a 128-row tile: one scale atom a 64-k block, N = 128
                const uint32_t idesc = half_n ? kIdescF4Half : kIdescF4;
                for (int ks = ks0; ks < ks1; ks++, it++) {
                    const int s = it % kF4Stages;
                    if (!tc_mbar_wait(full(s), (uint32_t)((it / kF4Stages) & 1))) { healthy = false; break; }
                    tc_fence_after();
                    const uint32_t st = sbase + (uint32_t)(s * kF4Stage);
                    const uint32_t at = st, asf = st + kF4AData, bt = st + kF4ARec, bsf = bt + kF4BData;
                    const uint32_t sfa = tmem + 256u + (uint32_t)(s * kF4SfCols), sfb = sfa + 16u;
#pragma unroll
                    for (int kb = 0; kb < 4; kb++) {
                        tmem_cp_sf(sfa + 4u * kb, umma_desc_rows16(asf + kb * 512));
                        if (PLANES && half_n) {
                            tmem_cp_sf(sfb + 8u * kb, umma_desc_rows16(bsf + kb * 512));
                        } else {
                            tmem_cp_sf(sfb + 8u * kb, umma_desc_rows16(bsf + (2 * kb) * 512));
                            tmem_cp_sf(sfb + 8u * kb + 4u, umma_desc_rows16(bsf + (2 * kb + 1) * 512));
                        }
                    }
#pragma unroll
                    for (int kb = 0; kb < 4; kb++)
                        umma_f4(tmem, umma_desc_sw128(at + kb * 32), umma_desc_sw128(bt + kb * 32),
                                (ks > ks0 || kb > 0) ? 1u : 0u, sfa + 4u * kb, sfb + 8u * kb, idesc);
                    umma_commit(empty(s));
                }
                if (healthy) umma_commit(acc_full);
            }
            // every MMA and scale copy this thread issued has completed before the TMEM is freed
            umma_commit(drain);
            if (!tc_mbar_wait(drain, 0)) healthy = false;
            if (!healthy) atomicOr(&g_nv4_error, 1);
        }
        __syncwarp();
    } else {
        // epilogue: warp w reads TMEM lanes 32 (w % 4).. (tile rows) and columns 128 ((w - 2) / 4)..
        const int q = warp & 3, half = (warp - 2) >> 2;
        const bool split = a.ksplit > 1;
        const int ld = split ? a.n : a.ldy;
        const float sc = split ? 1.f : a.s2;
        const bool vec = ((ld & 3) == 0) && ((reinterpret_cast<uintptr_t>(split ? a.part : a.y) & 15) == 0);
        int tl = 0;
        for (int tile = blockIdx.x; tile < tiles; tile += gridDim.x, tl++) {
            int mt, nt, ks0, ks1;
            item(tile, mt, nt, ks0, ks1);
            float* dst = split ? a.part + (size_t)(tile % a.ksplit) * a.T * a.n : a.y;
            if (!tc_mbar_wait(acc_full, (uint32_t)(tl & 1))) {
                if (lane == 0) atomicOr(&g_nv4_error, 1);
                break;
            }
            tc_fence_after();
            uint32_t v[4][32];
            const uint32_t base = tmem + ((uint32_t)(q * 32) << 16) + (uint32_t)(half * 128);
#pragma unroll
            for (int j = 0; j < 4; j++) tmem_ld32(base + 32u * j, v[j]);
            tmem_ld_wait();
            tc_fence_before();
            __syncwarp();
            if (lane == 0) tc_mbar_arrive(acc_empty);   // the accumulator may be overwritten now
            const int row = mt * kF4M + q * 32 + lane;
            const int col0 = nt * kF4N + half * 128;
            if (row < a.T) {
                float* yr = dst + (size_t)row * ld;
#pragma unroll
                for (int j = 0; j < 4; j++) {
#pragma unroll
                    for (int e = 0; e < 32; e += 4) {
                        const int col = col0 + 32 * j + e;
                        const float f0 = __uint_as_float(v[j][e]) * sc, f1 = __uint_as_float(v[j][e + 1]) * sc;
                        const float f2 = __uint_as_float(v[j][e + 2]) * sc, f3 = __uint_as_float(v[j][e + 3]) * sc;
                        if (vec && col + 4 <= a.n) {
                            *reinterpret_cast<float4*>(yr + col) = make_float4(f0, f1, f2, f3);
                        } else {
                            if (col < a.n) yr[col] = f0;
                            if (col + 1 < a.n) yr[col + 1] = f1;
                            if (col + 2 < a.n) yr[col + 2] = f2;
                            if (col + 3 < a.n) yr[col + 3] = f3;
                        }
                    }
                }
            }
        }
    }
    tc_fence_before();
    __syncthreads();
    if (warp == 1) {
        tc_fence_after();
        asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(kF4TmemCols));
    }
    pdl_trigger();
}

// y[t][c] = s2 * (part[0][t][c] + part[1][t][c] + ...), the slices added in order
__global__ void f4_splitk_sum_k(const float* __restrict__ part, int ksplit, int T, int n, float s2, float* __restrict__ y,
                                int ldy) {
    pdl_wait();
    const size_t i = (size_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (i < (size_t)T * n) {
        const int t = (int)(i / n), c = (int)(i % n);
        float acc = part[i];
        for (int sl = 1; sl < ksplit; sl++) acc += part[(size_t)sl * T * n + i];
        y[(size_t)t * ldy + c] = acc * s2;
    }
    pdl_trigger();
}

// K slices for a launch with at most a quarter of the SMs' worth of tiles (up to 4, at least 2 stages a slice).  A
// CTA's ring is bound by the latency of its bulk copies, so slicing pays only when most SMs would otherwise idle (out_proj
// at M = 512, 64 tiles on 148 SMs, measured slower sliced in two).
static int f4_ksplit(int tiles, int KS, int sms) {
    if (tiles * 4 > sms) return 1;
    int s = sms / tiles;
    if (s > 4) s = 4;
    if (s > KS / 2) s = KS / 2;
    return s < 2 ? 1 : s;
}

static int f4_num_sms() {
    static int sms[64] = {0};
    int dev = 0;
    cudaGetDevice(&dev);
    if (dev < 0 || dev >= 64) dev = 0;
    if (!sms[dev]) {
        int v = 0;
        cudaDeviceGetAttribute(&v, cudaDevAttrMultiProcessorCount, dev);
        sms[dev] = v > 0 ? v : 148;
    }
    return sms[dev];
}

static inline bool a16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15) == 0; }

static bool f4_opt_in() {
    static bool opted = false;
    if (!opted) {
        if (cudaFuncSetAttribute(nv4_gemm_k<false>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)kF4Smem) !=
                cudaSuccess ||
            cudaFuncSetAttribute(nv4_gemm_k<true>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)kF4Smem) !=
                cudaSuccess)
            return false;
        opted = true;
    }
    return true;
}

// ---- libbolt's BOLT_NV4_FP4 buffers (the shims in bolt_shim.cu) ----
// the weight planes into libbolt's tile buffers: qw n*k/2 bytes, sfw n*k/16 bytes; n % 128 == 0, k % 256 == 0
int nv4_planes_pack(const uint8_t* q, const uint8_t* sc, uint8_t* qw, uint8_t* sfw, int n, int k, cudaStream_t s) {
    if (!q || !sc || !qw || !sfw || n <= 0 || n % 128 || k <= 0 || k % kF4K || !a16(q) || !a16(qw) || !a16(sfw))
        return B200Q_EINVAL;
    const size_t th = (size_t)n * (k / 32);
    return status_from(launch(nv4_tc_pack_planes_k, dim3((unsigned)((th + 255) / 256)), dim3(256), 0, s, q, sc, n, k,
                              qw, sfw));
}
// fp32 rows -> libbolt's plain NVFP4 rows (q4 [T][k/2], sf [T][k/16])
int nv4_quant_plain(const float* x, int ldx, uint8_t* q4, uint8_t* sf, int T, int k, cudaStream_t s) {
    if (T <= 0) return B200Q_OK;
    if (!x || !q4 || !sf || k <= 0 || k % kF4K || ldx < k || ldx % 4 || !a16(x) || !a16(q4)) return B200Q_EINVAL;
    const size_t th = (size_t)T * (k / 32);
    return status_from(launch(quant_nv4_plain_k, dim3((unsigned)((th + 255) / 256)), dim3(256), 0, s, x, ldx, T, k, q4,
                              sf));
}
// y = s2 * planes-weights x plain rows; rows_img: b200q_nv4_rows_bytes(T, k) bytes of scratch (the rows image)
int nv4_gemm_planes(const uint8_t* qw, const uint8_t* sfw, int n, int k, float s2, const uint8_t* q4, const uint8_t* sf,
                    int T, uint8_t* rows_img, float* y, int ldy, cudaStream_t s) {
    if (T <= 0) return B200Q_OK;
    if (!qw || !sfw || !q4 || !sf || !rows_img || !y || n <= 0 || n % 128 || k <= 0 || k % kF4K || ldy < n ||
        !a16(qw) || !a16(sfw) || !a16(q4) || !a16(rows_img))
        return B200Q_EINVAL;
    if (!f4_opt_in()) return status_from(cudaGetLastError());
    const int Mp = (T + kF4M - 1) / kF4M * kF4M;
    const size_t th = (size_t)Mp * (k / 32);
    cudaError_t e = launch(f4_rows_from_plain_k, dim3((unsigned)((th + 255) / 256)), dim3(256), 0, s, q4, sf, T, k, Mp,
                           rows_img);
    if (e != cudaSuccess) return status_from(e);
    const int tiles = ((T + kF4M - 1) / kF4M) * ((n + kF4N - 1) / kF4N);
    const int grid = tiles < f4_num_sms() ? tiles : f4_num_sms();
    F4Args a{qw, sfw, rows_img, y, n, k, T, ldy, s2, 1, nullptr};
    return status_from(launch(nv4_gemm_k<true>, dim3(grid), dim3(kF4Threads), kF4Smem, s, a));
}

}  // namespace b200q

using namespace b200q;

extern "C" {

size_t b200q_nv4_tc_bytes(int64_t n, int k) {
    if (n <= 0 || k <= 0 || k % kF4K) return 0;
    return (size_t)((n + kF4N - 1) / kF4N) * (size_t)(k / kF4K) * kF4BRec;
}

int b200q_nv4_tc_pack(const void* q, const void* sc, void* packed, int64_t n, int k, void* stream) {
    if (!q || !sc || !packed || n <= 0 || k <= 0 || k % kF4K || !a16(q) || !a16(packed)) return B200Q_EINVAL;
    const int64_t Np = (n + kF4N - 1) / kF4N * kF4N;
    const size_t th = (size_t)Np * (k / 32);
    return status_from(launch(nv4_tc_pack_k, dim3((unsigned)((th + 255) / 256)), dim3(256), 0, (cudaStream_t)stream,
                              (const uint8_t*)q, (const uint8_t*)sc, n, k, Np, (uint8_t*)packed));
}

size_t b200q_nv4_rows_bytes(int T, int k) {
    if (T <= 0 || k <= 0 || k % kF4K) return 0;
    return (size_t)((T + kF4M - 1) / kF4M) * (size_t)(k / kF4K) * kF4ARec;
}

int b200q_quant_nv4_rows(const void* x, int x_dtype, int ldx, int T, int k, void* rows, void* stream) {
    if (!x || !rows || T <= 0 || k <= 0 || k % kF4K || ldx < k || !a16(x) || !a16(rows)) return B200Q_EINVAL;
    if (x_dtype != B200Q_F32 && x_dtype != B200Q_BF16) return B200Q_EINVAL;
    if ((x_dtype == B200Q_F32 && ldx % 4) || (x_dtype == B200Q_BF16 && ldx % 8)) return B200Q_EINVAL;
    const int Mp = (T + kF4M - 1) / kF4M * kF4M;
    const size_t th = (size_t)Mp * (k / 32);
    return status_from(launch(quant_nv4_rows_k, dim3((unsigned)((th + 255) / 256)), dim3(256), 0, (cudaStream_t)stream,
                              x, x_dtype, ldx, T, k, Mp, (uint8_t*)rows));
}

size_t b200q_nv4_gemm_workspace_bytes(int n, int k, int T) {
    if (n <= 0 || T <= 0 || k <= 0 || k % kF4K) return 0;
    const int tiles = ((T + kF4M - 1) / kF4M) * ((n + kF4N - 1) / kF4N);
    const int ks = f4_ksplit(tiles, k / kF4K, f4_num_sms());
    return ks > 1 ? (size_t)ks * T * n * sizeof(float) : 0;
}

int b200q_nv4_gemm(const void* w, int n, int k, float s2, const void* rows, int T, float* y, int ldy, void* workspace,
                   size_t workspace_bytes, void* stream) {
    if (!w || !rows || !y || n <= 0 || T <= 0 || k <= 0 || k % kF4K || ldy < n || !a16(w) || !a16(rows)) return B200Q_EINVAL;
    if (!f4_opt_in()) return status_from(cudaGetLastError());
    const int tiles = ((T + kF4M - 1) / kF4M) * ((n + kF4N - 1) / kF4N);
    int ks = f4_ksplit(tiles, k / kF4K, f4_num_sms());
    if (!workspace || workspace_bytes < (size_t)ks * T * n * sizeof(float) || !a16(workspace)) ks = 1;
    const int items = tiles * ks;
    const int grid = items < f4_num_sms() ? items : f4_num_sms();
    F4Args a{(const uint8_t*)w, nullptr, (const uint8_t*)rows, y, n, k, T, ldy, s2, ks, (float*)workspace};
    cudaError_t e = launch(nv4_gemm_k<false>, dim3(grid), dim3(kF4Threads), kF4Smem, (cudaStream_t)stream, a);
    if (e != cudaSuccess || ks == 1) return status_from(e);
    const size_t th = (size_t)T * n;
    return status_from(launch(f4_splitk_sum_k, dim3((unsigned)((th + 255) / 256)), dim3(256), 0, (cudaStream_t)stream,
                              (const float*)workspace, ks, T, n, s2, y, ldy));
}

}  // extern "C"
