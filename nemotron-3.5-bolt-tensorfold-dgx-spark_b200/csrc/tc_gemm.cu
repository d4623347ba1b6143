// Prompt-length GEMMs of the IQ2_XXS experts and the Q8_0 projections on the sm_100a tensor cores: tcgen05.mma
// kind::f16 (fp16 operands, fp32 accumulation in TMEM), the weights dequantised inside the kernel.
//
// C[m][n] = sum_k A[m][k] B[n][k]: A the activation rows (tokens, or the expert-sorted pairs of the MoE), B the weight
// rows.  A CTA computes a tile of up to 256 rows x 256 weight rows as two MMAs per k-step, each with M = 128 weight
// rows (one half of the dequantised weight tile) and N = the tile's rows (both 128-row activation records): two
// accumulators of 256 TMEM columns whose TMEM lanes are weight rows, so every dequantised weight feeds 256 rows and
// the epilogue's lanes hold 32 consecutive outputs of one row (each store a contiguous line).  Per 32-k stage of a 5-stage shared-memory ring:
//   A        the two 128-row halves (8 KB each), bulk-copied (cp.async.bulk, no tensor map) from an fp16 rows image
//            by one lane of warp 0;
//   B        256 weight rows x 32 k in fp16, written by 16 dequantising warps in two sets of 8 that take alternate
//            stages (warp w of a set: rows 32w..32w+31, lane = row), from the packed weights, which each lane
//            prefetches into registers ahead of use.  IQ2_XXS: a prmt picks every fp16 pair out of its chunk's three
//            scaled magnitudes and a xor sets its signs, the selectors and masks read as 128-bit entries from
//            replicated shared-memory tables (conflict-free).  Q8_0: a magic-number prmt makes the int8 exact in fp16
//            and one hmul2 applies the scale;
//   MMA      one lane of warp 1 issues the m128n256k16 (or n128 for tiles of at most 128 rows) MMAs of both weight
//            halves and commits them to the stage's barrier;
//   epilogue 8 warps drain the accumulators (tcgen05.ld: warp w reads lane quarter w % 4 of one accumulator), hand
//            them back to the MMA warp, and write the outputs.
// Tiles (up to 256 rows of one group x 256 weight rows) are handed out persistently, one CTA per SM.
//
// Shared-memory tiles are K-major with the 64-byte swizzle of the UMMA descriptors: rows of 64 B (32 fp16), 8-row
// atoms of 512 B, the 16-byte chunk c of row r at position c ^ ((r >> 1) & 3).
//
// Rows image: the activations of a launch in fp16, in slots of 128 rows; record (slot, 32-k block kk), 8 KB, is the
// shared-memory tile above, at (slot * K/32 + kk) * 8192.  For the MoE the slots of expert e hold its pairs in
// expert-sorted order, 128 a slot; the up projection's epilogue writes fp16(relu(v)^2) straight into the down
// projection's rows image.
//
// Numerics (libbolt's prompt fold, PQ8 bolt_mma.cu:234-254 and PIQ2 bolt_mma.cu:380-397, in fp16):
//   Q8_0   B = fp16(q * d), the scale folded and rounded once.
//   IQ2    B = fp16(d (0.5 + s4) / 4 * signed grid), rounded once.  (FP8 cannot hold the grid magnitudes 25 and 43.)
//   A      activations rounded to fp16 once; the MoE's intermediate act = fp16(relu(v)^2).
// Every barrier wait is bounded (%globaltimer); on a timeout the kernel records an error (b200q_device_error bit 4),
// waits for its own copies and MMAs, frees its TMEM and returns.
#include "tcgen05.cuh"

namespace b200q {

constexpr int kXM = 128;                        // rows of a slot and of an MMA half
constexpr int kXN = 256;                        // weight rows of a tile
constexpr int kXRec = kXM * 64;                 // 8 KB: a rows-image record (128 rows x 32 fp16)
constexpr int kXB = kXN * 64;                   // 16 KB: the B tile of a stage
constexpr int kXStage = 2 * kXRec + kXB;        // 32 KB: the two A halves, then the B tile
constexpr int kXStages = 5;
constexpr int kDeqWarps = 16, kXEpiWarps = 8;  // dequantisers (8 a stage: kDeqWarps / 8 sets taking stages in turn)
constexpr int kPhases = kDeqWarps / 8;
constexpr int kEpiParts = kXEpiWarps / 8;       // epilogue warps an (accumulator, lane quarter), splitting the tokens
constexpr int kXThreads = (2 + kDeqWarps + kXEpiWarps) * 32;   // 832
constexpr int kGridTbl = 256 * 8 * 16;          // 32 KB: grid entry -> four prmt selectors, 8 copies
constexpr int kSignTbl = 128 * 8 * 16;          // 16 KB: sign index -> four xor masks, 8 copies
constexpr size_t kXSmem = (size_t)kXStages * kXStage + kGridTbl + kSignTbl + 1024 /*align*/ + 256 /*barriers*/;
constexpr uint32_t kXTmemCols = 512;            // two 256-column accumulators

__device__ int g_tc_error;   // bit 0: a barrier wait timed out (reported by b200q_device_error)

int tc_error_read(int clear) {
    int v = 0;
    if (cudaMemcpyFromSymbol(&v, g_tc_error, sizeof(int)) != cudaSuccess) return -1;
    if (clear) {
        const int z = 0;
        cudaMemcpyToSymbol(g_tc_error, &z, sizeof(int));
    }
    return v;
}

// instruction descriptors, kind::f16: fp32 accumulator, fp16 A and B, both K-major, M = 128, N = 256 or 128
constexpr uint32_t kIdescF16N256 = (1u << 4) | (256u >> 3) << 17 | ((uint32_t)(kXM >> 4) << 24);
constexpr uint32_t kIdescF16N128 = (1u << 4) | (128u >> 3) << 17 | ((uint32_t)(kXM >> 4) << 24);

__device__ __forceinline__ void umma_f16(uint32_t tmem_d, uint64_t a, uint64_t b, uint32_t idesc, uint32_t accumulate) {
    asm volatile(
        "{ .reg .pred p; setp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, {%5, %6, %7, %8}, p; }"
        ::"r"(tmem_d), "l"(a), "l"(b), "r"(idesc), "r"(accumulate), "r"(0), "r"(0), "r"(0), "r"(0));
}
__device__ __forceinline__ uint32_t h2u(__half2 h) { return *reinterpret_cast<uint32_t*>(&h); }
__device__ __forceinline__ uint32_t prmt(uint32_t a, uint32_t b, uint32_t s) {
    uint32_t d;
    asm("prmt.b32 %0, %1, %2, %3;" : "=r"(d) : "r"(a), "r"(b), "r"(s));
    return d;
}
__device__ __forceinline__ uint4 ldg_nc(const void* p) {
    uint4 v;
    asm volatile("ld.global.nc.v4.u32 {%0,%1,%2,%3}, [%4];" : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w) : "l"(p));
    return v;
}
__device__ __forceinline__ uint2 ldg_nc64(const void* p) {
    uint2 v;
    asm volatile("ld.global.nc.v2.u32 {%0,%1}, [%2];" : "=r"(v.x), "=r"(v.y) : "l"(p));
    return v;
}
__device__ __forceinline__ uint4 lds128(uint32_t addr) {
    uint4 v;
    asm volatile("ld.shared.v4.u32 {%0,%1,%2,%3}, [%4];" : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w) : "r"(addr));
    return v;
}
__device__ __forceinline__ uint32_t ldg_u16(const void* p) {
    unsigned short v;
    asm volatile("ld.global.nc.u16 %0, [%1];" : "=h"(v) : "l"(p));
    return v;
}

// ---------------------------------------------------------------------------------------------------------
// launch description
// ---------------------------------------------------------------------------------------------------------
struct XArgs {
    const uint8_t* w;        // packed weights of group 0
    size_t wstride;          // bytes between the groups' weight matrices
    const uint8_t* a;        // rows image
    int N, K;
    const int4* tiles;       // grouped: {group, first slot, first row in the group, rows}; nullptr: dense
    const int* ntiles;       // grouped: number of tiles (device)
    int max_mtiles;          // grouped: capacity of `tiles`; dense: ceil(T / 256)
    int T;                   // dense: rows
};

__device__ __forceinline__ int4 x_tile(const XArgs& a, int mt) {
    if (a.tiles) return a.tiles[mt];
    const int m0 = mt * 2 * kXM;
    return make_int4(0, 2 * mt, m0, min(2 * kXM, a.T - m0));
}

// Epilogues.  kTokensM picks the MMA's orientation, and so which index a TMEM lane carries:
//   false: weights are M, tokens N.  put(t, n, tok0, lane, v): v[j] = (weight row n, the lane's; token tok0 + j); the
//          32 lanes hold 32 consecutive weight rows, so a token's store is one contiguous line, one element a lane.
//   true:  tokens are M, weights N.  put(t, h, r, col, N, v): v[j] = (token 128 h + r, the lane's; weight row col + j);
//          a lane holds 32 consecutive outputs of one row and stores them 16 bytes at a time.
struct EpiRows {             // fp32 y[orow][n]; orow = rowmap[row0[g] + m0 + token] (or the dense row)
    static constexpr bool kTokensM = false;
    float* y;
    int ldy;
    const int* row0;         // per-group first row in the row list (offsets), nullptr: 0
    const int* rowmap;       // nullptr: identity
    __device__ void put(int4 t, int n, int tok0, int lane, const uint32_t (&v)[32]) const {
        const int grow = (row0 ? row0[t.x] : 0) + t.z + tok0 + lane;
        const int mine = tok0 + lane < t.w ? (rowmap ? rowmap[grow] : grow) : -1;
        float* yn = y + n;
#pragma unroll
        for (int j = 0; j < 32; j++) {
            const int orow = __shfl_sync(0xffffffffu, mine, j);
            if (orow >= 0) yn[(size_t)orow * ldy] = __uint_as_float(v[j]);
        }
    }
};
struct EpiRowsT {            // EpiRows with tokens as M: a lane's 32 outputs of its row as eight 16-byte stores
    static constexpr bool kTokensM = true;
    float* y;
    int ldy;
    const int* row0;
    const int* rowmap;
    __device__ void put(int4 t, int h, int r, int col, int N, const uint32_t (&v)[32]) const {
        const int grow = (row0 ? row0[t.x] : 0) + t.z + h * kXM + r;
        const int orow = rowmap ? rowmap[grow] : grow;
        float* o = y + (size_t)orow * ldy + col;
        if (col + 32 <= N && ((ldy & 3) == 0) && ((reinterpret_cast<uintptr_t>(y) & 15) == 0)) {
#pragma unroll
            for (int i = 0; i < 32; i += 4)
                *reinterpret_cast<float4*>(o + i) =
                    make_float4(__uint_as_float(v[i]), __uint_as_float(v[i + 1]), __uint_as_float(v[i + 2]), __uint_as_float(v[i + 3]));
        } else {
#pragma unroll
            for (int i = 0; i < 32; i++)
                if (col + i < N) o[i] = __uint_as_float(v[i]);
        }
    }
};
struct EpiImg {              // fp16(relu(v)^2) into the next GEMM's rows image (its K = this GEMM's N), tokens as M:
    // a lane's 32 outputs are one 64-byte row of a record, and a warp's 32 lanes write 2 KB of it contiguously
    static constexpr bool kTokensM = true;
    uint8_t* img;
    int N;
    __device__ void put(int4 t, int h, int r, int col, int N_, const uint32_t (&v)[32]) const {
        uint8_t* rec = img + ((size_t)(t.y + h) * (N / 32) + col / 32) * kXRec;
#pragma unroll
        for (int c = 0; c < 4; c++) {
            uint32_t o[4];
#pragma unroll
            for (int j = 0; j < 4; j++) {
                const float a0 = __uint_as_float(v[8 * c + 2 * j]), a1 = __uint_as_float(v[8 * c + 2 * j + 1]);
                o[j] = h2u(__floats2half2_rn(a0 > 0.f ? a0 * a0 : 0.f, a1 > 0.f ? a1 * a1 : 0.f));
            }
            *reinterpret_cast<uint4*>(rec + sw64_off(r, c)) = make_uint4(o[0], o[1], o[2], o[3]);
        }
    }
};
struct EpiImgW {             // EpiImg with weights as M (one fp16 a lane per token row)
    static constexpr bool kTokensM = false;
    uint8_t* img;
    int N;
    __device__ void put(int4 t, int n, int tok0, int lane, const uint32_t (&v)[32]) const {
        const size_t kk = (size_t)(n >> 5), nkk = (size_t)(N >> 5);
        const uint32_t within = (uint32_t)((lane & 7) * 2);
#pragma unroll
        for (int j = 0; j < 32; j++) {
            const int tok = tok0 + j;
            if (tok < t.w) {
                const int r = tok & (kXM - 1);
                uint8_t* rec = img + ((size_t)(t.y + (tok >> 7)) * nkk + kk) * kXRec;
                const float a0 = __uint_as_float(v[j]);
                *reinterpret_cast<__half*>(rec + sw64_off(r, lane >> 3) + within) = __float2half_rn(a0 > 0.f ? a0 * a0 : 0.f);
            }
        }
    }
};

// ---------------------------------------------------------------------------------------------------------
// B dequantisers.  run() produces its phase's stages of one tile for the calling warp's 32 rows (lane = row): for
// each of those 32-k blocks it waits for the stage to be free, writes the row's 64 B, and arrives on the stage's "full"
// barrier.
// ---------------------------------------------------------------------------------------------------------
struct XRing {               // stage bookkeeping shared by the warps of one CTA
    uint32_t sbase, bars;
    __device__ uint32_t full(int it) const { return bars + 8u * (it % kXStages); }
    __device__ uint32_t empty(int it) const { return bars + 8u * (kXStages + it % kXStages); }
    __device__ uint32_t stage(int it) const { return sbase + (uint32_t)((it % kXStages) * kXStage); }
    static constexpr int kBars = 2 * kXStages;
};

// waits (lane 0) for the stage of iteration `it` to be free; false on a timeout (warp-uniform)
__device__ __forceinline__ bool x_wait_free(const XRing& R, int it, int lane) {
    const int use = it / kXStages;
    int ok = 1;
    if (use > 0 && lane == 0) ok = tc_mbar_wait(R.empty(it), (uint32_t)((use - 1) & 1)) ? 1 : 0;
    return __shfl_sync(0xffffffffu, ok, 0) != 0;
}
__device__ __forceinline__ void x_stage_done(const XRing& R, int it, int lane) {
    tc_fence_proxy_async();   // the generic-proxy writes are visible to the tensor core
    __syncwarp();
    if (lane == 0) tc_mbar_arrive(R.full(it));
}

// a lane's 16 bytes of a chunk pair (one phase: both chunks; two phases: only its own 8 bytes, in .x and .y)
__device__ __forceinline__ uint4 ld_pair(const uint8_t* p) {
    if (kPhases == 2) {
        const uint2 v = ldg_nc64(p);
        return make_uint4(v.x, v.y, 0u, 0u);
    }
    return ldg_nc(p);
}

struct DeqIQ2 {              // IQ2_XXS rt32 layout (common.cuh); sign words re-encoded by the packer
    static constexpr bool kTables = true;
    uint32_t gtbl, stbl;     // shared-memory tables (set in the kernel)
    // 8 fp16 of one 8-element group: each pair's magnitudes by prmt from {h8, h25, h43}, then its signs by xor.  A
    // 128-bit table entry per grid index (selectors) and per sign index (masks), 8 copies so that the 8 lanes of a
    // quarter-warp read 8 different bank groups.
    __device__ __forceinline__ uint4 group(uint32_t P0, uint32_t P1, uint32_t gi, uint32_t si, uint32_t lane8) const {
        const uint4 sel = lds128(gtbl + ((gi << 7) | lane8));
        const uint4 sg = lds128(stbl + ((si << 7) | lane8));
        return make_uint4(prmt(P0, P1, sel.x) ^ sg.x, prmt(P0, P1, sel.y) ^ sg.y, prmt(P0, P1, sel.z) ^ sg.z,
                          prmt(P0, P1, sel.w) ^ sg.w);
    }
    __device__ __forceinline__ void chunk(uint32_t qx, uint32_t qy, float d, uint32_t row_addr, int lane) const {
        const uint32_t s4 = ((qy >> 7) & 1u) | ((qy >> 14) & 2u) | ((qy >> 21) & 4u) | ((qy >> 28) & 8u);
        // (float)s4 without a conversion instruction: s4 in the mantissa of 2^23, minus 2^23 (exact)
        const float fs4 = __uint_as_float(0x4B000000u | s4) - 8388608.f;
        const float db = d * (0.5f + fs4) * 0.25f;
        const uint32_t P0 = h2u(__floats2half2_rn(8.f * db, 25.f * db));
        const uint32_t P1 = h2u(__floats2half2_rn(43.f * db, 0.f));
        const int sw = (lane >> 1) & 3;
        const uint32_t lane8 = (uint32_t)(lane & 7) << 4;
#pragma unroll
        for (int g = 0; g < 4; g++)
            sts128(row_addr + (uint32_t)((g ^ sw) << 4), group(P0, P1, (qx >> (8 * g)) & 255u, (qy >> (8 * g)) & 127u, lane8));
    }
    // the stages kk = phase, phase + 2, ... of one tile for the rows of row tile rt of the group's matrix wm (n x K);
    // stage kk is ring iteration it0 + kk.  valid: rt's rows exist.
    __device__ bool run(const XRing& R, int it0, const uint8_t* wm, int K, int rt, bool valid, int wd, int phase,
                        int lane) const {
        const int nb = K >> 8;
        const uint8_t* base = wm + (size_t)rt * nb * kIq2Unit + lane * 16 + (kPhases == 2 ? phase * 8 : 0);
        // this lane's chunk pairs j of the current / next super-block (with two phases only chunk 2j + phase)
        uint4 c[4], n[4];
        uint32_t dc = 0, dn = 0;
        if (valid) {
#pragma unroll
            for (int j = 0; j < 4; j++) c[j] = ld_pair(base + j * 512);
            dc = ldg_u16(wm + (size_t)rt * nb * kIq2Unit + 2048 + lane * 2);
        }
        for (int sb = 0; sb < nb; sb++) {
            if (valid && sb + 1 < nb) {
                const uint8_t* u = base + (size_t)(sb + 1) * kIq2Unit;
#pragma unroll
                for (int j = 0; j < 4; j++) n[j] = ld_pair(u + j * 512);
                dn = ldg_u16(wm + ((size_t)rt * nb + sb + 1) * kIq2Unit + 2048 + lane * 2);
            }
            const float d = __half2float(__ushort_as_half((unsigned short)dc));
#pragma unroll
            for (int j = 0; j < 4; j++) {
#pragma unroll
                for (int hh = 0; hh < 2 / kPhases; hh++) {
                    const int ch = kPhases == 2 ? 2 * j + phase : 2 * j + hh;
                    const int it = it0 + sb * 8 + ch;
                    if (!x_wait_free(R, it, lane)) return false;
                    const uint32_t row_addr = R.stage(it) + 2 * kXRec + (uint32_t)((wd * 32 + lane) * 64);
                    if (valid) {
                        if (hh == 0) chunk(c[j].x, c[j].y, d, row_addr, lane);
                        else chunk(c[j].z, c[j].w, d, row_addr, lane);
                    } else {
#pragma unroll
                        for (int g = 0; g < 4; g++) sts128(row_addr + g * 16, make_uint4(0, 0, 0, 0));
                    }
                    x_stage_done(R, it, lane);
                }
            }
#pragma unroll
            for (int j = 0; j < 4; j++) c[j] = n[j];
            dc = dn;
        }
        return true;
    }
};

// Q8_0 prompt layout ("q8 tc"): units (32-row tile t, 32-k block kb) of 1088 B, [32 lanes][32 int8] then [32] fp16 d,
// at (t * K/32 + kb) * 1088 -- a warp's step over one 32-k block reads 1088 contiguous bytes.
constexpr int kQ8Unit = 1088;
struct DeqQ8 {
    static constexpr bool kTables = false;
    uint32_t gtbl, stbl;
    // 0x64XX as fp16 is 1024 + XX exactly; with the int8's sign bit flipped XX = q + 128, so minus 1152 gives q exactly,
    // and one fp16 multiply by d rounds q * d once
    __device__ __forceinline__ static uint32_t pair(uint32_t x, uint32_t sel, __half2 d2) {
        const __half2 mg = __half2half2(__ushort_as_half((unsigned short)0x6480));   // 1152
        const uint32_t b = prmt(x, 0x64646464u, sel);
        const __half2 q = __hsub2(*reinterpret_cast<const __half2*>(&b), mg);
        return h2u(__hmul2(q, d2));
    }
    __device__ __forceinline__ static uint4 quad(uint32_t w0, uint32_t w1, __half2 d2) {
        const uint32_t x0 = w0 ^ 0x80808080u, x1 = w1 ^ 0x80808080u;
        return make_uint4(pair(x0, 0x4140u, d2), pair(x0, 0x4342u, d2), pair(x1, 0x4140u, d2), pair(x1, 0x4342u, d2));
    }
    // the stages kk = phase, phase + 2, ... of one tile (32-k blocks), prefetched three of this warp's blocks ahead
    __device__ bool run(const XRing& R, int it0, const uint8_t* wm, int K, int rt, bool valid, int wd, int phase,
                        int lane) const {
        const int nk = K >> 5;   // a multiple of 8
        const uint8_t* base = wm + (size_t)rt * nk * kQ8Unit;
        uint4 qa[4], qb[4];
        uint32_t dd[4];
        if (valid) {
#pragma unroll
            for (int u = 0; u < 3; u++) {
                const uint8_t* p = base + (size_t)(kPhases * u + phase) * kQ8Unit;
                qa[u] = ldg_nc(p + lane * 32);
                qb[u] = ldg_nc(p + lane * 32 + 16);
                dd[u] = ldg_u16(p + 1024 + lane * 2);
            }
        }
        for (int m0 = 0; m0 < nk / kPhases; m0 += 4) {
#pragma unroll
            for (int u = 0; u < 4; u++) {
                const int m = m0 + u, kb = kPhases * m + phase, nx = m + 3;
                if (valid && nx < nk / kPhases) {   // prefetch this warp's block m + 3 into its ring slot
                    const uint8_t* p = base + (size_t)(kPhases * nx + phase) * kQ8Unit;
                    qa[(u + 3) & 3] = ldg_nc(p + lane * 32);
                    qb[(u + 3) & 3] = ldg_nc(p + lane * 32 + 16);
                    dd[(u + 3) & 3] = ldg_u16(p + 1024 + lane * 2);
                }
                const int it = it0 + kb;
                if (!x_wait_free(R, it, lane)) return false;
                const uint32_t row_addr = R.stage(it) + 2 * kXRec + (uint32_t)((wd * 32 + lane) * 64);
                const int sw = (lane >> 1) & 3;
                if (valid) {
                    const __half2 d2 = __half2half2(__ushort_as_half((unsigned short)dd[u]));
                    sts128(row_addr + (uint32_t)((0 ^ sw) << 4), quad(qa[u].x, qa[u].y, d2));
                    sts128(row_addr + (uint32_t)((1 ^ sw) << 4), quad(qa[u].z, qa[u].w, d2));
                    sts128(row_addr + (uint32_t)((2 ^ sw) << 4), quad(qb[u].x, qb[u].y, d2));
                    sts128(row_addr + (uint32_t)((3 ^ sw) << 4), quad(qb[u].z, qb[u].w, d2));
                } else {
#pragma unroll
                    for (int g = 0; g < 4; g++) sts128(row_addr + g * 16, make_uint4(0, 0, 0, 0));
                }
                x_stage_done(R, it, lane);
            }
        }
        return true;
    }
};

// ---------------------------------------------------------------------------------------------------------
// the GEMM
// ---------------------------------------------------------------------------------------------------------
template <class Deq, class Epi>
__global__ void __launch_bounds__(kXThreads, 1) tcx_gemm_k(XArgs a, Epi epi) {
    extern __shared__ __align__(1024) unsigned char x_dyn[];
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const uint32_t raw = (uint32_t)__cvta_generic_to_shared(x_dyn);
    XRing R;
    R.sbase = (raw + 1023u) & ~1023u;
    const uint32_t gtbl = R.sbase + kXStages * kXStage, stbl = gtbl + kGridTbl;
    R.bars = stbl + kSignTbl;
    const uint32_t acc_full = R.bars + 8u * XRing::kBars, acc_empty = acc_full + 8u, drain = acc_full + 16u;
    const uint32_t tmem_slot = acc_full + 24u;
    unsigned char* tmem_slot_ptr = x_dyn + (tmem_slot - raw);

    if (Deq::kTables) {
        // grid selectors: entry g, copy c at (g * 8 + c) * 16: for each pair p of elements (2p, 2p + 1) the prmt
        // selector of their fp16 magnitudes out of {h8, h25, h43} (bytes 0-1, 2-3, 4-5)
        for (int i = tid; i < 256 * 8; i += kXThreads) {
            const unsigned long long gr = iq2xxs_grid[i >> 3];
            uint32_t w[4];
#pragma unroll
            for (int p = 0; p < 4; p++) {
                const uint32_t m0 = (uint32_t)((gr >> (16 * p)) & 255), m1 = (uint32_t)((gr >> (16 * p + 8)) & 255);
                const uint32_t a0 = m0 == 8 ? 0u : m0 == 25 ? 2u : 4u, a1 = m1 == 8 ? 0u : m1 == 25 ? 2u : 4u;
                w[p] = a0 | (a0 + 1) << 4 | a1 << 8 | (a1 + 1) << 12;
            }
            sts128(gtbl + (uint32_t)i * 16u, make_uint4(w[0], w[1], w[2], w[3]));
        }
        // sign masks: sign index i, copy c: for each pair p the fp16x2 sign bits of elements 2p (bit 15), 2p + 1 (bit 31)
        for (int i = tid; i < 128 * 8; i += kXThreads) {
            const uint32_t s = ksigns_iq2xs[i >> 3];
            uint32_t w[4];
#pragma unroll
            for (int p = 0; p < 4; p++) w[p] = ((s >> (2 * p)) & 1u) << 15 | ((s >> (2 * p + 1)) & 1u) << 31;
            sts128(stbl + (uint32_t)i * 16u, make_uint4(w[0], w[1], w[2], w[3]));
        }
    }
    if (tid == 0) {
        for (int s = 0; s < kXStages; s++) { tc_mbar_init(R.full(s), 1 + kDeqWarps / kPhases); tc_mbar_init(R.empty(s), 1); }
        tc_mbar_init(acc_full, 1);
        tc_mbar_init(acc_empty, kXEpiWarps);
        tc_mbar_init(drain, 1);
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    }
    if (warp == 1) {
        asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(tmem_slot), "r"(kXTmemCols));
        asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;");
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = *reinterpret_cast<volatile uint32_t*>(tmem_slot_ptr);
    pdl_wait();

    const int NT = (a.N + kXN - 1) / kXN, KK = a.K / 32;
    const int mtiles = a.tiles ? min(*a.ntiles, a.max_mtiles) : a.max_mtiles;
    const int total = mtiles * NT;

    if (warp == 0) {
        // rows producer: one lane bulk-copies each stage's A records
        if (lane == 0) {
            bool healthy = true;
            int it = 0;
            for (int L = blockIdx.x; L < total && healthy; L += gridDim.x) {
                const int4 t = x_tile(a, L / NT);
                const int halves = t.w > kXM ? 2 : 1;
                const uint8_t* a0 = a.a + (size_t)t.y * KK * kXRec;
                for (int kk = 0; kk < KK; kk++, it++) {
                    const int use = it / kXStages;
                    if (use > 0 && !tc_mbar_wait(R.empty(it), (uint32_t)((use - 1) & 1))) { healthy = false; break; }
                    const uint32_t st = R.stage(it);
                    tc_mbar_arrive_tx(R.full(it), (uint32_t)(halves * kXRec));
                    tc_bulk_g2s(st, a0 + (size_t)kk * kXRec, (uint32_t)kXRec, R.full(it));
                    if (halves == 2) tc_bulk_g2s(st + kXRec, a0 + ((size_t)KK + kk) * kXRec, (uint32_t)kXRec, R.full(it));
                }
            }
            // the copies of the last uses of every stage have landed before the CTA may exit
            for (int i = it - kXStages > 0 ? it - kXStages : 0; i < it; i++)
                if (!tc_mbar_wait(R.full(i), (uint32_t)((i / kXStages) & 1))) healthy = false;
            if (!healthy) atomicOr(&g_tc_error, 1);
        }
        __syncwarp();
    } else if (warp == 1) {
        // MMA issuer
        if (lane == 0) {
            bool healthy = true;
            int it = 0, tl = 0;
            for (int L = blockIdx.x; L < total && healthy; L += gridDim.x, tl++) {
                const int4 t = x_tile(a, L / NT);
                const uint32_t idesc = t.w > kXM ? kIdescF16N256 : kIdescF16N128;   // tokens: the MMAs' N
                const bool w2 = (L % NT) * kXN + kXM < a.N;                         // the second weight half exists
                if (tl > 0 && !tc_mbar_wait(acc_empty, (uint32_t)((tl - 1) & 1))) { healthy = false; break; }
                tc_fence_after();
                for (int kk = 0; kk < KK; kk++, it++) {
                    if (!tc_mbar_wait(R.full(it), (uint32_t)((it / kXStages) & 1))) { healthy = false; break; }
                    tc_fence_after();
                    const uint32_t st = R.stage(it), bt = st + 2 * kXRec;
                    if constexpr (Epi::kTokensM) {
                        // M = 128 tokens (A record h), N = the 256 weight rows of the B tile
#pragma unroll
                        for (int ki = 0; ki < 2; ki++)
                            umma_f16(tmem, umma_desc_sw64(st + ki * 32), umma_desc_sw64(bt + ki * 32), kIdescF16N256,
                                     (kk | ki) ? 1u : 0u);
                        if (t.w > kXM) {
#pragma unroll
                            for (int ki = 0; ki < 2; ki++)
                                umma_f16(tmem + 256u, umma_desc_sw64(st + kXRec + ki * 32), umma_desc_sw64(bt + ki * 32),
                                         kIdescF16N256, (kk | ki) ? 1u : 0u);
                        }
                    } else {
                        // M = 128 weight rows (half h of the B tile), N = the tile's tokens (both A records, contiguous)
#pragma unroll
                        for (int ki = 0; ki < 2; ki++)
                            umma_f16(tmem, umma_desc_sw64(bt + ki * 32), umma_desc_sw64(st + ki * 32), idesc, (kk | ki) ? 1u : 0u);
                        if (w2) {
#pragma unroll
                            for (int ki = 0; ki < 2; ki++)
                                umma_f16(tmem + 256u, umma_desc_sw64(bt + kXRec + ki * 32), umma_desc_sw64(st + ki * 32), idesc,
                                         (kk | ki) ? 1u : 0u);
                        }
                    }
                    umma_commit(R.empty(it));
                }
                if (healthy) umma_commit(acc_full);
            }
            // every MMA this thread issued has completed before the TMEM is freed
            umma_commit(drain);
            if (!tc_mbar_wait(drain, 0)) healthy = false;
            if (!healthy) atomicOr(&g_tc_error, 1);
        }
        __syncwarp();
    } else if (warp < 2 + kDeqWarps) {
        // dequantisers: warp 2 + 8 phase + wd owns weight rows 32 wd .. 32 wd + 31 of the even (phase 0) or odd
        // (phase 1) stages of every tile
        const int wd = (warp - 2) & 7, phase = (warp - 2) >> 3;   // phase 0 with one set
        Deq dq;
        dq.gtbl = gtbl;
        dq.stbl = stbl;
        int it0 = 0;
        for (int L = blockIdx.x; L < total; L += gridDim.x, it0 += KK) {
            const int4 t = x_tile(a, L / NT);
            const int n0 = (L % NT) * kXN + wd * 32;
            const uint8_t* wm = a.w + (size_t)t.x * a.wstride;
            if (!dq.run(R, it0, wm, a.K, n0 >> 5, n0 < a.N, wd, phase, lane)) {
                if (lane == 0) atomicOr(&g_tc_error, 1);
                break;
            }
        }
    } else {
        // epilogue: warp w reads TMEM lanes 32 (w % 4).. of accumulator h; kEpiParts warps share an (h, lane quarter),
        // each a contiguous part of its column blocks
        const int e = warp - 2 - kDeqWarps, q = warp & 3, h = (e >> 2) & 1, cpart = e >> 3;
        int tl = 0;
        for (int L = blockIdx.x; L < total; L += gridDim.x, tl++) {
            const int4 t = x_tile(a, L / NT);
            const int n = (L % NT) * kXN + h * kXM + q * 32 + lane;   // the lane's weight row (weights as M)
            if (!tc_mbar_wait(acc_full, (uint32_t)(tl & 1))) {
                if (lane == 0) atomicOr(&g_tc_error, 1);
                break;
            }
            tc_fence_after();
            if constexpr (Epi::kTokensM) {
                // lanes are tokens 128 h + 32 q + lane; columns the tile's weight rows, 8 blocks of 32 (split by part)
                const int r = q * 32 + lane, n0 = (L % NT) * kXN;
                const int cb0 = cpart * (8 / kEpiParts), cb1 = cb0 + 8 / kEpiParts;
                if (h == 0 || t.w > kXM) {
                    const bool row_ok = h * kXM + r < t.w;
#pragma unroll 1
                    for (int cb = cb0; cb < cb1; cb++) {
                        uint32_t v[32];
                        tmem_ld32(tmem + ((uint32_t)(q * 32) << 16) + (uint32_t)(h * 256 + cb * 32), v);
                        tmem_ld_wait();
                        if (cb == cb1 - 1) {
                            tc_fence_before();
                            __syncwarp();
                            if (lane == 0) tc_mbar_arrive(acc_empty);   // the accumulators may be overwritten now
                        }
                        const int col = n0 + cb * 32;
                        if (row_ok && col < a.N) epi.put(t, h, r, col, a.N, v);
                    }
                } else {
                    tc_fence_before();
                    __syncwarp();
                    if (lane == 0) tc_mbar_arrive(acc_empty);
                }
            } else {
                // lanes are weight rows; this warp's 32-token column blocks [cb0, cb1) of the tile's 8 (4 for a tile of
                // at most 128 tokens)
                const int nblk = t.w > kXM ? 8 : 4;
                const int cb0 = min(cpart * (8 / kEpiParts), nblk), cb1 = min(cb0 + 8 / kEpiParts, nblk);
                if ((L % NT) * kXN + h * kXM < a.N && cb0 < cb1) {
#pragma unroll 1
                    for (int cb = cb0; cb < cb1; cb++) {
                        uint32_t v[32];
                        tmem_ld32(tmem + ((uint32_t)(q * 32) << 16) + (uint32_t)(h * 256 + cb * 32), v);
                        tmem_ld_wait();
                        if (cb == cb1 - 1) {
                            tc_fence_before();
                            __syncwarp();
                            if (lane == 0) tc_mbar_arrive(acc_empty);   // the accumulators may be overwritten now
                        }
                        if (cb * 32 < t.w && n < a.N) epi.put(t, n, cb * 32, lane, v);
                    }
                } else {
                    tc_fence_before();
                    __syncwarp();
                    if (lane == 0) tc_mbar_arrive(acc_empty);
                }
            }
        }
    }
    tc_fence_before();
    __syncthreads();
    if (warp == 1) {
        tc_fence_after();
        asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(kXTmemCols));
    }
    pdl_trigger();
}

static int x_num_sms() {
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

template <class Deq, class Epi>
static cudaError_t launch_x(const XArgs& a, const Epi& epi, cudaStream_t s) {
    static bool opted = false;
    if (!opted) {
        const cudaError_t e = cudaFuncSetAttribute(tcx_gemm_k<Deq, Epi>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)kXSmem);
        if (e != cudaSuccess) return e;
        opted = true;
    }
    const long long work = (long long)a.max_mtiles * ((a.N + kXN - 1) / kXN);
    const int grid = (int)(work < x_num_sms() ? work : x_num_sms());
    if (grid <= 0) return cudaSuccess;
    return launch(tcx_gemm_k<Deq, Epi>, dim3(grid), dim3(kXThreads), kXSmem, s, a, epi);
}

// ---------------------------------------------------------------------------------------------------------
// rows images, tile tables, packing
// ---------------------------------------------------------------------------------------------------------
// rows image from activation rows.  Grouped (slots != nullptr): slot s = {expert e, local slot j}, row r is pair
// offsets[e] + 128 j + r of the expert-sorted list (if it exists), source row order[pair] / div.  Dense: slot s row r
// is source row 128 s + r (if < T).  Missing rows are zeros.  A thread converts 8 k.
__global__ void rows_image_k(const void* __restrict__ x, int dtype, int ldx, int K, int T, const int2* __restrict__ slots,
                             const int* __restrict__ nslots, int max_slots, const int* __restrict__ counts,
                             const int* __restrict__ offsets, const int* __restrict__ order, int div,
                             uint8_t* __restrict__ img) {
    pdl_wait();
    const int per = K >> 3;
    const size_t i = (size_t)blockIdx.x * blockDim.x + threadIdx.x;
    const int limit = slots ? min(*nslots, max_slots) : max_slots;
    if (i < (size_t)limit * kXM * per) {
        const int c8 = (int)(i % per);
        const int r = (int)((i / per) % kXM);
        const int s = (int)(i / ((size_t)per * kXM));
        int src = -1;
        if (slots) {
            const int2 sl = slots[s];
            const int local = sl.y * kXM + r;
            if (local < counts[sl.x]) src = order[offsets[sl.x] + local] / div;
        } else {
            const int row = s * kXM + r;
            if (row < T) src = row;
        }
        uint4 v = make_uint4(0, 0, 0, 0);
        if (src >= 0) {
            if (dtype == B200Q_BF16) {
                const uint4 u = __ldg(reinterpret_cast<const uint4*>(reinterpret_cast<const __nv_bfloat16*>(x) + (size_t)src * ldx + c8 * 8));
                const uint32_t uw[4] = {u.x, u.y, u.z, u.w};
                uint32_t o[4];
#pragma unroll
                for (int j = 0; j < 4; j++) o[j] = h2u(__floats2half2_rn(__uint_as_float(uw[j] << 16), __uint_as_float(uw[j] & 0xffff0000u)));
                v = make_uint4(o[0], o[1], o[2], o[3]);
            } else {
                const float4* f = reinterpret_cast<const float4*>(reinterpret_cast<const float*>(x) + (size_t)src * ldx + c8 * 8);
                const float4 f0 = __ldg(f), f1 = __ldg(f + 1);
                v = make_uint4(h2u(__floats2half2_rn(f0.x, f0.y)), h2u(__floats2half2_rn(f0.z, f0.w)),
                               h2u(__floats2half2_rn(f1.x, f1.y)), h2u(__floats2half2_rn(f1.z, f1.w)));
            }
        }
        *reinterpret_cast<uint4*>(img + ((size_t)s * (K / 32) + c8 / 4) * kXRec + sw64_off(r, c8 & 3)) = v;
    }
    pdl_trigger();
}

// tiles and slots of the grouped launch from the per-expert counts (one block): tiles[] = {e, first slot, first row,
// rows} in expert order, slots[] = {e, j}; meta = {tiles, slots}
__global__ void moe_tiles_k(const int* __restrict__ counts, int E, int4* __restrict__ tiles, int2* __restrict__ slots,
                            int* __restrict__ meta) {
    pdl_wait();
    __shared__ int s_t[512], s_s[512];
    const int e = threadIdx.x;
    const int c = e < E ? counts[e] : 0;
    const int nt = (c + 2 * kXM - 1) / (2 * kXM), ns = (c + kXM - 1) / kXM;
    s_t[e] = nt;
    s_s[e] = ns;
    __syncthreads();
    for (int off = 1; off < 512; off <<= 1) {   // inclusive scans
        const int a = e >= off ? s_t[e - off] : 0, b = e >= off ? s_s[e - off] : 0;
        __syncthreads();
        s_t[e] += a;
        s_s[e] += b;
        __syncthreads();
    }
    const int tb = s_t[e] - nt, sb = s_s[e] - ns;
    for (int i = 0; i < nt; i++) tiles[tb + i] = make_int4(e, sb + 2 * i, 2 * kXM * i, min(2 * kXM, c - 2 * kXM * i));
    for (int j = 0; j < ns; j++) slots[sb + j] = make_int2(e, j);
    if (e == 511) { meta[0] = s_t[511]; meta[1] = s_s[511]; }
    pdl_trigger();
}

// act image -> pair-indexed rows act[pair][F] fp16 (for inspection)
__global__ void act_rows_k(const uint8_t* __restrict__ img, int F, const int2* __restrict__ slots, const int* __restrict__ nslots,
                           int max_slots, const int* __restrict__ counts, const int* __restrict__ offsets,
                           const int* __restrict__ order, __half* __restrict__ act) {
    pdl_wait();
    const int per = F >> 3;
    const size_t i = (size_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (i < (size_t)min(*nslots, max_slots) * kXM * per) {
        const int c8 = (int)(i % per), r = (int)((i / per) % kXM), s = (int)(i / ((size_t)per * kXM));
        const int2 sl = slots[s];
        const int local = sl.y * kXM + r;
        if (local < counts[sl.x]) {
            const int pair = order[offsets[sl.x] + local];
            *reinterpret_cast<uint4*>(act + (size_t)pair * F + c8 * 8) =
                *reinterpret_cast<const uint4*>(img + ((size_t)s * (F / 32) + c8 / 4) * kXRec + sw64_off(r, c8 & 3));
        }
    }
    pdl_trigger();
}

// Q8_0 ggml blocks [n][k/32][34] -> the q8 tc layout; a thread moves one block
__global__ void q8_tc_pack_k(const uint8_t* __restrict__ raw, uint8_t* __restrict__ out, int64_t n, int k) {
    pdl_wait();
    const int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
    const int nb = k / 32;
    if (i < n * nb) {
        const int64_t row = i / nb;
        const int kb = (int)(i % nb);
        const uint8_t* blk = raw + (size_t)i * 34;
        uint8_t* u = out + ((size_t)(row >> 5) * nb + kb) * kQ8Unit;
        const int l = (int)(row & 31);
        u[1024 + 2 * l] = blk[0];
        u[1024 + 2 * l + 1] = blk[1];
        for (int j = 0; j < 32; j++) u[l * 32 + j] = blk[2 + j];
    }
    pdl_trigger();
}

static inline bool x16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15) == 0; }
static inline size_t x_align(size_t v) { return (v + 255) & ~(size_t)255; }

struct MoeWs {               // workspace of b200q_moe_prompt
    size_t tiles, slots, meta, aimg, actimg, total;
    int max_tiles, max_slots;
};
static MoeWs moe_ws(int pairs, int E, int H, int F) {
    MoeWs w{};
    w.max_tiles = pairs / (2 * kXM) + E;
    w.max_slots = pairs / kXM + E;
    w.tiles = 0;
    w.slots = x_align(w.tiles + (size_t)w.max_tiles * sizeof(int4));
    w.meta = x_align(w.slots + (size_t)w.max_slots * sizeof(int2));
    w.aimg = x_align(w.meta + 16);
    w.actimg = x_align(w.aimg + (size_t)w.max_slots * (H / 32) * kXRec);
    w.total = x_align(w.actimg + (size_t)w.max_slots * (F / 32) * kXRec);
    return w;
}

}  // namespace b200q

using namespace b200q;

extern "C" {

size_t b200q_q8_tc_bytes(int64_t n, int k) {
    if (n <= 0 || n % 32 || k <= 0 || k % 256) return 0;
    return (size_t)n * (k / 32) * 34;
}

int b200q_q8_tc_pack(const void* raw, void* packed, int64_t n, int k, void* stream) {
    if (!raw || !packed || n <= 0 || n % 32 || k <= 0 || k % 256 || !x16(packed)) return B200Q_EINVAL;
    const int64_t th = n * (k / 32);
    return status_from(launch(q8_tc_pack_k, dim3((unsigned)((th + 255) / 256)), dim3(256), 0, (cudaStream_t)stream,
                              (const uint8_t*)raw, (uint8_t*)packed, n, k));
}

size_t b200q_q8_gemm_workspace_bytes(int T, int k) {
    if (T <= 0 || k <= 0 || k % 256) return 0;
    return (size_t)((T + 2 * kXM - 1) / (2 * kXM)) * 2 * (k / 32) * kXRec;
}

int b200q_q8_gemm(const void* w, int n, int k, const void* x, int x_dtype, int ldx, int T, float* y, int ldy, void* workspace,
                  size_t workspace_bytes, void* stream) {
    if (!w || !x || !y || n <= 0 || n % 32 || k <= 0 || k % 256 || T <= 0 || ldx < k || ldy < n ||
        (x_dtype != B200Q_F32 && x_dtype != B200Q_BF16) || !x16(w) || !x16(x) || (ldx % 8) || !workspace || !x16(workspace))
        return B200Q_EINVAL;
    if (workspace_bytes < b200q_q8_gemm_workspace_bytes(T, k)) return B200Q_ENOSPACE;
    cudaStream_t s = (cudaStream_t)stream;
    const int mt = (T + 2 * kXM - 1) / (2 * kXM);
    const size_t th = (size_t)mt * 2 * kXM * (k / 8);
    cudaError_t e = launch(rows_image_k, dim3((unsigned)((th + 255) / 256)), dim3(256), 0, s, x, x_dtype, ldx, k, T,
                           (const int2*)nullptr, (const int*)nullptr, 2 * mt, (const int*)nullptr, (const int*)nullptr,
                           (const int*)nullptr, 1, (uint8_t*)workspace);
    if (e != cudaSuccess) return status_from(e);
    XArgs a{};
    a.w = (const uint8_t*)w;
    a.a = (const uint8_t*)workspace;
    a.N = n;
    a.K = k;
    a.max_mtiles = mt;
    a.T = T;
    return status_from(launch_x<DeqQ8>(a, EpiRows{y, ldy, nullptr, nullptr}, s));
}

size_t b200q_moe_prompt_workspace_bytes(int pairs, int E, int H, int F) {
    if (pairs <= 0 || E <= 0 || H <= 0 || F <= 0 || H % 256 || F % 256) return 0;
    return moe_ws(pairs, E, H, F).total;
}

int b200q_moe_prompt(const void* up, const void* down, int E, int H, int F, const int* counts, const int* offsets,
                     const int* order, int topk, int pairs, const void* x, int x_dtype, float* mo, void* act_rows,
                     void* workspace, size_t workspace_bytes, void* stream) {
    if (!up || !down || !counts || !offsets || !order || !x || !mo || !workspace || E <= 0 || E > 512 || topk <= 0 ||
        pairs <= 0 || H % 256 || F % 256 || H <= 0 || F <= 0 || (x_dtype != B200Q_F32 && x_dtype != B200Q_BF16) ||
        !x16(up) || !x16(down) || !x16(x) || !x16(workspace) || (act_rows && !x16(act_rows)))
        return B200Q_EINVAL;
    const MoeWs L = moe_ws(pairs, E, H, F);
    if (workspace_bytes < L.total) return B200Q_ENOSPACE;
    cudaStream_t s = (cudaStream_t)stream;
    uint8_t* ws = (uint8_t*)workspace;
    int4* tiles = (int4*)(ws + L.tiles);
    int2* slots = (int2*)(ws + L.slots);
    int* meta = (int*)(ws + L.meta);
    uint8_t* aimg = ws + L.aimg;
    uint8_t* actimg = ws + L.actimg;

    cudaError_t e = launch(moe_tiles_k, dim3(1), dim3(512), 0, s, counts, E, tiles, slots, meta);
    if (e != cudaSuccess) return status_from(e);
    size_t th = (size_t)L.max_slots * kXM * (H / 8);
    e = launch(rows_image_k, dim3((unsigned)((th + 255) / 256)), dim3(256), 0, s, x, x_dtype, H, H, 0, (const int2*)slots,
               (const int*)(meta + 1), L.max_slots, counts, offsets, order, topk, aimg);
    if (e != cudaSuccess) return status_from(e);

    XArgs a{};
    a.w = (const uint8_t*)up;
    a.wstride = iq2_bytes(F, H);
    a.a = aimg;
    a.N = F;
    a.K = H;
    a.tiles = tiles;
    a.ntiles = meta;
    a.max_mtiles = L.max_tiles;
    e = launch_x<DeqIQ2>(a, EpiImg{actimg, F}, s);
    if (e != cudaSuccess) return status_from(e);
    if (act_rows) {
        th = (size_t)L.max_slots * kXM * (F / 8);
        e = launch(act_rows_k, dim3((unsigned)((th + 255) / 256)), dim3(256), 0, s, (const uint8_t*)actimg, F,
                   (const int2*)slots, (const int*)(meta + 1), L.max_slots, counts, offsets, order, (__half*)act_rows);
        if (e != cudaSuccess) return status_from(e);
    }
    a.w = (const uint8_t*)down;
    a.wstride = iq2_bytes(H, F);
    a.a = actimg;
    a.N = H;
    a.K = F;
    return status_from(launch_x<DeqIQ2>(a, EpiRows{mo, H, offsets, order}, s));
}

}  // extern "C"
