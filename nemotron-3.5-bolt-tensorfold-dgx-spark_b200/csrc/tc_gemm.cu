// Prompt-length GEMMs of the IQ2_XXS experts and the Q8_0 projections on the sm_100a tensor cores: tcgen05.mma
// kind::f16 (fp16 operands, fp32 accumulation in TMEM), the weights dequantised inside the kernel, on SM pairs.
//
// C[n][m] = sum_k W[n][k] X[m][k]: W the weight rows (the MMA's M), X the activation rows (tokens, or the
// expert-sorted pairs of the MoE; the MMA's N).  A cluster of two CTAs computes a pair tile of 256 weight rows x 256
// rows (128 for a tile of at most 128 rows) with tcgen05.mma.cta_group::2 m256n256k16: CTA r of the pair holds
// weight rows 128 r .. 128 r + 127 (its half of A) and X rows 128 r .. (its half of B, 64 rows for N = 128), and its
// TMEM holds the accumulator of its 128 weight rows x all N columns.  So every SM dequantises 128 weight rows that
// feed 256 rows, each SM's tensor core reads only half of the B tile from its own shared memory, and the accumulator
// (256 columns) is double-buffered in the SM's 512 TMEM columns: the epilogue drains one tile while the MMAs of the
// next fill the other buffer.  Per 64-k stage of a 5-stage ring in each CTA (32 KB, identical offsets in both), two
// 32-k blocks of each operand:
//   X        the CTA's X rows (2 x 8 KB, or 2 x 4 KB for N = 128), bulk-copied (cp.async.bulk, no tensor map, one
//            destination) from an fp16 rows image by one lane of warp 0;
//   W        the CTA's 128 weight rows x 64 k in fp16, written by 16 dequantising warps in four sets of 4 that take
//            the stages in turn (warp w of a set: rows 32w..32w+31, lane = row), from the packed weights, which each
//            lane prefetches into registers ahead of use.  IQ2_XXS: a prmt picks every fp16 pair out of its chunk's
//            three scaled magnitudes and a xor sets its signs, the selectors and masks read as 128-bit entries from
//            replicated shared-memory tables (conflict-free).  Q8_0: a magic-number prmt makes the int8 exact in fp16
//            and one hmul2 applies the scale;
//   MMA      one lane of the leader CTA's warp 1 waits until both CTAs' stages are full, issues the four m256 MMAs
//            of the stage and commits them to both CTAs' "empty" barriers (a tcgen05.commit to each); in the peer CTA
//            warp 1 relays "stage full" to the leader (a remote mbarrier arrive);
//   epilogue 8 warps a CTA drain their accumulator buffer (tcgen05.ld: warp w reads lane quarter w % 4, half of the
//            columns), release it to the leader, and write the outputs.
// Pair tiles are handed out persistently, one cluster per SM pair.
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
//   Q8_0   W = fp16(q * d), the scale folded and rounded once.
//   IQ2    W = fp16(d (0.5 + s4) / 4 * signed grid), rounded once.  (FP8 cannot hold the grid magnitudes 25 and 43.)
//   X      activations rounded to fp16 once; the MoE's intermediate act = fp16(relu(v)^2).
// Every barrier wait is bounded (%globaltimer); on a timeout the kernel records an error (b200q_device_error bit 4),
// waits for its own copies and MMAs, frees its TMEM and returns.  Every copy has one destination, its own CTA.
#include "tcgen05.cuh"

namespace b200q {

constexpr int kXM = 128;                        // rows of a slot, and weight rows of a CTA
constexpr int kXN = 256;                        // weight rows of a pair tile
constexpr int kXRec = kXM * 64;                 // 8 KB: a rows-image record (128 rows x 32 fp16)
constexpr int kXStage = 4 * kXRec;              // 32 KB: the CTA's X rows (two 32-k blocks), then its W rows (two)
constexpr int kXWOff = 2 * kXRec;               // the W blocks' offset in a stage
#ifndef B200Q_TC_COPIES
#define B200Q_TC_COPIES 8
#endif
#ifndef B200Q_TC_IQ2_STAGES
#define B200Q_TC_IQ2_STAGES 5
#endif
constexpr int kDeqWarps = 16, kXEpiWarps = 8;   // dequantisers (4 a stage, in kPhases sets taking stages in turn)
constexpr int kPhases = kDeqWarps / 4;
constexpr int kXThreads = (2 + kDeqWarps + kXEpiWarps) * 32;   // 832
// shared memory of a CTA: the ring, the dequantiser's tables, alignment slack and the barriers
template <class Deq>
constexpr size_t x_smem() { return (size_t)Deq::kStages * kXStage + Deq::kTableBytes + 1024 + 256; }
constexpr uint32_t kXTmemCols = 512;            // two 256-column accumulator buffers
static_assert(kPhases == 4, "the dequantisers' chunk assignment assumes four sets");

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

// instruction descriptors, kind::f16: fp32 accumulator, fp16 A and B, both K-major, M = 256 (a CTA pair), N = 256 / 128
constexpr uint32_t kIdesc2N256 = (1u << 4) | (256u >> 3) << 17 | (256u >> 4) << 24;
constexpr uint32_t kIdesc2N128 = (1u << 4) | (128u >> 3) << 17 | (256u >> 4) << 24;

// one m256 MMA of a CTA pair, issued by the leader: A and B descriptors address the same offsets in both CTAs
__device__ __forceinline__ void umma2_f16(uint32_t tmem_d, uint64_t a, uint64_t b, uint32_t idesc, uint32_t accumulate) {
    asm volatile(
        "{ .reg .pred p; setp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::2.kind::f16 [%0], %1, %2, %3, {%5, %6, %7, %8, %9, %10, %11, %12}, p; }"
        ::"r"(tmem_d), "l"(a), "l"(b), "r"(idesc), "r"(accumulate), "r"(0), "r"(0), "r"(0), "r"(0), "r"(0), "r"(0),
          "r"(0), "r"(0));
}
// the completion of the leader's MMAs so far arrives on the barrier at `bar` (a shared::cluster address: the
// leader's own barrier, or the peer's from peer_addr); the leader commits to each CTA's copy of a barrier in turn
__device__ __forceinline__ void umma2_commit(uint32_t bar) {
    asm volatile("tcgen05.commit.cta_group::2.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(bar) : "memory");
}
__device__ __forceinline__ uint32_t cluster_rank() {
    uint32_t r;
    asm volatile("mov.u32 %0, %%cluster_ctarank;" : "=r"(r));
    return r;
}
// the shared::cluster address of `addr` (a shared::cta address) in the CTA of rank `rank`
__device__ __forceinline__ uint32_t peer_addr(uint32_t addr, uint32_t rank) {
    uint32_t r;
    asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(r) : "r"(addr), "r"(rank));
    return r;
}
// an arrive on the other CTA's barrier (default semantics: no cluster-wide fence before it, which would stall the
// relay a round trip per stage)
__device__ __forceinline__ void mbar_arrive_cluster(uint32_t cluster_addr) {
    asm volatile("mbarrier.arrive.shared::cluster.b64 _, [%0];" ::"r"(cluster_addr) : "memory");
}
__device__ __forceinline__ void cluster_sync_all() {
    asm volatile("barrier.cluster.arrive.release.aligned;\n\tbarrier.cluster.wait.acquire.aligned;" ::: "memory");
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

// Epilogues.  put(t, n, tok0, lane, v): v[j] = (weight row n, the lane's; row tok0 + j of the tile); the 32 lanes of
// a warp hold 32 consecutive weight rows, so every row's outputs from one warp are one contiguous line.
struct EpiRows {             // fp32 y[orow][n]; orow = rowmap[row0[g] + m0 + row] (or the dense row)
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
struct EpiRows16 {           // EpiRows with bf16 outputs (rounded to nearest even): a 64-byte line a row
    __nv_bfloat16* y;
    int ldy;
    const int* row0;
    const int* rowmap;
    __device__ void put(int4 t, int n, int tok0, int lane, const uint32_t (&v)[32]) const {
        const int grow = (row0 ? row0[t.x] : 0) + t.z + tok0 + lane;
        const int mine = tok0 + lane < t.w ? (rowmap ? rowmap[grow] : grow) : -1;
        __nv_bfloat16* yn = y + n;
#pragma unroll
        for (int j = 0; j < 32; j++) {
            const int orow = __shfl_sync(0xffffffffu, mine, j);
            if (orow >= 0) yn[(size_t)orow * ldy] = __float2bfloat16_rn(__uint_as_float(v[j]));
        }
    }
};
struct EpiImg {              // fp16(relu(v)^2) into the next GEMM's rows image (its K = this GEMM's N): for each row
    // the warp's 32 weight rows are one 64-byte row of a record (2 bytes a lane)
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
// W dequantisers.  run() produces its phase's stages of one tile for the calling warp's 32 rows (lane = row): for
// each of those 32-k blocks it waits for the stage to be free, writes the row's 64 B, and arrives on the stage's "full"
// barrier.
// ---------------------------------------------------------------------------------------------------------
template <int S>
struct XRing {               // stage bookkeeping shared by the warps of one CTA: S stages
    static constexpr int kStages = S;
    uint32_t sbase, bars;
    __device__ uint32_t full(int it) const { return bars + 8u * (it % S); }
    __device__ uint32_t empty(int it) const { return bars + 8u * (S + it % S); }
    __device__ uint32_t stage(int it) const { return sbase + (uint32_t)((it % S) * kXStage); }
    static constexpr int kBars = 2 * S;
};

// waits (lane 0) for the stage of iteration `it` to be free; false on a timeout (warp-uniform)
template <class Ring>
__device__ __forceinline__ bool x_wait_free(const Ring& R, int it, int lane) {
    const int use = it / Ring::kStages;
    int ok = 1;
    if (use > 0 && lane == 0) ok = tc_mbar_wait(R.empty(it), (uint32_t)((use - 1) & 1)) ? 1 : 0;
    return __shfl_sync(0xffffffffu, ok, 0) != 0;
}
template <class Ring>
__device__ __forceinline__ void x_stage_done(const Ring& R, int it, int lane) {
    tc_fence_proxy_async();   // the generic-proxy writes are visible to the tensor core
    __syncwarp();
    if (lane == 0) tc_mbar_arrive(R.full(it));
}

struct DeqIQ2 {              // IQ2_XXS rt32 layout (common.cuh); sign words re-encoded by the packer
    static constexpr bool kTables = true;
    static constexpr int kCopies = B200Q_TC_COPIES;            // replicas of each table entry
    static constexpr int kGridTbl = 256 * kCopies * 16;       // grid entry -> four prmt selectors
    static constexpr int kSignTbl = 128 * kCopies * 16;       // sign index -> four xor masks
    static constexpr int kTableBytes = kGridTbl + kSignTbl;
    static constexpr int kStages = B200Q_TC_IQ2_STAGES;
    uint32_t gtbl, stbl;     // shared-memory tables (set in the kernel)
    // 8 fp16 of one 8-element group: each pair's magnitudes by prmt from {h8, h25, h43}, then its signs by xor.  A
    // 128-bit table entry per grid index (selectors) and per sign index (masks), kCopies copies so that the lanes of a
    // quarter-warp read different bank groups.
    __device__ __forceinline__ uint4 group(uint32_t P0, uint32_t P1, uint32_t gi, uint32_t si, uint32_t lane8) const {
        const uint4 sel = lds128(gtbl + ((gi * kCopies) << 4 | lane8));
        const uint4 sg = lds128(stbl + ((si * kCopies) << 4 | lane8));
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
        const uint32_t lane8 = (uint32_t)(lane & (kCopies - 1)) << 4;
#pragma unroll
        for (int g = 0; g < 4; g++)
            sts128(row_addr + (uint32_t)((g ^ sw) << 4), group(P0, P1, (qx >> (8 * g)) & 255u, (qy >> (8 * g)) & 127u, lane8));
    }
    // the stages kk = phase, phase + 4, ... of one tile for the rows of row tile rt of the group's matrix wm (n x K):
    // stage kk (64 k) is chunk pair kk & 3 of super-block kk >> 2, so this warp reads chunk pair `phase` (16 bytes)
    // of every super-block, two super-blocks ahead of use.  Stage kk is ring iteration it0 + kk.  valid: rt's rows
    // exist.
    template <class Ring>
    __device__ bool run(const Ring& R, int it0, const uint8_t* wm, int K, int rt, bool valid, int wd, int phase,
                        int lane) const {
        const int nb = K >> 8;
        const uint8_t* unit0 = wm + (size_t)rt * nb * kIq2Unit;
        const uint32_t o = (uint32_t)(phase * 512 + lane * 16);
        uint4 c = make_uint4(0, 0, 0, 0), m = c, n = c;
        uint32_t dc = 0, dm = 0, dn = 0;
        if (valid) {
            c = ldg_nc(unit0 + o);
            dc = ldg_u16(unit0 + 2048 + lane * 2);
            if (nb > 1) {
                m = ldg_nc(unit0 + kIq2Unit + o);
                dm = ldg_u16(unit0 + kIq2Unit + 2048 + lane * 2);
            }
        }
        for (int sb = 0; sb < nb; sb++) {
            if (valid && sb + 2 < nb) {
                const uint8_t* u = unit0 + (size_t)(sb + 2) * kIq2Unit;
                n = ldg_nc(u + o);
                dn = ldg_u16(u + 2048 + lane * 2);
            }
            const float d = __half2float(__ushort_as_half((unsigned short)dc));
            const int it = it0 + sb * 4 + phase;
            if (!x_wait_free(R, it, lane)) return false;
            const uint32_t row_addr = R.stage(it) + kXWOff + (uint32_t)((wd * 32 + lane) * 64);
            if (valid) {
                chunk(c.x, c.y, d, row_addr, lane);
                chunk(c.z, c.w, d, row_addr + kXRec, lane);
            } else {
#pragma unroll
                for (int g = 0; g < 4; g++) {
                    sts128(row_addr + g * 16, make_uint4(0, 0, 0, 0));
                    sts128(row_addr + kXRec + g * 16, make_uint4(0, 0, 0, 0));
                }
            }
            x_stage_done(R, it, lane);
            c = m;
            dc = dm;
            m = n;
            dm = dn;
        }
        return true;
    }
};

// Q8_0 prompt layout ("q8 tc"): units (32-row tile t, 32-k block kb) of 1088 B, [32 lanes][32 int8] then [32] fp16 d,
// at (t * K/32 + kb) * 1088 -- a warp's step over one 32-k block reads 1088 contiguous bytes.
constexpr int kQ8Unit = 1088;
struct DeqQ8 {
    static constexpr bool kTables = false;
    static constexpr int kCopies = 1, kGridTbl = 0, kSignTbl = 0, kTableBytes = 0;
    static constexpr int kStages = 7;
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
    __device__ __forceinline__ static void put_block(uint32_t row_addr, uint4 qa, uint4 qb, uint32_t d, int lane) {
        const int sw = (lane >> 1) & 3;
        const __half2 d2 = __half2half2(__ushort_as_half((unsigned short)d));
        sts128(row_addr + (uint32_t)((0 ^ sw) << 4), quad(qa.x, qa.y, d2));
        sts128(row_addr + (uint32_t)((1 ^ sw) << 4), quad(qa.z, qa.w, d2));
        sts128(row_addr + (uint32_t)((2 ^ sw) << 4), quad(qb.x, qb.y, d2));
        sts128(row_addr + (uint32_t)((3 ^ sw) << 4), quad(qb.z, qb.w, d2));
    }
    // the stages kk = phase, phase + 4, ... of one tile (64 k: 32-k blocks 2kk, 2kk + 1), each prefetched one of
    // this warp's stages (four stages) ahead (two would not fit the registers of an 832-thread CTA)
    template <class Ring>
    __device__ bool run(const Ring& R, int it0, const uint8_t* wm, int K, int rt, bool valid, int wd, int phase,
                        int lane) const {
        constexpr int kAhead = 1, kRing = kAhead + 1;
        const int nm = (K >> 6) / kPhases;   // this warp's stages (K % 256 == 0: at least 1)
        const uint8_t* base = wm + (size_t)rt * (K >> 5) * kQ8Unit + lane * 32;
        const uint8_t* dbase = wm + (size_t)rt * (K >> 5) * kQ8Unit + 1024 + lane * 2;
        uint4 qa[kRing][2], qb[kRing][2];
        uint32_t dd[kRing][2];
        auto fetch = [&](int slot, int mm) {
#pragma unroll
            for (int h = 0; h < 2; h++) {
                const size_t off = (size_t)(2 * (kPhases * mm + phase) + h) * kQ8Unit;
                qa[slot][h] = ldg_nc(base + off);
                qb[slot][h] = ldg_nc(base + off + 16);
                dd[slot][h] = ldg_u16(dbase + off);
            }
        };
#pragma unroll
        for (int u = 0; u < kAhead; u++) {
            if (valid && u < nm) fetch(u, u);
        }
        for (int m0 = 0; m0 < nm; m0 += kRing) {
#pragma unroll
            for (int u = 0; u < kRing; u++) {
                const int m = m0 + u;
                if (m >= nm) break;
                if (valid && m + kAhead < nm) fetch((u + kAhead) % kRing, m + kAhead);
                const int it = it0 + kPhases * m + phase;
                if (!x_wait_free(R, it, lane)) return false;
                const uint32_t row_addr = R.stage(it) + kXWOff + (uint32_t)((wd * 32 + lane) * 64);
                if (valid) {
                    put_block(row_addr, qa[u][0], qb[u][0], dd[u][0], lane);
                    put_block(row_addr + kXRec, qa[u][1], qb[u][1], dd[u][1], lane);
                } else {
#pragma unroll
                    for (int g = 0; g < 4; g++) {
                        sts128(row_addr + g * 16, make_uint4(0, 0, 0, 0));
                        sts128(row_addr + kXRec + g * 16, make_uint4(0, 0, 0, 0));
                    }
                }
                x_stage_done(R, it, lane);
            }
        }
        return true;
    }
};

// ---------------------------------------------------------------------------------------------------------
// the GEMM: one cluster of two CTAs per SM pair
// ---------------------------------------------------------------------------------------------------------
template <class Deq, class Epi>
__global__ void __cluster_dims__(2, 1, 1) __launch_bounds__(kXThreads, 1) tcx_gemm_k(XArgs a, Epi epi) {
    extern __shared__ __align__(1024) unsigned char x_dyn[];
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const uint32_t rank = cluster_rank();   // 0: the leader, which issues the pair's MMAs; 1: the peer
    const uint32_t raw = (uint32_t)__cvta_generic_to_shared(x_dyn);
    constexpr int kXStages = Deq::kStages;
    using Ring = XRing<kXStages>;
    Ring R;
    R.sbase = (raw + 1023u) & ~1023u;
    const uint32_t gtbl = R.sbase + kXStages * kXStage, stbl = gtbl + Deq::kGridTbl;
    R.bars = stbl + Deq::kSignTbl;
    const uint32_t acc_full = R.bars + 8u * Ring::kBars;   // [2]
    const uint32_t acc_empty = acc_full + 16u;              // [2], arrived on in the leader by both CTAs' epilogues
    const uint32_t drain = acc_full + 32u, tmem_slot = acc_full + 40u;
    unsigned char* tmem_slot_ptr = x_dyn + (tmem_slot - raw);

    if (Deq::kTables) {
        // grid selectors: entry g, copy c at (g * 8 + c) * 16: for each pair p of elements (2p, 2p + 1) the prmt
        // selector of their fp16 magnitudes out of {h8, h25, h43} (bytes 0-1, 2-3, 4-5)
        for (int i = tid; i < 256 * Deq::kCopies; i += kXThreads) {
            const unsigned long long gr = iq2xxs_grid[i / Deq::kCopies];
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
        for (int i = tid; i < 128 * Deq::kCopies; i += kXThreads) {
            const uint32_t s = ksigns_iq2xs[i / Deq::kCopies];
            uint32_t w[4];
#pragma unroll
            for (int p = 0; p < 4; p++) w[p] = ((s >> (2 * p)) & 1u) << 15 | ((s >> (2 * p + 1)) & 1u) << 31;
            sts128(stbl + (uint32_t)i * 16u, make_uint4(w[0], w[1], w[2], w[3]));
        }
    }
    if (tid == 0) {
        // full: this CTA's producer (arrive + bytes) and the stage's 4 dequantising warps, and in the leader the peer's
        // relay; empty, acc_full, drain: one commit of the leader's MMAs; acc_empty (used in the leader): both CTAs'
        // epilogue warps
        for (int s = 0; s < kXStages; s++) {
            tc_mbar_init(R.full(s), 1 + 4 + (rank == 0 ? 1 : 0));
            tc_mbar_init(R.empty(s), 1);
        }
        for (int b = 0; b < 2; b++) {
            tc_mbar_init(acc_full + 8u * b, 1);
            tc_mbar_init(acc_empty + 8u * b, 2 * kXEpiWarps);
        }
        tc_mbar_init(drain, 1);
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    }
    if (warp == 1) {
        // both CTAs' warp 1 take the pair's TMEM: 512 columns in each SM
        asm volatile("tcgen05.alloc.cta_group::2.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(tmem_slot), "r"(kXTmemCols));
        asm volatile("tcgen05.relinquish_alloc_permit.cta_group::2.sync.aligned;");
    }
    tc_fence_before();
    __syncthreads();
    cluster_sync_all();   // both CTAs' barriers exist before either arrives on the other's
    tc_fence_after();
    const uint32_t tmem = *reinterpret_cast<volatile uint32_t*>(tmem_slot_ptr);
    pdl_wait();

    const int NT = (a.N + kXN - 1) / kXN, KK = a.K / 64;   // 64-k stages a tile
    const int mtiles = a.tiles ? min(*a.ntiles, a.max_mtiles) : a.max_mtiles;
    const int total = mtiles * NT;
    const int cl = (int)(blockIdx.x >> 1), ncl = (int)(gridDim.x >> 1);

    if (warp == 0) {
        // X producer: one lane bulk-copies this CTA's rows of each stage (its 128-row slot, or half of the tile's one
        // slot when the tile has at most 128 rows): the two 32-k records of a stage are adjacent in the image
        if (lane == 0) {
            bool healthy = true;
            int it = 0;
            for (int L = cl; L < total && healthy; L += ncl) {
                const int4 t = x_tile(a, L / NT);
                const bool wide = t.w > kXM;
                const uint8_t* src = wide ? a.a + (size_t)(t.y + (int)rank) * (2 * KK) * kXRec
                                          : a.a + (size_t)t.y * (2 * KK) * kXRec + rank * (kXRec / 2);
                for (int kk = 0; kk < KK; kk++, it++) {
                    const int use = it / kXStages;
                    if (use > 0 && !tc_mbar_wait(R.empty(it), (uint32_t)((use - 1) & 1))) { healthy = false; break; }
                    const uint8_t* blk = src + (size_t)(2 * kk) * kXRec;
                    if (wide) {
                        tc_mbar_arrive_tx(R.full(it), 2u * kXRec);
                        tc_bulk_g2s(R.stage(it), blk, 2u * kXRec, R.full(it));
                    } else {
                        tc_mbar_arrive_tx(R.full(it), (uint32_t)kXRec);
                        tc_bulk_g2s(R.stage(it), blk, (uint32_t)(kXRec / 2), R.full(it));
                        tc_bulk_g2s(R.stage(it) + kXRec, blk + kXRec, (uint32_t)(kXRec / 2), R.full(it));
                    }
                }
            }
            // every stage's last release (the leader's commits land in this CTA's barriers too) before the CTA may exit
            for (int i = it - kXStages > 0 ? it - kXStages : 0; i < it; i++)
                if (!tc_mbar_wait(R.empty(i), (uint32_t)((i / kXStages) & 1))) healthy = false;
            if (!healthy) atomicOr(&g_tc_error, 1);
        }
        __syncwarp();
    } else if (warp == 1) {
        if (lane == 0) {
            bool healthy = true;
            if (rank == 0) {
                // MMA issuer: per stage four m256 MMAs (k 16 each) into the tile's accumulator buffer
                const uint32_t p_empty0 = peer_addr(R.empty(0), 1), p_acc_full = peer_addr(acc_full, 1);
                int it = 0, tl = 0;
                for (int L = cl; L < total && healthy; L += ncl, tl++) {
                    const int4 t = x_tile(a, L / NT);
                    const uint32_t idesc = t.w > kXM ? kIdesc2N256 : kIdesc2N128;
                    const int b = tl & 1;
                    if (tl >= 2 && !tc_mbar_wait(acc_empty + 8u * b, (uint32_t)(((tl >> 1) - 1) & 1))) {
                        healthy = false;
                        break;
                    }
                    tc_fence_after();
                    const uint32_t dacc = tmem + (uint32_t)(b * 256);
                    for (int kk = 0; kk < KK; kk++, it++) {
                        if (!tc_mbar_wait(R.full(it), (uint32_t)((it / kXStages) & 1))) { healthy = false; break; }
                        tc_fence_after();
                        const uint32_t st = R.stage(it);
#pragma unroll
                        for (int ki = 0; ki < 4; ki++) {
                            const uint32_t o = (uint32_t)((ki >> 1) * kXRec + (ki & 1) * 32);
                            umma2_f16(dacc, umma_desc_sw64(st + kXWOff + o), umma_desc_sw64(st + o), idesc,
                                      (kk | ki) ? 1u : 0u);
                        }
                        umma2_commit(R.empty(it));
                        umma2_commit(p_empty0 + 8u * (uint32_t)(it % kXStages));
                    }
                    if (healthy) {
                        umma2_commit(acc_full + 8u * b);
                        umma2_commit(p_acc_full + 8u * b);
                    }
                }
                // the epilogues' last releases have landed before the leader may exit
                for (int j = tl - 2 > 0 ? tl - 2 : 0; j < tl && healthy; j++)
                    if (!tc_mbar_wait(acc_empty + 8u * (j & 1), (uint32_t)((j >> 1) & 1))) healthy = false;
                // every MMA issued has completed (and so no longer reads either CTA's stages) before TMEM is freed
                umma2_commit(drain);
                umma2_commit(peer_addr(drain, 1));
            } else {
                // relay: each stage of this CTA full (its X rows landed, its W rows written) -> the leader's barrier
                const uint32_t lead_full0 = peer_addr(R.full(0), 0);
                int it = 0;
                for (int L = cl; L < total && healthy; L += ncl)
                    for (int kk = 0; kk < KK; kk++, it++) {
                        if (!tc_mbar_wait(R.full(it), (uint32_t)((it / kXStages) & 1))) { healthy = false; break; }
                        mbar_arrive_cluster(lead_full0 + 8u * (uint32_t)(it % kXStages));
                    }
            }
            if (!tc_mbar_wait(drain, 0)) healthy = false;
            if (!healthy) atomicOr(&g_tc_error, 1);
        }
        __syncwarp();
    } else if (warp < 2 + kDeqWarps) {
        // dequantisers: warp 2 + 4 phase + wd owns this CTA's weight rows 32 wd .. 32 wd + 31 of the stages
        // kk = phase (mod 4) of every tile
        const int wd = (warp - 2) & 3, phase = (warp - 2) >> 2;
        Deq dq;
        dq.gtbl = gtbl;
        dq.stbl = stbl;
        int it0 = 0;
        for (int L = cl; L < total; L += ncl, it0 += KK) {
            const int4 t = x_tile(a, L / NT);
            const int n0 = (L % NT) * kXN + (int)rank * kXM + wd * 32;
            const uint8_t* wm = a.w + (size_t)t.x * a.wstride;
            if (!dq.run(R, it0, wm, a.K, n0 >> 5, n0 < a.N, wd, phase, lane)) {
                if (lane == 0) atomicOr(&g_tc_error, 1);
                break;
            }
        }
    } else {
        // epilogue: warp w reads TMEM lane quarter w % 4 (32 weight rows) and one half of the tile's 32-row column
        // blocks, from the tile's buffer; the last read releases the buffer to the leader's MMA
        const int e = warp - 2 - kDeqWarps, q = warp & 3, ch = e >> 2;
        const uint32_t lead_empty = rank == 0 ? 0u : peer_addr(acc_empty, 0);
        int tl = 0;
        for (int L = cl; L < total; L += ncl, tl++) {
            const int4 t = x_tile(a, L / NT);
            const int b = tl & 1;
            if (!tc_mbar_wait(acc_full + 8u * b, (uint32_t)((tl >> 1) & 1))) {
                if (lane == 0) atomicOr(&g_tc_error, 1);
                break;
            }
            tc_fence_after();
            const int nbase = (L % NT) * kXN + (int)rank * kXM;   // this CTA's first weight row
            const int n = nbase + q * 32 + lane;
            const int nblk = t.w > kXM ? 8 : 4, cb0 = ch * (nblk / 2), cb1 = cb0 + nblk / 2;
#pragma unroll 1
            for (int cb = cb0; cb < cb1; cb++) {
                uint32_t v[32];
                tmem_ld32(tmem + ((uint32_t)(q * 32) << 16) + (uint32_t)(b * 256 + cb * 32), v);
                tmem_ld_wait();
                if (cb == cb1 - 1) {
                    tc_fence_before();
                    __syncwarp();
                    if (lane == 0) {
                        if (rank == 0) tc_mbar_arrive(acc_empty + 8u * b);
                        else mbar_arrive_cluster(lead_empty + 8u * b);
                    }
                }
                if (nbase < a.N && cb * 32 < t.w && n < a.N) epi.put(t, n, cb * 32, lane, v);
            }
        }
    }
    tc_fence_before();
    __syncthreads();
    cluster_sync_all();   // neither CTA leaves while the other may still arrive on its barriers
    if (warp == 1) {
        tc_fence_after();
        asm volatile("tcgen05.dealloc.cta_group::2.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(kXTmemCols));
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

// SMs the persistent prompt GEMMs leave free on a device (b200q_set_sm_reserve): while a pipelined expert-parallel
// exchange runs, NCCL's kernels need SMs beside the GEMMs
static int g_sm_reserve[64];

template <class Deq, class Epi>
static cudaError_t launch_x(const XArgs& a, const Epi& epi, cudaStream_t s) {
    static int max_clusters = 0;   // SM pairs that can hold one cluster each
    if (!max_clusters) {
        const cudaError_t e = cudaFuncSetAttribute(tcx_gemm_k<Deq, Epi>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)x_smem<Deq>());
        if (e != cudaSuccess) return e;
        cudaLaunchConfig_t cfg = {};
        cfg.gridDim = dim3(2 * (x_num_sms() / 2));
        cfg.blockDim = dim3(kXThreads);
        cfg.dynamicSmemBytes = x_smem<Deq>();
        cudaLaunchAttribute at[1];
        at[0].id = cudaLaunchAttributeClusterDimension;
        at[0].val.clusterDim.x = 2;
        at[0].val.clusterDim.y = 1;
        at[0].val.clusterDim.z = 1;
        cfg.attrs = at;
        cfg.numAttrs = 1;
        int n = 0;
        if (cudaOccupancyMaxActiveClusters(&n, tcx_gemm_k<Deq, Epi>, &cfg) != cudaSuccess || n <= 0) {
            cudaGetLastError();
            n = x_num_sms() / 2;
        }
        max_clusters = n;
    }
    const long long work = (long long)a.max_mtiles * ((a.N + kXN - 1) / kXN);
    int dev = 0;
    cudaGetDevice(&dev);
    const int reserve = (dev >= 0 && dev < 64) ? g_sm_reserve[dev] : 0;
    const int avail = max_clusters - (reserve + 1) / 2 > 1 ? max_clusters - (reserve + 1) / 2 : 1;
    const int clusters = (int)(work < avail ? work : avail);
    if (clusters <= 0) return cudaSuccess;
    return launch(tcx_gemm_k<Deq, Epi>, dim3(2 * clusters), dim3(kXThreads), x_smem<Deq>(), s, a, epi);
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

extern "C" int b200q_set_sm_reserve(int sms) {
    int dev = 0;
    if (sms < 0 || sms > 128 || cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return B200Q_EINVAL;
    g_sm_reserve[dev] = sms;
    return B200Q_OK;
}

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
                     const int* order, int topk, int pairs, const void* x, int x_dtype, void* mo, int mo_dtype,
                     void* act_rows, void* workspace, size_t workspace_bytes, void* stream) {
    if (!up || !down || !counts || !offsets || !order || !x || !mo || !workspace || E <= 0 || E > 512 || topk <= 0 ||
        pairs <= 0 || H % 256 || F % 256 || H <= 0 || F <= 0 || (x_dtype != B200Q_F32 && x_dtype != B200Q_BF16) ||
        (mo_dtype != B200Q_F32 && mo_dtype != B200Q_BF16) ||
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
    if (mo_dtype == B200Q_BF16)
        return status_from(launch_x<DeqIQ2>(a, EpiRows16{(__nv_bfloat16*)mo, H, offsets, order}, s));
    return status_from(launch_x<DeqIQ2>(a, EpiRows{(float*)mo, H, offsets, order}, s));
}

}  // extern "C"
