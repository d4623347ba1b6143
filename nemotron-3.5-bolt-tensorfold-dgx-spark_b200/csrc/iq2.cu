// IQ2_XXS on sm_100a: the load-time packer, the synthetic generator and the HBM-streaming GEMVs over int8
// activation rows (dense, and grouped by expert for the routed MoE).
//
// Arithmetic (the routed-expert kernels moe_mma_k / moe_coop_k of the reference, bolt_kernels.cu:445-483 and
// 599-652): a row's 32-weight chunk holds four grid-index bytes, four 7-bit sign indices and a 4-bit sub-scale s4.
// Its weights are the signed grid integers (iq2xxs_grid bytes, negated where ksigns_iq2xs says); the chunk's exact
// int32 dot with the int8 activation row is scaled by dA * s, dA = d * (0.5 + s4) * 0.25 = (d / 8) * (2 s4 + 1)
// (both forms are exact in fp32) and s the row's activation scale of that chunk, and accumulated in chunk order:
// acc = fma(dA * s, (float)dot, acc).
//
// Mapping: a lane owns one weight row and walks K in order, so every output is the reference's own chunk-ordered
// sum, reproducible bit for bit by a scalar loop.  A warp owns 32 rows of one expert ("slot") and up to 3 of the
// slot's tokens: a work unit (at three, not four, the units of the 16-token shared expert no longer outlast the
// routed experts' second wave of units).  CTAs are persistent (one of 24 warps per SM); warps take units from a global counter
// as they go, the slots with the most tokens first, so the expensive units start early and every warp stays busy
// until the last units are handed out.
//
// Streaming: the (32-row tile, 256-k super-block) pieces of the layout are contiguous 2112-byte units, so each warp
// runs its own ring of kStages shared-memory stages filled by TMA bulk copies (cp.async.bulk, completion on an
// mbarrier): a stage holds one super-block of the warp's 32 rows plus the matching 256 bytes of int8 activations and
// 32 bytes of scales of each of the unit's tokens.  Lane 0 keeps kStages - 1 stages in flight across unit boundaries;
// every lane reads its row's 16-byte chunk pairs from the stage and every token's activation words as shared-memory
// broadcasts.  Waits are bounded (%globaltimer): on a timeout the kernel sets an error flag, lets its own copies
// land and returns.
//
// Dequantisation without bank conflicts: a 64 KB table in shared memory gives, per lane, its own copy of two 32-bit
// words for every grid index r: codes(r), the eight magnitude codes of grid entry r as nibbles (8 -> 0, 25 -> 1,
// 43 -> 2), and signs(r & 127), three times the eight sign bits of ksigns_iq2xs as nibbles.  The word of row r, lane
// l sits at r * 256 + l * 4 (+ 128 for signs): every lane reads its own bank, and one prmt turns a grid-index byte
// (or a sign-index byte) and the lane offset into the address.  codes + signs is a prmt selector into the six signed
// magnitudes {8, 25, 43, -8, -25, -43}: two prmt give eight int8 weights.  For the sign index to be a byte the packer
// re-encodes ggml's sign word (four 7-bit fields, s4 in bits 28-31) as four bytes, byte g = field g | bit g of s4 << 7;
// the spare top bit selects the table's second, identical half of sign words.
#include "iq2.cuh"
#include "moe.cuh"

#include <atomic>
#include <cstring>

namespace b200q {

// ---------------------------------------------------------------------------------------------------------
// small portable helpers (host and device give the same bits)
// ---------------------------------------------------------------------------------------------------------
__host__ __device__ inline uint64_t splitmix64(uint64_t x) {
    x += 0x9E3779B97F4A7C15ull;
    x = (x ^ (x >> 30)) * 0xBF58476D1CE4E5B9ull;
    x = (x ^ (x >> 27)) * 0x94D049BB133111EBull;
    return x ^ (x >> 31);
}

// float -> IEEE half bits, round to nearest even, for normal positive inputs below 65504 (the generator's range)
__host__ __device__ inline uint16_t f2h_bits_pos(float f) {
#ifdef __CUDA_ARCH__
    const uint32_t u = __float_as_uint(f);
#else
    uint32_t u;
    memcpy(&u, &f, 4);
#endif
    const int e = (int)((u >> 23) & 255) - 127;   // f = 1.m * 2^e
    uint32_t mant = (u & 0x7fffffu) | 0x800000u;  // 24 bits
    if (e < -14) {                                // half subnormal: multiples of 2^-24
        const int sh = -e - 14 + 13;
        const uint32_t q = mant >> sh, rem = mant & ((1u << sh) - 1), half = 1u << (sh - 1);
        return (uint16_t)(q + ((rem > half || (rem == half && (q & 1))) ? 1 : 0));
    }
    uint32_t q = mant >> 13;
    const uint32_t rem = mant & 0x1fffu;
    if (rem > 0x1000u || (rem == 0x1000u && (q & 1))) q++;
    int ee = e + 15;
    if (q == 0x800u) { q = 0x400u; ee++; }
    return (uint16_t)(((uint32_t)ee << 10) | (q & 0x3ffu));
}

// One ggml IQ2_XXS block of the synthetic distribution: d ~ U[1e-3, 1e-2] (fp16), grid indices U{0..255},
// sign indices U{0..127}, sub-scales U{0..15}.  Block i depends on (seed, i) only.
__host__ __device__ inline void synth_iq2_block(uint64_t seed, uint64_t i, uint8_t* b) {
    uint64_t h = splitmix64(seed ^ splitmix64(i * 0x100000001B3ull + 0x51ED27ull));
    const float u = (float)(h >> 40) * (1.f / 16777216.f);
    const uint16_t d = f2h_bits_pos(1e-3f + 9e-3f * u);
    b[0] = (uint8_t)(d & 255);
    b[1] = (uint8_t)(d >> 8);
    for (int c = 0; c < 8; c++) {
        h = splitmix64(h + (uint64_t)c);
        const uint32_t grid = (uint32_t)h;                 // four U{0..255} bytes
        const uint32_t aux = (uint32_t)(h >> 32);
        const uint32_t signs = aux & 0x0fffffffu;           // four U{0..127} fields
        const uint32_t s4 = (uint32_t)(splitmix64(h ^ 0xA5A5ull) & 15u);
        const uint32_t hi = signs | (s4 << 28);
        uint8_t* p = b + 2 + 8 * c;
        p[0] = (uint8_t)grid; p[1] = (uint8_t)(grid >> 8); p[2] = (uint8_t)(grid >> 16); p[3] = (uint8_t)(grid >> 24);
        p[4] = (uint8_t)hi; p[5] = (uint8_t)(hi >> 8); p[6] = (uint8_t)(hi >> 16); p[7] = (uint8_t)(hi >> 24);
    }
}

__global__ void synth_iq2_k(uint64_t seed, int64_t nblocks, uint8_t* __restrict__ out) {
    const int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (i < nblocks) synth_iq2_block(seed, (uint64_t)i, out + i * 66);
}

// ggml's sign word (four 7-bit sign indices, s4 in bits 28-31) -> four bytes: field g | (bit g of s4) << 7
__host__ __device__ inline uint32_t iq2_sign_bytes(uint32_t qy) {
    uint32_t r = 0;
    for (int g = 0; g < 4; g++) r |= ((((qy >> (7 * g)) & 127u) | (((qy >> (28 + g)) & 1u) << 7)) << (8 * g));
    return r;
}

// ---------------------------------------------------------------------------------------------------------
// packer: ggml blocks [n][k/256][66] -> rt32 units (see common.cuh), one thread per (row, chunk pair); the sign
// word of every chunk is re-encoded by iq2_sign_bytes
// ---------------------------------------------------------------------------------------------------------
// the split form: a unit's 2048 chunk bytes into qs (2048 a unit), its 32 rows' d into dq (64 bytes a unit)
__global__ void iq2_pack_split_k(const uint8_t* __restrict__ raw, uint8_t* __restrict__ qs, uint8_t* __restrict__ dq,
                                 int64_t n, int k) {
    pdl_wait();
    const int npair = k / 64, nb = k / 256;
    const int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (i < n * npair) {
        const int64_t row = i / npair;
        const int j = (int)(i - row * npair);
        const uint8_t* blk = raw + ((size_t)row * nb + j / 4) * 66;
        const uint8_t* src = blk + 2 + 16 * (j % 4);
        uint32_t w[4];
#pragma unroll
        for (int q = 0; q < 4; q++)
            w[q] = (uint32_t)src[4 * q] | (uint32_t)src[4 * q + 1] << 8 | (uint32_t)src[4 * q + 2] << 16 | (uint32_t)src[4 * q + 3] << 24;
        w[1] = iq2_sign_bytes(w[1]);
        w[3] = iq2_sign_bytes(w[3]);
        const int64_t rt = row / kIq2Tile;
        const int lane = (int)(row % kIq2Tile);
        const size_t unit = (size_t)rt * nb + j / 4;
        reinterpret_cast<uint4*>(qs + unit * 2048)[(j & 3) * kIq2Tile + lane] = make_uint4(w[0], w[1], w[2], w[3]);
        if ((j & 3) == 0) reinterpret_cast<uint16_t*>(dq + unit * 64)[lane] = (uint16_t)(blk[0] | blk[1] << 8);
    }
    pdl_trigger();
}

__global__ void iq2_pack_k(const uint8_t* __restrict__ raw, uint8_t* __restrict__ out, int64_t n, int k) {
    pdl_wait();
    const int npair = k / 64, nb = k / 256;
    const int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (i < n * npair) {
        const int64_t row = i / npair;
        const int j = (int)(i - row * npair);
        const uint8_t* blk = raw + ((size_t)row * nb + j / 4) * 66;
        const uint8_t* src = blk + 2 + 16 * (j % 4);
        uint32_t w[4];
#pragma unroll
        for (int q = 0; q < 4; q++)
            w[q] = (uint32_t)src[4 * q] | (uint32_t)src[4 * q + 1] << 8 | (uint32_t)src[4 * q + 2] << 16 | (uint32_t)src[4 * q + 3] << 24;
        w[1] = iq2_sign_bytes(w[1]);
        w[3] = iq2_sign_bytes(w[3]);
        const int64_t rt = row / kIq2Tile;
        const int lane = (int)(row % kIq2Tile);
        uint8_t* unit = out + ((size_t)rt * nb + j / 4) * kIq2Unit;
        reinterpret_cast<uint4*>(unit)[(j & 3) * kIq2Tile + lane] = make_uint4(w[0], w[1], w[2], w[3]);
        if ((j & 3) == 0) reinterpret_cast<uint16_t*>(unit + 2048)[lane] = (uint16_t)(blk[0] | blk[1] << 8);
    }
    pdl_trigger();
}

// ---------------------------------------------------------------------------------------------------------
// the GEMV
// ---------------------------------------------------------------------------------------------------------
constexpr int kGemvWarps = 24;              // one persistent CTA of 24 warps an SM (80 registers a thread)
constexpr int kStages = 2;                  // ring stages a warp (one super-block in flight while one is read)
constexpr int kUnitTok = kIq2UnitTok;       // most tokens a work unit dots
constexpr int kStageAct = kIq2Unit;                       // 2112: tokens' int8 rows (kUnitTok x 256 B)
constexpr int kStageScl = kStageAct + kUnitTok * 256;     // their scales (kUnitTok x 32 B)
constexpr int kStageBytes = kStageScl + kUnitTok * 32;    // 2976 at three tokens
constexpr int kMaxSlots = 520;
// Shared memory: the 64 KB table sits at the fixed shared address kTblAddr, so one prmt builds a lookup address
// (table base, index byte, lane offset) with no add.  Below it: the ring barriers, the slot counts and prefix, and
// the first stages; above it, the remaining stages.  The layout holds for a dynamic-memory base below 1 KB.
constexpr uint32_t kTblAddr = 0x10000;
constexpr int kQueue = kStages + 1;         // a warp's queue of units grabbed ahead (its producer is <= kStages ahead)
// barriers, slot counts / order / unit prefix, the warps' unit queues, the two magnitude words (8-byte aligned)
// the one-launch decode layer keeps its own schedule in shared memory: at most kLayerSlots slots and kLayerIds ids
// (pairs + shared-expert rows, also the most batches); larger layers take the three-launch path
constexpr int kLayerSlots = 257, kLayerIds = 512;
constexpr uint32_t kHdrBytes = kGemvWarps * kStages * 8 + (3 * kMaxSlots + 1) * 4 + kGemvWarps * kQueue * (3 + kUnitTok) * 4 +
                               (kLayerSlots + 1 + 2 * kLayerIds) * 4 + 12 + 16;
constexpr int kNumStages = kGemvWarps * kStages;
constexpr uint32_t kMaxDynBase = 1024;
constexpr int kStagesBelowMin = (int)((kTblAddr - kMaxDynBase - kHdrBytes - 16) / kStageBytes);
constexpr size_t kGemvSmem = (size_t)kTblAddr * 2 + (size_t)(kNumStages - kStagesBelowMin) * kStageBytes;
constexpr int kUnitCtrs = 64;               // launch slots of the unit counters (launches in flight at once)
constexpr unsigned long long kWaitNs = 2000000000ull;   // a ring stage not filled within 2 s: give up

enum Epi { kStore = 0, kRelu2 = 1, kRelu2Q8 = 2, kDots = 3 };

// bit 0: a ring wait timed out; bit 1: the shared-memory layout did not fit; bit 3: a fused launch's down unit
// waited more than 2 s for its batch's up rows; bit 4: a fused launch's batch order held an index out of range;
// bit 5: a wait of the one-launch decode layer (schedule, x's rows, the CTAs' units) gave up
__device__ int g_iq2_error;
#ifdef B200Q_X_TRACE
__device__ unsigned long long g_x_trace[160][16];   // per CTA: %globaltimer at the layer's phase points
#define XTRACE(i) do { if (threadIdx.x == 0) g_x_trace[blockIdx.x][i] = globaltimer(); } while (0)
#else
#define XTRACE(i) do { } while (0)
#endif
#ifdef B200Q_X_STATS
__device__ unsigned long long g_x_stats[4];   // pending waits, their ns, pending units taken, down units taken
#endif
// per launch slot: [0] the next unit to hand out, [1] the CTAs done (the last one resets the slot for its next
// launch), [6] set when a wait of the launch gave up (the other waits of the launch then give up at once); the
// one-launch decode layer also uses [4] the CTAs done quantising x and [5] the CTAs done with their units
__device__ int g_unit_ctr[kUnitCtrs][8];
// the one-launch decode layer's readiness counters per launch slot (one a batch), zero between the slot's launches
__device__ int g_layer_ready[kUnitCtrs][kLayerIds];

__device__ __forceinline__ uint32_t prmt(uint32_t a, uint32_t b, uint32_t s) {
    uint32_t d;
    asm("prmt.b32 %0, %1, %2, %3;" : "=r"(d) : "r"(a), "r"(b), "r"(s));
    return d;
}
__device__ __forceinline__ uint32_t lds32(uint32_t addr) {
    uint32_t v;
    asm volatile("ld.shared.u32 %0, [%1];" : "=r"(v) : "r"(addr));
    return v;
}
__device__ __forceinline__ uint4 lds128(uint32_t addr) {
    uint4 v;
    asm volatile("ld.shared.v4.u32 {%0,%1,%2,%3}, [%4];" : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w) : "r"(addr));
    return v;
}
__device__ __forceinline__ uint16_t lds16(uint32_t addr) {
    uint16_t v;
    asm volatile("ld.shared.u16 %0, [%1];" : "=h"(v) : "r"(addr));
    return v;
}
__device__ __forceinline__ unsigned long long globaltimer() {
    unsigned long long t;
    asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
    return t;
}
__device__ __forceinline__ void mbar_init(uint32_t bar, uint32_t count) {
    asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(bar), "r"(count) : "memory");
}
__device__ __forceinline__ void mbar_expect_tx(uint32_t bar, uint32_t bytes) {
    asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(bar), "r"(bytes) : "memory");
}
__device__ __forceinline__ bool mbar_try_wait(uint32_t bar, uint32_t parity) {
    uint32_t ok;
    asm volatile("{ .reg .pred p; mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2; selp.u32 %0, 1, 0, p; }"
                 : "=r"(ok) : "r"(bar), "r"(parity) : "memory");
    return ok != 0;
}
// bounded wait for a stage: false when it has not completed within `ns`
__device__ __forceinline__ bool mbar_wait(uint32_t bar, uint32_t parity, unsigned long long ns) {
    if (mbar_try_wait(bar, parity)) return true;
    const unsigned long long t0 = globaltimer();
    while (!mbar_try_wait(bar, parity))
        if (globaltimer() - t0 > ns) return false;
    return true;
}
// A weight copy, read once a step: marked to leave L2 first (an evict_first policy), so that the step's streamed
// weights do not push out what is read again (the code, the tables, the activation rows between the projections).
__device__ __forceinline__ uint64_t evict_first_policy() {
    uint64_t pol;
    asm volatile("createpolicy.fractional.L2::evict_first.b64 %0, 1.0;" : "=l"(pol));
    return pol;
}
__device__ __forceinline__ void bulk_g2s_stream(uint32_t dst, const void* src, uint32_t bytes, uint32_t bar, uint64_t pol) {
    asm volatile("cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes.L2::cache_hint [%0], [%1], %2, [%3], %4;"
                 ::"r"(dst), "l"(src), "r"(bytes), "r"(bar), "l"(pol) : "memory");
}
__device__ __forceinline__ void bulk_g2s(uint32_t dst, const void* src, uint32_t bytes, uint32_t bar) {
    asm volatile("cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];"
                 ::"r"(dst), "l"(src), "r"(bytes), "r"(bar) : "memory");
}

// the 64 KB table: row r (256 B) = [codes(r) x 32 lanes][signs(r & 127) x 32 lanes]
__device__ void build_table(uint32_t* tbl) {
    for (int i = threadIdx.x; i < 512; i += blockDim.x) {
        const int r = i & 255;
        uint32_t word = 0;
        if (i < 256) {
            const unsigned long long g = iq2xxs_grid[r];
#pragma unroll
            for (int j = 0; j < 8; j++) {
                const uint32_t mag = (uint32_t)(g >> (8 * j)) & 255u;
                word |= (mag == 8 ? 0u : mag == 25 ? 1u : 2u) << (4 * j);
            }
        } else {
            const uint32_t sg = ksigns_iq2xs[r & 127];
#pragma unroll
            for (int j = 0; j < 8; j++) word |= (((sg >> j) & 1u) * 3u) << (4 * j);
        }
        uint4* dst = reinterpret_cast<uint4*>(tbl + r * 64 + (i < 256 ? 0 : 32));
        const uint4 v = make_uint4(word, word, word, word);
#pragma unroll
        for (int q = 0; q < 8; q++) dst[q] = v;
    }
}

// the eight int8 weights of group g of a chunk (grid bytes qx, sign bytes qyp) as two words; lane_c = kTblAddr | lane*4,
// lane_s = lane_c | 128
__device__ __forceinline__ void group_weights(uint32_t lane_c, uint32_t lane_s, uint32_t qx, uint32_t qyp, int g,
                                              uint32_t& lo, uint32_t& hi) {
    // address = kTblAddr | (index byte << 8) | lane * 4 (| 128 for the sign half): bytes 0, 2, 3 from the lane word
    const uint32_t sel_b = 0x7604u | ((uint32_t)g << 4);
    const uint32_t ac = prmt(qx, lane_c, sel_b);
    const uint32_t as = prmt(qyp, lane_s, sel_b);
    const uint32_t sel = lds32(ac) + lds32(as);                // nibble j: code_j + 3 * sign_j, in 0..5
    lo = prmt(0xF82B1908u, 0x0000D5E7u, sel);                  // bytes 8, 25, 43, -8 | -25, -43
    hi = prmt(0xF82B1908u, 0x0000D5E7u, sel >> 16);
}

// Units: (slot s, token batch b0 of kUnitTok tokens, 32-row group g).  Every CTA orders the slots by token count,
// largest first, and numbers their units in that order (batch-major, then row group); warps take unit numbers from
// a global counter as they go, so the expensive units go first and the tail is short and shared by all warps.
//
// A fused launch runs two phases over the same slots and schedule: the up projection's units (ReLU^2 and the int8
// rows of the result), then the down projection's units over those rows.  A down unit of (slot, batch) needs the
// batch's up rows for every row group of the up output, so each up unit adds one to its batch's readiness counter
// once its rows are stored, and the producer of a down unit waits (bounded) for the counter to reach the up phase's
// row-group count before it issues the unit's first copy.  Units are handed out in order, so every up unit a down unit
// waits for is already held by a running warp, and nothing an up unit does waits on a down unit: the waits end.
struct Unit {
    int s, b0, g, nt, bidx;   // slot, first token, row group, tokens, the batch's index in schedule order
};

// The CTA's unit bookkeeping in shared memory: the slots by token count and the exclusive prefix of their batches.
struct Sched {
    const int *cnt, *order, *bpre;
    int nslots;
    int G, U;                // the (first) phase: row groups, units
    int G2, U2;              // a fused launch's down phase (U2 = 0 otherwise)
    const int* dorder;       // its order of batches
    const int* offs;         // the one-launch layer: the slots' offsets and the ids in slot order (shared memory;
    const int* ord;          // nullptr: read the arguments' offsets and order from global memory)
    uint32_t kc;             // shared address of the two words of signed magnitudes (prmt sources)
};

// unit u of a phase of G row groups
__device__ __forceinline__ Unit decode_unit(int u, const Sched& sc, int G) {
    int lo = 0, hi = sc.nslots;   // the last ordered slot whose first unit is <= u
    while (hi - lo > 1) {
        const int mid = (lo + hi) >> 1;
        if (sc.bpre[mid] * G <= u) lo = mid;
        else hi = mid;
    }
    Unit w;
    w.s = sc.order[lo];
    const int r = u - sc.bpre[lo] * G, b = r / G;
    w.bidx = sc.bpre[lo] + b;
    w.b0 = b * kUnitTok;
    w.g = r - b * G;
    w.nt = min(kUnitTok, sc.cnt[w.s] - w.b0);
    return w;
}

// A warp's ring: kStages shared-memory stages used in turn.  `slot` is the stage the warp reads next and `par` the
// parity of its barrier's next phase; consumed / issued count super-blocks (for the drain after a timeout, and for
// lane 0 to see that the ring ran empty).
struct Ring {
    uint32_t st[kStages];    // the stages' shared addresses
    uint32_t bar0;           // the first stage's barrier (the others 8 bytes apart)
    int slot, consumed, issued;
    uint32_t par;
    static_assert(kStages == 2 || kStages == 3, "stage() selects among two or three stages");
    __device__ __forceinline__ uint32_t stage_at(int sl) const {   // selects, so st stays in registers
        if constexpr (kStages == 2) return sl == 0 ? st[0] : st[1];
        else return sl == 0 ? st[0] : sl == 1 ? st[1] : st[2];
    }
    __device__ __forceinline__ uint32_t stage() const { return stage_at(slot); }
    __device__ __forceinline__ uint32_t bar() const { return bar0 + 8u * (uint32_t)slot; }
    __device__ __forceinline__ void advance() {
        consumed++;
        if (++slot == kStages) {
            slot = 0;
            par ^= 1u;
        }
    }
};

__device__ __forceinline__ const uint8_t* slot_weights(const GemvArgs& a, int s) {
    return (a.counts == nullptr || s < a.nslot_routed) ? a.slab + (size_t)s * a.expert_bytes : a.extra_w;
}

// A queue entry: the unit's row group (-1: no more units), its token count, its phase and batch index
// (phase | bidx << 1), then its token ids.
constexpr int kQEntry = 3 + kUnitTok;

__device__ __forceinline__ int ld_acquire(const int* p) {
    int v;
    asm volatile("ld.acquire.gpu.global.b32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
    return v;
}

// Lane 0's producer: takes units from the launch's counter, queues them for its warp (row group, token count, phase,
// ids), and fills the warp's ring with their super-blocks (weights, the tokens' int8 rows and, with kScl, their
// scales).  Every source pointer is set once a unit and advanced by a constant a stage.
//
// A fused launch's down unit whose batch is not complete when it is taken is `pending`: the producer issues nothing
// for it and never waits (its warp may still be reading an up unit that others wait for); the warp waits, bounded, only
// when its ring has run empty (force), when it holds no unfinished up unit.
template <bool kScl>
struct Producer {
    int* queue;              // this warp's kQueue entries of kQEntry ints
    int pn;                  // units grabbed
    int nt, left;            // the unit being issued: its tokens, and its super-blocks not yet issued (0: none)
    int pending;             // 1 + the batch index a pending down unit waits for, or 0
    bool split;              // its weights in the split layout
    const uint8_t* wsrc;     // its next super-block of weights
    const uint8_t* dsrc;     // the split layout: its next 64 bytes of d
    const int8_t* xq;        // its phase's int8 rows and scales
    const float* xs;
    int xoff[kUnitTok];      // element offsets of its tokens' next int8 blocks (from xq) and scales (from xs)
    int soff[kUnitTok];

    // the unit's queue entry and source pointers, from its phase's arguments
    __device__ __forceinline__ void fill(const GemvArgs& p, const Sched& sc, const Unit& w, int phase, int* e) {
        // offsets and order are read at L2 (cg): they may be taken before this grid waits for its predecessor
        const int base = sc.offs ? sc.offs[w.s] : p.counts ? __ldcg(p.offsets + w.s) : 0;
        e[0] = w.g;
        e[1] = w.nt;
        e[2] = phase | (w.bidx << 1);
#pragma unroll
        for (int m = 0; m < kUnitTok; m++) {
            const int mm = m < w.nt ? m : 0;
            const int id = sc.ord ? sc.ord[base + w.b0 + mm] : p.counts ? __ldcg(p.order + base + w.b0 + mm) : w.b0 + mm;
            const int arow = id < p.act_split ? id / p.act_div : id - p.act_split + p.act_base;
            e[3 + m] = id;
            xoff[m] = arow * p.k;
            if (kScl) soff[m] = arow * (p.k >> 5);
        }
        const size_t unit0 = (size_t)w.g * (p.k >> 8);   // the unit's first (tile, super-block)
        split = p.dplane != nullptr;
        if (split) {
            const bool routed = p.counts == nullptr || w.s < p.nslot_routed;   // as slot_weights
            wsrc = slot_weights(p, w.s) + unit0 * 2048;
            dsrc = (routed ? p.dplane + (size_t)w.s * p.dplane_stride : p.dplane_extra) + unit0 * 64;
        } else {
            wsrc = slot_weights(p, w.s) + unit0 * kIq2Unit;
        }
        xq = p.xq;
        xs = p.xs;
        nt = w.nt;
        left = p.k >> 8;
    }

    // A warp's first unit is fixed, warp w of CTA b taking unit w * gridDim + b (consecutive units, the heaviest
    // first, land on different SMs), so a launch does not open with every warp of the GPU contending for one
    // counter; the counter hands out the units after those.
    template <bool FUSED>
    __device__ __forceinline__ void grab(const GemvArgs& a, const GemvArgs& b, const Sched& sc, const int* ready,
                                         int ctr) {
        const int u = pn == 0 ? (int)(threadIdx.x >> 5) * (int)gridDim.x + (int)blockIdx.x
                              : (int)gridDim.x * kGemvWarps + atomicAdd(&g_unit_ctr[ctr][0], 1);
        int* e = queue + (pn % kQueue) * kQEntry;
        pn++;
        if (u >= sc.U + sc.U2) {
            // no units left for this warp: the next launch on the stream may be scheduled now (it still waits for
            // this grid's completion before it reads anything), so its CTAs build their tables during this tail
            pdl_trigger();
            e[0] = -1;
            left = 0;
            return;
        }
        if (!FUSED || u < sc.U) {
            fill(a, sc, decode_unit(u, sc, sc.G), 0, e);
            return;
        }
        // the down phase runs batch by batch in the prologue's order (iq2_schedule_batches), each batch's row groups
        // in turn
        const int uu = u - sc.U, p = uu / sc.G2;
        Unit w;
        w.bidx = sc.offs ? sc.dorder[p] : __ldcg(sc.dorder + p);
        if ((unsigned)w.bidx >= (unsigned)sc.bpre[sc.nslots]) {   // never, with a whole order: refuse, not read past it
            atomicOr(&g_iq2_error, 16);
            e[0] = -1;
            left = 0;
            return;
        }
        const int i = iq2_batch_slot(sc.bpre, sc.nslots, w.bidx);
        w.s = sc.order[i];
        w.b0 = (w.bidx - sc.bpre[i]) * kUnitTok;
        w.g = uu - p * sc.G2;
        w.nt = min(kUnitTok, sc.cnt[w.s] - w.b0);
        fill(b, sc, w, 1, e);
#ifdef B200Q_X_STATS
        atomicAdd(&g_x_stats[3], 1ull);
#endif
        if (ld_acquire(ready + w.bidx) < sc.G) pending = 1 + w.bidx;   // the batch's up rows are not all in
        else asm volatile("fence.proxy.async.global;" ::: "memory");   // rows read by the async proxy (bulk copies)
    }

    // the unit's next super-block into the stage at st (barrier bar), which the warp has finished reading
    template <bool FUSED>
    __device__ __forceinline__ void issue(const GemvArgs& a, const GemvArgs& b, const Sched& sc, const int* ready,
                                          int ctr, uint32_t st, uint32_t bar, Ring& r) {
        if (left == 0 || (FUSED && pending)) return;
        asm volatile("fence.proxy.async.shared::cta;" ::: "memory");   // the warp's reads of the stage come first
        mbar_expect_tx(bar, (uint32_t)(kIq2Unit + nt * (kScl ? 288 : 256)));
        if (split) {
            bulk_g2s_stream(st, wsrc, 2048, bar, evict_first_policy());
            bulk_g2s_stream(st + 2048, dsrc, 64, bar, evict_first_policy());
            wsrc += 2048;
            dsrc += 64;
        } else {
            bulk_g2s_stream(st, wsrc, kIq2Unit, bar, evict_first_policy());
            wsrc += kIq2Unit;
        }
#pragma unroll
        for (int m = 0; m < kUnitTok; m++) {
            if (m < nt) {
                bulk_g2s(st + kStageAct + m * 256, xq + xoff[m], 256, bar);
                xoff[m] += 256;
                if (kScl) {
                    bulk_g2s(st + kStageScl + m * 32, xs + soff[m], 32, bar);
                    soff[m] += 8;
                }
            }
        }
        r.issued++;
        if (--left == 0) grab<FUSED>(a, b, sc, ready, ctr);
    }

    // The ring is empty (every issued stage read): wait, bounded, for a pending unit's batch, then fill the ring from
    // the stage the warp reads next.  False when the wait timed out.
    template <bool FUSED>
    __device__ __forceinline__ bool force(const GemvArgs& a, const GemvArgs& b, const Sched& sc, const int* ready,
                                          int ctr, Ring& r) {
        if (FUSED && pending) {
            const int* c = ready + (pending - 1);
            const unsigned long long t0 = globaltimer();
#ifdef B200Q_X_STATS
            atomicAdd(&g_x_stats[0], 1ull);
#endif
            while (ld_acquire(c) < sc.G) {
                // give up after 2 s, or at once when another wait of this launch has (rows may never be released)
                if (globaltimer() - t0 > kWaitNs || *(volatile int*)&g_unit_ctr[ctr][6]) {
                    atomicOr(&g_iq2_error, 8);
                    atomicExch(&g_unit_ctr[ctr][6], 1);
                    return false;
                }
                __nanosleep(128);
            }
            asm volatile("fence.proxy.async.global;" ::: "memory");
#ifdef B200Q_X_STATS
            atomicAdd(&g_x_stats[1], globaltimer() - t0);
#endif
            pending = 0;
        }
#pragma unroll
        for (int i = 0; i < kStages; i++) {
            int sl = r.slot + i;
            if (sl >= kStages) sl -= kStages;
            issue<FUSED>(a, b, sc, ready, ctr, r.stage_at(sl), r.bar0 + 8u * (uint32_t)sl, r);
        }
        return true;
    }
};

// the table words are written once before the first barrier and never change: a plain (reorderable) load
__device__ __forceinline__ uint32_t lds_tbl(uint32_t addr) {
    uint32_t v;
    asm("ld.shared.u32 %0, [%1];" : "=r"(v) : "r"(addr));
    return v;
}
__device__ __forceinline__ uint2 lds64(uint32_t addr) {
    uint2 v;
    asm volatile("ld.shared.v2.u32 {%0,%1}, [%2];" : "=r"(v.x), "=r"(v.y) : "r"(addr));
    return v;
}

// dA = d (0.5 + s4) / 4 = (2 s4 + 1) d / 8 of a chunk, exactly.  s4 is the top bits of its four sign bytes: one
// multiply gathers bits 7, 15, 23, 31 into 28..31 (every partial product lands on its own bit, so nothing carries)
// and the added bit 27 is the +1; a funnel shift puts 2 s4 + 1 under the exponent of 2^23, f = 2^23 + 2 s4 + 1, and
// one fma gives f * d/8 - 2^23 * d/8 with no rounding (the result has at most 16 significant bits).
__device__ __forceinline__ float chunk_scale(uint32_t qy, float dh8, float dh8m) {
    const uint32_t p = (qy & 0x80808080u) * 0x00204081u + 0x08000000u;
    return fmaf(__uint_as_float(__funnelshift_r(p, 0x02580000u, 27)), dh8, dh8m);
}

// One unit: its 32 rows (a lane each) over K in chunk order, exactly NT token rows.  Every stage is one super-block,
// read as four chunk pairs (a loop kept rolled: the unrolled stage outgrows the instruction cache).  Returns false
// when a ring wait timed out.  `ready`: a fused launch's up unit adds one to its batch's counter once its rows are
// stored (nullptr otherwise).
struct Ids {
    int v[kUnitTok];
};

template <int NT, int EPI, bool FUSED, bool kScl, bool PTRS = false>
__device__ __forceinline__ bool unit_rows(const GemvArgs& a, const GemvArgs& pa, const GemvArgs& pb, int g,
                                          const Ids& ids, int lane, Ring& r, Producer<kScl>& pr, const Sched& sc,
                                          const int* ready, int* release, int ctr, int nsb) {
    static_assert(kScl == (EPI != kDots), "scales travel with every epilogue but the chunk dots");
    const int* id = ids.v;
    const uint32_t lane_c = kTblAddr | ((uint32_t)lane * 4u), lane_s = lane_c | 128u;
    const int row = g * kIq2Tile + lane, nc = a.k >> 5;
    // exact int -> float without a conversion instruction: an integer i with |i| < 2^22 added to the bits of 1.5 * 2^23
    // gives the float 1.5 * 2^23 + i (the dot's bound is 32 * 43 * 127 = 174752)
    constexpr int kBias = 0x4B400000;
    constexpr float kBiasF = 12582912.f;
    float acc[NT];
#pragma unroll
    for (int m = 0; m < NT; m++) acc[m] = 0.f;
    for (int sb = 0; sb < nsb; sb++) {
        if (FUSED) {
            // a pending unit reaches the front with nothing in flight: only now may the warp wait for its batch
            int fok = 1;
            if (lane == 0 && r.issued == r.consumed) fok = pr.template force<FUSED>(pa, pb, sc, ready, ctr, r);
            if (!__shfl_sync(0xffffffffu, fok, 0)) return false;
        }
        const uint32_t st = r.stage(), bar = r.bar();
        const bool ok = mbar_wait(bar, r.par, kWaitNs);
        if (__any_sync(0xffffffffu, !ok)) return false;
        const float dh8 = __half2float(__ushort_as_half(lds16(st + 2048 + lane * 2))) * 0.125f;
        const float dh8m = -8388608.f * dh8;   // exact: a power-of-two scaling
        // the signed magnitudes {8, 25, 43, -8 | -25, -43} as two words, loaded rather than written as immediates:
        // held in registers they cost two, rebuilt at each use they cost an instruction a prmt
        const uint2 tb = lds64(sc.kc);
#ifdef B200Q_X_UNROLL_J
#pragma unroll
#else
#pragma unroll 1
#endif
        for (int j = 0; j < 4; j++) {
            const uint4 q = lds128(st + j * 512 + lane * 16);
            float se[NT], so[NT];   // the tokens' scales of chunks 2j, 2j + 1
#pragma unroll
            for (int m = 0; m < NT; m++) {
                if constexpr (kScl) {
                    const uint2 v = lds64(st + kStageScl + m * 32 + j * 8);
                    se[m] = __uint_as_float(v.x);
                    so[m] = __uint_as_float(v.y);
                } else {
                    se[m] = so[m] = 0.f;
                }
            }
#pragma unroll
            for (int h = 0; h < 2; h++) {
                const int c8 = 2 * j + h;
                const uint32_t qx = h ? q.z : q.x, qy = h ? q.w : q.y;
                const float dA = chunk_scale(qy, dh8, dh8m);
                uint32_t wq[8];
#pragma unroll
                for (int gg = 0; gg < 4; gg++) {
                    // address = kTblAddr | (index byte << 8) | lane * 4 (| 128 for the sign half)
                    const uint32_t sel_b = 0x7604u | ((uint32_t)gg << 4);
                    const uint32_t sel = lds_tbl(prmt(qx, lane_c, sel_b)) + lds_tbl(prmt(qy, lane_s, sel_b));
                    wq[2 * gg] = prmt(tb.x, tb.y, sel);
#ifdef B200Q_X_UMULHI
                    wq[2 * gg + 1] = prmt(tb.x, tb.y, __umulhi(sel, 0x10000u));
#else
                    wq[2 * gg + 1] = prmt(tb.x, tb.y, sel >> 16);
#endif
                }
#pragma unroll
                for (int m = 0; m < NT; m++) {
                    const uint32_t xa = st + kStageAct + m * 256 + c8 * 32;
                    const uint4 x0 = lds128(xa), x1 = lds128(xa + 16);
                    // one chain of eight: the other tokens and the next chunk's dequantisation hide its latency
                    int da = __dp4a((int)wq[0], (int)x0.x, kBias);
                    da = __dp4a((int)wq[1], (int)x0.y, da);
                    da = __dp4a((int)wq[2], (int)x0.z, da);
                    da = __dp4a((int)wq[3], (int)x0.w, da);
                    da = __dp4a((int)wq[4], (int)x1.x, da);
                    da = __dp4a((int)wq[5], (int)x1.y, da);
                    da = __dp4a((int)wq[6], (int)x1.z, da);
                    da = __dp4a((int)wq[7], (int)x1.w, da);
                    const int dot = da;
                    if constexpr (EPI == kDots) {
                        a.dots[((size_t)id[m] * a.n + row) * nc + sb * 8 + c8] = dot - kBias;
                    } else {
                        const float s = h ? so[m] : se[m];
                        acc[m] = fmaf(dA * s, __int_as_float(dot) - kBiasF, acc[m]);
                    }
                }
            }
        }
        __syncwarp();   // every lane is done with the stage: lane 0 refills it
        if (lane == 0) pr.template issue<FUSED>(pa, pb, sc, ready, ctr, st, bar, r);
        r.advance();
    }
    if constexpr (EPI != kDots) {
#pragma unroll
        for (int m = 0; m < NT; m++) {
            float v = acc[m];
            if constexpr (EPI != kStore) v = v > 0.f ? v * v : 0.f;
            if constexpr (EPI == kRelu2Q8) {
                // quant_rows_k over this warp's 32 consecutive outputs (one 32-group of the output row)
                float am = v;   // v >= 0 after relu^2
#pragma unroll
                for (int o = 16; o > 0; o >>= 1) am = fmaxf(am, __shfl_xor_sync(0xffffffffu, am, o));
                const float inv = am > 0.f ? 127.f / am : 0.f;
                a.aq[(size_t)id[m] * a.n + row] = (int8_t)__float2int_rn(v * inv);
                if (lane == 0) a.as[(size_t)id[m] * (a.n >> 5) + g] = am / 127.f;
            } else if constexpr (PTRS) {   // every id's output row at its own address (GemvArgs::y_rows)
                unsigned char* dst = reinterpret_cast<unsigned char*>(a.y_rows[id[m]]);
                if (a.y_bf16) reinterpret_cast<__nv_bfloat16*>(dst)[row] = __float2bfloat16_rn(v);
                else reinterpret_cast<float*>(dst)[row] = v;
            } else {
                if (a.y_bf16) reinterpret_cast<__nv_bfloat16*>(a.y)[(size_t)id[m] * a.ldy + row] = __float2bfloat16_rn(v);
                else a.y[(size_t)id[m] * a.ldy + row] = v;
            }
        }
    }
    if (FUSED && EPI == kRelu2Q8 && release != nullptr) {
        // this unit's rows are stored: release them to the down units of its batch (bulk copies read them, so the
        // proxy fence orders the stores before the async proxy's reads as well)
        __syncwarp();
        if (lane == 0) {
            asm volatile("fence.proxy.async.global;" ::: "memory");
            __threadfence();
            atomicAdd(release, 1);
        }
    }
    return true;
}

__device__ __forceinline__ void st_release(int* p, int v) {
    asm volatile("st.release.gpu.global.b32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}

// a bounded wait of one thread until *p >= v; false (and an error bit) when it gave up, after 2 s or at once when
// another wait of the launch (slot ctr) has given up
__device__ __forceinline__ bool wait_at_least(const int* p, int v, int ctr) {
    if (ld_acquire(p) >= v) return true;
    const unsigned long long t0 = globaltimer();
    while (ld_acquire(p) < v) {
        if (globaltimer() - t0 > kWaitNs || *(volatile int*)&g_unit_ctr[ctr][6]) {
            atomicOr(&g_iq2_error, 32);
            atomicExch(&g_unit_ctr[ctr][6], 1);
            return false;
        }
        __nanosleep(256);
    }
    return true;
}

// The layer's prologue, every thread of the CTA.  After the wait for the preceding launch, the CTA quantises its
// share of x to int8 rows (a warp per 32-group) and counts itself done; then it routes every token, groups the pairs
// by expert and computes the GEMVs' schedule on its own, into shared memory (every CTA gets the same bytes; only CTA 0
// writes the routing to the caller's buffers); then it waits (bounded) until every CTA's share of x is written.
// Scratch: the ring stages, unused until the units start.  False when the wait gave up: the CTA takes no units.
__device__ bool layer_prologue(const LayerArgs& L, const GemvArgs& a, int nslots, int* scr, int ctr, int* s_cnt,
                               int* s_order, int* s_bpre, int* s_offs, int* s_ord, int* s_dord) {
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5, nw = blockDim.x >> 5;
    XTRACE(1);
    pdl_wait();
    XTRACE(2);
    // route (a warp a token) and quantise this CTA's share of x (a warp a 32-group) at once: with fewer tokens than
    // warps, the quantising warps are those without a token
    int* ridx_s = scr;                 // kLayerIds: the routing
    int* place_s = ridx_s + kLayerIds; // kLayerIds: the schedule's scratch
    float* rw_s = reinterpret_cast<float*>(place_s + kLayerIds);   // kLayerIds: the routing of CTAs other than 0
    const int pairs = L.T * L.topk;
    int* ridx_o = blockIdx.x == 0 ? L.ridx : reinterpret_cast<int*>(rw_s);   // CTA 0 writes the caller's buffers
    float* rw_o = blockIdx.x == 0 ? L.rw : rw_s;   // (the others write a scratch nobody reads)
    const int groups = L.H >> 5, ng = L.T * groups;
    const int qw0 = L.T < nw ? L.T : 0, nqw = nw - qw0;   // the quantising warps
    if (warp >= qw0)
        for (int gw = (int)blockIdx.x * nqw + (warp - qw0); gw < ng; gw += (int)gridDim.x * nqw) {
            const int r = gw / groups, g = gw - r * groups;
            const float v = load_act(L.x, B200Q_BF16, (size_t)r * L.H + g * 32 + lane);
            quant_group(v, lane, const_cast<int8_t*>(a.xq) + (size_t)r * L.H + g * 32,
                        const_cast<float*>(a.xs) + (size_t)r * groups + g);
        }
    for (int t = warp; t < L.T; t += nw) {
        if (L.route == B200Q_ROUTE_SOFTMAX && L.E <= 128)
            route_softmax_bf16(reinterpret_cast<const __nv_bfloat16*>(L.logits), L.E, L.topk, t, lane, ridx_o, rw_o,
                               ridx_s);
        else if (L.E <= 128) route_token<4>(L.logits, B200Q_BF16, L.E, L.bias, L.E, L.topk, L.route, L.scale, t, lane,
                                            ridx_o, rw_o, ridx_s);
        else route_token<16>(L.logits, B200Q_BF16, L.E, L.bias, L.E, L.topk, L.route, L.scale, t, lane, ridx_o, rw_o,
                             ridx_s);
    }
    __syncthreads();
    if (tid == 0) {   // this CTA's share of x is written
        __threadfence();
        atomicAdd(&g_unit_ctr[ctr][4], 1);
    }
    XTRACE(10);
    layer_schedule(ridx_s, pairs, L.E, L.extra, a.n >> 5, (int)gridDim.x * kGemvWarps, s_cnt, s_offs, s_ord, s_order,
                   s_bpre, s_dord, place_s);
    XTRACE(13);
    if (tid == 0) {
        const bool ok = wait_at_least(&g_unit_ctr[ctr][4], (int)gridDim.x, ctr);
        asm volatile("fence.proxy.async.global;" ::: "memory");   // x's rows are read by bulk copies
        scr[0] = ok ? 1 : 0;
    }
    __syncthreads();
    XTRACE(5);
    const bool ok = scr[0] != 0;
    __syncthreads();
    return ok;
}

// The layer's epilogue: once every CTA is done with its units (a bounded count), this CTA's share of
// out[t] = sum_k rw[t][k] mo[t * topk + k] (+ the shared expert's row), in combine_k's order.
__device__ void layer_epilogue(const LayerArgs& L, const GemvArgs& b, int ctr) {
    const int tid = threadIdx.x;
    __syncthreads();
    XTRACE(7);
    if (tid == 0) {
        __threadfence();
        atomicAdd(&g_unit_ctr[ctr][5], 1);
        wait_at_least(&g_unit_ctr[ctr][5], (int)gridDim.x, ctr);
    }
    __syncthreads();
    XTRACE(8);
    const int h4n = L.H >> 2, total = L.T * h4n, topk = L.topk;
    const float* mo = b.y;
    for (int i = (int)blockIdx.x + (int)gridDim.x * tid; i < total; i += (int)gridDim.x * blockDim.x) {   // every CTA a share
        const int t = i / h4n, h4 = i - t * h4n;
        float4 acc = make_float4(0.f, 0.f, 0.f, 0.f);
        float wk[16];
        float4 v[16];
#pragma unroll
        for (int kk = 0; kk < 16; kk++)   // every load issued before the sums (topk <= 16)
            if (kk < topk) {
                wk[kk] = __ldcg(L.rw + t * topk + kk);
                v[kk] = __ldcg(reinterpret_cast<const float4*>(mo + ((size_t)t * topk + kk) * L.H) + h4);
            }
#pragma unroll
        for (int kk = 0; kk < 16; kk++)
            if (kk < topk) {
                acc.x = fmaf(wk[kk], v[kk].x, acc.x); acc.y = fmaf(wk[kk], v[kk].y, acc.y);
                acc.z = fmaf(wk[kk], v[kk].z, acc.z); acc.w = fmaf(wk[kk], v[kk].w, acc.w);
            }
        if (L.extra) {
            const float4 sv = __ldcg(reinterpret_cast<const float4*>(mo + ((size_t)L.T * topk + t) * L.H) + h4);
            acc.x += sv.x; acc.y += sv.y; acc.z += sv.z; acc.w += sv.w;
        }
        if (L.out_dtype == B200Q_BF16) {
            __nv_bfloat162* o = reinterpret_cast<__nv_bfloat162*>(reinterpret_cast<__nv_bfloat16*>(L.out) + (size_t)t * L.H) + 2 * h4;
            o[0] = __floats2bfloat162_rn(acc.x, acc.y);
            o[1] = __floats2bfloat162_rn(acc.z, acc.w);
        } else {
            reinterpret_cast<float4*>(reinterpret_cast<float*>(L.out) + (size_t)t * L.H)[h4] = acc;
        }
    }
}

// One launch: the units of one phase (EPI), or a fused up (kRelu2Q8, args a) + down (kStore, args b) pair over the
// same slots, whose schedule the fused form requires (a.sched); LAYER: the whole decode layer around the fused pair.
template <int EPI, bool FUSED, bool LAYER, bool PTRS = false>
__device__ __forceinline__ void gemv_body(const GemvArgs& a, const GemvArgs& b, int* ready, int nslots,
                                          const LayerArgs& L) {
    static_assert(!FUSED || EPI == kRelu2Q8, "a fused launch is up (relu^2 + int8 rows) then down");
    static_assert(!LAYER || FUSED, "the layer runs the fused projections");
    extern __shared__ __align__(128) unsigned char dyn[];
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    // the layout around the table at kTblAddr (see kTblAddr): barriers, counts, prefix, stages below; stages above
    const uint32_t base = (uint32_t)__cvta_generic_to_shared(dyn);
    int* s_cnt = reinterpret_cast<int*>(dyn + kNumStages * 8);
    int* s_order = s_cnt + kMaxSlots;
    int* s_bpre = s_order + kMaxSlots;
    int* s_queue = s_bpre + kMaxSlots + 1;
    int* s_offs = s_queue + kGemvWarps * kQueue * kQEntry;   // the one-launch layer's schedule
    int* s_ord = s_offs + kLayerSlots + 1;
    int* s_dord = s_ord + kLayerIds;
    const uint32_t a0 = (base + kHdrBytes + 15u) & ~15u;
    int nA = a0 <= kTblAddr ? (int)((kTblAddr - a0) / kStageBytes) : 0;
    if (nA > kNumStages) nA = kNumStages;
    Ring r;
    r.bar0 = base + 8u * (uint32_t)(warp * kStages);
#pragma unroll
    for (int i = 0; i < kStages; i++) {
        const int q = warp * kStages + i;
        r.st[i] = q < nA ? a0 + (uint32_t)(q * kStageBytes) : 2u * kTblAddr + (uint32_t)((q - nA) * kStageBytes);
    }
    r.slot = r.consumed = r.issued = 0;
    r.par = 0;
    const uint32_t end = 2u * kTblAddr + (uint32_t)((kNumStages - nA) * kStageBytes);
    if (base + kHdrBytes > kTblAddr || (size_t)end > (size_t)base + kGemvSmem) {
        if (tid == 0) atomicOr(&g_iq2_error, 2);   // the dynamic shared memory does not start low enough
        return;
    }
    if (lane == 0) {
        for (int i = 0; i < kStages; i++) mbar_init(r.bar0 + 8u * (uint32_t)i, 1);
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    }
    XTRACE(0);
    build_table(reinterpret_cast<uint32_t*>(dyn + (kTblAddr - base)));
    const uint32_t kc = (base + (uint32_t)((const unsigned char*)(s_dord + kLayerIds) - dyn) + 7u) & ~7u;
    if (tid == 0) asm volatile("st.shared.v2.u32 [%0], {%1, %2};" ::"r"(kc), "r"(0xF82B1908u), "r"(0x0000D5E7u) : "memory");
    bool layer_ok = true;
    if constexpr (LAYER) {
        ready = &g_layer_ready[a.ctr][0];
        layer_ok = layer_prologue(L, a, nslots, reinterpret_cast<int*>(dyn + (2u * kTblAddr - base)), a.ctr, s_cnt,
                                  s_order, s_bpre, s_offs, s_ord, s_dord);
    }
    // With a schedule whose inputs an earlier launch wrote, the schedule and each warp's first unit are taken while
    // the preceding launch still runs; only the bulk copies wait for it.
    const bool early = !FUSED && a.sched != nullptr && a.sched_early;
    if (!early && !LAYER) pdl_wait();
    if (!LAYER)
        for (int s = tid; s < nslots; s += blockDim.x) {
            int cnt = a.counts ? __ldcg(a.counts + s) : a.dense_rows;
            if (slot_weights(a, s) == nullptr) cnt = 0;
            s_cnt[s] = cnt;
        }
    if (LAYER) {
        // the prologue computed the schedule in shared memory
    } else if (a.sched) {
        for (int i = tid; i <= nslots; i += blockDim.x) {
            if (i < nslots) s_order[i] = __ldcg(a.sched + i);
            s_bpre[i] = __ldcg(a.sched + nslots + i);
        }
    } else {
        __syncthreads();
        iq2_schedule_slots(s_cnt, nslots, s_order, s_bpre, s_order);
    }
    __syncthreads();
    Sched sc;
    sc.cnt = s_cnt;
    sc.order = s_order;
    sc.bpre = s_bpre;
    sc.nslots = nslots;
    sc.G = a.n / kIq2Tile;
    sc.U = s_bpre[nslots] * sc.G;
    sc.G2 = FUSED ? b.n / kIq2Tile : 0;
    sc.U2 = FUSED ? s_bpre[nslots] * sc.G2 : 0;
    sc.dorder = LAYER ? s_dord : a.sched + 2 * nslots + 1;
    sc.offs = LAYER ? s_offs : nullptr;
    sc.ord = LAYER ? s_ord : nullptr;
    if (!layer_ok) sc.U = sc.U2 = 0;   // a prologue wait gave up: no units (the error bit is set)
    sc.kc = kc;
    const int ctr = a.ctr;
    constexpr bool kScl = EPI != kDots;
    Producer<kScl> pr;
    pr.queue = s_queue + warp * kQueue * kQEntry;
    pr.pn = 0;
    pr.left = 0;
    pr.pending = 0;
    XTRACE(6);
    if (lane == 0) pr.template grab<FUSED>(a, b, sc, ready, ctr);
    if (early) pdl_wait();
    if (lane == 0) {
#pragma unroll
        for (int i = 0; i < kStages; i++)
            pr.template issue<FUSED>(a, b, sc, ready, ctr, r.st[i], r.bar0 + 8u * (uint32_t)i, r);
    }
    const int nsb = a.k >> 8, nsb2 = FUSED ? b.k >> 8 : 0;
    bool healthy = true;
    for (int cn = 0; healthy; cn++) {
        __syncwarp();   // lane 0's queue writes are visible to the warp
        const int* e = pr.queue + (cn % kQueue) * kQEntry;
        const int g = e[0];
        if (g < 0) break;
        const int nt = e[1];
        const int ph = e[2] & 1;
        int* rdy = FUSED ? ready + (e[2] >> 1) : nullptr;
        Ids id;
#pragma unroll
        for (int m = 0; m < kUnitTok; m++) id.v[m] = e[3 + m];
        static_assert(kUnitTok == 3, "one code path per token count 1 .. 3");
        bool down_unit = false;
        if constexpr (FUSED) down_unit = ph != 0;
        if constexpr (FUSED) {
            if (down_unit) {
                if (nt == 1) healthy = unit_rows<1, kStore, FUSED, kScl, PTRS>(b, a, b, g, id, lane, r, pr, sc, ready, nullptr, ctr, nsb2);
                else if (nt == 2) healthy = unit_rows<2, kStore, FUSED, kScl, PTRS>(b, a, b, g, id, lane, r, pr, sc, ready, nullptr, ctr, nsb2);
                else healthy = unit_rows<3, kStore, FUSED, kScl, PTRS>(b, a, b, g, id, lane, r, pr, sc, ready, nullptr, ctr, nsb2);
                continue;
            }
        }
        {
            if (nt == 1) healthy = unit_rows<1, EPI, FUSED, kScl>(a, a, b, g, id, lane, r, pr, sc, ready, rdy, ctr, nsb);
            else if (nt == 2) healthy = unit_rows<2, EPI, FUSED, kScl>(a, a, b, g, id, lane, r, pr, sc, ready, rdy, ctr, nsb);
            else healthy = unit_rows<3, EPI, FUSED, kScl>(a, a, b, g, id, lane, r, pr, sc, ready, rdy, ctr, nsb);
        }
    }
    if (!healthy) {
        // a stage never filled: flag it, and let this warp's copies in flight land before the CTA's memory goes away
        if (lane == 0) {
            atomicOr(&g_iq2_error, 1);
            for (int i = r.consumed; i < r.issued; i++)
                mbar_wait(r.bar0 + 8u * (uint32_t)(i % kStages), (uint32_t)((i / kStages) & 1), kWaitNs);
        }
        __syncwarp();
    }
    if constexpr (LAYER) layer_epilogue(L, b, ctr);
    XTRACE(9);
    // the last CTA out resets this launch slot's counters (and the layer's readiness counters) for its next launch
    __syncthreads();
    if (tid == 0) {
        __threadfence();
        const bool last = atomicAdd(&g_unit_ctr[ctr][1], 1) == (int)gridDim.x - 1;
        if (last) {
#pragma unroll
            for (int i = 0; i < 8; i++) g_unit_ctr[ctr][i] = 0;
            // every CTA wrote its outputs before its count (fence, then the add); this CTA's system-scope fence (the
            // acquire of those counts, cumulative) orders them before the flags that publish them to other ranks
            if (a.done_base) {
                const int e = *reinterpret_cast<volatile const int*>(a.done_epoch);
                fence_acq_rel_sys();
                for (int j = 0; j < a.done_n; j++) st_relaxed_sys(reinterpret_cast<int*>(a.done_base[j] + a.done_off), e);
            }
        }
        s_queue[0] = last;
    }
    if constexpr (LAYER) {
        __syncthreads();
        if (s_queue[0])
            for (int i = tid; i < kLayerIds; i += blockDim.x) g_layer_ready[ctr][i] = 0;
    }
    pdl_trigger();
}

template <int EPI, bool FUSED, bool PTRS = false>
__global__ void __launch_bounds__(kGemvWarps * 32, 1) iq2_gemv_k(GemvArgs a, GemvArgs b, int* ready, int nslots) {
    const LayerArgs none = {};
    gemv_body<EPI, FUSED, false, PTRS>(a, b, ready, nslots, none);
}

__global__ void __launch_bounds__(kGemvWarps * 32, 1) decode_layer_k(GemvArgs a, GemvArgs b, int* ready, int nslots,
                                                                     LayerArgs L) {
    gemv_body<kRelu2Q8, true, true>(a, b, ready, nslots, L);
}

static int num_sms() {
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

template <int EPI, bool FUSED, bool PTRS = false>
static cudaError_t launch_gemv_e(const GemvArgs& a, const GemvArgs& b, int* ready, int nslots, cudaStream_t s) {
    static bool opted = false;
    if (!opted) {
        cudaError_t e = cudaFuncSetAttribute(iq2_gemv_k<EPI, FUSED, PTRS>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                             (int)kGemvSmem);
        if (e != cudaSuccess) return e;
        opted = true;
    }
    return launch(iq2_gemv_k<EPI, FUSED, PTRS>, dim3(num_sms()), dim3(kGemvWarps * 32), kGemvSmem, s, a, b, ready,
                  nslots);
}

// launches take the counter slots in turn: kUnitCtrs launches can be in flight (on any streams) before a slot is
// reused, and a slot is back to zero when its launch ends
static int next_ctr() {
    static std::atomic<unsigned> next_slot{0};
    return (int)(next_slot.fetch_add(1u) % kUnitCtrs);
}

cudaError_t launch_iq2_gemv(const GemvArgs& a0, int nslots, int /*maxcnt*/, int epi, cudaStream_t s) {
    if (nslots <= 0 || nslots > kMaxSlots) return cudaErrorInvalidValue;
    GemvArgs a = a0;
    a.ctr = next_ctr();
    switch (epi) {
        case kStore: return launch_gemv_e<kStore, false>(a, a, nullptr, nslots, s);
        case kRelu2: return launch_gemv_e<kRelu2, false>(a, a, nullptr, nslots, s);
        case kRelu2Q8: return launch_gemv_e<kRelu2Q8, false>(a, a, nullptr, nslots, s);
        default: return launch_gemv_e<kDots, false>(a, a, nullptr, nslots, s);
    }
}

int iq2_first_wave() { return num_sms() * kGemvWarps; }

bool layer_fits(int T, int E, int topk, bool shared) {
    return T >= 1 && T <= 64 && E >= 1 && E + 1 <= kLayerSlots && T * topk + (shared ? T : 0) <= kLayerIds;
}

cudaError_t launch_decode_layer(const GemvArgs& up, const GemvArgs& down, int* ready, int nslots, const LayerArgs& L,
                                cudaStream_t s) {
    (void)ready;   // the launch keeps its readiness counters by launch slot
    if (!layer_fits(L.T, L.E, L.topk, L.extra > 0) || nslots != L.E + (L.extra > 0 ? 1 : 0)) return cudaErrorInvalidValue;
    static bool opted = false;
    if (!opted) {
        cudaError_t e = cudaFuncSetAttribute(decode_layer_k, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)kGemvSmem);
        if (e != cudaSuccess) return e;
        opted = true;
    }
    GemvArgs a = up;
    a.ctr = next_ctr();
    return launch(decode_layer_k, dim3(num_sms()), dim3(kGemvWarps * 32), kGemvSmem, s, a, down, ready, nslots, L);
}

cudaError_t launch_iq2_updown(const GemvArgs& up, const GemvArgs& down, int* ready, int nslots, cudaStream_t s) {
    if (nslots <= 0 || nslots > kMaxSlots || up.sched == nullptr || ready == nullptr) return cudaErrorInvalidValue;
    GemvArgs a = up;
    a.ctr = next_ctr();
    if (down.y_rows) return launch_gemv_e<kRelu2Q8, true, true>(a, down, ready, nslots, s);
    return launch_gemv_e<kRelu2Q8, true>(a, down, ready, nslots, s);
}

cudaError_t launch_iq2_pack_split(const uint8_t* raw, uint8_t* qs, uint8_t* dq, int64_t n, int k, cudaStream_t s) {
    const int64_t th = n * (k / 64);
    return launch(iq2_pack_split_k, dim3((unsigned)((th + 255) / 256)), dim3(256), 0, s, raw, qs, dq, n, k);
}

bool iq2_shape_ok(int64_t n, int k) { return n > 0 && n % kIq2Tile == 0 && n <= (1 << 24) && k > 0 && k % 256 == 0 && k <= 8192; }

// the GEMVs stream weights, int8 rows and scales with bulk copies, which need 16-byte aligned addresses
static bool a16(const void* p) { return ((uintptr_t)p & 15) == 0; }

int tc_error_read(int clear);   // tc_gemm.cu
int nv4_error_read(int clear);  // nv4_gemm.cu
int gemv_error_read(int clear); // gemv_tc.cu

}  // namespace b200q

using namespace b200q;

extern "C" {

size_t b200q_iq2_bytes(int64_t n, int k) { return iq2_bytes(n, k); }

int b200q_iq2_pack(const void* raw, void* packed, int64_t n, int k, void* stream) {
    if (!raw || !packed || !iq2_shape_ok(n, k)) return B200Q_EINVAL;
    const int64_t th = n * (k / 64);
    launch(iq2_pack_k, dim3((unsigned)((th + 255) / 256)), dim3(256), 0, (cudaStream_t)stream, (const uint8_t*)raw,
           (uint8_t*)packed, n, k);
    return launched();
}

void b200q_synth_iq2_host(uint64_t seed, int64_t nblocks, void* out) {
    uint8_t* o = (uint8_t*)out;
    for (int64_t i = 0; i < nblocks; i++) synth_iq2_block(seed, (uint64_t)i, o + i * 66);
}

int b200q_synth_iq2(uint64_t seed, int64_t nblocks, void* out, void* stream) {
    if (!out || nblocks < 0) return B200Q_EINVAL;
    if (nblocks == 0) return B200Q_OK;
    synth_iq2_k<<<(unsigned)((nblocks + 255) / 256), 256, 0, (cudaStream_t)stream>>>(seed, nblocks, (uint8_t*)out);
    return launched();
}

#ifdef B200Q_X_STATS
extern "C" int b200q_x_stats(unsigned long long* out, int clear) {
    cudaMemcpyFromSymbol(out, g_x_stats, sizeof(g_x_stats));
    if (clear) { unsigned long long z[4] = {0, 0, 0, 0}; cudaMemcpyToSymbol(g_x_stats, z, sizeof(z)); }
    return 0;
}
#endif

#ifdef B200Q_X_TRACE
extern "C" int b200q_x_trace(unsigned long long* out) {
    return (int)cudaMemcpyFromSymbol(out, g_x_trace, sizeof(g_x_trace));
}
#endif

int b200q_device_error(int clear) {
    int v = 0;
    if (cudaMemcpyFromSymbol(&v, g_iq2_error, sizeof(int)) != cudaSuccess) return -1;
    if (clear) {
        const int z = 0;
        cudaMemcpyToSymbol(g_iq2_error, &z, sizeof(int));
    }
    const int t = b200q::tc_error_read(clear), f = b200q::nv4_error_read(clear), d = b200q::gemv_error_read(clear);
    if (t < 0 || f < 0 || d < 0) return -1;
    return v | (t << 4) | (f << 8) | (d << 12);
}

int b200q_iq2_gemv(const void* w, int n, int k, const int8_t* xq, const float* xs, int T, float* y, int ldy, int epi,
                   void* stream) {
    if (!w || !xq || !xs || !y || !iq2_shape_ok(n, k) || T <= 0 || ldy < n || (epi != 0 && epi != 1) || !a16(w) ||
        !a16(xq) || !a16(xs))
        return B200Q_EINVAL;
    GemvArgs a = {};
    a.slab = (const uint8_t*)w; a.n = n; a.k = k; a.dense_rows = T;
    a.act_div = 1; a.act_split = 1 << 30; a.xq = xq; a.xs = xs; a.y = y; a.ldy = ldy;
    return status_from(launch_iq2_gemv(a, 1, T, epi, (cudaStream_t)stream));
}

int b200q_iq2_chunk_dots(const void* w, int n, int k, const int8_t* xq, int T, int32_t* dots, void* stream) {
    if (!w || !xq || !dots || !iq2_shape_ok(n, k) || T <= 0 || !a16(w) || !a16(xq)) return B200Q_EINVAL;
    GemvArgs a = {};
    a.slab = (const uint8_t*)w; a.n = n; a.k = k; a.dense_rows = T;
    a.act_div = 1; a.act_split = 1 << 30; a.xq = xq; a.dots = dots;
    return status_from(launch_iq2_gemv(a, 1, T, kDots, (cudaStream_t)stream));
}

int b200q_moe_up(const void* slab, int E, int n, int k, const int* counts, const int* offsets, const int* order,
                 int topk, const int8_t* xq, const float* xs, float* y, int ldy, int epi, void* stream) {
    if (!slab || !counts || !offsets || !order || !xq || !xs || !y || E <= 0 || E > 512 || topk <= 0 ||
        !iq2_shape_ok(n, k) || ldy < n || (epi != 0 && epi != 1) || !a16(slab) || !a16(xq) || !a16(xs))
        return B200Q_EINVAL;
    GemvArgs a = {};
    a.slab = (const uint8_t*)slab; a.expert_bytes = iq2_bytes(n, k); a.nslot_routed = E; a.n = n; a.k = k;
    a.counts = counts; a.offsets = offsets; a.order = order; a.act_div = topk; a.act_split = 1 << 30;
    a.xq = xq; a.xs = xs; a.y = y; a.ldy = ldy;
    return status_from(launch_iq2_gemv(a, E, 16, epi, (cudaStream_t)stream));
}

int b200q_moe_up_q8(const void* slab, int E, int n, int k, const int* counts, const int* offsets, const int* order,
                    int topk, const int8_t* xq, const float* xs, int8_t* aq, float* as, void* stream) {
    if (!slab || !counts || !offsets || !order || !xq || !xs || !aq || !as || E <= 0 || E > 512 || topk <= 0 ||
        !iq2_shape_ok(n, k) || !a16(slab) || !a16(xq) || !a16(xs))
        return B200Q_EINVAL;
    GemvArgs a = {};
    a.slab = (const uint8_t*)slab; a.expert_bytes = iq2_bytes(n, k); a.nslot_routed = E; a.n = n; a.k = k;
    a.counts = counts; a.offsets = offsets; a.order = order; a.act_div = topk; a.act_split = 1 << 30;
    a.xq = xq; a.xs = xs; a.aq = aq; a.as = as;
    return status_from(launch_iq2_gemv(a, E, 16, kRelu2Q8, (cudaStream_t)stream));
}

int b200q_moe_down(const void* slab, int E, int n, int k, const int* counts, const int* offsets, const int* order,
                   const int8_t* aq, const float* as, float* y, int ldy, void* stream) {
    if (!slab || !counts || !offsets || !order || !aq || !as || !y || E <= 0 || E > 512 || !iq2_shape_ok(n, k) || ldy < n ||
        !a16(slab) || !a16(aq) || !a16(as))
        return B200Q_EINVAL;
    GemvArgs a = {};
    a.slab = (const uint8_t*)slab; a.expert_bytes = iq2_bytes(n, k); a.nslot_routed = E; a.n = n; a.k = k;
    a.counts = counts; a.offsets = offsets; a.order = order; a.act_div = 1; a.act_split = 1 << 30;
    a.xq = aq; a.xs = as; a.y = y; a.ldy = ldy;
    return status_from(launch_iq2_gemv(a, E, 16, kStore, (cudaStream_t)stream));
}

}  // extern "C"
