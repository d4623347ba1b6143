// IQ2_XXS on sm_100a: the load-time packer, the synthetic generator and the HBM-streaming GEMVs over int8
// activation rows (dense, and grouped by expert for the routed MoE).
//
// Arithmetic (the routed-expert kernels moe_mma_k / moe_coop_k of the reference, bolt_kernels.cu:445-483 and
// 599-652): a row's 32-weight chunk c holds four grid-index bytes and a word of four 7-bit sign indices plus a 4-bit
// sub-scale.  Its weights are the signed grid integers (iq2xxs_grid bytes, negated where ksigns64 says); the chunk's
// exact int32 dot with the int8 activation row is scaled by dA * s, dA = d * (0.5 + s4) * 0.25 and s the row's
// activation scale of that chunk, and accumulated in chunk order:  acc = fma(dA * s, (float)dot, acc).
//
// Mapping: a warp owns 32 weight rows (lane l = row 32t + l) and walks K in order, so every lane's accumulation is
// the reference's own order and the result is reproducible bit for bit by a scalar loop.  A CTA of 8 warps covers
// 256 rows of one expert ("slot"); the slot's tokens (at most kMaxTok at a time) sit in shared memory as int8 rows
// and every lane reads the same activation word (a broadcast).  The weights stream once per slot: each lane
// keeps four 16-byte loads (64 weights each) in flight ahead of the math.
#include "iq2.cuh"

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
        const int sh = -e - 14 + 13;              // keep 24 - 13 - (-e - 14) bits
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

// ---------------------------------------------------------------------------------------------------------
// packer: ggml blocks [n][k/256][66] -> rt32 units (see common.cuh), one thread per (row, chunk pair)
// ---------------------------------------------------------------------------------------------------------
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
constexpr int kWarps = 8;                   // warps a CTA: 256 weight rows
constexpr int kPF = 4;                      // chunk pairs (16-byte loads) a lane keeps in flight: one super-block

enum Epi { kStore = 0, kRelu2 = 1, kRelu2Q8 = 2, kDots = 3 };



__device__ __forceinline__ uint4 ld_stream(const uint4* p) {
    uint4 v;
    asm volatile("ld.global.nc.L1::no_allocate.v4.u32 {%0,%1,%2,%3}, [%4];"
                 : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w) : "l"(p));
    return v;
}
__device__ __forceinline__ uint16_t ld_stream_u16(const uint16_t* p) {
    uint16_t v;
    asm volatile("ld.global.nc.L1::no_allocate.u16 %0, [%1];" : "=h"(v) : "l"(p));
    return v;
}

// the 32 signed grid integers of a chunk as 8 words of int8: (grid ^ mask) + (mask & 1s) negates a byte where the
// mask is 0xFF (grid bytes are at most 43, so no byte carries into the next)
__device__ __forceinline__ void iq2_chunk_weights(uint32_t qx, uint32_t qy, const uint2* __restrict__ grid,
                                                  const uint2* __restrict__ sgn, uint32_t (&w)[8]) {
#pragma unroll
    for (int g = 0; g < 4; g++) {
        const uint2 G = grid[(qx >> (8 * g)) & 255];
        const uint2 S = sgn[(qy >> (7 * g)) & 127];
        w[2 * g] = (G.x ^ S.x) + (S.x & 0x01010101u);
        w[2 * g + 1] = (G.y ^ S.y) + (S.y & 0x01010101u);
    }
}

// what a warp's walk over its 32 rows needs
struct RowCtx {
    const GemvArgs& a;
    const uint8_t* tile;     // the warp's row tile
    const int8_t* xsm;       // staged int8 rows [nt][k]
    const float* ssm;        // their scales [nt][k/32]
    const uint2* grid;
    const uint2* sgn;
    const int* ids;
    int k, n, nc, npair, lane, row, rt, nt;
};

// One warp, 32 rows (a lane each), K in chunk order, NT token rows (nt <= NT of them real; for NT in {1, 2} nt == NT).
template <int NT, int EPI>
__device__ __forceinline__ void iq2_rows(const RowCtx& c) {
    const int lane = c.lane;
    auto qptr = [&](int j) { return reinterpret_cast<const uint4*>(c.tile + (size_t)(j >> 2) * kIq2Unit) + (j & 3) * kIq2Tile + lane; };
    auto dptr = [&](int b) { return reinterpret_cast<const uint16_t*>(c.tile + (size_t)b * kIq2Unit + 2048) + lane; };
    float acc[NT];
#pragma unroll
    for (int m = 0; m < NT; m++) acc[m] = 0.f;

    uint4 buf[kPF];
    uint16_t dnext = ld_stream_u16(dptr(0));
#pragma unroll
    for (int i = 0; i < kPF; i++) buf[i] = ld_stream(qptr(i));

    for (int j0 = 0; j0 < c.npair; j0 += kPF) {
        uint4 cur[kPF];
#pragma unroll
        for (int i = 0; i < kPF; i++) cur[i] = buf[i];
        const float dh = __half2float(__ushort_as_half(dnext));
        if (j0 + kPF < c.npair) {
#pragma unroll
            for (int i = 0; i < kPF; i++) buf[i] = ld_stream(qptr(j0 + kPF + i));
            dnext = ld_stream_u16(dptr((j0 + kPF) >> 2));
        }
#pragma unroll
        for (int i = 0; i < 2 * kPF; i++) {
            const int ch = 2 * j0 + i;
            const uint32_t qx = (i & 1) ? cur[i >> 1].z : cur[i >> 1].x;
            const uint32_t qy = (i & 1) ? cur[i >> 1].w : cur[i >> 1].y;
            uint32_t w[8];
            iq2_chunk_weights(qx, qy, c.grid, c.sgn, w);
            const float dA = dh * (0.5f + (float)(qy >> 28)) * 0.25f;
#pragma unroll
            for (int m = 0; m < NT; m++) {
                if (NT <= 2 || m < c.nt) {
                    const int4* xa = reinterpret_cast<const int4*>(c.xsm + (size_t)m * c.k + ch * 32);
                    const int4 x0 = xa[0], x1 = xa[1];
                    int dot = __dp4a((int)w[0], x0.x, 0);
                    dot = __dp4a((int)w[1], x0.y, dot);
                    dot = __dp4a((int)w[2], x0.z, dot);
                    dot = __dp4a((int)w[3], x0.w, dot);
                    dot = __dp4a((int)w[4], x1.x, dot);
                    dot = __dp4a((int)w[5], x1.y, dot);
                    dot = __dp4a((int)w[6], x1.z, dot);
                    dot = __dp4a((int)w[7], x1.w, dot);
                    if constexpr (EPI == kDots) {
                        c.a.dots[((size_t)c.ids[m] * c.n + c.row) * c.nc + ch] = dot;
                    } else {
                        acc[m] = fmaf(dA * c.ssm[m * c.nc + ch], (float)dot, acc[m]);
                    }
                }
            }
        }
    }

    if constexpr (EPI != kDots) {
#pragma unroll
        for (int m = 0; m < NT; m++) {
            if (NT <= 2 || m < c.nt) {
                float v = acc[m];
                if constexpr (EPI != kStore) v = v > 0.f ? v * v : 0.f;
                const int id = c.ids[m];
                if constexpr (EPI == kRelu2Q8) {
                    // quant_rows_k over this warp's 32 consecutive outputs (one 32-group of the row)
                    float am = v;   // v >= 0 after relu^2
#pragma unroll
                    for (int o = 16; o > 0; o >>= 1) am = fmaxf(am, __shfl_xor_sync(0xffffffffu, am, o));
                    const float inv = am > 0.f ? 127.f / am : 0.f;
                    c.a.aq[(size_t)id * c.n + c.row] = (int8_t)__float2int_rn(v * inv);
                    if (lane == 0) c.a.as[(size_t)id * (c.n >> 5) + c.rt] = am / 127.f;
                } else {
                    c.a.y[(size_t)id * c.a.ldy + c.row] = v;
                }
            }
        }
    }
}

template <int MAXT, int EPI>
__global__ void __launch_bounds__(kWarps * 32, 2) iq2_gemv_k(GemvArgs a) {
    pdl_wait();
    __shared__ uint2 grid_s[256];
    __shared__ uint2 sgn_s[128];
    __shared__ int ids_s[MAXT];
    extern __shared__ __align__(16) unsigned char dyn[];
    const int k = a.k, n = a.n, nc = k >> 5, npair = k >> 6;
    int8_t* xsm = reinterpret_cast<int8_t*>(dyn);                                   // [MAXT][k]
    float* ssm = reinterpret_cast<float*>(dyn + (size_t)MAXT * k);                  // [MAXT][k/32]

    const int slot = blockIdx.y;
    int cnt, base;
    const uint8_t* W;
    if (a.counts == nullptr) { cnt = a.dense_rows; base = 0; W = a.slab; }
    else {
        cnt = a.counts[slot];
        base = a.offsets[slot];
        W = slot < a.nslot_routed ? a.slab + (size_t)slot * a.expert_bytes : a.extra_w;
    }
    if (cnt == 0 || W == nullptr) { pdl_trigger(); return; }

    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    for (int i = tid; i < 256; i += blockDim.x) {
        const unsigned long long g = iq2xxs_grid[i];
        grid_s[i] = make_uint2((uint32_t)g, (uint32_t)(g >> 32));
    }
    for (int i = tid; i < 128; i += blockDim.x) {
        const unsigned long long m = ksigns64[i];
        sgn_s[i] = make_uint2((uint32_t)m, (uint32_t)(m >> 32));
    }

    const int rt = blockIdx.x * kWarps + warp;     // this warp's row tile
    const bool active = rt * kIq2Tile < n;
    const int row = rt * kIq2Tile + lane;
    // super-block b of this tile: 4 x 512 bytes of chunk pairs, then 32 fp16 scales
    const uint8_t* tile = W + (size_t)rt * (k >> 8) * kIq2Unit;

    for (int b0 = 0; b0 < cnt; b0 += MAXT) {
        const int nt = min(MAXT, cnt - b0);
        __syncthreads();   // the previous batch is done with the staged rows
        if (tid < MAXT) ids_s[tid] = tid < nt ? (a.counts ? a.order[base + b0 + tid] : b0 + tid) : 0;
        __syncthreads();
        {   // stage the batch's int8 rows and their scales
            const int per = k >> 4;
            for (int idx = tid; idx < nt * per; idx += blockDim.x) {
                const int r = idx / per, i = idx - r * per;
                const int id = ids_s[r];
                const int arow = id < a.act_split ? id / a.act_div : id - a.act_split + a.act_base;
                reinterpret_cast<uint4*>(xsm + (size_t)r * k)[i] = __ldg(reinterpret_cast<const uint4*>(a.xq + (size_t)arow * k) + i);
            }
            for (int idx = tid; EPI != kDots && idx < nt * nc; idx += blockDim.x) {
                const int r = idx / nc, i = idx - r * nc;
                const int id = ids_s[r];
                const int arow = id < a.act_split ? id / a.act_div : id - a.act_split + a.act_base;
                ssm[r * nc + i] = __ldg(a.xs + (size_t)arow * nc + i);
            }
        }
        __syncthreads();
        if (!active) continue;
        RowCtx c{a, tile, xsm, ssm, grid_s, sgn_s, ids_s, k, n, nc, npair, lane, row, rt, nt};
        // the token count picks the code: a slot of one token runs the one-token loop, and so on
        if (nt == 1) iq2_rows<1, EPI>(c);
        else if (nt == 2) iq2_rows<2, EPI>(c);
        else if (MAXT >= 4 && nt <= 4) iq2_rows<(MAXT >= 4 ? 4 : 1), EPI>(c);
        else if (MAXT >= 8 && nt <= 8) iq2_rows<(MAXT >= 8 ? 8 : 1), EPI>(c);
        else if (MAXT >= 16) iq2_rows<(MAXT >= 16 ? 16 : 1), EPI>(c);
    }
    pdl_trigger();
}

static size_t gemv_smem(int maxt, int k) { return (size_t)maxt * k + (size_t)maxt * (k / 32) * 4; }

template <int MAXT, int EPI>
static cudaError_t launch_gemv_t(const GemvArgs& a, int nslots, cudaStream_t s) {
    const size_t sm = gemv_smem(MAXT, a.k);
    static size_t opted = 0;
    if (sm > 48 * 1024 && sm > opted) {
        cudaError_t e = cudaFuncSetAttribute(iq2_gemv_k<MAXT, EPI>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)sm);
        if (e != cudaSuccess) return e;
        opted = sm;
    }
    const dim3 grid((a.n / kIq2Tile + kWarps - 1) / kWarps, nslots);
    return launch(iq2_gemv_k<MAXT, EPI>, grid, dim3(kWarps * 32), sm, s, a);
}

template <int EPI>
static cudaError_t launch_gemv_e(const GemvArgs& a, int nslots, int maxcnt, cudaStream_t s) {
    if (maxcnt <= 1) return launch_gemv_t<1, EPI>(a, nslots, s);
    if (maxcnt <= 2) return launch_gemv_t<2, EPI>(a, nslots, s);
    if (maxcnt <= 4) return launch_gemv_t<4, EPI>(a, nslots, s);
    if (maxcnt <= 8) return launch_gemv_t<8, EPI>(a, nslots, s);
    return launch_gemv_t<16, EPI>(a, nslots, s);
}

cudaError_t launch_iq2_gemv(const GemvArgs& a, int nslots, int maxcnt, int epi, cudaStream_t s) {
    switch (epi) {
        case kStore: return launch_gemv_e<kStore>(a, nslots, maxcnt, s);
        case kRelu2: return launch_gemv_e<kRelu2>(a, nslots, maxcnt, s);
        case kRelu2Q8: return launch_gemv_e<kRelu2Q8>(a, nslots, maxcnt, s);
        default: return launch_gemv_e<kDots>(a, nslots, maxcnt, s);
    }
}

bool iq2_shape_ok(int64_t n, int k) { return n > 0 && n % kIq2Tile == 0 && k > 0 && k % 256 == 0 && k <= 8192; }

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

int b200q_iq2_gemv(const void* w, int n, int k, const int8_t* xq, const float* xs, int T, float* y, int ldy, int epi,
                   void* stream) {
    if (!w || !xq || !xs || !y || !iq2_shape_ok(n, k) || T <= 0 || ldy < n || (epi != 0 && epi != 1)) return B200Q_EINVAL;
    GemvArgs a = {};
    a.slab = (const uint8_t*)w; a.n = n; a.k = k; a.dense_rows = T;
    a.act_div = 1; a.act_split = 1 << 30; a.xq = xq; a.xs = xs; a.y = y; a.ldy = ldy;
    return status_from(launch_iq2_gemv(a, 1, T, epi, (cudaStream_t)stream));
}

int b200q_iq2_chunk_dots(const void* w, int n, int k, const int8_t* xq, int T, int32_t* dots, void* stream) {
    if (!w || !xq || !dots || !iq2_shape_ok(n, k) || T <= 0) return B200Q_EINVAL;
    GemvArgs a = {};
    a.slab = (const uint8_t*)w; a.n = n; a.k = k; a.dense_rows = T;
    a.act_div = 1; a.act_split = 1 << 30; a.xq = xq; a.dots = dots;
    return status_from(launch_iq2_gemv(a, 1, T, kDots, (cudaStream_t)stream));
}

int b200q_moe_up(const void* slab, int E, int n, int k, const int* counts, const int* offsets, const int* order,
                 int topk, const int8_t* xq, const float* xs, float* y, int ldy, int epi, void* stream) {
    if (!slab || !counts || !offsets || !order || !xq || !xs || !y || E <= 0 || E > 512 || topk <= 0 ||
        !iq2_shape_ok(n, k) || ldy < n || (epi != 0 && epi != 1))
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
        !iq2_shape_ok(n, k))
        return B200Q_EINVAL;
    GemvArgs a = {};
    a.slab = (const uint8_t*)slab; a.expert_bytes = iq2_bytes(n, k); a.nslot_routed = E; a.n = n; a.k = k;
    a.counts = counts; a.offsets = offsets; a.order = order; a.act_div = topk; a.act_split = 1 << 30;
    a.xq = xq; a.xs = xs; a.aq = aq; a.as = as;
    return status_from(launch_iq2_gemv(a, E, 16, kRelu2Q8, (cudaStream_t)stream));
}

int b200q_moe_down(const void* slab, int E, int n, int k, const int* counts, const int* offsets, const int* order,
                   const int8_t* aq, const float* as, float* y, int ldy, void* stream) {
    if (!slab || !counts || !offsets || !order || !aq || !as || !y || E <= 0 || E > 512 || !iq2_shape_ok(n, k) || ldy < n)
        return B200Q_EINVAL;
    GemvArgs a = {};
    a.slab = (const uint8_t*)slab; a.expert_bytes = iq2_bytes(n, k); a.nslot_routed = E; a.n = n; a.k = k;
    a.counts = counts; a.offsets = offsets; a.order = order; a.act_div = 1; a.act_split = 1 << 30;
    a.xq = aq; a.xs = as; a.y = y; a.ldy = ldy;
    return status_from(launch_iq2_gemv(a, E, 16, kStore, (cudaStream_t)stream));
}

}  // extern "C"
