// NVFP4 and Q8_0 decode GEMVs (T <= 16 activation rows): HBM-streaming, the dequantised weights fed to the tensor
// cores as the A operand of mma.m16n8k16 (fp16 in, fp32 accumulate), the activation rows as B.
//
// Numerics (exact operands, fp32 sums):
//   NVFP4  a = e2m1 * e4m3 scale, exact in fp16 (2 + 4 significant bits, the scale range 2^-9..448), the tensor
//          scale s2 applied to the fp32 result: the arithmetic of libbolt's PNV4 policy (bolt_mma.cu:98-175).
//   Q8_0   a = the int8 itself (exact in fp16); the per-32 scale d multiplies the fp32 partial of each 32-block,
//          FmtQ8's w = q * d (bolt_kernels.cu:41-52) with no rounding of the product (libbolt's PQ8 rounds
//          q * d to fp16, bolt_mma.cu:234-254).
//   The activations are converted to fp16 once (exact for bf16 inputs in fp16's normal range).
// Mapping: a warp owns one 16-row tile over one K slice; the eight warps of a CTA own eight consecutive tiles and
// share the slice's activations in shared memory.  grid.y splits K so that about four CTAs run per SM; the slices'
// fp32 partials are summed in slice order, so results do not depend on timing: by the last CTA of each column to
// finish (an arrival count a column) for NVFP4 at up to 8 rows, a call then being one launch; by a second kernel
// otherwise (measured faster there: the last CTA's sum is a serial tail the second kernel spreads over the GPU).
#include "common.cuh"

#include <atomic>
#include <mutex>

namespace b200q {

__device__ __forceinline__ uint32_t prmt(uint32_t a, uint32_t b, uint32_t s) {
    uint32_t d;
    asm("prmt.b32 %0, %1, %2, %3;" : "=r"(d) : "r"(a), "r"(b), "r"(s));
    return d;
}
__device__ __forceinline__ uint32_t hmul2(uint32_t a, uint32_t b) {
    uint32_t d;
    asm("mul.rn.f16x2 %0, %1, %2;" : "=r"(d) : "r"(a), "r"(b));
    return d;
}
__device__ __forceinline__ uint32_t hsub2(uint32_t a, uint32_t b) {
    uint32_t d;
    asm("sub.rn.f16x2 %0, %1, %2;" : "=r"(d) : "r"(a), "r"(b));
    return d;
}
// two e4m3 bytes (low byte -> low half) to f16x2, exact
__device__ __forceinline__ uint32_t e4m3x2_f16x2(uint32_t v) {
    uint32_t d;
    asm("{ .reg .b16 t; cvt.u16.u32 t, %1; cvt.rn.f16x2.e4m3x2 %0, t; }" : "=r"(d) : "r"(v));
    return d;
}
__device__ __forceinline__ void mma16816(float* c, uint32_t a0, uint32_t a1, uint32_t a2, uint32_t a3, uint32_t b0, uint32_t b1) {
    asm volatile("mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, {%0,%1,%2,%3};"
                 : "+f"(c[0]), "+f"(c[1]), "+f"(c[2]), "+f"(c[3])
                 : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
}
__device__ __forceinline__ uint4 ldg_stream(const void* p) {
    uint4 v;
    asm volatile("ld.global.nc.L1::no_allocate.v4.u32 {%0,%1,%2,%3}, [%4];" : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w) : "l"(p));
    return v;
}
__device__ __forceinline__ uint2 ldg_stream2(const void* p) {
    uint2 v;
    asm volatile("ld.global.nc.L1::no_allocate.v2.u32 {%0,%1}, [%2];" : "=r"(v.x), "=r"(v.y) : "l"(p));
    return v;
}
__device__ __forceinline__ uint32_t ldg_stream1(const void* p) {
    uint32_t v;
    asm volatile("ld.global.nc.L1::no_allocate.u32 %0, [%1];" : "=r"(v) : "l"(p));
    return v;
}

// ---------------------------------------------------------------------------------------------------------
// layouts ("t16"): rows in tiles of 16; lane (g, t) = (lane / 4, lane % 4) holds the m16n8k16 A fragment
//   a0 = (row g, k 2t..2t+1)  a1 = (row g+8, k 2t..)  a2 = (row g, k 2t+8..)  a3 = (row g+8, k 2t+8..)
// NVFP4: unit (tile, 64-k step s) = 576 B: [32 lanes][4 words] then [8 g][8 B].  Word j of a lane covers k16
//   step j: byte i is a_i, its low element in the low nibble (so one cvt.f16x2.e2m1x2 makes a_i).  The 8 bytes of
//   group g are the e4m3 scales of row g for the step's four 16-blocks, then those of row g+8.
// Q8_0: unit (tile, 32-k block b) = 544 B: [32 lanes][16 B] then [8 g][2 x fp16].  Bytes 8u..8u+7 of a lane are
//   a0, a1, a2, a3 (two int8 each, low k first) of k16 step u; group g's word holds d of row g, then of row g+8.
// ---------------------------------------------------------------------------------------------------------
constexpr int kNv4Unit = 576, kQ8Unit = 544;

// qo / so: a unit's 512 code bytes and 64 scale bytes, units qstride / sstride apart (the t16 unit: out, out + 512,
// both 576; the split form: two planes, 512 and 64)
__global__ void nv4_pack_k(const uint8_t* __restrict__ q, const uint8_t* __restrict__ sc, uint8_t* __restrict__ qo,
                           uint8_t* __restrict__ so, int qstride, int sstride, int n, int k) {
    pdl_wait();
    const int steps = k / 64;
    const int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (i < (int64_t)(n / 16) * steps * 32) {
        const int lane = (int)(i & 31);
        const int64_t unit = i >> 5;
        const int tile = (int)(unit / steps), s = (int)(unit % steps);
        const int g = lane >> 2, t = lane & 3;
        auto nib = [&](int row, int kk) { return (uint32_t)(q[(size_t)row * (k / 2) + kk / 2] >> (4 * (kk & 1))) & 15u; };
        uint32_t w[4];
        for (int j = 0; j < 4; j++) {
            const int k0 = 64 * s + 16 * j + 2 * t;
            const int rr[4] = {16 * tile + g, 16 * tile + g + 8, 16 * tile + g, 16 * tile + g + 8};
            const int kk[4] = {k0, k0, k0 + 8, k0 + 8};
            uint32_t v = 0;
            for (int r = 0; r < 4; r++) v |= (nib(rr[r], kk[r]) | nib(rr[r], kk[r] + 1) << 4) << (8 * r);
            w[j] = v;
        }
        reinterpret_cast<uint4*>(qo + (size_t)unit * qstride)[lane] = make_uint4(w[0], w[1], w[2], w[3]);
        uint8_t* us = so + (size_t)unit * sstride;
        if (t == 0) {
            for (int h = 0; h < 2; h++)
                for (int j = 0; j < 4; j++) us[8 * g + 4 * h + j] = sc[(size_t)(16 * tile + g + 8 * h) * (k / 16) + 4 * s + j];
        }
    }
    pdl_trigger();
}

// qo / so: a unit's 512 int8 bytes and 32 scale bytes, units qstride / sstride apart (t16: out, out + 512, both 544;
// the split form: two planes, 512 and 32)
__global__ void q8_pack_k(const uint8_t* __restrict__ raw, uint8_t* __restrict__ qo, uint8_t* __restrict__ so,
                          int qstride, int sstride, int n, int k) {
    pdl_wait();
    const int nb = k / 32;
    const int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (i < (int64_t)(n / 16) * nb * 32) {
        const int lane = (int)(i & 31);
        const int64_t unit = i >> 5;
        const int tile = (int)(unit / nb), b = (int)(unit % nb);
        const int g = lane >> 2, t = lane & 3;
        auto val = [&](int row, int kk) { return raw[((size_t)row * nb + b) * 34 + 2 + kk]; };
        uint8_t* u = qo + (size_t)unit * qstride;
        uint8_t* us = so + (size_t)unit * sstride;
        for (int uu = 0; uu < 2; uu++) {
            const int k0 = 16 * uu + 2 * t;
            const int rr[4] = {16 * tile + g, 16 * tile + g + 8, 16 * tile + g, 16 * tile + g + 8};
            const int kk[4] = {k0, k0, k0 + 8, k0 + 8};
            for (int r = 0; r < 4; r++) {
                u[16 * lane + 8 * uu + 2 * r] = val(rr[r], kk[r]);
                u[16 * lane + 8 * uu + 2 * r + 1] = val(rr[r], kk[r] + 1);
            }
        }
        if (t == 0) {
            for (int h = 0; h < 2; h++) {
                const uint8_t* blk = raw + ((size_t)(16 * tile + g + 8 * h) * nb + b) * 34;
                us[4 * g + 2 * h] = blk[0];
                us[4 * g + 2 * h + 1] = blk[1];
            }
        }
    }
    pdl_trigger();
}

// ---------------------------------------------------------------------------------------------------------
// the GEMV
// ---------------------------------------------------------------------------------------------------------
constexpr int kTcWarps = 8;

struct TcArgs {
    const uint8_t* w;
    int n, k;
    const void* x;
    int x_dtype, ldx, T;
    int L;          // K slice of a CTA (multiple of 256)
    float s2;       // NVFP4 tensor scale (1 for Q8_0)
    float* out;     // KS == 1: y [T][ldy]; else partials [KS][T][n]
    int ldo;
    const uint8_t* wsc;   // the split layout (libbolt's tile buffers): w holds the units' 512 code bytes, wsc their scales
    float* y;             // KS > 1: the result y [T][ldo], summed from the partials in the launch
    int* cols;            // KS > 1: an arrival count a column of CTAs (blockIdx.x), zero at entry, reset at exit
    int xvec;             // the staging loads x's alignment allows: 2 four values (rows on 4 elements), 1 pairs (rows on
                          // 2 elements), 0 single values
};

// The token rows of the CTA's K slice [k0, k0 + len) as fp16 into shared memory (row stride `stride` halves).  Only
// the `rows` rows that exist are staged: the MMA's output column n reads only B column n, and the columns of the
// absent rows are never stored, so those rows of B need no zeros.  No index needs a division: the four-value form
// walks (row, unit) positions across the CTA's threads, the pair and single-value forms go a row at a time.
__device__ __forceinline__ void stage_rows(const TcArgs& a, __half* xs, int stride, int k0, int len, int rows) {
    const bool bf = a.x_dtype == B200Q_BF16;
    const __nv_bfloat16* xb = reinterpret_cast<const __nv_bfloat16*>(a.x);
    const float* xf = reinterpret_cast<const float*>(a.x);
    if (a.xvec == 2) {
        // (row, four-value unit) positions in row-major order, thread p taking p, p + blockDim, ...: advanced without
        // a division (a row holds len / 4 >= 64 units, so one step crosses at most blockDim / 64 rows), and four loads
        // issued before their stores, so that they are in flight together
        const int nq = len >> 2;
        int r = 0, q = threadIdx.x;
        while (q >= nq) { q -= nq; r++; }
        while (r < rows) {
            int rr[4], qq[4];
            uint4 u[4];
#pragma unroll
            for (int b = 0; b < 4; b++) {
                rr[b] = r;
                qq[b] = q;
                if (r < rows) {
                    const size_t off = (size_t)r * a.ldx + k0 + 4 * q;
                    if (bf) {
                        const uint2 t = *reinterpret_cast<const uint2*>(xb + off);
                        u[b] = make_uint4(t.x, t.y, 0u, 0u);
                    } else {
                        u[b] = *reinterpret_cast<const uint4*>(xf + off);
                    }
                }
                q += blockDim.x;
                while (q >= nq) { q -= nq; r++; }
            }
#pragma unroll
            for (int b = 0; b < 4; b++) {
                if (rr[b] >= rows) break;
                float v[4];
                if (bf) {
                    const float2 f0 = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(&u[b].x));
                    const float2 f1 = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(&u[b].y));
                    v[0] = f0.x; v[1] = f0.y; v[2] = f1.x; v[3] = f1.y;
                } else {
                    v[0] = __uint_as_float(u[b].x); v[1] = __uint_as_float(u[b].y);
                    v[2] = __uint_as_float(u[b].z); v[3] = __uint_as_float(u[b].w);
                }
                const __half2 h0 = __floats2half2_rn(v[0], v[1]), h1 = __floats2half2_rn(v[2], v[3]);
                *reinterpret_cast<uint2*>(xs + (size_t)rr[b] * stride + 4 * qq[b]) =
                    make_uint2(*reinterpret_cast<const uint32_t*>(&h0), *reinterpret_cast<const uint32_t*>(&h1));
            }
        }
        return;
    }
    for (int r = 0; r < rows; r++) {
        const size_t row = (size_t)r * a.ldx + k0;
        __half* dst = xs + (size_t)r * stride;
        if (a.xvec == 1) {
            for (int c2 = threadIdx.x; c2 < len / 2; c2 += blockDim.x) {
                float v0, v1;
                if (bf) {
                    const __nv_bfloat162 b = *reinterpret_cast<const __nv_bfloat162*>(xb + row + 2 * c2);
                    v0 = __low2float(b); v1 = __high2float(b);
                } else {
                    const float2 f = *reinterpret_cast<const float2*>(xf + row + 2 * c2);
                    v0 = f.x; v1 = f.y;
                }
                *reinterpret_cast<__half2*>(dst + 2 * c2) = __floats2half2_rn(v0, v1);
            }
        } else {
            for (int c = threadIdx.x; c < len; c += blockDim.x)
                dst[c] = __float2half_rn(bf ? __bfloat162float(xb[row + c]) : xf[row + c]);
        }
    }
}

// The K split's sum inside the launch: the last CTA of a column to finish adds its rows' partials over the slices in
// slice order and scales by s2 (the arithmetic of a separate sum pass, s = part[0] + part[1] + ...), then resets the
// column's count for the next launch that takes the same counters.
// (No shared memory: a static array beside the launches' dynamic shared memory would cost a CTA an SM.)
__device__ __forceinline__ void tc_fold(const TcArgs& a) {
    __syncthreads();
    int last = 0;
    if (threadIdx.x == 0) {
        __threadfence();
        last = atomicAdd(a.cols + blockIdx.x, 1) == (int)gridDim.y - 1;
        __threadfence();
    }
    if (!__syncthreads_or(last)) return;
    const int r0 = blockIdx.x * kTcWarps * 16, rows = min(kTcWarps * 16, a.n - r0);
    for (int i = threadIdx.x; i < a.T * rows; i += blockDim.x) {
        const int tok = i / rows, row = r0 + (i - tok * rows);
        float s = 0.f;
        for (int ks = 0; ks < (int)gridDim.y; ks++) s += __ldcg(a.out + ((size_t)ks * a.T + tok) * a.n + row);
        a.y[(size_t)tok * a.ldo + row] = s * a.s2;
    }
    if (threadIdx.x == 0) a.cols[blockIdx.x] = 0;
}

enum { kFmtNv4 = 0, kFmtQ8 = 1 };
// units a lane keeps in flight, and the CTAs an SM the K split aims at, per format (measured on B200 over 4 / 8 / 16
// units and 4 / 8 CTAs at config 3's and the GQA projections' shapes, M 1 and 16: tc_gemv_k is fastest for NVFP4 at
// 4 and 4; Q8_0 runs the ring form, two stages at 4 CTAs an SM)
template <int FMT> struct TcTune;
template <> struct TcTune<kFmtNv4> { static constexpr int kPf = 4, kCtasPerSm = 4; };
template <> struct TcTune<kFmtQ8> { static constexpr int kPf = 8, kCtasPerSm = 4; };   // the ring form (below)

// two e2m1 codes (low nibble -> low half) to f16x2, exact (every e2m1 value is an fp16)
__device__ __forceinline__ uint32_t e2m1x2_f16x2(uint32_t v) {
    uint32_t d;
    asm("{ .reg .b8 t; cvt.u8.u32 t, %1; cvt.rn.f16x2.e2m1x2 %0, t; }" : "=r"(d) : "r"(v));
    return d;
}
// the four A fragments of one NVFP4 k16 step from word `w` (byte i = a_i), scaled by (hg, hg8) = the step's scales
// of rows g, g+8
__device__ __forceinline__ void nv4_frag(uint32_t w, uint32_t hg, uint32_t hg8, uint32_t (&a)[4]) {
    a[0] = hmul2(e2m1x2_f16x2(w), hg);
    a[1] = hmul2(e2m1x2_f16x2(w >> 8), hg8);
    a[2] = hmul2(e2m1x2_f16x2(w >> 16), hg);
    a[3] = hmul2(e2m1x2_f16x2(w >> 24), hg8);
}

// int8 pairs -> f16x2 exactly: 1152 + b as fp16 (0x64 high byte, b ^ 0x80 low byte), minus 1152
__device__ __forceinline__ void q8_frag(uint32_t w0, uint32_t w1, uint32_t (&a)[4]) {
    const uint32_t x0 = w0 ^ 0x80808080u, x1 = w1 ^ 0x80808080u;
    const uint32_t bias = 0x64806480u;   // 1152, 1152
    a[0] = hsub2(prmt(x0, 0x64646464u, 0x5140u), bias);
    a[1] = hsub2(prmt(x0, 0x64646464u, 0x7362u), bias);
    a[2] = hsub2(prmt(x1, 0x64646464u, 0x5140u), bias);
    a[3] = hsub2(prmt(x1, 0x64646464u, 0x7362u), bias);
}

template <int FMT, int NT, bool SPLIT, bool FOLD = false>
__global__ void __launch_bounds__(kTcWarps * 32) tc_gemv_k(TcArgs a) {
    pdl_wait();
    extern __shared__ __align__(16) unsigned char dyn[];
    const int L = a.L, stride = L + 8;   // halves a staged row (the padding spreads the B loads over the banks)
    __half* xs = reinterpret_cast<__half*>(dyn);
    const int ks = blockIdx.y, k0 = ks * L, len = min(L, a.k - k0);
    if (NT == 1 && a.xvec > 0) {
        // up to 8 rows on pair boundaries: the single loop over (row, pair) measured faster here than the
        // row-at-a-time form (NVFP4, M = 1: in_proj 2468 against 2336 GB/s, out_proj 1763 against 1527)
        const int srows = min(a.T, 8);
        for (int i = threadIdx.x; i < srows * (len / 2); i += blockDim.x) {
            const int r = i / (len / 2), c = 2 * (i - r * (len / 2));
            const size_t off = (size_t)r * a.ldx + k0 + c;
            float v0, v1;
            if (a.x_dtype == B200Q_BF16) {
                const __nv_bfloat162 b = *reinterpret_cast<const __nv_bfloat162*>(reinterpret_cast<const __nv_bfloat16*>(a.x) + off);
                v0 = __low2float(b); v1 = __high2float(b);
            } else {
                const float2 f = *reinterpret_cast<const float2*>(reinterpret_cast<const float*>(a.x) + off);
                v0 = f.x; v1 = f.y;
            }
            *reinterpret_cast<__half2*>(xs + (size_t)r * stride + c) = __floats2half2_rn(v0, v1);
        }
    } else {
        stage_rows(a, xs, stride, k0, len, min(a.T, NT * 8));
    }
    __syncthreads();
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, g = lane >> 2, t = lane & 3;
    const int tile = blockIdx.x * kTcWarps + warp;
    if (tile * 16 < a.n) {
        float acc[NT][4];
#pragma unroll
        for (int i = 0; i < NT; i++) acc[i][0] = acc[i][1] = acc[i][2] = acc[i][3] = 0.f;
        const __half* xb = xs + (size_t)g * stride + 2 * t;
        auto bfrag = [&](int nt, int kk, uint32_t& b0, uint32_t& b1) {
            const __half* p = xb + (size_t)nt * 8 * stride + kk;
            b0 = *reinterpret_cast<const uint32_t*>(p);
            b1 = *reinterpret_cast<const uint32_t*>(p + 8);
        };
        if constexpr (FMT == kFmtNv4) {
            const int steps = a.k / 64, s0 = k0 / 64, ns = len / 64;
            // a unit's codes and scales: one 576-byte unit, or the two planes of the split layout
            constexpr int QS = SPLIT ? 512 : kNv4Unit, SS = SPLIT ? 64 : kNv4Unit;
            const size_t u0 = (size_t)tile * steps + s0;
            const uint8_t* base = a.w + u0 * QS;
            const uint8_t* sbase = SPLIT ? a.wsc + u0 * SS : base + 512;
            constexpr int PF = TcTune<FMT>::kPf;
            uint4 qb[PF];
            uint2 sb[PF];
#pragma unroll
            for (int i = 0; i < PF; i++) {
                if (i < ns) {
                    qb[i] = ldg_stream(base + (size_t)i * QS + 16 * lane);
                    sb[i] = ldg_stream2(sbase + (size_t)i * SS + 8 * g);
                }
            }
            for (int s = 0; s < ns; s += PF) {
#pragma unroll
                for (int i = 0; i < PF; i++) {
                    if (s + i < ns) {
                        const uint4 q = qb[i];
                        const uint2 sc = sb[i];
                        if (s + i + PF < ns) {
                            qb[i] = ldg_stream(base + (size_t)(s + i + PF) * QS + 16 * lane);
                            sb[i] = ldg_stream2(sbase + (size_t)(s + i + PF) * SS + 8 * g);
                        }
                        // the step's scales: half2 (row g, row g + 8) for blocks 0,1 and 2,3, duplicated per row
                        const uint32_t h01 = e4m3x2_f16x2(prmt(sc.x, sc.y, 0x5140u));   // bytes g.0, g8.0 | g.1, g8.1
                        const uint32_t h23 = e4m3x2_f16x2(prmt(sc.x, sc.y, 0x7362u));
                        const uint32_t h01b = e4m3x2_f16x2(prmt(sc.x, sc.y, 0x5140u) >> 16);
                        const uint32_t h23b = e4m3x2_f16x2(prmt(sc.x, sc.y, 0x7362u) >> 16);
                        const uint32_t hs[4] = {h01, h01b, h23, h23b};   // block j: (row g, row g + 8)
                        const uint32_t words[4] = {q.x, q.y, q.z, q.w};
#pragma unroll
                        for (int j = 0; j < 4; j++) {
                            const uint32_t hg = prmt(hs[j], 0, 0x1010u), hg8 = prmt(hs[j], 0, 0x3232u);
                            uint32_t af[4];
                            nv4_frag(words[j], hg, hg8, af);
                            const int kk = (s + i) * 64 + 16 * j;
#pragma unroll
                            for (int nt = 0; nt < NT; nt++) {
                                uint32_t b0, b1;
                                bfrag(nt, kk, b0, b1);
                                mma16816(acc[nt], af[0], af[1], af[2], af[3], b0, b1);
                            }
                        }
                    }
                }
            }
        } else {
            const int nbk = a.k / 32, b0i = k0 / 32, nblk = len / 32;
            constexpr int QS = SPLIT ? 512 : kQ8Unit, SS = SPLIT ? 32 : kQ8Unit;
            const size_t u0 = (size_t)tile * nbk + b0i;
            const uint8_t* base = a.w + u0 * QS;
            const uint8_t* sbase = SPLIT ? a.wsc + u0 * SS : base + 512;
            constexpr int PF = TcTune<FMT>::kPf;
            uint4 qb[PF];
            uint32_t db[PF];
#pragma unroll
            for (int i = 0; i < PF; i++) {
                if (i < nblk) {
                    qb[i] = ldg_stream(base + (size_t)i * QS + 16 * lane);
                    db[i] = ldg_stream1(sbase + (size_t)i * SS + 4 * g);
                }
            }
            for (int b = 0; b < nblk; b += PF) {
#pragma unroll
                for (int i = 0; i < PF; i++) {
                    if (b + i < nblk) {
                        const uint4 q = qb[i];
                        const uint32_t dd = db[i];
                        if (b + i + PF < nblk) {
                            qb[i] = ldg_stream(base + (size_t)(b + i + PF) * QS + 16 * lane);
                            db[i] = ldg_stream1(sbase + (size_t)(b + i + PF) * SS + 4 * g);
                        }
                        const float dg = __half2float(__ushort_as_half((unsigned short)(dd & 0xffff)));
                        const float dg8 = __half2float(__ushort_as_half((unsigned short)(dd >> 16)));
                        float part[NT][4];
#pragma unroll
                        for (int nt = 0; nt < NT; nt++) part[nt][0] = part[nt][1] = part[nt][2] = part[nt][3] = 0.f;
#pragma unroll
                        for (int u = 0; u < 2; u++) {
                            uint32_t af[4];
                            q8_frag(u ? q.z : q.x, u ? q.w : q.y, af);
                            const int kk = (b + i) * 32 + 16 * u;
#pragma unroll
                            for (int nt = 0; nt < NT; nt++) {
                                uint32_t b0, b1;
                                bfrag(nt, kk, b0, b1);
                                mma16816(part[nt], af[0], af[1], af[2], af[3], b0, b1);
                            }
                        }
#pragma unroll
                        for (int nt = 0; nt < NT; nt++) {
                            acc[nt][0] = fmaf(dg, part[nt][0], acc[nt][0]);
                            acc[nt][1] = fmaf(dg, part[nt][1], acc[nt][1]);
                            acc[nt][2] = fmaf(dg8, part[nt][2], acc[nt][2]);
                            acc[nt][3] = fmaf(dg8, part[nt][3], acc[nt][3]);
                        }
                    }
                }
            }
        }
        // outputs: acc[nt][0..3] = (row g, tok 2t), (row g, tok 2t+1), (row g+8, tok 2t), (row g+8, tok 2t+1)
        const bool partial = gridDim.y > 1;
        const float sc = partial ? 1.f : a.s2;
#pragma unroll
        for (int nt = 0; nt < NT; nt++)
#pragma unroll
            for (int j = 0; j < 4; j++) {
                const int tok = nt * 8 + 2 * t + (j & 1);
                const int row = tile * 16 + g + ((j >> 1) ? 8 : 0);
                if (tok < a.T && row < a.n) {
                    float* o = partial ? a.out + ((size_t)ks * a.T + tok) * a.n + row : a.out + (size_t)tok * a.ldo + row;
                    *o = acc[nt][j] * sc;
                }
            }
    }
    if constexpr (FOLD) tc_fold(a);
    pdl_trigger();
}

// ---------------------------------------------------------------------------------------------------------
// The ring form, used for Q8_0: each warp's units reach shared memory by bulk copies into a ring of kRingStages
// stages of kRingUnits units (one mbarrier a stage, lane 0 refilling a stage once the warp has read it), so a warp
// keeps its slice's units in flight without holding them in registers.  The arithmetic is tc_gemv_k's, unit by unit.
// Measured on B200 against tc_gemv_k (CUDA graphs of 60 calls): Q8_0 q/k/v 6144 x 4096 at 2287 / 1638 GB/s (M 1 / 16)
// with three stages at 3 CTAs an SM against 2118 / 1532, and 2378 / 1690 with two stages at 4; NVFP4 mixed (two
// stages: in_proj M=1 2199 against 2072, M=16 1190 against 1452, out_proj M=1 1424 against 1513), so NVFP4 keeps
// tc_gemv_k.  Every wait is bounded: on a timeout the kernel records bit 0 of g_gemv_error (b200q_device_error bit
// 12), lets its copies in flight land and returns.
// ---------------------------------------------------------------------------------------------------------
constexpr int kRingStages = 2, kRingUnits = 4;
constexpr unsigned long long kRingWaitNs = 2000000000ull;   // a stage not filled within 2 s: give up
__device__ int g_gemv_error;                                // bit 0: a ring wait timed out

__device__ __forceinline__ void ring_init(uint32_t bar) {
    asm volatile("mbarrier.init.shared::cta.b64 [%0], 1;" ::"r"(bar) : "memory");
}
__device__ __forceinline__ void ring_expect(uint32_t bar, uint32_t bytes) {
    asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(bar), "r"(bytes) : "memory");
}
__device__ __forceinline__ bool ring_try(uint32_t bar, uint32_t parity) {
    uint32_t ok;
    asm volatile("{ .reg .pred p; mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2; selp.u32 %0, 1, 0, p; }"
                 : "=r"(ok) : "r"(bar), "r"(parity) : "memory");
    return ok != 0;
}
__device__ __forceinline__ unsigned long long ring_clock() {
    unsigned long long t;
    asm volatile("mov.u64 %0, %globaltimer;" : "=l"(t));
    return t;
}
__device__ __forceinline__ bool ring_wait(uint32_t bar, uint32_t parity) {
    if (ring_try(bar, parity)) return true;
    const unsigned long long t0 = ring_clock();
    while (!ring_try(bar, parity))
        if (ring_clock() - t0 > kRingWaitNs) return false;
    return true;
}
__device__ __forceinline__ void ring_copy(uint32_t dst, const void* src, uint32_t bytes, uint32_t bar) {
    asm volatile("cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];"
                 ::"r"(dst), "l"(src), "r"(bytes), "r"(bar) : "memory");
}
__device__ __forceinline__ uint4 ring_lds128(uint32_t addr) {
    uint4 v;
    asm volatile("ld.shared.v4.u32 {%0,%1,%2,%3}, [%4];" : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w) : "r"(addr));
    return v;
}
__device__ __forceinline__ uint32_t ring_lds32(uint32_t addr) {
    uint32_t v;
    asm volatile("ld.shared.u32 %0, [%1];" : "=r"(v) : "r"(addr));
    return v;
}

template <int FMT>
struct RingGeom {
    static constexpr int kKu = FMT == kFmtNv4 ? 64 : 32;                 // k a unit
    static constexpr int kUb = FMT == kFmtNv4 ? kNv4Unit : kQ8Unit;      // bytes a unit, joined
    static constexpr int kSsz = kUb - 512;                                // its scale bytes
    static constexpr int kStage = kRingUnits * kUb;                       // bytes a stage
};
// dynamic shared memory of a ring launch: barriers, the staged rows, the warps' rings
template <int FMT>
__host__ __device__ inline size_t ring_x_offset() { return 256; }
template <int FMT>
__host__ __device__ inline size_t ring_offset(int rows, int L) {
    return (ring_x_offset<FMT>() + (size_t)rows * (L + 8) * 2 + 127) / 128 * 128;
}
template <int FMT>
__host__ __device__ inline size_t ring_smem(int rows, int L) {
    return ring_offset<FMT>(rows, L) + (size_t)kTcWarps * kRingStages * RingGeom<FMT>::kStage;
}

template <int FMT, int NT, bool SPLIT>
__global__ void __launch_bounds__(kTcWarps * 32) tc_ring_k(TcArgs a) {
    static_assert(FMT == kFmtQ8, "the ring form is the Q8_0 decode GEMV");
    using G = RingGeom<FMT>;
    extern __shared__ __align__(16) unsigned char dyn[];
    const int L = a.L, stride = L + 8;
    const int ks = blockIdx.y, k0 = ks * L, len = min(L, a.k - k0);
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, g = lane >> 2, t = lane & 3;
    const int tile = blockIdx.x * kTcWarps + warp;
    const bool live = tile * 16 < a.n;
    const uint32_t sb0 = (uint32_t)__cvta_generic_to_shared(dyn);
    const uint32_t bar0 = sb0 + 8u * (uint32_t)(warp * kRingStages);
    const uint32_t ring = sb0 + (uint32_t)ring_offset<FMT>(NT * 8, L) + (uint32_t)(warp * kRingStages * G::kStage);
    __half* xs = reinterpret_cast<__half*>(dyn + ring_x_offset<FMT>());
    // the warp's units: nun consecutive units from u0, in stages of kRingUnits
    const int nun = live ? len / G::kKu : 0;
    const int nst = (nun + kRingUnits - 1) / kRingUnits;
    const size_t u0 = (size_t)tile * (a.k / G::kKu) + k0 / G::kKu;
    // smem of unit i of a stage: codes at st + i * CQ, scales at st + SOFF + i * CS
    constexpr int CQ = SPLIT ? 512 : G::kUb, SOFF = SPLIT ? kRingUnits * 512 : 512, CS = SPLIT ? G::kSsz : G::kUb;
    auto issue = [&](int q) {   // stage q of the slice into its ring slot (lane 0)
        const int u = q * kRingUnits, n = min(kRingUnits, nun - u);
        const uint32_t st = ring + (uint32_t)((q % kRingStages) * G::kStage), bar = bar0 + 8u * (uint32_t)(q % kRingStages);
        asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
        ring_expect(bar, (uint32_t)(n * G::kUb));
        if constexpr (SPLIT) {
            ring_copy(st, a.w + (u0 + u) * 512, (uint32_t)(n * 512), bar);
            ring_copy(st + SOFF, a.wsc + (u0 + u) * G::kSsz, (uint32_t)(n * G::kSsz), bar);
        } else {
            ring_copy(st, a.w + (u0 + u) * G::kUb, (uint32_t)(n * G::kUb), bar);
        }
    };
    if (lane == 0 && nst > 0) {
        for (int i = 0; i < kRingStages; i++) ring_init(bar0 + 8u * (uint32_t)i);
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    }
    __syncwarp();
    pdl_wait();
    if (lane == 0)
        for (int q = 0; q < kRingStages && q < nst; q++) issue(q);
    stage_rows(a, xs, stride, k0, len, min(a.T, NT * 8));
    __syncthreads();
    if (nst > 0) {
        float acc[NT][4];
#pragma unroll
        for (int i = 0; i < NT; i++) acc[i][0] = acc[i][1] = acc[i][2] = acc[i][3] = 0.f;
        const __half* xb = xs + (size_t)g * stride + 2 * t;
        auto bfrag = [&](int nt, int kk, uint32_t& b0, uint32_t& b1) {
            const __half* p = xb + (size_t)nt * 8 * stride + kk;
            b0 = *reinterpret_cast<const uint32_t*>(p);
            b1 = *reinterpret_cast<const uint32_t*>(p + 8);
        };
        bool healthy = true;
        int q = 0;
        for (; q < nst; q++) {
            const uint32_t st = ring + (uint32_t)((q % kRingStages) * G::kStage), bar = bar0 + 8u * (uint32_t)(q % kRingStages);
            const bool ok = ring_wait(bar, (uint32_t)((q / kRingStages) & 1));
            if (__any_sync(0xffffffffu, !ok)) {
                healthy = false;
                break;
            }
            const int n = min(kRingUnits, nun - q * kRingUnits);
#pragma unroll 1
            for (int i = 0; i < n; i++) {
                const uint4 qv = ring_lds128(st + (uint32_t)(i * CQ + 16 * lane));
                const int ku = (q * kRingUnits + i) * G::kKu;   // the unit's first k within the slice
                const uint32_t dd = ring_lds32(st + (uint32_t)(SOFF + i * CS + 4 * g));
                const float dg = __half2float(__ushort_as_half((unsigned short)(dd & 0xffff)));
                const float dg8 = __half2float(__ushort_as_half((unsigned short)(dd >> 16)));
                float part[NT][4];
#pragma unroll
                for (int nt = 0; nt < NT; nt++) part[nt][0] = part[nt][1] = part[nt][2] = part[nt][3] = 0.f;
#pragma unroll
                for (int u = 0; u < 2; u++) {
                    uint32_t af[4];
                    q8_frag(u ? qv.z : qv.x, u ? qv.w : qv.y, af);
                    const int kk = ku + 16 * u;
#pragma unroll
                    for (int nt = 0; nt < NT; nt++) {
                        uint32_t b0, b1;
                        bfrag(nt, kk, b0, b1);
                        mma16816(part[nt], af[0], af[1], af[2], af[3], b0, b1);
                    }
                }
#pragma unroll
                for (int nt = 0; nt < NT; nt++) {
                    acc[nt][0] = fmaf(dg, part[nt][0], acc[nt][0]);
                    acc[nt][1] = fmaf(dg, part[nt][1], acc[nt][1]);
                    acc[nt][2] = fmaf(dg8, part[nt][2], acc[nt][2]);
                    acc[nt][3] = fmaf(dg8, part[nt][3], acc[nt][3]);
                }
            }
            __syncwarp();   // every lane is done with the stage: lane 0 refills it
            if (lane == 0 && q + kRingStages < nst) issue(q + kRingStages);
        }
        if (!healthy) {
            // a stage never filled: flag it, and let this warp's copies in flight land before the CTA's memory goes
            if (lane == 0) {
                atomicOr(&g_gemv_error, 1);
                for (int i = q; i < nst && i < q + kRingStages; i++)
                    ring_wait(bar0 + 8u * (uint32_t)(i % kRingStages), (uint32_t)((i / kRingStages) & 1));
            }
            __syncwarp();
        } else {
            const bool partial = gridDim.y > 1;
            const float sc = partial ? 1.f : a.s2;
#pragma unroll
            for (int nt = 0; nt < NT; nt++)
#pragma unroll
                for (int j = 0; j < 4; j++) {
                    const int tok = nt * 8 + 2 * t + (j & 1);
                    const int row = tile * 16 + g + ((j >> 1) ? 8 : 0);
                    if (tok < a.T && row < a.n) {
                        float* o = partial ? a.out + ((size_t)ks * a.T + tok) * a.n + row : a.out + (size_t)tok * a.ldo + row;
                        *o = acc[nt][j] * sc;
                    }
                }
        }
    }
    pdl_trigger();
}

// The ring form over several column tiles a CTA, for 16 token rows: staging 16 rows of a long K slice is a large
// share of a call, and a launch of one CTA a column tile re-staged them in every wave after the first (lm_head at
// M = 16: 1024 column tiles, one K slice).  Each CTA stages its rows once; each warp runs its tiles' units through
// its ring as one sequence.  At one row the single-tile form stays faster (its staging is cheap, and its code
// leaner: lm_head M = 1 5820 against 5423 GB/s).
template <int FMT, int NT, bool SPLIT>
__global__ void __launch_bounds__(kTcWarps * 32, 4) tc_ring_tiles_k(TcArgs a) {
    static_assert(FMT == kFmtQ8 && NT == 2, "the tiled ring form is the Q8_0 decode GEMV at 16 rows");
    using G = RingGeom<FMT>;
    extern __shared__ __align__(16) unsigned char dyn[];
    const int L = a.L, stride = L + 8;
    const int ks = blockIdx.y, k0 = ks * L, len = min(L, a.k - k0);
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, g = lane >> 2, t = lane & 3;
    // the warp's tiles: tile0, tile0 + step, ... (a launch with fewer CTAs than column tiles: each CTA stages its rows
    // of x once for all of its tiles), and their units in this K slice, nun a tile in stages of kRingUnits.  Stage
    // Q of the warp's sequence is stage Q % nst of its tile Q / nst, in ring slot Q % kRingStages.
    const int tile0 = blockIdx.x * kTcWarps + warp, step = gridDim.x * kTcWarps, ntile = (a.n + 15) / 16;
    const int mine = tile0 < ntile ? (ntile - 1 - tile0) / step + 1 : 0;
    const int nun = len / G::kKu;
    const int nst = (nun + kRingUnits - 1) / kRingUnits;
    const int total = mine * nst;
    const uint32_t sb0 = (uint32_t)__cvta_generic_to_shared(dyn);
    const uint32_t bar0 = sb0 + 8u * (uint32_t)(warp * kRingStages);
    const uint32_t ring = sb0 + (uint32_t)ring_offset<FMT>(NT * 8, L) + (uint32_t)(warp * kRingStages * G::kStage);
    __half* xs = reinterpret_cast<__half*>(dyn + ring_x_offset<FMT>());
    // smem of unit i of a stage: codes at st + i * CQ, scales at st + SOFF + i * CS
    constexpr int CQ = SPLIT ? 512 : G::kUb, SOFF = SPLIT ? kRingUnits * 512 : 512, CS = SPLIT ? G::kSsz : G::kUb;
    auto issue = [&](int Q) {   // stage Q of the warp's sequence into its ring slot (lane 0)
        const int j = Q / nst, q = Q - j * nst;
        const size_t u0 = (size_t)(tile0 + j * step) * (a.k / G::kKu) + k0 / G::kKu;
        const int u = q * kRingUnits, n = min(kRingUnits, nun - u);
        const uint32_t st = ring + (uint32_t)((Q % kRingStages) * G::kStage), bar = bar0 + 8u * (uint32_t)(Q % kRingStages);
        asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
        ring_expect(bar, (uint32_t)(n * G::kUb));
        if constexpr (SPLIT) {
            ring_copy(st, a.w + (u0 + u) * 512, (uint32_t)(n * 512), bar);
            ring_copy(st + SOFF, a.wsc + (u0 + u) * G::kSsz, (uint32_t)(n * G::kSsz), bar);
        } else {
            ring_copy(st, a.w + (u0 + u) * G::kUb, (uint32_t)(n * G::kUb), bar);
        }
    };
    if (lane == 0 && total > 0) {
        for (int i = 0; i < kRingStages; i++) ring_init(bar0 + 8u * (uint32_t)i);
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    }
    __syncwarp();
    pdl_wait();
    if (lane == 0)
        for (int Q = 0; Q < kRingStages && Q < total; Q++) issue(Q);
    stage_rows(a, xs, stride, k0, len, min(a.T, NT * 8));
    __syncthreads();
    if (total > 0) {
        const __half* xb = xs + (size_t)g * stride + 2 * t;
        auto bfrag = [&](int nt, int kk, uint32_t& b0, uint32_t& b1) {
            const __half* p = xb + (size_t)nt * 8 * stride + kk;
            b0 = *reinterpret_cast<const uint32_t*>(p);
            b1 = *reinterpret_cast<const uint32_t*>(p + 8);
        };
        const bool partial = gridDim.y > 1;
        const float sc = partial ? 1.f : a.s2;
        bool healthy = true;
        int Q = 0;
        for (int j = 0; j < mine && healthy; j++) {
            const int tile = tile0 + j * step;
            float acc[NT][4];
#pragma unroll
            for (int i = 0; i < NT; i++) acc[i][0] = acc[i][1] = acc[i][2] = acc[i][3] = 0.f;
            for (int q = 0; q < nst; q++, Q++) {
                const uint32_t st = ring + (uint32_t)((Q % kRingStages) * G::kStage), bar = bar0 + 8u * (uint32_t)(Q % kRingStages);
                const bool ok = ring_wait(bar, (uint32_t)((Q / kRingStages) & 1));
                if (__any_sync(0xffffffffu, !ok)) {
                    healthy = false;
                    break;
                }
                const int n = min(kRingUnits, nun - q * kRingUnits);
#pragma unroll 1
                for (int i = 0; i < n; i++) {
                    const uint4 qv = ring_lds128(st + (uint32_t)(i * CQ + 16 * lane));
                    const int ku = (q * kRingUnits + i) * G::kKu;   // the unit's first k within the slice
                    const uint32_t dd = ring_lds32(st + (uint32_t)(SOFF + i * CS + 4 * g));
                    const float dg = __half2float(__ushort_as_half((unsigned short)(dd & 0xffff)));
                    const float dg8 = __half2float(__ushort_as_half((unsigned short)(dd >> 16)));
                    float part[NT][4];
#pragma unroll
                    for (int nt = 0; nt < NT; nt++) part[nt][0] = part[nt][1] = part[nt][2] = part[nt][3] = 0.f;
#pragma unroll
                    for (int u = 0; u < 2; u++) {
                        uint32_t af[4];
                        q8_frag(u ? qv.z : qv.x, u ? qv.w : qv.y, af);
                        const int kk = ku + 16 * u;
#pragma unroll
                        for (int nt = 0; nt < NT; nt++) {
                            uint32_t b0, b1;
                            bfrag(nt, kk, b0, b1);
                            mma16816(part[nt], af[0], af[1], af[2], af[3], b0, b1);
                        }
                    }
#pragma unroll
                    for (int nt = 0; nt < NT; nt++) {
                        acc[nt][0] = fmaf(dg, part[nt][0], acc[nt][0]);
                        acc[nt][1] = fmaf(dg, part[nt][1], acc[nt][1]);
                        acc[nt][2] = fmaf(dg8, part[nt][2], acc[nt][2]);
                        acc[nt][3] = fmaf(dg8, part[nt][3], acc[nt][3]);
                    }
                }
                __syncwarp();   // every lane is done with the stage: lane 0 refills it
                if (lane == 0 && Q + kRingStages < total) issue(Q + kRingStages);
            }
            if (!healthy) break;
#pragma unroll
            for (int nt = 0; nt < NT; nt++)
#pragma unroll
                for (int jj = 0; jj < 4; jj++) {
                    const int tok = nt * 8 + 2 * t + (jj & 1);
                    const int row = tile * 16 + g + ((jj >> 1) ? 8 : 0);
                    if (tok < a.T && row < a.n) {
                        float* o = partial ? a.out + ((size_t)ks * a.T + tok) * a.n + row : a.out + (size_t)tok * a.ldo + row;
                        *o = acc[nt][jj] * sc;
                    }
                }
        }
        if (!healthy) {
            // a stage never filled: flag it, and let this warp's copies in flight land before the CTA's memory goes
            if (lane == 0) {
                atomicOr(&g_gemv_error, 1);
                for (int i = Q; i < total && i < Q + kRingStages; i++)
                    ring_wait(bar0 + 8u * (uint32_t)(i % kRingStages), (uint32_t)((i / kRingStages) & 1));
            }
            __syncwarp();
        }
    }
    pdl_trigger();
}

int gemv_error_read(int clear) {
    int v = 0;
    if (cudaMemcpyFromSymbol(&v, g_gemv_error, sizeof(int)) != cudaSuccess) return -1;
    if (clear) {
        const int z = 0;
        cudaMemcpyToSymbol(g_gemv_error, &z, sizeof(int));
    }
    return v;
}

__global__ void splitk_sum_k(const float* __restrict__ part, int KS, int T, int n, float s2, float* __restrict__ y, int ldy) {
    pdl_wait();
    const int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (i < (int64_t)T * n) {
        const int tok = (int)(i / n), row = (int)(i - (int64_t)tok * n);
        float s = 0.f;
        for (int ks = 0; ks < KS; ks++) s += part[((size_t)ks * T + tok) * n + row];
        y[(size_t)tok * ldy + row] = s * s2;
    }
    pdl_trigger();
}

// the K-split launches' column counts: kTcSlots launch slots taken in turn (so that launches in flight on different
// streams do not share counts), kTcMaxCols columns each; zero at load, every launch leaves its slot's counts at zero
constexpr int kTcSlots = 32, kTcMaxCols = 2048;
__device__ int g_tc_cols[kTcSlots][kTcMaxCols];

static int* tc_cols_slot() {
    static std::mutex mu;
    static int* base[64] = {nullptr};
    static std::atomic<unsigned> next{0};
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return nullptr;
    {
        std::lock_guard<std::mutex> lock(mu);
        if (!base[dev] && cudaGetSymbolAddress((void**)&base[dev], g_tc_cols) != cudaSuccess) {
            cudaGetLastError();
            return nullptr;
        }
    }
    return base[dev] + (size_t)(next.fetch_add(1u) % kTcSlots) * kTcMaxCols;
}

// K slice: about TcTune<FMT>::kCtasPerSm CTAs an SM over the row tiles, slices a multiple of 256
static int slice_len(int fmt, int n, int k) {
    const int ctas_x = (n / 16 + kTcWarps - 1) / kTcWarps;
    const int per_sm = fmt == kFmtNv4 ? TcTune<kFmtNv4>::kCtasPerSm : TcTune<kFmtQ8>::kCtasPerSm;
    const int want = (per_sm * 148 + ctas_x - 1) / ctas_x;
    int L = (k + want - 1) / want;
    L = ((L + 255) / 256) * 256;
    // Q8_0 with enough column tiles for one slice (lm_head): four slices from K = 2048 on, so that a CTA stages a
    // quarter of the rows' length and more CTAs fit an SM (measured on B200, lm_head 131072 x 4096, one / two / four
    // slices: M = 1 5817 / 6213 / 6360 GB/s, M = 16 2886 / 4004 / 4005; the projections with fewer columns already
    // take several slices)
    if (fmt == kFmtQ8 && L >= k && k >= 2048) L = ((k / 4 + 255) / 256) * 256;
    return L > k ? k : L;
}

static size_t splitk_ws(int fmt, int n, int k, int T) {
    const int L = slice_len(fmt, n, k), KS = (k + L - 1) / L;
    return KS > 1 ? (size_t)KS * T * n * sizeof(float) : 0;
}

// dynamic shared memory of a launch over `rows` staged rows (8 or 16) and slices of L
template <int FMT>
static size_t tc_smem(int rows, int L) {
    return FMT == kFmtQ8 ? ring_smem<FMT>(rows, L) : (size_t)rows * (L + 8) * 2;
}
constexpr size_t kMaxSmem = 232448;   // 227 KB, the opt-in limit a CTA

template <int FMT, int NT, bool SPLIT>
static cudaError_t launch_tc(const TcArgs& a, dim3 grid, cudaStream_t s) {
    static size_t opted = 0, opted_fold = 0;
    const size_t smem = tc_smem<FMT>(NT * 8, a.L);
    if constexpr (FMT == kFmtQ8 && NT == 2) {
        // 16 rows: the tiled form where the column tiles outnumber the CTAs resident at once (each CTA stages its rows
        // of x once for all of its tiles), one CTA a column tile where they fit (measured faster there: q/k/v
        // M = 16 2146 against 2117 GB/s)
        void (*tiles)(TcArgs) = tc_ring_tiles_k<FMT, NT, SPLIT>;
        void (*one)(TcArgs) = tc_ring_k<FMT, NT, SPLIT>;
        static size_t opt_tiles = 0, opt_one = 0, cap_smem = 0;
        static int per_sm = 0;
        if (smem > 48 * 1024 && smem > opt_tiles) {
            const cudaError_t e = cudaFuncSetAttribute(tiles, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
            if (e != cudaSuccess) return e;
            opt_tiles = smem;
        }
        if (smem > 48 * 1024 && smem > opt_one) {
            const cudaError_t e = cudaFuncSetAttribute(one, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
            if (e != cudaSuccess) return e;
            opt_one = smem;
        }
        if (cap_smem != smem) {
            int nb = 0;
            if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&nb, tiles, kTcWarps * 32, smem) != cudaSuccess) {
                cudaGetLastError();
                nb = 1;
            }
            per_sm = nb > 0 ? nb : 1;
            cap_smem = smem;
        }
        int dev = 0, sms = 0;
        if (cudaGetDevice(&dev) != cudaSuccess || cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess ||
            sms <= 0)
            sms = 148;
        const unsigned cap = (unsigned)(per_sm * sms) / grid.y;
        if (cap >= 1 && grid.x > cap) {
            grid.x = cap;
            return launch(tiles, grid, dim3(kTcWarps * 32), smem, s, a);
        }
        return launch(one, grid, dim3(kTcWarps * 32), smem, s, a);
    }
    void (*kern)(TcArgs);
    const bool fold = a.cols != nullptr;   // NVFP4 at up to 8 rows: the K split's sum in the launch
    if constexpr (FMT == kFmtQ8) kern = tc_ring_k<FMT, NT, SPLIT>;
    else if constexpr (NT == 1) kern = fold ? tc_gemv_k<FMT, NT, SPLIT, true> : tc_gemv_k<FMT, NT, SPLIT, false>;
    else kern = tc_gemv_k<FMT, NT, SPLIT>;
    if (fold && smem > 48 * 1024 && smem > opted_fold) {
        const cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
        if (e != cudaSuccess) return e;
        opted_fold = smem;
        return launch(kern, grid, dim3(kTcWarps * 32), smem, s, a);
    }
    if (fold) return launch(kern, grid, dim3(kTcWarps * 32), smem, s, a);
    if (smem > 48 * 1024 && smem > opted) {
        const cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
        if (e != cudaSuccess) return e;
        opted = smem;
    }
    return launch(kern, grid, dim3(kTcWarps * 32), smem, s, a);
}

template <int FMT>
static int run_tc(const uint8_t* w, float s2, int n, int k, const void* x, int x_dtype, int ldx, int T, float* y, int ldy,
                  void* ws, size_t ws_bytes, cudaStream_t s, const uint8_t* wsc = nullptr) {
    int L = slice_len(FMT, n, k);
    int KS = (k + L - 1) / L;
    if (KS > 1 && (!ws || ws_bytes < (size_t)KS * T * n * sizeof(float))) { L = k; KS = 1; }   // no workspace: one slice
    if (((uintptr_t)w | (uintptr_t)wsc) & 15) return B200Q_EINVAL;   // the ring's bulk copies start on 16-byte boundaries
    const size_t xe = x_dtype == B200Q_BF16 ? 2 : 4;
    if ((uintptr_t)x % xe) return B200Q_EINVAL;   // x not on its element size
    if (T > 8 && tc_smem<FMT>(16, L) > kMaxSmem) {
        // one slice's 16 staged rows do not fit (a long K without a workspace): two passes of at most 8 rows
        const int st = run_tc<FMT>(w, s2, n, k, x, x_dtype, ldx, 8, y, ldy, ws, ws_bytes, s, wsc);
        if (st != B200Q_OK) return st;
        return run_tc<FMT>(w, s2, n, k, (const char*)x + 8 * (size_t)ldx * xe, x_dtype, ldx, T - 8, y + 8 * (size_t)ldy, ldy,
                           ws, ws_bytes, s, wsc);
    }
    const dim3 grid((n / 16 + kTcWarps - 1) / kTcWarps, KS);
    // the sum in the launch: NVFP4 at up to 8 rows (measured on B200, M = 1: in_proj 2083 against 2062 GB/s, out_proj
    // 1618 against 1511; at M = 16, and for Q8_0 at M = 1 and 16, the second kernel was faster)
    const bool fold = FMT == kFmtNv4 && T <= 8 && KS > 1 && grid.x <= (unsigned)kTcMaxCols;
    int* cols = fold ? tc_cols_slot() : nullptr;
    // the widest staging load x's base and row pitch allow
    const uintptr_t xa = (uintptr_t)x;
    const int xvec = (xa % (4 * xe) == 0 && ldx % 4 == 0) ? 2 : (xa % (2 * xe) == 0 && ldx % 2 == 0) ? 1 : 0;
    TcArgs a{w, n, k, x, x_dtype, ldx, T, L, s2, KS > 1 ? (float*)ws : y, ldy, wsc, y, cols, xvec};
    const dim3 grid2((n / 16 + kTcWarps - 1) / kTcWarps, KS);
    cudaError_t e;
    if (wsc) e = T > 8 ? launch_tc<FMT, 2, true>(a, grid2, s) : launch_tc<FMT, 1, true>(a, grid2, s);
    else e = T > 8 ? launch_tc<FMT, 2, false>(a, grid2, s) : launch_tc<FMT, 1, false>(a, grid2, s);
    if (e != cudaSuccess) return status_from(e);
    if (KS > 1 && !cols) {
        const int64_t tot = (int64_t)T * n;
        e = launch(splitk_sum_k, dim3((unsigned)((tot + 255) / 256)), dim3(256), 0, s, (const float*)ws, KS, T, n, s2, y, ldy);
        if (e != cudaSuccess) return status_from(e);
    }
    return B200Q_OK;
}

static bool tc_shape_ok(int64_t n, int k) { return n > 0 && n % 16 == 0 && k > 0 && k % 256 == 0; }

// the split forms of the t16 layouts, for libbolt's tile buffers (bolt_shim.cu)
cudaError_t launch_nv4_pack_split(const uint8_t* q, const uint8_t* sc, uint8_t* qt, uint8_t* sct, int n, int k,
                                  cudaStream_t s) {
    const int64_t th = (int64_t)(n / 16) * (k / 64) * 32;
    return launch(nv4_pack_k, dim3((unsigned)((th + 255) / 256)), dim3(256), 0, s, q, sc, qt, sct, 512, 64, n, k);
}
cudaError_t launch_q8_pack_split(const uint8_t* raw, uint8_t* qt, uint8_t* dt, int n, int k, cudaStream_t s) {
    const int64_t th = (int64_t)(n / 16) * (k / 32) * 32;
    return launch(q8_pack_k, dim3((unsigned)((th + 255) / 256)), dim3(256), 0, s, raw, qt, dt, 512, 32, n, k);
}
// the decode GEMVs over split planes; ws may be null (one K slice)
int tc_gemv_split(int fmt, const uint8_t* qt, const uint8_t* sct, float s2, int n, int k, const float* x, int ldx, int T,
                  float* y, int ldy, void* ws, size_t ws_bytes, cudaStream_t s) {
    if (!qt || !sct || !x || !y || !tc_shape_ok(n, k) || T <= 0 || T > 16 || ldx < k || ldy < n) return B200Q_EINVAL;
    return fmt == kFmtNv4 ? run_tc<kFmtNv4>(qt, s2, n, k, x, B200Q_F32, ldx, T, y, ldy, ws, ws_bytes, s, sct)
                          : run_tc<kFmtQ8>(qt, 1.f, n, k, x, B200Q_F32, ldx, T, y, ldy, ws, ws_bytes, s, sct);
}
size_t tc_split_ws(int fmt, int n, int k, int T) { return tc_shape_ok(n, k) && T > 0 ? splitk_ws(fmt, n, k, T) : 0; }

}  // namespace b200q

using namespace b200q;

extern "C" {

size_t b200q_nv4_bytes(int64_t n, int k) { return nv4_bytes(n, k); }
size_t b200q_q8_bytes(int64_t n, int k) { return q8_bytes(n, k); }

int b200q_nv4_pack(const void* q, const void* sc, void* packed, int64_t n, int k, void* stream) {
    if (!q || !sc || !packed || !tc_shape_ok(n, k) || n > (1 << 30)) return B200Q_EINVAL;
    const int64_t th = (n / 16) * (k / 64) * 32;
    launch(nv4_pack_k, dim3((unsigned)((th + 255) / 256)), dim3(256), 0, (cudaStream_t)stream, (const uint8_t*)q,
           (const uint8_t*)sc, (uint8_t*)packed, (uint8_t*)packed + 512, kNv4Unit, kNv4Unit, (int)n, k);
    return launched();
}

int b200q_q8_pack(const void* raw, void* packed, int64_t n, int k, void* stream) {
    if (!raw || !packed || !tc_shape_ok(n, k) || n > (1 << 30)) return B200Q_EINVAL;
    const int64_t th = (n / 16) * (k / 32) * 32;
    launch(q8_pack_k, dim3((unsigned)((th + 255) / 256)), dim3(256), 0, (cudaStream_t)stream, (const uint8_t*)raw,
           (uint8_t*)packed, (uint8_t*)packed + 512, kQ8Unit, kQ8Unit, (int)n, k);
    return launched();
}

size_t b200q_nv4_gemv_workspace_bytes(int n, int k, int T) { return tc_split_ws(kFmtNv4, n, k, T); }
size_t b200q_q8_gemv_workspace_bytes(int n, int k, int T) { return tc_split_ws(kFmtQ8, n, k, T); }

int b200q_nv4_gemv(const void* w, float s2, int n, int k, const void* x, int x_dtype, int ldx, int T, float* y, int ldy,
                   void* workspace, size_t workspace_bytes, void* stream) {
    if (!w || !x || !y || !tc_shape_ok(n, k) || T <= 0 || T > 16 || ldx < k || ldy < n ||
        (x_dtype != B200Q_F32 && x_dtype != B200Q_BF16))
        return B200Q_EINVAL;
    return run_tc<kFmtNv4>((const uint8_t*)w, s2, n, k, x, x_dtype, ldx, T, y, ldy, workspace, workspace_bytes, (cudaStream_t)stream);
}

int b200q_q8_gemv(const void* w, int n, int k, const void* x, int x_dtype, int ldx, int T, float* y, int ldy,
                  void* workspace, size_t workspace_bytes, void* stream) {
    if (!w || !x || !y || !tc_shape_ok(n, k) || T <= 0 || T > 16 || ldx < k || ldy < n ||
        (x_dtype != B200Q_F32 && x_dtype != B200Q_BF16))
        return B200Q_EINVAL;
    return run_tc<kFmtQ8>((const uint8_t*)w, 1.f, n, k, x, x_dtype, ldx, T, y, ldy, workspace, workspace_bytes, (cudaStream_t)stream);
}

}  // extern "C"
