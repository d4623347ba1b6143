// Prompt-length GEMMs on the sm_100a tensor cores: tcgen05.mma (kind::f16, fp32 accumulation in TMEM).
//
// C[m][n] = sum_k A[m][k] * B[n][k]: A the activation rows (tokens), B the weight rows, both K-major.  A CTA owns one
// 128 x 256 output tile (tokens x weight rows); its accumulator is 256 TMEM columns.  Eight producer warps fill a
// ring of kStages shared-memory stages: the 128 x 64 fp16 A tile (activation rows converted from bf16 or fp32, or
// gathered for the grouped MoE) and the 256 x 64 fp16 B tile (weights dequantised from their packed format), both in
// the 128-byte-swizzled K-major layout the UMMA descriptors name (8-row atoms of 1024 B, row r's 16-byte chunk c at
// position c ^ (r & 7)).  One thread issues the four m128n256k16 MMAs of a stage and commits them to the stage's
// "empty" barrier; after the last stage a commit to the "done" barrier releases four epilogue warps, which read the
// accumulator with tcgen05.ld (warp w: TMEM lanes 32w..32w+31 = tile rows) and write the outputs.
//
// Numerics: fp16 operands, fp32 accumulation.
//   Q8_0   B = fp16(q * d): the scale folded and rounded once (2^-11), libbolt's PQ8 (bolt_mma.cu:234-254).
//   IQ2    B = fp16(d (0.5 + s4) 0.25 * signed grid): the chunk scale folded and rounded once, libbolt's PIQ2
//          (bolt_mma.cu:380-397) in fp16 instead of bf16.  (FP8 cannot hold the grid magnitudes 25 and 43.)
//   A      activations rounded to fp16 once (exact for bf16 inputs in fp16's normal range).
// Every barrier wait is bounded (%globaltimer); on a timeout the kernel records an error (b200q_device_error), frees
// its TMEM and returns.
#include "tcgen05.cuh"

namespace b200q {

constexpr int kTM = 128, kTN = 256, kTK = 64;
constexpr int kTcStages = 4;
constexpr int kATile = kTM * kTK * 2;           // 16 KB
constexpr int kBTile = kTN * kTK * 2;           // 32 KB
constexpr int kStage = kATile + kBTile;         // 48 KB
constexpr int kProdWarps = 8, kEpiWarps = 4;
constexpr int kTcThreads = (kEpiWarps + 1 + kProdWarps) * 32;   // epilogue warps, the MMA warp, producer warps
constexpr size_t kTcSmem = (size_t)kTcStages * kStage + 1024 /*align*/ + 256 /*barriers*/;

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

// instruction descriptor, kind::f16: fp32 accumulator, fp16 A and B, both K-major, N = 256, M = 128
constexpr uint32_t kIdescF16 = (1u << 4) | (0u << 7) | (0u << 10) | ((uint32_t)(kTN >> 3) << 17) | ((uint32_t)(kTM >> 4) << 24);

__device__ __forceinline__ void umma_f16(uint32_t tmem_d, uint64_t a, uint64_t b, uint32_t accumulate) {
    asm volatile(
        "{ .reg .pred p; setp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, {%5, %6, %7, %8}, p; }"
        ::"r"(tmem_d), "l"(a), "l"(b), "r"(kIdescF16), "r"(accumulate), "r"(0), "r"(0), "r"(0), "r"(0));
}
__device__ __forceinline__ uint32_t h2u(__half2 h) { return *reinterpret_cast<uint32_t*>(&h); }

// ---------------------------------------------------------------------------------------------------------
// operands
// ---------------------------------------------------------------------------------------------------------
struct TcA {                 // activation rows: row m of the tile is source row rows[m] (or m0 + m), K-major
    const void* x;           // [rows][ldx], bf16 (dtype 1), fp32 (0) or fp16 (2)
    int dtype, ldx;
    const int* gather;       // nullptr: row = m0 + m; else row = gather[m0 + m]
    int gather_div;          // row = gather[..] / gather_div (pairs -> tokens)
};

// B producers: fill 8 chunks (64 k) of one weight row into the swizzled tile
struct ProdQ8 {              // Q8_0 "rows" layout: q [n][k] int8 then d [n][k/32] fp16
    const int8_t* q;
    const __half* d;
    int n, k;
    __device__ void row(uint32_t tile, int r, int nrow, int ks) const {
        if (nrow >= n) {
            for (int c = 0; c < 8; c++) sts128(sw128(tile, r, c), make_uint4(0, 0, 0, 0));
            return;
        }
        const uint4* src = reinterpret_cast<const uint4*>(q + (size_t)nrow * k + ks * kTK);
        const __half2 d0 = __half2half2(d[(size_t)nrow * (k >> 5) + ks * 2]);
        const __half2 d1 = __half2half2(d[(size_t)nrow * (k >> 5) + ks * 2 + 1]);
#pragma unroll
        for (int h = 0; h < 4; h++) {
            const uint4 v = __ldg(src + h);   // 16 int8 = two chunks
            const uint32_t w[4] = {v.x, v.y, v.z, v.w};
            const __half2 ds = h < 2 ? d0 : d1;
            uint32_t o[8];
#pragma unroll
            for (int j = 0; j < 4; j++) {
                const int8_t b0 = (int8_t)(w[j] & 255), b1 = (int8_t)((w[j] >> 8) & 255), b2 = (int8_t)((w[j] >> 16) & 255),
                             b3 = (int8_t)(w[j] >> 24);
                o[2 * j] = h2u(__hmul2(__halves2half2(__short2half_rn(b0), __short2half_rn(b1)), ds));
                o[2 * j + 1] = h2u(__hmul2(__halves2half2(__short2half_rn(b2), __short2half_rn(b3)), ds));
            }
            sts128(sw128(tile, r, 2 * h), make_uint4(o[0], o[1], o[2], o[3]));
            sts128(sw128(tile, r, 2 * h + 1), make_uint4(o[4], o[5], o[6], o[7]));
        }
    }
};

struct ProdIQ2 {             // IQ2_XXS rt32 layout (see common.cuh); sign words re-encoded by the packer
    const uint8_t* w;        // the matrix (an expert) [n][k]
    int n, k;
    __device__ void row(uint32_t tile, int r, int nrow, int ks) const {
        if (nrow >= n) {
            for (int c = 0; c < 8; c++) sts128(sw128(tile, r, c), make_uint4(0, 0, 0, 0));
            return;
        }
        const int nb = k >> 8, rt = nrow >> 5, lane = nrow & 31, sb = ks >> 2, j = ks & 3;
        const uint8_t* unit = w + ((size_t)rt * nb + sb) * kIq2Unit;
        const uint4 qv = __ldg(reinterpret_cast<const uint4*>(unit + j * 512 + lane * 16));
        const float d = __half2float(__ushort_as_half(__ldg(reinterpret_cast<const unsigned short*>(unit + 2048) + lane)));
#pragma unroll
        for (int h = 0; h < 2; h++) {
            const uint32_t qx = h ? qv.z : qv.x, qy = h ? qv.w : qv.y;
            const uint32_t s4 = ((qy >> 7) & 1u) | ((qy >> 14) & 2u) | ((qy >> 21) & 4u) | ((qy >> 28) & 8u);
            const float db = d * (0.5f + (float)s4) * 0.25f;
#pragma unroll
            for (int g = 0; g < 4; g++) {
                const unsigned long long gr = iq2xxs_grid[(qx >> (8 * g)) & 255];
                const uint32_t sg = ksigns_iq2xs[(qy >> (8 * g)) & 127];
                float v[8];
#pragma unroll
                for (int e = 0; e < 8; e++) {
                    const float mag = (float)((gr >> (8 * e)) & 255);
                    v[e] = ((sg >> e) & 1) ? -mag * db : mag * db;
                }
                sts128(sw128(tile, r, 4 * h + g),
                       make_uint4(h2u(__floats2half2_rn(v[0], v[1])), h2u(__floats2half2_rn(v[2], v[3])),
                                  h2u(__floats2half2_rn(v[4], v[5])), h2u(__floats2half2_rn(v[6], v[7]))));
            }
        }
    }
};

// epilogues: out[row][col] for the tile's real rows / cols
struct EpiStore {            // fp32 [rows][ldo] (rows scattered by `scatter` when given)
    float* out;
    int ldo;
    const int* scatter;
    float scale;
    __device__ void put(int grow, int col, const float* v, int nv) const {
        const int orow = scatter ? scatter[grow] : grow;
        float* o = out + (size_t)orow * ldo + col;
        for (int i = 0; i < nv; i++) o[i] = v[i] * scale;
    }
};
struct EpiRelu2H {           // relu(v)^2 as fp16 [rows][ldo] (the next GEMM's A)
    __half* out;
    int ldo;
    const int* scatter;
    float scale;
    __device__ void put(int grow, int col, const float* v, int nv) const {
        const int orow = scatter ? scatter[grow] : grow;
        __half* o = out + (size_t)orow * ldo + col;
        for (int i = 0; i < nv; i++) { const float t = v[i] > 0.f ? v[i] * v[i] : 0.f; o[i] = __float2half_rn(t); }
    }
};

// The work of one launch: a list of (group, m-tile) tiles times n-tiles.  Group g has rows [row0[g], row0[g] + cnt[g])
// of the A source list and weight matrix wbase + g * wstride; with groups == nullptr there is one group of M rows.
struct TcGroups {
    const int* counts;       // per group rows (nullptr: one group)
    const int* offsets;      // per group first row
    int ngroups;
    int M;                   // rows of the single group
};

template <class Prod, class Epi>
struct TcArgsT {
    TcA a;
    Prod b;                  // b.w / b.q advanced by g * wstride per group
    size_t wstride;          // bytes (IQ2) between groups' weight matrices
    Epi epi;
    TcGroups grp;
    int N, K;
};

template <class Prod>
__device__ __forceinline__ Prod prod_for_group(const Prod& p, size_t wstride, int g);
template <>
__device__ __forceinline__ ProdQ8 prod_for_group<ProdQ8>(const ProdQ8& p, size_t, int) { return p; }
template <>
__device__ __forceinline__ ProdIQ2 prod_for_group<ProdIQ2>(const ProdIQ2& p, size_t wstride, int g) {
    ProdIQ2 q = p;
    q.w = p.w + (size_t)g * wstride;
    return q;
}

template <class Prod, class Epi>
__global__ void __launch_bounds__(kTcThreads, 1) tc_gemm_k(TcArgsT<Prod, Epi> a) {
    extern __shared__ __align__(1024) unsigned char tc_dyn[];
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const uint32_t raw = (uint32_t)__cvta_generic_to_shared(tc_dyn);
    const uint32_t sbase = (raw + 1023u) & ~1023u;                   // stages, 1024-byte aligned
    const uint32_t bars = sbase + kTcStages * kStage;                // full[s], empty[s], done, tmem slot
    auto full = [&](int s) { return bars + 8u * s; };
    auto empty = [&](int s) { return bars + 8u * (kTcStages + s); };
    const uint32_t done = bars + 8u * (2 * kTcStages);
    const uint32_t tmem_slot = done + 8u;
    unsigned char* tmem_slot_ptr = tc_dyn + (tmem_slot - raw);

    // which tile: blockIdx.x = n-tile, blockIdx.y = tile index over the groups' m-tiles
    const int ntn = (a.N + kTN - 1) / kTN;
    int g = 0, m0 = 0, rows = a.grp.M;
    if (a.grp.counts) {
        pdl_wait();
        int t = blockIdx.y;
        rows = 0;
        for (g = 0; g < a.grp.ngroups; g++) {
            const int c = a.grp.counts[g];
            const int mt = (c + kTM - 1) / kTM;
            if (t < mt) { m0 = t * kTM; rows = c - m0; break; }
            t -= mt;
        }
        if (g >= a.grp.ngroups) { pdl_trigger(); return; }   // past the last tile
    } else {
        m0 = blockIdx.y * kTM;
        rows = a.grp.M - m0;
        if (rows <= 0) return;
    }
    if (rows > kTM) rows = kTM;
    const int row_base = a.grp.counts ? a.grp.offsets[g] + m0 : m0;   // index into the A row list
    const int n0 = (blockIdx.x % ntn) * kTN;
    const Prod prod = prod_for_group(a.b, a.wstride, g);
    const int nk = a.K / kTK;

    if (tid == 0) {
        for (int s = 0; s < kTcStages; s++) { tc_mbar_init(full(s), kProdWarps * 32); tc_mbar_init(empty(s), 1); }
        tc_mbar_init(done, 1);
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    }
    if (warp == 0) {   // the whole warp allocates the accumulator's 256 TMEM columns
        asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(tmem_slot), "r"(kTN));
        asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;");
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = *reinterpret_cast<volatile uint32_t*>(tmem_slot_ptr);
    if (!a.grp.counts) pdl_wait();
    bool healthy = true;

    if (warp >= kEpiWarps + 1) {
        // producers: 256 threads; A: 128 rows x 8 chunks (4 a thread), B: 256 rows (one a thread)
        const int p = tid - (kEpiWarps + 1) * 32;
        for (int i = 0; i < nk && healthy; i++) {
            const int s = i % kTcStages, use = i / kTcStages;
            if (use > 0 && !tc_mbar_wait(empty(s), (uint32_t)((use - 1) & 1))) { healthy = false; break; }
            const uint32_t at = sbase + (uint32_t)(s * kStage), bt = at + kATile;
            for (int q = p; q < kTM * 8; q += kProdWarps * 32) {
                const int r = q >> 3, c = q & 7;
                uint4 v = make_uint4(0, 0, 0, 0);
                if (r < rows) {
                    int src = row_base + r;
                    if (a.a.gather) src = a.a.gather[src] / a.a.gather_div;
                    const size_t off = (size_t)src * a.a.ldx + (size_t)i * kTK + c * 8;
                    if (a.a.dtype == 2) {
                        v = __ldg(reinterpret_cast<const uint4*>(reinterpret_cast<const __half*>(a.a.x) + off));
                    } else if (a.a.dtype == B200Q_BF16) {
                        const uint4 u = __ldg(reinterpret_cast<const uint4*>(reinterpret_cast<const __nv_bfloat16*>(a.a.x) + off));
                        const uint32_t uw[4] = {u.x, u.y, u.z, u.w};
                        uint32_t o[4];
#pragma unroll
                        for (int j = 0; j < 4; j++)
                            o[j] = h2u(__floats2half2_rn(__uint_as_float(uw[j] << 16), __uint_as_float(uw[j] & 0xffff0000u)));
                        v = make_uint4(o[0], o[1], o[2], o[3]);
                    } else {
                        const float4* f = reinterpret_cast<const float4*>(reinterpret_cast<const float*>(a.a.x) + off);
                        const float4 f0 = __ldg(f), f1 = __ldg(f + 1);
                        v = make_uint4(h2u(__floats2half2_rn(f0.x, f0.y)), h2u(__floats2half2_rn(f0.z, f0.w)),
                                       h2u(__floats2half2_rn(f1.x, f1.y)), h2u(__floats2half2_rn(f1.z, f1.w)));
                    }
                }
                sts128(sw128(at, r, c), v);
            }
            prod.row(bt, p, n0 + p, i);
            tc_fence_proxy_async();   // the generic-proxy writes are visible to the tensor core's reads
            tc_mbar_arrive(full(s));
        }
        if (!healthy) atomicOr(&g_tc_error, 1);
    } else if (warp == kEpiWarps) {
        // the MMA issuer
        if (lane == 0) {
            for (int i = 0; i < nk; i++) {
                const int s = i % kTcStages;
                if (!tc_mbar_wait(full(s), (uint32_t)((i / kTcStages) & 1))) { healthy = false; break; }
                tc_fence_after();
                const uint32_t at = sbase + (uint32_t)(s * kStage), bt = at + kATile;
#pragma unroll
                for (int kk = 0; kk < kTK / 16; kk++)
                    umma_f16(tmem, umma_desc_sw128(at + kk * 32), umma_desc_sw128(bt + kk * 32), (i | kk) ? 1u : 0u);
                umma_commit(empty(s));   // the stage is free once these MMAs have read it
            }
            umma_commit(done);           // all MMAs issued so far: the accumulator is final when this arrives
            if (!healthy) atomicOr(&g_tc_error, 1);
        }
        __syncwarp();
    } else {
        // epilogue: warp w reads TMEM lanes 32w.. (tile rows), 32 columns at a time
        if (tc_mbar_wait(done, 0)) {
            tc_fence_after();
            const int r = warp * 32 + lane;
            for (int cb = 0; cb < kTN; cb += 32) {
                uint32_t v[32];
                tmem_ld32(tmem + ((uint32_t)(warp * 32) << 16) + (uint32_t)cb, v);
                tmem_ld_wait();
                const int col = n0 + cb;
                if (r < rows && col < a.N) {
                    float f[32];
#pragma unroll
                    for (int i = 0; i < 32; i++) f[i] = __uint_as_float(v[i]);
                    a.epi.put(row_base + r, col, f, min(32, a.N - col));
                }
            }
        } else {
            if (lane == 0) atomicOr(&g_tc_error, 1);
        }
    }
    tc_fence_before();
    __syncthreads();
    if (warp == 0) {
        tc_fence_after();
        asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(kTN));
    }
    pdl_trigger();
}

template <class Prod, class Epi>
static cudaError_t launch_tc(const TcArgsT<Prod, Epi>& a, int m_tiles, cudaStream_t s) {
    static bool opted = false;
    if (!opted) {
        cudaError_t e = cudaFuncSetAttribute(tc_gemm_k<Prod, Epi>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)kTcSmem);
        if (e != cudaSuccess) return e;
        opted = true;
    }
    const int ntn = (a.N + kTN - 1) / kTN;
    return launch(tc_gemm_k<Prod, Epi>, dim3(ntn, m_tiles), dim3(kTcThreads), kTcSmem, s, a);
}

// ---------------------------------------------------------------------------------------------------------
// Q8_0 "rows" packing for the prompt GEMM: q [n][k] int8, then d [n][k/32] fp16
// ---------------------------------------------------------------------------------------------------------
__global__ void q8_rows_pack_k(const uint8_t* __restrict__ raw, int8_t* __restrict__ q, __half* __restrict__ d, int64_t n, int k) {
    pdl_wait();
    const int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;   // one block of 32
    const int nb = k / 32;
    if (i < n * nb) {
        const uint8_t* blk = raw + (size_t)i * 34;
        d[i] = __ushort_as_half((unsigned short)(blk[0] | blk[1] << 8));
        for (int j = 0; j < 32; j++) q[(size_t)i * 32 + j] = (int8_t)blk[2 + j];
    }
    pdl_trigger();
}

}  // namespace b200q

using namespace b200q;

extern "C" {

size_t b200q_q8_rows_bytes(int64_t n, int k) { return (size_t)n * k + (size_t)n * (k / 32) * 2; }

int b200q_q8_rows_pack(const void* raw, void* packed, int64_t n, int k, void* stream) {
    if (!raw || !packed || n <= 0 || k <= 0 || k % 64 || ((uintptr_t)packed & 15)) return B200Q_EINVAL;
    int8_t* q = (int8_t*)packed;
    __half* d = (__half*)((char*)packed + (size_t)n * k);
    const int64_t th = n * (k / 32);
    launch(q8_rows_pack_k, dim3((unsigned)((th + 255) / 256)), dim3(256), 0, (cudaStream_t)stream, (const uint8_t*)raw, q,
           d, n, k);
    return launched();
}

int b200q_q8_gemm(const void* w, int n, int k, const void* x, int x_dtype, int ldx, int T, float* y, int ldy, void* stream) {
    if (!w || !x || !y || n <= 0 || k <= 0 || k % 64 || T <= 0 || ldx < k || ldy < n ||
        (x_dtype != B200Q_F32 && x_dtype != B200Q_BF16) || ((uintptr_t)w & 15) || ((uintptr_t)x & 15) || (ldx % 8))
        return B200Q_EINVAL;
    TcArgsT<ProdQ8, EpiStore> a{};
    a.a = TcA{x, x_dtype, ldx, nullptr, 1};
    a.b = ProdQ8{(const int8_t*)w, (const __half*)((const char*)w + (size_t)n * k), n, k};
    a.epi = EpiStore{y, ldy, nullptr, 1.f};
    a.grp = TcGroups{nullptr, nullptr, 1, T};
    a.N = n;
    a.K = k;
    return status_from(launch_tc(a, (T + kTM - 1) / kTM, (cudaStream_t)stream));
}

// Grouped IQ2_XXS prompt GEMMs over expert-sorted rows (order from b200q_moe_group_large):
//  up:   act[p][0..n) = relu(W_up[e] . x[p / topk])^2 as fp16, for the pairs p of each expert e
//  down: y[p][0..n) = W_down[e] . act[p] (fp32)
int b200q_moe_up_tc(const void* slab, int E, int n, int k, const int* counts, const int* offsets, const int* order, int topk,
                    const void* x, int x_dtype, void* act_f16, int max_tiles, void* stream) {
    if (!slab || !counts || !offsets || !order || !x || !act_f16 || E <= 0 || E > 512 || topk <= 0 || n % 32 || k % 256 ||
        (x_dtype != B200Q_F32 && x_dtype != B200Q_BF16) || ((uintptr_t)slab & 15) || ((uintptr_t)x & 15) || max_tiles <= 0)
        return B200Q_EINVAL;
    TcArgsT<ProdIQ2, EpiRelu2H> a{};
    a.a = TcA{x, x_dtype, k, order, topk};
    a.b = ProdIQ2{(const uint8_t*)slab, n, k};
    a.wstride = iq2_bytes(n, k);
    a.epi = EpiRelu2H{(__half*)act_f16, n, order, 1.f};
    a.grp = TcGroups{counts, offsets, E, 0};
    a.N = n;
    a.K = k;
    return status_from(launch_tc(a, max_tiles, (cudaStream_t)stream));
}

int b200q_moe_down_tc(const void* slab, int E, int n, int k, const int* counts, const int* offsets, const int* order,
                      const void* act_f16, float* y, int max_tiles, void* stream) {
    if (!slab || !counts || !offsets || !order || !act_f16 || !y || E <= 0 || E > 512 || n % 32 || k % 256 ||
        ((uintptr_t)slab & 15) || ((uintptr_t)act_f16 & 15) || max_tiles <= 0)
        return B200Q_EINVAL;
    TcArgsT<ProdIQ2, EpiStore> a{};
    a.a = TcA{act_f16, 2, k, order, 1};
    a.b = ProdIQ2{(const uint8_t*)slab, n, k};
    a.wstride = iq2_bytes(n, k);
    a.epi = EpiStore{y, n, order, 1.f};
    a.grp = TcGroups{counts, offsets, E, 0};
    a.N = n;
    a.K = k;
    return status_from(launch_tc(a, max_tiles, (cudaStream_t)stream));
}

}  // extern "C"
