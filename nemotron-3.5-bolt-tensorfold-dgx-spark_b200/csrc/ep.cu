// The expert-parallel decode exchange around the local expert GEMVs, in its fixed-capacity layout: the dispatch
// pack (routing table lookup, each pair's place in its destination's block, the token rows and local indices into
// the send buffer) and the return combine (the pairs' outputs gathered back from the return buffer, weighted and
// summed).  Each replaces a chain of small tensor operations with one launch, so that a decode step around the two
// all-to-alls is a handful of kernels.
#include "common.cuh"

namespace b200q {

__device__ __forceinline__ float ld_elem(const void* p, int dtype, size_t i) {
    return dtype == B200Q_BF16 ? __bfloat162float(reinterpret_cast<const __nv_bfloat16*>(p)[i])
                               : reinterpret_cast<const float*>(p)[i];
}
__device__ __forceinline__ void st_elem(void* p, int dtype, size_t i, float v) {
    if (dtype == B200Q_BF16) reinterpret_cast<__nv_bfloat16*>(p)[i] = __float2bfloat16_rn(v);
    else reinterpret_cast<float*>(p)[i] = v;
}

// One CTA a send row j = (destination d, position pos).  The CTA walks the pairs in order, counting those bound for
// d with a block-wide running count, and the pair whose count reaches pos fills the row; a row no pair reaches gets
// the discard index.  pairs <= 1024, so the walk is a few ballots.
__global__ void __launch_bounds__(128) ep_pack_k(const void* __restrict__ x, int xdt, int T, int H,
                                                 const int* __restrict__ ridx, int topk, const int* __restrict__ dest,
                                                 const int* __restrict__ lidx, const int* __restrict__ nrep, int max_rep,
                                                 int cap, int discard, void* __restrict__ send, int sdt, int ldsend,
                                                 int* __restrict__ slot) {
    pdl_wait();
    __shared__ int warp_cnt[4];
    __shared__ int found_p, found_l;
    const int j = blockIdx.x, d = j / cap, pos = j - d * cap;
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    const int pairs = T * topk;
    if (threadIdx.x == 0) found_p = -1;
    __syncthreads();
    int base = 0;
    for (int p0 = 0; p0 < pairs; p0 += 128) {
        const int p = p0 + threadIdx.x;
        int mine = 0, l = 0;
        if (p < pairs) {
            const int e = ridx[p], t = p / topk;
            const int q = e * max_rep + t % nrep[e];
            mine = dest[q] == d;
            l = lidx[q];
        }
        const unsigned b = __ballot_sync(0xffffffffu, mine);
        if (lane == 0) warp_cnt[warp] = __popc(b);
        __syncthreads();
        int before = base, total = 0;
#pragma unroll
        for (int w = 0; w < 4; w++) {
            before += w < warp ? warp_cnt[w] : 0;
            total += warp_cnt[w];
        }
        before += __popc(b & ((1u << lane) - 1u));
        if (mine && before == pos) {
            found_p = p;
            found_l = l;
        }
        base += total;
        __syncthreads();
    }
    const int p = found_p;
    const int elt = sdt == B200Q_BF16 ? 2 : 4;
    unsigned char* row = reinterpret_cast<unsigned char*>(send) + (size_t)j * ldsend * elt;
    if (threadIdx.x == 0) {
        *reinterpret_cast<int*>(row + (size_t)H * elt) = p < 0 ? discard : found_l;
        if (p >= 0) slot[p] = j;
    }
    if (p >= 0) {
        const int t = p / topk;
        for (int h = threadIdx.x; h < H; h += blockDim.x) st_elem(row, sdt, h, ld_elem(x, xdt, (size_t)t * H + h));
    }
    pdl_trigger();
}

// combine_k's arithmetic (bolt_kernels.cu:1714-1727) over the return buffer: k in order, fma, then the shared row
__global__ void ep_combine_k(const void* __restrict__ back, int bdt, int ldb, const int* __restrict__ slot,
                             const float* __restrict__ rw, const float* __restrict__ shared, int T, int topk, int H,
                             void* __restrict__ out, int odt) {
    pdl_wait();
    const int t = blockIdx.y;
    const int h = blockIdx.x * blockDim.x + threadIdx.x;
    if (h < H) {
        float acc = 0.f;
        for (int kk = 0; kk < topk; kk++) {
            const float wk = rw[t * topk + kk];
            acc = fmaf(wk, ld_elem(back, bdt, (size_t)slot[t * topk + kk] * ldb + h), acc);
        }
        if (shared) acc += shared[(size_t)t * H + h];
        st_elem(out, odt, (size_t)t * H + h, acc);
    }
    pdl_trigger();
}

}  // namespace b200q

using namespace b200q;

extern "C" {

int b200q_ep_pack(const void* x, int x_dtype, int T, int H, const int* ridx, int topk, const int* dest,
                  const int* lidx, const int* nrep, int max_rep, int world, int cap, int discard, void* send,
                  int send_dtype, int ldsend, int* slot, void* stream) {
    const int elt = send_dtype == B200Q_BF16 ? 2 : 4;
    if (!x || !ridx || !dest || !lidx || !nrep || !send || !slot || T <= 0 || H <= 0 || topk <= 0 || T * topk > 1024 ||
        max_rep <= 0 || world <= 0 || cap < T * topk || (x_dtype != B200Q_F32 && x_dtype != B200Q_BF16) ||
        (send_dtype != B200Q_F32 && send_dtype != B200Q_BF16) || (size_t)ldsend * elt < (size_t)H * elt + 16 ||
        ((uintptr_t)send & 15) || ((size_t)ldsend * elt) % 16)
        return B200Q_EINVAL;
    launch(ep_pack_k, dim3((unsigned)(world * cap)), dim3(128), 0, (cudaStream_t)stream, x, x_dtype, T, H, ridx, topk,
           dest, lidx, nrep, max_rep, cap, discard, send, send_dtype, ldsend, slot);
    return launched();
}

int b200q_ep_combine(const void* back, int back_dtype, int ldb, const int* slot, const float* rw, const float* shared,
                     int T, int topk, int H, void* out, int out_dtype, void* stream) {
    if (!back || !slot || !rw || !out || T < 0 || topk <= 0 || H <= 0 || ldb < H ||
        (back_dtype != B200Q_F32 && back_dtype != B200Q_BF16) || (out_dtype != B200Q_F32 && out_dtype != B200Q_BF16))
        return B200Q_EINVAL;
    if (T == 0) return B200Q_OK;
    launch(ep_combine_k, dim3((H + 255) / 256, T), dim3(256), 0, (cudaStream_t)stream, back, back_dtype, ldb, slot, rw,
           shared, T, topk, H, out, out_dtype);
    return launched();
}

}  // extern "C"
