// Shared pieces of libb200q: the ggml IQ2_XXS tables, launch plumbing (programmatic dependent launch), status
// codes and the device layouts of the packed weights.
#pragma once
#include <cuda_runtime.h>
#include <cuda_fp16.h>
#include <cuda_bf16.h>
#include <cstdint>
#include <cstddef>

#include "../../include/b200q.h"

// The ggml tables are taken from the reference's own table file by path at build time (B200Q_IQ2_TABLES), never
// re-typed: kmask_iq2xs[8], ksigns_iq2xs[128], ksigns64[128], iq2xxs_grid[256] (engine/iq2_tables.inc:1-117).
#define GGML_TABLE_BEGIN(type, name, size) static __device__ const type name[size] = {
#define GGML_TABLE_END() };
#include B200Q_IQ2_TABLES
#undef GGML_TABLE_BEGIN
#undef GGML_TABLE_END

namespace b200q {

// ---------------------------------------------------------------------------------------------------------
// Programmatic dependent launch: every kernel waits at entry for the writes of the kernel before it on the
// stream (a no-op when launched plainly) and lets the next one be scheduled once its own blocks are done, the
// plumbing of libbolt's launch_pdl / pdl_wait / pdl_trigger (bolt_common.h:84-110).
// ---------------------------------------------------------------------------------------------------------
__device__ __forceinline__ void pdl_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }
__device__ __forceinline__ void pdl_trigger() { asm volatile("griddepcontrol.launch_dependents;" ::: "memory"); }

bool pdl_enabled();

template <typename... KArgs, typename... Args>
inline cudaError_t launch(void (*kern)(KArgs...), dim3 grid, dim3 block, size_t smem, cudaStream_t s, Args... args) {
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = grid;
    cfg.blockDim = block;
    cfg.dynamicSmemBytes = smem;
    cfg.stream = s;
    cudaLaunchAttribute at[1];
    at[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    at[0].val.programmaticStreamSerializationAllowed = pdl_enabled() ? 1 : 0;
    cfg.attrs = at;
    cfg.numAttrs = 1;
    return cudaLaunchKernelEx(&cfg, kern, static_cast<KArgs>(args)...);
}

// Status of the last launch (no synchronisation): B200Q_OK or B200Q_ECUDA, the CUDA error kept for
// b200q_last_cuda_error().
int status_from(cudaError_t e);
inline int launched() { return status_from(cudaGetLastError()); }

// ---------------------------------------------------------------------------------------------------------
// IQ2_XXS device layout ("rt32"): rows in tiles of 32, so that lane l of a warp owns row 32*t + l and one
// 16-byte load of every lane fetches two consecutive 32-weight chunks of each of the warp's 32 rows (512
// contiguous bytes a warp).
//   qs  [n/32][k/64][32][16 B]   lane l's 16 bytes: chunks 2j, 2j+1 of its row; each chunk is ggml's 8 bytes
//                                (4 grid-index bytes, then a u32 of four 7-bit sign indices + the 4-bit sub-scale)
//   d   [n/32][k/256][32] fp16   the super-block scale of each row
// The two planes share one buffer: qs first (n*k/4 bytes), then d (n*k/128 bytes); n*k/256*66 bytes in all, the
// same bytes as ggml's blocks.  A slab of E experts is E such buffers back to back.
// ---------------------------------------------------------------------------------------------------------
constexpr int kIq2Tile = 32;
__host__ __device__ inline size_t iq2_qs_bytes(int64_t n, int k) { return (size_t)n * (size_t)(k / 4); }
__host__ __device__ inline size_t iq2_bytes(int64_t n, int k) { return (size_t)n * (size_t)(k / 256) * 66; }

// Q8_0 device layout ("rt32"): rows in tiles of 32; lane l owns row 32*t + l.
//   q  [n/32][k/32][32][32 B]  the row's 32 int8 of block b
//   d  [n/32][k/32][32] fp16
// n*k/32*34 bytes in all.
__host__ __device__ inline size_t q8_q_bytes(int64_t n, int k) { return (size_t)n * (size_t)k; }
__host__ __device__ inline size_t q8_bytes(int64_t n, int k) { return (size_t)n * (size_t)(k / 32) * 34; }

// NVFP4 device layout ("rt32"): rows in tiles of 32; lane l owns row 32*t + l.
//   q   [n/32][k/32][32][16 B]  32 e2m1 nibbles of the row (element 2j low nibble of byte j)
//   sc  [n/32][k/32][32][2 B]   the two e4m3 scales of those 32 elements
// n*k*9/16 bytes in all; the fp32 tensor scale is an argument.
__host__ __device__ inline size_t nv4_q_bytes(int64_t n, int k) { return (size_t)n * (size_t)(k / 2); }
__host__ __device__ inline size_t nv4_bytes(int64_t n, int k) { return (size_t)n * (size_t)(k / 2) + (size_t)n * (size_t)(k / 16); }

}  // namespace b200q
