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
// IQ2_XXS device layout ("rt32"): rows in tiles of 32, so that lane l of a warp owns row 32*t + l.  Every
// (row tile t, super-block b of 256 k) is one contiguous unit of 2112 bytes:
//   [4 chunk pairs j][32 lanes][16 B]   lane l's 16 bytes: chunks 2j, 2j+1 of its row in the super-block; each
//                                       chunk is ggml's 8 bytes (4 grid-index bytes, then a u32 of four 7-bit sign
//                                       indices + the 4-bit sub-scale in bits 28-31)
//   [32 lanes] fp16                     the super-block scale d of each row
// Units are ordered t-major: unit (t, b) at (t * k/256 + b) * 2112.  A warp's step over one super-block reads 2112
// contiguous bytes; n*k/256*66 bytes in all, ggml's byte count.  A row tile is self-contained, so a slab of E
// experts of n rows (n % 32 == 0) packed as one matrix of E*n rows has expert e at e * iq2_bytes(n, k).
// ---------------------------------------------------------------------------------------------------------
constexpr int kIq2Tile = 32;
constexpr int kIq2Unit = 2112;   // bytes of a (32-row tile, 256-k super-block) unit
__host__ __device__ inline size_t iq2_bytes(int64_t n, int k) { return (size_t)n * (size_t)(k / 256) * 66; }

// Q8_0 and NVFP4 device layouts ("t16", tiles of 16 rows in the tensor cores' A-fragment order): gemv_tc.cu.
__host__ __device__ inline size_t q8_bytes(int64_t n, int k) { return (size_t)n * (size_t)(k / 32) * 34; }
__host__ __device__ inline size_t nv4_bytes(int64_t n, int k) { return (size_t)n * (size_t)(k / 2) + (size_t)n * (size_t)(k / 16); }

}  // namespace b200q
