// Read-only HBM streaming probes: the read roof the memory-bound kernels are
// measured against (the counterpart of the reference's bandwidth probe op,
// ascend-kernel/csrc/register.cpp:32-33, rebuilt for this GPU's load paths).
//
//   mode 0  plain loads: persistent CTAs of 512 threads, each thread keeps
//           8 independent 16-byte non-caching loads in flight (64 KB per CTA,
//           four CTAs per SM), over one contiguous buffer;
//   mode 1  bulk-copy engine: one thread per CTA streams 32 KB contiguous
//           chunks into a 4-stage shared-memory ring with cp.async.bulk
//           (128 KB in flight per CTA, one CTA per SM);
//   mode 2  the paged KV pattern of the decode kernel without its math: the
//           buffer is viewed as rows of `row_bytes` (kv heads x 256 bytes),
//           and a CTA streams one kv head's 256-byte slice of 64-row tiles
//           with 2-D TMA boxes [64 rows x 64 x 16-bit] (two per 128 dims,
//           128-byte swizzle, L2 evict-first) into a 3-stage ring, two CTAs
//           per SM, work items (kv head, 512 rows) taken in order;
//   mode 3  mode 2 with the items ordered kv head first, so no two CTAs read
//           the same rows at once (the DRAM-locality contrast to mode 2).
// Every probe folds what it reads into one word per CTA (written to `sink`),
// so no load can be dropped. All waits are bounded (ptx.cuh).
#include <cuda_runtime.h>

#include <algorithm>
#include <cstdio>
#include <cstring>

#include "../../include/cascade_b200.h"
#include "kernels.h"
#include "ptx.cuh"

namespace cascade {
namespace {

constexpr int kPlainThreads = 512;
constexpr int kPlainUnroll = 8;

__global__ void __launch_bounds__(kPlainThreads) read_plain_kernel(const uint4* __restrict__ src, size_t n16,
                                                                   uint32_t* sink) {
  uint32_t acc = 0;
  const size_t stride = static_cast<size_t>(gridDim.x) * kPlainThreads;
  size_t i = static_cast<size_t>(blockIdx.x) * kPlainThreads + threadIdx.x;
  for (; i + (kPlainUnroll - 1) * stride < n16; i += kPlainUnroll * stride) {
    uint4 v[kPlainUnroll];
#pragma unroll
    for (int u = 0; u < kPlainUnroll; ++u) {
      const uint4* p = src + i + u * stride;
      asm volatile("ld.global.nc.L1::no_allocate.v4.u32 {%0,%1,%2,%3}, [%4];"
                   : "=r"(v[u].x), "=r"(v[u].y), "=r"(v[u].z), "=r"(v[u].w)
                   : "l"(p));
    }
#pragma unroll
    for (int u = 0; u < kPlainUnroll; ++u) acc ^= v[u].x ^ v[u].y ^ v[u].z ^ v[u].w;
  }
  for (; i < n16; i += stride) {
    const uint4 v = src[i];
    acc ^= v.x ^ v.y ^ v.z ^ v.w;
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) acc ^= __shfl_xor_sync(0xffffffffu, acc, o);
  if ((threadIdx.x & 31) == 0) atomicXor(sink + blockIdx.x, acc);
}

// ---------------------------------------------------------------- mode 1
constexpr int kBulkChunk = 32768;
constexpr int kBulkStages = 4;
constexpr int kBulkSmem = kBulkStages * kBulkChunk + 1024 + 256;

__device__ __forceinline__ void bulk_load_1d(void* dst, const void* src, uint32_t bytes, uint64_t* bar) {
  asm volatile("cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(
                   smem_u32(dst)),
               "l"(src), "r"(bytes), "r"(smem_u32(bar))
               : "memory");
}

__global__ void __launch_bounds__(64, 1) read_bulk_kernel(const uint8_t* __restrict__ src, size_t chunks,
                                                          uint32_t* sink) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + kBulkStages * kBulkChunk);
  uint64_t* empty = full + kBulkStages;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  if (threadIdx.x == 0) {
    for (int s = 0; s < kBulkStages; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    fence_mbar_init();
    cta_wait_init();
  }
  __syncthreads();
  // this CTA's chunks: blockIdx.x, blockIdx.x + gridDim.x, ...
  const size_t mine = chunks > blockIdx.x ? (chunks - blockIdx.x + gridDim.x - 1) / gridDim.x : 0;
  uint32_t acc = 0;
  if (warp == 0) {
    if (lane == 0) {
      size_t it = 0;
      for (; it < mine; ++it) {
        const int st = it % kBulkStages;
        if (it >= kBulkStages) mbar_wait(&empty[st], ((it / kBulkStages) - 1) & 1);
        if (cta_aborted()) break;
        mbar_arrive_expect_tx(&full[st], kBulkChunk);
        bulk_load_1d(smem + st * kBulkChunk, src + (blockIdx.x + it * gridDim.x) * kBulkChunk, kBulkChunk, &full[st]);
      }
      if (cta_aborted())
        for (size_t j = it > kBulkStages ? it - kBulkStages : 0; j < it; ++j)
          mbar_wait_drain(&full[j % kBulkStages], (j / kBulkStages) & 1);
    }
  } else {
    // consumer warp: touch one word per 1 KB of each chunk, then free the slot
    for (size_t it = 0; it < mine; ++it) {
      const int st = it % kBulkStages;
      mbar_wait(&full[st], (it / kBulkStages) & 1);
      acc ^= reinterpret_cast<const uint32_t*>(smem + st * kBulkChunk)[lane * 256];
      __syncwarp();
      if (lane == 0) mbar_arrive(&empty[st]);
    }
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) acc ^= __shfl_xor_sync(0xffffffffu, acc, o);
  if (threadIdx.x == 32) atomicXor(sink + blockIdx.x, acc);
}

// ---------------------------------------------------------------- mode 2
constexpr int kPagedTile = 64;                       // rows per stage
constexpr int kPagedStages = 3;
constexpr int kPagedHalf = kPagedTile * 128;         // [64 rows x 64 x 16-bit]
constexpr int kPagedStage = 2 * kPagedHalf;          // one head's 256 bytes x 64 rows
constexpr int kPagedItemRows = 512;
constexpr int kPagedSmem = kPagedStages * kPagedStage + 1024 + 256;

struct PagedProbe {
  CUtensorMap tmap;      // [rows, heads * 128] 16-bit, box {64, 64}, SW128
  int32_t rows, heads;
  int32_t head_major;    // mode 3: items ordered kv head first (no two CTAs read the same rows at once)
  uint32_t* sink;
};

__global__ void __launch_bounds__(64, 2) read_paged_kernel(const __grid_constant__ PagedProbe p) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + kPagedStages * kPagedStage);
  uint64_t* empty = full + kPagedStages;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  if (threadIdx.x == 0) {
    for (int s = 0; s < kPagedStages; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    fence_mbar_init();
    cta_wait_init();
  }
  __syncthreads();
  const int row_blocks = (p.rows + kPagedItemRows - 1) / kPagedItemRows;
  const int items = row_blocks * p.heads;
  // tiles of this CTA in order: items blockIdx.x, +gridDim.x, ...; within an
  // item, its 512 rows in 64-row tiles
  uint32_t acc = 0;
  if (warp == 0) {
    if (lane == 0) {
      tma_prefetch_desc(&p.tmap);
      const uint64_t pol = policy_evict_first();
      uint32_t it = 0;
      for (int item = blockIdx.x; item < items && !cta_aborted(); item += gridDim.x) {
        const int g = p.head_major ? item / row_blocks : item % p.heads;
        const int r0 = (p.head_major ? item % row_blocks : item / p.heads) * kPagedItemRows;
        const int r1 = min(p.rows, r0 + kPagedItemRows);
        for (int r = r0; r < r1; r += kPagedTile, ++it) {
          const int st = it % kPagedStages;
          if (it >= kPagedStages) mbar_wait(&empty[st], ((it / kPagedStages) - 1) & 1);
          if (cta_aborted()) break;
          mbar_arrive_expect_tx(&full[st], kPagedStage);
          uint8_t* d = smem + st * kPagedStage;
          tma_load_2d_hint(d, &p.tmap, &full[st], g * 128, r, pol);
          tma_load_2d_hint(d + kPagedHalf, &p.tmap, &full[st], g * 128 + 64, r, pol);
        }
      }
      if (cta_aborted())
        for (uint32_t j = it > kPagedStages ? it - kPagedStages : 0; j < it; ++j)
          mbar_wait_drain(&full[j % kPagedStages], (j / kPagedStages) & 1);
    }
  } else {
    uint32_t it = 0;
    for (int item = blockIdx.x; item < items; item += gridDim.x) {
      const int r0 = (p.head_major ? item % row_blocks : item / p.heads) * kPagedItemRows;
      const int r1 = min(p.rows, r0 + kPagedItemRows);
      for (int r = r0; r < r1; r += kPagedTile, ++it) {
        const int st = it % kPagedStages;
        mbar_wait(&full[st], (it / kPagedStages) & 1);
        acc ^= reinterpret_cast<const uint32_t*>(smem + st * kPagedStage)[lane * 128];
        __syncwarp();
        if (lane == 0) mbar_arrive(&empty[st]);
      }
    }
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) acc ^= __shfl_xor_sync(0xffffffffu, acc, o);
  if (threadIdx.x == 32) atomicXor(p.sink + blockIdx.x, acc);
}

}  // namespace
}  // namespace cascade

using namespace cascade;

extern "C" int cascade_probe_hbm_read(const void* src, size_t bytes, int32_t mode, int64_t row_bytes, uint32_t* sink,
                                      size_t sink_words, cascade_stream_t stream) {
  const char* op = "cascade_probe_hbm_read";
  cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
  if (!src || !sink || (reinterpret_cast<uintptr_t>(src) & 255))
    return set_error(CASCADE_ERR_INVALID, "cascade_probe_hbm_read: src (256-byte aligned) and sink required");
  if (sink_words < 2 * kNumSMs * 4)
    return set_error(CASCADE_ERR_INVALID, "cascade_probe_hbm_read: sink needs 4 * 2 * 148 words");
  cudaError_t e = cudaSuccess;
  if (mode == 0) {
    const size_t n16 = bytes / 16;
    read_plain_kernel<<<4 * kNumSMs, kPlainThreads, 0, st>>>(static_cast<const uint4*>(src), n16, sink);
    e = cudaGetLastError();
  } else if (mode == 1) {
    const size_t chunks = bytes / kBulkChunk;
    e = ensure_smem_limit(reinterpret_cast<const void*>(read_bulk_kernel), kBulkSmem);
    if (e == cudaSuccess) {
      read_bulk_kernel<<<kNumSMs, 64, kBulkSmem, st>>>(static_cast<const uint8_t*>(src), chunks, sink);
      e = cudaGetLastError();
    }
  } else if (mode == 2 || mode == 3) {
    if (row_bytes <= 0 || row_bytes % 256 != 0)
      return set_error(CASCADE_ERR_INVALID, "cascade_probe_hbm_read: mode 2 needs row_bytes a multiple of 256");
    PagedProbe p;
    std::memset(&p, 0, sizeof(p));
    p.rows = static_cast<int32_t>(std::min<size_t>(bytes / row_bytes, INT32_MAX));
    p.heads = static_cast<int32_t>(row_bytes / 256);
    p.head_major = mode == 3 ? 1 : 0;
    p.sink = sink;
    if (!encode_tmap_2d(&p.tmap, src, static_cast<uint64_t>(row_bytes / 2), static_cast<uint64_t>(p.rows),
                        static_cast<uint64_t>(row_bytes), 64, kPagedTile, true, CU_TENSOR_MAP_L2_PROMOTION_L2_256B))
      return set_error(CASCADE_ERR_CUDA, "cascade_probe_hbm_read: cuTensorMapEncodeTiled failed");
    e = ensure_smem_limit(reinterpret_cast<const void*>(read_paged_kernel), kPagedSmem);
    if (e == cudaSuccess) {
      read_paged_kernel<<<2 * kNumSMs, 64, kPagedSmem, st>>>(p);
      e = cudaGetLastError();
    }
  } else {
    return set_error(CASCADE_ERR_INVALID, "cascade_probe_hbm_read: mode must be 0, 1, 2 or 3");
  }
  if (e != cudaSuccess) {
    char msg[160];
    snprintf(msg, sizeof(msg), "%s: CUDA error %d (%s)", op, static_cast<int>(e), cudaGetErrorString(e));
    return set_error(CASCADE_ERR_CUDA, msg);
  }
  return CASCADE_OK;
}
