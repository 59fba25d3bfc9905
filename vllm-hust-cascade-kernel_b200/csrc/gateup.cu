// gate_up GEMM with the SwiGLU epilogue fused, on tcgen05/TMEM.
//
//   C = X W^T,  X [M, K] bf16, W [2I, K] bf16 (nn.Linear layout: gate rows
//   [0, I), up rows [I, 2I)); mode 1 writes D = silu(C_gate) * C_up in bf16
//   ([M, I]) and never materialises C -- the fusion the reference only hooked
//   (ascend-kernel/csrc/ops/f3_floor/op_kernel/kernel_f3_floor.cpp:276-282,
//   intended chain f3_floor/design.md:107-109). Modes 0/2/4 also write C.
//
// Persistent kernel, one CTA per SM, 6 warps:
//   warp 0    TMA producer: per 64-wide K block, the X tile [128 x 64] (two of
//             them, rows [m0, m0+256), in the 256-row form used for M <= 256) and the
//             paired W tile = gate rows [n0, n0+BN) followed by up rows
//             [I+n0, I+n0+BN) ([2BN x 64]), 128-byte swizzle, 4-stage ring;
//   warp 1    MMA issuer: one tcgen05.mma M=128, N=2*BN, K=16 per K step, so
//             a single TMEM accumulator holds gate (columns [0,BN)) and up
//             (columns [BN,2BN)) of the same output tile; two accumulators
//             (2 x 2BN = 512 columns) let the epilogue of tile t overlap the
//             MMAs of tile t+1;
//   warps 2-5 epilogue: thread = output row = TMEM lane; tcgen05.ld gate and
//             up columns, silu(g) * u in fp32, RNE to bf16, swizzled smem
//             staging, TMA tensor store (rows past M are clipped by TMA).
// Tiles are visited m-fastest so the CTAs in flight share W tiles in L2 and
// X stays L2-resident. No TMA multicast: every CTA loads its own tiles.
#include "kernels.h"
#include "ptx.cuh"

#include <cudaTypedefs.h>

#include <algorithm>
#include <cstring>

namespace cascade {
namespace {

constexpr int kBM = 128;
constexpr int kBK = 64;
constexpr int kStages = 4;
constexpr int kThreads = 6 * 32;

// MT = 128-row halves of X per CTA tile. MT = 1: the M=128 x N=2BN tile, two
// TMEM accumulators (the epilogue of tile t overlaps the MMAs of tile t+1).
// MT = 2: both 128-row halves of a 256-row tile share every W tile load (a
// third less load traffic per FLOP), one accumulator per half, so the
// epilogue of a tile is not overlapped.
template <int BN, int MT = 1>
struct GemmCfg {
  static constexpr int kStagesN = MT == 1 ? kStages : 3;
  static constexpr int kABytes = MT * kBM * kBK * 2;     // 16 KB per half
  static constexpr int kBBytes = 2 * BN * kBK * 2;       // 32 KB for BN=128
  static constexpr int kStageBytes = kABytes + kBBytes;
  static constexpr int kStageOff = 0;
  static constexpr int kStagingOff = kStagesN * kStageBytes;  // [128 rows x BN] bf16, SW128 halves
  static constexpr int kStagingBytes = kBM * BN * 2;
  static constexpr int kBarOff = kStagingOff + kStagingBytes;
  static_assert(kBarOff % 16 == 0, "mbarriers need 8-byte alignment");
  static constexpr int kSmem = kBarOff + 256 + 1024;
  static_assert(kSmem <= 227 * 1024, "shared memory budget");
  static constexpr int kAccSlots = MT == 1 ? 2 : 1;      // accumulator sets in TMEM
  static constexpr uint32_t kTmemCols = 4 * BN;           // 2 x 2BN columns either way
};

struct __align__(8) GemmBars {
  uint64_t full[kStages];   // the MT = 2 form uses the first 3
  uint64_t empty[kStages];
  uint64_t acc_full[2];
  uint64_t acc_empty[2];
  uint64_t drain;           // an aborting MMA issuer's last commit
  uint32_t tmem_base;
};

// Teardown of an aborting CTA's producer: wait (bounded) for the TMA loads of
// the last NS ring positions it issued, [0, issued), one per stage.
template <int NS>
__device__ __forceinline__ void drain_loads(uint64_t* full, int issued) {
  for (int it = issued > NS ? issued - NS : 0; it < issued; ++it) mbar_wait_drain(&full[it % NS], (it / NS) & 1);
}

struct GemmParams {
  CUtensorMap tm_a;   // X [M, K], box {64, 128}
  CUtensorMap tm_b;   // W [2I, K], box {64, BN}
  CUtensorMap tm_d;   // D [M, I] row stride d_stride, box {64, 128}
  CUtensorMap tm_c;   // C [M, 2I], box {64, 128}
  int32_t M, K, I;
  int32_t num_m, num_n, num_kb;
  int32_t mode;
};

__device__ __forceinline__ float silu_mul(float g, float u) {
  // silu(g) = g / (1 + exp(-g)), exp via ex2; 1/(1+e) with an IEEE reciprocal
  const float e = ex2(-g * 1.4426950408889634f);
  return g * __frcp_rn(1.f + e) * u;
}

template <int BN, int MT>
__global__ void __launch_bounds__(kThreads, 1) gateup_kernel(const __grid_constant__ GemmParams p) {
  using C = GemmCfg<BN, MT>;
  constexpr int NS = C::kStagesN;
  constexpr int NA = C::kAccSlots;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  GemmBars* bars = reinterpret_cast<GemmBars*>(smem + C::kBarOff);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int num_tiles = p.num_m * p.num_n;

  if (threadIdx.x == 0) {
    for (int s = 0; s < NS; ++s) {
      mbar_init(&bars->full[s], 1);
      mbar_init(&bars->empty[s], 1);
    }
    for (int a = 0; a < 2; ++a) {
      mbar_init(&bars->acc_full[a], 1);
      mbar_init(&bars->acc_empty[a], 4 * 32);
    }
    mbar_init(&bars->drain, 1);
    fence_mbar_init();
    cta_wait_init();
  }
  if (warp == 1) {
    tmem_alloc(&bars->tmem_base, C::kTmemCols);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tbase = bars->tmem_base;

  if (warp == 0) {
    if (lane == 0) {
      tma_prefetch_desc(&p.tm_a);
      tma_prefetch_desc(&p.tm_b);
      int it = 0;
      for (int tile = blockIdx.x; tile < num_tiles && !cta_aborted(); tile += gridDim.x) {
        const int m0 = (tile % p.num_m) * (MT * kBM);
        const int n0 = (tile / p.num_m) * BN;
        for (int kb = 0; kb < p.num_kb; ++kb, ++it) {
          const int st = it % NS;
          if (it >= NS) mbar_wait(&bars->empty[st], ((it / NS) - 1) & 1);
          if (cta_aborted()) break;
          uint8_t* sa = smem + C::kStageOff + st * C::kStageBytes;
          uint8_t* sb = sa + C::kABytes;
          mbar_arrive_expect_tx(&bars->full[st], C::kStageBytes);
#pragma unroll
          for (int h = 0; h < MT; ++h) tma_load_2d(sa + h * (kBM * kBK * 2), &p.tm_a, &bars->full[st], kb * kBK, m0 + h * kBM);
          tma_load_2d(sb, &p.tm_b, &bars->full[st], kb * kBK, n0);
          tma_load_2d(sb + BN * 128, &p.tm_b, &bars->full[st], kb * kBK, p.I + n0);
        }
      }
      if (cta_aborted()) drain_loads<NS>(bars->full, it);
    }
  } else if (warp == 1) {
    if (lane == 0) {
      const uint32_t idesc = make_idesc_f16(128, 2 * BN, 1, 0, 0);
      const uint32_t sbase = smem_u32(smem + C::kStageOff);
      int it = 0, tc = 0;
      for (int tile = blockIdx.x; tile < num_tiles && !cta_aborted(); tile += gridDim.x, ++tc) {
        const int ab = tc % NA;
        if (tc >= NA) mbar_wait(&bars->acc_empty[ab], ((tc / NA) - 1) & 1);
        tc_fence_after();
        const uint32_t acc = tbase + ab * 2 * BN;   // MT = 2: half h at acc + h * 2BN
        for (int kb = 0; kb < p.num_kb; ++kb, ++it) {
          const int st = it % NS;
          mbar_wait(&bars->full[st], (it / NS) & 1);
          if (cta_aborted()) break;
          tc_fence_after();
          const uint32_t a0 = sbase + st * C::kStageBytes;
          const uint32_t b0 = a0 + C::kABytes;
#pragma unroll
          for (int h = 0; h < MT; ++h) {
#pragma unroll
            for (int k = 0; k < kBK / 16; ++k) {
              umma_f16_ss(acc + h * 2 * BN, make_smem_desc(a0 + h * (kBM * kBK * 2) + k * 32, 16, 1024, 2),
                          make_smem_desc(b0 + k * 32, 16, 1024, 2), idesc, (kb > 0 || k > 0) ? 1u : 0u);
            }
          }
          umma_commit(&bars->empty[st]);
        }
        umma_commit(&bars->acc_full[ab]);
      }
      if (cta_aborted()) {
        umma_commit(&bars->drain);
        mbar_wait_drain(&bars->drain, 0);
      }
    }
  } else {
    // ------------------------------------------------------------ epilogue
    const int q = warp & 3;                 // TMEM lane quarter of this warp
    const int r = q * 32 + lane;            // tile row == TMEM lane
    const uint32_t lane_off = static_cast<uint32_t>(q * 32) << 16;
    const int etid = threadIdx.x - 64;      // 0..127 within the epilogue group
    uint8_t* stg = smem + C::kStagingOff;
    int tc = 0;
    for (int tile = blockIdx.x; tile < num_tiles; tile += gridDim.x, ++tc) {
      const int ab = tc % NA;
      mbar_wait(&bars->acc_full[ab], (tc / NA) & 1);
      tc_fence_after();
      for (int h = 0; h < MT; ++h) {
      const int m0 = (tile % p.num_m) * (MT * kBM) + h * kBM;
      const int n0 = (tile / p.num_m) * BN;
      const uint32_t acc = tbase + lane_off + (ab + h) * 2 * BN;
      // passes: mode 1 -> {silu*up -> D}; mode 2 -> {gate -> C, up -> C};
      // mode 0 -> {gate -> C, up -> C, gate -> D}; mode 4 -> {gate -> C, up -> C, up -> D}
      const int npass = p.mode == 1 ? 1 : (p.mode == 2 ? 2 : 3);
      for (int pass = 0; pass < npass; ++pass) {
        // the staging buffer must be free: previous bulk stores finished reading it
        if (etid == 0) bulk_wait_group_read0();
        asm volatile("bar.sync 1, 128;" ::: "memory");
        const int what = p.mode == 1 ? 2 : (pass < 2 ? pass : (p.mode == 0 ? 0 : 1));  // 0 gate, 1 up, 2 swiglu
#pragma unroll
        for (int c = 0; c < BN / 16; ++c) {
          uint32_t g[16], u[16];
          if (what != 1) tmem_ld_32x32b_x16(acc + c * 16, g);
          if (what != 0) tmem_ld_32x32b_x16(acc + BN + c * 16, u);
          tmem_wait_ld();
          uint32_t pk[8];
#pragma unroll
          for (int e = 0; e < 16; e += 2) {
            float a0, a1;
            if (what == 2) {
              a0 = silu_mul(__uint_as_float(g[e]), __uint_as_float(u[e]));
              a1 = silu_mul(__uint_as_float(g[e + 1]), __uint_as_float(u[e + 1]));
            } else if (what == 0) {
              a0 = __uint_as_float(g[e]);
              a1 = __uint_as_float(g[e + 1]);
            } else {
              a0 = __uint_as_float(u[e]);
              a1 = __uint_as_float(u[e + 1]);
            }
            pk[e >> 1] = pack2<false>(a0, a1);
          }
          // column chunk (16 bytes = 8 outputs) index within the BN-wide tile
#pragma unroll
          for (int h = 0; h < 2; ++h) {
            const int ch = c * 2 + h;
            *reinterpret_cast<uint4*>(stg + (ch >> 3) * (kBM * 128) + sw128(r, ch & 7)) =
                make_uint4(pk[4 * h], pk[4 * h + 1], pk[4 * h + 2], pk[4 * h + 3]);
          }
        }
        if (pass == npass - 1 && h == MT - 1) {
          // all TMEM reads of this accumulator (set) are done: hand it back
          tc_fence_before();
          mbar_arrive(&bars->acc_empty[ab]);
        }
        fence_proxy_async_smem();
        asm volatile("bar.sync 1, 128;" ::: "memory");
        if (etid == 0) {
          const bool to_d = (p.mode == 1) || pass == 2;
#pragma unroll
          for (int h = 0; h < BN / 64; ++h) {
            if (to_d) {
              tma_store_2d(&p.tm_d, stg + h * (kBM * 128), n0 + h * 64, m0);
            } else {
              const int col = (pass == 0 ? 0 : p.I) + n0 + h * 64;
              tma_store_2d(&p.tm_c, stg + h * (kBM * 128), col, m0);
            }
          }
          bulk_commit_group();
        }
      }
      }  // half h
    }
    if (etid == 0) bulk_wait_group0();
  }

  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tbase, C::kTmemCols);
  }
}

// Modes 3/5/7/8: the epilogue's window traffic on an existing workspace.
__global__ void gateup_window_kernel(const uint16_t* __restrict__ ws, uint16_t* __restrict__ d, int64_t d_stride,
                                     int32_t M, int32_t I, int32_t mode) {
  const int64_t chunks = static_cast<int64_t>(M) * (I / 8);
  for (int64_t c = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; c < chunks;
       c += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    const int64_t row = c / (I / 8), col = (c % (I / 8)) * 8;
    if (mode == 7) {
      // read-only rung: volatile loads of both windows, nothing written
      const volatile uint4* gp = reinterpret_cast<const volatile uint4*>(ws + row * 2 * I + col);
      const volatile uint4* up = reinterpret_cast<const volatile uint4*>(ws + row * 2 * I + I + col);
      (void)gp->x;
      (void)up->x;
      continue;
    }
    uint4 g = make_uint4(0, 0, 0, 0);
    if (mode != 8) g = *reinterpret_cast<const uint4*>(ws + row * 2 * I + col);
    *reinterpret_cast<uint4*>(d + row * d_stride + col) = g;
  }
}

bool enc(CUtensorMap* m, const void* base, uint64_t inner, uint64_t rows, uint64_t stride_bytes, uint32_t box_rows) {
  return encode_tmap_2d(m, base, inner, rows, stride_bytes, 64, box_rows, true, CU_TENSOR_MAP_L2_PROMOTION_L2_256B);
}

template <int BN, int MT = 1>
cudaError_t launch_bn(const GateUpLaunch& L, const void* a, const void* b, cudaStream_t stream) {
  using C = GemmCfg<BN, MT>;
  GemmParams p;
  std::memset(&p, 0, sizeof(p));
  p.M = L.M;
  p.K = L.K;
  p.I = L.I;
  p.num_m = (L.M + MT * kBM - 1) / (MT * kBM);
  p.num_n = L.I / BN;
  p.num_kb = (L.K + kBK - 1) / kBK;
  p.mode = L.mode;
  if (!enc(&p.tm_a, a, L.K, L.M, static_cast<uint64_t>(L.K) * 2, kBM)) return cudaErrorInvalidValue;
  if (!enc(&p.tm_b, b, L.K, 2ull * L.I, static_cast<uint64_t>(L.K) * 2, BN)) return cudaErrorInvalidValue;
  if (L.mode != 2) {
    if (!enc(&p.tm_d, L.d, L.I, L.M, static_cast<uint64_t>(L.d_stride) * 2, kBM)) return cudaErrorInvalidValue;
  }
  if (L.mode != 1) {
    if (!enc(&p.tm_c, L.ws, 2ull * L.I, L.M, 4ull * L.I, kBM)) return cudaErrorInvalidValue;
  }
  int dev = 0, sms = kNumSMs;
  cudaGetDevice(&dev);
  cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
  const int tiles = p.num_m * p.num_n;
  const int grid = tiles < sms ? tiles : sms;
  cudaError_t e = ensure_smem_limit(reinterpret_cast<const void*>(gateup_kernel<BN, MT>), C::kSmem);
  if (e != cudaSuccess) return e;
  gateup_kernel<BN, MT><<<grid, kThreads, C::kSmem, stream>>>(p);
  return cudaGetLastError();
}

// ---------------------------------------------------------------------------
// CTA-pair form for SwiGLU over 129..256 rows: a cluster of two CTAs computes
// a 256-row x 2C-column output tile (C = 128 or 112) with
// tcgen05.mma.cta_group::2 (M = 256, N = 2C, issued by rank 0). Per K block
// each CTA loads its own 128 rows of X and 2C rows of W -- rank 0 the gate
// rows [n0, n0+2C), rank 1 the up rows [I+n0, I+n0+2C) -- so one pair
// instruction on the first C of each CTA's W rows yields gate | up of output
// columns [n0, n0+C) for all 256 rows, and a second one on the next C rows
// those of [n0+C, n0+2C). Each CTA holds its 128 rows of both accumulators
// (2 x 2C TMEM columns) and runs the SwiGLU epilogue on them. With C = 128 a
// CTA moves 48 KB per K block for 128 x 512 accumulator outputs, against
// 64 KB for 256 x 256 in the one-CTA 256-row form; C = 112 trades a little of
// that for tile counts that fit the SMs (I = 14336: 128 CTAs instead of 112).
// ---------------------------------------------------------------------------
template <int C>
struct PairCfg {
  static_assert(C == 128 || C == 112, "pair tile: 2 x 128 or 2 x 112 output columns");
  static constexpr int kStages = 4;
  static constexpr int kABytes = kBM * kBK * 2;             // 16 KB: this CTA's X rows
  static constexpr int kBHalf = C * kBK * 2;                // one MMA's W rows of this CTA
  static constexpr int kStageBytes = kABytes + 2 * kBHalf;  // 48 KB (C = 128) / 44 KB (C = 112)
  static constexpr int kStagingOff = kStages * kStageBytes;
  static constexpr int kStagingBytes = kBM * C * 2;         // [128 rows x C cols] bf16
  static constexpr int kBarOff = kStagingOff + kStagingBytes;
  static constexpr int kSmem = kBarOff + 256 + 1024;
  static_assert(kSmem <= 227 * 1024, "shared memory budget");
  static_assert(kBHalf % 1024 == 0, "the second W block starts on a swizzle atom");
};
constexpr int kPairStages = 4;

struct __align__(8) PairBars {
  uint64_t full[kPairStages];   // rank 0's: both CTAs' loads of a stage
  uint64_t empty[kPairStages];  // each CTA's: the pair's MMAs read the stage
  uint64_t acc_full;            // each CTA's: the tile's MMAs are done
  uint64_t acc_empty;           // rank 0's: both CTAs' epilogues read TMEM
  uint64_t drain;               // rank 0's: an aborting MMA issuer's last commit
  uint32_t tmem_base;
};

template <int C>
__global__ void __launch_bounds__(kThreads, 1) gateup_pair_kernel(const __grid_constant__ GemmParams p) {
  using Cfg = PairCfg<C>;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  PairBars* bars = reinterpret_cast<PairBars*>(smem + Cfg::kBarOff);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const uint32_t rank = cluster_cta_rank();
  const int cluster = blockIdx.x >> 1, nclusters = gridDim.x >> 1;
  const int num_tiles = p.num_n;  // 2C-column tiles; M <= 256 is one row tile

  if (threadIdx.x == 0) {
    for (int s = 0; s < kPairStages; ++s) {
      mbar_init(&bars->full[s], 1);
      mbar_init(&bars->empty[s], 1);
    }
    mbar_init(&bars->acc_full, 1);
    mbar_init(&bars->acc_empty, 2);
    mbar_init(&bars->drain, 1);
    fence_mbar_init();
    cta_wait_init();
  }
  if (warp == 1) {
    tmem_alloc_pair(&bars->tmem_base, 512);
    tmem_relinquish_pair();
  }
  tc_fence_before();
  __syncwarp();
  cluster_sync_all();  // barriers and TMEM of both CTAs are ready
  tc_fence_after();
  const uint32_t tbase = bars->tmem_base;

  if (warp == 0) {
    if (lane == 0) {
      tma_prefetch_desc(&p.tm_a);
      tma_prefetch_desc(&p.tm_b);
      int it = 0;
      for (int tile = cluster; tile < num_tiles && !cta_aborted(); tile += nclusters) {
        const int wrow = (rank == 0 ? 0 : p.I) + tile * 2 * C;  // gate rows (rank 0) or up rows (rank 1)
        for (int kb = 0; kb < p.num_kb; ++kb, ++it) {
          const int st = it % kPairStages;
          if (it >= kPairStages) mbar_wait_cluster(&bars->empty[st], ((it / kPairStages) - 1) & 1);
          if (cta_aborted()) break;
          const uint32_t full_l = mapa_shared(smem_u32(&bars->full[st]), 0);
          if (rank == 0) mbar_arrive_expect_tx(&bars->full[st], 2 * Cfg::kStageBytes);
          uint8_t* sa = smem + st * Cfg::kStageBytes;
          uint8_t* sb = sa + Cfg::kABytes;
          tma_load_2d_pair(sa, &p.tm_a, full_l, kb * kBK, static_cast<int>(rank) * kBM);
          tma_load_2d_pair(sb, &p.tm_b, full_l, kb * kBK, wrow);
          tma_load_2d_pair(sb + Cfg::kBHalf, &p.tm_b, full_l, kb * kBK, wrow + C);
        }
      }
      if (cta_aborted()) {
        if (rank == 0) {
          // both CTAs' loads of a stage complete on rank 0's barrier
          for (int i = it > kPairStages ? it - kPairStages : 0; i < it; ++i)
            mbar_wait_cluster_drain(&bars->full[i % kPairStages], (i / kPairStages) & 1);
        } else {
          // rank 1 cannot observe rank 0's barriers: give its own last loads
          // time to land (a TMA copy takes microseconds) before teardown
          const uint64_t t0 = globaltimer_ns();
          while (globaltimer_ns() - t0 < 200000) {
          }
        }
      }
    }
  } else if (warp == 1) {
    if (lane == 0 && rank == 0) {
      const uint32_t idesc = make_idesc_f16(256, 2 * C, 1, 0, 0);
      int it = 0, tc = 0;
      for (int tile = cluster; tile < num_tiles && !cta_aborted(); tile += nclusters, ++tc) {
        if (tc > 0) mbar_wait_cluster(&bars->acc_empty, (tc - 1) & 1);
        tc_fence_after();
        for (int kb = 0; kb < p.num_kb; ++kb, ++it) {
          const int st = it % kPairStages;
          mbar_wait_cluster(&bars->full[st], (it / kPairStages) & 1);
          if (cta_aborted()) break;
          tc_fence_after();
          const uint32_t a0 = smem_u32(smem + st * Cfg::kStageBytes);
          const uint32_t b0 = a0 + Cfg::kABytes;
#pragma unroll
          for (int k = 0; k < kBK / 16; ++k) {
            const uint64_t ad = make_smem_desc(a0 + k * 32, 16, 1024, 2);
            const uint32_t acc = (kb > 0 || k > 0) ? 1u : 0u;
            umma_f16_ss_pair(tbase, ad, make_smem_desc(b0 + k * 32, 16, 1024, 2), idesc, acc);
            umma_f16_ss_pair(tbase + 2 * C, ad, make_smem_desc(b0 + Cfg::kBHalf + k * 32, 16, 1024, 2), idesc, acc);
          }
          umma_commit_pair(&bars->empty[st], 3);
        }
        umma_commit_pair(&bars->acc_full, 3);
      }
      if (cta_aborted()) {
        umma_commit_pair(&bars->drain, 1);
        mbar_wait_cluster_drain(&bars->drain, 0);
      }
    }
  } else {
    // ------------------------------------------------------------ epilogue
    const int q = warp & 3;
    const int r = q * 32 + lane;
    const uint32_t lane_off = static_cast<uint32_t>(q * 32) << 16;
    const int etid = threadIdx.x - 64;
    const uint32_t acc_empty_l = mapa_shared(smem_u32(&bars->acc_empty), 0);
    uint8_t* stg = smem + Cfg::kStagingOff;
    int tc = 0;
    for (int tile = cluster; tile < num_tiles; tile += nclusters, ++tc) {
      mbar_wait_cluster(&bars->acc_full, tc & 1);
      tc_fence_after();
      const int m0 = static_cast<int>(rank) * kBM;
      for (int h = 0; h < 2; ++h) {
        const int n0 = tile * 2 * C + h * C;
        const uint32_t acc = tbase + lane_off + h * 2 * C;
        if (etid == 0) bulk_wait_group_read0();   // the staging buffer's previous stores have read it
        asm volatile("bar.sync 1, 128;" ::: "memory");
#pragma unroll
        for (int c = 0; c < C / 16; ++c) {
          uint32_t g[16], u[16];
          tmem_ld_32x32b_x16(acc + c * 16, g);
          tmem_ld_32x32b_x16(acc + C + c * 16, u);
          tmem_wait_ld();
          uint32_t pk[8];
#pragma unroll
          for (int e = 0; e < 16; e += 2) {
            pk[e >> 1] = pack2<false>(silu_mul(__uint_as_float(g[e]), __uint_as_float(u[e])),
                                      silu_mul(__uint_as_float(g[e + 1]), __uint_as_float(u[e + 1])));
          }
#pragma unroll
          for (int hh = 0; hh < 2; ++hh) {
            const int ch = c * 2 + hh;
            // C = 128: two 64-column SW128 halves; C = 112: plain [128][112] rows
            uint8_t* dst = C == 128 ? stg + (ch >> 3) * (kBM * 128) + sw128(r, ch & 7) : stg + r * (C * 2) + ch * 16;
            *reinterpret_cast<uint4*>(dst) = make_uint4(pk[4 * hh], pk[4 * hh + 1], pk[4 * hh + 2], pk[4 * hh + 3]);
          }
        }
        fence_proxy_async_smem();
        tc_fence_before();
        asm volatile("bar.sync 1, 128;" ::: "memory");
        if (etid == 0) {
          // this CTA's TMEM reads of the tile are done after the second half
          if (h == 1) mbar_arrive_remote(acc_empty_l);
          tma_store_2d(&p.tm_d, stg, n0, m0);
          if (C == 128) tma_store_2d(&p.tm_d, stg + kBM * 128, n0 + 64, m0);
          bulk_commit_group();
        }
      }
    }
    if (etid == 0) bulk_wait_group0();
  }

  tc_fence_before();
  __syncwarp();
  cluster_sync_all();  // no MMA of the pair still writes either CTA's TMEM
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc_pair(tbase, 512);
  }
}

template <int C>
cudaError_t launch_pair(const GateUpLaunch& L, const void* a, const void* b, cudaStream_t stream) {
  using Cfg = PairCfg<C>;
  GemmParams p;
  std::memset(&p, 0, sizeof(p));
  p.M = L.M;
  p.K = L.K;
  p.I = L.I;
  p.num_m = 1;
  p.num_n = L.I / (2 * C);
  p.num_kb = (L.K + kBK - 1) / kBK;
  p.mode = L.mode;
  if (!enc(&p.tm_a, a, L.K, L.M, static_cast<uint64_t>(L.K) * 2, kBM)) return cudaErrorInvalidValue;
  if (!enc(&p.tm_b, b, L.K, 2ull * L.I, static_cast<uint64_t>(L.K) * 2, C)) return cudaErrorInvalidValue;
  // D: C = 128 stores two 64-column SW128 boxes, C = 112 one plain 112-column box
  if (!encode_tmap_2d(&p.tm_d, L.d, L.I, L.M, static_cast<uint64_t>(L.d_stride) * 2, C == 128 ? 64 : C, kBM, C == 128,
                      CU_TENSOR_MAP_L2_PROMOTION_L2_256B))
    return cudaErrorInvalidValue;
  cudaError_t e = ensure_smem_limit(reinterpret_cast<const void*>(gateup_pair_kernel<C>), Cfg::kSmem);
  if (e != cudaSuccess) return e;
  cudaLaunchConfig_t cfg = {};
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = 2;
  attr[0].val.clusterDim.y = 1;
  attr[0].val.clusterDim.z = 1;
  cfg.blockDim = dim3(kThreads);
  cfg.dynamicSmemBytes = Cfg::kSmem;
  cfg.stream = stream;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  // persistent: as many pairs as can be resident at once (per device), at
  // most one per tile
  static int max_clusters[64] = {};  // per C instantiation
  int dev = 0;
  cudaGetDevice(&dev);
  int& mc = max_clusters[dev & 63];
  if (mc == 0) {
    cfg.gridDim = dim3(kNumSMs);
    int n = 0;
    if (cudaOccupancyMaxActiveClusters(&n, reinterpret_cast<const void*>(gateup_pair_kernel<C>), &cfg) !=
            cudaSuccess ||
        n <= 0) {
      cudaGetLastError();
      n = kNumSMs / 2;
    }
    mc = std::min(n, kNumSMs / 2);
  }
  cfg.gridDim = dim3(2 * std::min(p.num_n, mc));
  return cudaLaunchKernelEx(&cfg, gateup_pair_kernel<C>, p);
}

// ---------------------------------------------------------------------------
// Split-K CTA-pair form for SwiGLU over 129..256 rows on narrow shards (few
// 256-column pair tiles: a Llama-3-70B MLP shard over 4 or 8 GPUs has
// I = 7168 / 3584, 28 / 14 tiles). The pair tile already fills TMEM (512
// accumulator columns per CTA), so more tiles per SM would move more operand
// bytes through L2 per FLOP; splitting K instead puts more SMs on each tile at
// the pair tile's traffic per FLOP. A cluster of 2S CTAs = S pairs computes
// one 256 x 256 output tile: pair s (cluster ranks 2s, 2s+1; its leader 2s
// issues the MMAs) accumulates K blocks [s*kb/S, (s+1)*kb/S) exactly as the
// pair form does. The S partial accumulators are reduced through distributed
// shared memory: output columns [s*W, (s+1)*W) of the tile (W = 256 / S)
// belong to pair s; each CTA of another pair reads the gate and up columns of
// that range for its 128 rows from TMEM and stores them into the owner's
// operand ring, free once every pair's MMAs are done (one [128 x 2W] fp32
// slot per sender, in 16-column blocks; each warp transposes its rows through
// a small local buffer so that every remote store instruction writes 512
// contiguous bytes); the owner adds its own columns and the slots in a
// fixed order (its own, then the senders by split index: the result does not
// depend on timing), applies SwiGLU and TMA-stores its [128 x W] bf16 block.
// No global scratch: mode 1 keeps its workspace-free contract. Three cluster
// barriers, taken by every thread of every CTA on every path (an aborted CTA
// included), order the exchange: rings free / slots written / TMEM and peer
// stores done before teardown.
// ---------------------------------------------------------------------------
template <int S>
struct SplitCfg {
  static_assert(S == 2 || S == 4, "K splits per cluster: 2 or 4 (clusters of 4 or 8 CTAs)");
  static constexpr int C = 128;
  static constexpr int W = 2 * C / S;               // output columns one pair reduces
  static constexpr int kRingBytes = PairCfg<C>::kStagingOff;
  // A receive slot holds one sender's gate | up columns of the owner's range
  // for the 128 rows as 2W/16 blocks of [128 rows x 16 fp32] (8 KB each),
  // the 16-byte chunk k of row r stored at chunk k ^ ((r >> 1) & 3): 8
  // consecutive rows of one chunk fall in 8 different bank groups.
  static constexpr int kBlocks = 2 * W / 16;
  static constexpr int kSlotBytes = kBlocks * kBM * 64;
  static constexpr int kSendOff = (S - 1) * kSlotBytes;  // per-warp [32 rows x 16 fp32] transpose buffers
  static constexpr int kSendBytes = 4 * 32 * 64;
  static constexpr int kStgOff = kSendOff + kSendBytes;
  static constexpr int kStgBytes = kBM * W * 2;     // [128 x W] bf16 in 64-column SW128 boxes
  static constexpr int kBarOff = (kStgOff + kStgBytes > kRingBytes ? kStgOff + kStgBytes : kRingBytes);
  static constexpr int kSmem = kBarOff + 256 + 1024;
  static_assert(kStgOff % 1024 == 0, "staging boxes start on a swizzle atom");
  static_assert(kSmem <= 227 * 1024, "shared memory budget");
};

template <int S>
__global__ void __launch_bounds__(kThreads, 1) gateup_pair_split_kernel(const __grid_constant__ GemmParams p) {
  using Cfg = SplitCfg<S>;
  using PC = PairCfg<128>;
  constexpr int C = 128, W = Cfg::W;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  PairBars* bars = reinterpret_cast<PairBars*>(smem + Cfg::kBarOff);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const uint32_t crank = cluster_cta_rank();
  const uint32_t prank = crank & 1u, leader = crank & ~1u;  // role in the pair, the pair's MMA issuer
  const int split = static_cast<int>(crank >> 1);
  const int tile = static_cast<int>(blockIdx.x) / (2 * S);
  const int kb0 = split * p.num_kb / S, kb1 = (split + 1) * p.num_kb / S;
  const uint16_t pair_mask = static_cast<uint16_t>(3u << leader);

  if (threadIdx.x == 0) {
    for (int s = 0; s < kPairStages; ++s) {
      mbar_init(&bars->full[s], 1);
      mbar_init(&bars->empty[s], 1);
    }
    mbar_init(&bars->acc_full, 1);
    mbar_init(&bars->drain, 1);
    fence_mbar_init();
    cta_wait_init();
  }
  if (warp == 1) {
    tmem_alloc_pair(&bars->tmem_base, 512);
    tmem_relinquish_pair();
  }
  tc_fence_before();
  __syncwarp();
  cluster_sync_all();  // barriers and TMEM of every CTA are ready
  tc_fence_after();
  const uint32_t tbase = bars->tmem_base;

  if (warp == 0) {
    if (lane == 0) {
      tma_prefetch_desc(&p.tm_a);
      tma_prefetch_desc(&p.tm_b);
      const int wrow = (prank == 0 ? 0 : p.I) + tile * 2 * C;  // gate rows (even rank) or up rows (odd)
      int it = 0;
      for (int kb = kb0; kb < kb1; ++kb, ++it) {
        const int st = it % kPairStages;
        if (it >= kPairStages) mbar_wait_cluster(&bars->empty[st], ((it / kPairStages) - 1) & 1);
        if (cta_aborted()) break;
        const uint32_t full_l = mapa_shared(smem_u32(&bars->full[st]), leader);
        if (prank == 0) mbar_arrive_expect_tx(&bars->full[st], 2 * PC::kStageBytes);
        uint8_t* sa = smem + st * PC::kStageBytes;
        uint8_t* sb = sa + PC::kABytes;
        tma_load_2d_pair(sa, &p.tm_a, full_l, kb * kBK, static_cast<int>(prank) * kBM);
        tma_load_2d_pair(sb, &p.tm_b, full_l, kb * kBK, wrow);
        tma_load_2d_pair(sb + PC::kBHalf, &p.tm_b, full_l, kb * kBK, wrow + C);
      }
      if (cta_aborted()) {
        if (prank == 0) {
          for (int i = it > kPairStages ? it - kPairStages : 0; i < it; ++i)
            mbar_wait_cluster_drain(&bars->full[i % kPairStages], (i / kPairStages) & 1);
        } else {
          // the odd CTA cannot observe the leader's barriers: give its own
          // last loads time to land before teardown
          const uint64_t t0 = globaltimer_ns();
          while (globaltimer_ns() - t0 < 200000) {
          }
        }
      }
    }
  } else if (warp == 1) {
    if (lane == 0 && prank == 0) {
      const uint32_t idesc = make_idesc_f16(256, 2 * C, 1, 0, 0);
      int it = 0;
      tc_fence_after();
      for (int kb = kb0; kb < kb1; ++kb, ++it) {
        const int st = it % kPairStages;
        mbar_wait_cluster(&bars->full[st], (it / kPairStages) & 1);
        if (cta_aborted()) break;
        tc_fence_after();
        const uint32_t a0 = smem_u32(smem + st * PC::kStageBytes);
        const uint32_t b0 = a0 + PC::kABytes;
#pragma unroll
        for (int k = 0; k < kBK / 16; ++k) {
          const uint64_t ad = make_smem_desc(a0 + k * 32, 16, 1024, 2);
          const uint32_t acc = (kb > kb0 || k > 0) ? 1u : 0u;
          umma_f16_ss_pair(tbase, ad, make_smem_desc(b0 + k * 32, 16, 1024, 2), idesc, acc);
          umma_f16_ss_pair(tbase + 2 * C, ad, make_smem_desc(b0 + PC::kBHalf + k * 32, 16, 1024, 2), idesc, acc);
        }
        umma_commit_pair(&bars->empty[st], pair_mask);
      }
      umma_commit_pair(&bars->acc_full, pair_mask);
      if (cta_aborted()) {
        umma_commit_pair(&bars->drain, static_cast<uint16_t>(1u << leader));
        mbar_wait_cluster_drain(&bars->drain, 0);
      }
    }
  } else {
    mbar_wait_cluster(&bars->acc_full, 0);  // this pair's partial sums are in TMEM
  }

  // ---- exchange: every CTA's ring is free once every pair's MMAs are done
  __syncwarp();
  tc_fence_before();
  cluster_sync_all();
  tc_fence_after();
  const int q = warp & 3;
  const int r = q * 32 + lane;  // this thread's TMEM lane = row of the CTA's 128
  const uint32_t lane_off = static_cast<uint32_t>(q * 32) << 16;
  // Row r's 16-byte chunk k within a [rows x 16 fp32] block (see SplitCfg).
  const uint32_t row_chunk = static_cast<uint32_t>(r) * 64;
  const uint32_t swz = static_cast<uint32_t>((r >> 1) & 3);
  if (warp >= 2) {
    // Each warp moves its 32 rows one 16-column block at a time: TMEM ->
    // registers -> its transpose buffer (local, swizzled) -> 512 contiguous
    // bytes per remote store instruction (a warp-wide store that scatters
    // over 32 rows is about twice as slow through the cluster network).
    uint8_t* xb = smem + Cfg::kSendOff + q * 2048;
    const uint32_t xrow = static_cast<uint32_t>(lane) * 64;
    for (int j = 0; j < S; ++j) {
      if (j == split) continue;
      const int slot = split < j ? split : split - 1;
      const uint32_t dst = mapa_shared(smem_u32(smem + slot * Cfg::kSlotBytes + q * 2048 + lane * 16),
                                       static_cast<uint32_t>(2 * j) + prank);
      const int col0 = j * W;
      const uint32_t gsrc = tbase + lane_off + (col0 / C) * 2 * C + (col0 % C);
#pragma unroll 1
      for (int b = 0; b < Cfg::kBlocks; ++b) {
        // blocks [0, W/16): gate columns; [W/16, 2W/16): the same up columns
        uint32_t v[16];
        tmem_ld_32x32b_x16(gsrc + (b < W / 16 ? b * 16 : C + (b - W / 16) * 16), v);
        tmem_wait_ld();
#pragma unroll
        for (int k = 0; k < 4; ++k)
          *reinterpret_cast<uint4*>(xb + xrow + ((k ^ swz) << 4)) = make_uint4(v[4 * k], v[4 * k + 1], v[4 * k + 2], v[4 * k + 3]);
        __syncwarp();
#pragma unroll
        for (int k = 0; k < 4; ++k) {
          const uint4 w4 = *reinterpret_cast<const uint4*>(xb + k * 512 + lane * 16);
          st_cluster_v4(dst + b * (kBM * 64) + k * 512, w4.x, w4.y, w4.z, w4.w);
        }
        __syncwarp();
      }
    }
  }
  __syncwarp();
  tc_fence_before();
  cluster_sync_all();  // the slots are written (release / acquire)
  tc_fence_after();
  if (warp >= 2) {
    const int etid = threadIdx.x - 64;
    const int col0 = split * W;
    const uint32_t gsrc = tbase + lane_off + (col0 / C) * 2 * C + (col0 % C);
    uint8_t* stg = smem + Cfg::kStgOff;
#pragma unroll 1
    for (int c = 0; c < W / 16; ++c) {
      uint32_t gr[16], ur[16];
      tmem_ld_32x32b_x16(gsrc + c * 16, gr);
      tmem_ld_32x32b_x16(gsrc + C + c * 16, ur);
      tmem_wait_ld();
      float g[16], u[16];
#pragma unroll
      for (int e = 0; e < 16; ++e) {
        g[e] = __uint_as_float(gr[e]);
        u[e] = __uint_as_float(ur[e]);
      }
#pragma unroll
      for (int s = 0; s < S - 1; ++s) {
        const uint8_t* gb = smem + s * Cfg::kSlotBytes + c * (kBM * 64) + row_chunk;
        const uint8_t* ub = gb + (W / 16) * (kBM * 64);
#pragma unroll
        for (int k = 0; k < 4; ++k) {
          const float4 gv = *reinterpret_cast<const float4*>(gb + ((k ^ swz) << 4));
          const float4 uv = *reinterpret_cast<const float4*>(ub + ((k ^ swz) << 4));
          const int e = 4 * k;
          g[e] += gv.x, g[e + 1] += gv.y, g[e + 2] += gv.z, g[e + 3] += gv.w;
          u[e] += uv.x, u[e + 1] += uv.y, u[e + 2] += uv.z, u[e + 3] += uv.w;
        }
      }
      uint32_t pk[8];
#pragma unroll
      for (int e = 0; e < 16; e += 2) pk[e >> 1] = pack2<false>(silu_mul(g[e], u[e]), silu_mul(g[e + 1], u[e + 1]));
#pragma unroll
      for (int hh = 0; hh < 2; ++hh) {
        const int ch = c * 2 + hh;  // 16-byte chunk of the row's W bf16
        *reinterpret_cast<uint4*>(stg + (ch >> 3) * (kBM * 128) + sw128(r, ch & 7)) =
            make_uint4(pk[4 * hh], pk[4 * hh + 1], pk[4 * hh + 2], pk[4 * hh + 3]);
      }
    }
    fence_proxy_async_smem();
    asm volatile("bar.sync 1, 128;" ::: "memory");
    if (etid == 0) {
      const int n0 = tile * 2 * C + col0;
#pragma unroll
      for (int b = 0; b < W / 64; ++b) tma_store_2d(&p.tm_d, stg + b * (kBM * 128), n0 + b * 64, static_cast<int>(prank) * kBM);
      bulk_commit_group();
      bulk_wait_group0();
    }
  }

  tc_fence_before();
  __syncwarp();
  cluster_sync_all();  // no CTA still reads TMEM or stores into a peer's shared memory
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc_pair(tbase, 512);
  }
}

template <int S>
cudaError_t launch_pair_split(const GateUpLaunch& L, const void* a, const void* b, cudaStream_t stream) {
  using Cfg = SplitCfg<S>;
  GemmParams p;
  std::memset(&p, 0, sizeof(p));
  p.M = L.M;
  p.K = L.K;
  p.I = L.I;
  p.num_m = 1;
  p.num_n = L.I / 256;
  p.num_kb = (L.K + kBK - 1) / kBK;
  p.mode = L.mode;
  if (!enc(&p.tm_a, a, L.K, L.M, static_cast<uint64_t>(L.K) * 2, kBM)) return cudaErrorInvalidValue;
  if (!enc(&p.tm_b, b, L.K, 2ull * L.I, static_cast<uint64_t>(L.K) * 2, Cfg::C)) return cudaErrorInvalidValue;
  if (!encode_tmap_2d(&p.tm_d, L.d, L.I, L.M, static_cast<uint64_t>(L.d_stride) * 2, 64, kBM, true,
                      CU_TENSOR_MAP_L2_PROMOTION_L2_256B))
    return cudaErrorInvalidValue;
  cudaError_t e = ensure_smem_limit(reinterpret_cast<const void*>(gateup_pair_split_kernel<S>), Cfg::kSmem);
  if (e != cudaSuccess) return e;
  cudaLaunchConfig_t cfg = {};
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = 2 * S;
  attr[0].val.clusterDim.y = 1;
  attr[0].val.clusterDim.z = 1;
  cfg.gridDim = dim3(2 * S * p.num_n);
  cfg.blockDim = dim3(kThreads);
  cfg.dynamicSmemBytes = Cfg::kSmem;
  cfg.stream = stream;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  return cudaLaunchKernelEx(&cfg, gateup_pair_split_kernel<S>, p);
}

// ---------------------------------------------------------------------------
// Small-M variant (M <= 128, the weight-streaming regime): swap the operands so
// the paired weight tile fills the 128-row MMA side. D^T[128 x MP] =
// W_tile[128 x K] X^T[K x MP], W_tile = gate rows [n0, n0+64) followed by the
// same up rows [I+n0, I+n0+64); MP = M rounded up to 16. One 64-column output
// tile per CTA (I/64 CTAs, two per SM), so every SM streams weights; TMEM
// lanes 0-63 hold gate, 64-127 up; the up half is handed to the gate warps
// through shared memory; D^T is transposed into swizzled smem and TMA-stored
// (rows past M clipped).
// ---------------------------------------------------------------------------
template <int MP>
struct SwapCfg {
  // deep enough to keep ~17 MB of weight tiles in flight over the 224 CTAs of
  // an 8B-sized call, within two CTAs per SM
  static constexpr int kStages = MP <= 32 ? 5 : (MP <= 64 ? 4 : 2);
  static constexpr int kABytes = 128 * kBK * 2;            // W tile: 16 KB
  static constexpr int kBBytes = MP * kBK * 2;             // X tile
  static constexpr int kStageBytes = kABytes + kBBytes;
  static constexpr int kStagingOff = kStages * kStageBytes;  // [MP rows][64 cols] bf16, SW128
  static constexpr int kStagingBytes = MP * 128;
  static constexpr int kXchgOff = kStagingOff + kStagingBytes;  // up values [64][16] fp32
  static constexpr int kXchgBytes = 64 * 16 * 4;
  static constexpr int kBarOff = kXchgOff + kXchgBytes;
  static_assert(kBarOff % 16 == 0, "mbarriers need 8-byte alignment");
  static constexpr int kSmem = kBarOff + 256 + 1024;
  static_assert(2 * (kSmem + 1024) <= 228 * 1024, "two CTAs per SM");
  static_assert(kStages <= 5, "SwapBars holds 5 stages");
  static constexpr uint32_t kTmemCols = MP < 32 ? 32 : MP;
};

struct __align__(8) SwapBars {
  uint64_t full[5];
  uint64_t empty[5];
  uint64_t acc_full;
  uint64_t drain;
  uint32_t tmem_base;
};

template <int MP>
__global__ void __launch_bounds__(kThreads, 2) gateup_swap_kernel(const __grid_constant__ GemmParams p) {
  using C = SwapCfg<MP>;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  SwapBars* bars = reinterpret_cast<SwapBars*>(smem + C::kBarOff);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int n0 = blockIdx.x * 64;

  if (threadIdx.x == 0) {
    for (int s = 0; s < C::kStages; ++s) {
      mbar_init(&bars->full[s], 1);
      mbar_init(&bars->empty[s], 1);
    }
    mbar_init(&bars->acc_full, 1);
    mbar_init(&bars->drain, 1);
    fence_mbar_init();
    cta_wait_init();
  }
  if (warp == 1) {
    tmem_alloc(&bars->tmem_base, C::kTmemCols);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tbase = bars->tmem_base;

  if (warp == 0) {
    if (lane == 0) {
      tma_prefetch_desc(&p.tm_a);
      tma_prefetch_desc(&p.tm_b);
      const uint64_t pol = policy_evict_first();  // weights are streamed once
      int kb = 0;
      for (; kb < p.num_kb; ++kb) {
        const int st = kb % C::kStages;
        if (kb >= C::kStages) mbar_wait(&bars->empty[st], ((kb / C::kStages) - 1) & 1);
        if (cta_aborted()) break;
        uint8_t* sa = smem + st * C::kStageBytes;
        uint8_t* sb = sa + C::kABytes;
        mbar_arrive_expect_tx(&bars->full[st], C::kStageBytes);
        tma_load_2d_hint(sa, &p.tm_b, &bars->full[st], kb * kBK, n0, pol);               // gate rows
        tma_load_2d_hint(sa + 64 * 128, &p.tm_b, &bars->full[st], kb * kBK, p.I + n0, pol);  // up rows
        tma_load_2d(sb, &p.tm_a, &bars->full[st], kb * kBK, 0);                           // X rows
      }
      if (cta_aborted()) drain_loads<C::kStages>(bars->full, kb);
    }
  } else if (warp == 1) {
    if (lane == 0) {
      const uint32_t idesc = make_idesc_f16(128, MP, 1, 0, 0);
      const uint32_t sbase = smem_u32(smem);
      for (int kb = 0; kb < p.num_kb; ++kb) {
        const int st = kb % C::kStages;
        mbar_wait(&bars->full[st], (kb / C::kStages) & 1);
        if (cta_aborted()) break;
        tc_fence_after();
        const uint32_t a0 = sbase + st * C::kStageBytes;
        const uint32_t b0 = a0 + C::kABytes;
#pragma unroll
        for (int k = 0; k < kBK / 16; ++k) {
          umma_f16_ss(tbase, make_smem_desc(a0 + k * 32, 16, 1024, 2), make_smem_desc(b0 + k * 32, 16, 1024, 2),
                      idesc, (kb > 0 || k > 0) ? 1u : 0u);
        }
        umma_commit(&bars->empty[st]);
      }
      umma_commit(&bars->acc_full);
      if (cta_aborted()) {
        umma_commit(&bars->drain);
        mbar_wait_drain(&bars->drain, 0);
      }
    }
  } else {
    // epilogue warps 2-5: TMEM lane quarter q = warp & 3 (2,3 -> up rows; 0,1 -> gate rows)
    const int q = warp & 3;
    const int r = q * 32 + lane;
    const uint32_t lane_off = static_cast<uint32_t>(q * 32) << 16;
    const int etid = threadIdx.x - 64;
    float* xchg = reinterpret_cast<float*>(smem + C::kXchgOff);   // [64][16]
    uint8_t* stg = smem + C::kStagingOff;
    mbar_wait(&bars->acc_full, 0);
    tc_fence_after();
#pragma unroll 1
    for (int c = 0; c < MP / 16; ++c) {
      uint32_t v[16];
      tmem_ld_32x32b_x16(tbase + lane_off + c * 16, v);
      tmem_wait_ld();
      if (r >= 64) {
#pragma unroll
        for (int j = 0; j < 16; ++j) xchg[(r - 64) * 16 + j] = __uint_as_float(v[j]);
      }
      asm volatile("bar.sync 1, 128;" ::: "memory");
      if (r < 64) {
#pragma unroll
        for (int j = 0; j < 16; ++j) {
          const int m = c * 16 + j;
          const float h = silu_mul(__uint_as_float(v[j]), xchg[r * 16 + j]);
          __nv_bfloat16 hb = __float2bfloat16_rn(h);
          // staging row m (token), column r (output col), 128-byte swizzle
          *reinterpret_cast<__nv_bfloat16*>(stg + m * 128 + (((r >> 3) ^ (m & 7)) << 4) + (r & 7) * 2) = hb;
        }
      }
      asm volatile("bar.sync 1, 128;" ::: "memory");
    }
    tc_fence_before();
    fence_proxy_async_smem();
    asm volatile("bar.sync 1, 128;" ::: "memory");
    if (etid == 0) {
      tma_store_2d(&p.tm_d, stg, n0, 0);
      bulk_commit_group();
      bulk_wait_group0();
    }
  }

  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tbase, C::kTmemCols);
  }
}

template <int MP>
cudaError_t launch_swap(const GateUpLaunch& L, const void* a, const void* b, cudaStream_t stream) {
  using C = SwapCfg<MP>;
  GemmParams p;
  std::memset(&p, 0, sizeof(p));
  p.M = L.M;
  p.K = L.K;
  p.I = L.I;
  p.num_kb = (L.K + kBK - 1) / kBK;
  p.mode = 1;
  if (!enc(&p.tm_a, a, L.K, L.M, static_cast<uint64_t>(L.K) * 2, MP)) return cudaErrorInvalidValue;
  if (!enc(&p.tm_b, b, L.K, 2ull * L.I, static_cast<uint64_t>(L.K) * 2, 64)) return cudaErrorInvalidValue;
  if (!enc(&p.tm_d, L.d, L.I, L.M, static_cast<uint64_t>(L.d_stride) * 2, MP)) return cudaErrorInvalidValue;
  cudaError_t e = ensure_smem_limit(reinterpret_cast<const void*>(gateup_swap_kernel<MP>), C::kSmem);
  if (e != cudaSuccess) return e;
  gateup_swap_kernel<MP><<<L.I / 64, kThreads, C::kSmem, stream>>>(p);
  return cudaGetLastError();
}

}  // namespace

cudaError_t launch_gateup(const GateUpLaunch& L, const void* a, const void* b, cudaStream_t stream) {
  // fused SwiGLU with few rows: weight streaming over all SMs
  if (L.mode == 1 && L.M <= 128) {
    if (L.M <= 16) return launch_swap<16>(L, a, b, stream);
    if (L.M <= 32) return launch_swap<32>(L, a, b, stream);
    if (L.M <= 64) return launch_swap<64>(L, a, b, stream);
    return launch_swap<128>(L, a, b, stream);
  }
  // up to 256 rows: one 256-row tile per CTA shares each W tile between both
  // halves (measured: equal at K=4096, 4% faster at K=8192); beyond, the
  // overlapped-epilogue form wins (684 vs 725 us at M=4096)
  if (L.M <= 2 * kBM) {
    // Narrow SwiGLU shards: K split over a cluster of pairs when the pair
    // tiles alone would leave most SMs idle and the split still fits one wave
    // of clusters (16 clusters of 8 / 32 of 4 CTAs on 148 SMs), each split
    // keeping at least 4 K blocks.
    if (L.mode == 1 && L.M > kBM && L.I % 256 == 0) {
      const int64_t pair_tiles = L.I / 256;
      const int num_kb = (L.K + kBK - 1) / kBK;
      if (pair_tiles * 8 <= 128 && num_kb >= 16) return launch_pair_split<4>(L, a, b, stream);
      if (pair_tiles * 4 <= 128 && num_kb >= 8) return launch_pair_split<2>(L, a, b, stream);
    }
    // Few rows: the weight stream is spread over as many CTAs as there are
    // SMs. Of the tile forms (256 x 128 with a shared W tile, 128 x 128,
    // 128 x 64), take the one with the most tiles that still fits in one
    // wave; if none fits, the one with the fewest. Measured at M=256 (us):
    // K=8192 I=3584 [100 / 66 / 61], I=7168 [103 / 70 / 111], I=28672
    // [227 / 240 / 350]; K=4096 I=14336 [70 / 72 / 109].
    int dev = 0, sms = kNumSMs;
    cudaGetDevice(&dev);
    cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
    const int64_t cand[3] = {
        L.M > kBM && L.I % 128 == 0 ? (L.M + 2 * kBM - 1) / (2 * kBM) * (L.I / 128) : -1,
        L.I % 128 == 0 ? (L.M + kBM - 1) / kBM * (L.I / 128) : -1,
        L.I % 64 == 0 ? (L.M + kBM - 1) / kBM * (L.I / 64) : -1};
    int best = -1;
    for (int c = 0; c < 3; ++c)
      if (cand[c] > 0 && cand[c] <= sms && (best < 0 || cand[c] > cand[best])) best = c;
    if (best < 0)
      for (int c = 0; c < 3; ++c)
        if (cand[c] > 0 && (best < 0 || cand[c] < cand[best])) best = c;
    if (best == 0) {
      // SwiGLU with 256-column pair tiles (the same CTA count): the CTA-pair form
      if (L.mode == 1 && L.M > kBM) {
        // of the pair tiles (256 / 224 columns), the one with the least
        // column work per SM: rounds of resident pairs x tile width
        const int64_t pairs = sms / 2;
        const int64_t w256 = L.I % 256 == 0 ? (L.I / 256 + pairs - 1) / pairs * 256 : -1;
        const int64_t w224 = L.I % 224 == 0 ? (L.I / 224 + pairs - 1) / pairs * 224 : -1;
        if (w224 > 0 && (w256 < 0 || w224 < w256)) return launch_pair<112>(L, a, b, stream);
        if (w256 > 0) return launch_pair<128>(L, a, b, stream);
      }
      return launch_bn<128, 2>(L, a, b, stream);
    }
    if (best == 2) return launch_bn<64, 1>(L, a, b, stream);
  }
  return launch_bn<128>(L, a, b, stream);
}

cudaError_t launch_gateup_window(const void* ws, void* d, int64_t d_stride, int32_t M, int32_t I, int32_t mode,
                                 cudaStream_t stream) {
  const int64_t chunks = static_cast<int64_t>(M) * (I / 8);
  const int blocks = static_cast<int>(std::min<int64_t>((chunks + 255) / 256, 148 * 16));
  gateup_window_kernel<<<blocks, 256, 0, stream>>>(static_cast<const uint16_t*>(ws), static_cast<uint16_t*>(d),
                                                   d_stride, M, I, mode);
  return cudaGetLastError();
}

}  // namespace cascade
