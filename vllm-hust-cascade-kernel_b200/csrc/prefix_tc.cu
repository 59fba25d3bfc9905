// Stage-1 shared-prefix paged attention on the 5th-generation tensor cores
// (tcgen05 + TMEM), for more than 16 query rows per (request, kv head).
//
// In the cascade the whole decode batch of a prefix group is flattened into
// one request with q_len = group size, so every kv head sees
// q_len * (H/KVH) query rows against the same prefix pages: a dense
// QK^T / PV contraction (the shared-prefix stage of the reference,
// ascend-kernel/csrc/ops/fa_fp32_stage1/op_kernel/kernel_fa_fp32_stage1.cpp:143-745).
//
// One CTA = (KV split, kv head x 128-row tile, request); 6 warps:
//   warp 4    TMA producer: 128-token K and V tiles, gathered page by page
//             through block_table (2-D boxes of [min(bs,128) rows x 64 dims],
//             128-byte swizzle), double-buffered;
//   warp 5    MMA issuer (one thread): S = Q K^T (M=128, N=128, K=128) into a
//             TMEM S buffer, then O_tile = P V into a TMEM PV buffer; every
//             completion is signalled with tcgen05.commit to an mbarrier;
//   warps 0-3 softmax + correction: thread i owns query row i == TMEM lane i.
//             Reads S with tcgen05.ld, keeps the running max / row sum, writes
//             P = bf16/fp16(exp(S - m)) (RNE, the reference's quantisation
//             point, block_epilogue_online_softmax_no_mask.hpp:578-591) into
//             swizzled smem as the A operand of PV, and accumulates
//             O = dm * O + PV in registers (the reference's rescale,
//             block_epilogue_rescale_o_no_split_row.hpp:144-268).
// TMEM: S[2] at columns 0/128, PV[2] at 256/384 (512 columns, 1 CTA per SM).
// Shared memory: Q 32 KB, K 2x32 KB, V 2x32 KB, P 2x32 KB.
// Final O/l and LSE = ln(l) + m (natural log), written 8x per row (stage-1
// padded layout) or as a split partial merged by the combine kernel.
#include "kernels.h"
#include "ptx.cuh"

namespace cascade {
namespace {

constexpr int kRows = 128;
constexpr int kTok = 128;
constexpr int kThreads = 6 * 32;
constexpr int kHalf = 16384;            // [128 rows][64 x 16-bit] swizzled region
constexpr int kTileBytes = 2 * kHalf;   // [128 rows][128 x 16-bit]
constexpr int kOffQ = 0;
constexpr int kOffK = kOffQ + kTileBytes;
constexpr int kOffV = kOffK + 2 * kTileBytes;
constexpr int kOffP = kOffV + 2 * kTileBytes;
constexpr int kOffBar = kOffP + 2 * kTileBytes;
constexpr int kSmemBytes = kOffBar + 256 + 1024;
constexpr uint32_t kTmemCols = 512;

struct __align__(8) PrefixBars {
  uint64_t q_full;
  uint64_t k_full[2], k_empty[2], v_full[2], v_empty[2];
  uint64_t s_full[2], s_free[2], p_full[2], p_free[2], pv_full[2], pv_free[2];
  uint32_t tmem_base;
};

__device__ __forceinline__ int token_offset(const PagedAttnLaunch& p, int b) {
  if (p.q_seqlen_value > 0) return b * p.q_seqlen_value;
  const int lane = threadIdx.x & 31;
  long long acc = 0;
  for (int i = lane; i < b; i += 32) acc += p.q_seqlens[i];
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) acc += __shfl_xor_sync(0xffffffffu, acc, o);
  return static_cast<int>(acc);
}

__device__ __forceinline__ void store_row(const PagedAttnLaunch& p, size_t row, const float* o, float scale) {
  if (p.out_dtype == 2) {
    float4* dst = reinterpret_cast<float4*>(static_cast<float*>(p.out) + row * kHeadDim);
#pragma unroll
    for (int i = 0; i < kHeadDim / 4; ++i)
      dst[i] = make_float4(o[4 * i] * scale, o[4 * i + 1] * scale, o[4 * i + 2] * scale, o[4 * i + 3] * scale);
  } else {
    uint4* dst = reinterpret_cast<uint4*>(static_cast<uint16_t*>(p.out) + row * kHeadDim);
    const bool h = p.out_dtype == 1;
#pragma unroll
    for (int i = 0; i < kHeadDim / 8; ++i) {
      uint32_t w[4];
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        const float a = o[8 * i + 2 * j] * scale, b = o[8 * i + 2 * j + 1] * scale;
        w[j] = h ? pack2<true>(a, b) : pack2<false>(a, b);
      }
      dst[i] = make_uint4(w[0], w[1], w[2], w[3]);
    }
  }
}

template <bool kFp16>
__global__ void __launch_bounds__(kThreads, 1) paged_prefix_tc_kernel(const __grid_constant__ PagedAttnLaunch p) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  PrefixBars* bars = reinterpret_cast<PrefixBars*>(smem + kOffBar);

  const int split = blockIdx.x;
  const int g = blockIdx.y % p.kv_heads;
  const int mt = blockIdx.y / p.kv_heads;
  const int b = blockIdx.z;
  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const int tid = threadIdx.x;

  const int kv = static_cast<int>(p.kv_seqlens[b]);
  const int q_len = p.q_seqlen_value > 0 ? p.q_seqlen_value : static_cast<int>(p.q_seqlens[b]);
  const int nrows = q_len * p.group;
  const int row0 = mt * kRows;
  const int unit_rows = min(kRows, nrows - row0);
  const int tok0 = token_offset(p, b);
  if (unit_rows <= 0) return;  // this request has fewer row tiles
  const int s_begin = split * p.split_tokens;
  const int s_end = min(kv, s_begin + p.split_tokens);
  const int ntiles = s_end > s_begin ? (s_end - s_begin + kTok - 1) / kTok : 0;
  const size_t plane = static_cast<size_t>(p.num_tokens) * p.num_heads;

  auto out_row = [&](int r) -> size_t {
    const int rr = row0 + r;
    return static_cast<size_t>(tok0 + rr / p.group) * p.num_heads + g * p.group + rr % p.group;
  };

  if (ntiles == 0) {
    // split beyond this request's kv (or kv == 0)
    for (int r = tid; r < unit_rows; r += blockDim.x) {
      const size_t row = out_row(r);
      if (p.num_splits > 1) {
        p.part_lse[static_cast<size_t>(split) * plane + row] = -INFINITY;
      } else {
        float z[kHeadDim];
#pragma unroll
        for (int i = 0; i < kHeadDim; ++i) z[i] = 0.f;
        store_row(p, row, z, 1.f);
        for (int c = 0; c < p.lse_stride; ++c) p.lse[row * p.lse_stride + c] = -INFINITY;
      }
    }
    return;
  }

  if (tid == 0) {
    mbar_init(&bars->q_full, 1);
    for (int s = 0; s < 2; ++s) {
      mbar_init(&bars->k_full[s], 1);
      mbar_init(&bars->k_empty[s], 1);
      mbar_init(&bars->v_full[s], 1);
      mbar_init(&bars->v_empty[s], 1);
      mbar_init(&bars->s_full[s], 1);
      mbar_init(&bars->s_free[s], 4 * 32);
      mbar_init(&bars->p_full[s], 4 * 32);
      mbar_init(&bars->p_free[s], 1);
      mbar_init(&bars->pv_full[s], 1);
      mbar_init(&bars->pv_free[s], 4 * 32);
    }
    fence_mbar_init();
  }
  if (warp == 5) {
    tmem_alloc(&bars->tmem_base, kTmemCols);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tbase = bars->tmem_base;
  const uint32_t sQ = smem_u32(smem + kOffQ);
  const uint32_t sK = smem_u32(smem + kOffK);
  const uint32_t sV = smem_u32(smem + kOffV);
  const uint32_t sP = smem_u32(smem + kOffP);

  if (warp == 4) {
    // ------------------------------------------------------------ producer
    if (lane == 0) {
      tma_prefetch_desc(&p.tmap_k);
      tma_prefetch_desc(&p.tmap_v);
      const int bs = p.block_size;
      const int box_rows = bs < kTok ? bs : kTok;
      const int oob_row = p.num_blocks * bs;
      const int32_t* bt = p.block_table + static_cast<size_t>(b) * p.block_cols;
      const int npages = (kv + bs - 1) / bs;
      const int x0 = g * kHeadDim;
      for (int j = 0; j < ntiles; ++j) {
        const int st = j & 1, u = j >> 1;
        const int t_tile = s_begin + j * kTok;
        for (int kvsel = 0; kvsel < 2; ++kvsel) {
          uint64_t* full = kvsel ? &bars->v_full[st] : &bars->k_full[st];
          uint64_t* empty = kvsel ? &bars->v_empty[st] : &bars->k_empty[st];
          const CUtensorMap* tm = kvsel ? &p.tmap_v : &p.tmap_k;
          uint8_t* dst = smem + (kvsel ? kOffV : kOffK) + st * kTileBytes;
          if (j >= 2) mbar_wait(empty, (u - 1) & 1);
          mbar_arrive_expect_tx(full, kTileBytes);
          for (int off = 0; off < kTok; off += box_rows) {
            const int t = t_tile + off;
            const int page = t / bs;
            const int row = page < npages ? bt[page] * bs + (t % bs) : oob_row;
            tma_load_2d(dst + off * 128, tm, full, x0, row);
            tma_load_2d(dst + kHalf + off * 128, tm, full, x0 + 64, row);
          }
        }
      }
    }
  } else if (warp == 5) {
    // ------------------------------------------------------------- MMA issuer
    if (lane == 0) {
      constexpr uint32_t fmt = kFp16 ? 0u : 1u;
      const uint32_t idesc_s = make_idesc_f16(128, 128, fmt, 0, 0);
      const uint32_t idesc_pv = make_idesc_f16(128, 128, fmt, 0, 1);
      mbar_wait(&bars->q_full, 0);
      tc_fence_after();
      for (int j = 0; j <= ntiles; ++j) {
        if (j < ntiles) {
          const int st = j & 1, u = j >> 1;
          mbar_wait(&bars->k_full[st], u & 1);
          if (j >= 2) mbar_wait(&bars->s_free[st], (u - 1) & 1);
          tc_fence_after();
          const uint32_t kb = sK + st * kTileBytes;
#pragma unroll
          for (int k = 0; k < 8; ++k) {
            const uint32_t koff = (k >> 2) * kHalf + (k & 3) * 32;
            umma_f16_ss(tbase + st * 128, make_smem_desc(sQ + koff, 16, 1024, 2),
                        make_smem_desc(kb + koff, 16, 1024, 2), idesc_s, k > 0 ? 1u : 0u);
          }
          umma_commit(&bars->s_full[st]);
          umma_commit(&bars->k_empty[st]);
        }
        if (j >= 1) {
          const int i = j - 1;
          const int st = i & 1, u = i >> 1;
          mbar_wait(&bars->v_full[st], u & 1);
          mbar_wait(&bars->p_full[st], u & 1);
          if (i >= 2) mbar_wait(&bars->pv_free[st], (u - 1) & 1);
          tc_fence_after();
          const uint32_t pb = sP + st * kTileBytes;
          const uint32_t vb = sV + st * kTileBytes;
#pragma unroll
          for (int k = 0; k < 8; ++k) {
            umma_f16_ss(tbase + 256 + st * 128,
                        make_smem_desc(pb + (k >> 2) * kHalf + (k & 3) * 32, 16, 1024, 2),
                        make_smem_desc(vb + k * 2048, kHalf, 1024, 2), idesc_pv, k > 0 ? 1u : 0u);
          }
          umma_commit(&bars->pv_full[st]);
          umma_commit(&bars->v_empty[st]);
          umma_commit(&bars->p_free[st]);
        }
      }
    }
  } else {
    // ------------------------------------------------ softmax / correction
    // Q row -> swizzled smem (K-major A operand); rows past the unit are zero
    {
      uint8_t* q_s = smem + kOffQ;
      if (tid < unit_rows) {
        const uint4* src = reinterpret_cast<const uint4*>(static_cast<const uint16_t*>(p.query) +
                                                           out_row(tid) * kHeadDim);
#pragma unroll
        for (int c = 0; c < 16; ++c)
          *reinterpret_cast<uint4*>(q_s + (c >> 3) * kHalf + sw128(tid, c & 7)) = __ldg(src + c);
      } else {
#pragma unroll
        for (int c = 0; c < 16; ++c)
          *reinterpret_cast<uint4*>(q_s + (c >> 3) * kHalf + sw128(tid, c & 7)) = make_uint4(0, 0, 0, 0);
      }
      fence_proxy_async_smem();
      asm volatile("bar.sync 1, 128;" ::: "memory");
      if (tid == 0) mbar_arrive(&bars->q_full);
    }

    const uint32_t lane_off = static_cast<uint32_t>(warp * 32) << 16;
    const float sl2 = p.scale_log2;
    float o[kHeadDim];
#pragma unroll
    for (int i = 0; i < kHeadDim; ++i) o[i] = 0.f;
    float m = -INFINITY, l = 0.f, dm_prev = 0.f;

    auto accumulate = [&](int i, float d) {
      const int st = i & 1, u = i >> 1;
      mbar_wait(&bars->pv_full[st], u & 1);
      tc_fence_after();
#pragma unroll
      for (int c = 0; c < 8; ++c) {
        uint32_t r[16];
        tmem_ld_32x32b_x16(tbase + lane_off + 256 + st * 128 + c * 16, r);
        tmem_wait_ld();
#pragma unroll
        for (int e = 0; e < 16; ++e) o[c * 16 + e] = fmaf(d, o[c * 16 + e], __uint_as_float(r[e]));
      }
      tc_fence_before();
      mbar_arrive(&bars->pv_free[st]);
    };

    for (int j = 0; j < ntiles; ++j) {
      const int st = j & 1, u = j >> 1;
      const int n_valid = min(kTok, s_end - (s_begin + j * kTok));
      mbar_wait(&bars->s_full[st], u & 1);
      tc_fence_after();
      const uint32_t s_addr = tbase + lane_off + st * 128;
      float mx = -INFINITY;
#pragma unroll
      for (int c = 0; c < 4; ++c) {
        uint32_t r[32];
        tmem_ld_32x32b_x32(s_addr + c * 32, r);
        tmem_wait_ld();
#pragma unroll
        for (int e = 0; e < 32; ++e) {
          const float v = (c * 32 + e < n_valid) ? __uint_as_float(r[e]) : -INFINITY;
          mx = fmaxf(mx, v);
        }
      }
      const float m_new = fmaxf(m, mx * sl2);
      const float dm = (m == -INFINITY) ? 0.f : ex2(m - m_new);
      if (j >= 2) mbar_wait(&bars->p_free[st], (u - 1) & 1);
      uint8_t* pbuf = smem + kOffP + st * kTileBytes;
      float rs = 0.f;
#pragma unroll
      for (int c = 0; c < 8; ++c) {
        uint32_t r[16];
        tmem_ld_32x32b_x16(s_addr + c * 16, r);
        tmem_wait_ld();
        uint32_t pk[8];
#pragma unroll
        for (int e = 0; e < 16; e += 2) {
          const float x0 = (c * 16 + e < n_valid) ? ex2(fmaf(__uint_as_float(r[e]), sl2, -m_new)) : 0.f;
          const float x1 = (c * 16 + e + 1 < n_valid) ? ex2(fmaf(__uint_as_float(r[e + 1]), sl2, -m_new)) : 0.f;
          rs += x0 + x1;
          pk[e >> 1] = pack2<kFp16>(x0, x1);
        }
#pragma unroll
        for (int q = 0; q < 2; ++q) {
          const int tc = c * 2 + q;  // 16-byte chunk index along the 128 tokens
          *reinterpret_cast<uint4*>(pbuf + (tc >> 3) * kHalf + sw128(tid, tc & 7)) =
              make_uint4(pk[4 * q], pk[4 * q + 1], pk[4 * q + 2], pk[4 * q + 3]);
        }
      }
      tc_fence_before();
      mbar_arrive(&bars->s_free[st]);
      fence_proxy_async_smem();
      mbar_arrive(&bars->p_full[st]);
      l = dm * l + rs;
      m = m_new;
      if (j >= 1) accumulate(j - 1, dm_prev);
      dm_prev = dm;
    }
    accumulate(ntiles - 1, dm_prev);

    if (tid < unit_rows) {
      const size_t row = out_row(tid);
      const float inv = 1.f / l;
      const float lse_nat = (m + __log2f(l)) * 0.6931471805599453f;
      if (p.num_splits > 1) {
        float4* dst = reinterpret_cast<float4*>(p.part_o + (static_cast<size_t>(split) * plane + row) * kHeadDim);
#pragma unroll
        for (int i = 0; i < kHeadDim / 4; ++i)
          dst[i] = make_float4(o[4 * i] * inv, o[4 * i + 1] * inv, o[4 * i + 2] * inv, o[4 * i + 3] * inv);
        p.part_lse[static_cast<size_t>(split) * plane + row] = lse_nat;
      } else {
        store_row(p, row, o, inv);
        for (int c = 0; c < p.lse_stride; ++c) p.lse[row * p.lse_stride + c] = lse_nat;
      }
    }
  }

  tc_fence_before();
  __syncthreads();
  if (warp == 5) {
    tc_fence_after();
    tmem_dealloc(tbase, kTmemCols);
  }
}

}  // namespace

cudaError_t launch_paged_prefix_tc(const PagedAttnLaunch& p, bool fp16, cudaStream_t stream) {
  const int mtiles = (p.max_q_seqlen * p.group + kRows - 1) / kRows;
  dim3 grid(p.num_splits, p.kv_heads * mtiles, p.batch);
  auto kern = fp16 ? paged_prefix_tc_kernel<true> : paged_prefix_tc_kernel<false>;
  cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, kSmemBytes);
  if (e != cudaSuccess) return e;
  kern<<<grid, kThreads, kSmemBytes, stream>>>(p);
  return cudaGetLastError();
}

}  // namespace cascade
