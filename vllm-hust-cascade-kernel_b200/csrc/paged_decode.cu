// Paged decode attention for the cascade: <= 16 query rows per (request, kv
// head) -- the per-request suffix stage (q_len = 1, GQA group <= 16) and the
// small-row forms of the stage-1 op.
//
// Memory-bound design (KV bytes dominate):
//  * one CTA per (split of 512 kv tokens, kv head, request); the split's
//    partial (O, LSE) is merged by launch_split_combine when a request has
//    more than one split. For wide ragged batches a planned form instead
//    lists the non-empty (request, split) items on the device
//    (decode_plan_kernel) and runs two persistent CTAs per SM over them
//    (paged_decode_stream_kernel: a fetcher warp prepares the next item in
//    shared memory while the current one streams through a ring that never
//    drains between items), with the same tile and merge code;
//  * a producer warp streams 64-token K/V tiles with 2-D TMA (one box per page
//    segment and 64-element half of the head dim, 128-byte swizzle) into a
//    3-stage ring: 32 KB per stage, 96 KB per CTA, two CTAs per SM;
//  * four consumer warps each own 16 tokens of every tile: QK^T and PV with
//    m16n8k16 mma.sync (rows = the <= 16 query rows of the GQA group), P kept
//    in registers (fp32 -> 16-bit RNE, the reference's quantisation point,
//    kernel_fa_fp32_stage1.cpp / block_epilogue_online_softmax_no_mask.hpp:578-591),
//    row sums from the unquantised fp32 exps, warp-shuffle row reductions;
//  * the 4 warps' (m, l, O) are merged through shared memory at the end.
// Each warp runs its own online softmax over its tokens in 16-token steps;
// the CPU oracle reproduces this structure exactly (chunk 16, segments =
// the warp's token subsets).
#include <algorithm>

#include "kernels.h"
#include "ptx.cuh"

namespace cascade {

namespace {

constexpr int kTile = 64;              // kv tokens per pipeline stage
constexpr int kStages = 3;
constexpr int kConsumerWarps = 4;
constexpr int kThreads = (kConsumerWarps + 1) * 32;
constexpr int kHalfBytes = kTile * 128;          // one [64 tokens x 64 dims] 16-bit box region
constexpr int kKBytes = 2 * kHalfBytes;           // K tile, both dim halves
constexpr int kStageBytes = 2 * kKBytes;          // K + V
constexpr int kSmemBytes = kStages * kStageBytes + 1024 /*align*/ + 512 /*barriers, block-table cache*/;

constexpr int kBtCache = 48;  // block-table entries of one split kept in smem

struct __align__(8) DecodeBarriers {
  uint64_t full[kStages];
  uint64_t empty[kStages];
  uint64_t stall;  // never completed: the debug_stall test hook waits on it
  int32_t bt[kBtCache];
};

__device__ __forceinline__ int request_token_offset(const PagedAttnLaunch& p, int b) {
  if (p.q_seqlen_value > 0) return b * p.q_seqlen_value;
  // per-request q lengths: prefix sum over the first b entries (warp-parallel)
  int lane = threadIdx.x & 31;
  long long acc = 0;
  for (int i = lane; i < b; i += 32) acc += p.q_seqlens[i];
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) acc += __shfl_xor_sync(0xffffffffu, acc, o);
  return static_cast<int>(acc);
}

template <bool kFp16>
__device__ __forceinline__ void store_out(void* out, int out_dtype, size_t idx, float v0, float v1) {
  if (out_dtype == 2) {
    *reinterpret_cast<float2*>(static_cast<float*>(out) + idx) = make_float2(v0, v1);
  } else if (out_dtype == 1) {
    *reinterpret_cast<__half2*>(static_cast<__half*>(out) + idx) = __floats2half2_rn(v0, v1);
  } else {
    *reinterpret_cast<__nv_bfloat162*>(static_cast<__nv_bfloat16*>(out) + idx) = __floats2bfloat162_rn(v0, v1);
  }
}

__device__ __forceinline__ void init_decode_barriers(const PagedAttnLaunch& p, DecodeBarriers* bars) {
  for (int s = 0; s < kStages; ++s) {
    mbar_init(&bars->full[s], 1);
    mbar_init(&bars->empty[s], kConsumerWarps);
  }
  mbar_init(&bars->stall, 1);
  fence_mbar_init();
  cta_wait_init(static_cast<uint64_t>(p.wait_limit_us) * 1000);
}

// Teardown of an aborting CTA (lane 0 of the producer warp): wait, bounded,
// for the TMA loads of ring positions [begin, end) that may still be in
// flight -- the last NS of them, one per stage -- so no copy lands in shared
// memory after the CTA has exited.
template <int NS>
__device__ __forceinline__ void drain_ring(uint64_t* full, uint32_t begin, uint32_t end) {
  for (uint32_t gi = (end - begin > NS ? end - NS : begin); gi < end; ++gi) mbar_wait_drain(&full[gi % NS], (gi / NS) & 1);
}

// Producer warp of one item: pulls the split's block-table entries
// (bt_pre0/1 = entries lane and lane + 32, loaded earlier by this warp) into
// shared memory, then lane 0 streams the item's tiles into the NS-stage ring
// at ring positions it0, it0 + 1, ... Returns (in lane 0) the number of tiles
// issued: fewer than ntiles only when the CTA is aborting.
template <int NS, bool kBtFilled = false>
__device__ __forceinline__ int produce_tiles(const PagedAttnLaunch& p, uint8_t* smem, uint64_t* full, uint64_t* empty,
                                              int32_t* bt_smem, int b, int g, int s_begin, int s_end, int kv,
                                              int ntiles, uint32_t it0, int bt_pre0, int bt_pre1) {
  const int lane = threadIdx.x & 31;
  const int first_page = s_begin / p.block_size;
  // The whole warp first pulls this split's block-table entries into shared
  // memory, so the TMA issue loop never waits on a dependent global load.
  const int bs = p.block_size;
  const int32_t* bt = p.block_table + static_cast<size_t>(b) * p.block_cols;
  const int npages = (kv + bs - 1) / bs;
  const int last_page = min(npages, (s_end + bs - 1) / bs);  // exclusive
  const int nbt = last_page - first_page;
  const bool cached = nbt <= kBtCache;
  if (cached && !kBtFilled) {
    static_assert(kBtCache <= 64, "two prefetched entries per lane");
    if (lane < nbt) bt_smem[lane] = bt_pre0;
    if (lane + 32 < nbt) bt_smem[lane + 32] = bt_pre1;
  }
  __syncwarp();
  int issued = 0;
  if (lane == 0) {
    tma_prefetch_desc(&p.tmap_k);
    tma_prefetch_desc(&p.tmap_v);
    const int box_rows = bs < kTile ? bs : kTile;
    const int oob_row = p.num_blocks * bs;  // fully out of range -> zero fill
    const uint64_t pol = policy_evict_first();
    for (int i = 0; i < ntiles; ++i, ++issued) {
      const uint32_t gi = it0 + i;  // ring position of this tile in the CTA's lifetime
      const int st = gi % NS;
      if (gi >= NS) mbar_wait(&empty[st], ((gi / NS) - 1) & 1);
      if (cta_aborted()) break;
      uint8_t* sk = smem + st * kStageBytes;
      uint8_t* sv = sk + kKBytes;
      mbar_arrive_expect_tx(&full[st], kStageBytes);
      const int t_tile = s_begin + i * kTile;
      for (int off = 0; off < kTile; off += box_rows) {
        const int t = t_tile + off;
        const int page = t / bs;
        int row = oob_row;
        if (page < npages) row = paged_row(cached ? bt_smem[page - first_page] : bt[page], t, bs, p.num_blocks, oob_row);
        const int x0 = g * kHeadDim;
        uint8_t* dk = sk + off * 128;
        uint8_t* dv = sv + off * 128;
        tma_load_2d_hint(dk, &p.tmap_k, &full[st], x0, row, pol);
        tma_load_2d_hint(dk + kHalfBytes, &p.tmap_k, &full[st], x0 + 64, row, pol);
        tma_load_2d_hint(dv, &p.tmap_v, &full[st], x0, row, pol);
        tma_load_2d_hint(dv + kHalfBytes, &p.tmap_v, &full[st], x0 + 64, row, pol);
      }
    }
  }
  return issued;
}

// Q A-fragments of this thread (rows gq and gq+8, 8 k-steps over the 128
// dims), from the query tensor or, when q_rows is given, from a copy of the
// item's nrows query rows ([row][128], 16-bit) in shared memory.
__device__ __forceinline__ void load_q_frags(const PagedAttnLaunch& p, const uint16_t* q_rows, int nrows, int tok0,
                                             int g, uint32_t (&qa)[8][4]) {
  const int lane = threadIdx.x & 31;
  const int gq = lane >> 2;
  const int tq = lane & 3;
  {
    const uint16_t* q = static_cast<const uint16_t*>(p.query);
    const int rows[2] = {gq, gq + 8};
    uint32_t v[2][8][2];
#pragma unroll
    for (int ri = 0; ri < 2; ++ri) {
      const int r = rows[ri];
#pragma unroll
      for (int ks = 0; ks < 8; ++ks) {
        v[ri][ks][0] = 0;
        v[ri][ks][1] = 0;
      }
      if (r < nrows) {
        const int t = tok0 + r / p.group, h = g * p.group + r % p.group;
        const uint16_t* src =
            q_rows != nullptr ? q_rows + r * kHeadDim : q + (static_cast<size_t>(t) * p.num_heads + h) * kHeadDim;
#pragma unroll
        for (int ks = 0; ks < 8; ++ks) {
          v[ri][ks][0] = *reinterpret_cast<const uint32_t*>(src + ks * 16 + 2 * tq);
          v[ri][ks][1] = *reinterpret_cast<const uint32_t*>(src + ks * 16 + 8 + 2 * tq);
        }
      }
    }
#pragma unroll
    for (int ks = 0; ks < 8; ++ks) {
      qa[ks][0] = v[0][ks][0];
      qa[ks][1] = v[1][ks][0];
      qa[ks][2] = v[0][ks][1];
      qa[ks][3] = v[1][ks][1];
    }
  }
}

// Consumer warps of one item: the item's tiles from the ring (positions
// it0, it0 + 1, ...) against the Q fragments qa; leaves this thread's O fragments, row
// maxima (log2 units) and quad-reduced row sums.
template <bool kFp16, int NS>
__device__ __forceinline__ void consume_tiles(const PagedAttnLaunch& p, uint8_t* smem, uint64_t* full, uint64_t* empty,
                                              uint64_t* stall, uint32_t it0, int ntiles, int s_begin, int s_end,
                                              const uint32_t (&qa)[8][4], float (&o)[16][4], float& m0, float& m1,
                                              float& l0, float& l1) {
  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const int tq = lane & 3;  // thread in quad

#pragma unroll
  for (int n = 0; n < 16; ++n) o[n][0] = o[n][1] = o[n][2] = o[n][3] = 0.f;
  m0 = -INFINITY;  // running max (log2 units) rows gq, gq+8
  m1 = -INFINITY;
  l0 = 0.f;        // this thread's share of the row sums
  l1 = 0.f;

  if (p.debug_stall) mbar_wait(stall, 0);  // test hook: runs into the wait limit, the CTA aborts
  const uint32_t smem_base = smem_u32(smem);
  const int wrow = warp * 16;  // this warp's first token row within a tile
  // ldmatrix row addresses (matrix index = lane / 8, row = lane % 8)
  const int mi = lane >> 3, mr = lane & 7;

  for (int i = 0; i < ntiles; ++i) {
    const uint32_t gi = it0 + i;
    const int st = gi % NS;
    mbar_wait(&full[st], (gi / NS) & 1);
    const uint32_t kbase = smem_base + st * kStageBytes;
    const uint32_t vbase = kbase + kKBytes;

    // S = Q K^T over this warp's 16 tokens (two n8 tiles)
    float s[2][4] = {{0.f, 0.f, 0.f, 0.f}, {0.f, 0.f, 0.f, 0.f}};
    {
      const int trow = wrow + (mi >> 1) * 8 + mr;  // token row of this lane's ldmatrix address
#pragma unroll
      for (int ks = 0; ks < 8; ++ks) {
        const int dim = ks * 16 + (mi & 1) * 8;
        const uint32_t addr = kbase + (dim >> 6) * kHalfBytes + sw128(trow, (dim & 63) >> 3);
        uint32_t r[4];
        ldmatrix_x4(r, addr);
        mma_16816<kFp16>(s[0], qa[ks], r[0], r[1]);
        mma_16816<kFp16>(s[1], qa[ks], r[2], r[3]);
      }
    }

    // mask tokens beyond kv, scale to log2 units, online softmax
    const int tbase = s_begin + i * kTile + wrow;
    float mx0 = -INFINITY, mx1 = -INFINITY;
#pragma unroll
    for (int n = 0; n < 2; ++n) {
      const int tk = tbase + n * 8 + 2 * tq;
      s[n][0] = (tk < s_end) ? s[n][0] * p.scale_log2 : -INFINITY;
      s[n][1] = (tk + 1 < s_end) ? s[n][1] * p.scale_log2 : -INFINITY;
      s[n][2] = (tk < s_end) ? s[n][2] * p.scale_log2 : -INFINITY;
      s[n][3] = (tk + 1 < s_end) ? s[n][3] * p.scale_log2 : -INFINITY;
      mx0 = fmaxf(mx0, fmaxf(s[n][0], s[n][1]));
      mx1 = fmaxf(mx1, fmaxf(s[n][2], s[n][3]));
    }
    mx0 = fmaxf(mx0, __shfl_xor_sync(0xffffffffu, mx0, 1));
    mx0 = fmaxf(mx0, __shfl_xor_sync(0xffffffffu, mx0, 2));
    mx1 = fmaxf(mx1, __shfl_xor_sync(0xffffffffu, mx1, 1));
    mx1 = fmaxf(mx1, __shfl_xor_sync(0xffffffffu, mx1, 2));
    const float mn0 = fmaxf(m0, mx0), mn1 = fmaxf(m1, mx1);
    const float ms0 = mn0 == -INFINITY ? 0.f : mn0;  // all-masked-so-far guard
    const float ms1 = mn1 == -INFINITY ? 0.f : mn1;
    const float al0 = m0 == -INFINITY ? 0.f : ex2(m0 - ms0);
    const float al1 = m1 == -INFINITY ? 0.f : ex2(m1 - ms1);
    m0 = mn0;
    m1 = mn1;
    float ps0 = 0.f, ps1 = 0.f;
#pragma unroll
    for (int n = 0; n < 2; ++n) {
      s[n][0] = ex2(s[n][0] - ms0);
      s[n][1] = ex2(s[n][1] - ms0);
      s[n][2] = ex2(s[n][2] - ms1);
      s[n][3] = ex2(s[n][3] - ms1);
      ps0 += s[n][0] + s[n][1];
      ps1 += s[n][2] + s[n][3];
    }
    l0 = al0 * l0 + ps0;
    l1 = al1 * l1 + ps1;
#pragma unroll
    for (int n = 0; n < 16; ++n) {
      o[n][0] *= al0;
      o[n][1] *= al0;
      o[n][2] *= al1;
      o[n][3] *= al1;
    }
    // P (16-bit, RNE) as the A operand of PV: C-fragment layout == A layout
    uint32_t pa[4];
    pa[0] = pack2<kFp16>(s[0][0], s[0][1]);
    pa[1] = pack2<kFp16>(s[0][2], s[0][3]);
    pa[2] = pack2<kFp16>(s[1][0], s[1][1]);
    pa[3] = pack2<kFp16>(s[1][2], s[1][3]);

    {
      const int trow = wrow + (mi & 1) * 8 + mr;
#pragma unroll
      for (int pp = 0; pp < 8; ++pp) {
        const int dim = pp * 16 + (mi >> 1) * 8;
        const uint32_t addr = vbase + (dim >> 6) * kHalfBytes + sw128(trow, (dim & 63) >> 3);
        uint32_t r[4];
        ldmatrix_x4_trans(r, addr);
        mma_16816<kFp16>(o[2 * pp], pa, r[0], r[1]);
        mma_16816<kFp16>(o[2 * pp + 1], pa, r[2], r[3]);
      }
    }
    __syncwarp();
    if (lane == 0) mbar_arrive(&empty[st]);
  }

  // row sums over the quad
  l0 += __shfl_xor_sync(0xffffffffu, l0, 1);
  l0 += __shfl_xor_sync(0xffffffffu, l0, 2);
  l1 += __shfl_xor_sync(0xffffffffu, l1, 1);
  l1 += __shfl_xor_sync(0xffffffffu, l1, 2);
}

// Merge of the 4 consumer warps' (m, l, O) through shared memory at
// merge_smem (merge_bytes(mrows): rows [0, mrows) of each warp, mrows >=
// nrows), then the item's output: a split partial (O, LSE) or, for a single
// split, the final O and LSE.
constexpr int kSoStride = kHeadDim + 8;
__host__ __device__ constexpr int merge_bytes(int mrows) {
  return (kConsumerWarps * mrows * kSoStride + 2 * kConsumerWarps * mrows) * 4;
}
template <bool kFp16>
__device__ __forceinline__ void merge_store(const PagedAttnLaunch& p, float* merge_smem, int mrows,
                                            const float (&o)[16][4], float m0, float m1, float l0, float l1,
                                            int nrows, int tok0, int g, int split) {
  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const int gq = lane >> 2;
  const int tq = lane & 3;
  asm volatile("bar.sync 1, %0;" ::"r"(kConsumerWarps * 32) : "memory");
  // Rows are padded to 136 floats: the 8 rows of one fragment store then fall
  // on distinct banks (row r starts at bank 8r mod 32), and only the query
  // rows that exist are written.
  float* so = merge_smem;                                      // [4][mrows][kSoStride]
  float* sm = so + kConsumerWarps * mrows * kSoStride;        // [4][mrows]
  float* sl = sm + kConsumerWarps * mrows;                    // [4][mrows]
  if (gq < nrows) {
    float* dst = so + (warp * mrows + gq) * kSoStride + 2 * tq;
#pragma unroll
    for (int n = 0; n < 16; ++n) *reinterpret_cast<float2*>(dst + n * 8) = make_float2(o[n][0], o[n][1]);
  }
  if (gq + 8 < nrows) {
    float* dst = so + (warp * mrows + gq + 8) * kSoStride + 2 * tq;
#pragma unroll
    for (int n = 0; n < 16; ++n) *reinterpret_cast<float2*>(dst + n * 8) = make_float2(o[n][2], o[n][3]);
  }
  if (tq == 0) {
    if (gq < nrows) {
      sm[warp * mrows + gq] = m0;
      sl[warp * mrows + gq] = l0;
    }
    if (gq + 8 < nrows) {
      sm[warp * mrows + gq + 8] = m1;
      sl[warp * mrows + gq + 8] = l1;
    }
  }
  asm volatile("bar.sync 1, %0;" ::"r"(kConsumerWarps * 32) : "memory");

  // 128 threads, one float4 of one row each: a warp covers one 512-byte row
  // (conflict-free smem reads, coalesced global stores).
  const int tid = threadIdx.x;
  for (int idx = tid; idx < nrows * (kHeadDim / 4); idx += kConsumerWarps * 32) {
    const int r = idx / (kHeadDim / 4);
    const int d0 = (idx % (kHeadDim / 4)) * 4;
    float M = -INFINITY;
#pragma unroll
    for (int w = 0; w < kConsumerWarps; ++w) M = fmaxf(M, sm[w * mrows + r]);
    float wsum = 0.f, wt[kConsumerWarps];
#pragma unroll
    for (int w = 0; w < kConsumerWarps; ++w) {
      const float mw = sm[w * mrows + r];
      wt[w] = (mw == -INFINITY) ? 0.f : ex2(mw - M);
      wsum += wt[w] * sl[w * mrows + r];
    }
    const float inv = wsum > 0.f ? 1.f / wsum : 0.f;
    const float lse_nat = (wsum > 0.f) ? (M + log2f(wsum)) * 0.6931471805599453f : -INFINITY;
    const int t = tok0 + r / p.group, h = g * p.group + r % p.group;
    const size_t row = static_cast<size_t>(t) * p.num_heads + h;
    float4 acc = make_float4(0.f, 0.f, 0.f, 0.f);
#pragma unroll
    for (int w = 0; w < kConsumerWarps; ++w) {
      if (wt[w] == 0.f) continue;
      const float4 v = *reinterpret_cast<const float4*>(&so[(w * mrows + r) * kSoStride + d0]);
      acc.x += wt[w] * v.x;
      acc.y += wt[w] * v.y;
      acc.z += wt[w] * v.z;
      acc.w += wt[w] * v.w;
    }
    const int c = idx % (kHeadDim / 4);
    if (p.num_splits > 1 || p.partial_out) {
      float* dst = p.part_o + (static_cast<size_t>(split) * p.num_tokens * p.num_heads + row) * kHeadDim + d0;
      *reinterpret_cast<float4*>(dst) = make_float4(acc.x * inv, acc.y * inv, acc.z * inv, acc.w * inv);
      if (c == 0) p.part_lse[static_cast<size_t>(split) * p.num_tokens * p.num_heads + row] = lse_nat;
    } else {
      store_out<kFp16>(p.out, p.out_dtype, row * kHeadDim + d0, acc.x * inv, acc.y * inv);
      store_out<kFp16>(p.out, p.out_dtype, row * kHeadDim + d0 + 2, acc.z * inv, acc.w * inv);
      for (int cc = c; cc < p.lse_stride; cc += kHeadDim / 4) p.lse[row * p.lse_stride + cc] = lse_nat;
    }
  }
}

// One (split, kv head, request) item. `it0` = tiles this CTA consumed in
// earlier items (the ring's barrier phases continue across items);
// `init_bars` initialises the ring barriers first (one item per CTA). Returns
// the tiles consumed. All 160 threads call it; on return every tile of the
// item has landed and the ring's shared memory is free again only after a
// CTA barrier (the merge reuses it).
template <bool kFp16>
__device__ __forceinline__ int paged_decode_item(const PagedAttnLaunch& p, uint8_t* smem, DecodeBarriers* bars,
                                                 int split, int g, int b, uint32_t it0, bool init_bars) {
  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;

  // The split's block-table entries do not depend on the kv length: the
  // producer warp issues their load first, so it overlaps the length load.
  const int s_begin = split * p.split_tokens;
  const int first_page = s_begin / p.block_size;
  const int bt_avail = min(kBtCache, p.block_cols - first_page);
  int bt_pre0 = 0, bt_pre1 = 0;
  if (warp == kConsumerWarps) {
    const int32_t* btrow = p.block_table + static_cast<size_t>(b) * p.block_cols + first_page;
    if (lane < bt_avail) bt_pre0 = btrow[lane];
    if (lane + 32 < bt_avail) bt_pre1 = btrow[lane + 32];
  }

  // kv is clamped to the block table's capacity, so no entry past a row is read
  const int kv = static_cast<int>(min(p.kv_seqlens[b], static_cast<int64_t>(p.block_cols) * p.block_size));
  const int q_len = p.q_seqlen_value > 0 ? p.q_seqlen_value : static_cast<int>(p.q_seqlens[b]);
  const int nrows = q_len * p.group;
  const int tok0 = request_token_offset(p, b);
  const int s_end = min(kv, s_begin + p.split_tokens);
  const int ntiles = s_end > s_begin ? (s_end - s_begin + kTile - 1) / kTile : 0;

  // Empty split (kv shorter than this split's start, or no query rows):
  // write -inf partials so the combine step skips it.
  if (ntiles == 0 || nrows == 0) {
    if (p.num_splits > 1 || p.partial_out) {
      for (int r = threadIdx.x; r < nrows; r += blockDim.x) {
        int t = tok0 + r / p.group, h = g * p.group + r % p.group;
        p.part_lse[static_cast<size_t>(split) * p.num_tokens * p.num_heads + static_cast<size_t>(t) * p.num_heads + h] =
            -INFINITY;
      }
    } else {
      // single split: kv == 0 -> out = 0, lse = -inf
      for (int i = threadIdx.x; i < nrows * kHeadDim / 2; i += blockDim.x) {
        int r = i / (kHeadDim / 2), d = (i % (kHeadDim / 2)) * 2;
        int t = tok0 + r / p.group, h = g * p.group + r % p.group;
        store_out<kFp16>(p.out, p.out_dtype, (static_cast<size_t>(t) * p.num_heads + h) * kHeadDim + d, 0.f, 0.f);
      }
      for (int i = threadIdx.x; i < nrows * p.lse_stride; i += blockDim.x) {
        int r = i / p.lse_stride, c = i % p.lse_stride;
        int t = tok0 + r / p.group, h = g * p.group + r % p.group;
        p.lse[(static_cast<size_t>(t) * p.num_heads + h) * p.lse_stride + c] = -INFINITY;
      }
    }
    return 0;
  }

  if (init_bars) {
    if (threadIdx.x == 0) init_decode_barriers(p, bars);
    __syncthreads();
  }

  if (warp == kConsumerWarps) {
    const int issued = produce_tiles<kStages>(p, smem, bars->full, bars->empty, bars->bt, b, g, s_begin, s_end, kv,
                                              ntiles, it0, bt_pre0, bt_pre1);
    if (lane == 0 && cta_aborted()) drain_ring<kStages>(bars->full, it0, it0 + issued);
    return ntiles;
  }

  uint32_t qa[8][4];
  load_q_frags(p, nullptr, nrows, tok0, g, qa);
  float o[16][4];
  float m0, m1, l0, l1;
  consume_tiles<kFp16, kStages>(p, smem, bars->full, bars->empty, &bars->stall, it0, ntiles, s_begin, s_end, qa, o, m0,
                                m1, l0, l1);
  // All tiles are consumed (every full barrier was waited by every warp), so
  // the stage ring is free for the merge once all consumer warps reach its
  // first barrier.
  merge_store<kFp16>(p, reinterpret_cast<float*>(smem), 16, o, m0, m1, l0, l1, nrows, tok0, g, split);
  return ntiles;
}
__device__ __forceinline__ uint8_t* decode_smem() {
  extern __shared__ uint8_t smem_raw[];
  return reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
}

// One CTA per (split, kv head, request).
template <bool kFp16>
__global__ void __launch_bounds__(kThreads, 2) paged_decode_kernel(const __grid_constant__ PagedAttnLaunch p) {
  pdl_launch_dependents();
  uint8_t* smem = decode_smem();
  DecodeBarriers* bars = reinterpret_cast<DecodeBarriers*>(smem + kStages * kStageBytes);
  paged_decode_item<kFp16>(p, smem, bars, blockIdx.x, blockIdx.y, blockIdx.z, 0u, true);
  // pdl 1: every CTA waits for the primary before exiting; pdl 2: only the
  // grid's last CTA does (enough for "this grid completed => the primary
  // completed" without holding every slot while a long primary runs)
  const bool last = blockIdx.x == gridDim.x - 1 && blockIdx.y == gridDim.y - 1 && blockIdx.z == gridDim.z - 1;
  if ((p.pdl == 1 || (p.pdl == 2 && last)) && threadIdx.x == 0) pdl_wait();
}

// Streaming form of the planned decode, three roles:
//   warp 5 (fetcher) takes the items (per-kv-head counter) and prepares each
//     in one of two shared-memory slots: the item code, its kv length, the
//     split's block-table entries and the item's query rows;
//   warp 4 (producer) streams each slot's tiles into an NS-stage ring whose
//     positions continue across items (3 stages when the rows of an item are
//     few enough for two CTAs per SM, else 2);
//   warps 0-3 (consumers) take Q from the slot, consume the tiles and merge
//     through their own shared-memory area.
// The ring never drains between items and no role waits on a global load
// at an item boundary: the next item's metadata and rows arrive while the
// current one streams. A slot is free again once the producer has issued its
// tiles and every consumer warp has read its Q. Two CTAs per SM.
constexpr int kStreamThreads = kThreads + 32;

struct __align__(16) StreamSlot {
  int32_t code;  // (b << 8) | split, or -1: no more items
  int32_t kv;
  int32_t pad[2];
  int32_t bt[kBtCache];
};

struct __align__(16) StreamBarriers {
  uint64_t full[3];
  uint64_t empty[3];
  uint64_t item_full[2];   // slot written (32 fetcher lanes)
  uint64_t item_empty[2];  // slot consumed (producer + one arrive per consumer warp)
  uint64_t stall;          // never completed: the debug_stall test hook waits on it
  int32_t code_bcast;      // the consumers' item code, read once and shared (named barrier 1)
  int32_t pad[1];
  StreamSlot slot[2];
};

// Shared memory of the streaming form for items of `rows` query rows: the
// NS-stage ring, the consumers' merge area (rows per warp = rows), the
// barriers and slots, then each slot's query rows (rows x 256 bytes).
__host__ __device__ constexpr int stream_smem_bytes(int ns, int rows) {
  return ns * kStageBytes + merge_bytes(rows) + static_cast<int>(sizeof(StreamBarriers)) + 2 * rows * kHeadDim * 2 +
         1024 /*align*/;
}

template <bool kFp16, int NS>
__global__ void __launch_bounds__(kStreamThreads, 2)
    paged_decode_stream_kernel(const __grid_constant__ PagedAttnLaunch p) {
  pdl_launch_dependents();
  uint8_t* smem = decode_smem();
  const int nrows = p.q_seqlen_value * p.group;
  float* merge_smem = reinterpret_cast<float*>(smem + NS * kStageBytes);
  StreamBarriers* bars = reinterpret_cast<StreamBarriers*>(smem + NS * kStageBytes + merge_bytes(nrows));
  uint16_t* qrows = reinterpret_cast<uint16_t*>(bars + 1);  // [2 slots][nrows][128]
  const int g = blockIdx.y;
  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  if (threadIdx.x == 0) {
    for (int s = 0; s < NS; ++s) {
      mbar_init(&bars->full[s], 1);
      mbar_init(&bars->empty[s], kConsumerWarps);
    }
    for (int q = 0; q < 2; ++q) {
      mbar_init(&bars->item_full[q], 32);
      mbar_init(&bars->item_empty[q], 1 + kConsumerWarps);
    }
    mbar_init(&bars->stall, 1);
    fence_mbar_init();
    cta_wait_init(static_cast<uint64_t>(p.wait_limit_us) * 1000);
  }
  pdl_wait();  // the item list, its count and the zeroed counters are complete
  __syncthreads();
  const size_t plane = static_cast<size_t>(p.num_tokens) * p.num_heads;
  const int cap = p.block_cols * p.block_size;
  for (int b = blockIdx.x; b < p.batch; b += gridDim.x) {
    const int kv = static_cast<int>(min(p.kv_seqlens[b], static_cast<int64_t>(cap)));
    const int used = kv > 0 ? min(p.num_splits, (kv + p.split_tokens - 1) / p.split_tokens) : 0;
    const int tok0 = b * p.q_seqlen_value;
    for (int i = threadIdx.x; i < (p.num_splits - used) * nrows; i += blockDim.x) {
      const int s = used + i / nrows, r = i % nrows;
      const int t = tok0 + r / p.group, h = g * p.group + r % p.group;
      p.part_lse[static_cast<size_t>(s) * plane + static_cast<size_t>(t) * p.num_heads + h] = -INFINITY;
    }
  }
  uint32_t it0 = 0;  // ring position of the next tile
  if (warp == kConsumerWarps + 1) {
    // ------------------------------------------------------------- fetcher
    const int count = *p.plan_count;
    for (int j = 0;; ++j) {
      const int q = j & 1;
      StreamSlot& sl = bars->slot[q];
      if (j >= 2) mbar_wait(&bars->item_empty[q], ((j >> 1) - 1) & 1);
      // an aborting CTA takes no more items: it writes the end code at once
      int item = 0;
      if (lane == 0) item = cta_aborted() ? count : atomicAdd(p.plan_counters + g, 1);
      item = __shfl_sync(0xffffffffu, item, 0);
      const int code = item < count ? p.plan_items[item] : -1;
      if (code >= 0) {
        const int split = code & 0xFF, b = code >> 8;
        const int first_page = split * p.split_tokens / p.block_size;
        const int bt_avail = min(kBtCache, p.block_cols - first_page);
        const int32_t* btrow = p.block_table + static_cast<size_t>(b) * p.block_cols + first_page;
        static_assert(kBtCache <= 64, "two block-table entries per lane");
        if (lane < bt_avail) sl.bt[lane] = btrow[lane];
        if (lane + 32 < bt_avail) sl.bt[lane + 32] = btrow[lane + 32];
        if (lane == 0) sl.kv = static_cast<int>(min(p.kv_seqlens[b], static_cast<int64_t>(cap)));
        // query rows: nrows x 256 bytes as 16-byte chunks over the warp
        const uint4* qsrc = static_cast<const uint4*>(p.query);
        uint4* qdst = reinterpret_cast<uint4*>(qrows + q * nrows * kHeadDim);
        for (int c = lane; c < nrows * (kHeadDim / 8); c += 32) {
          const int r = c / (kHeadDim / 8), w = c % (kHeadDim / 8);
          const int t = b * p.q_seqlen_value + r / p.group, h = g * p.group + r % p.group;
          qdst[c] = qsrc[(static_cast<size_t>(t) * p.num_heads + h) * (kHeadDim / 8) + w];
        }
      }
      if (lane == 0) sl.code = code;
      mbar_arrive(&bars->item_full[q]);  // each lane releases its own stores
      if (code < 0) break;
    }
  } else if (warp == kConsumerWarps) {
    // ------------------------------------------------------------ producer
    for (int j = 0;; ++j) {
      const int q = j & 1;
      StreamSlot& sl = bars->slot[q];
      mbar_wait(&bars->item_full[q], (j >> 1) & 1);
      // one lane decides for the warp (an aborting CTA's slots are not
      // protected by their barriers any more)
      int code = 0;
      if (lane == 0) code = cta_aborted() ? -1 : sl.code;
      code = __shfl_sync(0xffffffffu, code, 0);
      if (code < 0) break;
      const int split = code & 0xFF, b = code >> 8;
      const int s_begin = split * p.split_tokens;
      const int kv = sl.kv;
      const int s_end = min(kv, s_begin + p.split_tokens);
      const int ntiles = s_end > s_begin ? (s_end - s_begin + kTile - 1) / kTile : 0;
      int issued = produce_tiles<NS, true>(p, smem, bars->full, bars->empty, sl.bt, b, g, s_begin, s_end, kv, ntiles,
                                           it0, 0, 0);
      issued = __shfl_sync(0xffffffffu, issued, 0);
      __syncwarp();  // lane 0 has issued every tile: the slot's entries are no longer read
      if (lane == 0) mbar_arrive(&bars->item_empty[q]);
      it0 += issued;
    }
    if (lane == 0 && cta_aborted()) drain_ring<NS>(bars->full, 0, it0);
  } else {
    // ----------------------------------------------------------- consumers
    for (int j = 0;; ++j) {
      const int q = j & 1;
      StreamSlot& sl = bars->slot[q];
      mbar_wait(&bars->item_full[q], (j >> 1) & 1);
      // one thread reads the code for all four warps, so they all take the
      // same branch into merge_store's named barriers even when an aborting
      // CTA's fetcher rewrites the slot
      if (threadIdx.x == 0) bars->code_bcast = cta_aborted() ? -1 : sl.code;
      asm volatile("bar.sync 1, %0;" ::"r"(kConsumerWarps * 32) : "memory");
      const int code = bars->code_bcast;
      if (code < 0) break;
      const int split = code & 0xFF, b = code >> 8;
      const int s_begin = split * p.split_tokens;
      const int s_end = min(sl.kv, s_begin + p.split_tokens);
      const int ntiles = s_end > s_begin ? (s_end - s_begin + kTile - 1) / kTile : 0;
      const int tok0 = b * p.q_seqlen_value;
      uint32_t qa[8][4];
      load_q_frags(p, qrows + q * nrows * kHeadDim, nrows, tok0, g, qa);
      __syncwarp();
      if (lane == 0) mbar_arrive(&bars->item_empty[q]);
      float o[16][4];
      float m0, m1, l0, l1;
      consume_tiles<kFp16, NS>(p, smem, bars->full, bars->empty, &bars->stall, it0, ntiles, s_begin, s_end, qa, o, m0,
                               m1, l0, l1);
      merge_store<kFp16>(p, merge_smem, nrows, o, m0, m1, l0, l1, nrows, tok0, g, split);
      it0 += ntiles;
    }
  }
}

// Lists the non-empty (request, split) items of a planned decode: request b
// contributes min(num_splits, ceil(kv_b / split_tokens)) items (none for
// kv_b = 0), coded (b << 8) | split, in request order; also the count, and
// zeroes the per-kv-head item counters. One CTA of 1024 threads.
__global__ void __launch_bounds__(1024) decode_plan_kernel(const __grid_constant__ PagedAttnLaunch p) {
  pdl_launch_dependents();
  if (p.pdl) pdl_wait();  // the seqlens may come from the kernel before
  __shared__ int32_t wsum[32];
  __shared__ int32_t carry;
  const int tid = threadIdx.x, lane = tid & 31, w = tid >> 5;
  if (tid == 0) carry = 0;
  for (int i = tid; i < p.kv_heads; i += blockDim.x) p.plan_counters[i] = 0;
  __syncthreads();
  for (int base = 0; base < p.batch; base += blockDim.x) {
    const int b = base + tid;
    int n = 0;
    if (b < p.batch) {
      const int kv = static_cast<int>(min(p.kv_seqlens[b], static_cast<int64_t>(p.block_cols) * p.block_size));
      n = kv > 0 ? min(p.num_splits, (kv + p.split_tokens - 1) / p.split_tokens) : 0;
    }
    int x = n;  // inclusive scan: warp, then warp totals
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      const int y = __shfl_up_sync(0xffffffffu, x, o);
      if (lane >= o) x += y;
    }
    if (lane == 31) wsum[w] = x;
    __syncthreads();
    if (w == 0) {
      int v = lane < (blockDim.x >> 5) ? wsum[lane] : 0;
#pragma unroll
      for (int o = 1; o < 32; o <<= 1) {
        const int y = __shfl_up_sync(0xffffffffu, v, o);
        if (lane >= o) v += y;
      }
      wsum[lane] = v;  // inclusive prefix of warp totals
    }
    __syncthreads();
    const int excl = carry + (w > 0 ? wsum[w - 1] : 0) + x - n;
    for (int s = 0; s < n; ++s) p.plan_items[excl + s] = (b << 8) | s;
    __syncthreads();
    if (tid == 0) carry += wsum[(blockDim.x >> 5) - 1];
    __syncthreads();
  }
  if (tid == 0) *p.plan_count = carry;
}

// One warp per (token, head) row: merge the split partials.
__global__ void split_combine_kernel(const __grid_constant__ PagedAttnLaunch p) {
  const int warps_per_block = blockDim.x >> 5;
  const size_t row = static_cast<size_t>(blockIdx.x) * warps_per_block + (threadIdx.x >> 5);
  const int lane = threadIdx.x & 31;
  const size_t rows = static_cast<size_t>(p.num_tokens) * p.num_heads;
  if (row >= rows) return;
  const size_t plane = rows;
  float M = -INFINITY;
  for (int s = 0; s < p.num_splits; ++s) M = fmaxf(M, p.part_lse[s * plane + row]);
  float acc0 = 0.f, acc1 = 0.f, acc2 = 0.f, acc3 = 0.f, wsum = 0.f;
  if (M != -INFINITY) {
    for (int s = 0; s < p.num_splits; ++s) {
      const float l = p.part_lse[s * plane + row];
      if (l == -INFINITY) continue;
      const float w = __expf(l - M);
      const float4 v = *reinterpret_cast<const float4*>(p.part_o + (s * plane + row) * kHeadDim + lane * 4);
      acc0 += w * v.x;
      acc1 += w * v.y;
      acc2 += w * v.z;
      acc3 += w * v.w;
      wsum += w;
    }
  }
  const float inv = wsum > 0.f ? 1.f / wsum : 0.f;
  const float lse = wsum > 0.f ? M + __logf(wsum) : -INFINITY;
  const size_t o = row * kHeadDim + lane * 4;
  if (p.out_dtype == 2) {
    *reinterpret_cast<float4*>(static_cast<float*>(p.out) + o) =
        make_float4(acc0 * inv, acc1 * inv, acc2 * inv, acc3 * inv);
  } else if (p.out_dtype == 1) {
    __half2 a = __floats2half2_rn(acc0 * inv, acc1 * inv), c = __floats2half2_rn(acc2 * inv, acc3 * inv);
    uint2 u = make_uint2(*reinterpret_cast<uint32_t*>(&a), *reinterpret_cast<uint32_t*>(&c));
    *reinterpret_cast<uint2*>(static_cast<__half*>(p.out) + o) = u;
  } else {
    __nv_bfloat162 a = __floats2bfloat162_rn(acc0 * inv, acc1 * inv), c = __floats2bfloat162_rn(acc2 * inv, acc3 * inv);
    uint2 u = make_uint2(*reinterpret_cast<uint32_t*>(&a), *reinterpret_cast<uint32_t*>(&c));
    *reinterpret_cast<uint2*>(static_cast<__nv_bfloat16*>(p.out) + o) = u;
  }
  if (lane < p.lse_stride) {
    for (int c = lane; c < p.lse_stride; c += 32) p.lse[row * p.lse_stride + c] = lse;
  }
}

}  // namespace

cudaError_t launch_paged_decode(const PagedAttnLaunch& p, bool fp16, cudaStream_t stream) {
  if (p.plan_items != nullptr) {
    // plan (one CTA), then the persistent decode as its programmatic
    // dependent: two CTAs per SM in all, split evenly over the kv heads
    launch_maybe_pdl(decode_plan_kernel, dim3(1), dim3(1024), 0, stream, p.pdl != 0, p);
    cudaError_t e = cudaGetLastError();
    if (e != cudaSuccess) return e;
    // three ring stages when two CTAs per SM still fit (up to 228 KB of
    // shared memory per SM, 1 KB reserved per CTA), else two
    const int rows = p.q_seqlen_value * p.group;
    const bool three = 2 * (stream_smem_bytes(3, rows) + 1024) <= 228 * 1024;
    const int smem = stream_smem_bytes(three ? 3 : 2, rows);
    auto kern = three ? (fp16 ? paged_decode_stream_kernel<true, 3> : paged_decode_stream_kernel<false, 3>)
                      : (fp16 ? paged_decode_stream_kernel<true, 2> : paged_decode_stream_kernel<false, 2>);
    e = ensure_smem_limit(reinterpret_cast<const void*>(kern), smem);
    if (e != cudaSuccess) return e;
    const int per_head = std::max(1, (2 * kNumSMs) / std::max(1, p.kv_heads));
    return launch_maybe_pdl(kern, dim3(per_head, p.kv_heads, 1), dim3(kStreamThreads), smem, stream, true,
                            p);
  }
  dim3 grid(p.num_splits, p.kv_heads, p.batch);
  auto kern = fp16 ? paged_decode_kernel<true> : paged_decode_kernel<false>;
  cudaError_t e = ensure_smem_limit(reinterpret_cast<const void*>(kern), kSmemBytes);
  if (e != cudaSuccess) return e;
  return launch_maybe_pdl(kern, grid, dim3(kThreads), kSmemBytes, stream, p.pdl != 0, p);
}

cudaError_t launch_split_combine(const PagedAttnLaunch& p, cudaStream_t stream) {
  const size_t rows = static_cast<size_t>(p.num_tokens) * p.num_heads;
  const int wpb = 8;
  const unsigned blocks = static_cast<unsigned>((rows + wpb - 1) / wpb);
  if (blocks == 0) return cudaSuccess;
  split_combine_kernel<<<blocks, wpb * 32, 0, stream>>>(p);
  return cudaGetLastError();
}

}  // namespace cascade
