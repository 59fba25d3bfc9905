// Stage-1 shared-prefix paged attention on the 5th-generation tensor cores
// (tcgen05 + TMEM), for more than 16 query rows per (request, kv head).
//
// In the cascade the whole decode batch of a prefix group is flattened into
// one request with q_len = group size, so every kv head sees
// q_len * (H/KVH) query rows against the same prefix pages: a dense
// QK^T / PV contraction (the shared-prefix stage of the reference,
// ascend-kernel/csrc/ops/fa_fp32_stage1/op_kernel/kernel_fa_fp32_stage1.cpp:143-745).
//
// One CTA = (KV split, kv head x 128-row tile, request); 11 warps:
//   warp 8    K producer, warp 10 V producer: 128-token K and V tiles gathered
//             page by page through block_table (2-D boxes [min(bs,128) rows x
//             64 dims], 128-byte swizzle) into two 3-stage rings. Two issuing
//             threads: one thread's TMA issue rate caps a CTA near 76 GB/s;
//   warp 9    MMA issuer (one thread): S_j = Q K_j^T (M=N=K=128) into a TMEM S
//             buffer and O += P_j V_j into the TMEM O accumulator, both with
//             the A operand (Q, P) read from tensor memory;
//   warps 0-3 softmax: thread i owns query row i == TMEM lane i. One
//             tcgen05.ld of the 128-column S row, running max and
//             unquantised row sum, P = round16(exp(S - m)) (RNE: the
//             reference's quantisation point,
//             block_epilogue_online_softmax_no_mask.hpp:578-591) written back
//             over the first 64 columns of the same S buffer (two 16-bit
//             values per column) as the A operand of PV;
//   warps 4-7 correction + epilogue: they load Q into tensor memory, and
//             before P_j V_j is accumulated they rescale the TMEM accumulator
//             O = dm_j * O (the reference's rescale,
//             block_epilogue_rescale_o_no_split_row.hpp:144-268) -- skipped,
//             exactly, for a warp whose 32 rows all kept their max (dm == 1);
//             at the end they write O / l and the LSE.
// TMEM: S[2] at columns 0/128 (P_j aliases S_j), O at 256, Q at 384. Shared
// memory: K 3x32 KB, V 3x32 KB. LSE = ln(l) + m (natural log), written 8x per
// row (stage-1 padded layout) or as a split partial for a later combine.
#include "kernels.h"
#include "ptx.cuh"

namespace cascade {
namespace {

constexpr int kRows = 128;
constexpr int kTok = 128;
constexpr int kThreads = 11 * 32;
constexpr int kKProducerWarp = 8;
constexpr int kMmaWarp = 9;
constexpr int kVProducerWarp = 10;
constexpr int kStages = 3;              // K and V ring depth
constexpr int kHalf = 16384;            // [128 rows][64 x 16-bit] swizzled region
constexpr int kTileBytes = 2 * kHalf;   // [128 rows][128 x 16-bit]
constexpr int kOffK = 0;
constexpr int kOffV = kOffK + kStages * kTileBytes;
constexpr int kOffAux = kOffV + kStages * kTileBytes;   // dm[2][128], l[128], m[128], block table, barriers
constexpr int kBtCache = 256;                 // block-table entries of one split kept in smem
constexpr int kOffBars = kOffAux + 4 * 128 * 4 + kBtCache * 4;
static_assert(kOffBars % 16 == 0, "mbarriers need 8-byte alignment");
constexpr int kSmemBytes = kOffBars + 256 + 1024;
static_assert(kSmemBytes <= 227 * 1024, "shared memory per CTA");
constexpr uint32_t kTmemCols = 512;
constexpr uint32_t kColO = 256;
constexpr uint32_t kColQ = 384;         // Q as 64 columns of 16-bit pairs

// Phase rules (each barrier is waited in tile order and can never complete
// two phases ahead of its waiter):
//   s_full[j&1]   S_j complete (commit)                  -> softmax
//   p_full[j&1]   P_j written to TMEM (128 softmax rows)  -> MMA, before PV_j
//   corr_go[j&1]  tile j's row maxima known (128 softmax rows) AND PV_{j-1}
//                 complete (commit; a plain arrive for j = 0) -> correction
//   o_ready[j&1]  O rescaled for tile j (128 rows)        -> MMA, before PV_j
struct __align__(8) PrefixBars {
  uint64_t q_full;
  uint64_t k_full[kStages], k_empty[kStages], v_full[kStages], v_empty[kStages];
  uint64_t s_full[2], p_full[2], corr_go[2], o_ready[2];
  uint64_t o_final, fin;
  uint64_t stall;   // never completed: the debug_stall test hook waits on it
  uint64_t drain;   // an aborting MMA issuer's last commit
  uint32_t tmem_base;
};
static_assert(sizeof(PrefixBars) <= 256, "barrier block");

__device__ __forceinline__ int token_offset(const PagedAttnLaunch& p, int b) {
  if (p.q_seqlen_value > 0) return b * p.q_seqlen_value;
  const int lane = threadIdx.x & 31;
  long long acc = 0;
  for (int i = lane; i < b; i += 32) acc += p.q_seqlens[i];
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) acc += __shfl_xor_sync(0xffffffffu, acc, o);
  return static_cast<int>(acc);
}

__device__ __forceinline__ void tmem_st_32x32b_x32(uint32_t taddr, const uint32_t (&r)[32]) {
  asm volatile(
      "tcgen05.st.sync.aligned.32x32b.x32.b32 [%0], "
      "{%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,%16,"
      "%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31,%32};" ::"r"(taddr),
      "r"(r[0]), "r"(r[1]), "r"(r[2]), "r"(r[3]), "r"(r[4]), "r"(r[5]), "r"(r[6]), "r"(r[7]), "r"(r[8]),
      "r"(r[9]), "r"(r[10]), "r"(r[11]), "r"(r[12]), "r"(r[13]), "r"(r[14]), "r"(r[15]), "r"(r[16]),
      "r"(r[17]), "r"(r[18]), "r"(r[19]), "r"(r[20]), "r"(r[21]), "r"(r[22]), "r"(r[23]), "r"(r[24]),
      "r"(r[25]), "r"(r[26]), "r"(r[27]), "r"(r[28]), "r"(r[29]), "r"(r[30]), "r"(r[31])
      : "memory");
}

__device__ __forceinline__ void tmem_st_32x32b_x16(uint32_t taddr, const uint32_t (&r)[16]) {
  asm volatile(
      "tcgen05.st.sync.aligned.32x32b.x16.b32 [%0], "
      "{%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,%16};" ::"r"(taddr),
      "r"(r[0]), "r"(r[1]), "r"(r[2]), "r"(r[3]), "r"(r[4]), "r"(r[5]), "r"(r[6]), "r"(r[7]), "r"(r[8]),
      "r"(r[9]), "r"(r[10]), "r"(r[11]), "r"(r[12]), "r"(r[13]), "r"(r[14]), "r"(r[15])
      : "memory");
}

__device__ __forceinline__ void tmem_wait_st() { asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory"); }

// Columns [nv, 64) of a 64-column S chunk (two 32-column loads) -> -inf.
__device__ __forceinline__ void mask_cols(uint32_t (&sa)[32], uint32_t (&sb)[32], int nv) {
  const uint32_t ninf = __float_as_uint(-INFINITY);
#pragma unroll
  for (int e = 0; e < 32; ++e) {
    sa[e] = e < nv ? sa[e] : ninf;
    sb[e] = 32 + e < nv ? sb[e] : ninf;
  }
}

// Stores 32 consecutive output elements of one row (fp32 or 16-bit).
__device__ __forceinline__ void store_chunk(const PagedAttnLaunch& p, size_t elem, const uint32_t (&r)[32],
                                            float scale) {
  if (p.out_dtype == 2) {
    float4* dst = reinterpret_cast<float4*>(static_cast<float*>(p.out) + elem);
#pragma unroll
    for (int i = 0; i < 8; ++i)
      dst[i] = make_float4(__uint_as_float(r[4 * i]) * scale, __uint_as_float(r[4 * i + 1]) * scale,
                           __uint_as_float(r[4 * i + 2]) * scale, __uint_as_float(r[4 * i + 3]) * scale);
  } else {
    uint4* dst = reinterpret_cast<uint4*>(static_cast<uint16_t*>(p.out) + elem);
    const bool h = p.out_dtype == 1;
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      uint32_t w[4];
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        const float a = __uint_as_float(r[8 * i + 2 * j]) * scale, b = __uint_as_float(r[8 * i + 2 * j + 1]) * scale;
        w[j] = h ? pack2<true>(a, b) : pack2<false>(a, b);
      }
      dst[i] = make_uint4(w[0], w[1], w[2], w[3]);
    }
  }
}

template <bool kFp16>
__device__ __forceinline__ void paged_prefix_tc_body(const PagedAttnLaunch& p) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  float* dmbuf = reinterpret_cast<float*>(smem + kOffAux);   // [2][128]
  float* lbuf = dmbuf + 2 * kRows;                            // [128]
  float* mbuf = lbuf + kRows;                                 // [128]
  int32_t* btc = reinterpret_cast<int32_t*>(mbuf + kRows);   // [kBtCache]
  PrefixBars* bars = reinterpret_cast<PrefixBars*>(btc + kBtCache);

  const int split = blockIdx.x;
  const int g = blockIdx.y % p.kv_heads;
  const int mt = blockIdx.y / p.kv_heads;
  const int b = blockIdx.z;
  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const int tid = threadIdx.x;

  // kv is clamped to the block table's capacity, so no entry past a row is read
  const int kv = static_cast<int>(min(p.kv_seqlens[b], static_cast<int64_t>(p.block_cols) * p.block_size));
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
  const bool partial = p.num_splits > 1 || p.partial_out;

  auto out_row = [&](int r) -> size_t {
    const int rr = row0 + r;
    return static_cast<size_t>(tok0 + rr / p.group) * p.num_heads + g * p.group + rr % p.group;
  };

  if (ntiles == 0) {
    // split beyond this request's kv (or kv == 0)
    for (int r = tid; r < unit_rows; r += blockDim.x) {
      const size_t row = out_row(r);
      if (partial) {
        p.part_lse[static_cast<size_t>(split) * plane + row] = -INFINITY;
      } else {
        uint32_t z[32];
#pragma unroll
        for (int i = 0; i < 32; ++i) z[i] = 0u;
#pragma unroll
        for (int c = 0; c < 4; ++c) store_chunk(p, row * kHeadDim + c * 32, z, 1.f);
        for (int c = 0; c < p.lse_stride; ++c) p.lse[row * p.lse_stride + c] = -INFINITY;
      }
    }
    return;
  }

  // The split's block-table entries -> smem (warp 8, one round trip) before
  // the CTA barrier, so both producers see them.
  const int bs = p.block_size;
  const int32_t* bt = p.block_table + static_cast<size_t>(b) * p.block_cols;
  const int npages = (kv + bs - 1) / bs;
  const int first_page = s_begin / bs;
  const int nbt = min(npages, (s_end + bs - 1) / bs) - first_page;
  const bool cached = nbt <= kBtCache;
  if (warp == kKProducerWarp && cached) {
    for (int i = lane; i < nbt; i += 32) btc[i] = bt[first_page + i];
  }
  if (tid == 0) {
    mbar_init(&bars->q_full, 1);
    for (int s = 0; s < kStages; ++s) {
      mbar_init(&bars->k_full[s], 1);
      mbar_init(&bars->k_empty[s], 1);
      mbar_init(&bars->v_full[s], 1);
      mbar_init(&bars->v_empty[s], 1);
    }
    for (int s = 0; s < 2; ++s) {
      mbar_init(&bars->s_full[s], 1);
      mbar_init(&bars->p_full[s], 128);
      mbar_init(&bars->corr_go[s], 129);
      mbar_init(&bars->o_ready[s], 128);
    }
    mbar_init(&bars->o_final, 1);
    mbar_init(&bars->fin, 128);
    mbar_init(&bars->stall, 1);
    mbar_init(&bars->drain, 1);
    fence_mbar_init();
    cta_wait_init(static_cast<uint64_t>(p.wait_limit_us) * 1000);
  }
  if (warp == kMmaWarp) {
    tmem_alloc(&bars->tmem_base, kTmemCols);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tbase = bars->tmem_base;

  if (warp == kKProducerWarp || warp == kVProducerWarp) {
    // ---------------------------------------------------- K / V producers
    if (lane == 0) {
      const bool is_v = warp == kVProducerWarp;
      const CUtensorMap* tm = is_v ? &p.tmap_v : &p.tmap_k;
      uint64_t* full = is_v ? bars->v_full : bars->k_full;
      uint64_t* empty = is_v ? bars->v_empty : bars->k_empty;
      uint8_t* ring = smem + (is_v ? kOffV : kOffK);
      tma_prefetch_desc(tm);
      const int box_rows = bs < kTok ? bs : kTok;
      const int oob_row = p.num_blocks * bs;
      const int x0 = g * kHeadDim;
      int issued = 0;
      for (int j = 0; j < ntiles; ++j, ++issued) {
        const int st = j % kStages, u = j / kStages;
        const int t_tile = s_begin + j * kTok;
        uint8_t* dst = ring + st * kTileBytes;
        if (j >= kStages) mbar_wait(&empty[st], (u - 1) & 1);
        if (cta_aborted()) break;
        mbar_arrive_expect_tx(&full[st], kTileBytes);
        for (int off = 0; off < kTok; off += box_rows) {
          const int t = t_tile + off;
          const int page = t / bs;
          const int row =
              page < npages ? paged_row(cached ? btc[page - first_page] : bt[page], t, bs, p.num_blocks, oob_row)
                            : oob_row;
          tma_load_2d(dst + off * 128, tm, &full[st], x0, row);
          tma_load_2d(dst + kHalf + off * 128, tm, &full[st], x0 + 64, row);
        }
      }
      // aborting: wait (bounded) for the loads still in flight, the last
      // kStages issued, before the CTA can exit
      if (cta_aborted())
        for (int j = issued > kStages ? issued - kStages : 0; j < issued; ++j)
          mbar_wait_drain(&full[j % kStages], (j / kStages) & 1);
    }
  } else if (warp == kMmaWarp) {
    // ------------------------------------------------------------- MMA issuer
    if (lane == 0) {
      constexpr uint32_t fmt = kFp16 ? 0u : 1u;
      const uint32_t idesc_s = make_idesc_f16(128, 128, fmt, 0, 0);
      const uint32_t idesc_pv = make_idesc_f16(128, 128, fmt, 0, 1);
      const uint32_t sK = smem_u32(smem + kOffK);
      const uint32_t sV = smem_u32(smem + kOffV);
      mbar_arrive(&bars->corr_go[0]);  // tile 0 has no PV_{-1} to wait for
      mbar_wait(&bars->q_full, 0);
      tc_fence_after();
      for (int j = 0; j <= ntiles; ++j) {
        if (j < ntiles) {
          // S_j overwrites S buffer j&1, whose P_{j-2} was read by PV_{j-2}:
          // issued earlier by this thread, so it executes first.
          const int st = j % kStages, u = j / kStages;
          mbar_wait(&bars->k_full[st], u & 1);
          if (cta_aborted()) break;
          tc_fence_after();
          const uint32_t kb = sK + st * kTileBytes;
#pragma unroll
          for (int k = 0; k < 8; ++k) {
            const uint32_t koff = (k >> 2) * kHalf + (k & 3) * 32;
            umma_f16_ts(tbase + (j & 1) * 128, tbase + kColQ + k * 8, make_smem_desc(kb + koff, 16, 1024, 2),
                        idesc_s, k > 0 ? 1u : 0u);
          }
          umma_commit(&bars->s_full[j & 1]);
          umma_commit(&bars->k_empty[st]);
        }
        if (j >= 1) {
          const int i = j - 1;
          const int st = i % kStages, u = i / kStages;
          mbar_wait(&bars->v_full[st], u & 1);
          mbar_wait(&bars->p_full[i & 1], (i >> 1) & 1);
          mbar_wait(&bars->o_ready[i & 1], (i >> 1) & 1);
          if (cta_aborted()) break;
          tc_fence_after();
          const uint32_t vb = sV + st * kTileBytes;
#pragma unroll
          for (int k = 0; k < 8; ++k) {
            umma_f16_ts(tbase + kColO, tbase + (i & 1) * 128 + k * 8, make_smem_desc(vb + k * 2048, kHalf, 1024, 2),
                        idesc_pv, (i > 0 || k > 0) ? 1u : 0u);
          }
          umma_commit(&bars->v_empty[st]);
          if (i + 1 < ntiles) umma_commit(&bars->corr_go[(i + 1) & 1]);
          if (i == ntiles - 1) umma_commit(&bars->o_final);
        }
      }
      if (cta_aborted()) {
        // no MMA may still write TMEM (or read shared memory) when it is freed
        umma_commit(&bars->drain);
        mbar_wait_drain(&bars->drain, 0);
      }
    }
  } else if (warp < 4) {
    // ---------------------------------------------------------------- softmax
    const uint32_t lane_off = static_cast<uint32_t>(warp * 32) << 16;
    const float sl2 = p.scale_log2;
    float m = -INFINITY, l = 0.f;
    if (p.debug_stall) mbar_wait(&bars->stall, 0);  // test hook: runs into the wait limit, the CTA aborts
    for (int j = 0; j < ntiles; ++j) {
      const int st = j & 1, u = j >> 1;
      const int n_valid = min(kTok, s_end - (s_begin + j * kTok));
      mbar_wait(&bars->s_full[st], u & 1);
      tc_fence_after();
      uint32_t s0[32], s1[32], s2[32], s3[32];
      tmem_ld_32x32b_x32(tbase + lane_off + st * 128 + 0, s0);
      tmem_ld_32x32b_x32(tbase + lane_off + st * 128 + 32, s1);
      tmem_ld_32x32b_x32(tbase + lane_off + st * 128 + 64, s2);
      tmem_ld_32x32b_x32(tbase + lane_off + st * 128 + 96, s3);
      tmem_wait_ld();
      float s[128];
#pragma unroll
      for (int e = 0; e < 32; ++e) {
        s[e] = __uint_as_float(s0[e]);
        s[32 + e] = __uint_as_float(s1[e]);
        s[64 + e] = __uint_as_float(s2[e]);
        s[96 + e] = __uint_as_float(s3[e]);
      }
      if (n_valid < kTok) {
#pragma unroll
        for (int e = 0; e < kTok; ++e) s[e] = e < n_valid ? s[e] : -INFINITY;
      }
      float m0 = -INFINITY, m1 = -INFINITY, m2 = -INFINITY, m3 = -INFINITY;
#pragma unroll
      for (int e = 0; e < kTok; e += 8) {
        m0 = fmax3f(m0, s[e], s[e + 1]);
        m1 = fmax3f(m1, s[e + 2], s[e + 3]);
        m2 = fmax3f(m2, s[e + 4], s[e + 5]);
        m3 = fmax3f(m3, s[e + 6], s[e + 7]);
      }
      const float mx = fmax3f(m0, m1, fmaxf(m2, m3));
      const float m_new = fmaxf(m, mx * sl2);
      const float dm = (m == -INFINITY) ? 1.f : ex2(m - m_new);
      dmbuf[st * kRows + tid] = dm;
      mbar_arrive(&bars->corr_go[st]);
      // P_j over the first 64 columns of S_j (already in registers), in two
      // 32-column halves. PV_{j-2}, the last reader of this buffer,
      // completed before S_j did.
      float r0 = 0.f, r1 = 0.f, r2 = 0.f, r3 = 0.f;  // two packed row-sum accumulators
      const float neg_m = -m_new;
#pragma unroll
      for (int q4 = 0; q4 < 4; ++q4) {
        uint32_t pk[16];
#pragma unroll
        for (int e = 0; e < 32; e += 4) {
          const float* sv = s + q4 * 32 + e;
          float y0, y1, y2, y3;
          ffma2_bcast(y0, y1, sv[0], sv[1], sl2, neg_m);
          ffma2_bcast(y2, y3, sv[2], sv[3], sl2, neg_m);
          const float x0 = ex2(y0), x1 = ex2(y1), x2 = ex2(y2), x3 = ex2(y3);  // masked: ex2(-inf) = 0
          fadd2(r0, r1, x0, x1);
          fadd2(r2, r3, x2, x3);
          pk[e >> 1] = pack2<kFp16>(x0, x1);
          pk[(e >> 1) + 1] = pack2<kFp16>(x2, x3);
        }
        tmem_st_32x32b_x16(tbase + lane_off + st * 128 + q4 * 16, pk);
      }
      const float rs = (r0 + r1) + (r2 + r3);
      tmem_wait_st();
      tc_fence_before();
      mbar_arrive(&bars->p_full[st]);
      l = dm * l + rs;
      m = m_new;
    }
    lbuf[tid] = l;
    mbuf[tid] = m;
    mbar_arrive(&bars->fin);
  } else {
    // -------------------------------------------- correction + epilogue (4-7)
    const int r = tid - 128;  // row == TMEM lane (warp % 4 selects the lane quarter)
    const uint32_t lane_off = static_cast<uint32_t>((warp & 3) * 32) << 16;
    {
      // Q row -> tensor memory (A operand of S = Q K^T: 64 columns of 16-bit
      // pairs); rows past the unit are zero
      const uint4* src = reinterpret_cast<const uint4*>(static_cast<const uint16_t*>(p.query) +
                                                         out_row(r < unit_rows ? r : 0) * kHeadDim);
#pragma unroll
      for (int hf = 0; hf < 2; ++hf) {
        uint32_t qv[32];
#pragma unroll
        for (int c = 0; c < 8; ++c) {
          const uint4 v = r < unit_rows ? __ldg(src + hf * 8 + c) : make_uint4(0u, 0u, 0u, 0u);
          qv[4 * c] = v.x;
          qv[4 * c + 1] = v.y;
          qv[4 * c + 2] = v.z;
          qv[4 * c + 3] = v.w;
        }
        tmem_st_32x32b_x32(tbase + lane_off + kColQ + hf * 32, qv);
      }
      tmem_wait_st();
      tc_fence_before();
      asm volatile("bar.sync 2, 128;" ::: "memory");
      if (r == 0) mbar_arrive(&bars->q_full);
    }
    for (int j = 0; j < ntiles; ++j) {
      const int st = j & 1, u = j >> 1;
      // tile j's dm is in smem and PV_{j-1} has completed
      mbar_wait(&bars->corr_go[st], u & 1);
      const float dm = dmbuf[st * kRows + r];
      if (j >= 1 && __any_sync(0xffffffffu, dm != 1.f)) {
        tc_fence_after();
#pragma unroll
        for (int c = 0; c < 4; ++c) {
          uint32_t o[32];
          tmem_ld_32x32b_x32(tbase + lane_off + kColO + c * 32, o);
          tmem_wait_ld();
#pragma unroll
          for (int e = 0; e < 32; ++e) o[e] = __float_as_uint(__uint_as_float(o[e]) * dm);
          tmem_st_32x32b_x32(tbase + lane_off + kColO + c * 32, o);
        }
        tmem_wait_st();
      }
      tc_fence_before();
      mbar_arrive(&bars->o_ready[st]);
    }
    // epilogue: O / l once the last PV is done. The rows go through shared
    // memory (the K tiles are free by now) so that the global stores are whole
    // 512-byte rows per warp instruction rather than one 16-byte piece per
    // thread and row. Staging layout: [128 rows][32 x 16-byte chunks], chunk
    // j of row r at position j ^ (r % 32): conflict-free both ways.
    mbar_wait(&bars->fin, 0);
    mbar_wait(&bars->o_final, 0);
    tc_fence_after();
    const float l = lbuf[r], m = mbuf[r];
    const float inv = 1.f / l;
    const float lse_nat = (m + __log2f(l)) * 0.6931471805599453f;
    if (partial || p.out_dtype == 2) {
      // fp32 rows: stage unswizzled with a 528-byte row pitch (conflict-free
      // for the row-per-thread writes) and let the bulk-copy engine move each
      // 512-byte row to global memory.
      constexpr int kPitch = kHeadDim + 4;
      float* stage = reinterpret_cast<float*>(smem + kOffK);
#pragma unroll
      for (int c = 0; c < 4; ++c) {
        uint32_t o[32];
        tmem_ld_32x32b_x32(tbase + lane_off + kColO + c * 32, o);
        tmem_wait_ld();
#pragma unroll
        for (int i = 0; i < 8; ++i)
          *reinterpret_cast<float4*>(stage + r * kPitch + c * 32 + i * 4) =
              make_float4(__uint_as_float(o[4 * i]) * inv, __uint_as_float(o[4 * i + 1]) * inv,
                          __uint_as_float(o[4 * i + 2]) * inv, __uint_as_float(o[4 * i + 3]) * inv);
      }
      fence_proxy_async_smem();
      __syncwarp();
      if (r < unit_rows) {
        const size_t row = out_row(r);
        float* dst = partial ? p.part_o + (static_cast<size_t>(split) * plane + row) * kHeadDim
                             : static_cast<float*>(p.out) + row * kHeadDim;
        bulk_store_1d(dst, stage + r * kPitch, kHeadDim * 4);
        bulk_commit_group();
        if (partial) {
          p.part_lse[static_cast<size_t>(split) * plane + row] = lse_nat;
        } else {
          for (int c = 0; c < p.lse_stride; ++c) p.lse[row * p.lse_stride + c] = lse_nat;
        }
        bulk_wait_group0();
      }
    } else {
    float* stage = reinterpret_cast<float*>(smem + kOffK);
  #pragma unroll
      for (int c = 0; c < 4; ++c) {
        uint32_t o[32];
        tmem_ld_32x32b_x32(tbase + lane_off + kColO + c * 32, o);
        tmem_wait_ld();
  #pragma unroll
        for (int i = 0; i < 8; ++i)
          *reinterpret_cast<float4*>(stage + r * kHeadDim + (((c * 8 + i) ^ (r & 31)) << 2)) =
              make_float4(__uint_as_float(o[4 * i]) * inv, __uint_as_float(o[4 * i + 1]) * inv,
                          __uint_as_float(o[4 * i + 2]) * inv, __uint_as_float(o[4 * i + 3]) * inv);
      }
      if (r < unit_rows) {
        const size_t row = out_row(r);
        if (partial) {
          p.part_lse[static_cast<size_t>(split) * plane + row] = lse_nat;
        } else {
          for (int c = 0; c < p.lse_stride; ++c) p.lse[row * p.lse_stride + c] = lse_nat;
        }
      }
      asm volatile("bar.sync 2, 128;" ::: "memory");
      // warp w of the group stores rows [32w, 32w + 32); lane = 16-byte chunk.
      // Rows are walked as (query token, head) without divisions, 8 loads in
      // flight before their stores.
      {
        const int rbeg = (warp & 3) * 32;
        int tq_ = (row0 + rbeg) / p.group, hq_ = (row0 + rbeg) % p.group;
        const size_t head0 = static_cast<size_t>(g) * p.group;
  #pragma unroll
        for (int k0 = 0; k0 < 32; k0 += 8) {
          float4 v[8];
          size_t rows[8];
  #pragma unroll
          for (int k = 0; k < 8; ++k) {
            const int rr = rbeg + k0 + k;
            v[k] = *reinterpret_cast<const float4*>(stage + rr * kHeadDim + ((lane ^ (rr & 31)) << 2));
            rows[k] = static_cast<size_t>(tok0 + tq_) * p.num_heads + head0 + hq_;
            if (++hq_ == p.group) {
              hq_ = 0;
              ++tq_;
            }
          }
  #pragma unroll
          for (int k = 0; k < 8; ++k) {
            if (rbeg + k0 + k >= unit_rows) break;
            const size_t row = rows[k];
            if (partial) {
              *reinterpret_cast<float4*>(p.part_o + (static_cast<size_t>(split) * plane + row) * kHeadDim + lane * 4) =
                  v[k];
            } else if (p.out_dtype == 2) {
              *reinterpret_cast<float4*>(static_cast<float*>(p.out) + row * kHeadDim + lane * 4) = v[k];
            } else {
              const bool h = p.out_dtype == 1;
              const uint32_t a = h ? pack2<true>(v[k].x, v[k].y) : pack2<false>(v[k].x, v[k].y);
              const uint32_t bb = h ? pack2<true>(v[k].z, v[k].w) : pack2<false>(v[k].z, v[k].w);
              *reinterpret_cast<uint2*>(static_cast<uint16_t*>(p.out) + row * kHeadDim + lane * 4) = make_uint2(a, bb);
            }
          }
        }
      }
    }
  
      }
  tc_fence_before();
  __syncthreads();
  if (warp == kMmaWarp) {
    tc_fence_after();
    tmem_dealloc(tbase, kTmemCols);
  }
}

template <bool kFp16>
__global__ void __launch_bounds__(kThreads, 1) paged_prefix_tc_kernel(const __grid_constant__ PagedAttnLaunch p) {
  pdl_launch_dependents();
  paged_prefix_tc_body<kFp16>(p);
  if (p.pdl && threadIdx.x == 0) pdl_wait();
}

// ---------------------------------------------------------------------------
// Two-tile form: one CTA = (KV split, kv head x PAIR of 128-row tiles,
// request). Both row tiles (A = rows [256 p, 256 p + 128), B = the next 128)
// read the same K/V tiles, and two softmax warpgroups alternate so that the
// tensor pipe always has the other tile's MMAs while one softmax runs:
//   warps 0-3   softmax + epilogue of tile A (thread = row = TMEM lane)
//   warps 4-7   softmax + epilogue of tile B
//   warps 8-11  Q staging (both tiles, shared memory), O rescale of both tiles
//   warp 12     K producer (2-slot ring), warp 13 V producer (3-slot ring)
//   warp 14     MMA issuer (one thread)
// TMEM: S_A [0,128), S_B [128,256), O_A [256,384), O_B [384,512); P_X over the
// first 64 columns of S_X. Q_A, Q_B in shared memory (SS MMA for S). Per KV
// tile j the issue order is PV_A(j), S_A(j+1), PV_B(j), S_B(j+1): S_X(j+1)
// overwrites P_X(j) only after PV_X(j) (same issuing thread, executed in
// order). The arithmetic per row tile is the one-tile kernel's (S per 128
// tokens, running max, P = round16(exp(S - m)), unquantised row sums,
// O = dm O + P V with the rescale skipped exactly when no row of a warp moved
// its max), so both forms give the same quantisation structure.
constexpr int kPpThreads = 16 * 32;
// K slots free after S_B(j + 1) and are next needed by S_A(j + 3); V slots
// free after PV_B(j) and are next needed by PV_A(j + 3): the third V slot
// gives the V loads the same lookahead as the K loads (with two, PV_A waited
// for V on long prefixes).
constexpr int kPpKStages = 2;
constexpr int kPpVStages = 3;
constexpr int kPpBtCache = 128;
constexpr int kPpOffQ = 0;                                    // Q_A, Q_B: 2 x 32 KB
constexpr int kPpOffK = kPpOffQ + 2 * kTileBytes;             // K ring
constexpr int kPpOffV = kPpOffK + kPpKStages * kTileBytes;    // V ring
constexpr int kPpOffAux = kPpOffV + kPpVStages * kTileBytes;  // dm[2 tiles][128], block table
constexpr int kPpOffBars = kPpOffAux + 2 * 128 * 4 + kPpBtCache * 4;
static_assert(kPpOffBars % 16 == 0, "mbarriers need 8-byte alignment");
constexpr int kPpSmemBytes = kPpOffBars + 256 + 1024;
// static shared memory (the 16-byte wait state) counts against the same limit
static_assert(kPpSmemBytes + 16 <= 227 * 1024, "shared memory per CTA");
constexpr int kPpStagePitch = kHeadDim + 4;                   // fp32 epilogue staging row pitch (floats)
static_assert(2 * kRows * kPpStagePitch * 4 <= kPpOffAux, "both tiles' epilogue staging fit below the aux area");

struct __align__(8) PpBars {
  uint64_t q_full;
  uint64_t k_full[kPpKStages], k_empty[kPpKStages], v_full[kPpVStages], v_empty[kPpVStages];
  uint64_t s_full[2], p_full[2];          // per tile
  uint64_t corr_go[2][2], o_ready[2][2];  // [tile][j & 1]
  uint64_t o_final[2];
  uint64_t stall, drain;
  uint32_t tmem_base;
  int64_t ov_ta;  // segment A's tile count of an overlapped stage-1 (ov_seg != 0)
};
static_assert(sizeof(PpBars) <= 256, "barrier block");
constexpr int kPpNumBars = static_cast<int>(offsetof(PpBars, tmem_base) / sizeof(uint64_t));

// One piece of a two-tile CTA's work: request b, kv head g, row-tile pair mp
// against KV tokens [s_begin, min(kv_b, s_lim)), written as split-partial
// plane `split` (or as the final output when the call has one split and no
// partials). fill_to > split + 1: this CTA holds the unit's last piece, and
// planes (split, fill_to) of the unit's rows get -inf LSEs. The barriers are
// (re)initialised here (bars_live: they hold a previous piece's state and
// are invalidated first); TMEM is allocated by the caller. All threads call
// it; it returns whether the barriers are initialised, after a CTA barrier
// when it used them.
template <bool kFp16>
__device__ __forceinline__ bool paged_prefix_pp_piece(const PagedAttnLaunch& p, uint8_t* smem, uint32_t tbase,
                                                      int b, int g, int mp, int split, int s_begin, int s_lim,
                                                      int fill_to, bool bars_live) {
  // dm of tile t's current KV tile: written by the softmax (pass 1 of tile
  // j), read by the rescale before it releases PV(j); the next write (tile
  // j + 1) needs S(j + 1), which is issued after PV(j), so one slot per
  // row tile suffices
  float* dmbuf = reinterpret_cast<float*>(smem + kPpOffAux);          // [2 tiles][128]
  int32_t* btc = reinterpret_cast<int32_t*>(dmbuf + 2 * kRows);       // [kPpBtCache]
  PpBars* bars = reinterpret_cast<PpBars*>(smem + kPpOffBars);

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const int tid = threadIdx.x;

  const int kv = static_cast<int>(min(p.kv_seqlens[b], static_cast<int64_t>(p.block_cols) * p.block_size));
  const int q_len = p.q_seqlen_value > 0 ? p.q_seqlen_value : static_cast<int>(p.q_seqlens[b]);
  const int nrows = q_len * p.group;
  const int row0[2] = {mp * 2 * kRows, mp * 2 * kRows + kRows};
  const int unit_rows[2] = {min(kRows, nrows - row0[0]), min(kRows, nrows - row0[1])};
  const int tok0 = token_offset(p, b);
  if (unit_rows[0] <= 0) return bars_live;  // this request has fewer row tiles
  const int s_end = min(kv, s_lim);
  const int ntiles = s_end > s_begin ? (s_end - s_begin + kTok - 1) / kTok : 0;
  const size_t plane = static_cast<size_t>(p.num_tokens) * p.num_heads;
  const bool partial = p.num_splits > 1 || p.partial_out;

  auto out_row = [&](int t, int r) -> size_t {
    const int rr = row0[t] + r;
    return static_cast<size_t>(tok0 + rr / p.group) * p.num_heads + g * p.group + rr % p.group;
  };

  // planes past the unit's last piece hold no work
  for (int i = tid; i < 2 * kRows && fill_to > split + 1; i += blockDim.x) {
    const int t = i / kRows, r = i % kRows;
    if (r >= unit_rows[t]) continue;
    const size_t row = out_row(t, r);
    for (int sl = split + 1; sl < fill_to; ++sl) p.part_lse[static_cast<size_t>(sl) * plane + row] = -INFINITY;
  }

  if (ntiles == 0) {
    // split beyond this request's kv (or kv == 0)
    for (int i = tid; i < 2 * kRows; i += blockDim.x) {
      const int t = i / kRows, r = i % kRows;
      if (r >= unit_rows[t]) continue;
      const size_t row = out_row(t, r);
      if (partial) {
        p.part_lse[static_cast<size_t>(split) * plane + row] = -INFINITY;
      } else {
        float* o = static_cast<float*>(p.out) + row * kHeadDim;
        for (int c = 0; c < kHeadDim; ++c) o[c] = 0.f;
        for (int c = 0; c < p.lse_stride; ++c) p.lse[row * p.lse_stride + c] = -INFINITY;
      }
    }
    return bars_live;
  }

  const int bs = p.block_size;
  const int32_t* bt = p.block_table + static_cast<size_t>(b) * p.block_cols;
  const int npages = (kv + bs - 1) / bs;
  const int first_page = s_begin / bs;
  const int nbt = min(npages, (s_end + bs - 1) / bs) - first_page;
  const bool cached = nbt <= kPpBtCache;
  if (warp == 12 && cached) {
    for (int i = lane; i < nbt; i += 32) btc[i] = bt[first_page + i];
  }
  if (tid == 0) {
    if (bars_live) {
      uint64_t* all = reinterpret_cast<uint64_t*>(bars);
      for (int i = 0; i < kPpNumBars; ++i) mbar_inval(all + i);
    }
    mbar_init(&bars->q_full, 1);
    for (int s = 0; s < kPpKStages; ++s) {
      mbar_init(&bars->k_full[s], 1);
      mbar_init(&bars->k_empty[s], 1);
    }
    for (int s = 0; s < kPpVStages; ++s) {
      mbar_init(&bars->v_full[s], 1);
      mbar_init(&bars->v_empty[s], 1);
    }
    for (int t = 0; t < 2; ++t) {
      mbar_init(&bars->s_full[t], 1);
      mbar_init(&bars->p_full[t], 128);
      mbar_init(&bars->o_final[t], 1);
      for (int s = 0; s < 2; ++s) {
        mbar_init(&bars->corr_go[t][s], 129);
        mbar_init(&bars->o_ready[t][s], 128);
      }
    }
    mbar_init(&bars->stall, 1);
    mbar_init(&bars->drain, 1);
    fence_mbar_init();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();

  if (warp == 12 || warp == 13) {
    // ---------------------------------------------------- K / V producers
    if (lane == 0) {
      const bool is_v = warp == 13;
      const CUtensorMap* tm = is_v ? &p.tmap_v : &p.tmap_k;
      uint64_t* full = is_v ? bars->v_full : bars->k_full;
      uint64_t* empty = is_v ? bars->v_empty : bars->k_empty;
      uint8_t* ring = smem + (is_v ? kPpOffV : kPpOffK);
      tma_prefetch_desc(tm);
      const int box_rows = bs < kTok ? bs : kTok;
      const int oob_row = p.num_blocks * bs;
      const int x0 = g * kHeadDim;
      const int stages = is_v ? kPpVStages : kPpKStages;
      int issued = 0;
      for (int j = 0; j < ntiles; ++j, ++issued) {
        const int st = j % stages, u = j / stages;
        if (j >= stages) mbar_wait(&empty[st], (u - 1) & 1);
        if (cta_aborted()) break;
        mbar_arrive_expect_tx(&full[st], kTileBytes);
        uint8_t* dst = ring + st * kTileBytes;
        for (int off = 0; off < kTok; off += box_rows) {
          const int t = s_begin + j * kTok + off;
          const int page = t / bs;
          const int row =
              page < npages ? paged_row(cached ? btc[page - first_page] : bt[page], t, bs, p.num_blocks, oob_row)
                            : oob_row;
          tma_load_2d(dst + off * 128, tm, &full[st], x0, row);
          tma_load_2d(dst + kHalf + off * 128, tm, &full[st], x0 + 64, row);
        }
      }
      if (cta_aborted())
        for (int j = issued > stages ? issued - stages : 0; j < issued; ++j)
          mbar_wait_drain(&full[j % stages], (j / stages) & 1);
    }
  } else if (warp == 14) {
    // ------------------------------------------------------------- MMA issuer
    if (lane == 0) {
      constexpr uint32_t fmt = kFp16 ? 0u : 1u;
      const uint32_t idesc_s = make_idesc_f16(128, 128, fmt, 0, 0);
      const uint32_t idesc_pv = make_idesc_f16(128, 128, fmt, 0, 1);
      const uint32_t sQ = smem_u32(smem + kPpOffQ);
      const uint32_t sK = smem_u32(smem + kPpOffK);
      const uint32_t sV = smem_u32(smem + kPpOffV);
      auto issue_s = [&](int t, int kst) {
        const uint32_t qb = sQ + t * kTileBytes, kb = sK + kst * kTileBytes;
#pragma unroll
        for (int k = 0; k < 8; ++k) {
          const uint32_t koff = (k >> 2) * kHalf + (k & 3) * 32;
          umma_f16_ss(tbase + t * 128, make_smem_desc(qb + koff, 16, 1024, 2), make_smem_desc(kb + koff, 16, 1024, 2),
                      idesc_s, k > 0 ? 1u : 0u);
        }
        umma_commit(&bars->s_full[t]);
      };
      auto issue_pv = [&](int t, int vst, int j) {
        const uint32_t vb = sV + vst * kTileBytes;
#pragma unroll
        for (int k = 0; k < 8; ++k) {
          umma_f16_ts(tbase + 256 + t * 128, tbase + t * 128 + k * 8, make_smem_desc(vb + k * 2048, kHalf, 1024, 2),
                      idesc_pv, (j > 0 || k > 0) ? 1u : 0u);
        }
      };
      mbar_arrive(&bars->corr_go[0][0]);  // tile 0 has no PV_{-1} to wait for
      mbar_arrive(&bars->corr_go[1][0]);
      mbar_wait(&bars->q_full, 0);
      mbar_wait(&bars->k_full[0], 0);
      tc_fence_after();
      if (!cta_aborted()) {
        issue_s(0, 0);
        issue_s(1, 0);
        umma_commit(&bars->k_empty[0]);
      }
      for (int j = 0; j < ntiles && !cta_aborted(); ++j) {
        const int vst = j % kPpVStages;
        const bool more = j + 1 < ntiles;
        const int kst = (j + 1) % kPpKStages;
        mbar_wait(&bars->v_full[vst], (j / kPpVStages) & 1);
        for (int t = 0; t < 2; ++t) {
          mbar_wait(&bars->p_full[t], j & 1);
          mbar_wait(&bars->o_ready[t][j & 1], (j >> 1) & 1);
          if (cta_aborted()) break;
          tc_fence_after();
          issue_pv(t, vst, j);
          if (t == 1) umma_commit(&bars->v_empty[vst]);
          umma_commit(more ? &bars->corr_go[t][(j + 1) & 1] : &bars->o_final[t]);
          if (more) {
            if (t == 0) mbar_wait(&bars->k_full[kst], ((j + 1) / kPpKStages) & 1);
            if (cta_aborted()) break;
            tc_fence_after();
            issue_s(t, kst);
            if (t == 1) umma_commit(&bars->k_empty[kst]);
          }
        }
      }
      if (cta_aborted()) {
        umma_commit(&bars->drain);
        mbar_wait_drain(&bars->drain, 0);
      }
    }
  } else if (warp < 8) {
    // ------------------------------------------------- softmax + epilogue, tile t
    const int t = warp >> 2;
    const int r = tid & 127;  // row == TMEM lane
    const uint32_t lane_off = static_cast<uint32_t>((warp & 3) * 32) << 16;
    const uint32_t scol = tbase + lane_off + t * 128;
    const float sl2 = p.scale_log2;
    float m = -INFINITY, l = 0.f;
    if (p.debug_stall && t == 0) mbar_wait(&bars->stall, 0);  // test hook: runs into the wait limit
    for (int j = 0; j < ntiles; ++j) {
      const int n_valid = min(kTok, s_end - (s_begin + j * kTok));
      mbar_wait(&bars->s_full[t], j & 1);
      tc_fence_after();
      // pass 1: the tile's row max, 64 columns per TMEM round trip; four
      // independent three-input max chains. Columns past the split's end
      // (only in its last tile) read as -inf.
      const bool full = n_valid == kTok;
      float mx;
      {
        float m0 = -INFINITY, m1 = -INFINITY, m2 = -INFINITY, m3 = -INFINITY;
#pragma unroll 1
        for (int h = 0; h < 2; ++h) {
          uint32_t sa[32], sb[32];
          tmem_ld_32x32b_x32(scol + h * 64, sa);
          tmem_ld_32x32b_x32(scol + h * 64 + 32, sb);
          tmem_wait_ld();
          if (!full) mask_cols(sa, sb, n_valid - h * 64);
#pragma unroll
          for (int e = 0; e < 32; e += 4) {
            m0 = fmax3f(m0, __uint_as_float(sa[e]), __uint_as_float(sa[e + 1]));
            m1 = fmax3f(m1, __uint_as_float(sa[e + 2]), __uint_as_float(sa[e + 3]));
            m2 = fmax3f(m2, __uint_as_float(sb[e]), __uint_as_float(sb[e + 1]));
            m3 = fmax3f(m3, __uint_as_float(sb[e + 2]), __uint_as_float(sb[e + 3]));
          }
        }
        mx = fmax3f(m0, m1, fmaxf(m2, m3));
      }
      const float m_new = fmaxf(m, mx * sl2);
      const float dm = (m == -INFINITY) ? 1.f : ex2(m - m_new);
      dmbuf[t * kRows + r] = dm;
      mbar_arrive(&bars->corr_go[t][j & 1]);
      // pass 2: P = round16(exp(S - m)) over the first 64 columns, row sum of
      // the unrounded exps (two packed accumulators); 64 columns per round
      // trip (P of columns [64h, 64h + 64) goes to [32h, 32h + 32): never over
      // an S column a later load still reads). A masked column gives
      // exp2(-inf) = 0.
      float r0 = 0.f, r1 = 0.f, r2 = 0.f, r3 = 0.f;
      const float neg_m = -m_new;
#pragma unroll 1
      for (int h = 0; h < 2; ++h) {
        uint32_t sa[32], sb[32];
        tmem_ld_32x32b_x32(scol + h * 64, sa);
        tmem_ld_32x32b_x32(scol + h * 64 + 32, sb);
        tmem_wait_ld();
        if (!full) mask_cols(sa, sb, n_valid - h * 64);
#pragma unroll
        for (int q = 0; q < 2; ++q) {
          const uint32_t(&sv)[32] = q ? sb : sa;
          uint32_t pk[16];
#pragma unroll
          for (int e = 0; e < 32; e += 4) {
            float y0, y1, y2, y3;
            ffma2_bcast(y0, y1, __uint_as_float(sv[e]), __uint_as_float(sv[e + 1]), sl2, neg_m);
            ffma2_bcast(y2, y3, __uint_as_float(sv[e + 2]), __uint_as_float(sv[e + 3]), sl2, neg_m);
            const float x0 = ex2(y0), x1 = ex2(y1), x2 = ex2(y2), x3 = ex2(y3);
            fadd2(r0, r1, x0, x1);
            fadd2(r2, r3, x2, x3);
            pk[e >> 1] = pack2<kFp16>(x0, x1);
            pk[(e >> 1) + 1] = pack2<kFp16>(x2, x3);
          }
          tmem_st_32x32b_x16(scol + h * 32 + q * 16, pk);
        }
      }
      const float rs = (r0 + r1) + (r2 + r3);
      tmem_wait_st();
      tc_fence_before();
      mbar_arrive(&bars->p_full[t]);
      l = dm * l + rs;
      m = m_new;
    }
    // epilogue of tile t: O / l once its last PV is done, fp32 rows staged in
    // shared memory (whole 512-byte rows for the bulk-copy engine)
    mbar_wait(&bars->o_final[t], 0);
    tc_fence_after();
    const float inv = 1.f / l;
    const float lse_nat = (m + __log2f(l)) * 0.6931471805599453f;
    float* stage = reinterpret_cast<float*>(smem) + t * kRows * kPpStagePitch;
#pragma unroll
    for (int c = 0; c < 4; ++c) {
      uint32_t o[32];
      tmem_ld_32x32b_x32(tbase + lane_off + 256 + t * 128 + c * 32, o);
      tmem_wait_ld();
#pragma unroll
      for (int i = 0; i < 8; ++i)
        *reinterpret_cast<float4*>(stage + r * kPpStagePitch + c * 32 + i * 4) =
            make_float4(__uint_as_float(o[4 * i]) * inv, __uint_as_float(o[4 * i + 1]) * inv,
                        __uint_as_float(o[4 * i + 2]) * inv, __uint_as_float(o[4 * i + 3]) * inv);
    }
    fence_proxy_async_smem();
    __syncwarp();
    if (r < unit_rows[t]) {
      const size_t row = out_row(t, r);
      float* dst = partial ? p.part_o + (static_cast<size_t>(split) * plane + row) * kHeadDim
                           : static_cast<float*>(p.out) + row * kHeadDim;
      bulk_store_1d(dst, stage + r * kPpStagePitch, kHeadDim * 4);
      bulk_commit_group();
      if (partial) {
        p.part_lse[static_cast<size_t>(split) * plane + row] = lse_nat;
      } else {
        for (int c = 0; c < p.lse_stride; ++c) p.lse[row * p.lse_stride + c] = lse_nat;
      }
      bulk_wait_group0();
    }
  } else if (warp < 12) {
    // ----------------------------------- Q staging + O rescale of both tiles
    const int r = tid - 256;
    const uint32_t lane_off = static_cast<uint32_t>((warp & 3) * 32) << 16;
    {
      // Q rows -> shared memory in the K tiles' layout ([128 rows][64 x 16-bit]
      // halves, 128-byte swizzle); rows past the unit are zero
#pragma unroll 1
      for (int t = 0; t < 2; ++t) {
        const bool ok = r < unit_rows[t];
        const uint4* src = reinterpret_cast<const uint4*>(static_cast<const uint16_t*>(p.query) +
                                                           out_row(t, ok ? r : 0) * kHeadDim);
        uint8_t* qt = smem + kPpOffQ + t * kTileBytes;
#pragma unroll 4
        for (int c = 0; c < 16; ++c) {
          const uint4 v = ok ? __ldg(src + c) : make_uint4(0u, 0u, 0u, 0u);
          *reinterpret_cast<uint4*>(qt + (c >> 3) * kHalf + sw128(r, c & 7)) = v;
        }
      }
      fence_proxy_async_smem();
      asm volatile("bar.sync 2, 128;" ::: "memory");
      if (r == 0) mbar_arrive(&bars->q_full);
    }
    for (int j = 0; j < ntiles; ++j) {
#pragma unroll
      for (int t = 0; t < 2; ++t) {
        mbar_wait(&bars->corr_go[t][j & 1], (j >> 1) & 1);
        const float dm = dmbuf[t * kRows + r];
        if (j >= 1 && __any_sync(0xffffffffu, dm != 1.f)) {
          tc_fence_after();
#pragma unroll
          for (int h = 0; h < 2; ++h) {
            uint32_t oa[32], ob[32];
            const uint32_t a = tbase + lane_off + 256 + t * 128 + h * 64;
            tmem_ld_32x32b_x32(a, oa);
            tmem_ld_32x32b_x32(a + 32, ob);
            tmem_wait_ld();
#pragma unroll
            for (int e = 0; e < 32; ++e) {
              oa[e] = __float_as_uint(__uint_as_float(oa[e]) * dm);
              ob[e] = __float_as_uint(__uint_as_float(ob[e]) * dm);
            }
            tmem_st_32x32b_x32(a, oa);
            tmem_st_32x32b_x32(a + 32, ob);
          }
          tmem_wait_st();
        }
        tc_fence_before();
        mbar_arrive(&bars->o_ready[t][j & 1]);
      }
    }
  }
  tc_fence_before();
  __syncthreads();
  return true;
}

template <bool kFp16>
__global__ void __launch_bounds__(kPpThreads, 1) paged_prefix_pp_kernel(const __grid_constant__ PagedAttnLaunch p) {
  pdl_launch_dependents();
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  PpBars* bars = reinterpret_cast<PpBars*>(smem + kPpOffBars);
  if (threadIdx.x == 0) cta_wait_init(static_cast<uint64_t>(p.wait_limit_us) * 1000);
  if (threadIdx.x >> 5 == 14) {
    tmem_alloc(&bars->tmem_base, kTmemCols);
    tmem_relinquish();
  }
  const int64_t mtiles = (static_cast<int64_t>(p.max_q_seqlen) * p.group + kRows - 1) / kRows;
  const int64_t pairs = (mtiles + 1) / 2;
  const int64_t T = static_cast<int64_t>(p.batch) * p.kv_heads * p.piece_unit_tiles;
  if (p.ov_seg != 0 && threadIdx.x < 32) {
    // overlapped with the suffix decode: segment A's share of the tiles from
    // the suffix's kv tokens (the same sum, hence the same value, in every CTA)
    long long tok = 0;
    for (int b = threadIdx.x; b < p.ov_nlens; b += 32) tok += p.ov_lens[b];
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) tok += __shfl_xor_sync(0xffffffffu, tok, o);
    if (threadIdx.x == 0) bars->ov_ta = overlap_tiles(tok, p.kv_heads, p.ov_runs_a, p.ov_runs_b, T, p.piece_unit_tiles);
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tbase = bars->tmem_base;
  if (p.piece_ctas == 0) {
    // split grid: (split, kv head x row-tile pair, request)
    const int split = blockIdx.x;
    paged_prefix_pp_piece<kFp16>(p, smem, tbase, blockIdx.z, blockIdx.y % p.kv_heads, blockIdx.y / p.kv_heads,
                                 split, split * p.split_tokens, split * p.split_tokens + p.split_tokens, 0, false);
  } else {
    // equal runs of the concatenated (request, kv head) KV streams' tiles, each
    // run taken by `pairs` adjacent CTAs (one per row-tile pair of the
    // stream), so the pairs that read the same K/V tiles run in lock step and
    // share them through L2. One segment: G runs over [0, T). Overlapped with
    // the suffix decode: ga runs over [0, TA) (segment A) and gb runs over
    // [TA, T) (segment B), run numbers continuing from A into B. A stream's
    // pieces are numbered by the runs that hold them, starting at the run that
    // holds its first tile: run_of(x) = the largest r with bnd(r) <= x.
    const int64_t tc = p.piece_unit_tiles;
    int64_t ga, gb, TA, run;
    if (p.ov_seg == 0) {
      ga = gridDim.x / pairs, gb = 0, TA = T;
      run = blockIdx.x / pairs;
    } else {
      ga = p.ov_runs_a, gb = p.ov_runs_b, TA = bars->ov_ta;
      run = (p.ov_seg == 2 ? ga : 0) + blockIdx.x / pairs;
    }
    auto bnd = [&](int64_t r) -> int64_t { return r <= ga ? r * TA / ga : TA + (r - ga) * (T - TA) / gb; };
    auto run_of = [&](int64_t x) -> int64_t {
      return x < TA ? ((x + 1) * ga + TA - 1) / TA - 1 : ga + ((x - TA + 1) * gb + (T - TA) - 1) / (T - TA) - 1;
    };
    const int mp = static_cast<int>(blockIdx.x % pairs);
    const int64_t hi = bnd(run + 1);
    bool live = false;
    for (int64_t x = bnd(run); x < hi;) {
      const int64_t u = x / tc;
      const int64_t ue = (u + 1) * tc;
      const int64_t end = min(hi, ue);
      const int64_t plane = run - run_of(u * tc);
      if (plane >= p.num_splits) {  // outside the planned planes (the planner's bound rules this out)
        if (threadIdx.x == 0) atomicOr(&g_cascade_device_error, kErrBadPlan);
        break;
      }
      live = paged_prefix_pp_piece<kFp16>(p, smem, tbase, static_cast<int>(u / p.kv_heads),
                                          static_cast<int>(u % p.kv_heads), mp, static_cast<int>(plane),
                                          static_cast<int>((x - u * tc) * kTok), static_cast<int>((end - u * tc) * kTok),
                                          end == ue ? p.num_splits : 0, live);
      x = end;
      if (cta_aborted()) break;  // read after the piece's CTA barrier: the same in every thread
    }
  }
  tc_fence_before();
  __syncthreads();
  if (threadIdx.x >> 5 == 14) {
    tc_fence_after();
    tmem_dealloc(tbase, kTmemCols);
  }
  if (p.pdl && threadIdx.x == 0) pdl_wait();
}

}  // namespace

cudaError_t launch_paged_prefix_tc(const PagedAttnLaunch& p, bool fp16, cudaStream_t stream) {
  const int mtiles = (p.max_q_seqlen * p.group + kRows - 1) / kRows;
  if (mtiles >= 2 && (p.num_splits > 1 || p.partial_out || p.out_dtype == 2)) {
    // two row tiles per CTA (fp32 output or split partials)
    const dim3 grid = p.piece_ctas ? dim3(p.piece_ctas) : dim3(p.num_splits, p.kv_heads * ((mtiles + 1) / 2), p.batch);
    auto kern = fp16 ? paged_prefix_pp_kernel<true> : paged_prefix_pp_kernel<false>;
    cudaError_t e = ensure_smem_limit(reinterpret_cast<const void*>(kern), kPpSmemBytes);
    if (e != cudaSuccess) return e;
    return launch_maybe_pdl(kern, grid, dim3(kPpThreads), kPpSmemBytes, stream, p.pdl != 0, p);
  }
  dim3 grid(p.num_splits, p.kv_heads * mtiles, p.batch);
  auto kern = fp16 ? paged_prefix_tc_kernel<true> : paged_prefix_tc_kernel<false>;
  cudaError_t e = ensure_smem_limit(reinterpret_cast<const void*>(kern), kSmemBytes);
  if (e != cudaSuccess) return e;
  return launch_maybe_pdl(kern, grid, dim3(kThreads), kSmemBytes, stream, p.pdl != 0, p);
}

}  // namespace cascade
