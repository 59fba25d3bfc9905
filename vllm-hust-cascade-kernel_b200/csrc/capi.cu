// C ABI of the cascade-decode operator set (include/cascade_b200.h):
// validation (mirroring the reference op hosts' checks and messages),
// planning (kernel choice and KV splits, shape-only so workspaces can be
// sized without reading device memory), tensor-map encoding and launches.
#include <cuda.h>
#include <cuda_runtime.h>
#include <cudaTypedefs.h>

#include <algorithm>
#include <cstdarg>
#include <cstdint>
#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <mutex>
#include <string>
#include <vector>

#include "../../include/cascade_b200.h"
#include "kernels.h"
#include "ptx.cuh"

namespace cascade {

__device__ unsigned int g_cascade_device_error = 0;

namespace {

thread_local std::string g_last_error;

int fail(int code, const char* fmt, ...) {
  char buf[512];
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(buf, sizeof(buf), fmt, ap);
  va_end(ap);
  g_last_error = buf;
  return code;
}

int cuda_fail(const char* op, cudaError_t e) {
  return fail(CASCADE_ERR_CUDA, "%s: CUDA error %d (%s)", op, static_cast<int>(e), cudaGetErrorString(e));
}

PFN_cuTensorMapEncodeTiled_v12000 get_encode_fn() {
  static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void* ptr = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &ptr, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess) {
      fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(ptr);
    }
  });
  return fn;
}

bool block_size_ok(int64_t bs) {
  return bs == 16 || bs == 32 || bs == 64 || bs == 128 || bs == 256 || bs == 512;
}

constexpr int kDecodeSplit = 512;  // kv tokens per decode split (multiple of its 64-token tile)
constexpr int kTcTile = 128;       // kv tokens per tcgen05 tile
constexpr int kMaxSplits = 32;     // per request; the step combine merges up to 64 partials per row

int64_t ceil_div(int64_t a, int64_t b) { return (a + b - 1) / b; }

// Planned decode (kernel 2): uniform-q requests whose one-CTA-per-item grid
// at 512-token splits would exceed 16384 CTAs (~55 waves of two per SM). That
// grid is sized by the LONGEST request, so on such wide ragged batches most
// of its split CTAs find no work (C5: 36,864 CTAs, 4,968 with work); the
// planned form lists the non-empty items on the device and runs two
// persistent CTAs per SM over them. Narrower grids keep the per-item kernel
// (C4-like, 8,192 slots: 186 us widened per-item vs 202 us planned).
bool decode_planned(const cascade_paged_attn_t* p) {
  const int64_t cap = p->block_cols * p->block_size;
  return p->q_seqlen_value > 0 && cap > kDecodeSplit &&
         p->batch * p->kv_heads * ceil_div(cap, kDecodeSplit) > 16384;
}

// Equal-run schedule of the two-tile stage-1 (uniform q only): the 128-token
// KV tiles of all (request, kv head) streams, concatenated, are cut into
// equal runs, one per group of `pairs` CTAs (one CTA per row-tile pair of
// the stream, so the pairs that read the same K/V tiles stay in lock step),
// as many groups as fill the SMs once: every CTA does the same number of
// tiles whatever the stream count (the split grid can leave SMs idle: C4 ran
// 128 CTAs on 148 SMs). A run may end in one stream and start the next; a
// stream's pieces go to consecutive partial planes. Used when a run is
// shorter than a stream and at least kMinRunTiles long (the CTA's pipeline
// refills at each piece boundary). *ctas = runs x pairs.
constexpr int64_t kMinRunTiles = 8;
bool pp_pieces(const cascade_paged_attn_t* p, int64_t* ctas, int64_t* unit_tiles, int64_t* planes) {
  if (p->q_seqlen_value <= 0) return false;
  const int64_t rows = p->q_seqlen_value * (p->num_heads / p->kv_heads);
  if (rows <= 128) return false;
  const int64_t cap = std::max<int64_t>(1, p->block_cols * p->block_size);
  const int64_t pairs = ceil_div(rows, 256);
  const int64_t streams = p->kv_heads * p->batch;
  const int64_t tc = ceil_div(cap, kTcTile);
  const int64_t T = streams * tc;
  const int64_t G = std::min<int64_t>(kNumSMs / pairs, T);
  if (G <= streams || T < G * kMinRunTiles) return false;
  // the run [floor(r T / G), floor((r + 1) T / G)) that holds tile x
  auto run_of = [&](int64_t x) { return ((x + 1) * G + T - 1) / T - 1; };
  int64_t most = 1;
  for (int64_t u = 0; u < streams; ++u) most = std::max(most, run_of(u * tc + tc - 1) - run_of(u * tc) + 1);
  if (most > kMaxSplits) return false;
  *ctas = G * pairs;
  *unit_tiles = tc;
  *planes = most;
  return true;
}

// Stage-1 overlapped with the suffix decode in a decode-first cascade step
// (PagedAttnLaunch::ov_seg): stage-1 on the equal-run schedule, the decode on
// its per-item grid (the persistent planned decode keeps the serial order:
// held SMs stall its fixed grid, C5 decode 206 -> 351 us with 24 SMs held).
// Segment A = kOvCtas / pairs runs over the first TA tiles (TA decided on the
// device, 0 or at least kOvMinRunTiles per run and at most 3/5 of the
// tiles), segment B = the equal-run schedule's G runs over the rest. Every
// run is then at least `minrun` tiles long, so a unit of tc tiles meets at
// most ceil(tc / minrun) + 1 runs: *planes bounds its partial planes.
bool overlap_plan(const cascade_paged_attn_t* a, int kernel_a, int kernel_b, int64_t n2, int64_t* runs_a,
                  int64_t* runs_b, int64_t* planes) {
  int64_t ctas, tc, pl;
  if (kernel_a != 1 || kernel_b != 0 || n2 <= 0 || !pp_pieces(a, &ctas, &tc, &pl)) return false;
  const int64_t pairs = ceil_div(a->q_seqlen_value * (a->num_heads / a->kv_heads), 256);
  const int64_t ga = std::max<int64_t>(1, kOvCtas / pairs), gb = ctas / pairs;
  const int64_t T = a->kv_heads * a->batch * tc;
  const int64_t minrun = std::min<int64_t>(kOvMinRunTiles, (T - (3 * T) / 5) / gb);
  if (minrun < kMinRunTiles) return false;
  const int64_t np = ceil_div(tc, minrun) + 1;
  if (np > kMaxSplits || np + n2 > 64) return false;
  *runs_a = ga;
  *runs_b = gb;
  *planes = np;
  return true;
}

// Shape-only split rule of each kernel.
void split_rule(const cascade_paged_attn_t* p, int kernel, int64_t* split_tokens, int64_t* num_splits) {
  const int64_t cap = std::max<int64_t>(1, p->block_cols * p->block_size);
  if (kernel == 2) {
    *split_tokens = std::max<int64_t>(kDecodeSplit, ceil_div(ceil_div(cap, kMaxSplits), 64) * 64);
  } else if (kernel == 0) {
    // 512-token splits, widened (in 64-token tiles) so no request has more than
    // kMaxSplits. When the (request, kv head) pairs alone fill the GPU many
    // times over, splits of 1024 (>= 2048 pairs) or 2048 tokens (>= 4096
    // pairs): the grid's split dimension is sized by the LONGEST request, so
    // short requests leave most of their split CTAs empty, and each empty CTA
    // still holds a 99 KB slot while it reads its length and exits.
    const int64_t widen = std::min<int64_t>(4, std::max<int64_t>(1, p->batch * p->kv_heads / 1024));
    *split_tokens = std::max<int64_t>(kDecodeSplit * widen, ceil_div(ceil_div(cap, kMaxSplits), 64) * 64);
  } else {
    int64_t G, tc, planes;
    if (pp_pieces(p, &G, &tc, &planes)) {
      // equal runs: the longest piece, and one partial plane per piece of a unit
      const int64_t pairs = ceil_div(p->q_seqlen_value * (p->num_heads / p->kv_heads), 256);
      *split_tokens = ceil_div(tc * p->kv_heads * p->batch, G / pairs) * kTcTile;
      *num_splits = planes;
      return;
    }
    const int64_t group = p->num_heads / p->kv_heads;
    const int64_t rows_req = p->q_seqlen_value > 0 ? p->q_seqlen_value * group : 0;
    int64_t want;
    if (rows_req > 128) {
      // two-tile form: units = (kv head, pair of 128-row tiles); as many splits
      // as keep the grid within one wave of one CTA per SM (C4: 64 units x 2
      // splits = 128 CTAs; 3 splits would run 192 CTAs in two rounds), at least two
      const int64_t units = p->kv_heads * p->batch * ceil_div(rows_req, 256);
      want = std::max<int64_t>(2, kNumSMs / std::max<int64_t>(1, units));
    } else {
      const int64_t mtiles = std::max<int64_t>(p->batch, ceil_div(p->num_tokens * group, 128));
      const int64_t units = p->kv_heads * mtiles;
      // Enough splits for one 225 KB CTA per SM, and at least two: the grid is
      // sized by the longest request, and on ragged prefixes (C5) the longest
      // requests' CTAs set the kernel's length (C5 step 297 -> 276 us with two
      // splits; uniform shapes with >= 148 row tiles lose ~4% to the extra wave).
      want = std::max<int64_t>(2, ceil_div(kNumSMs, units));
    }
    int64_t ns = std::min<int64_t>(std::min<int64_t>(want, ceil_div(cap, kTcTile)), kMaxSplits);
    *split_tokens = ceil_div(ceil_div(cap, ns), kTcTile) * kTcTile;
  }
  *num_splits = ceil_div(cap, *split_tokens);
}

// The fused step's prefix-first rule: when the stage-1 grid has few (request,
// kv head, 128-row tile) units, splits are chosen so that about
// kPrefixFirstCtas CTAs of stage-1 run first, concurrently with the suffix
// decode on the remaining SMs. Measured on the C2 step (16 units): 2 splits
// (32 CTAs) 39.3 us, 4 splits 41.1 us, 1 split 64.7 us (stage-1 becomes the
// long pole); larger stage-1 grids (C4: 128 units, C5: 256) keep the
// decode-first order, where stage-1 needs most SMs anyway.
constexpr int64_t kPrefixFirstCtas = 32;
constexpr int64_t kPrefixFirstMaxUnits = 24;
bool prefix_first_splits(const cascade_paged_attn_t* p, int64_t* splits) {
  if (p->q_seqlen_value <= 0) return false;
  const int64_t group = p->num_heads / p->kv_heads;
  const int64_t rows = p->q_seqlen_value * group;
  const int64_t units = p->kv_heads * p->batch * ceil_div(rows, rows > 128 ? 256 : 128);
  if (units > kPrefixFirstMaxUnits) return false;
  const int64_t cap = std::max<int64_t>(1, p->block_cols * p->block_size);
  *splits = std::min(ceil_div(kPrefixFirstCtas, units), ceil_div(cap, kTcTile));
  return true;
}

// Partials [nsplit][rows][128] fp32 + LSE [nsplit][rows]; a planned decode
// adds its item list [batch * nsplit], the item count and one counter per kv
// head (int32).
size_t workspace_for(const cascade_paged_attn_t* p, int64_t num_splits, int kernel) {
  if (num_splits <= 1 && !(p->flags & CASCADE_FLAG_PARTIALS_ONLY)) return 0;
  const size_t rows = static_cast<size_t>(p->num_tokens) * p->num_heads;
  size_t bytes = static_cast<size_t>(num_splits) * rows * (kHeadDim + 1) * sizeof(float);
  if (kernel == 2) bytes += (static_cast<size_t>(p->batch) * num_splits + 1 + p->kv_heads) * sizeof(int32_t);
  return bytes;
}

// Validation common to both paged-attention entry points; `op` prefixes messages.
int validate_paged(const cascade_paged_attn_t* p, const char* op) {
  if (p == nullptr) return fail(CASCADE_ERR_INVALID, "%s: null argument", op);
  if (p->dtype != CASCADE_BF16 && p->dtype != CASCADE_FP16)
    return fail(CASCADE_ERR_INVALID, "%s: query/key/value must be bf16 or fp16", op);
  if (p->q_seqlen_value < 0)
    return fail(CASCADE_ERR_INVALID, "%s: q_seqlen_value must be >= 0 (0 = read seqlens from device)", op);
  if (p->head_dim != kHeadDim)
    return fail(CASCADE_ERR_UNSUPPORTED, "%s: only head dim 128 is supported (L1TileShape::K constraint)", op);
  if (!block_size_ok(p->block_size))
    return fail(CASCADE_ERR_UNSUPPORTED, "%s: paged blockSize must be one of 16, 32, 64, 128, 256, 512", op);
  if (p->kv_heads <= 0 || p->num_heads % p->kv_heads != 0)
    return fail(CASCADE_ERR_INVALID, "%s: numHeads must be a multiple of kvHeads", op);
  if (p->num_tokens < 0 || p->batch < 0 || p->num_blocks < 0 || p->block_cols < 0)
    return fail(CASCADE_ERR_INVALID, "%s: negative size", op);
  if (p->num_tokens * p->num_heads > (int64_t(1) << 31) / kHeadDim ||
      p->num_blocks * p->block_size >= (int64_t(1) << 31))
    return fail(CASCADE_ERR_UNSUPPORTED, "%s: problem too large for 32-bit row indices", op);
  if (p->q_seqlen_value > 0 && p->num_tokens != p->batch * p->q_seqlen_value)
    return fail(CASCADE_ERR_INVALID,
                "%s: with q_seqlen_value=%lld, query.size(0) must equal batch * q_seqlen_value", op,
                static_cast<long long>(p->q_seqlen_value));
  return CASCADE_OK;
}

int validate_pointers(const cascade_paged_attn_t* p, const char* op) {
  if (p->batch > 0 && p->num_tokens > 0) {
    if (!p->query || !p->key || !p->value || !p->block_table || !p->actual_q_seqlens || !p->actual_kv_seqlens)
      return fail(CASCADE_ERR_INVALID, "%s: null device pointer", op);
    if ((reinterpret_cast<uintptr_t>(p->key) | reinterpret_cast<uintptr_t>(p->value)) & 15)
      return fail(CASCADE_ERR_INVALID, "%s: key/value must be 16-byte aligned", op);
    if (reinterpret_cast<uintptr_t>(p->query) & 3)
      return fail(CASCADE_ERR_INVALID, "%s: query must be 4-byte aligned", op);
  }
  return CASCADE_OK;
}

// Legacy path: read the seqlens back and apply the reference's host checks
// (op_host/fa_fp32_stage1.cpp:223-241). `allow_zero_kv` relaxes kv >= 1.
int read_and_check_seqlens(const cascade_paged_attn_t* p, const char* op, bool allow_zero_kv, cudaStream_t stream,
                           int64_t* max_q) {
  std::vector<int64_t> q(p->batch), kv(p->batch);
  cudaError_t e = cudaMemcpyAsync(q.data(), p->actual_q_seqlens, p->batch * sizeof(int64_t),
                                  cudaMemcpyDeviceToHost, stream);
  if (e == cudaSuccess)
    e = cudaMemcpyAsync(kv.data(), p->actual_kv_seqlens, p->batch * sizeof(int64_t), cudaMemcpyDeviceToHost,
                        stream);
  if (e == cudaSuccess) e = cudaStreamSynchronize(stream);
  if (e != cudaSuccess) return cuda_fail(op, e);
  int64_t sum_q = 0, mq = 0, mkv = 0;
  for (int64_t b = 0; b < p->batch; ++b) {
    if (q[b] < 1 || kv[b] < (allow_zero_kv ? 0 : 1))
      return fail(CASCADE_ERR_INVALID, "%s: seqlens must be >= 1", op);
    sum_q += q[b];
    mq = std::max(mq, q[b]);
    mkv = std::max(mkv, kv[b]);
  }
  if (sum_q != p->num_tokens)
    return fail(CASCADE_ERR_INVALID, "%s: query.size(0) must equal sum(actual_q_seqlens)", op);
  if (ceil_div(mkv, p->block_size) > p->block_cols)
    return fail(CASCADE_ERR_INVALID, "%s: block_table cols too small for max kv seqlen", op);
  *max_q = mq;
  return CASCADE_OK;
}

int check_table(const char* op, const int32_t* bt, int64_t rows, int64_t cols, const int64_t* kv_lens,
                int64_t block_size, int64_t num_blocks, int64_t* bad_row, int64_t* bad_col) {
  for (int64_t r = 0; r < rows; ++r) {
    const int64_t kv = kv_lens[r] < 0 ? 0 : kv_lens[r];
    const int64_t pages = ceil_div(kv, block_size);
    if (pages > cols) {
      if (bad_row) *bad_row = r;
      if (bad_col) *bad_col = cols;
      return fail(CASCADE_ERR_INVALID, "%s: block_table row %lld needs %lld pages for kv %lld but has %lld columns",
                  op, static_cast<long long>(r), static_cast<long long>(pages), static_cast<long long>(kv),
                  static_cast<long long>(cols));
    }
    for (int64_t c = 0; c < pages; ++c) {
      const int32_t id = bt[r * cols + c];
      if (id < 0 || id >= num_blocks) {
        if (bad_row) *bad_row = r;
        if (bad_col) *bad_col = c;
        return fail(CASCADE_ERR_INVALID, "%s: block_table[%lld][%lld] = %d is outside [0, num_blocks=%lld)", op,
                    static_cast<long long>(r), static_cast<long long>(c), static_cast<int>(id),
                    static_cast<long long>(num_blocks));
      }
    }
  }
  return CASCADE_OK;
}

// Debug mode (CASCADE_FLAG_CHECK_BLOCK_IDS): read the block table and the kv
// lengths back and check every page the call will read.
int read_and_check_table(const cascade_paged_attn_t* p, const char* op, cudaStream_t stream) {
  std::vector<int32_t> bt(static_cast<size_t>(p->batch * p->block_cols));
  std::vector<int64_t> kv(static_cast<size_t>(p->batch));
  cudaError_t e = cudaSuccess;
  if (!bt.empty())
    e = cudaMemcpyAsync(bt.data(), p->block_table, bt.size() * sizeof(int32_t), cudaMemcpyDeviceToHost, stream);
  if (e == cudaSuccess)
    e = cudaMemcpyAsync(kv.data(), p->actual_kv_seqlens, kv.size() * sizeof(int64_t), cudaMemcpyDeviceToHost, stream);
  if (e == cudaSuccess) e = cudaStreamSynchronize(stream);
  if (e != cudaSuccess) return cuda_fail(op, e);
  return check_table(op, bt.data(), p->batch, p->block_cols, kv.data(), p->block_size, p->num_blocks, nullptr,
                     nullptr);
}

// Validation, seqlen read-back (legacy path), planning and tensor maps of one
// paged-attention call. On success *L holds everything but the output and
// workspace pointers. Returns CASCADE_OK with plan->num_splits == 0 for an
// empty problem (nothing to launch).
int prepare_paged(const cascade_paged_attn_t* p, const char* op, bool suffix, cudaStream_t stream,
                  cascade_attn_plan_t* plan, PagedAttnLaunch* L) {
  int rc = validate_paged(p, op);
  if (rc == CASCADE_OK) rc = validate_pointers(p, op);
  if (rc) return rc;
  std::memset(L, 0, sizeof(*L));
  if (p->batch == 0 || p->num_tokens == 0) {
    plan->num_splits = 0;
    return CASCADE_OK;
  }
  int64_t max_q = p->q_seqlen_value;
  if (p->q_seqlen_value == 0) {
    rc = read_and_check_seqlens(p, op, suffix, stream, &max_q);
    if (rc) return rc;
  }
  if (p->flags & CASCADE_FLAG_CHECK_BLOCK_IDS) {
    rc = read_and_check_table(p, op, stream);
    if (rc) return rc;
  }
  rc = cascade_plan_paged_attn(p, max_q, suffix ? 1 : 0, plan);
  if (rc) return rc;
  const bool tc = plan->kernel == 1;
  const uint32_t box_rows = static_cast<uint32_t>(std::min<int64_t>(p->block_size, tc ? 128 : 64));
  const uint64_t inner = static_cast<uint64_t>(p->kv_heads) * kHeadDim;
  const uint64_t rows = static_cast<uint64_t>(p->num_blocks) * p->block_size;
  if (rows == 0) return fail(CASCADE_ERR_INVALID, "%s: empty KV pool", op);
  if (!encode_tmap_2d(&L->tmap_k, p->key, inner, rows, inner * 2, 64, box_rows, true,
                      CU_TENSOR_MAP_L2_PROMOTION_L2_256B) ||
      !encode_tmap_2d(&L->tmap_v, p->value, inner, rows, inner * 2, 64, box_rows, true,
                      CU_TENSOR_MAP_L2_PROMOTION_L2_256B))
    return fail(CASCADE_ERR_CUDA, "%s: cuTensorMapEncodeTiled failed", op);
  L->query = p->query;
  L->block_table = p->block_table;
  L->q_seqlens = p->actual_q_seqlens;
  L->kv_seqlens = p->actual_kv_seqlens;
  L->num_tokens = static_cast<int32_t>(p->num_tokens);
  L->num_heads = static_cast<int32_t>(p->num_heads);
  L->kv_heads = static_cast<int32_t>(p->kv_heads);
  L->group = static_cast<int32_t>(p->num_heads / p->kv_heads);
  L->batch = static_cast<int32_t>(p->batch);
  L->block_cols = static_cast<int32_t>(p->block_cols);
  L->block_size = static_cast<int32_t>(p->block_size);
  L->num_blocks = static_cast<int32_t>(p->num_blocks);
  L->q_seqlen_value = static_cast<int32_t>(p->q_seqlen_value);
  L->max_q_seqlen = static_cast<int32_t>(max_q);
  L->split_tokens = static_cast<int32_t>(plan->split_tokens);
  L->num_splits = static_cast<int32_t>(plan->num_splits);
  int64_t pc, put, planes;
  if (tc && pp_pieces(p, &pc, &put, &planes)) {
    L->piece_ctas = static_cast<int32_t>(pc);
    L->piece_unit_tiles = static_cast<int32_t>(put);
  }
  L->out_dtype = suffix ? p->dtype : CASCADE_FP32;
  L->lse_stride = suffix ? 1 : 8;
  L->partial_out = (p->flags & CASCADE_FLAG_PARTIALS_ONLY) ? 1 : 0;
  L->debug_stall = (p->flags & CASCADE_FLAG_DEBUG_STALL) ? 1 : 0;

  L->wait_limit_us = L->debug_stall ? 1000u : 0u;
  L->scale_log2 = static_cast<float>(1.0 / std::sqrt(static_cast<double>(kHeadDim)) * 1.4426950408889634);
  return CASCADE_OK;
}

int check_workspace(const char* op, void* ws, size_t ws_bytes, size_t need) {
  if (need == 0) return CASCADE_OK;
  if (ws == nullptr || ws_bytes < need)
    return fail(CASCADE_ERR_WORKSPACE, "%s: workspace of %zu bytes required, %zu given", op, need, ws_bytes);
  if (reinterpret_cast<uintptr_t>(ws) & 15) return fail(CASCADE_ERR_INVALID, "%s: workspace must be 16-byte aligned", op);
  return CASCADE_OK;
}

void set_partials(PagedAttnLaunch* L, void* ws, int kernel) {
  const size_t nrows = static_cast<size_t>(L->num_tokens) * L->num_heads;
  L->part_o = static_cast<float*>(ws);
  L->part_lse = ws ? static_cast<float*>(ws) + static_cast<size_t>(L->num_splits) * nrows * kHeadDim : nullptr;
  L->plan_items = L->plan_count = L->plan_counters = nullptr;
  if (kernel == 2 && ws) {
    L->plan_items = reinterpret_cast<int32_t*>(L->part_lse + static_cast<size_t>(L->num_splits) * nrows);
    L->plan_count = L->plan_items + static_cast<size_t>(L->batch) * L->num_splits;
    L->plan_counters = L->plan_count + 1;
  }
}

cudaError_t launch_attention(const PagedAttnLaunch& L, int kernel, bool fp16, cudaStream_t stream) {
  return kernel == 1 ? launch_paged_prefix_tc(L, fp16, stream) : launch_paged_decode(L, fp16, stream);
}

int run_paged(const cascade_paged_attn_t* p, const char* op, bool suffix, void* out, float* lse, void* ws,
              size_t ws_bytes, cudaStream_t stream) {
  cascade_attn_plan_t plan;
  PagedAttnLaunch L;
  int rc = prepare_paged(p, op, suffix, stream, &plan, &L);
  if (rc || plan.num_splits == 0) return rc;
  const bool partials_only = L.partial_out != 0;
  if (!partials_only && (!out || !lse)) return fail(CASCADE_ERR_INVALID, "%s: null output pointer", op);
  rc = check_workspace(op, ws, ws_bytes, plan.workspace_bytes);
  if (rc) return rc;
  L.out = out;
  L.lse = lse;
  set_partials(&L, ws, plan.kernel);
  cudaError_t e = launch_attention(L, plan.kernel, p->dtype == CASCADE_FP16, stream);
  if (e == cudaSuccess && plan.num_splits > 1 && !partials_only) e = launch_split_combine(L, stream);
  if (e != cudaSuccess) return cuda_fail(op, e);
  return CASCADE_OK;
}

}  // namespace

bool encode_tmap_2d(CUtensorMap* map, const void* base, uint64_t inner, uint64_t rows, uint64_t row_stride_bytes,
                    uint32_t box_inner, uint32_t box_rows, bool swizzle128, CUtensorMapL2promotion promo) {
  auto fn = get_encode_fn();
  if (!fn) return false;
  cuuint64_t dims[2] = {inner, rows};
  cuuint64_t strides[1] = {row_stride_bytes};
  cuuint32_t box[2] = {box_inner, box_rows};
  cuuint32_t estr[2] = {1, 1};
  CUresult r = fn(map, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, const_cast<void*>(base), dims, strides, box, estr,
                  CU_TENSOR_MAP_INTERLEAVE_NONE,
                  swizzle128 ? CU_TENSOR_MAP_SWIZZLE_128B : CU_TENSOR_MAP_SWIZZLE_NONE, promo,
                  CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  return r == CUDA_SUCCESS;
}

cudaError_t ensure_smem_limit(const void* kernel, int bytes) {
  static std::mutex mu;
  static std::vector<std::pair<std::pair<const void*, int>, int>> done;  // ((kernel, device), bytes)
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return e;
  std::lock_guard<std::mutex> lock(mu);
  for (const auto& d : done)
    if (d.first.first == kernel && d.first.second == dev && d.second >= bytes) return cudaSuccess;
  e = cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, bytes);
  if (e == cudaSuccess) done.push_back({{kernel, dev}, bytes});
  return e;
}

int set_error(int code, const char* msg) {
  g_last_error = msg;
  return code;
}

}  // namespace cascade

using namespace cascade;

extern "C" {

const char* cascade_last_error(void) { return g_last_error.c_str(); }

int cascade_version(void) { return 100; }

int cascade_device_error(uint32_t* word) {
  unsigned int v = 0, zero = 0;
  cudaError_t e = cudaDeviceSynchronize();
  if (e == cudaSuccess) e = cudaMemcpyFromSymbol(&v, g_cascade_device_error, sizeof(v));
  if (e == cudaSuccess) e = cudaMemcpyToSymbol(g_cascade_device_error, &zero, sizeof(zero));
  if (e != cudaSuccess) return cuda_fail("cascade_device_error", e);
  if (word) *word = v;
  return CASCADE_OK;
}

int cascade_check_block_table(const int32_t* bt, int64_t rows, int64_t cols, const int64_t* kv_lens,
                              int64_t block_size, int64_t num_blocks, int64_t* bad_row, int64_t* bad_col) {
  const char* op = "cascade_check_block_table";
  if (rows < 0 || cols < 0 || block_size <= 0 || num_blocks < 0)
    return fail(CASCADE_ERR_INVALID, "%s: negative size", op);
  if (rows > 0 && (!kv_lens || (cols > 0 && !bt))) return fail(CASCADE_ERR_INVALID, "%s: null pointer", op);
  return check_table(op, bt, rows, cols, kv_lens, block_size, num_blocks, bad_row, bad_col);
}

int cascade_plan_paged_attn(const cascade_paged_attn_t* p, int64_t max_q_seqlen, int32_t suffix_mode,
                            cascade_attn_plan_t* plan) {
  const char* op = suffix_mode ? "cascade_suffix_decode" : "fa_fp32_stage1";
  int rc = validate_paged(p, op);
  if (rc) return rc;
  if (!plan) return fail(CASCADE_ERR_INVALID, "%s: null plan", op);
  const int64_t group = p->num_heads / p->kv_heads;
  const int64_t rows = std::max<int64_t>(1, max_q_seqlen) * group;
  plan->kernel = rows <= 16 ? (decode_planned(p) ? 2 : 0) : 1;
  plan->rows_per_group = static_cast<int32_t>(std::min<int64_t>(rows, INT32_MAX));
  split_rule(p, plan->kernel, &plan->split_tokens, &plan->num_splits);
  plan->workspace_bytes = workspace_for(p, plan->num_splits, plan->kernel);
  return CASCADE_OK;
}

static size_t workspace_size_any(const cascade_paged_attn_t* p, int suffix) {
  if (validate_paged(p, suffix ? "cascade_suffix_decode" : "fa_fp32_stage1")) return 0;
  if (p->batch == 0 || p->num_tokens == 0) return 0;
  if (p->q_seqlen_value > 0) {
    cascade_attn_plan_t plan;
    if (cascade_plan_paged_attn(p, p->q_seqlen_value, suffix, &plan)) return 0;
    return plan.workspace_bytes;
  }
  // per-request q lengths: the kernel is chosen after reading them, so size
  // for whichever kernel needs more
  size_t best = 0;
  for (int k = 0; k < 2; ++k) {
    int64_t st, ns;
    split_rule(p, k, &st, &ns);
    best = std::max(best, workspace_for(p, ns, k));
  }
  return best;
}

size_t cascade_fa_fp32_stage1_workspace_size(const cascade_paged_attn_t* p) { return workspace_size_any(p, 0); }

size_t cascade_suffix_decode_workspace_size(const cascade_paged_attn_t* p) { return workspace_size_any(p, 1); }

int cascade_fa_fp32_stage1(const cascade_paged_attn_t* p, float* out, float* lse, void* workspace,
                           size_t workspace_bytes, cascade_stream_t stream) {
  return run_paged(p, "fa_fp32_stage1", false, out, lse, workspace, workspace_bytes,
                   reinterpret_cast<cudaStream_t>(stream));
}

int cascade_suffix_decode(const cascade_paged_attn_t* p, void* out, float* lse, void* workspace,
                          size_t workspace_bytes, cascade_stream_t stream) {
  return run_paged(p, "cascade_suffix_decode", true, out, lse, workspace, workspace_bytes,
                   reinterpret_cast<cudaStream_t>(stream));
}

static size_t align_up(size_t x, size_t a) { return (x + a - 1) / a * a; }

size_t cascade_decode_step_workspace_size(const cascade_paged_attn_t* prefix, const cascade_paged_attn_t* suffix) {
  if (!prefix || !suffix) return 0;
  cascade_paged_attn_t a = *prefix, b = *suffix;
  a.flags |= CASCADE_FLAG_PARTIALS_ONLY;
  b.flags |= CASCADE_FLAG_PARTIALS_ONLY;
  size_t need_a = workspace_size_any(&a, 1);
  cascade_attn_plan_t pa, pb;
  int64_t ra, rb, planes;
  if (a.q_seqlen_value > 0 && b.q_seqlen_value > 0 && a.batch > 0 && b.batch > 0 && a.num_tokens > 0 &&
      cascade_plan_paged_attn(&a, a.q_seqlen_value, 1, &pa) == CASCADE_OK &&
      cascade_plan_paged_attn(&b, b.q_seqlen_value, 1, &pb) == CASCADE_OK &&
      overlap_plan(&a, pa.kernel, pb.kernel, pb.num_splits, &ra, &rb, &planes))
    need_a = std::max(need_a, workspace_for(&a, planes, 1));
  return align_up(need_a, 256) + align_up(workspace_size_any(&b, 1), 256);
}

int cascade_decode_step(const cascade_paged_attn_t* prefix, const cascade_paged_attn_t* suffix, void* out,
                        int32_t out_dtype, float* lse_out, void* workspace, size_t workspace_bytes,
                        cascade_stream_t stream) {
  const char* op = "cascade_decode_step";
  if (!prefix || !suffix) return fail(CASCADE_ERR_INVALID, "%s: null argument", op);
  if (out_dtype != CASCADE_BF16 && out_dtype != CASCADE_FP16 && out_dtype != CASCADE_FP32)
    return fail(CASCADE_ERR_INVALID, "%s: out dtype must be bf16, fp16 or fp32", op);
  if (prefix->num_tokens != suffix->num_tokens || prefix->num_heads != suffix->num_heads ||
      prefix->dtype != suffix->dtype || prefix->head_dim != suffix->head_dim)
    return fail(CASCADE_ERR_INVALID, "%s: prefix and suffix must describe the same query tensor", op);
  const size_t rows = static_cast<size_t>(suffix->num_tokens) * suffix->num_heads;
  if (rows == 0) return CASCADE_OK;
  if (!out) return fail(CASCADE_ERR_INVALID, "%s: null output pointer", op);
  cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
  cascade_paged_attn_t a = *prefix, b = *suffix;
  a.flags |= CASCADE_FLAG_PARTIALS_ONLY;
  b.flags |= CASCADE_FLAG_PARTIALS_ONLY;
  cascade_attn_plan_t pa, pb;
  PagedAttnLaunch La, Lb;
  int rc = prepare_paged(&a, op, true, st, &pa, &La);
  if (rc == CASCADE_OK) rc = prepare_paged(&b, op, true, st, &pb, &Lb);
  if (rc) return rc;
  const bool fp16 = suffix->dtype == CASCADE_FP16;
  // Prefix-first schedule (a small stage-1 grid, e.g. the Llama-3-8B step):
  // stage-1 runs first on about kPrefixFirstCtas SMs with fewer, longer
  // splits, and the suffix decode is its programmatic dependent on the other
  // SMs, so the shared prefix is read while the suffixes stream instead of
  // after them (C2 step 43.7 -> 39.3 us against the decode-first order).
  int64_t pf_splits = 0;
  const bool prefix_first = pa.num_splits && pa.kernel == 1 && pb.num_splits &&
                            prefix_first_splits(&a, &pf_splits);
  // Overlap (decode-first steps with a long stage-1): stage-1 segment A first
  // on kOvCtas SMs, the decode as its programmatic dependent on the others
  // (only its last CTA waits for segment A), segment B after the decode on
  // all SMs (each CTA waits for the decode before exiting), so the
  // tensor-bound stage-1 runs beside the HBM-bound decode instead of after it.
  // Its stage-1 partial planes are sized by overlap_plan's bound (the same
  // rule cascade_decode_step_workspace_size applies).
  int64_t ov_a = 0, ov_b = 0, ov_planes = 0;
  const bool overlap = !prefix_first && pa.num_splits && pb.num_splits && a.q_seqlen_value > 0 &&
                       b.q_seqlen_value > 0 &&
                       overlap_plan(&a, pa.kernel, pb.kernel, Lb.num_splits, &ov_a, &ov_b, &ov_planes);
  size_t need_a = pa.num_splits ? align_up(pa.workspace_bytes, 256) : 0;
  if (overlap) need_a = std::max(need_a, align_up(workspace_for(&a, ov_planes, pa.kernel), 256));
  const size_t need_b = pb.num_splits ? align_up(pb.workspace_bytes, 256) : 0;
  rc = check_workspace(op, workspace, workspace_bytes, need_a + need_b);
  if (rc) return rc;
  if (prefix_first) {
    const int64_t cap = std::max<int64_t>(1, a.block_cols * a.block_size);
    La.split_tokens = static_cast<int32_t>(ceil_div(ceil_div(cap, pf_splits), kTcTile) * kTcTile);
    La.num_splits = static_cast<int32_t>(ceil_div(cap, La.split_tokens));
    La.piece_ctas = 0;  // the split grid
  }
  if (overlap) {
    La.num_splits = static_cast<int32_t>(ov_planes);
    La.ov_runs_a = static_cast<int32_t>(ov_a);
    La.ov_runs_b = static_cast<int32_t>(ov_b);
    La.ov_lens = b.actual_kv_seqlens;
    La.ov_nlens = static_cast<int32_t>(b.batch);
  }
  set_partials(&La, workspace, pa.kernel);
  set_partials(&Lb, static_cast<uint8_t*>(workspace) + need_a, pb.kernel);
  if ((pa.num_splits ? La.num_splits : 0) + (pb.num_splits ? Lb.num_splits : 0) > 64)
    return fail(CASCADE_ERR_UNSUPPORTED, "%s: more than 64 KV splits per row", op);
  cudaError_t e = cudaSuccess;
  // The suffix decode (the long KV stream) goes first; stage-1 is launched as
  // its programmatic dependent, so its CTAs take over SMs as the decode's
  // ragged tail drains instead of waiting for the whole grid, and the combine
  // is the programmatic dependent of stage-1 (each kernel's CTAs wait for the
  // kernel before them only when they exit; the combine waits at its start).
  if (prefix_first) {
    e = launch_attention(La, pa.kernel, fp16, st);
    Lb.pdl = 2;  // only its last CTA waits for stage-1: no slot is held while stage-1 runs
    if (e == cudaSuccess) e = launch_attention(Lb, pb.kernel, fp16, st);
  } else if (overlap) {
    const int64_t pairs = ceil_div(a.q_seqlen_value * (a.num_heads / a.kv_heads), 256);
    PagedAttnLaunch LA = La, LB = La;
    LA.ov_seg = 1;
    LA.piece_ctas = static_cast<int32_t>(ov_a * pairs);
    LA.pdl = 0;
    LB.ov_seg = 2;
    LB.piece_ctas = static_cast<int32_t>(ov_b * pairs);
    LB.pdl = 1;
    Lb.pdl = 2;
    e = launch_attention(LA, pa.kernel, fp16, st);
    if (e == cudaSuccess) e = launch_attention(Lb, pb.kernel, fp16, st);
    if (e == cudaSuccess) e = launch_attention(LB, pa.kernel, fp16, st);
  } else {
    if (pb.num_splits) e = launch_attention(Lb, pb.kernel, fp16, st);
    La.pdl = pb.num_splits ? 1 : 0;
    if (e == cudaSuccess && pa.num_splits) e = launch_attention(La, pa.kernel, fp16, st);
  }
  if (e == cudaSuccess) {
    CascadeCombineLaunch C;
    std::memset(&C, 0, sizeof(C));
    C.pdl = (pa.num_splits || pb.num_splits) ? 1 : 0;
    C.o1 = La.part_o;
    C.l1 = La.part_lse;
    C.n1 = pa.num_splits ? La.num_splits : 0;
    C.o2 = Lb.part_o;
    C.l2 = Lb.part_lse;
    C.n2 = pb.num_splits ? Lb.num_splits : 0;
    C.rows = static_cast<int64_t>(rows);
    C.out = out;
    C.out_dtype = out_dtype;
    C.lse_out = lse_out;
    e = launch_cascade_combine(C, st);
  }
  if (e != cudaSuccess) return cuda_fail(op, e);
  return CASCADE_OK;
}

int cascade_lse_merge(const void* o1, int32_t o1_dtype, const void* o2, int32_t o2_dtype, const float* lse1,
                      int64_t stride1, const float* lse2, int64_t stride2, void* out, int32_t out_dtype,
                      int64_t rows, int64_t dim, cascade_stream_t stream) {
  const char* op = "lse_merge";
  auto dt_ok = [](int32_t d) { return d == CASCADE_BF16 || d == CASCADE_FP16 || d == CASCADE_FP32; };
  if (!dt_ok(o1_dtype) || !dt_ok(o2_dtype) || !dt_ok(out_dtype))
    return fail(CASCADE_ERR_INVALID, "%s: dtypes must be bf16, fp16 or fp32", op);
  if (dim <= 0 || dim % 16 != 0)
    return fail(CASCADE_ERR_INVALID, "%s: head dim must be a multiple of 16 (MTE 32B alignment)", op);
  if (rows < 0) return fail(CASCADE_ERR_INVALID, "%s: negative row count", op);
  if (rows == 0) return CASCADE_OK;
  if (stride1 < 1 || stride1 > 64 || stride2 < 1 || stride2 > 64)
    return fail(CASCADE_ERR_INVALID, "%s: lse row stride must be in [1, 64]", op);
  if (!o1 || !o2 || !lse1 || !lse2 || !out) return fail(CASCADE_ERR_INVALID, "%s: null pointer", op);
  if ((reinterpret_cast<uintptr_t>(o1) | reinterpret_cast<uintptr_t>(o2) | reinterpret_cast<uintptr_t>(out)) & 15)
    return fail(CASCADE_ERR_INVALID, "%s: o1/o2/out must be 16-byte aligned", op);
  LseMergeLaunch L;
  L.o1 = o1;
  L.o2 = o2;
  L.lse1 = lse1;
  L.lse2 = lse2;
  L.out = out;
  L.rows = rows;
  L.dim = static_cast<int32_t>(dim);
  L.stride1 = static_cast<int32_t>(stride1);
  L.stride2 = static_cast<int32_t>(stride2);
  L.o1_dtype = o1_dtype;
  L.o2_dtype = o2_dtype;
  L.out_dtype = out_dtype;
  cudaError_t e = launch_lse_merge(L, reinterpret_cast<cudaStream_t>(stream));
  if (e != cudaSuccess) return cuda_fail(op, e);
  return CASCADE_OK;
}

int cascade_add_rms_norm_stats(const void* x1, const void* x2, const void* gamma, const void* beta, void* x_out,
                               float* rstd, void* y, int64_t M, int64_t K, int32_t dtype, int32_t mode, float eps,
                               cascade_stream_t stream) {
  // op_host/add_rms_norm_stats.cpp:64-104, same limits and texts
  const char* op = "add_rms_norm_stats";
  if (mode < 0 || mode > 2) return fail(CASCADE_ERR_INVALID, "%s: mode must be 0, 1 or 2", op);
  if (!(eps > 0.f)) return fail(CASCADE_ERR_INVALID, "%s: eps must be > 0", op);
  if (dtype != CASCADE_BF16 && dtype != CASCADE_FP16)
    return fail(CASCADE_ERR_INVALID, "%s: x1 must be bf16 or fp16", op);
  if (M <= 0) return fail(CASCADE_ERR_INVALID, "%s: empty row count", op);
  if (K <= 0 || K > 5120) return fail(CASCADE_ERR_INVALID, "%s: K must be in (0, 5120] (one row resident in UB)", op);
  if (K % 16 != 0) return fail(CASCADE_ERR_INVALID, "%s: K must be a multiple of 16 (32B row copies)", op);
  if (M > INT32_MAX) return fail(CASCADE_ERR_UNSUPPORTED, "%s: more than 2^31-1 rows", op);
  if (!x1 || !rstd) return fail(CASCADE_ERR_INVALID, "%s: null pointer", op);
  if (mode != 1 && !x2) return fail(CASCADE_ERR_INVALID, "%s: x2 must be contiguous, same shape and dtype as x1", op);
  if (mode == 0 && !x_out) return fail(CASCADE_ERR_INVALID, "%s: null x_out", op);
  if (mode == 1 && (!gamma || !y))
    return fail(CASCADE_ERR_INVALID, "%s: mode 1 needs a contiguous gamma of K elements, same dtype", op);
  auto mis = [](const void* q) { return (reinterpret_cast<uintptr_t>(q) & 15) != 0; };
  if (mis(x1) || (mode != 1 && mis(x2)) || (mode == 0 && mis(x_out)) ||
      (mode == 1 && (mis(gamma) || mis(y) || (beta && mis(beta)))))
    return fail(CASCADE_ERR_INVALID, "%s: tensors must be 16-byte aligned", op);
  RmsNormLaunch L;
  L.x1 = x1;
  L.x2 = mode == 1 ? nullptr : x2;
  L.gamma = mode == 1 ? gamma : nullptr;
  L.beta = mode == 1 ? beta : nullptr;
  L.x_out = mode == 0 ? x_out : nullptr;
  L.rstd = rstd;
  L.y = mode == 1 ? y : nullptr;
  L.M = static_cast<int32_t>(M);
  L.K = static_cast<int32_t>(K);
  L.m_padded = static_cast<int32_t>((M + 7) / 8 * 8);
  L.mode = mode;
  L.eps = eps;
  cudaError_t e = launch_add_rms_norm_stats(L, dtype == CASCADE_FP16, reinterpret_cast<cudaStream_t>(stream));
  if (e != cudaSuccess) return cuda_fail(op, e);
  return CASCADE_OK;
}

int cascade_f3_gateup_epilogue(const void* a, const void* b, void* ws, void* d, int64_t d_stride, int64_t M,
                               int64_t K, int64_t I, int32_t mode, cascade_stream_t stream) {
  const char* op = "f3_gateup_epilogue";
  if (!((mode >= 0 && mode <= 5) || mode == 7 || mode == 8))
    return fail(CASCADE_ERR_INVALID, "%s: mode must be 0..5, 7 or 8", op);
  if (M <= 0 || K <= 0) return fail(CASCADE_ERR_INVALID, "%s: empty input", op);
  if (K % 16 != 0) return fail(CASCADE_ERR_INVALID, "%s: K must be a multiple of 16", op);
  if (I <= 0 || I % 128 != 0) return fail(CASCADE_ERR_INVALID, "%s: I must be a multiple of the N tile", op);
  if (K < 64) return fail(CASCADE_ERR_INVALID, "%s: K must be >= 64 (L0 K tile)", op);
  if (M > INT32_MAX || K > INT32_MAX || I > INT32_MAX / 2)
    return fail(CASCADE_ERR_UNSUPPORTED, "%s: dimension too large", op);
  const bool needs_ws = mode != 1;
  const bool needs_d = mode != 2 && mode != 7;
  if (needs_ws && !ws) return fail(CASCADE_ERR_WORKSPACE, "%s: workspace must be contiguous bf16 [M, 2I]", op);
  if (needs_d && (!d || d_stride < I)) return fail(CASCADE_ERR_INVALID, "%s: d must be bf16 [M, I]", op);
  if (needs_d && (d_stride % 8 != 0 || (reinterpret_cast<uintptr_t>(d) & 15)))
    return fail(CASCADE_ERR_INVALID, "%s: d must be 16-byte aligned with a row stride multiple of 8", op);
  cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
  if (mode == 3 || mode == 5 || mode == 7 || mode == 8) {
    cudaError_t e = launch_gateup_window(ws, d, d_stride, static_cast<int32_t>(M), static_cast<int32_t>(I), mode, st);
    if (e != cudaSuccess) return cuda_fail(op, e);
    return CASCADE_OK;
  }
  if (!a || !b) return fail(CASCADE_ERR_INVALID, "%s: null input", op);
  if ((reinterpret_cast<uintptr_t>(a) | reinterpret_cast<uintptr_t>(b)) & 15)
    return fail(CASCADE_ERR_INVALID, "%s: a/b must be 16-byte aligned", op);
  GateUpLaunch L;
  std::memset(&L, 0, sizeof(L));
  L.ws = ws;
  L.d = d;
  L.d_stride = d_stride;
  L.M = static_cast<int32_t>(M);
  L.K = static_cast<int32_t>(K);
  L.I = static_cast<int32_t>(I);
  L.mode = mode;
  cudaError_t e = launch_gateup(L, a, b, st);
  if (e != cudaSuccess) return cuda_fail(op, e);
  return CASCADE_OK;
}

}  // extern "C"
