// Internal launch interface between the C ABI (capi.cu) and the kernels.
#pragma once

#include <cuda.h>
#include <cuda_runtime.h>
#include <cstdint>

namespace cascade {

constexpr int kHeadDim = 128;
constexpr int kNumSMs = 148;

// Stage-1 overlapped with a cascade step's suffix decode (PagedAttnLaunch::
// ov_seg): segment A runs on kOvCtas SMs beside the decode, sized so that its
// runs last about as long as the decode: the suffix's kv bytes at
// kOvDecodeBytesPerNs (the decode's HBM rate on the SMs segment A leaves it:
// the C4 decode took 221 instead of 206 us with 48 SMs held, 254 with 64)
// over kOvTileNs per 128-token KV tile of a two-tile stage-1 CTA (C4: 55
// tiles in ~175 us). Within 40% of that estimate, the segment A whose
// segment-B runs are a whole fraction of a stream (tc >> k tiles, TA = T -
// runs_b * (tc >> k)) is taken instead: no segment-B run then straddles two
// (request, kv head) streams and every segment-B CTA does one piece (C4:
// 343 us at TA = 1,728 tiles, 32-tile runs, against 345-361 us for segments
// whose runs straddle streams). No segment A below kOvMinRunTiles tiles per
// run (16: the 2-rank shard of C4, 4 kv heads, gets a segment A of 864 tiles,
// 203 instead of 206 us serial; with 32 it had none); at most 3/5 of the
// tiles.
constexpr int kOvCtas = 64;
constexpr int64_t kOvMinRunTiles = 16;
constexpr double kOvDecodeBytesPerNs = 6000.0;  // 6 TB/s
constexpr double kOvTileNs = 3300.0;
__host__ __device__ inline int64_t overlap_tiles(int64_t suffix_tokens, int64_t kv_heads, int64_t runs_a,
                                                 int64_t runs_b, int64_t T, int64_t tc) {
  const double t_dec = static_cast<double>(suffix_tokens) * static_cast<double>(kv_heads) * 512.0 /
                       kOvDecodeBytesPerNs;
  int64_t per_run = static_cast<int64_t>(t_dec / kOvTileNs);
  const int64_t cap = (3 * T) / 5 / runs_a;
  if (per_run > cap) per_run = cap;
  if (per_run < kOvMinRunTiles) return 0;
  const int64_t est = per_run * runs_a;
  int64_t best = -1;
  for (int k = 0; k < 4; ++k) {
    const int64_t lb = tc >> k;
    if (lb < 8 || (lb << k) != tc) break;
    const int64_t ta = T - runs_b * lb;
    if (ta < kOvMinRunTiles * runs_a || ta > (3 * T) / 5 || 5 * (ta > est ? ta - est : est - ta) > 2 * est) continue;
    if (best < 0 || (ta > est ? ta - est : est - ta) < (best > est ? best - est : est - best)) best = ta;
  }
  return best >= 0 ? best : est;
}

// ----------------------------------------------------------------------------
// paged attention (decode path: <= 16 query rows per (request, kv head))
// ----------------------------------------------------------------------------
struct PagedAttnLaunch {
  CUtensorMap tmap_k;  // 2-D view [num_blocks*block_size, kv_heads*128], box {64, box_rows}, SW128
  CUtensorMap tmap_v;
  const void* query;
  const int32_t* block_table;
  const int64_t* q_seqlens;
  const int64_t* kv_seqlens;
  void* out;            // final output (nsplit == 1) in out_dtype
  float* lse;           // final lse (nsplit == 1), row stride lse_stride
  float* part_o;        // [nsplit][T*H][128] fp32 (nsplit > 1)
  float* part_lse;      // [nsplit][T*H]
  int32_t num_tokens, num_heads, kv_heads, group;
  int32_t batch, block_cols, block_size, num_blocks;
  int32_t q_seqlen_value;  // > 0 uniform, 0 = per-request (prefix-summed in kernel)
  int32_t max_q_seqlen;
  int32_t split_tokens, num_splits;
  // two-tile stage-1 over equal runs of KV tiles (0 = the split grid): the
  // grid has piece_ctas CTAs; (request, kv head, row-tile pair) units of
  // piece_unit_tiles 128-token tiles are concatenated and cut into piece_ctas
  // equal runs, each CTA taking one run (one or two pieces of units); a
  // piece's partial goes to plane "its index among the unit's pieces"
  int32_t piece_ctas, piece_unit_tiles;
  // Equal runs in two segments around a cascade step's suffix decode
  // (ov_seg 0: one segment of piece_ctas / pairs runs). The first TA tiles
  // are cut into ov_runs_a runs (segment A, launched before the decode on few
  // SMs: ov_seg 1), the rest into ov_runs_b runs (segment B, launched after
  // it: ov_seg 2). Every CTA of both launches computes the same TA from the
  // suffix's kv lengths (ov_lens, ov_nlens requests).
  int32_t ov_seg, ov_runs_a, ov_runs_b, ov_nlens;
  const int64_t* ov_lens;
  int32_t out_dtype;    // 0 bf16, 1 fp16, 2 fp32
  int32_t lse_stride;   // 8 (reference padded rows) or 1 (compact)
  int32_t partial_out;  // 1: always write split partials (a later combine produces the output)
  int32_t pdl;          // launched as a programmatic dependent of the previous kernel in the stream:
                        // 1 = every CTA waits for it before exiting, 2 = only the grid's last CTA does
  int32_t debug_stall;  // 1 (test hook): the consumers first wait on a barrier nothing completes
  uint32_t wait_limit_us;  // limit of one mbarrier wait (0 = the default, kWaitLimitNs)

  float scale_log2;     // softmax scale * log2(e)
  // planned decode (kernel 2): workspace arrays after the partials, or null
  int32_t* plan_items;     // [batch * num_splits] (request << 8) | split of the non-empty items
  int32_t* plan_count;     // number of items
  int32_t* plan_counters;  // [kv_heads] next item per kv head
};

cudaError_t launch_paged_decode(const PagedAttnLaunch& p, bool fp16, cudaStream_t stream);

// Launch `kern` with the programmatic-dependent attribute when `pdl` is set.
template <typename Arg>
cudaError_t launch_maybe_pdl(void (*kern)(Arg), dim3 grid, dim3 block, size_t smem, cudaStream_t stream, bool pdl,
                             const Arg& arg) {
  if (!pdl) {
    kern<<<grid, block, smem, stream>>>(arg);
    return cudaGetLastError();
  }
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = block;
  cfg.dynamicSmemBytes = smem;
  cfg.stream = stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  return cudaLaunchKernelEx(&cfg, kern, arg);
}


// Stage-1 tensor-core path (tcgen05, > 16 rows per (request, kv head)).
cudaError_t launch_paged_prefix_tc(const PagedAttnLaunch& p, bool fp16, cudaStream_t stream);

// Merge the nsplit partials of every (token, head) row into the final output.
cudaError_t launch_split_combine(const PagedAttnLaunch& p, cudaStream_t stream);

// One combine for a whole cascade step: merges the split partials of stage-1
// and of the suffix for every (token, head) row and writes the final output.
struct CascadeCombineLaunch {
  const float* o1;      // [n1][rows][128]
  const float* l1;      // [n1][rows]
  const float* o2;      // [n2][rows][128]
  const float* l2;      // [n2][rows]
  int32_t n1, n2;
  int64_t rows;
  void* out;            // [rows][128] in out_dtype
  int32_t out_dtype;    // 0 bf16, 1 fp16, 2 fp32
  float* lse_out;       // [rows] or null
  int32_t pdl;          // 1: launched as a programmatic dependent (waits for its primary first)
};

cudaError_t launch_cascade_combine(const CascadeCombineLaunch& p, cudaStream_t stream);

// ----------------------------------------------------------------------------
// LSE merge
// ----------------------------------------------------------------------------
struct LseMergeLaunch {
  const void* o1;
  const void* o2;
  const float* lse1;
  const float* lse2;
  void* out;
  int64_t rows;
  int32_t dim;
  int32_t stride1, stride2;
  int32_t o1_dtype, o2_dtype, out_dtype;  // 0 bf16, 1 fp16, 2 fp32
};

cudaError_t launch_lse_merge(const LseMergeLaunch& p, cudaStream_t stream);

// ----------------------------------------------------------------------------
// gate_up GEMM + epilogue
// ----------------------------------------------------------------------------
struct GateUpLaunch {
  void* ws;            // [M, 2I] bf16 (modes that write C)
  void* d;             // [M, I] bf16
  int64_t d_stride;
  int32_t M, K, I;
  int32_t mode;
};

cudaError_t launch_gateup(const GateUpLaunch& p, const void* a, const void* b, cudaStream_t stream);
// Modes 3/5/7/8: epilogue window traffic on an existing workspace (no GEMM).
cudaError_t launch_gateup_window(const void* ws, void* d, int64_t d_stride, int32_t M, int32_t I, int32_t mode,
                                 cudaStream_t stream);

// ----------------------------------------------------------------------------
// Residual add + RMSNorm statistics
// ----------------------------------------------------------------------------
struct RmsNormLaunch {
  const void* x1;      // [M, K] 16-bit
  const void* x2;      // [M, K] (modes 0 and 2)
  const void* gamma;   // [K] (mode 1)
  const void* beta;    // [K] or nullptr (mode 1)
  void* x_out;         // [M, K] (mode 0)
  float* rstd;         // [m_padded] (rows >= M zeroed)
  void* y;             // [M, K] (mode 1)
  int32_t M, K, m_padded, mode;
  float eps;
};

cudaError_t launch_add_rms_norm_stats(const RmsNormLaunch& p, bool fp16, cudaStream_t stream);

// Host: raise a kernel's dynamic shared memory limit once per (kernel,
// device) instead of on every launch.
cudaError_t ensure_smem_limit(const void* kernel, int bytes);

// Host: record `msg` as this thread's cascade_last_error() text; returns `code`.
int set_error(int code, const char* msg);

// Host: encode a 2-D bf16/fp16 tiled tensor map (SW128 when inner box is 64).
bool encode_tmap_2d(CUtensorMap* map, const void* base, uint64_t inner, uint64_t rows, uint64_t row_stride_bytes,
                    uint32_t box_inner, uint32_t box_rows, bool swizzle128, CUtensorMapL2promotion promo);

}  // namespace cascade
