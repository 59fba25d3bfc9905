/*
 * cascade_b200.h -- C ABI of the B200 (sm_100a) cascade-decode operator set.
 *
 * Plain pointers and sizes only: no torch, no C++ types. Every entry point
 * runs asynchronously on the given CUDA stream and returns 0 on success or a
 * cascade_status code; cascade_last_error() gives the message of the last
 * failure on the calling thread (messages start with the reference op name,
 * e.g. "fa_fp32_stage1: ...", matching the reference's TORCH_CHECK texts).
 *
 * Device pointers are CUDA device (or managed) memory on the current device.
 * `stream` is a cudaStream_t (0 = legacy default stream).
 */
#ifndef CASCADE_B200_H
#define CASCADE_B200_H

#include <stddef.h>
#include <stdint.h>

#if defined(__GNUC__)
#define CASCADE_API __attribute__((visibility("default")))
#else
#define CASCADE_API
#endif

#ifdef __cplusplus
extern "C" {
#endif

typedef struct CUstream_st *cascade_stream_t; /* == cudaStream_t */

enum cascade_dtype {
  CASCADE_BF16 = 0,
  CASCADE_FP16 = 1,
  CASCADE_FP32 = 2,
};

enum cascade_status {
  CASCADE_OK = 0,
  CASCADE_ERR_INVALID = 1,     /* argument rejected by validation */
  CASCADE_ERR_CUDA = 2,        /* a CUDA runtime / driver call failed */
  CASCADE_ERR_WORKSPACE = 3,   /* workspace missing or too small */
  CASCADE_ERR_UNSUPPORTED = 4, /* shape outside the supported domain */
};

/* Paged-attention problem description shared by stage-1 and the suffix.
 * Layouts follow the reference op (ascend-kernel/csrc/ops.h:26-38,
 * ascend-kernel/README.md:122-131):
 *   query        [num_tokens, num_heads, head_dim], contiguous
 *   key / value  [num_blocks, block_size, kv_heads, head_dim], contiguous
 *   block_table  int32 [batch, block_cols]; block_cols is the row stride
 *   actual_q_seqlens / actual_kv_seqlens  int64 [batch], DEVICE memory
 * q_seqlen_value > 0: every request has that many query tokens (no device->
 * host reads; graph-capture safe). q_seqlen_value == 0: the seqlens are read
 * back to the host and validated (the reference's legacy path,
 * ascend-kernel/csrc/ops/fa_fp32_stage1/op_host/fa_fp32_stage1.cpp:215-246).
 */
typedef struct cascade_paged_attn {
  const void *query;
  const void *key;
  const void *value;
  const int32_t *block_table;
  const int64_t *actual_q_seqlens;
  const int64_t *actual_kv_seqlens;
  int64_t num_tokens;
  int64_t num_heads;
  int64_t head_dim;
  int64_t num_blocks;
  int64_t block_size;
  int64_t kv_heads;
  int64_t batch;
  int64_t block_cols;
  int64_t q_seqlen_value;
  int32_t dtype; /* cascade_dtype of query/key/value: BF16 or FP16 */
  int32_t flags; /* CASCADE_FLAG_* bits, normally 0 */
} cascade_paged_attn_t;

/* cascade_paged_attn_t.flags bit: write the split-KV partials
 * (workspace layout below) and skip the final combine; out/lse are not
 * touched. Used to time or chain the attention kernel alone. */
#define CASCADE_FLAG_PARTIALS_ONLY 1

/* cascade_paged_attn_t.flags bit, a test hook for the kernels' bounded waits
 * (no counterpart in the reference): the attention kernel's consumer warps
 * first wait on a barrier that nothing completes, with a 1 ms limit instead
 * of the default 100 ms. The wait runs out, the CTA aborts (its other waits
 * return at once, producers stop and drain their copies in flight, TMEM is
 * freed) and the call ends with (word & 1) set in cascade_device_error(). The
 * outputs of such a call are garbage. */
#define CASCADE_FLAG_DEBUG_STALL 2

/* cascade_paged_attn_t.flags bit, a debug mode: before launching, read the
 * block table and the kv lengths back to the host (a synchronising copy) and
 * reject the call with CASCADE_ERR_INVALID if a page a request reads has a
 * block id outside [0, num_blocks) (cascade_check_block_table below). Without
 * it the kernels still never read outside the pool: such a page reads as
 * zeros and the word cascade_device_error() reads has (word & 2) set. */
#define CASCADE_FLAG_CHECK_BLOCK_IDS 4

/* Host-side check of a block table against the paging contract (no CUDA
 * calls; host memory): every page a request reads -- entries
 * [0, ceil(kv_lens[r] / block_size)) of row r -- must hold a block id in
 * [0, num_blocks), and ceil(kv_lens[r] / block_size) must not exceed cols.
 * bt: int32 [rows, cols] (row stride cols); kv_lens: int64 [rows].
 * Returns 0, or CASCADE_ERR_INVALID with the first offending (row, column)
 * in *bad_row / *bad_col (either may be NULL) and a message naming them. The
 * reference guards the same contract statically
 * (ascend-kernel/csrc/ops/fa_fp32_stage1/op_kernel/kernel_fa_fp32_stage1.cpp:107-112). */
CASCADE_API int cascade_check_block_table(const int32_t *bt, int64_t rows, int64_t cols, const int64_t *kv_lens,
                                          int64_t block_size, int64_t num_blocks, int64_t *bad_row,
                                          int64_t *bad_col);

/* Bytes of device workspace a call with this description needs (split-KV
 * partials). Depends on shapes only, never on the seqlen values. 0 = none. */
CASCADE_API size_t cascade_fa_fp32_stage1_workspace_size(const cascade_paged_attn_t *p);

/* Stage-1 shared-prefix paged attention, fp32 out + padded LSE.
 * Replaces ascend_kernel::fa_fp32_stage1
 *   (ascend-kernel/csrc/ops/fa_fp32_stage1/op_host/fa_fp32_stage1.cpp:178-329,
 *    schema ascend-kernel/csrc/register.cpp:25-26).
 * out: fp32 [num_tokens, num_heads, head_dim]
 * lse: fp32 [num_tokens * num_heads * 8]; row (token*H + head) holds 8 copies
 *      of ln(sum exp) + max (the reference's 32-byte padded LSE rows).
 * A request with kv length 0 (accepted only when q_seqlen_value > 0) yields
 * out = 0 and lse = -inf. */
CASCADE_API int cascade_fa_fp32_stage1(const cascade_paged_attn_t *p, float *out, float *lse, void *workspace,
                           size_t workspace_bytes, cascade_stream_t stream);

/* Stage-2 per-request suffix decode: same problem description, output in the
 * query dtype and a compact fp32 LSE. Replaces the closed CANN
 * npu_fused_infer_attention_score_v2 call of the cascade consumer
 * (ascend-kernel/README.md:180-199; (o2, l2) = (bf16 [B,H,1,D], fp32 [B,H,1])).
 * out: [num_tokens, num_heads, head_dim] in p->dtype; lse: fp32 [num_tokens*num_heads].
 * kv length 0 is allowed in both q_seqlen modes: out = 0, lse = -inf. */
CASCADE_API size_t cascade_suffix_decode_workspace_size(const cascade_paged_attn_t *p);
CASCADE_API int cascade_suffix_decode(const cascade_paged_attn_t *p, void *out, float *lse, void *workspace,
                          size_t workspace_bytes, cascade_stream_t stream);

/* One whole cascade decode step (stage-1 over the shared prefixes, the
 * per-request suffixes, and the merge) with a single final combine: both
 * attention kernels write split partials into the workspace and one kernel
 * merges all partials of each (token, head) row in LSE space and writes
 * `out` ([num_tokens, num_heads, 128] in out_dtype) and, if lse_out is not
 * NULL, the merged natural-log LSE ([num_tokens*num_heads] fp32).
 * Equivalent to cascade_fa_fp32_stage1 + cascade_suffix_decode +
 * cascade_lse_merge (the consumer's chain, ascend-kernel/README.md:158-201)
 * without the intermediate outputs; the suffix partial is not rounded to the
 * query dtype before the merge. `prefix` and `suffix` describe the same
 * query tensor (same num_tokens / num_heads / dtype); zero-length prefixes or
 * suffixes are allowed. The workspace size depends on the shapes alone; when a
 * long stage-1 runs beside the suffix decode (stage-1 split into two launches
 * around it) it covers that schedule's extra partial planes, so it can exceed
 * the two standalone workspace sizes summed: size it with
 * cascade_decode_step_workspace_size. */
CASCADE_API size_t cascade_decode_step_workspace_size(const cascade_paged_attn_t *prefix,
                                                      const cascade_paged_attn_t *suffix);
CASCADE_API int cascade_decode_step(const cascade_paged_attn_t *prefix, const cascade_paged_attn_t *suffix, void *out,
                                    int32_t out_dtype, float *lse_out, void *workspace, size_t workspace_bytes,
                                    cascade_stream_t stream);

/* Row-wise LSE-space merge of two attention partials.
 * Replaces ascend_kernel::lse_merge
 *   (ascend-kernel/csrc/ops/lse_merge/op_host/lse_merge.cpp:32-70,
 *    schema ascend-kernel/csrc/register.cpp:24).
 * o1: [rows, dim] BF16 / FP16 / FP32; o2: [rows, dim] BF16 / FP16 / FP32;
 * lse1/lse2: fp32 with row strides stride1/stride2 (value = element 0 of the row);
 * out: [rows, dim] in out_dtype. m = max(l1,l2); w = exp(l-m);
 * out = (o1 w1 + o2 w2) / (w1 + w2) in fp32; a side whose lse is -inf gets
 * weight 0 (both -inf -> 0). */
CASCADE_API int cascade_lse_merge(const void *o1, int32_t o1_dtype, const void *o2, int32_t o2_dtype, const float *lse1,
                      int64_t stride1, const float *lse2, int64_t stride2, void *out, int32_t out_dtype,
                      int64_t rows, int64_t dim, cascade_stream_t stream);

/* Gate/up GEMM with the f3 epilogue modes.
 * Replaces ascend_kernel::f3_gateup_epilogue
 *   (ascend-kernel/csrc/ops/f3_floor/op_host/f3_floor.cpp:59-125,
 *    schema ascend-kernel/csrc/register.cpp:30-31).
 * a: bf16 [M, K] (row stride K); b: bf16 [2I, K] (gate rows [0,I), up rows [I,2I));
 * ws: bf16 [M, 2I] C workspace (may be NULL for mode 1); d: bf16 [M, I] with row stride d_stride.
 * mode 1: d = silu(a b_gate^T) * (a b_up^T), fp32 epilogue, RNE to bf16, ws untouched.
 * mode 2: ws = a b^T (bf16), d untouched.
 * mode 0: ws = a b^T and d = gate half of ws; mode 4: ws = a b^T and d = up half.
 * mode 3: d = gate half of the existing ws (no GEMM); mode 5: same, gate half only read;
 * mode 7: read gate+up halves of ws, write nothing; mode 8: write d (zeros), read nothing. */
CASCADE_API int cascade_f3_gateup_epilogue(const void *a, const void *b, void *ws, void *d, int64_t d_stride, int64_t M,
                               int64_t K, int64_t I, int32_t mode, cascade_stream_t stream);

/* Residual add + RMSNorm statistics, three modes over contiguous (M, K) rows.
 * Replaces ascend_kernel::add_rms_norm_stats
 *   (ascend-kernel/csrc/ops/add_rms_norm_stats/op_host/add_rms_norm_stats.cpp:59-150,
 *    schema ascend-kernel/csrc/register.cpp:27-28).
 * x1, x2, x_out, y: [M, K] in `dtype` (CASCADE_BF16 / CASCADE_FP16), row stride K,
 * 16-byte aligned; gamma, beta: [K] in `dtype` (beta may be NULL);
 * rstd: fp32 [ceil(M/8)*8], rows >= M are written as 0.
 *   mode 0: x_out = round(x1 + x2), rstd = 1/sqrt(mean(x_out^2) + eps)
 *           (x2 and x_out required; gamma, beta, y unused)
 *   mode 1: rstd from x1, y = round(round(x1 * rstd) * gamma + beta)
 *           (gamma and y required; x2 and x_out unused)
 *   mode 2: rstd from round(x1 + x2) only (x2 required).
 * Limits (as the reference): 0 < K <= 5120, K % 16 == 0, M > 0, eps > 0. */
CASCADE_API int cascade_add_rms_norm_stats(const void *x1, const void *x2, const void *gamma, const void *beta,
                                           void *x_out, float *rstd, void *y, int64_t M, int64_t K, int32_t dtype,
                                           int32_t mode, float eps, cascade_stream_t stream);

/* Suffix decode that allocates nothing (no counterpart in the reference).
 * For callers that cannot allocate device memory when they run the step: a
 * host binding the C ABI without a device allocator, or a serving loop whose
 * memory is fixed before it starts. Same inputs, outputs and results as
 * cascade_suffix_decode, but the split-KV partials go to a scratch array
 * built into the library: 16 MiB, reserved on every GPU that loads the
 * library until the process exits. Limits: q_seqlen_value must be > 0, and a
 * call whose cascade_suffix_decode_workspace_size() exceeds 16 MiB is
 * rejected with CASCADE_ERR_UNSUPPORTED before anything runs. The first call
 * on each device looks up the array's device address (cudaGetSymbolAddress
 * with that device current); make that first call before any stream capture.
 * All calls share the one array and nothing in it needs clearing (each call
 * writes every partial it reads), but calls that overlap on the GPU (other
 * streams, other host threads) race on it: serialise them. */
CASCADE_API int cascade_suffix_decode_noalloc(const cascade_paged_attn_t *p, void *out, float *lse,
                                              cascade_stream_t stream);

/* Read-only HBM streaming probe, the read roof of the memory-bound kernels
 * (the role of the reference's bandwidth probe op, ascend-kernel/csrc/register.cpp:32-33;
 * interface of its own). Reads `bytes` of device memory at `src` (256-byte
 * aligned) once and folds them into `sink` (device uint32, at least 1184
 * words; its contents are meaningless). mode 0: plain 16-byte loads, 8 in
 * flight per thread, 4 x 148 CTAs of 512 threads; mode 1: 32 KB bulk copies
 * into a 4-stage shared-memory ring, one CTA per SM; mode 2: the decode
 * kernel's paged pattern without its math -- rows of `row_bytes` (a multiple
 * of 256: kv heads x 256 bytes), one kv head's 256-byte slice of 64-row tiles
 * per 2-D TMA stage, 512-row items, two CTAs per SM; mode 3: mode 2 with the
 * items in kv-head-major order (no two CTAs read the same rows at once).
 * Time it with events. */
CASCADE_API int cascade_probe_hbm_read(const void *src, size_t bytes, int32_t mode, int64_t row_bytes, uint32_t *sink,
                                       size_t sink_words, cascade_stream_t stream);

/* Last error message of this thread ("" if none). */
CASCADE_API const char *cascade_last_error(void);

/* Reads and clears the device error word. Bits: 1 = a kernel's bounded wait
 * gave up; 2 = a block id outside the pool was read as a zero page; 4 = a
 * stage-1 piece fell outside its planned partial planes and was skipped (its
 * rows are garbage; the planner's bound rules this out). Synchronises the
 * current device. */
CASCADE_API int cascade_device_error(uint32_t *word);

/* Library version (major*10000 + minor*100 + patch). */
CASCADE_API int cascade_version(void);

/* Host-only planner used by the entry points (exposed for tests and callers
 * that size grids): which kernel serves a paged-attention call and how it is
 * split. No CUDA calls. Returns 0 or CASCADE_ERR_*; the fields are:
 *   kernel: 0 = decode path (<= 16 query rows per request and kv head),
 *           1 = tcgen05 tile path (more rows),
 *           2 = planned decode path (decode rows, uniform q length, at least
 *               2048 (request, kv head) pairs and more than one 512-token
 *               split: a device-built list of the non-empty (request, split)
 *               items, two persistent CTAs per SM);
 *   rows_per_group: max query rows per (request, kv head) = q_len * H/KVH;
 *   split_tokens: kv tokens per split (a multiple of the kernel's KV tile);
 *   num_splits: splits per request; workspace_bytes: as the *_workspace_size
 *   functions report. max_q_seqlen: the host-known maximum q length
 *   (== q_seqlen_value on the uniform path). */
typedef struct cascade_attn_plan {
  int32_t kernel;
  int32_t rows_per_group;
  int64_t split_tokens;
  int64_t num_splits;
  size_t workspace_bytes;
} cascade_attn_plan_t;

CASCADE_API int cascade_plan_paged_attn(const cascade_paged_attn_t *p, int64_t max_q_seqlen, int32_t suffix_mode,
                            cascade_attn_plan_t *plan);

#ifdef __cplusplus
}
#endif

#endif /* CASCADE_B200_H */
