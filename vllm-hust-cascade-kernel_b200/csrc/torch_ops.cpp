// torch op registration: the reference's schemas in namespace `npu`
// (ascend-kernel/csrc/register.cpp:22-36) served for CUDA tensors, plus
// extended-domain siblings. Every op validates like the reference op host
// (same checks, same "<op>: ..." messages), allocates its outputs with the
// caching allocator on the input's device, and calls the C ABI on the current
// CUDA stream. There is no CPU kernel: a CPU tensor fails dispatch.
#include <ATen/ATen.h>
#include <c10/cuda/CUDAGuard.h>
#include <c10/cuda/CUDAStream.h>
#include <torch/library.h>

#include <tuple>

#include "../../include/cascade_b200.h"

namespace cascade_torch {
namespace {

void check_rc(int rc) { TORCH_CHECK(rc == CASCADE_OK, cascade_last_error()); }

int32_t dtype_code(at::ScalarType t) {
  switch (t) {
    case at::kBFloat16: return CASCADE_BF16;
    case at::kHalf: return CASCADE_FP16;
    case at::kFloat: return CASCADE_FP32;
    default: return -1;
  }
}

cascade_stream_t current_stream(const at::Tensor& t) {
  return reinterpret_cast<cascade_stream_t>(c10::cuda::getCurrentCUDAStream(t.get_device()).stream());
}

// Shared argument handling of the paged-attention ops. `strict` = the
// reference's fa_fp32_stage1 domain (bf16, blockSize 128).
cascade_paged_attn_t paged_desc(const char* op, bool strict, const at::Tensor& query, const at::Tensor& key,
                                const at::Tensor& value, const at::Tensor& block_table,
                                const at::Tensor& actual_q_seqlens, const at::Tensor& actual_kv_seqlens,
                                int64_t q_seqlen_value) {
  // op_host/fa_fp32_stage1.cpp:184-208, same order and texts
  TORCH_CHECK(query.is_contiguous() && key.is_contiguous() && value.is_contiguous() &&
                  block_table.is_contiguous() && actual_q_seqlens.is_contiguous() &&
                  actual_kv_seqlens.is_contiguous(),
              op, ": all inputs must be contiguous");
  if (strict) {
    TORCH_CHECK(query.scalar_type() == at::kBFloat16, op, ": query must be bf16");
    TORCH_CHECK(key.scalar_type() == at::kBFloat16 && value.scalar_type() == at::kBFloat16, op,
                ": key/value must be bf16");
  } else {
    TORCH_CHECK(query.scalar_type() == at::kBFloat16 || query.scalar_type() == at::kHalf, op,
                ": query must be bf16 or fp16");
    TORCH_CHECK(key.scalar_type() == query.scalar_type() && value.scalar_type() == query.scalar_type(), op,
                ": key/value must have the query dtype");
  }
  TORCH_CHECK(block_table.scalar_type() == at::kInt, op, ": block_table must be int32");
  TORCH_CHECK(actual_q_seqlens.scalar_type() == at::kLong && actual_kv_seqlens.scalar_type() == at::kLong, op,
              ": seqlens must be int64");
  TORCH_CHECK(query.dim() == 3, op, ": query must be (T, H, D)");
  TORCH_CHECK(key.dim() == 4 && value.dim() == 4, op, ": key/value must be (numBlocks, blockSize, KVH, D)");
  TORCH_CHECK(key.sizes() == value.sizes(), op, ": key/value shapes must match");
  TORCH_CHECK(q_seqlen_value >= 0, op, ": q_seqlen_value must be >= 0 (0 = read seqlens from device)");
  TORCH_CHECK(block_table.dim() == 2, op, ": block_table must be (B, cols)");
  const int64_t batch = actual_q_seqlens.numel();
  TORCH_CHECK(actual_kv_seqlens.numel() == batch, op, ": seqlen tensors must have batch entries");
  TORCH_CHECK(query.size(2) == 128, op, ": only head dim 128 is supported (L1TileShape::K constraint)");
  if (strict) TORCH_CHECK(key.size(1) == 128, op, ": only paged blockSize 128 is supported");
  TORCH_CHECK(key.size(2) > 0 && query.size(1) % key.size(2) == 0, op, ": numHeads must be a multiple of kvHeads");
  TORCH_CHECK(query.is_cuda() && key.is_cuda() && value.is_cuda() && block_table.is_cuda() &&
                  actual_q_seqlens.is_cuda() && actual_kv_seqlens.is_cuda(),
              op, ": all inputs must be CUDA tensors");
  const auto dev = query.get_device();
  TORCH_CHECK(key.get_device() == dev && value.get_device() == dev && block_table.get_device() == dev &&
                  actual_q_seqlens.get_device() == dev && actual_kv_seqlens.get_device() == dev,
              op, ": all inputs must be on one device");
  TORCH_CHECK(block_table.size(0) >= batch || batch == 0, op, ": block_table must have a row per request");

  cascade_paged_attn_t d{};
  d.query = query.data_ptr();
  d.key = key.data_ptr();
  d.value = value.data_ptr();
  d.block_table = block_table.data_ptr<int32_t>();
  d.actual_q_seqlens = actual_q_seqlens.data_ptr<int64_t>();
  d.actual_kv_seqlens = actual_kv_seqlens.data_ptr<int64_t>();
  d.num_tokens = query.size(0);
  d.num_heads = query.size(1);
  d.head_dim = query.size(2);
  d.num_blocks = key.size(0);
  d.block_size = key.size(1);
  d.kv_heads = key.size(2);
  d.batch = batch;
  d.block_cols = block_table.size(1);
  d.q_seqlen_value = q_seqlen_value;
  d.dtype = dtype_code(query.scalar_type());
  d.flags = 0;
  return d;
}

std::tuple<at::Tensor, at::Tensor> prefix_impl(const char* op, bool strict, const at::Tensor& query,
                                               const at::Tensor& key, const at::Tensor& value,
                                               const at::Tensor& block_table, const at::Tensor& actual_q_seqlens,
                                               const at::Tensor& actual_kv_seqlens, int64_t q_seqlen_value) {
  cascade_paged_attn_t d = paged_desc(op, strict, query, key, value, block_table, actual_q_seqlens,
                                      actual_kv_seqlens, q_seqlen_value);
  const c10::cuda::CUDAGuard guard(query.device());
  const int64_t T = d.num_tokens, H = d.num_heads, D = d.head_dim;
  if (d.batch == 0 || T == 0) {
    return {at::empty({T, H, D}, query.options().dtype(at::kFloat)), at::empty({0}, query.options().dtype(at::kFloat))};
  }
  auto out = at::empty({T, H, D}, query.options().dtype(at::kFloat));
  auto lse = at::empty({T * H * 8}, query.options().dtype(at::kFloat));
  const size_t ws_bytes = cascade_fa_fp32_stage1_workspace_size(&d);
  at::Tensor ws;
  if (ws_bytes) ws = at::empty({static_cast<int64_t>(ws_bytes)}, query.options().dtype(at::kByte));
  check_rc(cascade_fa_fp32_stage1(&d, out.data_ptr<float>(), lse.data_ptr<float>(),
                                  ws_bytes ? ws.data_ptr() : nullptr, ws_bytes, current_stream(query)));
  return {out, lse};
}

// torch.ops.npu.fa_fp32_stage1 -- reference domain (ops.h:26-38).
std::tuple<at::Tensor, at::Tensor> fa_fp32_stage1(const at::Tensor& query, const at::Tensor& key,
                                                  const at::Tensor& value, const at::Tensor& block_table,
                                                  const at::Tensor& actual_q_seqlens,
                                                  const at::Tensor& actual_kv_seqlens, int64_t q_seqlen_value) {
  return prefix_impl("fa_fp32_stage1", true, query, key, value, block_table, actual_q_seqlens, actual_kv_seqlens,
                     q_seqlen_value);
}

// torch.ops.npu.cascade_prefix_attention -- same contract, extended domain:
// fp16 or bf16, blockSize in {16,...,512}, kv length 0 (-> out 0, lse -inf)
// on the uniform-q path.
std::tuple<at::Tensor, at::Tensor> cascade_prefix_attention(const at::Tensor& query, const at::Tensor& key,
                                                            const at::Tensor& value, const at::Tensor& block_table,
                                                            const at::Tensor& actual_q_seqlens,
                                                            const at::Tensor& actual_kv_seqlens,
                                                            int64_t q_seqlen_value) {
  return prefix_impl("cascade_prefix_attention", false, query, key, value, block_table, actual_q_seqlens,
                     actual_kv_seqlens, q_seqlen_value);
}

// torch.ops.npu.cascade_suffix_decode -- the stage-2 suffix attention the
// reference's consumer obtains from CANN FIA v2 (README.md:180-199):
// returns (out in the query dtype [T,H,D], compact fp32 lse [T*H]).
std::tuple<at::Tensor, at::Tensor> cascade_suffix_decode(const at::Tensor& query, const at::Tensor& key,
                                                         const at::Tensor& value, const at::Tensor& block_table,
                                                         const at::Tensor& actual_q_seqlens,
                                                         const at::Tensor& actual_kv_seqlens, int64_t q_seqlen_value) {
  const char* op = "cascade_suffix_decode";
  cascade_paged_attn_t d = paged_desc(op, false, query, key, value, block_table, actual_q_seqlens,
                                      actual_kv_seqlens, q_seqlen_value);
  const c10::cuda::CUDAGuard guard(query.device());
  const int64_t T = d.num_tokens, H = d.num_heads, D = d.head_dim;
  auto out = at::empty({T, H, D}, query.options());
  auto lse = at::empty({T * H}, query.options().dtype(at::kFloat));
  if (d.batch == 0 || T == 0) return {out, lse};
  const size_t ws_bytes = cascade_suffix_decode_workspace_size(&d);
  at::Tensor ws;
  if (ws_bytes) ws = at::empty({static_cast<int64_t>(ws_bytes)}, query.options().dtype(at::kByte));
  check_rc(cascade_suffix_decode(&d, out.data_ptr(), lse.data_ptr<float>(), ws_bytes ? ws.data_ptr() : nullptr,
                                 ws_bytes, current_stream(query)));
  return {out, lse};
}

// torch.ops.npu.cascade_decode_step -- the whole cascade step with one final
// combine (C ABI cascade_decode_step). Returns the merged output [T,H,D] in
// the dtype selected by out_code (1 bf16, 2 fp32, 3 fp16).
at::Tensor cascade_decode_step(const at::Tensor& query, const at::Tensor& key, const at::Tensor& value,
                               const at::Tensor& prefix_block_table, const at::Tensor& prefix_q_seqlens,
                               const at::Tensor& prefix_kv_seqlens, const at::Tensor& suffix_block_table,
                               const at::Tensor& suffix_q_seqlens, const at::Tensor& suffix_kv_seqlens,
                               int64_t prefix_q_seqlen_value, int64_t out_code) {
  const char* op = "cascade_decode_step";
  TORCH_CHECK(out_code >= 1 && out_code <= 3, op, ": out_code must be 1 (bf16), 2 (fp32) or 3 (fp16)");
  cascade_paged_attn_t a = paged_desc(op, false, query, key, value, prefix_block_table, prefix_q_seqlens,
                                      prefix_kv_seqlens, prefix_q_seqlen_value);
  cascade_paged_attn_t b = paged_desc(op, false, query, key, value, suffix_block_table, suffix_q_seqlens,
                                      suffix_kv_seqlens, 1);
  const c10::cuda::CUDAGuard guard(query.device());
  const at::ScalarType out_type = out_code == 1 ? at::kBFloat16 : out_code == 2 ? at::kFloat : at::kHalf;
  auto out = at::empty(query.sizes(), query.options().dtype(out_type));
  if (query.numel() == 0) return out;
  const size_t ws_bytes = cascade_decode_step_workspace_size(&a, &b);
  at::Tensor ws;
  if (ws_bytes) ws = at::empty({static_cast<int64_t>(ws_bytes)}, query.options().dtype(at::kByte));
  check_rc(cascade_decode_step(&a, &b, out.data_ptr(), dtype_code(out_type), nullptr,
                               ws_bytes ? ws.data_ptr() : nullptr, ws_bytes, current_stream(query)));
  return out;
}

at::Tensor merge_impl(const char* op, bool strict, const at::Tensor& o1, const at::Tensor& o2, const at::Tensor& lse1,
                      const at::Tensor& lse2, int64_t out_code) {
  // op_host/lse_merge.cpp:35-60, same order and texts
  TORCH_CHECK(o1.is_contiguous() && o2.is_contiguous() && lse1.is_contiguous() && lse2.is_contiguous(), op,
              ": all inputs must be contiguous");
  if (strict) {
    TORCH_CHECK(o1.scalar_type() == at::kBFloat16 || o1.scalar_type() == at::kFloat, op,
                ": o1 must be bf16 or fp32");
    TORCH_CHECK(o2.scalar_type() == at::kBFloat16, op, ": o2 must be bf16");
  } else {
    TORCH_CHECK(dtype_code(o1.scalar_type()) >= 0, op, ": o1 must be bf16, fp16 or fp32");
    TORCH_CHECK(dtype_code(o2.scalar_type()) >= 0, op, ": o2 must be bf16, fp16 or fp32");
  }
  TORCH_CHECK(lse1.scalar_type() == at::kFloat && lse2.scalar_type() == at::kFloat, op,
              ": lse1/lse2 must be fp32");
  if (strict) {
    TORCH_CHECK(out_code >= 0 && out_code <= 2, op, ": out_code must be 0 (follow o1), 1 (bf16) or 2 (fp32)");
  } else {
    TORCH_CHECK(out_code >= 0 && out_code <= 3, op,
                ": out_code must be 0 (follow o1), 1 (bf16), 2 (fp32) or 3 (fp16)");
  }
  const at::ScalarType out_type = out_code == 1   ? at::kBFloat16
                                  : out_code == 2 ? at::kFloat
                                  : out_code == 3 ? at::kHalf
                                                  : o1.scalar_type();
  TORCH_CHECK(o1.dim() >= 1 && o1.size(-1) % 16 == 0, op,
              ": head dim must be a multiple of 16 (MTE 32B alignment)");
  TORCH_CHECK(o2.numel() == o1.numel(), op, ": o1 and o2 must have the same number of elements");
  TORCH_CHECK(o1.is_cuda() && o2.is_cuda() && lse1.is_cuda() && lse2.is_cuda(), op,
              ": all inputs must be CUDA tensors");
  const c10::cuda::CUDAGuard guard(o1.device());
  auto out = at::empty(o1.sizes(), o1.options().dtype(out_type));
  const int64_t dim = o1.size(-1);
  const int64_t rows = o1.numel() / dim;
  if (rows == 0) return out;
  TORCH_CHECK(lse1.numel() % rows == 0 && lse2.numel() % rows == 0, op,
              ": lse numel must be a multiple of the row count (row-stride packing)");
  const int64_t s1 = lse1.numel() / rows, s2 = lse2.numel() / rows;
  TORCH_CHECK(s1 >= 1 && s1 <= 64 && s2 >= 1 && s2 <= 64, op, ": lse row stride must be in [1, 64]");
  check_rc(cascade_lse_merge(o1.data_ptr(), dtype_code(o1.scalar_type()), o2.data_ptr(),
                             dtype_code(o2.scalar_type()), lse1.data_ptr<float>(), s1, lse2.data_ptr<float>(), s2,
                             out.data_ptr(), dtype_code(out_type), rows, dim, current_stream(o1)));
  return out;
}

at::Tensor lse_merge(const at::Tensor& o1, const at::Tensor& o2, const at::Tensor& lse1, const at::Tensor& lse2,
                     int64_t out_code) {
  return merge_impl("lse_merge", true, o1, o2, lse1, lse2, out_code);
}

at::Tensor cascade_lse_merge(const at::Tensor& o1, const at::Tensor& o2, const at::Tensor& lse1,
                             const at::Tensor& lse2, int64_t out_code) {
  return merge_impl("cascade_lse_merge", false, o1, o2, lse1, lse2, out_code);
}

// torch.ops.npu.f3_gateup_epilogue (f3_floor/op_host/f3_floor.cpp:59-125).
std::tuple<at::Tensor, at::Tensor> f3_gateup_epilogue(const at::Tensor& a, const at::Tensor& b,
                                                      const c10::optional<at::Tensor>& workspace,
                                                      const c10::optional<at::Tensor>& out_d, int64_t mode) {
  const char* op = "f3_gateup_epilogue";
  TORCH_CHECK(a.dim() == 2 && a.is_contiguous() && a.scalar_type() == at::kBFloat16, op,
              ": a must be a contiguous bf16 [M, K]");
  TORCH_CHECK(b.dim() == 2 && b.is_contiguous() && b.scalar_type() == at::kBFloat16, op,
              ": b must be a contiguous bf16 [2I, K]");
  TORCH_CHECK((mode >= 0 && mode <= 5) || mode == 7 || mode == 8, op, ": mode must be 0..5, 7 or 8");
  const int64_t M = a.size(0), K = a.size(1);
  TORCH_CHECK(b.size(0) % 2 == 0, op, ": b.size(0) must be even (gate | up)");
  const int64_t I = b.size(0) / 2;
  TORCH_CHECK(b.size(1) == K, op, ": a.size(1) must equal b.size(1)");
  TORCH_CHECK(M > 0 && K > 0, op, ": empty input");
  TORCH_CHECK(K % 16 == 0, op, ": K must be a multiple of 16");
  TORCH_CHECK(M % 16 == 0, op, ": M must be a multiple of 16");
  TORCH_CHECK(I % 128 == 0, op, ": I must be a multiple of the N tile");
  TORCH_CHECK(K >= 64, op, ": K must be >= 64 (L0 K tile)");
  TORCH_CHECK(a.is_cuda() && b.is_cuda() && a.get_device() == b.get_device(), op,
              ": a and b must be CUDA tensors on one device");
  const c10::cuda::CUDAGuard guard(a.device());
  at::Tensor ws;
  if (workspace.has_value() && workspace->defined()) {
    ws = *workspace;
    TORCH_CHECK(ws.is_contiguous() && ws.scalar_type() == at::kBFloat16 && ws.dim() == 2 && ws.size(0) == M &&
                    ws.size(1) == 2 * I,
                op, ": workspace must be contiguous bf16 [M, 2I]");
  } else {
    ws = at::empty({M, 2 * I}, a.options());
  }
  at::Tensor d;
  int64_t d_stride = I;
  if (out_d.has_value() && out_d->defined()) {
    d = *out_d;
    TORCH_CHECK(d.scalar_type() == at::kBFloat16 && d.dim() == 2 && d.size(0) == M && d.size(1) == I, op,
                ": d must be bf16 [M, I]");
    TORCH_CHECK(d.stride(1) == 1, op, ": d rows must be contiguous");
    d_stride = d.stride(0);
  } else {
    d = at::empty({M, I}, a.options());
  }
  check_rc(cascade_f3_gateup_epilogue(a.data_ptr(), b.data_ptr(), ws.data_ptr(), d.data_ptr(), d_stride, M, K, I,
                                      static_cast<int32_t>(mode), current_stream(a)));
  return {d, ws};
}

// torch.ops.npu.cascade_gateup_swiglu(x [M,K], w [2I,K]) -> silu(x w_gate^T) * (x w_up^T)
// as bf16 [M, I]: the fused mode-1 GEMM for any M >= 1 (no C workspace).
at::Tensor cascade_gateup_swiglu(const at::Tensor& x, const at::Tensor& w) {
  const char* op = "cascade_gateup_swiglu";
  TORCH_CHECK(x.dim() == 2 && x.is_contiguous() && x.scalar_type() == at::kBFloat16, op,
              ": x must be a contiguous bf16 [M, K]");
  TORCH_CHECK(w.dim() == 2 && w.is_contiguous() && w.scalar_type() == at::kBFloat16, op,
              ": w must be a contiguous bf16 [2I, K]");
  TORCH_CHECK(w.size(0) % 2 == 0 && w.size(1) == x.size(1), op, ": w must be [2I, K] with K = x.size(1)");
  TORCH_CHECK(x.is_cuda() && w.is_cuda() && x.get_device() == w.get_device(), op,
              ": x and w must be CUDA tensors on one device");
  const c10::cuda::CUDAGuard guard(x.device());
  const int64_t M = x.size(0), K = x.size(1), I = w.size(0) / 2;
  auto d = at::empty({M, I}, x.options());
  if (M == 0) return d;
  check_rc(cascade_f3_gateup_epilogue(x.data_ptr(), w.data_ptr(), nullptr, d.data_ptr(), I, M, K, I, 1,
                                      current_stream(x)));
  return d;
}

// torch.ops.npu.add_rms_norm_stats: checks, their order and texts and the
// output allocation of op_host/add_rms_norm_stats.cpp:59-104 -- unused
// outputs come back as 0-element tensors and rstd is (ceil(M/8)*8, 1) fp32
// with zeroed padding rows.
std::tuple<at::Tensor, at::Tensor, at::Tensor> add_rms_norm_stats(const at::Tensor& x1, const at::Tensor& x2,
                                                                  const c10::optional<at::Tensor>& gamma,
                                                                  const c10::optional<at::Tensor>& beta, double eps,
                                                                  int64_t mode) {
  TORCH_CHECK(x1.dim() == 2, "add_rms_norm_stats: x1 must be 2D (M, K)");
  TORCH_CHECK(x1.is_contiguous(), "add_rms_norm_stats: x1 must be contiguous");
  TORCH_CHECK(mode >= 0 && mode <= 2, "add_rms_norm_stats: mode must be 0, 1 or 2");
  TORCH_CHECK(eps > 0.0, "add_rms_norm_stats: eps must be > 0");
  const bool is_bf16 = x1.scalar_type() == at::kBFloat16;
  const bool is_fp16 = x1.scalar_type() == at::kHalf;
  TORCH_CHECK(is_bf16 || is_fp16, "add_rms_norm_stats: x1 must be bf16 or fp16");
  if (mode != 1) {
    TORCH_CHECK(x2.defined() && x2.is_contiguous() && x2.sizes() == x1.sizes() &&
                    x2.scalar_type() == x1.scalar_type(),
                "add_rms_norm_stats: x2 must be contiguous, same shape and dtype as x1");
  }
  const int64_t M = x1.size(0), K = x1.size(1);
  TORCH_CHECK(M > 0, "add_rms_norm_stats: empty row count");
  TORCH_CHECK(K > 0 && K <= 5120, "add_rms_norm_stats: K must be in (0, ", 5120, "] (one row resident in UB)");
  TORCH_CHECK(K % 16 == 0, "add_rms_norm_stats: K must be a multiple of 16 (32B row copies)");
  const bool has_beta = mode == 1 && beta.has_value() && beta->defined() && beta->numel() > 0;
  if (mode == 1) {
    TORCH_CHECK(gamma.has_value() && gamma->defined() && gamma->is_contiguous() && gamma->numel() == K &&
                    gamma->scalar_type() == x1.scalar_type(),
                "add_rms_norm_stats: mode 1 needs a contiguous gamma of K elements, same dtype");
    if (has_beta) {
      TORCH_CHECK(beta->is_contiguous() && beta->numel() == K && beta->scalar_type() == x1.scalar_type(),
                  "add_rms_norm_stats: beta must be contiguous, K elements, same dtype");
    }
  }
  TORCH_CHECK(x1.is_cuda(), "add_rms_norm_stats: x1 must be a CUDA tensor");
  const int dev = x1.get_device();
  TORCH_CHECK(mode == 1 || (x2.is_cuda() && x2.get_device() == dev), "add_rms_norm_stats: x2 must be on x1's device");
  TORCH_CHECK(mode != 1 || (gamma->is_cuda() && gamma->get_device() == dev &&
                            (!has_beta || (beta->is_cuda() && beta->get_device() == dev))),
              "add_rms_norm_stats: gamma/beta must be on x1's device");
  const c10::cuda::CUDAGuard guard(x1.device());
  const int64_t m_padded = (M + 7) / 8 * 8;
  auto x_out = mode == 0 ? at::empty_like(x1) : at::empty({0}, x1.options());
  auto rstd = at::empty({m_padded, 1}, x1.options().dtype(at::kFloat));
  auto y = mode == 1 ? at::empty_like(x1) : at::empty({0}, x1.options());
  check_rc(cascade_add_rms_norm_stats(x1.data_ptr(), mode == 1 ? nullptr : x2.data_ptr(),
                                      mode == 1 ? gamma->data_ptr() : nullptr, has_beta ? beta->data_ptr() : nullptr,
                                      mode == 0 ? x_out.data_ptr() : nullptr, rstd.data_ptr<float>(),
                                      mode == 1 ? y.data_ptr() : nullptr, M, K, dtype_code(x1.scalar_type()),
                                      static_cast<int32_t>(mode), static_cast<float>(eps), current_stream(x1)));
  return {x_out, rstd, y};
}

}  // namespace
}  // namespace cascade_torch

TORCH_LIBRARY_FRAGMENT(npu, m) {
  m.def(
      "add_rms_norm_stats(Tensor x1, Tensor x2, Tensor? gamma, Tensor? beta, float eps, "
      "int mode) -> (Tensor, Tensor, Tensor)");
  m.def("lse_merge(Tensor o1, Tensor o2, Tensor lse1, Tensor lse2, int out_code=0) -> Tensor");
  m.def(
      "fa_fp32_stage1(Tensor query, Tensor key, Tensor value, Tensor block_table, "
      "Tensor actual_q_seqlens, Tensor actual_kv_seqlens, int q_seqlen_value=0) -> (Tensor, Tensor)");
  m.def(
      "f3_gateup_epilogue(Tensor a, Tensor b, Tensor? workspace, Tensor? out_d, int mode) "
      "-> (Tensor, Tensor)");
  m.def(
      "cascade_prefix_attention(Tensor query, Tensor key, Tensor value, Tensor block_table, "
      "Tensor actual_q_seqlens, Tensor actual_kv_seqlens, int q_seqlen_value=0) -> (Tensor, Tensor)");
  m.def(
      "cascade_suffix_decode(Tensor query, Tensor key, Tensor value, Tensor block_table, "
      "Tensor actual_q_seqlens, Tensor actual_kv_seqlens, int q_seqlen_value=0) -> (Tensor, Tensor)");
  m.def("cascade_lse_merge(Tensor o1, Tensor o2, Tensor lse1, Tensor lse2, int out_code=0) -> Tensor");
  m.def("cascade_gateup_swiglu(Tensor x, Tensor w) -> Tensor");
  m.def(
      "cascade_decode_step(Tensor query, Tensor key, Tensor value, Tensor prefix_block_table, "
      "Tensor prefix_q_seqlens, Tensor prefix_kv_seqlens, Tensor suffix_block_table, Tensor suffix_q_seqlens, "
      "Tensor suffix_kv_seqlens, int prefix_q_seqlen_value=0, int out_code=1) -> Tensor");
}

TORCH_LIBRARY_IMPL(npu, CUDA, m) {
  m.impl("lse_merge", TORCH_FN(cascade_torch::lse_merge));
  m.impl("fa_fp32_stage1", TORCH_FN(cascade_torch::fa_fp32_stage1));
  m.impl("f3_gateup_epilogue", TORCH_FN(cascade_torch::f3_gateup_epilogue));
  m.impl("cascade_prefix_attention", TORCH_FN(cascade_torch::cascade_prefix_attention));
  m.impl("cascade_suffix_decode", TORCH_FN(cascade_torch::cascade_suffix_decode));
  m.impl("cascade_lse_merge", TORCH_FN(cascade_torch::cascade_lse_merge));
  m.impl("cascade_gateup_swiglu", TORCH_FN(cascade_torch::cascade_gateup_swiglu));
  m.impl("cascade_decode_step", TORCH_FN(cascade_torch::cascade_decode_step));
  m.impl("add_rms_norm_stats", TORCH_FN(cascade_torch::add_rms_norm_stats));
}
