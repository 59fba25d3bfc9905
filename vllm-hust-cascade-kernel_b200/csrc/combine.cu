// Final combine of a cascade decode step: for every (token, head) row, merge
// the split-KV partials of stage-1 (shared prefix) and of the suffix in LSE
// space and write the output once. This replaces the reference chain's three
// passes (stage-1 output, suffix output, lse_merge: README.md:174-200) with
// one: m = max_i lse_i; w_i = exp(lse_i - m); out = sum_i w_i O_i / sum_i w_i
// (the lse_merge formula, kernel_lse_merge.cpp:16-20, over all partials).
// Partials with lse = -inf (empty splits, zero-length suffixes) get weight 0.
//
// One warp per row: lane i reads lse_i, the weights come from warp
// reductions, each lane then owns 4 of the 128 dims and issues the partial
// loads (16 B each) for every non-empty split.
#include "kernels.h"
#include "ptx.cuh"

namespace cascade {
namespace {

constexpr int kWarpsPerBlock = 8;

__global__ void __launch_bounds__(kWarpsPerBlock * 32) cascade_combine_kernel(const CascadeCombineLaunch p) {
  const int64_t row = static_cast<int64_t>(blockIdx.x) * kWarpsPerBlock + (threadIdx.x >> 5);
  const int lane = threadIdx.x & 31;
  if (p.pdl) pdl_wait();  // partials come from the kernels before this one
  if (row >= p.rows) return;
  const int n = p.n1 + p.n2;
  // Every load of the row is issued before any result is needed: the lse of
  // partial `lane` / `lane+32`, and this lane's 4 dims of the first 16
  // partials. A partial with lse = -inf may hold anything: it is selected
  // out, never multiplied.
  auto part_ptr = [&](int i) -> const float4* {
    const float* base = i < p.n1 ? p.o1 + (static_cast<int64_t>(i) * p.rows + row) * kHeadDim
                                 : p.o2 + (static_cast<int64_t>(i - p.n1) * p.rows + row) * kHeadDim;
    return reinterpret_cast<const float4*>(base) + lane;
  };
  float la = -INFINITY, lb = -INFINITY;
  if (lane < n) la = lane < p.n1 ? p.l1[lane * p.rows + row] : p.l2[(lane - p.n1) * p.rows + row];
  if (lane + 32 < n) {
    const int i = lane + 32;
    lb = i < p.n1 ? p.l1[i * p.rows + row] : p.l2[(i - p.n1) * p.rows + row];
  }
  constexpr int kPre = 16;
  float4 v[kPre];
#pragma unroll
  for (int k = 0; k < kPre; ++k) v[k] = k < n ? __ldg(part_ptr(k)) : make_float4(0.f, 0.f, 0.f, 0.f);
  float m = fmaxf(la, lb);
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, o));
  const float wa = (la == -INFINITY) ? 0.f : __expf(la - m);
  const float wb = (lb == -INFINITY) ? 0.f : __expf(lb - m);
  float wsum = wa + wb;
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) wsum += __shfl_xor_sync(0xffffffffu, wsum, o);
  float4 acc = make_float4(0.f, 0.f, 0.f, 0.f);
  auto add = [&](float w, const float4& x) {
    if (w != 0.f) {
      acc.x += w * x.x;
      acc.y += w * x.y;
      acc.z += w * x.z;
      acc.w += w * x.w;
    }
  };
#pragma unroll
  for (int k = 0; k < kPre; ++k) add(__shfl_sync(0xffffffffu, wa, k), v[k]);
  for (int i = kPre; i < n; ++i) {  // rare: more than 16 partials per row
    const float w = __shfl_sync(0xffffffffu, i < 32 ? wa : wb, i & 31);
    if (w != 0.f) add(w, __ldg(part_ptr(i)));
  }
  const float inv = wsum > 0.f ? 1.f / wsum : 0.f;
  const int64_t o = row * kHeadDim + lane * 4;
  if (p.out_dtype == 2) {
    *reinterpret_cast<float4*>(static_cast<float*>(p.out) + o) =
        make_float4(acc.x * inv, acc.y * inv, acc.z * inv, acc.w * inv);
  } else {
    const bool h = p.out_dtype == 1;
    const uint32_t a = h ? pack2<true>(acc.x * inv, acc.y * inv) : pack2<false>(acc.x * inv, acc.y * inv);
    const uint32_t b = h ? pack2<true>(acc.z * inv, acc.w * inv) : pack2<false>(acc.z * inv, acc.w * inv);
    *reinterpret_cast<uint2*>(static_cast<uint16_t*>(p.out) + o) = make_uint2(a, b);
  }
  if (p.lse_out != nullptr && lane == 0) p.lse_out[row] = wsum > 0.f ? m + __logf(wsum) : -INFINITY;
}

}  // namespace

cudaError_t launch_cascade_combine(const CascadeCombineLaunch& p, cudaStream_t stream) {
  if (p.rows == 0) return cudaSuccess;
  const unsigned blocks = static_cast<unsigned>((p.rows + kWarpsPerBlock - 1) / kWarpsPerBlock);
  return launch_maybe_pdl(cascade_combine_kernel, dim3(blocks), dim3(kWarpsPerBlock * 32), 0, stream, p.pdl != 0, p);
}

}  // namespace cascade
