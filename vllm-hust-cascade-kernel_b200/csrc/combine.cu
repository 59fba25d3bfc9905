// Final combine of a cascade decode step: for every (token, head) row, merge
// the split-KV partials of stage-1 (shared prefix) and of the suffix in LSE
// space and write the output once. This replaces the reference chain's three
// passes (stage-1 output, suffix output, lse_merge: README.md:174-200) with
// one: m = max_i lse_i; w_i = exp(lse_i - m); out = sum_i w_i O_i / sum_i w_i
// (the lse_merge formula, kernel_lse_merge.cpp:16-20, over all partials).
// Partials with lse = -inf (empty splits, zero-length suffixes) get weight 0.
//
// One warp per row: lane i reads lse_i, the weights come from warp
// reductions, each lane then owns 4 of the 128 dims. The kernel is
// latency-bound (a round of dependent loads per row), so its form follows
// the step's shape (n = n1 + n2 planes):
//  * dense (kPre = 4, 8 or 16 >= n): every partial is loaded before the
//    weights are known, one round per row. Grids of at most two blocks per
//    SM take the 16-deep form, whose 93 registers keep two blocks per SM and
//    so spread the rows over the most SMs (C2: 2,048 rows, 35.6 us step
//    against 36.4 with the 55-register form, whose blocks land four or more
//    to an SM); larger grids take the smallest depth that holds n, so no
//    register waits for a load never issued and more rows are in flight;
//  * sparse (kPre = 0, n > 8 on larger grids): ragged suffixes make many
//    splits but leave most of a row's partials empty, so the weights come
//    first and only the partials with a non-zero weight are loaded, eight
//    per round (C5 step 297-307 -> 278-284 us; C4, 8 planes on 16,384 rows,
//    372.7 -> 369.1 us).
#include "kernels.h"
#include "ptx.cuh"

namespace cascade {
namespace {

constexpr int kWarpsPerBlock = 8;

template <int kPre>
__global__ void __launch_bounds__(kWarpsPerBlock * 32, kPre == 4 ? 6 : kPre == 16 ? 2 : 4)
    cascade_combine_kernel(const CascadeCombineLaunch p) {
  const int64_t row = static_cast<int64_t>(blockIdx.x) * kWarpsPerBlock + (threadIdx.x >> 5);
  const int lane = threadIdx.x & 31;
  if (p.pdl) pdl_wait();  // partials come from the kernels before this one
  if (row >= p.rows) return;
  const int n = p.n1 + p.n2;
  // The lse of partial `lane` / `lane+32`, and (dense form) this lane's 4
  // dims of every partial, all issued before any result is needed. A partial
  // with lse = -inf may hold anything: it is selected out, never multiplied.
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
  constexpr int kHeld = kPre > 0 ? kPre : 1;
  float4 v[kHeld];
  if constexpr (kPre > 0) {
#pragma unroll
    for (int k = 0; k < kPre; ++k) v[k] = k < n ? __ldg(part_ptr(k)) : make_float4(0.f, 0.f, 0.f, 0.f);
  }
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
  if constexpr (kPre > 0) {
#pragma unroll
    for (int k = 0; k < kPre; ++k) add(__shfl_sync(0xffffffffu, wa, k), v[k]);
  } else {
    // Partials with a non-zero weight, as a warp-uniform bit set over the
    // (at most 64) planes; eight of them loaded per round.
    uint64_t live = static_cast<uint64_t>(__ballot_sync(0xffffffffu, wa != 0.f)) |
                    (static_cast<uint64_t>(__ballot_sync(0xffffffffu, wb != 0.f)) << 32);
    constexpr int kBatch = 8;
    while (live != 0) {
      float4 x[kBatch];
      float w[kBatch];
#pragma unroll
      for (int k = 0; k < kBatch; ++k) {
        w[k] = 0.f;
        x[k] = make_float4(0.f, 0.f, 0.f, 0.f);
        if (live != 0) {
          const int i = __ffsll(static_cast<long long>(live)) - 1;
          live &= live - 1;
          w[k] = __shfl_sync(0xffffffffu, i < 32 ? wa : wb, i & 31);
          x[k] = __ldg(part_ptr(i));
        }
      }
#pragma unroll
      for (int k = 0; k < kBatch; ++k) add(w[k], x[k]);
    }
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
  const int n = p.n1 + p.n2;
  const bool one_wave = blocks <= 2u * kNumSMs;
  auto kern = one_wave && n <= 16 ? cascade_combine_kernel<16>
              : n <= 4            ? cascade_combine_kernel<4>
              : n <= 8            ? cascade_combine_kernel<8>
                                  : cascade_combine_kernel<0>;
  return launch_maybe_pdl(kern, dim3(blocks), dim3(kWarpsPerBlock * 32), 0, stream, p.pdl != 0, p);
}

}  // namespace cascade
