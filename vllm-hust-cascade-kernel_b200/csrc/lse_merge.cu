// Row-wise LSE-space merge of two attention partials (cascade combine step).
//
// Semantics of the reference kernel (ascend-kernel/csrc/ops/lse_merge/
// op_kernel/kernel_lse_merge.cpp:16-20, :237-290): per row r
//   m = max(l1, l2); w1 = exp(l1 - m); w2 = exp(l2 - m);
//   out = (o1*w1 + o2*w2) * (1 / (w1 + w2))       all in fp32,
// a 16-bit output is rounded to nearest even. LSE rows are read with a row
// stride (1 = compact, 8 = the stage-1 padded rows).
// Extension: a side with lse = -inf has weight 0 and its O does not enter
// the result (a NaN there cannot leak).
//
// HBM-bound: each thread moves one 16-byte chunk of o2 (8 x 16-bit) and the
// matching 8 elements of o1 (16 or 32 bytes); the two LSE loads per row hit
// L1/L2 for the 16 threads sharing the row. Grid = ceil(rows*dim/8 / 256).
#include "kernels.h"
#include "ptx.cuh"

namespace cascade {
namespace {

template <int kDt>
__device__ __forceinline__ void load8(const void* base, size_t idx, float (&v)[8]) {
  if constexpr (kDt == 2) {
    const float4* p = reinterpret_cast<const float4*>(static_cast<const float*>(base) + idx);
    float4 a = __ldg(p), b = __ldg(p + 1);
    v[0] = a.x; v[1] = a.y; v[2] = a.z; v[3] = a.w;
    v[4] = b.x; v[5] = b.y; v[6] = b.z; v[7] = b.w;
  } else {
    uint4 u = __ldg(reinterpret_cast<const uint4*>(static_cast<const uint16_t*>(base) + idx));
    const uint32_t w[4] = {u.x, u.y, u.z, u.w};
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      if constexpr (kDt == 0) {
        v[2 * i] = __uint_as_float(w[i] << 16);
        v[2 * i + 1] = __uint_as_float(w[i] & 0xFFFF0000u);
      } else {
        __half2 h = *reinterpret_cast<const __half2*>(&w[i]);
        float2 f = __half22float2(h);
        v[2 * i] = f.x;
        v[2 * i + 1] = f.y;
      }
    }
  }
}

template <int kDt>
__device__ __forceinline__ void store8(void* base, size_t idx, const float (&v)[8]) {
  if constexpr (kDt == 2) {
    float4* p = reinterpret_cast<float4*>(static_cast<float*>(base) + idx);
    p[0] = make_float4(v[0], v[1], v[2], v[3]);
    p[1] = make_float4(v[4], v[5], v[6], v[7]);
  } else {
    uint32_t w[4];
#pragma unroll
    for (int i = 0; i < 4; ++i) w[i] = pack2<kDt == 1>(v[2 * i], v[2 * i + 1]);
    *reinterpret_cast<uint4*>(static_cast<uint16_t*>(base) + idx) = make_uint4(w[0], w[1], w[2], w[3]);
  }
}

template <int kO1, int kO2, int kOut>
__global__ void __launch_bounds__(256) lse_merge_kernel(const LseMergeLaunch p) {
  const int chunks_per_row = p.dim >> 3;
  const size_t gid = static_cast<size_t>(blockIdx.x) * blockDim.x + threadIdx.x;
  const size_t total = static_cast<size_t>(p.rows) * chunks_per_row;
  if (gid >= total) return;
  const size_t row = gid / chunks_per_row;
  const size_t idx = gid * 8;  // == row*dim + chunk*8
  // issue every load up front: the O loads do not wait on the LSE values
  const float l1 = __ldg(p.lse1 + row * p.stride1);
  const float l2 = __ldg(p.lse2 + row * p.stride2);
  float a[8], b[8];
  load8<kO1>(p.o1, idx, a);
  load8<kO2>(p.o2, idx, b);
  const float m = fmaxf(l1, l2);
  float w1, w2;
  if (m == -INFINITY) {
    w1 = 0.f;
    w2 = 0.f;
  } else {
    w1 = (l1 == -INFINITY) ? 0.f : __expf(l1 - m);
    w2 = (l2 == -INFINITY) ? 0.f : __expf(l2 - m);
  }
  const float s = w1 + w2;
  const float inv = s > 0.f ? 1.f / s : 0.f;
  // a zero-weight side contributes exactly 0 (its O, possibly NaN, is not used)
  float o[8];
#pragma unroll
  for (int i = 0; i < 8; ++i) {
    const float x = w1 != 0.f ? a[i] * w1 : 0.f;
    const float y = w2 != 0.f ? b[i] * w2 : 0.f;
    o[i] = (x + y) * inv;
  }
  store8<kOut>(p.out, idx, o);
}

template <int kO1, int kO2>
cudaError_t dispatch_out(const LseMergeLaunch& p, dim3 grid, cudaStream_t st) {
  switch (p.out_dtype) {
    case 0: lse_merge_kernel<kO1, kO2, 0><<<grid, 256, 0, st>>>(p); break;
    case 1: lse_merge_kernel<kO1, kO2, 1><<<grid, 256, 0, st>>>(p); break;
    default: lse_merge_kernel<kO1, kO2, 2><<<grid, 256, 0, st>>>(p); break;
  }
  return cudaGetLastError();
}

template <int kO1>
cudaError_t dispatch_o2(const LseMergeLaunch& p, dim3 grid, cudaStream_t st) {
  switch (p.o2_dtype) {
    case 0: return dispatch_out<kO1, 0>(p, grid, st);
    case 1: return dispatch_out<kO1, 1>(p, grid, st);
    default: return dispatch_out<kO1, 2>(p, grid, st);
  }
}

}  // namespace

cudaError_t launch_lse_merge(const LseMergeLaunch& p, cudaStream_t stream) {
  const size_t total = static_cast<size_t>(p.rows) * (p.dim >> 3);
  if (total == 0) return cudaSuccess;
  dim3 grid(static_cast<unsigned>((total + 255) / 256));
  switch (p.o1_dtype) {
    case 0: return dispatch_o2<0>(p, grid, stream);
    case 1: return dispatch_o2<1>(p, grid, stream);
    default: return dispatch_o2<2>(p, grid, stream);
  }
}

}  // namespace cascade
