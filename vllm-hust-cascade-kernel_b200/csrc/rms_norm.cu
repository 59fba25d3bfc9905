// Residual add + RMSNorm statistics (the norm stage of the reference's
// AddRmsNormBias -> GEMM fusion line), three modes over contiguous (M, K)
// rows of bf16 / fp16:
//   mode 0: x_out = round(x1 + x2), rstd = rms_stats(x_out)
//   mode 1: rstd = rms_stats(x1), y = round(round(x1 * rstd) * gamma + beta)
//   mode 2: rstd = rms_stats(round(x1 + x2)), nothing else written
// rms_stats(v) = 1 / sqrt(mean_k(v^2) + eps), returned in fp32, where v is the
// ROUNDED residual (the reference golden squares x_out after its rounding to
// the data type: ascend-kernel/csrc/ops/add_rms_norm_stats/test/
// add_rms_norm_stats_ref.py:130-156, design.md section 1).
// Precision: the residual add is exact in fp32 and rounded once (RNE) to the
// data type. The sum of squares and 1/sqrt are carried in fp64, the golden's
// own precision (one conversion and one fp64 fma per element). x * rstd must
// be the fp32 rounding of the fp64 product (the golden rounds it to fp32 and
// then to the data type): rstd is split into two fp32 parts rh + rl and
//   ph = x * rh,  v = ph + fma(x, rl, fma(x, rh, -ph))
// (the inner fma is the exact error of ph) gives that rounding in fp32
// arithmetic, off only within ~2^-46 of an fp32 rounding boundary. mid * gamma
// is exact in fp32 and + beta is one fma rounding, so y reproduces the fp64
// golden bit for bit except where the fp64 sums differ in order by ~1e-16.
// rstd is returned as the fp32 rounding of the fp64 value.
//
// HBM-bound: one CTA of 128 threads per row, the row held in registers (at
// most 5 16-byte chunks per input and thread, K <= 5120), so every input byte
// is read once and every output byte written once; the row's sum of squares
// is reduced with warp shuffles and 4 shared-memory slots. rstd is written
// for M rows and its padding rows [M, ceil(M/8)*8) are zeroed, the
// reference's output layout (op_host/add_rms_norm_stats.cpp:18-25).
#include "kernels.h"
#include "ptx.cuh"

namespace cascade {
namespace {

constexpr int kNormThreads = 128;
constexpr int kNormMaxChunks = 5;  // 5 x 8 elements x 128 threads = 5120 = the K limit

template <bool kFp16>
__device__ __forceinline__ float to_f32(uint16_t v) {
  if constexpr (kFp16) {
    return __half2float(__ushort_as_half(v));
  } else {
    return __bfloat162float(__ushort_as_bfloat16(v));
  }
}

template <bool kFp16>
__device__ __forceinline__ uint16_t from_f32(float v) {
  if constexpr (kFp16) {
    return __half_as_ushort(__float2half_rn(v));
  } else {
    return __bfloat16_as_ushort(__float2bfloat16_rn(v));
  }
}

// two fp32 values -> one 32-bit word of two RNE-rounded 16-bit values (low =
// first), one packed conversion instruction
template <bool kFp16>
__device__ __forceinline__ uint32_t pack2_rn(float lo, float hi) {
  if constexpr (kFp16) {
    const __half2 h = __floats2half2_rn(lo, hi);
    return *reinterpret_cast<const uint32_t*>(&h);
  } else {
    const __nv_bfloat162 h = __floats2bfloat162_rn(lo, hi);
    return *reinterpret_cast<const uint32_t*>(&h);
  }
}

// element e (0..7) of a 16-byte chunk of 16-bit values
__device__ __forceinline__ uint16_t elem(const uint32_t (&w)[4], int e) {
  return static_cast<uint16_t>(w[e >> 1] >> ((e & 1) * 16));
}

template <bool kFp16>
__global__ void __launch_bounds__(kNormThreads) add_rms_norm_stats_kernel(const __grid_constant__ RmsNormLaunch p) {
  const int row = blockIdx.x;
  const int tid = threadIdx.x;
  const int nchunks = p.K / 8;
  const size_t base = static_cast<size_t>(row) * p.K;
  const uint4* x1 = reinterpret_cast<const uint4*>(static_cast<const uint16_t*>(p.x1) + base);
  const uint4* x2 = p.mode == 1 ? nullptr : reinterpret_cast<const uint4*>(static_cast<const uint16_t*>(p.x2) + base);

  // load the row (all loads issued before any use)
  uint32_t a[kNormMaxChunks][4], b[kNormMaxChunks][4];
#pragma unroll
  for (int i = 0; i < kNormMaxChunks; ++i) {
    const int c = tid + i * kNormThreads;
    uint4 va = make_uint4(0u, 0u, 0u, 0u), vb = make_uint4(0u, 0u, 0u, 0u);
    if (c < nchunks) {
      va = __ldcs(x1 + c);
      if (x2) vb = __ldcs(x2 + c);
    }
    a[i][0] = va.x; a[i][1] = va.y; a[i][2] = va.z; a[i][3] = va.w;
    b[i][0] = vb.x; b[i][1] = vb.y; b[i][2] = vb.z; b[i][3] = vb.w;
  }

  // residual (rounded to the data type) and this thread's sum of squares
  double ss = 0.0;
#pragma unroll
  for (int i = 0; i < kNormMaxChunks; ++i) {
    if (tid + i * kNormThreads >= nchunks) continue;
#pragma unroll
    for (int e = 0; e < 8; e += 2) {
      if (x2) {
        a[i][e >> 1] = pack2_rn<kFp16>(to_f32<kFp16>(elem(a[i], e)) + to_f32<kFp16>(elem(b[i], e)),
                                       to_f32<kFp16>(elem(a[i], e + 1)) + to_f32<kFp16>(elem(b[i], e + 1)));
      }
      const double f0 = to_f32<kFp16>(elem(a[i], e)), f1 = to_f32<kFp16>(elem(a[i], e + 1));
      ss = fma(f0, f0, ss);
      ss = fma(f1, f1, ss);
    }
  }

  // row reduction: warp shuffles, then the 4 warps through shared memory
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, o);
  __shared__ double part[kNormThreads / 32];
  if ((tid & 31) == 0) part[tid >> 5] = ss;
  __syncthreads();
  const double total = (part[0] + part[1]) + (part[2] + part[3]);
  const double rstd = 1.0 / sqrt(total / static_cast<double>(p.K) + static_cast<double>(p.eps));

  if (tid == 0) {
    p.rstd[row] = static_cast<float>(rstd);
    if (row == p.M - 1) {
      for (int r = p.M; r < p.m_padded; ++r) p.rstd[r] = 0.f;
    }
  }

  if (p.mode == 0) {
    uint4* xo = reinterpret_cast<uint4*>(static_cast<uint16_t*>(p.x_out) + base);
#pragma unroll
    for (int i = 0; i < kNormMaxChunks; ++i) {
      const int c = tid + i * kNormThreads;
      if (c < nchunks) __stcs(xo + c, make_uint4(a[i][0], a[i][1], a[i][2], a[i][3]));
    }
  } else if (p.mode == 1) {
    const float rh = static_cast<float>(rstd);
    const float rl = static_cast<float>(rstd - static_cast<double>(rh));
    const uint4* gm = static_cast<const uint4*>(p.gamma);
    const uint4* bt = static_cast<const uint4*>(p.beta);
    uint4* yo = reinterpret_cast<uint4*>(static_cast<uint16_t*>(p.y) + base);
#pragma unroll
    for (int i = 0; i < kNormMaxChunks; ++i) {
      const int c = tid + i * kNormThreads;
      if (c >= nchunks) continue;
      const uint4 gv = __ldg(gm + c);
      const uint4 bv = bt ? __ldg(bt + c) : make_uint4(0u, 0u, 0u, 0u);
      const uint32_t g4[4] = {gv.x, gv.y, gv.z, gv.w}, b4[4] = {bv.x, bv.y, bv.z, bv.w};
      uint32_t out[4];
#pragma unroll
      for (int e = 0; e < 8; e += 2) {
        float xr[2];
#pragma unroll
        for (int k = 0; k < 2; ++k) {
          const float x = to_f32<kFp16>(elem(a[i], e + k));
          const float ph = x * rh;
          xr[k] = ph + fmaf(x, rl, fmaf(x, rh, -ph));
        }
        const uint32_t mid2[1] = {pack2_rn<kFp16>(xr[0], xr[1])};
        float v[2];
#pragma unroll
        for (int k = 0; k < 2; ++k) {
          const float mid = to_f32<kFp16>(static_cast<uint16_t>(mid2[0] >> (16 * k)));
          const float gmm = to_f32<kFp16>(elem(g4, e + k));
          v[k] = bt ? fmaf(mid, gmm, to_f32<kFp16>(elem(b4, e + k))) : mid * gmm;
        }
        out[e >> 1] = pack2_rn<kFp16>(v[0], v[1]);
      }
      __stcs(yo + c, make_uint4(out[0], out[1], out[2], out[3]));
    }
  }
}

}  // namespace

cudaError_t launch_add_rms_norm_stats(const RmsNormLaunch& p, bool fp16, cudaStream_t stream) {
  if (p.M <= 0) return cudaSuccess;
  auto kern = fp16 ? add_rms_norm_stats_kernel<true> : add_rms_norm_stats_kernel<false>;
  kern<<<static_cast<unsigned>(p.M), kNormThreads, 0, stream>>>(p);
  return cudaGetLastError();
}

}  // namespace cascade
