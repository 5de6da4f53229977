// CUDA-core throughput probes: the roofline denominators of the CUDA-core GEMM
// (fp32 / complex64 on FFMA, int16 / int32 on 32-bit IMAD, int64 on 64-bit
// multiply-add).  NVIDIA publishes no B200 figure for these pipes, so the
// library measures them: every thread runs CHAINS independent multiply-add
// chains for `iters` steps, enough independent work per warp to keep the pipe
// busy, on a grid of 4 CTAs of 256 threads per SM.
#pragma once
#include "mb_common.cuh"

namespace mb {

constexpr int kPeakChains = 8;

template <class T>
__device__ __forceinline__ T peak_mad(T a, T b, T c) { return a * b + c; }
template <>
__device__ __forceinline__ float peak_mad<float>(float a, float b, float c) { return fmaf(a, b, c); }

template <class T>
__global__ void __launch_bounds__(256) peak_mad_kernel(T *out, T seed, long long iters) {
  T acc[kPeakChains];
  const T mul = seed + (T)threadIdx.x;  // not a compile-time constant
#pragma unroll
  for (int i = 0; i < kPeakChains; ++i) acc[i] = seed + (T)(i + 1);
  for (long long it = 0; it < iters; ++it) {
#pragma unroll
    for (int u = 0; u < 16; ++u)
#pragma unroll
      for (int i = 0; i < kPeakChains; ++i) acc[i] = peak_mad<T>(acc[i], mul, acc[(i + 1) % kPeakChains]);
  }
  T s = acc[0];
#pragma unroll
  for (int i = 1; i < kPeakChains; ++i) s = s + acc[i];
  // practically never true; keeps the chains live
  if (s == (T)123456789) out[blockIdx.x * blockDim.x + threadIdx.x] = s;
}

}  // namespace mb
