// Operand packing for the tensor-core path: a strided (batched) matrix copied
// into dense row-major rows of pitch `ld` elements, so that TMA can load it.
// Used for views TMA cannot address in place (unaligned base or pitch, no unit
// stride); the reference copies such views with .contiguous()
// (metalblas/dispatch.py:33-35).
#pragma once
#include "mb_common.cuh"

namespace mb {

struct PackArgs {
  const void *src;
  void *dst;
  int64_t rows, cols;   // logical extents
  int64_t rs, cs, bs;   // source strides in elements (bs: batch)
  int64_t batch, ld;    // batches copied; destination row pitch in elements
};

// Grid-stride over batch * rows * cols elements, columns fastest, so a warp
// reads consecutive columns of one row (coalesced when cs == 1) and writes them
// consecutively.  U is the element's storage type (same-size unsigned).
template <class U>
__global__ void __launch_bounds__(256) pack_matrix_kernel(const PackArgs a) {
  const U *src = static_cast<const U *>(a.src);
  U *dst = static_cast<U *>(a.dst);
  const int64_t per_batch = a.rows * a.cols;
  const int64_t total = a.batch * per_batch;
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < total; i += (int64_t)gridDim.x * blockDim.x) {
    const int64_t b = i / per_batch;
    const int64_t rem = i - b * per_batch;
    const int64_t r = rem / a.cols;
    const int64_t c = rem - r * a.cols;
    dst[(b * a.rows + r) * a.ld + c] = src[b * a.bs + r * a.rs + c * a.cs];
  }
}

// Row-contiguous sources (cs == 1, the offset / odd-pitch views): each thread
// moves one 16-byte group of a destination row, reading its elements one by
// one (the source may be unaligned) and writing one aligned 16-byte store.  The
// destination pitch `ld` is a multiple of 16 bytes; the group past the end of a
// row spills into its padding, which the tensor maps never read.
template <class U>
__global__ void __launch_bounds__(256) pack_rows16_kernel(const PackArgs a) {
  constexpr int G = 16 / (int)sizeof(U);
  const U *src = static_cast<const U *>(a.src);
  U *dst = static_cast<U *>(a.dst);
  const int64_t groups = (a.cols + G - 1) / G;
  const int64_t per_batch = a.rows * groups;
  const int64_t total = a.batch * per_batch;
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < total; i += (int64_t)gridDim.x * blockDim.x) {
    const int64_t b = i / per_batch;
    const int64_t rem = i - b * per_batch;
    const int64_t r = rem / groups;
    const int64_t c0 = (rem - r * groups) * G;
    const U *s = src + b * a.bs + r * a.rs + c0;
    union { uint4 q; U e[G]; } v;
#pragma unroll
    for (int j = 0; j < G; ++j) v.e[j] = (c0 + j < a.cols) ? s[j] : U(0);
    *reinterpret_cast<uint4 *>(dst + (b * a.rows + r) * a.ld + c0) = v.q;
  }
}

}  // namespace mb
