// complex32 on the tensor cores: operand preparation.
//
// The reference computes complex GEMMs as four real products plus split and
// combine passes (metalblas/complex_dispatch.py:69-115,
// shaders/complex_pack.h:9-59).  Here one real fp16 GEMM does it:
//
//   A'[m][2k + c]          = component c of A(m, k)       (interleaved = the
//                                                          storage of A itself)
//   B'[2k][2n], B'[2k][2n+1]     = b_re,        b_im'
//   B'[2k+1][2n], B'[2k+1][2n+1] = -s * b_im',  s * b_re
//   C'[m][2n + c]          = component c of C(m, n)       (the storage of C)
//
// with b_im' = -b_im when B is conjugated and s = -1 when A is conjugated, so
// C' = A' B' is exactly C = op(A) op(B) with fp32 accumulation on the fp16
// tensor cores (kind::f16).  B' is built once per call in the workspace; A' is
// A's own memory when A is row-major, otherwise a packed copy (pack.cuh).
#pragma once
#include "mb_common.cuh"

namespace mb {

struct C32Prep {
  const __half2 *src;
  __half2 *dst;
  int64_t rows, cols;        // complex extents of the source matrix
  int64_t rs, cs, bs;        // source element strides (complex units), batch stride
  int64_t batch;
  int conj_a, conj_b;
};

// B (K x N complex) -> B' (2K x 2N real fp16, row-major, row pitch `ld` half2
// pairs, dense per batch).  Grid (ceil(N / 1024), min(K, 65535), batch): each
// thread takes four consecutive complex elements of one row of B (one 16-byte
// load when B is row-major and aligned) and writes its 2 x 2 blocks as two
// 16-byte stores, one to each of the rows 2k and 2k + 1 of B'.  In a half2
// word (low = re, high = im) the conjugations are sign-bit flips, so the
// result is exact: row 2k holds (re, im'), row 2k + 1 the halves swapped with
// im' (s = 1) or re (s = -1) negated.
__device__ __forceinline__ void c32_pair_words(uint32_t w, int conj_a, int conj_b, uint32_t &r0, uint32_t &r1) {
  if (conj_b) w ^= 0x80000000u;                       // im' = -im
  r0 = w;                                             // (re, im')
  const uint32_t sw = __byte_perm(w, 0, 0x1032);      // (im', re)
  r1 = sw ^ (conj_a ? 0x80000000u : 0x00008000u);     // (-s im', s re)
}

__global__ void __launch_bounds__(256) c32_build_b_kernel(const C32Prep p, int64_t ld) {
  const int64_t b = blockIdx.z;
  const int64_t n0 = ((int64_t)blockIdx.x * blockDim.x + threadIdx.x) * 4;
  if (n0 >= p.cols) return;
  const bool vec = p.cs == 1 && n0 + 4 <= p.cols && (ld & 3) == 0;
  for (int64_t k = blockIdx.y; k < p.rows; k += gridDim.y) {
    const __half2 *src = p.src + b * p.bs + k * p.rs;
    __half2 *out0 = p.dst + (b * 2 * p.rows + 2 * k) * ld;
    __half2 *out1 = out0 + ld;
    if (vec && (reinterpret_cast<uintptr_t>(src + n0) & 15) == 0) {
      const uint4 v = __ldg(reinterpret_cast<const uint4 *>(src + n0));
      uint4 a, c;
      c32_pair_words(v.x, p.conj_a, p.conj_b, a.x, c.x);
      c32_pair_words(v.y, p.conj_a, p.conj_b, a.y, c.y);
      c32_pair_words(v.z, p.conj_a, p.conj_b, a.z, c.z);
      c32_pair_words(v.w, p.conj_a, p.conj_b, a.w, c.w);
      *reinterpret_cast<uint4 *>(out0 + n0) = a;
      *reinterpret_cast<uint4 *>(out1 + n0) = c;
    } else {
      for (int j = 0; j < 4 && n0 + j < p.cols; ++j) {
        const __half2 v = src[(n0 + j) * p.cs];
        uint32_t r0, r1;
        c32_pair_words(*reinterpret_cast<const uint32_t *>(&v), p.conj_a, p.conj_b, r0, r1);
        reinterpret_cast<uint32_t *>(out0)[n0 + j] = r0;
        reinterpret_cast<uint32_t *>(out1)[n0 + j] = r1;
      }
    }
  }
}

}  // namespace mb
