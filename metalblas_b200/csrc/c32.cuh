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
// pairs, dense per batch).  Grid-stride over batch * K * N elements.
__global__ void __launch_bounds__(256) c32_build_b_kernel(const C32Prep p, int64_t ld) {
  const int64_t total = p.batch * p.rows * p.cols;
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < total; i += (int64_t)gridDim.x * blockDim.x) {
    const int64_t n = i % p.cols;
    const int64_t k = (i / p.cols) % p.rows;
    const int64_t b = i / (p.cols * p.rows);
    const __half2 v = p.src[b * p.bs + k * p.rs + n * p.cs];
    const __half re = __low2half(v);
    const __half im = p.conj_b ? __hneg(__high2half(v)) : __high2half(v);
    const __half s_re = p.conj_a ? __hneg(re) : re;
    const __half s_im = p.conj_a ? im : __hneg(im);
    __half2 *out = p.dst + b * (2 * p.rows) * ld;
    out[(2 * k) * ld + n] = __halves2half2(re, im);
    out[(2 * k + 1) * ld + n] = __halves2half2(s_im, s_re);
  }
}

}  // namespace mb
