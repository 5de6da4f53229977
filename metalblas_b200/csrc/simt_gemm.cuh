// CUDA-core register-tiled GEMM for every dtype and every stride pattern.
//
// This is the B200 counterpart of three reference kernels that do not use the
// Apple tensor unit: the simdgroup GEMM behind backend="simd"
// (metalblas/shaders/simd_gemm.h:153-300), the integer GEMM
// (metalblas/shaders/int_gemm.h:41-154, accumulate in ACC_T then truncate) and
// the complex four-product path (metalblas/complex_dispatch.py:69-115), which
// here is fused: interleaved complex operands are read once and multiplied as
// complex numbers in fp32.  It serves fp32 and complex64 (FFMA keeps the 1e-5
// tolerance), int16/int32/int64 (IMAD with two's-complement wrap), and any
// operand whose strides the TMA path cannot take (for example the reference's
// "offset" [1:,1:] view with lda=K+1, or a view with no unit stride, which the
// reference copies with .contiguous() in metalblas/dispatch.py:33-35 and which
// we read in place).
//
// Layout: 256 threads, a BM x BN tile per CTA, a TM x TN micro-tile per thread,
// BK-deep K slices double-buffered in shared memory with a register prefetch of
// the next slice.  Operands are converted to the accumulator type when they are
// staged, so the inner loop is pure FFMA / IMAD.
#pragma once
#include "mb_common.cuh"

namespace mb {

struct SimtParams {
  const void *A, *B, *bias;
  void *C;
  int64_t M, N, K, batch;
  int64_t a_rs, a_cs, sA, b_rs, b_cs, sB, c_rs, c_cs, sC;
  int64_t bias_rs, bias_cs, bias_bs;
  int conj_a, conj_b;
  EpiScalars epi;
};

template <class T, int BM, int BN, int BK, int TM, int TN>
__global__ void __launch_bounds__(256) simt_gemm_kernel(const SimtParams p) {
  using E = Elem<T>;
  using Acc = typename E::acc;
  constexpr int NT = 256;
  constexpr int TX = BN / TN, TY = BM / TM;
  static_assert(TX * TY == NT, "micro-tile grid must cover 256 threads");
  constexpr int A_PER = BM * BK / NT, B_PER = BK * BN / NT;
  static_assert(A_PER * NT == BM * BK && B_PER * NT == BK * BN, "tile/thread mismatch");
  constexpr int PAD = (sizeof(Acc) == 4) ? 4 : 2;

  __shared__ Acc As[2][BK][BM + PAD];
  __shared__ Acc Bs[2][BK][BN + PAD];

  const int tid = threadIdx.x;
  const int tx = tid % TX, ty = tid / TX;
  const int64_t m0 = (int64_t)blockIdx.y * BM, n0 = (int64_t)blockIdx.x * BN;
  // Stage the contiguous dimension fastest so global loads coalesce.
  const bool a_kfast = p.a_cs == 1 || (p.a_rs != 1 && (p.a_cs < 0 ? -p.a_cs : p.a_cs) <= (p.a_rs < 0 ? -p.a_rs : p.a_rs));
  const bool b_nfast = p.b_cs == 1 || (p.b_rs != 1 && (p.b_cs < 0 ? -p.b_cs : p.b_cs) <= (p.b_rs < 0 ? -p.b_rs : p.b_rs));
  const int64_t num_kt = (p.K + BK - 1) / BK;

  for (int64_t bz = blockIdx.z; bz < p.batch; bz += gridDim.z) {
    const T *A = (const T *)p.A + bz * p.sA;
    const T *B = (const T *)p.B + bz * p.sB;

    Acc acc[TM][TN];
#pragma unroll
    for (int i = 0; i < TM; ++i)
#pragma unroll
      for (int j = 0; j < TN; ++j) acc[i][j] = E::zero();

    Acc ra[A_PER], rb[B_PER];
    auto load_tile = [&](int64_t kt) {
      const int64_t k0 = kt * BK;
#pragma unroll
      for (int q = 0; q < A_PER; ++q) {
        const int idx = tid + q * NT;
        const int mm = a_kfast ? idx / BK : idx % BM;
        const int kk = a_kfast ? idx % BK : idx / BM;
        const int64_t gm = m0 + mm, gk = k0 + kk;
        ra[q] = (gm < p.M && gk < p.K) ? E::load(A[gm * p.a_rs + gk * p.a_cs], p.conj_a) : E::zero();
      }
#pragma unroll
      for (int q = 0; q < B_PER; ++q) {
        const int idx = tid + q * NT;
        const int nn = b_nfast ? idx % BN : idx / BK;
        const int kk = b_nfast ? idx / BN : idx % BK;
        const int64_t gn = n0 + nn, gk = k0 + kk;
        rb[q] = (gn < p.N && gk < p.K) ? E::load(B[gk * p.b_rs + gn * p.b_cs], p.conj_b) : E::zero();
      }
    };
    auto store_tile = [&](int buf) {
#pragma unroll
      for (int q = 0; q < A_PER; ++q) {
        const int idx = tid + q * NT;
        const int mm = a_kfast ? idx / BK : idx % BM;
        const int kk = a_kfast ? idx % BK : idx / BM;
        As[buf][kk][mm] = ra[q];
      }
#pragma unroll
      for (int q = 0; q < B_PER; ++q) {
        const int idx = tid + q * NT;
        const int nn = b_nfast ? idx % BN : idx / BK;
        const int kk = b_nfast ? idx / BN : idx % BK;
        Bs[buf][kk][nn] = rb[q];
      }
    };

    if (num_kt > 0) {
      load_tile(0);
      store_tile(0);
    }
    __syncthreads();
    for (int64_t kt = 0; kt < num_kt; ++kt) {
      const int cur = (int)(kt & 1);
      if (kt + 1 < num_kt) load_tile(kt + 1);
#pragma unroll
      for (int kk = 0; kk < BK; ++kk) {
        Acc av[TM], bv[TN];
#pragma unroll
        for (int i = 0; i < TM; ++i) av[i] = As[cur][kk][ty * TM + i];
#pragma unroll
        for (int j = 0; j < TN; ++j) bv[j] = Bs[cur][kk][tx * TN + j];
#pragma unroll
        for (int i = 0; i < TM; ++i)
#pragma unroll
          for (int j = 0; j < TN; ++j) E::mad(acc[i][j], av[i], bv[j]);
      }
      if (kt + 1 < num_kt) store_tile(cur ^ 1);
      __syncthreads();
    }

    T *C = (T *)p.C + bz * p.sC;
    const T *bias = (const T *)p.bias + (p.epi.enabled ? bz * p.bias_bs : 0);
#pragma unroll
    for (int i = 0; i < TM; ++i) {
      const int64_t gm = m0 + ty * TM + i;
      if (gm >= p.M) continue;
#pragma unroll
      for (int j = 0; j < TN; ++j) {
        const int64_t gn = n0 + tx * TN + j;
        if (gn >= p.N) continue;
        Acc v = acc[i][j];
        if (p.epi.enabled) v = EpiOps<T>::apply(v, bias + gm * p.bias_rs + gn * p.bias_cs, p.epi);
        C[gm * p.c_rs + gn * p.c_cs] = E::store(v);
      }
    }
    __syncthreads();
  }
}

}  // namespace mb
