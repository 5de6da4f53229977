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
__global__ void __launch_bounds__(256, 2) simt_gemm_kernel(const SimtParams p) {
  using E = Elem<T>;
  using Acc = typename E::acc;
  constexpr int NT = 256;
  constexpr int TX = BN / TN, TY = BM / TM;
  static_assert(TX * TY == NT, "micro-tile grid must cover 256 threads");
  // Staging: every thread moves one run of 4 consecutive elements of A and of B
  // per K slice, along that operand's contiguous dimension.
  static_assert(BM * BK == 4 * NT && BK * BN == 4 * NT, "one 4-element run per thread and operand");
  constexpr int PAD = (sizeof(Acc) == 4) ? 4 : 2;

  __shared__ __align__(16) Acc As[2][BK][BM + PAD];
  __shared__ __align__(16) Acc Bs[2][BK][BN + PAD];

  const int tid = threadIdx.x;
  const int tx = tid % TX, ty = tid / TX;
  const int64_t m0 = (int64_t)blockIdx.y * BM, n0 = (int64_t)blockIdx.x * BN;
  // A: k contiguous (row-major) -> run along k; otherwise run along m.
  const bool a_kfast = p.a_cs == 1 || (p.a_rs != 1 && (p.a_cs < 0 ? -p.a_cs : p.a_cs) <= (p.a_rs < 0 ? -p.a_rs : p.a_rs));
  // B: n contiguous (row-major) -> run along n; otherwise run along k.
  const bool b_nfast = p.b_cs == 1 || (p.b_rs != 1 && (p.b_cs < 0 ? -p.b_cs : p.b_cs) <= (p.b_rs < 0 ? -p.b_rs : p.b_rs));
  // this thread's run: (row or column, first k) inside the tile
  const int a_m = a_kfast ? tid % BM : (tid % (BM / 4)) * 4;
  const int a_k = a_kfast ? (tid / BM) * 4 : tid / (BM / 4);
  const int b_n = b_nfast ? (tid % (BN / 4)) * 4 : tid % BN;
  const int b_k = b_nfast ? tid / (BN / 4) : (tid / BN) * 4;
  const int64_t a_step = a_kfast ? p.a_cs : p.a_rs;   // stride along the run
  const int64_t b_step = b_nfast ? p.b_cs : p.b_rs;
  const int64_t num_kt = (p.K + BK - 1) / BK;

  for (int64_t bz = blockIdx.z; bz < p.batch; bz += gridDim.z) {
    // run bases for k0 = 0
    const T *Ab = (const T *)p.A + bz * p.sA + (m0 + a_m) * p.a_rs + (int64_t)a_k * p.a_cs;
    const T *Bb = (const T *)p.B + bz * p.sB + (int64_t)b_k * p.b_rs + (n0 + b_n) * p.b_cs;
    const int64_t a_kt_step = (int64_t)BK * p.a_cs, b_kt_step = (int64_t)BK * p.b_rs;

    Acc acc[TM][TN];
#pragma unroll
    for (int i = 0; i < TM; ++i)
#pragma unroll
      for (int j = 0; j < TN; ++j) acc[i][j] = E::zero();

    Acc ra[4], rb[4];
    auto load_tile = [&](int64_t kt) {
      const int64_t k0 = kt * BK;
      const T *ap = Ab + kt * a_kt_step;
      const T *bp = Bb + kt * b_kt_step;
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        const int64_t gm = m0 + a_m + (a_kfast ? 0 : j), gk = k0 + a_k + (a_kfast ? j : 0);
        ra[j] = (gm < p.M && gk < p.K) ? E::load(ap[j * a_step], p.conj_a) : E::zero();
      }
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        const int64_t gn = n0 + b_n + (b_nfast ? j : 0), gk = k0 + b_k + (b_nfast ? 0 : j);
        rb[j] = (gn < p.N && gk < p.K) ? E::load(bp[j * b_step], p.conj_b) : E::zero();
      }
    };
    auto store_tile = [&](int buf) {
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        if (a_kfast) As[buf][a_k + j][a_m] = ra[j];
        else As[buf][a_k][a_m + j] = ra[j];
      }
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        if (b_nfast) Bs[buf][b_k][b_n + j] = rb[j];
        else Bs[buf][b_k + j][b_n] = rb[j];
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
