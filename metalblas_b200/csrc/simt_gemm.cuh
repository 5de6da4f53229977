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
// Layout: 256 threads, a BM x BN tile per CTA, a TM x TN micro-tile per thread
// made of two TM/2 x TN/2 quadrant pairs (rows ty*TM/2 and BM/2 + ty*TM/2, and
// likewise for columns) so that a warp's shared-memory reads of a K row are
// contiguous 16-byte vectors.  BK-deep K slices are double-buffered in shared
// memory with a register prefetch of the next slice; every thread stages runs
// of 4 elements along each operand's contiguous dimension, with one aligned
// vector load per run when the layout allows it.  Operands are converted to
// the accumulator type when they are staged, so the inner loop is pure FFMA /
// IMAD.
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
  int a_vec, b_vec;  // 4-element runs along the contiguous dimension are aligned vectors
  EpiScalars epi;
  const int *gate;   // non-null: the kernel runs only if *gate != 0 (set on the device)
};

// Four consecutive elements from an address aligned to 4 * sizeof(T).
template <class T>
__device__ __forceinline__ void load_run4(const T *p, T (&v)[4]) {
  constexpr int B = 4 * (int)sizeof(T);
  if constexpr (B == 32) {
    union { uint4 q[2]; T t[4]; } u;
    u.q[0] = __ldg(reinterpret_cast<const uint4 *>(p));
    u.q[1] = __ldg(reinterpret_cast<const uint4 *>(p) + 1);
#pragma unroll
    for (int i = 0; i < 4; ++i) v[i] = u.t[i];
  } else if constexpr (B == 16) {
    union { uint4 q; T t[4]; } u;
    u.q = __ldg(reinterpret_cast<const uint4 *>(p));
#pragma unroll
    for (int i = 0; i < 4; ++i) v[i] = u.t[i];
  } else if constexpr (B == 8) {
    union { uint2 q; T t[4]; } u;
    u.q = __ldg(reinterpret_cast<const uint2 *>(p));
#pragma unroll
    for (int i = 0; i < 4; ++i) v[i] = u.t[i];
  } else {
    static_assert(B == 4, "element size");
    union { unsigned q; T t[4]; } u;
    u.q = __ldg(reinterpret_cast<const unsigned *>(p));
#pragma unroll
    for (int i = 0; i < 4; ++i) v[i] = u.t[i];
  }
}

// Four accumulators to a 16-byte aligned shared-memory address as vectors.
template <class Acc>
__device__ __forceinline__ void sts_run4(Acc *dst, const Acc (&v)[4]) {
  struct alignas(16) V4 { Acc a[4]; };
  V4 t;
#pragma unroll
  for (int i = 0; i < 4; ++i) t.a[i] = v[i];
  *reinterpret_cast<V4 *>(dst) = t;
}

template <class T, int BM, int BN, int BK, int TM, int TN>
__global__ void __launch_bounds__(256, 2) simt_gemm_kernel(const SimtParams p) {
  using E = Elem<T>;
  using Acc = typename E::acc;
  constexpr int NT = 256;
  constexpr int TX = BN / TN, TY = BM / TM;
  static_assert(TX * TY == NT, "micro-tile grid must cover 256 threads");
  constexpr int HM = TM / 2, HN = TN / 2;
  static_assert(HM * (int)sizeof(Acc) % 16 == 0 && HN * (int)sizeof(Acc) % 16 == 0, "16-byte fragment reads");
  // runs of 4 elements per thread and operand per K slice
  constexpr int RA = BM * BK / (4 * NT), RB = BK * BN / (4 * NT);
  static_assert(RA * 4 * NT == BM * BK && RB * 4 * NT == BK * BN && RA >= 1 && RB >= 1, "run tiling");
  constexpr int PAD = 16 / (int)sizeof(Acc);  // keeps rows 16-byte aligned

  __shared__ __align__(16) Acc As[2][BK][BM + PAD];
  __shared__ __align__(16) Acc Bs[2][BK][BN + PAD];

  if (p.gate != nullptr && *reinterpret_cast<const volatile int *>(p.gate) == 0) return;  // uniform per CTA
  const int tid = threadIdx.x;
  // Each warp covers an 8 (x) by 4 (y) block of micro-tiles, so one K row's
  // fragment reads touch 4 distinct 16-byte A vectors and 8 B vectors: one
  // shared-memory wavefront per read instead of two for a 16 x 2 layout.
  static_assert(TX % 8 == 0 && TY % 4 == 0 && (TX / 8) * (TY / 4) == NT / 32, "8 x 4 warp blocks");
  const int lane = tid & 31, wid = tid >> 5;
  const int tx = (wid % (TX / 8)) * 8 + (lane & 7), ty = (wid / (TX / 8)) * 4 + (lane >> 3);
  const int64_t m0 = (int64_t)blockIdx.y * BM, n0 = (int64_t)blockIdx.x * BN;
  // A: k contiguous (row-major) -> runs along k; otherwise runs along m.
  const bool a_kfast = p.a_cs == 1 || (p.a_rs != 1 && (p.a_cs < 0 ? -p.a_cs : p.a_cs) <= (p.a_rs < 0 ? -p.a_rs : p.a_rs));
  // B: n contiguous (row-major) -> runs along n; otherwise runs along k.
  const bool b_nfast = p.b_cs == 1 || (p.b_rs != 1 && (p.b_cs < 0 ? -p.b_cs : p.b_cs) <= (p.b_rs < 0 ? -p.b_rs : p.b_rs));
  const bool a_vec = p.a_vec != 0, b_vec = p.b_vec != 0;
  // this thread's run r: (row or column, first k) inside the tile; recomputed
  // where used (a few integer ops) rather than held in registers
  auto a_m = [&](int r) { const int q = tid + r * NT; return a_kfast ? q % BM : (q % (BM / 4)) * 4; };
  auto a_k = [&](int r) { const int q = tid + r * NT; return a_kfast ? (q / BM) * 4 : q / (BM / 4); };
  auto b_n = [&](int r) { const int q = tid + r * NT; return b_nfast ? (q % (BN / 4)) * 4 : q % BN; };
  auto b_k = [&](int r) { const int q = tid + r * NT; return b_nfast ? q / (BN / 4) : (q / BN) * 4; };
  const int64_t a_step = a_kfast ? p.a_cs : p.a_rs;  // stride along a run
  const int64_t b_step = b_nfast ? p.b_cs : p.b_rs;
  const int64_t num_kt = (p.K + BK - 1) / BK;

  for (int64_t bz = blockIdx.z; bz < p.batch; bz += gridDim.z) {
    const T *A0 = (const T *)p.A + bz * p.sA;
    const T *B0 = (const T *)p.B + bz * p.sB;

    Acc acc[TM][TN];
#pragma unroll
    for (int i = 0; i < TM; ++i)
#pragma unroll
      for (int j = 0; j < TN; ++j) acc[i][j] = E::zero();

    Acc ra[RA][4], rb[RB][4];
    auto load_tile = [&](int64_t kt) {
      const int64_t k0 = kt * BK;
#pragma unroll
      for (int r = 0; r < RA; ++r) {
        const int64_t gm = m0 + a_m(r), gk = k0 + a_k(r);
        const T *ap = A0 + gm * p.a_rs + gk * p.a_cs;
        const bool full = a_kfast ? (gm < p.M && gk + 3 < p.K) : (gm + 3 < p.M && gk < p.K);
        if (a_vec && full) {
          T v[4];
          load_run4<T>(ap, v);
#pragma unroll
          for (int j = 0; j < 4; ++j) ra[r][j] = E::load(v[j], p.conj_a);
        } else {
#pragma unroll
          for (int j = 0; j < 4; ++j) {
            const bool in = a_kfast ? (gm < p.M && gk + j < p.K) : (gm + j < p.M && gk < p.K);
            ra[r][j] = in ? E::load(ap[j * a_step], p.conj_a) : E::zero();
          }
        }
      }
#pragma unroll
      for (int r = 0; r < RB; ++r) {
        const int64_t gn = n0 + b_n(r), gk = k0 + b_k(r);
        const T *bp = B0 + gk * p.b_rs + gn * p.b_cs;
        const bool full = b_nfast ? (gn + 3 < p.N && gk < p.K) : (gn < p.N && gk + 3 < p.K);
        if (b_vec && full) {
          T v[4];
          load_run4<T>(bp, v);
#pragma unroll
          for (int j = 0; j < 4; ++j) rb[r][j] = E::load(v[j], p.conj_b);
        } else {
#pragma unroll
          for (int j = 0; j < 4; ++j) {
            const bool in = b_nfast ? (gn + j < p.N && gk < p.K) : (gn < p.N && gk + j < p.K);
            rb[r][j] = in ? E::load(bp[j * b_step], p.conj_b) : E::zero();
          }
        }
      }
    };
    auto store_tile = [&](int buf) {
#pragma unroll
      for (int r = 0; r < RA; ++r) {
        if (a_kfast) {
#pragma unroll
          for (int j = 0; j < 4; ++j) As[buf][a_k(r) + j][a_m(r)] = ra[r][j];
        } else {
          sts_run4<Acc>(&As[buf][a_k(r)][a_m(r)], ra[r]);
        }
      }
#pragma unroll
      for (int r = 0; r < RB; ++r) {
        if (b_nfast) {
          sts_run4<Acc>(&Bs[buf][b_k(r)][b_n(r)], rb[r]);
        } else {
#pragma unroll
          for (int j = 0; j < 4; ++j) Bs[buf][b_k(r) + j][b_n(r)] = rb[r][j];
        }
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
        for (int i = 0; i < HM; ++i) {
          av[i] = As[cur][kk][ty * HM + i];
          av[HM + i] = As[cur][kk][BM / 2 + ty * HM + i];
        }
#pragma unroll
        for (int j = 0; j < HN; ++j) {
          bv[j] = Bs[cur][kk][tx * HN + j];
          bv[HN + j] = Bs[cur][kk][BN / 2 + tx * HN + j];
        }
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
      const int64_t gm = m0 + (i < HM ? ty * HM + i : BM / 2 + ty * HM + (i - HM));
      if (gm >= p.M) continue;
#pragma unroll
      for (int j = 0; j < TN; ++j) {
        const int64_t gn = n0 + (j < HN ? tx * HN + j : BN / 2 + tx * HN + (j - HN));
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
