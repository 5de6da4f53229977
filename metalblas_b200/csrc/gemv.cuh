// Bandwidth-bound matrix-vector kernels (the M==1 / N==1 products).
//
// Two orientations cover every unit-stride layout, as in the reference:
//  * gemv_cols: y[r] = sum_k x[k] * W[k*ld + r]   (vector times a matrix whose
//    output index is contiguous) — the B200 form of gemv_t
//    (metalblas/shaders/gemv_t.h:15-99): lanes own 16-byte column vectors, the
//    warps of a CTA split K, partial sums meet in shared memory, and, when the
//    column count alone cannot fill 148 SMs, K is also split across CTAs with
//    fp32 partials in a caller-provided workspace reduced by the last CTA to
//    arrive (an atomic ticket, no waiting).
//  * gemv_rows: y[r] = sum_k W[r*ld + k] * x[k]   (rows contiguous along K) —
//    the B200 form of gemv_nt (metalblas/shaders/gemv_nt.h:16-101): one warp
//    per row, 16-byte loads, a warp-shuffle reduction.
// Orientation is chosen by the host like the reference's _dispatch_gemv
// (metalblas/dispatch.py:49-70).  Loads of W use ld.global.nc with L1
// no-allocate (W is streamed once); x is small and re-read from L1/L2.
#pragma once
#include "mb_common.cuh"

namespace mb {

struct GemvParams {
  const void *W, *X, *bias;
  void *Y;
  int64_t R, K;          // outputs, reduction length
  int64_t w_ld;          // cols: W(k,r) = W[k*w_ld + r];  rows: W(r,k) = W[r*w_ld + k]
  int64_t x_s;           // x(k) = X[k*x_s]
  int64_t y_s;           // y(r) = Y[r*y_s]
  int64_t bias_s;        // bias(r) = bias[r*bias_s]
  int64_t batch, sW, sX, sY, sBias;
  int conj_w, conj_x;
  int x_vec;             // rows kernel: x is unit-stride and 16-byte aligned in every batch
  EpiScalars epi;
  int ksplit;            // cols and staged-x rows kernels: CTAs along K
  int64_t kchunk;        // K elements per CTA (a multiple of 16 bytes of W for the rows kernel)
  void *ws;              // ksplit*batch*mrows*R accumulators
  unsigned *tickets;     // batch * gridDim.x counters, zero on entry and exit
  // cols kernel with several x rows (thin M): x row m at X + m*x_rs, y row m at
  // Y + m*y_rs, bias row m at bias + m*bias_rs; rows in mrb blocks of the
  // kernel's MR (grid x = column blocks * mrb, the row block varying fastest)
  int mrows, mrb;
  int64_t x_rs, y_rs, bias_rs;
};

template <class T, int VEC>
struct VecLoad {
  union U { uint4 u; T v[VEC]; };
  static_assert(sizeof(T) * VEC == 16, "16-byte vectors");
  __device__ static __forceinline__ void load(const T *p, T (&out)[VEC]) {
    U x;
    asm volatile("ld.global.nc.L1::no_allocate.v4.u32 {%0,%1,%2,%3}, [%4];"
                 : "=r"(x.u.x), "=r"(x.u.y), "=r"(x.u.z), "=r"(x.u.w) : "l"(p));
#pragma unroll
    for (int i = 0; i < VEC; ++i) out[i] = x.v[i];
  }
  __device__ static __forceinline__ uint4 raw(const T *p) {
    uint4 q;
    asm volatile("ld.global.nc.L1::no_allocate.v4.u32 {%0,%1,%2,%3}, [%4];"
                 : "=r"(q.x), "=r"(q.y), "=r"(q.z), "=r"(q.w) : "l"(p));
    return q;
  }
};

// acc += dot(w, x) over one 16-byte vector of each.  Generic form: unpack and
// multiply in the accumulator type.
template <class T, int VEC>
struct Dot16 {
  __device__ static __forceinline__ void run(typename Elem<T>::acc &acc, const uint4 &w, const uint4 &x, int cw, int cx) {
    union { uint4 q; T v[VEC]; } wu, xu;
    wu.q = w;
    xu.q = x;
#pragma unroll
    for (int i = 0; i < VEC; ++i) Elem<T>::mad(acc, Elem<T>::load(wu.v[i], cw), Elem<T>::load(xu.v[i], cx));
  }
};
// 16-bit floats: the sm_100 mixed-precision FMA (fp16/bf16 inputs, fp32 addend
// and result, one rounding) takes the packed halves directly, so no conversion
// instructions are issued; the result equals fmaf(float(w), float(x), acc).
#define MB_DOT16_MIXED(TYPE, PTXT)                                                                      \
  template <>                                                                                           \
  struct Dot16<TYPE, 8> {                                                                               \
    __device__ static __forceinline__ void run(float &acc, const uint4 &w, const uint4 &x, int, int) {  \
      const unsigned wv[4] = {w.x, w.y, w.z, w.w}, xv[4] = {x.x, x.y, x.z, x.w};                        \
      _Pragma("unroll") for (int i = 0; i < 4; ++i)                                                     \
        asm("{.reg .b16 wl, wh, xl, xh;\n\t"                                                            \
            "mov.b32 {wl, wh}, %1;\n\t"                                                                 \
            "mov.b32 {xl, xh}, %2;\n\t"                                                                 \
            "fma.rn.f32." PTXT " %0, wl, xl, %0;\n\t"                                                   \
            "fma.rn.f32." PTXT " %0, wh, xh, %0;}"                                                      \
            : "+f"(acc) : "r"(wv[i]), "r"(xv[i]));                                                      \
    }                                                                                                   \
  };
MB_DOT16_MIXED(__nv_bfloat16, "bf16")
MB_DOT16_MIXED(__half, "f16")
#undef MB_DOT16_MIXED

template <class Acc> __device__ __forceinline__ void acc_add(Acc &a, const Acc &b) { a += b; }
template <> __device__ __forceinline__ void acc_add<cf32>(cf32 &a, const cf32 &b) { a.re += b.re; a.im += b.im; }

template <class Acc> __device__ __forceinline__ Acc shfl_xor(Acc v, int m) { return __shfl_xor_sync(0xffffffffu, v, m); }
template <> __device__ __forceinline__ cf32 shfl_xor<cf32>(cf32 v, int m) {
  return cf32{__shfl_xor_sync(0xffffffffu, v.re, m), __shfl_xor_sync(0xffffffffu, v.im, m)};
}

template <class T>
__device__ __forceinline__ void gemv_store(const GemvParams &p, int64_t b, int64_t r, typename Elem<T>::acc v) {
  if (p.epi.enabled) {
    const T *bias = (const T *)p.bias + b * p.sBias + r * p.bias_s;
    v = EpiOps<T>::apply(v, bias, p.epi);
  }
  ((T *)p.Y)[b * p.sY + r * p.y_s] = Elem<T>::store(v);
}

// gemv_store for row m of a thin-M product (cols kernel).
template <class T>
__device__ __forceinline__ void gemv_store_m(const GemvParams &p, int64_t b, int64_t m, int64_t r,
                                             typename Elem<T>::acc v) {
  if (p.epi.enabled) {
    const T *bias = (const T *)p.bias + b * p.sBias + m * p.bias_rs + r * p.bias_s;
    v = EpiOps<T>::apply(v, bias, p.epi);
  }
  ((T *)p.Y)[b * p.sY + m * p.y_rs + r * p.y_s] = Elem<T>::store(v);
}

// One K row of gemv_cols: acc[i] += x * w[i] for VEC consecutive columns.
// Generic form: widen and multiply in the accumulator type.
template <class T, int VEC>
struct ColRow {
  using Acc = typename Elem<T>::acc;
  struct X { Acc v; };
  __device__ static __forceinline__ X prep(T x, int conj_x, int) { return X{Elem<T>::load(x, conj_x)}; }
  __device__ static __forceinline__ void run(Acc (&acc)[VEC], const T (&w)[VEC], const X &x, int conj_w) {
#pragma unroll
    for (int i = 0; i < VEC; ++i) Elem<T>::mad(acc[i], x.v, Elem<T>::load(w[i], conj_w));
  }
};
// 16-bit floats: the sm_100 mixed-precision FMA takes w's halves directly
// (fp32 addend and result, one rounding: the same value as fmaf on the widened
// operands).
#define MB_COLROW_MIXED(TYPE, PTXT)                                                           \
  template <>                                                                                 \
  struct ColRow<TYPE, 8> {                                                                    \
    struct X { unsigned short h; };                                                           \
    __device__ static __forceinline__ X prep(TYPE x, int, int) {                              \
      return X{*reinterpret_cast<const unsigned short *>(&x)};                                \
    }                                                                                         \
    __device__ static __forceinline__ void run(float (&acc)[8], const TYPE (&w)[8], const X &x, int) { \
      const unsigned *wv = reinterpret_cast<const unsigned *>(w);                             \
      _Pragma("unroll") for (int i = 0; i < 4; ++i)                                           \
        asm("{.reg .b16 wl, wh;\n\t"                                                          \
            "mov.b32 {wl, wh}, %2;\n\t"                                                       \
            "fma.rn.f32." PTXT " %0, wl, %3, %0;\n\t"                                         \
            "fma.rn.f32." PTXT " %1, wh, %3, %1;}"                                            \
            : "+f"(acc[2 * i]), "+f"(acc[2 * i + 1]) : "r"(wv[i]), "h"(x.h));                 \
    }                                                                                         \
  };
MB_COLROW_MIXED(__nv_bfloat16, "bf16")
MB_COLROW_MIXED(__half, "f16")
#undef MB_COLROW_MIXED
// complex32: acc += op(w) * x with four mixed-precision FMAs per element on the
// packed (re, im) halves; x is turned once into the half coefficients
// (P, Q, R, S) with re += w.re*P + w.im*Q and im += w.re*R + w.im*S, which fold
// the conjugations of x and of w into signs (negating a half is exact).
template <>
struct ColRow<__half2, 4> {
  struct X { unsigned pq, rs; };
  __device__ static __forceinline__ X prep(__half2 x, int conj_x, int conj_w) {
    const __half xr = __low2half(x);
    const __half xi = conj_x ? __hneg(__high2half(x)) : __high2half(x);
    const __half2 pq = conj_w ? __halves2half2(xr, xi) : __halves2half2(xr, __hneg(xi));
    const __half2 rs = conj_w ? __halves2half2(xi, __hneg(xr)) : __halves2half2(xi, xr);
    return X{*reinterpret_cast<const unsigned *>(&pq), *reinterpret_cast<const unsigned *>(&rs)};
  }
  __device__ static __forceinline__ void run(cf32 (&acc)[4], const __half2 (&w)[4], const X &x, int) {
    const unsigned *wv = reinterpret_cast<const unsigned *>(w);
#pragma unroll
    for (int i = 0; i < 4; ++i)
      asm("{.reg .b16 wr, wi, p, q, r, s;\n\t"
          "mov.b32 {wr, wi}, %2;\n\t"
          "mov.b32 {p, q}, %3;\n\t"
          "mov.b32 {r, s}, %4;\n\t"
          "fma.rn.f32.f16 %0, wr, p, %0;\n\t"
          "fma.rn.f32.f16 %0, wi, q, %0;\n\t"
          "fma.rn.f32.f16 %1, wr, r, %1;\n\t"
          "fma.rn.f32.f16 %1, wi, s, %1;}"
          : "+f"(acc[i].re), "+f"(acc[i].im) : "r"(wv[i]), "r"(x.pq), "r"(x.rs));
  }
};

// ---------------------------------------------------------------------------
// gemv_cols: grid (ceil(R / (32*VEC)), ksplit, batch), NW warps per CTA.
// VEC == 1 is the unaligned fallback (scalar loads).  MR > 1: thin M, a block
// of up to MR rows of x shares every 16-byte load of W (each W element feeds
// MR FMAs; rows past the block's last re-read it and their sums are dropped).
// Grid x = column blocks * p.mrb with the row block varying fastest, so the
// row blocks of one column stripe run together and share it through L2.
template <class T, int VEC, int NW, int MR = 1>
__global__ void __launch_bounds__(NW * 32) gemv_cols_kernel(const GemvParams p) {
  using E = Elem<T>;
  using Acc = typename E::acc;
  constexpr int COLS = 32 * VEC;
  __shared__ Acc red[NW][COLS];
  __shared__ unsigned s_ticket;

  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int mrb = MR == 1 ? 1 : p.mrb;
  const int64_t b = blockIdx.z;
  const int row0 = (int)(blockIdx.x % mrb) * MR;
  const int64_t cblk = blockIdx.x / mrb;
  const int64_t c0 = cblk * COLS + lane * VEC;
  const int64_t kbeg = (int64_t)blockIdx.y * p.kchunk;
  const int64_t kend = min(p.K, kbeg + p.kchunk);
  const T *W = (const T *)p.W + b * p.sW;
  const T *X = (const T *)p.X + b * p.sX;
  if constexpr (VEC > 1) {
    // The first 32 KB of this CTA's stripe of W (COLS columns of its rows,
    // one 16-byte aligned run per row) into L2 while the previous kernel
    // drains: enough to keep DRAM busy across the kernel boundary, too little
    // to evict what the running kernels read.
    constexpr int PF_ROWS = 32768 / (COLS * (int)sizeof(T));
    const int64_t cb = cblk * COLS;
    if (cb + COLS <= p.R && row0 == 0)
      for (int64_t kk = kbeg + threadIdx.x; kk < min(kend, kbeg + PF_ROWS); kk += NW * 32)
        prefetch_l2_bulk(W + kk * p.w_ld + cb, COLS * (uint32_t)sizeof(T));
  }
  pdl_wait();
  const int mrows = MR == 1 ? 1 : p.mrows;          // rows of x in all
  const int rows = MR == 1 ? 1 : min(MR, mrows - row0);  // rows in this CTA's block
  int64_t xoff[MR];
#pragma unroll
  for (int r = 0; r < MR; ++r) xoff[r] = (int64_t)(row0 + min(r, rows - 1)) * p.x_rs;

  Acc acc[MR][VEC];
#pragma unroll
  for (int r = 0; r < MR; ++r)
#pragma unroll
    for (int i = 0; i < VEC; ++i) acc[r][i] = E::zero();

  const bool full = (c0 + VEC <= p.R);
  constexpr int U = MR == 1 ? 8 : 4;  // independent 16-byte loads of W in flight per thread
  int64_t k = kbeg + warp;
  bool done = false;
  if constexpr (VEC > 1 && MR > 1) {
    if (full) {
      // Several x rows: each warp walks a contiguous K range so that its x
      // reads run along K through L1 lines (interleaved warps would take every
      // x element from L2 once per CTA).
      done = true;
      using CR = ColRow<T, VEC>;
      const int64_t span = ((kend - kbeg + NW - 1) / NW + U - 1) / U * U;
      k = kbeg + warp * span;
      const int64_t kw = min(kend, k + span);
      for (; k + U <= kw; k += U) {
        T w[U][VEC];
        typename CR::X xv[U][MR];
#pragma unroll
        for (int u = 0; u < U; ++u) VecLoad<T, VEC>::load(W + (k + u) * p.w_ld + c0, w[u]);
#pragma unroll
        for (int u = 0; u < U; ++u)
#pragma unroll
          for (int r = 0; r < MR; ++r) xv[u][r] = CR::prep(X[xoff[r] + (k + u) * p.x_s], p.conj_x, p.conj_w);
#pragma unroll
        for (int u = 0; u < U; ++u)
#pragma unroll
          for (int r = 0; r < MR; ++r) CR::run(acc[r], w[u], xv[u][r], p.conj_w);
      }
      for (; k < kw; ++k) {
        T w[VEC];
        VecLoad<T, VEC>::load(W + k * p.w_ld + c0, w);
#pragma unroll
        for (int r = 0; r < MR; ++r) CR::run(acc[r], w, CR::prep(X[xoff[r] + k * p.x_s], p.conj_x, p.conj_w), p.conj_w);
      }
    }
  } else if constexpr (VEC > 1) {
    if (full) {
      done = true;
      using CR = ColRow<T, VEC>;
      for (; k + (U - 1) * NW < kend; k += U * NW) {
        T w[U][VEC];
        typename CR::X xv[U][MR];
#pragma unroll
        for (int u = 0; u < U; ++u) VecLoad<T, VEC>::load(W + (k + u * NW) * p.w_ld + c0, w[u]);
#pragma unroll
        for (int u = 0; u < U; ++u)
#pragma unroll
          for (int r = 0; r < MR; ++r) xv[u][r] = CR::prep(X[xoff[r] + (k + u * NW) * p.x_s], p.conj_x, p.conj_w);
#pragma unroll
        for (int u = 0; u < U; ++u)
#pragma unroll
          for (int r = 0; r < MR; ++r) CR::run(acc[r], w[u], xv[u][r], p.conj_w);
      }
      for (; k < kend; k += NW) {
        T w[VEC];
        VecLoad<T, VEC>::load(W + k * p.w_ld + c0, w);
#pragma unroll
        for (int r = 0; r < MR; ++r) CR::run(acc[r], w, CR::prep(X[xoff[r] + k * p.x_s], p.conj_x, p.conj_w), p.conj_w);
      }
    }
  }
  if (!done) {
    for (; k < kend; k += NW) {
#pragma unroll
      for (int r = 0; r < MR; ++r) {
        const Acc xv = E::load(X[xoff[r] + k * p.x_s], p.conj_x);
#pragma unroll
        for (int i = 0; i < VEC; ++i)
          if (c0 + i < p.R) E::mad(acc[r][i], xv, E::load(W[k * p.w_ld + c0 + i], p.conj_w));
      }
    }
  }

  // W is streamed: the next kernel on the stream may start its set-up and
  // prefetch (launched once every CTA of this grid has passed here).
  pdl_trigger();
  // Sum the warps' partials row by row through one shared buffer.  ksplit == 1
  // stores the result; otherwise the partial is published for the last CTA.
  const int64_t cbase = cblk * COLS;
  Acc *ws = p.ksplit > 1 ? (Acc *)p.ws + ((b * p.ksplit + blockIdx.y) * mrows + row0) * p.R : nullptr;
#pragma unroll
  for (int r = 0; r < MR; ++r) {
    if (r >= rows) break;
    if (r) __syncthreads();  // the previous row's sums have been read
#pragma unroll
    for (int i = 0; i < VEC; ++i) red[warp][lane * VEC + i] = acc[r][i];
    __syncthreads();
    for (int c = threadIdx.x; c < COLS; c += NW * 32) {
      if (cbase + c >= p.R) continue;
      Acc s = red[0][c];
#pragma unroll
      for (int w = 1; w < NW; ++w) acc_add(s, red[w][c]);
      if (p.ksplit == 1) gemv_store_m<T>(p, b, row0 + r, cbase + c, s);
      else ws[r * p.R + cbase + c] = s;
    }
  }
  if (p.ksplit == 1) return;

  // Split K across CTAs: publish this CTA's partial, take a ticket; the CTA
  // that draws the last ticket sums all partials in split order (deterministic)
  // and resets the ticket for the next launch.
  __threadfence();
  __syncthreads();
  unsigned *ticket = p.tickets + b * gridDim.x + blockIdx.x;
  if (threadIdx.x == 0) s_ticket = atomicAdd(ticket, 1u);
  __syncthreads();
  if (s_ticket != (unsigned)(p.ksplit - 1)) return;
  __threadfence();
  const Acc *ws0 = (const Acc *)p.ws + b * p.ksplit * mrows * p.R;
  for (int m = row0; m < row0 + rows; ++m) {
    for (int c = threadIdx.x; c < COLS; c += NW * 32) {
      const int64_t r = cbase + c;
      if (r >= p.R) continue;
      Acc s = E::zero();
      for (int sp = 0; sp < p.ksplit; ++sp) {
        const Acc *src = ws0 + ((int64_t)sp * mrows + m) * p.R + r;
        Acc v;
        if constexpr (sizeof(Acc) == 8 && !E::is_int) {
          float2 f = __ldcg((const float2 *)src);
          v = *reinterpret_cast<Acc *>(&f);
        } else {
          v = __ldcg(src);
        }
        acc_add(s, v);
      }
      gemv_store_m<T>(p, b, m, r, s);
    }
  }
  if (threadIdx.x == 0) *ticket = 0u;
}

// ---------------------------------------------------------------------------
// gemv_rows: one warp per output row, grid (ceil(R / NW), 1, batch).
// VEC == 1 is the unaligned fallback.
template <class T, int VEC, int NW>
__global__ void __launch_bounds__(NW * 32) gemv_rows_kernel(const GemvParams p) {
  using E = Elem<T>;
  using Acc = typename E::acc;
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int64_t b = blockIdx.z;
  const int64_t r = (int64_t)blockIdx.x * NW + warp;
  pdl_wait();
  if (r >= p.R) { pdl_trigger(); return; }
  const T *W = (const T *)p.W + b * p.sW + r * p.w_ld;
  const T *X = (const T *)p.X + b * p.sX;

  Acc acc = E::zero();
  int64_t k = (int64_t)lane * VEC;
  if constexpr (VEC > 1) {
    constexpr int U = 4;
    constexpr int64_t STEP = 32 * VEC;
    const int64_t kvec_end = (p.K / VEC) * VEC;  // vector part
    const bool x_vec = p.x_vec != 0;
    for (; k + (U - 1) * STEP + VEC <= kvec_end; k += U * STEP) {
      T w[U][VEC];
#pragma unroll
      for (int u = 0; u < U; ++u) VecLoad<T, VEC>::load(W + k + u * STEP, w[u]);
#pragma unroll
      for (int u = 0; u < U; ++u) {
        const int64_t kk = k + u * STEP;
        if (x_vec) {
          T xv[VEC];
          const T *xp = X + kk;
          union { uint4 q; T v[VEC]; } xu;
          xu.q = __ldg(reinterpret_cast<const uint4 *>(xp));
#pragma unroll
          for (int i = 0; i < VEC; ++i) xv[i] = xu.v[i];
#pragma unroll
          for (int i = 0; i < VEC; ++i) E::mad(acc, E::load(w[u][i], p.conj_w), E::load(xv[i], p.conj_x));
        } else {
#pragma unroll
          for (int i = 0; i < VEC; ++i)
            E::mad(acc, E::load(w[u][i], p.conj_w), E::load(X[(kk + i) * p.x_s], p.conj_x));
        }
      }
    }
    for (; k + VEC <= kvec_end; k += STEP) {
      T w[VEC];
      VecLoad<T, VEC>::load(W + k, w);
#pragma unroll
      for (int i = 0; i < VEC; ++i)
        E::mad(acc, E::load(w[i], p.conj_w), E::load(X[(k + i) * p.x_s], p.conj_x));
    }
    // scalar tail beyond the last full vector
    for (int64_t kk = kvec_end + lane; kk < p.K; kk += 32)
      E::mad(acc, E::load(W[kk], p.conj_w), E::load(X[kk * p.x_s], p.conj_x));
  } else {
    for (int64_t kk = lane; kk < p.K; kk += 32)
      E::mad(acc, E::load(W[kk], p.conj_w), E::load(X[kk * p.x_s], p.conj_x));
  }
  pdl_trigger();  // W is streamed: the next kernel may start its set-up
#pragma unroll
  for (int m = 16; m >= 1; m >>= 1) acc_add(acc, shfl_xor(acc, m));
  if (lane == 0) gemv_store<T>(p, b, r, acc);
}

// ---------------------------------------------------------------------------
// gemv_rows with x staged in shared memory: W rows contiguous along K, x unit
// stride and 16-byte aligned.  Each warp owns RPW rows; x is read from global
// memory once per CTA (in 16 KB chunks) instead of once per row, so the only
// streamed global traffic is W.  grid (ceil(R / (NW * RPW)), ksplit, batch):
// CTA (x, y) covers rows [x*NW*RPW, +NW*RPW) over K range [y*kchunk, +kchunk).
// Splitting K keeps every CTA short, so the last partial wave of a long row
// sweep does not leave most SMs idle; partials are summed in split order by
// the CTA that draws the last ticket, as in gemv_cols.
template <class T, int VEC, int NW, int RPW>
__global__ void __launch_bounds__(NW * 32, sizeof(typename Elem<T>::acc) == 8 ? 2 : 3)
gemv_rows_smem_kernel(const GemvParams p) {
  using E = Elem<T>;
  using Acc = typename E::acc;
  constexpr int KC = 16384 / (int)sizeof(T);  // x elements per staged chunk
  constexpr int U = 4;                        // K vectors in flight per row and lane
  constexpr int STEP = 32 * VEC;
  __shared__ __align__(16) T xs[KC];
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int64_t b = blockIdx.z;
  const int64_t r0 = ((int64_t)blockIdx.x * NW + warp) * RPW;
  const T *X = (const T *)p.X + b * p.sX;
  const T *W = (const T *)p.W + b * p.sW;
  Acc acc[RPW];
#pragma unroll
  for (int r = 0; r < RPW; ++r) acc[r] = E::zero();
  const T *wrow[RPW];
  bool live[RPW];
#pragma unroll
  for (int r = 0; r < RPW; ++r) {
    live[r] = r0 + r < p.R;
    wrow[r] = W + (live[r] ? (r0 + r) : 0) * p.w_ld;
  }

  const int64_t kbeg = (int64_t)blockIdx.y * p.kchunk;
  const int64_t kend = min(p.K, kbeg + p.kchunk);
  if constexpr (VEC > 1) {
    // the first 4 KB of each of this warp's rows over [kbeg, kend) into L2
    // while the previous kernel drains (lane 0 of each row)
    const int64_t kv = min((int64_t)4096, ((kend - kbeg) * (int64_t)sizeof(T)) & ~int64_t(15));
#pragma unroll
    for (int r = 0; r < RPW; ++r)
      if (lane == 0 && live[r] && kv > 0 && (reinterpret_cast<uintptr_t>(wrow[r] + kbeg) & 15) == 0)
        prefetch_l2_bulk(wrow[r] + kbeg, (uint32_t)kv);
  }
  pdl_wait();
  for (int64_t kc = kbeg; kc < kend; kc += KC) {
    const int kn = (int)min((int64_t)KC, kend - kc);
    __syncthreads();  // previous chunk fully consumed
    for (int i = threadIdx.x * VEC; i < kn; i += NW * 32 * VEC) {
      if (i + VEC <= kn) {
        *reinterpret_cast<uint4 *>(&xs[i]) = __ldg(reinterpret_cast<const uint4 *>(X + kc + i));
      } else {
        for (int j = 0; j < VEC && i + j < kn; ++j) xs[i + j] = X[kc + i + j];
      }
    }
    __syncthreads();
    const int kvec = (kn / VEC) * VEC;
    int k = lane * VEC;
    for (; k + (U - 1) * STEP + VEC <= kvec; k += U * STEP) {
      uint4 w[RPW][U];
#pragma unroll
      for (int r = 0; r < RPW; ++r)
#pragma unroll
        for (int u = 0; u < U; ++u)
          w[r][u] = live[r] ? VecLoad<T, VEC>::raw(wrow[r] + kc + k + u * STEP) : make_uint4(0, 0, 0, 0);
#pragma unroll
      for (int u = 0; u < U; ++u) {
        const uint4 xq = *reinterpret_cast<const uint4 *>(&xs[k + u * STEP]);
#pragma unroll
        for (int r = 0; r < RPW; ++r)
          if (live[r]) Dot16<T, VEC>::run(acc[r], w[r][u], xq, p.conj_w, p.conj_x);
      }
    }
    for (; k + VEC <= kvec; k += STEP) {
      const uint4 xq = *reinterpret_cast<const uint4 *>(&xs[k]);
#pragma unroll
      for (int r = 0; r < RPW; ++r)
        if (live[r]) Dot16<T, VEC>::run(acc[r], VecLoad<T, VEC>::raw(wrow[r] + kc + k), xq, p.conj_w, p.conj_x);
    }
    for (int kk = kvec + lane; kk < kn; kk += 32)
#pragma unroll
      for (int r = 0; r < RPW; ++r)
        if (live[r]) E::mad(acc[r], E::load(wrow[r][kc + kk], p.conj_w), E::load(xs[kk], p.conj_x));
  }
  pdl_trigger();  // W is streamed: the next kernel may start its set-up
#pragma unroll
  for (int r = 0; r < RPW; ++r)
#pragma unroll
    for (int m = 16; m >= 1; m >>= 1) acc_add(acc[r], shfl_xor(acc[r], m));
  if (p.ksplit == 1) {
#pragma unroll
    for (int r = 0; r < RPW; ++r)
      if (lane == 0 && live[r]) gemv_store<T>(p, b, r0 + r, acc[r]);
    return;
  }
  Acc *ws = (Acc *)p.ws + (b * p.ksplit + blockIdx.y) * p.R;
#pragma unroll
  for (int r = 0; r < RPW; ++r)
    if (lane == 0 && live[r]) ws[r0 + r] = acc[r];
  __shared__ unsigned s_ticket;
  __threadfence();
  __syncthreads();
  unsigned *ticket = p.tickets + b * gridDim.x + blockIdx.x;
  if (threadIdx.x == 0) s_ticket = atomicAdd(ticket, 1u);
  __syncthreads();
  if (s_ticket != (unsigned)(p.ksplit - 1)) return;
  __threadfence();
  const Acc *ws0 = (const Acc *)p.ws + b * p.ksplit * p.R;
  if (threadIdx.x < NW * RPW) {
    const int64_t r = (int64_t)blockIdx.x * NW * RPW + threadIdx.x;
    if (r < p.R) {
      Acc s = E::zero();
      for (int sp = 0; sp < p.ksplit; ++sp) {
        Acc v;
        if constexpr (sizeof(Acc) == 8 && !E::is_int) {
          float2 f = __ldcg((const float2 *)(ws0 + sp * p.R + r));
          v = *reinterpret_cast<Acc *>(&f);
        } else {
          v = __ldcg(ws0 + sp * p.R + r);
        }
        acc_add(s, v);
      }
      gemv_store<T>(p, b, r, s);
    }
  }
  if (threadIdx.x == 0) *ticket = 0u;
}

}  // namespace mb
