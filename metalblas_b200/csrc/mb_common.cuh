// Element traits, epilogue arithmetic and small device helpers shared by every
// kernel of the library.
//
// Arithmetic contract (reference semantics):
//  * floats accumulate in fp32 and round once on store
//    (metalblas/float_dispatch.py:25-29 PROFILE: in/acc/out = T/float/T);
//  * complex64/complex32 accumulate as fp32 complex
//    (metalblas/complex_dispatch.py:10-13, shaders/complex_pack.h:37-38);
//  * integers accumulate in a wrapping accumulator (int8/int16/int32 -> 32 bit,
//    uint8 -> 32 bit unsigned, int64 -> 64 bit) and truncate on store, which is
//    the two's-complement result of the exact product mod 2^bits
//    (metalblas/integer_dispatch.py:13-19, shaders/int_gemm.h:122-150).
//    We accumulate in unsigned types so that overflow is defined behaviour.
//  * the addmm epilogue v = alpha*acc + beta*bias is computed in the scalar type
//    (fp32 for floats, complex fp32, the accumulator for integers) with the
//    alpha_nz / beta_nz switches of shaders/mb_epi.h:16-26.
#pragma once
#include <cuda_runtime.h>
#include <cuda_fp16.h>
#include <cuda_bf16.h>
#include <stdint.h>

namespace mb {

struct cf32 {
  float re, im;
};

__device__ __forceinline__ cf32 cmul(cf32 a, cf32 b) {
  return cf32{a.re * b.re - a.im * b.im, a.re * b.im + a.im * b.re};
}

// Elem<T>: storage type T -> accumulator `acc`, epilogue scalar `scal`,
// conversions, and multiply-accumulate.
template <class T> struct Elem;

template <> struct Elem<float> {
  using acc = float; using scal = float;
  static constexpr bool is_int = false, is_cplx = false;
  __device__ static __forceinline__ acc load(float v, bool) { return v; }
  __device__ static __forceinline__ float store(acc v) { return v; }
  __device__ static __forceinline__ void mad(acc &c, acc a, acc b) { c = fmaf(a, b, c); }
  __device__ static __forceinline__ acc zero() { return 0.f; }
};
template <> struct Elem<__half> {
  using acc = float; using scal = float;
  static constexpr bool is_int = false, is_cplx = false;
  __device__ static __forceinline__ acc load(__half v, bool) { return __half2float(v); }
  __device__ static __forceinline__ __half store(acc v) { return __float2half_rn(v); }
  __device__ static __forceinline__ void mad(acc &c, acc a, acc b) { c = fmaf(a, b, c); }
  __device__ static __forceinline__ acc zero() { return 0.f; }
};
template <> struct Elem<__nv_bfloat16> {
  using acc = float; using scal = float;
  static constexpr bool is_int = false, is_cplx = false;
  __device__ static __forceinline__ acc load(__nv_bfloat16 v, bool) { return __bfloat162float(v); }
  __device__ static __forceinline__ __nv_bfloat16 store(acc v) { return __float2bfloat16_rn(v); }
  __device__ static __forceinline__ void mad(acc &c, acc a, acc b) { c = fmaf(a, b, c); }
  __device__ static __forceinline__ acc zero() { return 0.f; }
};
template <> struct Elem<float2> {  // complex64
  using acc = cf32; using scal = cf32;
  static constexpr bool is_int = false, is_cplx = true;
  __device__ static __forceinline__ acc load(float2 v, bool conj) { return cf32{v.x, conj ? -v.y : v.y}; }
  __device__ static __forceinline__ float2 store(acc v) { return make_float2(v.re, v.im); }
  __device__ static __forceinline__ void mad(acc &c, acc a, acc b) {
    c.re = fmaf(a.re, b.re, c.re); c.re = fmaf(-a.im, b.im, c.re);
    c.im = fmaf(a.re, b.im, c.im); c.im = fmaf(a.im, b.re, c.im);
  }
  __device__ static __forceinline__ acc zero() { return cf32{0.f, 0.f}; }
};
template <> struct Elem<__half2> {  // complex32 (interleaved half re, half im)
  using acc = cf32; using scal = cf32;
  static constexpr bool is_int = false, is_cplx = true;
  __device__ static __forceinline__ acc load(__half2 v, bool conj) {
    float2 f = __half22float2(v); return cf32{f.x, conj ? -f.y : f.y};
  }
  __device__ static __forceinline__ __half2 store(acc v) { return __floats2half2_rn(v.re, v.im); }
  __device__ static __forceinline__ void mad(acc &c, acc a, acc b) { Elem<float2>::mad(c, a, b); }
  __device__ static __forceinline__ acc zero() { return cf32{0.f, 0.f}; }
};

#define MB_INT_ELEM(T, ACC)                                                              \
  template <> struct Elem<T> {                                                           \
    using acc = ACC; using scal = ACC;                                                   \
    static constexpr bool is_int = true, is_cplx = false;                                \
    __device__ static __forceinline__ acc load(T v, bool) { return (acc)(v); }           \
    __device__ static __forceinline__ T store(acc v) { return (T)(v); }                  \
    __device__ static __forceinline__ void mad(acc &c, acc a, acc b) { c += a * b; }     \
    __device__ static __forceinline__ acc zero() { return (acc)0; }                      \
  };
// Signed loads sign-extend into the unsigned accumulator: (uint32_t)(int8_t)-3
// == 2^32-3, so the wrapped sum is the two's-complement sum.
MB_INT_ELEM(int8_t, uint32_t)
MB_INT_ELEM(uint8_t, uint32_t)
MB_INT_ELEM(int16_t, uint32_t)
MB_INT_ELEM(int32_t, uint32_t)
MB_INT_ELEM(int64_t, uint64_t)
#undef MB_INT_ELEM

// Epilogue scalars as passed to every kernel.
struct EpiScalars {
  float alpha_re, alpha_im, beta_re, beta_im;
  int64_t ialpha, ibeta;
  int alpha_nz, beta_nz, enabled;
  int cplx;  // tensor-core complex32: columns (2j, 2j+1) are one complex value, bias is half2
};

template <class T> struct EpiOps;
template <class T> struct EpiOpsReal {
  using A = typename Elem<T>::acc;
  __device__ static __forceinline__ A apply(A acc, const T *bias, const EpiScalars &e) {
    A v = 0.f;
    if (e.alpha_nz) v = e.alpha_re * acc;
    if (e.beta_nz) v = fmaf(e.beta_re, Elem<T>::load(*bias, false), v);
    return v;
  }
};
template <class T> struct EpiOpsCplx {
  using A = cf32;
  __device__ static __forceinline__ A apply(A acc, const T *bias, const EpiScalars &e) {
    A v{0.f, 0.f};
    if (e.alpha_nz) v = cmul(cf32{e.alpha_re, e.alpha_im}, acc);
    if (e.beta_nz) {
      cf32 b = cmul(cf32{e.beta_re, e.beta_im}, Elem<T>::load(*bias, false));
      v.re += b.re; v.im += b.im;
    }
    return v;
  }
};
template <class T> struct EpiOpsInt {
  using A = typename Elem<T>::acc;
  __device__ static __forceinline__ A apply(A acc, const T *bias, const EpiScalars &e) {
    A v = 0;
    if (e.alpha_nz) v = (A)e.ialpha * acc;
    if (e.beta_nz) v += (A)e.ibeta * Elem<T>::load(*bias, false);
    return v;
  }
};
template <> struct EpiOps<float> : EpiOpsReal<float> {};
template <> struct EpiOps<__half> : EpiOpsReal<__half> {};
template <> struct EpiOps<__nv_bfloat16> : EpiOpsReal<__nv_bfloat16> {};
template <> struct EpiOps<float2> : EpiOpsCplx<float2> {};
template <> struct EpiOps<__half2> : EpiOpsCplx<__half2> {};
template <> struct EpiOps<int8_t> : EpiOpsInt<int8_t> {};
template <> struct EpiOps<uint8_t> : EpiOpsInt<uint8_t> {};
template <> struct EpiOps<int16_t> : EpiOpsInt<int16_t> {};
template <> struct EpiOps<int32_t> : EpiOpsInt<int32_t> {};
template <> struct EpiOps<int64_t> : EpiOpsInt<int64_t> {};

// Device status word: set to a non-zero mb_status when a bounded wait gives up.
// (The library is one translation unit, so this is its only definition.)
__device__ int g_mb_status = 0;

__device__ __forceinline__ uint64_t globaltimer_ns() {
  uint64_t t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}

// Programmatic dependent launch.  The GEMV and tcgen05 kernels are launched
// with programmatic stream serialization: a kernel may start while the
// previous kernel on its stream is still finishing, once every CTA of that
// kernel has called pdl_trigger (or exited).  The GEMV kernels trigger when
// their stream of W is done (earlier, the next grid could take free CTA slots
// and its prefetches be evicted before use); the tcgen05 kernel, whose CTAs
// fill their SMs, triggers on entry.  pdl_wait blocks until the
// previous kernel has completed and its memory operations are visible; every
// thread calls it before its first global load or store of data another
// kernel may write, so only set-up work (barriers, TMEM, tensor-map and L2
// prefetches) overlaps.  Both are no-ops for a launch without the attribute.
__device__ __forceinline__ void pdl_trigger() { asm volatile("griddepcontrol.launch_dependents;" ::: "memory"); }
__device__ __forceinline__ void pdl_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }
// L2 prefetch of `bytes` (a multiple of 16) at a 16-byte aligned address: a
// hint with no effect on the memory model, so it may run before pdl_wait.
__device__ __forceinline__ void prefetch_l2_bulk(const void *p, uint32_t bytes) {
  asm volatile("cp.async.bulk.prefetch.L2.global [%0], %1;" ::"l"(p), "r"(bytes) : "memory");
}

}  // namespace mb
