// Operand packing for the tensor-core path: a strided (batched) matrix copied
// into dense row-major rows of pitch `ld` elements, so that TMA can load it.
// Used for views TMA cannot address in place (unaligned base or pitch, no unit
// stride); the reference copies such views with .contiguous()
// (metalblas/dispatch.py:33-35).
#pragma once
#include "mb_common.cuh"

#include <type_traits>

namespace mb {

struct PackArgs {
  const void *src;
  void *dst;
  int64_t rows, cols;   // logical extents
  int64_t rs, cs, bs;   // source strides in elements (bs: batch)
  int64_t batch, ld;    // batches copied; destination row pitch in elements
};

// Any strides: 32 x 32 tiles through shared memory, read along whichever of
// rows / columns has the smaller source stride (coalesced for a column-major
// or transposed view) and written along the destination rows.  Block 32 x 8,
// grid-stride over tiles.  U is the element's storage type (same-size unsigned).
template <class U>
__global__ void __launch_bounds__(256) pack_matrix_kernel(const PackArgs a) {
  __shared__ U tile[32][33];
  const U *src = static_cast<const U *>(a.src);
  U *dst = static_cast<U *>(a.dst);
  const int tx = threadIdx.x, ty = threadIdx.y;
  const int64_t rt = (a.rows + 31) / 32, ct = (a.cols + 31) / 32;
  const int64_t tiles = a.batch * rt * ct;
  const bool c_fast = a.cs == 1 || (a.rs != 1 && (a.cs < 0 ? -a.cs : a.cs) <= (a.rs < 0 ? -a.rs : a.rs));
  for (int64_t t = blockIdx.x; t < tiles; t += gridDim.x) {
    const int64_t b = t / (rt * ct);
    const int64_t rem = t - b * rt * ct;
    const int64_t r0 = (rem / ct) * 32, c0 = (rem % ct) * 32;
    const U *sb = src + b * a.bs;
#pragma unroll
    for (int i = ty; i < 32; i += 8) {
      const int64_t r = r0 + (c_fast ? i : tx), c = c0 + (c_fast ? tx : i);
      const U v = (r < a.rows && c < a.cols) ? sb[r * a.rs + c * a.cs] : U(0);
      if (c_fast) tile[i][tx] = v; else tile[tx][i] = v;
    }
    __syncthreads();
#pragma unroll
    for (int i = ty; i < 32; i += 8) {
      const int64_t r = r0 + i, c = c0 + tx;
      if (r < a.rows && c < a.cols) dst[(b * a.rows + r) * a.ld + c] = tile[i][tx];
    }
    __syncthreads();
  }
}

// 16 bytes starting `off` bytes into the 32 bytes w0:w1 (little-endian words).
__device__ __forceinline__ uint4 bytes_at(const uint4 &w0, const uint4 &w1, uint32_t off) {
  uint32_t x0, x1, x2, x3, x4;
  switch (off >> 2) {
    case 0: x0 = w0.x; x1 = w0.y; x2 = w0.z; x3 = w0.w; x4 = w1.x; break;
    case 1: x0 = w0.y; x1 = w0.z; x2 = w0.w; x3 = w1.x; x4 = w1.y; break;
    case 2: x0 = w0.z; x1 = w0.w; x2 = w1.x; x3 = w1.y; x4 = w1.z; break;
    default: x0 = w0.w; x1 = w1.x; x2 = w1.y; x3 = w1.z; x4 = w1.w; break;
  }
  const uint32_t sh = (off & 3) * 8;
  return make_uint4(__funnelshift_r(x0, x1, sh), __funnelshift_r(x1, x2, sh), __funnelshift_r(x2, x3, sh),
                    __funnelshift_r(x3, x4, sh));
}

// Row-contiguous sources (cs == 1, the offset / odd-pitch views): each thread
// moves one 16-byte group of a destination row with one aligned 16-byte store.
// A full group is read as the two aligned 16-byte words it straddles (both hold
// bytes of the group, so they lie inside the source allocation) and shifted
// into place; the last group of a row is read element by element.  The
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
    if (c0 + G <= a.cols) {
      const uintptr_t addr = reinterpret_cast<uintptr_t>(s);
      const uint32_t off = (uint32_t)(addr & 15);
      const uint4 *w = reinterpret_cast<const uint4 *>(addr - off);
      const uint4 w0 = __ldg(w);
      v.q = off ? bytes_at(w0, __ldg(w + 1), off) : w0;
    } else {
#pragma unroll
      for (int j = 0; j < G; ++j) v.e[j] = (c0 + j < a.cols) ? s[j] : U(0);
    }
    *reinterpret_cast<uint4 *>(dst + (b * a.rows + r) * a.ld + c0) = v.q;
  }
}

}  // namespace mb

namespace mb {

// fp32 -> 3xTF32 operand split for the tensor cores: x = hi + lo + r with
// hi = x rounded to tf32 (nearest, ties away; cvt.rna), lo = (x - hi) rounded to
// tf32, |r| <= 2^-22 |x|.  Products hi*hi + hi*lo + lo*hi then reproduce x*y to
// about 2^-21 relative, inside the fp32 tolerance of the reference's tests.
// Non-finite x keep hi = x and lo = 0, and the split reports them: the cross
// terms inf * lo can turn into NaN where FFMA gives inf, so the caller then
// recomputes that product on the CUDA cores.  A finite x that rounds up to inf
// is truncated instead.
__device__ __forceinline__ float tf32_rna(float x) {
  uint32_t r;
  asm("cvt.rna.tf32.f32 %0, %1;" : "=r"(r) : "f"(x));
  return __uint_as_float(r);
}
__device__ __forceinline__ void tf32_split(float x, float &hi, float &lo) {
  if (!isfinite(x)) { hi = x; lo = 0.f; return; }
  hi = tf32_rna(x);
  if (isinf(hi)) hi = __uint_as_float(__float_as_uint(x) & 0xffffe000u);
  lo = tf32_rna(x - hi);
}

struct SplitArgs {
  const float *src;
  float *hi, *lo;
  int *nonfinite;       // set to 1 when any input value is inf or NaN
  int64_t rows, cols;   // output rows x cols (cols is the K dimension)
  int64_t rs, cs, bs;   // source strides of element (row, col) and batch (complex units in modes 1, 2)
  int64_t batch, ld;    // batches; destination row pitch (elements, 16-byte multiple)
  // complex64 as one real GEMM (the c32.cuh block form):
  //   mode 0: real source, element (r, c) at src[r*rs + c*cs]
  //   mode 1: A' = component c&1 of complex A(r, c/2) at complex index r*rs + (c/2)*cs
  //   mode 2: B'ᵀ (2N x 2K) from complex B(k = c/2, n = r/2) at complex index
  //           (r/2)*rs + (c/2)*cs: the 2 x 2 block [[re, -s*im'], [im', s*re]]
  //           (rows r&1, columns c&1) with im' = -im for conj(B), s = -1 for conj(A)
  int mode, conj_a, conj_b;
};

__device__ __forceinline__ float split_load(const SplitArgs &a, const float *src, int64_t r, int64_t c) {
  if (a.mode == 0) return src[r * a.rs + c * a.cs];
  const int64_t q = (a.mode == 1 ? r : (r >> 1)) * a.rs + (c >> 1) * a.cs;
  const float2 v = reinterpret_cast<const float2 *>(src)[q];
  if (a.mode == 1) return (c & 1) ? v.y : v.x;
  const float im = a.conj_b ? -v.y : v.y;
  const float s = a.conj_a ? -1.f : 1.f;
  if ((r & 1) == 0) return (c & 1) ? -s * im : v.x;
  return (c & 1) ? s * v.x : im;
}

// dst[b][r][c] = split(src(b, r, c)) through a shared-memory tile, so both the
// source read (along whichever of r / c is contiguous) and the destination rows
// are coalesced.  Block 32 x 8, grid-stride over tiles.
__global__ void __launch_bounds__(256) split_tf32_kernel(const SplitArgs a) {
  // 32 rows x 128 columns per tile; each thread then splits 4 consecutive
  // columns of a row and writes them with one 16-byte store per part
  __shared__ float tile[32][129];
  const int tx = threadIdx.x, ty = threadIdx.y;
  const int64_t rt = (a.rows + 31) / 32, ct = (a.cols + 127) / 128;
  const int64_t tiles = a.batch * rt * ct;
  const bool c_fast = a.cs == 1 || (a.rs != 1 && (a.cs < 0 ? -a.cs : a.cs) <= (a.rs < 0 ? -a.rs : a.rs));
  for (int64_t t = blockIdx.x; t < tiles; t += gridDim.x) {
    const int64_t b = t / (rt * ct);
    const int64_t rem = t - b * rt * ct;
    const int64_t r0 = (rem / ct) * 32, c0 = (rem % ct) * 128;
    const float *src = a.src + b * a.bs * (a.mode ? 2 : 1);
    if (c_fast) {
#pragma unroll
      for (int i = ty; i < 32; i += 8) {
        const int64_t r = r0 + i;
#pragma unroll
        for (int u = 0; u < 4; ++u) {
          const int cc = u * 32 + tx;
          const int64_t c = c0 + cc;
          tile[i][cc] = (r < a.rows && c < a.cols) ? split_load(a, src, r, c) : 0.f;
        }
      }
    } else {
      const int64_t r = r0 + tx;
#pragma unroll
      for (int u = 0; u < 16; ++u) {
        const int cc = u * 8 + ty;
        const int64_t c = c0 + cc;
        tile[tx][cc] = (r < a.rows && c < a.cols) ? split_load(a, src, r, c) : 0.f;
      }
    }
    __syncthreads();
    const int64_t c = c0 + 4 * tx;
    bool bad = false;
#pragma unroll
    for (int i = ty; i < 32; i += 8) {
      const int64_t r = r0 + i;
      if (r < a.rows && c < a.cols) {
        float hi[4], lo[4];
#pragma unroll
        for (int e = 0; e < 4; ++e) {
          const float x = tile[i][4 * tx + e];
          bad |= !isfinite(x);
          tf32_split(x, hi[e], lo[e]);
        }
        const int64_t o = (b * a.rows + r) * a.ld + c;
        if (c + 4 <= a.cols) {  // ld is a multiple of 4 floats and the parts are 256-byte aligned
          *reinterpret_cast<float4 *>(a.hi + o) = make_float4(hi[0], hi[1], hi[2], hi[3]);
          *reinterpret_cast<float4 *>(a.lo + o) = make_float4(lo[0], lo[1], lo[2], lo[3]);
        } else {
#pragma unroll
          for (int e = 0; e < 4; ++e)
            if (c + e < a.cols) { a.hi[o + e] = hi[e]; a.lo[o + e] = lo[e]; }
        }
      }
    }
    if (bad) *a.nonfinite = 1;
    __syncthreads();
  }
}

// ---------------------------------------------------------------------------
// Integer products on the 8-bit tensor cores: byte planes of 16/32/64-bit
// operands.  For one K chunk [k0, k0 + kc) of src (rows x K, element (r, k) at
// src[b*bs + r*rs + k*cs]), dst[b][r][seg(l)*kp + c] = byte l of src(r, k0 + c)
// (two's-complement bits, unsigned), zero for c >= kc, with seg(l) = l for A
// and L-1-l for B (its planes stacked in reverse).  A shared-memory tile makes
// the source read coalesced along whichever of r / k is contiguous and each
// plane row is written along k in 4-byte words (kp and ld are multiples of
// 16, the destination 256-byte aligned).  Block 32 x 8, grid-stride over tiles.
struct LimbArgs {
  const void *src;
  uint8_t *dst;
  int64_t rows, kc, k0;    // rows, K chunk length and start
  int64_t rs, cs, bs;      // source strides (elements)
  int64_t batch, kp, ld;   // batches; plane width (kc rounded up to 16); dst row pitch (L * kp)
  int planes, rev;
};

// Tiles of one operand's planes (32 rows x 128 columns of K each).
__host__ __device__ inline int64_t limb_tiles(const LimbArgs &a) {
  return a.batch * ((a.rows + 31) / 32) * ((a.kp + 127) / 128);
}

// Both operands in one launch: tiles [0, tiles(A)) are A's, the rest B's.
template <class S>
__global__ void __launch_bounds__(256) limb_split_kernel(const LimbArgs a0, const LimbArgs a1) {
  // 32 rows x 128 columns of K per tile; each thread then writes one 4-byte
  // word (4 consecutive k) per plane and row, 128 bytes per warp
  __shared__ S tile[32][129];
  const int tx = threadIdx.x, ty = threadIdx.y;
  const int64_t tiles0 = limb_tiles(a0), tiles = tiles0 + limb_tiles(a1);
  for (int64_t tt = blockIdx.x; tt < tiles; tt += gridDim.x) {
    const bool second = tt >= tiles0;
    const LimbArgs &a = second ? a1 : a0;
    const int64_t t = second ? tt - tiles0 : tt;
    const int64_t rt = (a.rows + 31) / 32, ct = (a.kp + 127) / 128;
    const bool c_fast = a.cs == 1 || (a.rs != 1 && (a.cs < 0 ? -a.cs : a.cs) <= (a.rs < 0 ? -a.rs : a.rs));
    const int64_t b = t / (rt * ct);
    const int64_t rem = t - b * rt * ct;
    const int64_t r0 = (rem / ct) * 32, c0 = (rem % ct) * 128;
    const S *src = (const S *)a.src + b * a.bs;
    if (c_fast) {
#pragma unroll
      for (int i = ty; i < 32; i += 8) {
        const int64_t r = r0 + i;
#pragma unroll
        for (int u = 0; u < 4; ++u) {
          const int cc = u * 32 + tx;
          const int64_t c = c0 + cc;
          tile[i][cc] = (r < a.rows && c < a.kc) ? src[r * a.rs + (a.k0 + c) * a.cs] : S(0);
        }
      }
    } else {
      const int64_t r = r0 + tx;
#pragma unroll
      for (int u = 0; u < 16; ++u) {
        const int cc = u * 8 + ty;
        const int64_t c = c0 + cc;
        tile[tx][cc] = (r < a.rows && c < a.kc) ? src[r * a.rs + (a.k0 + c) * a.cs] : S(0);
      }
    }
    __syncthreads();
    const int64_t c = c0 + 4 * tx;
#pragma unroll
    for (int i = ty; i < 32; i += 8) {
      const int64_t r = r0 + i;
      if (r < a.rows && c < a.kp) {
        using U = typename std::make_unsigned<S>::type;
        uint64_t v[4];
#pragma unroll
        for (int e = 0; e < 4; ++e) v[e] = (uint64_t)(U)tile[i][4 * tx + e];
        uint8_t *row = a.dst + (b * a.rows + r) * a.ld + c;
        for (int l = 0; l < a.planes; ++l) {
          const uint32_t word = (uint32_t)((v[0] >> (8 * l)) & 0xff) | (uint32_t)((v[1] >> (8 * l)) & 0xff) << 8 |
                                (uint32_t)((v[2] >> (8 * l)) & 0xff) << 16 | (uint32_t)((v[3] >> (8 * l)) & 0xff) << 24;
          *reinterpret_cast<uint32_t *>(row + (int64_t)(a.rev ? a.planes - 1 - l : l) * a.kp) = word;
        }
      }
    }
    __syncthreads();
  }
}

}  // namespace mb
