// tcgen05 / TMEM / TMA tensor-core GEMM for bf16, fp16, int8 and uint8.
//
// B200 replacement for the reference's Apple tensor-unit kernel
// mpp_tensor_gemm (metalblas/shaders/mpp_tensor.h:58-142: tiled GEMM, fp32
// accumulate, transposes via strides, batch via tgid.z + int4 strides, fused
// addmm epilogue in MB_STORE_TILE :38-55), of its split-K sibling
// (metalblas/shaders/splitk.h:21-82) and of the thin-M streaming kernel gemv_bt
// (metalblas/shaders/gemv_bt.h:47-269), which here is the same kernel run on
// Cᵀ = Bᵀ·Aᵀ so that the thin dimension becomes the UMMA N (16..64).
//
// Structure (one CTA per SM, persistent over work units):
//   warp 0      TMA producer: cp.async.bulk.tensor 3-D loads (no multicast)
//               into a STAGES-deep ring of 128B-swizzled shared-memory tiles,
//               completion tracked by mbarrier transaction counts.
//   warp 1      allocates TMEM, and one elected lane issues tcgen05.mma
//               (M=128, N=BN, K=16 for 16-bit / 32 for 8-bit) into one of two
//               TMEM accumulators, releasing each smem stage with
//               tcgen05.commit -> empty barrier.
//   warps 2..9  epilogue, two warps per TMEM lane quarter (each takes half of
//               the tile's columns): tcgen05.ld, alpha/beta/bias (mb_epi
//               semantics), convert, then either a 128B-swizzled staging tile in
//               shared memory written back by a TMA store (row-major outputs)
//               or direct stores (transposed / unaligned outputs).  For a
//               split-K unit the raw accumulators go to the workspace and the
//               last warp to draw a ticket for its slice reduces them in order.
// The two TMEM accumulators let the epilogue of tile i overlap the mainloop of
// tile i+1.
//
// Schedule: units are whole output tiles, except that when the tiles do not
// fill the last wave of the grid, the leftover tiles ("tail") are cut so the
// last wave is full as well: dp_tiles whole tiles first, then either
//  * half-width units (two per tail tile),
//  * fixed K splits ((tiles - dp_tiles) * splits split units), or
//  * stream-K: the tail's tiles x K-blocks iterations are divided into equal
//    contiguous ranges, one per CTA; a range is cut at tile boundaries into
//    pieces, and a tile's pieces (at most `splits`) are summed in K order by
//    the warp that draws the last ticket.  Every CTA does the same number of
//    K-blocks, whatever the tile count.
// Partials are stored lane-interleaved (a warp's 32 rows of 4 columns form one
// 512-byte run) so both the writes and the reduction are coalesced.  Thin tiles
// (BN <= 32) whose splits all fit in one wave run each tile's splits on the
// CTAs of one thread-block cluster instead (TcParams::csplit): the partials
// then travel through rank 0's shared memory, not the workspace.
//
// Operand layouts: each operand may be K-major or MN-major in global memory;
// TMA copies it into the matching canonical SWIZZLE_128B layout and the UMMA
// instruction descriptor's major bits say which.  Tile edges in M, N and K are
// zero-filled by TMA (out-of-bounds fill); TMA stores clip at the edges and the
// direct-store path masks.
//
// Every mbarrier wait is bounded by a %globaltimer deadline; a wait that runs
// out records MB_ERR_DEVICE_TIMEOUT in g_mb_status, raises a CTA-wide abort
// flag so every role leaves its loop, drains what it issued (bounded), frees
// TMEM and returns.  Nothing traps.
#pragma once
#include <cuda.h>
#include "mb_common.cuh"
#include <type_traits>

namespace mb {
namespace tc {

constexpr int BM = 128;                 // UMMA M (cta_group::1)
constexpr int kMaxPeers = 7;            // peer copies of C a replicating kernel writes (8 GPUs per node)
constexpr int NUM_EPI_WARPS = 8;
constexpr int NUM_THREADS = 64 + 32 * NUM_EPI_WARPS;
constexpr int SMEM_LIMIT = 232448;      // max dynamic shared memory per CTA on sm_100
constexpr int STAGING_ROW = 64;             // bytes per staged output row (SWIZZLE_64B)
constexpr int STAGING_BUF = 32 * STAGING_ROW;  // one 32-row box
constexpr int STAGING_PER_WARP = 2 * STAGING_BUF;  // double-buffered

struct TcParams {
  CUtensorMap tmA;   // UMMA-A operand (rows of C), 3-D {inner, outer, batch}
  CUtensorMap tmB;   // UMMA-B operand (cols of C)
  CUtensorMap tmA2;  // fp32 (3xTF32): the low tf32 parts of A and B, same geometry
  CUtensorMap tmB2;
  CUtensorMap tmC;   // output, 3-D {N, M, batch}, box {64 B, 32 rows}, SWIZZLE_64B; valid when c_tma
  int M, N, K, batch;
  int a_mn, b_mn;        // operand is MN-major in global memory
  int a_bcast, b_bcast;  // batch stride 0: always load batch 0
  int tiles_m, tiles_n, splits, kb_total, kb_per_split;
  int dp_tiles;          // tiles [0, dp_tiles) run whole; later ("tail") tiles are either
  int tail_half;         //   split into two half-width (BN/2) units (tail_half = 1) or
                         //   split along K `splits` ways (tail_half = 0)
  int num_units, group_m;
  void *C;
  int64_t c_rs, c_cs, sC;
  const void *bias;
  int64_t bias_rs, bias_cs, bias_bs;
  EpiScalars epi;
  int c_vec;             // c_cs == 1 and every row start is 16-byte aligned
  int c_tma;             // write C through tmC
  void *ws;              // split-K partials: tail_tiles * splits * PAIR * BM * BN * 4 bytes
  unsigned *tickets;     // NUM_EPI_WARPS per tail tile and CTA of a pair, zero on entry and exit
  int sk;                // tail tiles partitioned stream-K (splits = partial slots per tile)
  long long sk_iters;    // tail tiles * kb_total: the K-block iterations shared out
  unsigned long long timeout_ns;
  // Cluster split-K: the grid is one unit per CTA, every tile split `splits`
  // ways along K, and the CTAs of a cluster (cluster rank = split index) share
  // one tile: ranks 1.. store their partials into rank 0's shared memory
  // instead of the workspace, and rank 0 sums them in K order.
  int csplit;
  // Peer replication (kernels instantiated with PEER = true): every output
  // element is also stored, with plain st.global over NVLink, at the same
  // element offset from each peer_C[i] (another GPU's copy of C, mapped into
  // this process).  Loads and tensor maps only ever touch this GPU's memory.
  int npeers;
  void *peer_C[kMaxPeers];
  // NVSwitch multicast address of C (all ranks' copies at once), or null.
  // When set, whole 16-byte chunks go to every peer with one multimem.st
  // through it (the switch replicates the write); partial chunks still take
  // the per-peer stores.
  void *mc_C;
};

// One 16-byte store to every GPU bound to the multicast address `mc`.
__device__ __forceinline__ void multimem_st16(void *mc, const uint4 &v) {
  asm volatile("multimem.st.relaxed.sys.global.v4.f32 [%0], {%1, %2, %3, %4};" ::"l"(mc), "r"(v.x), "r"(v.y),
               "r"(v.z), "r"(v.w)
               : "memory");
}

template <int BN, int ESZ, int PAIR = 1>
struct Cfg {
  static constexpr int BK = 128 / ESZ;          // one 128-byte swizzle row of K
  static constexpr int UMMA_K = 32 / ESZ;       // K per tcgen05.mma
  static constexpr int KSTEPS = BK / UMMA_K;    // 4
  static constexpr int A_BYTES = BM * 128;
  static constexpr int B_BYTES = (BN / PAIR) * 128;  // this CTA's share of B's columns
  // fp32 runs as 3xTF32: each stage holds the high and the low tf32 parts of
  // both operands (A_hi, A_lo, B_hi, B_lo)
  static constexpr int NPART = ESZ == 4 ? 2 : 1;
  // K-blocks accumulated in TMEM before the epilogue takes the sum: the tensor
  // core's fp32 accumulation drifts over long chains, so fp32 (3xTF32) sums
  // chunks of 16 K-blocks (512 elements of K) in registers with IEEE adds.
  static constexpr int KCHUNK = ESZ == 4 ? 16 : (1 << 30);
  // fp32 running sums per epilogue thread (whole-width unit: BN/2 columns)
  static constexpr int RUN = ESZ == 4 ? BN / 2 : 1;
  static constexpr int STAGE_BYTES = NPART * (A_BYTES + B_BYTES);
  static constexpr int HALF = BN / 2;           // columns per epilogue warp (whole-tile unit)
  static constexpr int QUART = BN / 4;          // columns per epilogue warp (half-width unit)
  static constexpr int CC = STAGING_ROW / ESZ;  // columns per staged row
  static constexpr bool TMA_STORE = ESZ <= 2 && (QUART % CC) == 0;  // fp32 outputs: direct stores
  static constexpr int STAGING_BYTES = TMA_STORE ? NUM_EPI_WARPS * STAGING_PER_WARP : 0;
  static constexpr int BAR_BYTES = 256;
  // Cluster split-K (thin tiles): rank 0 of a cluster receives the raw
  // partials of ranks 1 .. CSPLIT_MAX-1 here, one BM x BN 4-byte slot each.
  static constexpr int CSPLIT_MAX = 4;
  static constexpr int RED_BYTES = (BN <= 32 && PAIR == 1 && ESZ <= 2) ? (CSPLIT_MAX - 1) * BM * BN * 4 : 0;
  static constexpr int STAGES_RAW = (SMEM_LIMIT - 1024 - STAGING_BYTES - RED_BYTES - BAR_BYTES) / STAGE_BYTES;
  static constexpr int STAGES = STAGES_RAW > 8 ? 8 : STAGES_RAW;
  // The 512-wide CTA-pair tile issues two N = 256 MMAs per K-step (tile
  // columns [0, 256) and [256, 512)); its accumulator fills all 512 TMEM
  // columns, so it has one accumulator instead of two.
  static constexpr int UMMA_N = BN > 256 ? 256 : BN;  // N per tcgen05.mma
  static constexpr int NMMA = BN / UMMA_N;            // MMAs per K-step
  static constexpr int NACC = 2 * BN <= 512 ? 2 : 1;  // TMEM accumulators (two: epilogue overlaps the next tile)
  static constexpr int ACC_COLS = BN;           // fp32/s32: one column per N
  static constexpr int TMEM_COLS = (NACC * BN <= 32) ? 32 : (NACC * BN <= 64) ? 64 : (NACC * BN <= 128) ? 128
                                 : (NACC * BN <= 256) ? 256 : 512;
  static constexpr int SMEM_BYTES = 1024 /*align slack*/ + STAGES * STAGE_BYTES + STAGING_BYTES + RED_BYTES + BAR_BYTES;
  // columns per tcgen05.ld on the direct-store and split-K paths (16 for 16- and
  // 32-bit outputs keeps the epilogue within the register budget of 320 threads)
  static constexpr int RCH = QUART < (ESZ >= 2 ? 16 : 32) ? (QUART < 8 ? 8 : QUART) : (ESZ >= 2 ? 16 : 32);
  static_assert(BN % 16 == 0 && BN >= 16 && (BN <= 256 || (BN == 512 && PAIR == 2 && ESZ <= 2)), "UMMA N");
  static_assert(STAGES >= 2, "need a pipeline");
  static_assert(SMEM_BYTES <= SMEM_LIMIT, "shared memory");
  static_assert(2 * STAGES + 6 + 1 <= BAR_BYTES / 8, "barrier area");
};

// ---------------------------------------------------------------------------
// PTX wrappers
__device__ __forceinline__ uint32_t smem_u32(const void *p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}
__device__ __forceinline__ void mbar_init(uint32_t bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(bar), "r"(count) : "memory");
}
__device__ __forceinline__ void fence_mbar_init() {
  asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}
__device__ __forceinline__ void mbar_arrive_expect_tx(uint32_t bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(bar), "r"(bytes) : "memory");
}
__device__ __forceinline__ void mbar_arrive(uint32_t bar) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(bar) : "memory");
}
__device__ __forceinline__ bool mbar_try_wait(uint32_t bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(ok)
      : "r"(bar), "r"(parity)
      : "memory");
  return ok != 0;
}
// Bounded wait: true when the phase with `parity` completed; false on abort
// (another role gave up) or deadline (this one gives up and raises abort).
__device__ __forceinline__ bool mbar_wait(uint32_t bar, uint32_t parity, volatile int *abort_flag,
                                          unsigned long long timeout_ns) {
  if (mbar_try_wait(bar, parity)) return true;
  const uint64_t t0 = globaltimer_ns();
  for (uint32_t it = 1;; ++it) {
    if (mbar_try_wait(bar, parity)) return true;
    if ((it & 63) == 0) {
      if (*abort_flag) return false;
      if (globaltimer_ns() - t0 > timeout_ns) {
        *abort_flag = 1;
        atomicExch(&g_mb_status, 4 /*MB_ERR_DEVICE_TIMEOUT*/);
        return false;
      }
    }
  }
}

__device__ __forceinline__ void tma_load_3d(uint32_t dst, const CUtensorMap *map, uint32_t bar, int c0, int c1,
                                            int c2) {
  asm volatile(
      "cp.async.bulk.tensor.3d.shared::cluster.global.tile.mbarrier::complete_tx::bytes"
      " [%0], [%1, {%3, %4, %5}], [%2];" ::"r"(dst),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(bar), "r"(c0), "r"(c1), "r"(c2)
      : "memory");
}
// CTA-pair form: the copy lands in this CTA's shared memory and its bytes are
// counted on `bar_cluster`, the pair leader's barrier (cluster address).  No
// multicast: each CTA fetches its own tiles.
__device__ __forceinline__ void tma_load_3d_pair(uint32_t dst, const CUtensorMap *map, uint32_t bar_cluster, int c0,
                                                 int c1, int c2) {
  asm volatile(
      "cp.async.bulk.tensor.3d.cta_group::2.shared::cluster.global.tile.mbarrier::complete_tx::bytes"
      " [%0], [%1, {%3, %4, %5}], [%2];" ::"r"(dst),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(bar_cluster), "r"(c0), "r"(c1), "r"(c2)
      : "memory");
}
__device__ __forceinline__ void prefetch_tmap(const CUtensorMap *map) {
  asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(map)) : "memory");
}

__device__ __forceinline__ void tmem_alloc(uint32_t dst_smem, uint32_t ncols) {
  asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(dst_smem), "r"(ncols)
               : "memory");
}
__device__ __forceinline__ void tmem_relinquish() {
  asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
}
__device__ __forceinline__ void tmem_dealloc(uint32_t taddr, uint32_t ncols) {
  asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(taddr), "r"(ncols) : "memory");
}
__device__ __forceinline__ void tc_fence_before() { asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory"); }
__device__ __forceinline__ void tc_fence_after() { asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory"); }

template <int ESZ>
__device__ __forceinline__ void umma(uint32_t d_tmem, uint64_t adesc, uint64_t bdesc, uint32_t idesc, uint32_t accum) {
  if constexpr (ESZ == 4) {
    asm volatile(
        "{\n\t.reg .pred p;\n\tsetp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::1.kind::tf32 [%0], %1, %2, %3, p;\n\t}" ::"r"(d_tmem),
        "l"(adesc), "l"(bdesc), "r"(idesc), "r"(accum)
        : "memory");
  } else if constexpr (ESZ == 2) {
    asm volatile(
        "{\n\t.reg .pred p;\n\tsetp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n\t}" ::"r"(d_tmem),
        "l"(adesc), "l"(bdesc), "r"(idesc), "r"(accum)
        : "memory");
  } else {
    asm volatile(
        "{\n\t.reg .pred p;\n\tsetp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::1.kind::i8 [%0], %1, %2, %3, p;\n\t}" ::"r"(d_tmem),
        "l"(adesc), "l"(bdesc), "r"(idesc), "r"(accum)
        : "memory");
  }
}
__device__ __forceinline__ void umma_commit(uint32_t bar) {
  asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(bar) : "memory");
}

// 32 lanes x 32 consecutive 32-bit TMEM columns -> 32 registers per thread.
__device__ __forceinline__ void tmem_ld_x32(uint32_t taddr, uint32_t (&r)[32]) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x32.b32 "
      "{%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,"
      "%16,%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31}, [%32];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
        "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15]),
        "=r"(r[16]), "=r"(r[17]), "=r"(r[18]), "=r"(r[19]), "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]),
        "=r"(r[24]), "=r"(r[25]), "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]), "=r"(r[30]), "=r"(r[31])
      : "r"(taddr));
}
__device__ __forceinline__ void tmem_ld_x16(uint32_t taddr, uint32_t (&r)[32]) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x16.b32 "
      "{%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15}, [%16];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
        "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15])
      : "r"(taddr));
}
// ---- CTA-pair (cluster of 2) helpers
__device__ __forceinline__ uint32_t cluster_rank() {
  uint32_t r;
  asm volatile("mov.u32 %0, %%cluster_ctarank;" : "=r"(r));
  return r;
}
// Address of the same shared-memory offset in CTA `rank` of the cluster.
__device__ __forceinline__ uint32_t mapa_shared(uint32_t addr, uint32_t rank) {
  uint32_t r;
  asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(r) : "r"(addr), "r"(rank));
  return r;
}
__device__ __forceinline__ void mbar_arrive_cluster(uint32_t cluster_addr) {
  asm volatile("mbarrier.arrive.release.cluster.shared::cluster.b64 _, [%0];" ::"r"(cluster_addr) : "memory");
}
__device__ __forceinline__ bool mbar_try_wait_cluster(uint32_t bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.try_wait.parity.acquire.cluster.shared::cta.b64 p, [%1], %2;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(ok)
      : "r"(bar), "r"(parity)
      : "memory");
  return ok != 0;
}
// Bounded wait on a barrier that receives arrivals from the peer CTA.
__device__ __forceinline__ bool mbar_wait_cluster(uint32_t bar, uint32_t parity, volatile int *abort_flag,
                                                  unsigned long long timeout_ns) {
  if (mbar_try_wait_cluster(bar, parity)) return true;
  const uint64_t t0 = globaltimer_ns();
  for (uint32_t it = 1;; ++it) {
    if (mbar_try_wait_cluster(bar, parity)) return true;
    if ((it & 63) == 0) {
      if (*abort_flag) return false;
      if (globaltimer_ns() - t0 > timeout_ns) {
        *abort_flag = 1;
        atomicExch(&g_mb_status, 4 /*MB_ERR_DEVICE_TIMEOUT*/);
        return false;
      }
    }
  }
}
// 16-byte store to shared memory of another CTA of the cluster (a mapa address).
__device__ __forceinline__ void st_cluster_v4(uint32_t addr, uint32_t a, uint32_t b, uint32_t c, uint32_t d) {
  asm volatile("st.shared::cluster.v4.u32 [%0], {%1, %2, %3, %4};" ::"r"(addr), "r"(a), "r"(b), "r"(c), "r"(d)
               : "memory");
}
__device__ __forceinline__ uint4 ld_shared_v4(uint32_t addr) {
  uint4 v;
  asm volatile("ld.shared.v4.u32 {%0, %1, %2, %3}, [%4];" : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w) : "r"(addr)
               : "memory");
  return v;
}
__device__ __forceinline__ void cluster_sync_all() {
  asm volatile("barrier.cluster.arrive.release.aligned;\n\tbarrier.cluster.wait.acquire.aligned;" ::: "memory");
}
template <int PAIR>
__device__ __forceinline__ void tmem_alloc_g(uint32_t dst_smem, uint32_t ncols) {
  if constexpr (PAIR == 2)
    asm volatile("tcgen05.alloc.cta_group::2.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(dst_smem), "r"(ncols)
                 : "memory");
  else
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(dst_smem), "r"(ncols)
                 : "memory");
}
template <int PAIR>
__device__ __forceinline__ void tmem_relinquish_g() {
  if constexpr (PAIR == 2) asm volatile("tcgen05.relinquish_alloc_permit.cta_group::2.sync.aligned;" ::: "memory");
  else asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
}
template <int PAIR>
__device__ __forceinline__ void tmem_dealloc_g(uint32_t taddr, uint32_t ncols) {
  if constexpr (PAIR == 2)
    asm volatile("tcgen05.dealloc.cta_group::2.sync.aligned.b32 %0, %1;" ::"r"(taddr), "r"(ncols) : "memory");
  else
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(taddr), "r"(ncols) : "memory");
}
// MMA issue: cta_group::2 runs one M=256 instruction over the CTA pair (each CTA
// supplies 128 rows of A and half of B's columns, and holds its 128 rows of D).
template <int ESZ, int PAIR>
__device__ __forceinline__ void umma_g(uint32_t d_tmem, uint64_t adesc, uint64_t bdesc, uint32_t idesc,
                                       uint32_t accum) {
  if constexpr (PAIR == 1) {
    umma<ESZ>(d_tmem, adesc, bdesc, idesc, accum);
  } else if constexpr (ESZ == 4) {
    asm volatile(
        "{\n\t.reg .pred p;\n\tsetp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::2.kind::tf32 [%0], %1, %2, %3, p;\n\t}" ::"r"(d_tmem),
        "l"(adesc), "l"(bdesc), "r"(idesc), "r"(accum)
        : "memory");
  } else if constexpr (ESZ == 2) {
    asm volatile(
        "{\n\t.reg .pred p;\n\tsetp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::2.kind::f16 [%0], %1, %2, %3, p;\n\t}" ::"r"(d_tmem),
        "l"(adesc), "l"(bdesc), "r"(idesc), "r"(accum)
        : "memory");
  } else {
    asm volatile(
        "{\n\t.reg .pred p;\n\tsetp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::2.kind::i8 [%0], %1, %2, %3, p;\n\t}" ::"r"(d_tmem),
        "l"(adesc), "l"(bdesc), "r"(idesc), "r"(accum)
        : "memory");
  }
}
// Commit: arrive once on the barrier at this offset in every CTA of the pair
// (tcgen05.commit with multicast; the loads themselves never multicast).
template <int PAIR>
__device__ __forceinline__ void umma_commit_g(uint32_t bar) {
  if constexpr (PAIR == 1) {
    umma_commit(bar);
  } else {
    asm volatile(
        "{\n\t.reg .b16 m;\n\tmov.b16 m, 3;\n\t"
        "tcgen05.commit.cta_group::2.mbarrier::arrive::one.shared::cluster.multicast::cluster.b64 [%0], m;\n\t}" ::"r"(
            bar)
        : "memory");
  }
}
// Commit to this CTA's barrier only (drain on abort).
template <int PAIR>
__device__ __forceinline__ void umma_commit_self(uint32_t bar) {
  if constexpr (PAIR == 1) {
    umma_commit(bar);
  } else {
    asm volatile(
        "{\n\t.reg .b16 m;\n\tmov.b16 m, 1;\n\t"
        "tcgen05.commit.cta_group::2.mbarrier::arrive::one.shared::cluster.multicast::cluster.b64 [%0], m;\n\t}" ::"r"(
            bar)
        : "memory");
  }
}

__device__ __forceinline__ void tmem_ld_x8(uint32_t taddr, uint32_t (&r)[32]) {
  asm volatile("tcgen05.ld.sync.aligned.32x32b.x8.b32 {%0,%1,%2,%3,%4,%5,%6,%7}, [%8];"
               : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7])
               : "r"(taddr));
}
template <int N>
__device__ __forceinline__ void tmem_ld(uint32_t taddr, uint32_t (&r)[32]) {
  if constexpr (N == 32) tmem_ld_x32(taddr, r);
  else if constexpr (N == 16) tmem_ld_x16(taddr, r);
  else tmem_ld_x8(taddr, r);
}
// TMA store of a shared-memory box to global (bulk async-group completion).
__device__ __forceinline__ void tma_store_3d(const CUtensorMap *map, uint32_t src, int c0, int c1, int c2) {
  asm volatile(
      "cp.async.bulk.tensor.3d.global.shared::cta.tile.bulk_group [%0, {%2, %3, %4}], [%1];" ::"l"(
          reinterpret_cast<uint64_t>(map)),
      "r"(src), "r"(c0), "r"(c1), "r"(c2)
      : "memory");
}
__device__ __forceinline__ void bulk_commit() { asm volatile("cp.async.bulk.commit_group;" ::: "memory"); }
// The source shared memory of every committed bulk store may be reused.
__device__ __forceinline__ void bulk_wait_read0() { asm volatile("cp.async.bulk.wait_group.read 0;" ::: "memory"); }
// Every committed bulk store has completed.
__device__ __forceinline__ void bulk_wait0() { asm volatile("cp.async.bulk.wait_group 0;" ::: "memory"); }
// Generic-proxy shared-memory writes become visible to the async (TMA) proxy.
__device__ __forceinline__ void fence_proxy_async_smem() {
  asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}
__device__ __forceinline__ void tmem_wait_ld() { asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory"); }

// Shared-memory matrix descriptor, SWIZZLE_128B, sm100 version bits.
__device__ __forceinline__ uint64_t sdesc(uint32_t saddr, uint32_t lbo, uint32_t sbo) {
  uint64_t d = 0;
  d |= (uint64_t)((saddr >> 4) & 0x3FFFu);
  d |= (uint64_t)((lbo >> 4) & 0x3FFFu) << 16;
  d |= (uint64_t)((sbo >> 4) & 0x3FFFu) << 32;
  d |= (uint64_t)1 << 46;
  d |= (uint64_t)2 << 61;
  return d;
}

// Instruction descriptor: D f32 (f16 kind) or s32 (i8 kind), operand formats,
// major-ness, N>>3 at bit 17, M>>4 at bit 24.
template <class T> struct UFmt;
template <> struct UFmt<__half> { static constexpr uint32_t d = 1, ab = 0; };
template <> struct UFmt<__nv_bfloat16> { static constexpr uint32_t d = 1, ab = 1; };
template <> struct UFmt<uint8_t> { static constexpr uint32_t d = 2, ab = 0; };
template <> struct UFmt<int8_t> { static constexpr uint32_t d = 2, ab = 1; };
template <> struct UFmt<float> { static constexpr uint32_t d = 1, ab = 2; };  // tf32 operands, f32 accumulator

template <class T, int BN, int UM = BM>
__device__ __forceinline__ uint32_t make_idesc(int a_mn, int b_mn) {
  return (UFmt<T>::d << 4) | (UFmt<T>::ab << 7) | (UFmt<T>::ab << 10) | ((uint32_t)a_mn << 15) |
         ((uint32_t)b_mn << 16) | ((uint32_t)(BN >> 3) << 17) | ((uint32_t)(UM >> 4) << 24);
}

struct Unit {
  int b, tm, tn;
  int tile;          // raster index over all output tiles
  int s;             // split / piece index (0 unless a K-split unit)
  int nparts;        // partial sums of this tile (split units)
  int kb0, kb1;      // K-blocks of this unit
  bool split;        // partial-sum unit (tail tile split along K)
  int half;          // -1: whole tile; 0/1: which half-width (BN/2 columns) of the tile
  int tail;          // tile - dp_tiles (valid for tail units)
};
__device__ __forceinline__ void tile_coords(const TcParams &p, Unit &r);
__device__ __forceinline__ Unit decode_unit(const TcParams &p, int u) {
  Unit r;
  r.s = 0; r.split = false; r.half = -1; r.tail = 0; r.nparts = 1;
  r.kb0 = 0; r.kb1 = p.kb_total;
  if (u < p.dp_tiles) {
    r.tile = u;
  } else if (p.tail_half) {
    const int v = u - p.dp_tiles;
    r.tail = v >> 1;
    r.tile = p.dp_tiles + r.tail;
    r.half = v & 1;
  } else {
    const int v = u - p.dp_tiles;
    r.tail = v / p.splits;
    r.tile = p.dp_tiles + r.tail;
    r.s = v % p.splits;
    r.split = true;
    r.nparts = p.splits;
    r.kb0 = r.s * p.kb_per_split;
    r.kb1 = min(p.kb_total, r.kb0 + p.kb_per_split);
  }
  tile_coords(p, r);
  return r;
}
// (batch, tile row, tile column) of r.tile: grouped raster, group_m tile rows
// per group so that concurrently running tiles share A and B panels in L2.
__device__ __forceinline__ void tile_coords(const TcParams &p, Unit &r) {
  const int per_batch = p.tiles_m * p.tiles_n;
  r.b = r.tile / per_batch;
  const int q = r.tile % per_batch;
  const int per_group = p.group_m * p.tiles_n;
  const int g = q / per_group;
  const int first_m = g * p.group_m;
  const int gsz = min(p.tiles_m - first_m, p.group_m);
  const int w = q % per_group;
  r.tm = first_m + w % gsz;
  r.tn = w / gsz;
}

// The stream-K CTA that owns iteration i of the tail (ranges [g*I/G, (g+1)*I/G)).
__device__ __forceinline__ long long sk_owner(long long i, long long I, int G) {
  return ((i + 1) * (long long)G - 1) / I;
}

// The sequence of units one CTA (or CTA pair) works through; every role of the
// CTA walks the same sequence.
struct UnitIter {
  int u;                // next strided unit
  long long i, iend;    // remaining stream-K range
};
__device__ __forceinline__ UnitIter unit_iter(const TcParams &p, int id, int n) {
  UnitIter it;
  it.u = id;
  it.i = it.iend = 0;
  if (p.sk) {
    it.i = (long long)id * p.sk_iters / n;
    it.iend = (long long)(id + 1) * p.sk_iters / n;
  }
  return it;
}
__device__ __forceinline__ bool unit_next(const TcParams &p, UnitIter &it, int n, Unit &r) {
  if (it.u < p.num_units) {
    r = decode_unit(p, it.u);
    it.u += n;
    return true;
  }
  if (it.i >= it.iend) return false;
  const long long KB = p.kb_total;
  const int tail = (int)(it.i / KB);
  const long long t0 = (long long)tail * KB, t1 = t0 + KB;
  const long long end = min(it.iend, t1);
  r.tail = tail;
  r.tile = p.dp_tiles + tail;
  r.half = -1;
  r.kb0 = (int)(it.i - t0);
  r.kb1 = (int)(end - t0);
  const long long first = sk_owner(t0, p.sk_iters, n);
  r.s = (int)(sk_owner(it.i, p.sk_iters, n) - first);
  r.nparts = (int)(sk_owner(t1 - 1, p.sk_iters, n) - first) + 1;
  r.split = r.nparts > 1;
  it.i = end;
  tile_coords(p, r);
  return true;
}

template <class T>
__device__ __forceinline__ typename Elem<T>::acc acc_from_bits(uint32_t bits) {
  if constexpr (Elem<T>::is_int) return bits;
  else return __uint_as_float(bits);
}

// Epilogue value of C(m, n) from its raw accumulator bits.
template <class T>
__device__ __forceinline__ T epi_value(const TcParams &p, int b, int m, int n, uint32_t bits) {
  typename Elem<T>::acc v = acc_from_bits<T>(bits);
  if (p.epi.enabled && m < p.M && n < p.N) {
    const T *bias = (const T *)p.bias + (int64_t)b * p.bias_bs;
    v = EpiOps<T>::apply(v, bias + (int64_t)m * p.bias_rs + (int64_t)n * p.bias_cs, p.epi);
  }
  return Elem<T>::store(v);
}

// complex32 epilogue on one interleaved pair: real columns (n, n+1) of C' are
// (re, im) of complex C(m, n/2); bias is complex32 with complex strides.
__device__ __forceinline__ void epi_cplx_pair(const TcParams &p, int b, int m, int n, uint32_t re_bits,
                                              uint32_t im_bits, __half &o_re, __half &o_im) {
  const float re = __uint_as_float(re_bits), im = __uint_as_float(im_bits);
  float vr = 0.f, vi = 0.f;
  if (p.epi.alpha_nz) {
    vr = p.epi.alpha_re * re - p.epi.alpha_im * im;
    vi = p.epi.alpha_re * im + p.epi.alpha_im * re;
  }
  if (p.epi.beta_nz && m < p.M && n < p.N) {
    const __half2 *bias = (const __half2 *)p.bias + (int64_t)b * p.bias_bs + (int64_t)m * p.bias_rs +
                          (int64_t)(n >> 1) * p.bias_cs;
    const float2 bv = __half22float2(*bias);
    vr += p.epi.beta_re * bv.x - p.epi.beta_im * bv.y;
    vi += p.epi.beta_re * bv.y + p.epi.beta_im * bv.x;
  }
  o_re = __float2half_rn(vr);
  o_im = __float2half_rn(vi);
}

// Epilogue values of NC consecutive columns n0.. of one row (real or complex pairs).
template <class T, int NC>
__device__ __forceinline__ void epi_values(const TcParams &p, int b, int m, int n0, const uint32_t (&r)[32],
                                           T (&out)[NC]) {
  if constexpr (std::is_same_v<T, __half>) {
    if (p.epi.cplx) {
#pragma unroll
      for (int j = 0; j < NC; j += 2) epi_cplx_pair(p, b, m, n0 + j, r[j], r[j + 1], out[j], out[j + 1]);
      return;
    }
  }
#pragma unroll
  for (int j = 0; j < NC; ++j) out[j] = epi_value<T>(p, b, m, n0 + j, r[j]);
}

// Real epilogue on NC (<= 32) consecutive columns n0.. of row m, in place: the
// raw accumulator bits in v become the bits of alpha * acc + beta * bias in the
// accumulator type (fp32 or wrapping u32), mb_epi semantics.  The row's bias values are fetched with
// 16-byte vector loads when they are contiguous and aligned (the usual bias[N]
// broadcast of addmm, or a row-major bias matrix), else one load per element.
template <class T, int NC>
__device__ __forceinline__ void epi_real(const TcParams &p, int b, int m, int n0, uint32_t (&v)[32]) {
  using E = Elem<T>;
  using Acc = typename E::acc;
  constexpr int BYTES = NC * (int)sizeof(T);
  constexpr int NQ = BYTES / 16 > 0 ? BYTES / 16 : 1;
  union { uint4 q[NQ]; T t[NQ * 16 / sizeof(T)]; } u;  // the bias values, packed
  const bool use_bias = p.epi.beta_nz && m < p.M;
  if (use_bias) {
    const T *row = (const T *)p.bias + (int64_t)b * p.bias_bs + (int64_t)m * p.bias_rs;
    if (BYTES % 16 == 0 && p.bias_cs == 1 && n0 + NC <= p.N && (reinterpret_cast<uintptr_t>(row + n0) & 15) == 0) {
#pragma unroll
      for (int i = 0; i < NQ; ++i) u.q[i] = __ldg(reinterpret_cast<const uint4 *>(row + n0) + i);
    } else {
#pragma unroll
      for (int j = 0; j < NC; ++j) u.t[j] = (n0 + j < p.N) ? row[(int64_t)(n0 + j) * p.bias_cs] : T();
    }
  }
#pragma unroll
  for (int j = 0; j < NC; ++j) {
    if constexpr (E::is_int) {
      Acc x = p.epi.alpha_nz ? (Acc)p.epi.ialpha * v[j] : Acc(0);
      if (use_bias) x += (Acc)p.epi.ibeta * E::load(u.t[j], false);
      v[j] = x;
    } else {
      float x = p.epi.alpha_nz ? p.epi.alpha_re * __uint_as_float(v[j]) : 0.f;
      if (use_bias) x = fmaf(p.epi.beta_re, E::load(u.t[j], false), x);
      v[j] = __float_as_uint(x);
    }
  }
}

// Write NC consecutive output values of row m (columns n0..) to a copy of C at
// `base` (C's strides): 16-byte stores when the row run is aligned and whole,
// else one store per element.
template <class T, int NC>
__device__ __forceinline__ void put_row_chunk(const TcParams &p, T *base, int b, int m, int n0, const T (&out)[NC]) {
  T *C = base + (int64_t)b * p.sC;
  constexpr int PER16 = 16 / sizeof(T);
  if (NC % PER16 == 0 && p.c_vec && n0 + NC <= p.N) {
    uint4 *dst = reinterpret_cast<uint4 *>(C + (int64_t)m * p.c_rs + n0);
#pragma unroll
    for (int v = 0; v < NC / PER16; ++v) dst[v] = *reinterpret_cast<const uint4 *>(&out[v * PER16]);
  } else {
#pragma unroll
    for (int j = 0; j < NC; ++j)
      if (n0 + j < p.N) C[(int64_t)m * p.c_rs + (int64_t)(n0 + j) * p.c_cs] = out[j];
  }
}

// Direct stores of NC (<= 32) consecutive columns of one output row (r is
// consumed: the epilogue is applied to it in place).  PEER: the same values
// also go to every peer copy of C.
template <class T, int NC, bool PEER = false>
__device__ __forceinline__ void store_row_chunk(const TcParams &p, int b, int m, int n0, uint32_t (&r)[32]) {
  T out[NC];
  bool cplx = false;
  if constexpr (std::is_same_v<T, __half>) cplx = p.epi.cplx != 0;
  if constexpr (Elem<T>::is_int && sizeof(T) == 8) {
    // 64-bit integer output of an 8-bit product (integer limbs): the s32
    // accumulator sign-extends, then alpha*acc + beta*bias wraps modulo 2^64
    const bool use_bias = p.epi.enabled && p.epi.beta_nz && m < p.M;
    const T *brow = (const T *)p.bias + (int64_t)b * p.bias_bs + (int64_t)m * p.bias_rs;
#pragma unroll
    for (int j = 0; j < NC; ++j) {
      const uint64_t acc = (uint64_t)(int64_t)(int32_t)r[j];
      uint64_t x = !p.epi.enabled ? acc : (p.epi.alpha_nz ? (uint64_t)p.epi.ialpha * acc : 0ull);
      if (use_bias && n0 + j < p.N) x += (uint64_t)p.epi.ibeta * (uint64_t)brow[(int64_t)(n0 + j) * p.bias_cs];
      out[j] = (T)x;
    }
  } else if (p.epi.enabled && !cplx) {
    epi_real<T, NC>(p, b, m, n0, r);
#pragma unroll
    for (int j = 0; j < NC; ++j) out[j] = Elem<T>::store(acc_from_bits<T>(r[j]));
  } else {
    epi_values<T, NC>(p, b, m, n0, r, out);
  }
  put_row_chunk<T, NC>(p, (T *)p.C, b, m, n0, out);
  if constexpr (PEER) {
    constexpr int PER16 = 16 / sizeof(T);
    if (p.mc_C && NC % PER16 == 0 && p.c_vec && n0 + NC <= p.N) {
      T *dst = (T *)p.mc_C + (int64_t)b * p.sC + (int64_t)m * p.c_rs + n0;
#pragma unroll
      for (int v = 0; v < NC / PER16; ++v)
        multimem_st16(dst + v * PER16, *reinterpret_cast<const uint4 *>(&out[v * PER16]));
    } else {
#pragma unroll 1
      for (int i = 0; i < p.npeers; ++i) put_row_chunk<T, NC>(p, (T *)p.peer_C[i], b, m, n0, out);
    }
  }
}

// Peer copies of one staged 32-row x 64-byte output box (the SWIZZLE_64B
// staging layout of the TMA-store epilogue: 16-byte chunk c of row r at chunk
// c ^ ((r >> 1) & 3)).  Lane l moves chunk l & 3 of rows l / 4, l / 4 + 8, ...,
// so each warp-wide store writes eight whole 64-byte row runs.  Rows past M and
// columns past N are skipped, as the TMA store clips them.
template <class T>
__device__ __forceinline__ void peer_store_box(const TcParams &p, uint32_t stg, int lane, int b, int row0, int col0) {
  constexpr int EPC = 16 / (int)sizeof(T);   // elements per 16-byte chunk
  const int rr = lane >> 2, ch = lane & 3;
  const int n = col0 + ch * EPC;
  if (n >= p.N) return;
  uint4 v[4];
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const int r = i * 8 + rr;
    const uint32_t addr = stg + (uint32_t)(r * STAGING_ROW) + ((uint32_t)(ch ^ ((r >> 1) & 3)) << 4);
    asm volatile("ld.shared.v4.b32 {%0, %1, %2, %3}, [%4];"
                 : "=r"(v[i].x), "=r"(v[i].y), "=r"(v[i].z), "=r"(v[i].w)
                 : "r"(addr));
  }
  const bool whole = n + EPC <= p.N;
  if (whole && p.mc_C) {
    T *C = (T *)p.mc_C + (int64_t)b * p.sC;
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const int m = row0 + i * 8 + rr;
      if (m < p.M) multimem_st16(C + (int64_t)m * p.c_rs + n, v[i]);
    }
    return;
  }
#pragma unroll 1
  for (int pi = 0; pi < p.npeers; ++pi) {
    T *C = (T *)p.peer_C[pi] + (int64_t)b * p.sC;
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const int m = row0 + i * 8 + rr;
      if (m >= p.M) break;
      T *dst = C + (int64_t)m * p.c_rs + n;
      if (whole) {
        *reinterpret_cast<uint4 *>(dst) = v[i];
      } else {
        const T *e = reinterpret_cast<const T *>(&v[i]);
#pragma unroll
        for (int j = 0; j < EPC; ++j)
          if (n + j < p.N) dst[j] = e[j];
      }
    }
  }
}

// Convert 32 raw accumulators of C(m, n0..n0+31) to packed output words
// (32 * sizeof(T) / 4 words).  The plain product (no epilogue) is branch-free:
// pairs of fp32 round with one cvt to bf16x2 / f16x2, 8-bit outputs keep the
// low byte of each s32 (two's-complement wrap) via byte permutes.
template <class T>
__device__ __forceinline__ void pack_bits32(const uint32_t (&r)[32], uint32_t (&pk)[32 * sizeof(T) / 4]) {
  if constexpr (sizeof(T) == 2) {
#pragma unroll
    for (int j = 0; j < 16; ++j) {
      if constexpr (std::is_same_v<T, __nv_bfloat16>) {
        __nv_bfloat162 h = __floats2bfloat162_rn(__uint_as_float(r[2 * j]), __uint_as_float(r[2 * j + 1]));
        pk[j] = *reinterpret_cast<uint32_t *>(&h);
      } else {
        __half2 h = __floats2half2_rn(__uint_as_float(r[2 * j]), __uint_as_float(r[2 * j + 1]));
        pk[j] = *reinterpret_cast<uint32_t *>(&h);
      }
    }
  } else {
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      const uint32_t lo = __byte_perm(r[4 * j], r[4 * j + 1], 0x0040);
      const uint32_t hi = __byte_perm(r[4 * j + 2], r[4 * j + 3], 0x0040);
      pk[j] = __byte_perm(lo, hi, 0x5410);
    }
  }
}

// (r is consumed: the epilogue is applied to it in place.)
template <class T>
__device__ __forceinline__ void pack32(const TcParams &p, int b, int m, int n0, uint32_t (&r)[32],
                                       uint32_t (&pk)[32 * sizeof(T) / 4]) {
  if (!p.epi.enabled) {
    pack_bits32<T>(r, pk);
    return;
  }
  bool cplx = false;
  if constexpr (std::is_same_v<T, __half>) cplx = p.epi.cplx != 0;
  if (!cplx) {
    epi_real<T, 32>(p, b, m, n0, r);
    pack_bits32<T>(r, pk);
    return;
  }
  T out[32];
  epi_values<T, 32>(p, b, m, n0, r, out);
#pragma unroll
  for (int j = 0; j < 32 * (int)sizeof(T) / 4; ++j) pk[j] = reinterpret_cast<const uint32_t *>(out)[j];
}

// Peer copies of two consecutive staged boxes (the previous box `stg_a`, then
// `stg_b`, CC columns each, adjacent in C): each row is one 128-byte run, so
// lane l moves chunk l & 7 of rows l / 8, l / 8 + 4, ...: a warp-wide store
// writes four whole 128-byte lines (the single-box copy writes 64-byte halves,
// twice the store requests per byte, and remote stores are bound by requests).
template <class T>
__device__ __forceinline__ void peer_store_box2(const TcParams &p, uint32_t stg_a, uint32_t stg_b, int lane, int b,
                                                int row0, int col0) {
  constexpr int EPC = 16 / (int)sizeof(T);   // elements per 16-byte chunk
  const int rr = lane >> 3, ch = lane & 7;
  const int n = col0 + ch * EPC;
  if (n >= p.N) return;
  const uint32_t buf = ch < 4 ? stg_a : stg_b;
  uint4 v[8];
#pragma unroll
  for (int i = 0; i < 8; ++i) {
    const int r = i * 4 + rr;
    const uint32_t addr = buf + (uint32_t)(r * STAGING_ROW) + ((uint32_t)((ch & 3) ^ ((r >> 1) & 3)) << 4);
    asm volatile("ld.shared.v4.b32 {%0, %1, %2, %3}, [%4];"
                 : "=r"(v[i].x), "=r"(v[i].y), "=r"(v[i].z), "=r"(v[i].w)
                 : "r"(addr));
  }
  const bool whole = n + EPC <= p.N;
  if (whole && p.mc_C) {
    T *C = (T *)p.mc_C + (int64_t)b * p.sC;
#pragma unroll
    for (int i = 0; i < 8; ++i) {
      const int m = row0 + i * 4 + rr;
      if (m < p.M) multimem_st16(C + (int64_t)m * p.c_rs + n, v[i]);
    }
    return;
  }
#pragma unroll 1
  for (int pi = 0; pi < p.npeers; ++pi) {
    T *C = (T *)p.peer_C[pi] + (int64_t)b * p.sC;
#pragma unroll
    for (int i = 0; i < 8; ++i) {
      const int m = row0 + i * 4 + rr;
      if (m >= p.M) break;
      T *dst = C + (int64_t)m * p.c_rs + n;
      if (whole) {
        *reinterpret_cast<uint4 *>(dst) = v[i];
      } else {
        const T *e = reinterpret_cast<const T *>(&v[i]);
#pragma unroll
        for (int j = 0; j < EPC; ++j)
          if (n + j < p.N) dst[j] = e[j];
      }
    }
  }
}

// Partial-sum slot of piece s of tail tile `tail` for CTA `rank` of its pair:
// slots are BM x BN 4-byte values, ordered (tail, piece, rank).  A CTA pair
// shares a 256-row tile, and each CTA publishes and reduces its own 128 rows.
template <int PAIR>
__device__ __forceinline__ int64_t slot_of(const TcParams &p, int tail, int s, int rank) {
  return ((int64_t)tail * p.splits + s) * PAIR + rank;
}

// Split-K / stream-K epilogue after a warp published its partial: take a ticket
// for (tail tile, warp); the warp that draws the last one sums every partial of
// its 32 rows x wcols columns in K order and stores the result.
template <class T, int BN, int RCH, bool PEER = false, int PAIR = 1>
__device__ __forceinline__ void split_finish(const TcParams &p, const Unit &w, int ew, int lane, int m, int nbase,
                                             int wcols, int rank) {
  const int64_t slot_words = (int64_t)BM * BN;
  const int64_t warp_off = (int64_t)ew * 32 * wcols;
  // Each warp owns 32 rows x wcols columns of the tile and reduces them on
  // its own: per-(tail tile, warp) tickets, so no cross-warp barrier exists
  // that an aborting warp could leave the others waiting at.
  __threadfence();
  __syncwarp();
  unsigned tk = 0;
  unsigned *ticket = p.tickets + ((int64_t)w.tail * PAIR + rank) * NUM_EPI_WARPS + ew;
  if (lane == 0) tk = atomicAdd(ticket, 1u);
  tk = __shfl_sync(0xffffffffu, tk, 0);
  if (tk == (unsigned)(w.nparts - 1)) {
    __threadfence();
    const uint4 *base = reinterpret_cast<const uint4 *>(reinterpret_cast<const uint32_t *>(p.ws) +
                                                        slot_of<PAIR>(p, w.tail, 0, rank) * slot_words + warp_off) + lane;
    const int64_t slot_vec = PAIR * slot_words / 4;   // from piece s to piece s + 1
    constexpr int NV = RCH / 4;                  // uint4 per lane per partial and chunk
    constexpr int PB = NV >= 8 ? 2 : (NV >= 4 ? 4 : 8);  // partials in flight: 16 loads per lane
#pragma unroll 1
    for (int c = 0; c < wcols; c += RCH) {
      uint32_t r[32];
#pragma unroll
      for (int j = 0; j < 32; ++j) r[j] = 0;
      const uint4 *src = base + (c >> 2) * 32;
#pragma unroll 1
      for (int s0 = 0; s0 < w.nparts; s0 += PB) {
        uint4 v[PB][NV];
#pragma unroll
        for (int b = 0; b < PB; ++b)
#pragma unroll
          for (int q = 0; q < NV; ++q)
            v[b][q] = (s0 + b < w.nparts) ? __ldcg(src + (int64_t)(s0 + b) * slot_vec + q * 32) : make_uint4(0, 0, 0, 0);
        // summed in K order: partial s0, s0+1, ...
#pragma unroll
        for (int b = 0; b < PB; ++b) {
          if (s0 + b >= w.nparts) break;
#pragma unroll
          for (int q = 0; q < NV; ++q) {
            const uint4 x = v[b][q];
            if constexpr (Elem<T>::is_int) {
              r[4 * q] += x.x; r[4 * q + 1] += x.y; r[4 * q + 2] += x.z; r[4 * q + 3] += x.w;
            } else {
              r[4 * q] = __float_as_uint(__uint_as_float(r[4 * q]) + __uint_as_float(x.x));
              r[4 * q + 1] = __float_as_uint(__uint_as_float(r[4 * q + 1]) + __uint_as_float(x.y));
              r[4 * q + 2] = __float_as_uint(__uint_as_float(r[4 * q + 2]) + __uint_as_float(x.z));
              r[4 * q + 3] = __float_as_uint(__uint_as_float(r[4 * q + 3]) + __uint_as_float(x.w));
            }
          }
        }
      }
      const int n0 = nbase + c;
      if (m < p.M && n0 < p.N) store_row_chunk<T, RCH, PEER>(p, w.b, m, n0, r);
    }
    if (lane == 0) *ticket = 0u;
  }
}

// ---------------------------------------------------------------------------
// TO: the output element type.  It is T except for the integer limb products,
// whose u8 x u8 GEMMs write 16/32/64-bit integers (direct stores only).
// PEER: also write every output element to the peer copies of C (TcParams::peer_C).
template <class T, int BN, int PAIR = 1, class TO = T, bool PEER = false>
__global__ void __launch_bounds__(NUM_THREADS, 1) tc_gemm_kernel(const __grid_constant__ TcParams p) {
  constexpr int ESZ = sizeof(T);
  using C_ = Cfg<BN, ESZ, PAIR>;
  // columns per TMEM read on the direct-store and split paths: wider outputs
  // take 16 so the converted row chunk stays within the register budget
  constexpr int RCHO = (sizeof(TO) > (size_t)ESZ && C_::RCH > 16) ? 16 : C_::RCH;
  constexpr int TM_ROWS = BM * PAIR;  // output rows per tile (256 for a CTA pair)
  constexpr int BK = C_::BK, STAGES = C_::STAGES;
  constexpr uint32_t A_BYTES = C_::A_BYTES, STAGE_BYTES = C_::STAGE_BYTES;
  constexpr int RCH = C_::RCH, CC = C_::CC;

  extern __shared__ __align__(1024) uint8_t smem_raw[];
  // 1024-byte alignment for the swizzled operand and staging tiles.
  uint8_t *smem = reinterpret_cast<uint8_t *>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t *ring = smem;
  uint8_t *staging = ring + STAGES * STAGE_BYTES;
  uint8_t *red = staging + C_::STAGING_BYTES;   // cluster split-K partials (rank 0)
  uint64_t *bars = reinterpret_cast<uint64_t *>(red + C_::RED_BYTES);
  // bars: full[STAGES], empty[STAGES], tfull[2], tempty[2], drain, red
  uint32_t *tmem_slot = reinterpret_cast<uint32_t *>(bars + 2 * STAGES + 6);
  volatile int *abort_flag = reinterpret_cast<volatile int *>(tmem_slot + 1);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const uint32_t ring_u32 = smem_u32(ring);
  const uint32_t bar_u32 = smem_u32(bars);
  auto full_bar = [&](int s) { return bar_u32 + 8u * s; };
  auto empty_bar = [&](int s) { return bar_u32 + 8u * (STAGES + s); };
  auto tfull_bar = [&](int a) { return bar_u32 + 8u * (2 * STAGES + a); };
  auto tempty_bar = [&](int a) { return bar_u32 + 8u * (2 * STAGES + 2 + a); };
  const uint32_t drain_bar = bar_u32 + 8u * (2 * STAGES + 4);
  const uint32_t red_bar = bar_u32 + 8u * (2 * STAGES + 5);
  const uint32_t red_u32 = smem_u32(red);
  const uint32_t rank = PAIR == 2 ? cluster_rank() : 0u;
  // the pair leader's full barrier of stage s, as a cluster address
  auto leader_full = [&](int s) { return mapa_shared(full_bar(s), 0); };
  const int pair_id = blockIdx.x / PAIR, npairs = gridDim.x / PAIR;
  // Waits on barriers that the peer CTA (or the pair's MMA) arrives on use
  // cluster-scope acquire.
  auto wait_x = [&](uint32_t bar, uint32_t parity) {
    if constexpr (PAIR == 2) return mbar_wait_cluster(bar, parity, abort_flag, p.timeout_ns);
    else return mbar_wait(bar, parity, abort_flag, p.timeout_ns);
  };

  // The next kernel on the stream may begin its own set-up now; this kernel's
  // set-up (barriers, TMEM, tensor maps) overlaps the previous kernel's end,
  // and pdl_wait below orders every global access after that kernel.
  pdl_trigger();
  if (threadIdx.x == 0) {
    for (int s = 0; s < STAGES; ++s) {
      mbar_init(full_bar(s), 1);
      mbar_init(empty_bar(s), 1);
    }
    for (int a = 0; a < 2; ++a) {
      mbar_init(tfull_bar(a), 1);
      mbar_init(tempty_bar(a), NUM_EPI_WARPS * PAIR);
    }
    mbar_init(drain_bar, 1);
    // cluster split-K: every lane of every epilogue warp of ranks 1.. arrives once
    if (p.csplit) mbar_init(red_bar, NUM_EPI_WARPS * 32 * (p.splits - 1));
    *abort_flag = 0;
    fence_mbar_init();
    prefetch_tmap(&p.tmA);
    prefetch_tmap(&p.tmB);
    if (p.c_tma) prefetch_tmap(&p.tmC);
  }
  if (warp == 1) {
    tmem_alloc_g<PAIR>(smem_u32(tmem_slot), C_::TMEM_COLS);
    tmem_relinquish_g<PAIR>();
  }
  tc_fence_before();
  __syncthreads();
  if constexpr (PAIR == 2) cluster_sync_all();  // peer barriers initialised before any remote arrive
  if constexpr (PAIR == 1 && C_::RED_BYTES > 0) {
    if (p.csplit) cluster_sync_all();  // rank 0's reduction barrier initialised before any remote arrive
  }
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;
  pdl_wait();

  if (warp == 0) {
    // ------------------------------------------------------------ producer
    if (lane == 0) {
      int stage = 0;
      uint32_t phase = 0;
      int issued_stage = -1;
      uint32_t issued_phase = 0;
      UnitIter it = unit_iter(p, pair_id, npairs);
      Unit w;
      while (unit_next(p, it, npairs, w)) {
        const int ba = p.a_bcast ? 0 : w.b, bb = p.b_bcast ? 0 : w.b;
        // This CTA's columns of B: its share (1/PAIR) of the unit's columns.  A
        // half-width unit loads only its BN/2 columns of an MN-major B; a
        // K-major B share is one box, loaded whole.
        const bool half_b = w.half >= 0 && p.b_mn;
        const int ccols = (half_b ? BN / 2 : BN) / PAIR;
        const uint32_t b_bytes = (uint32_t)ccols * 128u;
        const int b_boxes = ccols * ESZ / 128;
        const int b_col0 = w.tn * BN + (half_b ? w.half * (BN / 2) : 0) + (int)rank * ccols;
        const int a_row0 = w.tm * TM_ROWS + (int)rank * BM;
        for (int kb = w.kb0; kb < w.kb1; ++kb) {
          if (!wait_x(empty_bar(stage), phase ^ 1u)) goto producer_done;
          // Both CTAs' bytes of this stage are counted on the leader's full barrier.
          if (rank == 0) mbar_arrive_expect_tx(full_bar(stage), C_::NPART * (A_BYTES + b_bytes) * PAIR);
          const uint32_t sa = ring_u32 + stage * STAGE_BYTES;
          const uint32_t sb = sa + C_::NPART * A_BYTES;
          auto load = [&](uint32_t dst, const CUtensorMap *map, int c0, int c1, int c2) {
            if constexpr (PAIR == 2) tma_load_3d_pair(dst, map, leader_full(stage), c0, c1, c2);
            else tma_load_3d(dst, map, full_bar(stage), c0, c1, c2);
          };
          if (!p.a_mn) {
            load(sa, &p.tmA, kb * BK, a_row0, ba);
          } else {
#pragma unroll
            for (int j = 0; j < BM * ESZ / 128; ++j) load(sa + j * (BK * 128), &p.tmA, a_row0 + j * (128 / ESZ), kb * BK, ba);
          }
          if constexpr (C_::NMMA == 2) {
            // 512-wide pair tile: for MMA h this CTA holds tile columns
            // [h * 256 + rank * 128, + 128), at byte offset h * 16 KB of the stage
            constexpr int HB = (C_::UMMA_N / PAIR) * 128;
#pragma unroll
            for (int h = 0; h < 2; ++h) {
              const int col = w.tn * BN + h * C_::UMMA_N + (int)rank * (C_::UMMA_N / PAIR);
              if (!p.b_mn) {
                load(sb + h * HB, &p.tmB, kb * BK, col, bb);
              } else {
#pragma unroll
                for (int j = 0; j < (C_::UMMA_N / PAIR) * ESZ / 128; ++j)
                  load(sb + h * HB + j * (BK * 128), &p.tmB, col + j * (128 / ESZ), kb * BK, bb);
              }
            }
          } else if (!p.b_mn) {
            load(sb, &p.tmB, kb * BK, w.tn * BN + (int)rank * (BN / PAIR), bb);
          } else {
            for (int j = 0; j < b_boxes; ++j) load(sb + j * (BK * 128), &p.tmB, b_col0 + j * (128 / ESZ), kb * BK, bb);
          }
          if constexpr (C_::NPART == 2) {  // low parts (both operands K-major)
            load(sa + A_BYTES, &p.tmA2, kb * BK, a_row0, ba);
            load(sb + b_bytes, &p.tmB2, kb * BK, w.tn * BN + (int)rank * (BN / PAIR), bb);
          }
          issued_stage = stage;
          issued_phase = phase;
          if (++stage == STAGES) { stage = 0; phase ^= 1u; }
        }
      }
    producer_done:
      // Drain: the last issued stage's copies must land before the CTA can exit.
      // The leader sees them on its full barrier; the peer's are counted there
      // too, so the peer waits until the pair's MMA has consumed that stage.
      if (issued_stage >= 0) {
        volatile int no_abort = 0;
        if (rank == 0) mbar_wait(full_bar(issued_stage), issued_phase, &no_abort, p.timeout_ns);
        else mbar_wait_cluster(empty_bar(issued_stage), issued_phase, &no_abort, p.timeout_ns);
      }
    }
  } else if (warp == 1) {
    // ------------------------------------------------------------ MMA issuer
    if (rank == 0 && lane == 0) {
      const uint32_t idesc_full = make_idesc<T, C_::UMMA_N, TM_ROWS>(p.a_mn, p.b_mn);
      const uint32_t idesc_half = make_idesc<T, (BN >= 32 ? BN / 2 : BN), TM_ROWS>(p.a_mn, p.b_mn);
      // Canonical SW128 layouts: K-major SBO = 8 rows * 128 B; MN-major
      // LBO = next 128-byte MN column block (one TMA box), SBO = 8 K rows.
      const uint32_t a_lbo = p.a_mn ? BK * 128 : 16, b_lbo = p.b_mn ? BK * 128 : 16;
      const uint32_t a_kstep = p.a_mn ? C_::UMMA_K * 128 : 32, b_kstep = p.b_mn ? C_::UMMA_K * 128 : 32;
      int stage = 0;
      uint32_t phase = 0;
      int abuf = 0;
      uint32_t aphase = 0;
      bool issued_any = false;
      UnitIter it = unit_iter(p, pair_id, npairs);
      Unit w;
      while (unit_next(p, it, npairs, w)) {
        const uint32_t idesc = w.half >= 0 ? idesc_half : idesc_full;
        // K-major B holds the whole tile: a half-width unit starts BN/2 rows in.
        const uint32_t b_off = (w.half > 0 && !p.b_mn) ? (uint32_t)(BN / 2) * 128u : 0u;
        bool aborted = false;
        // One TMEM accumulation per K chunk (the whole unit, except for fp32:
        // see C_::KCHUNK); each chunk is handed to the epilogue.
        for (int c0 = w.kb0; c0 < w.kb1 && !aborted; c0 += C_::KCHUNK) {
          const int c1 = min(w.kb1, c0 + C_::KCHUNK);
          if (!wait_x(tempty_bar(abuf), aphase ^ 1u)) { aborted = true; break; }
          tc_fence_after();
          const uint32_t d_tmem = tmem_base + (uint32_t)(abuf * C_::ACC_COLS);
          for (int kb = c0; kb < c1; ++kb) {
            if (!wait_x(full_bar(stage), phase)) { aborted = true; break; }
            tc_fence_after();
            const uint32_t sa = ring_u32 + stage * STAGE_BYTES;
            const uint32_t sb = sa + C_::NPART * A_BYTES + b_off;
#pragma unroll
            for (int ks = 0; ks < C_::KSTEPS; ++ks) {
              const uint64_t ad = sdesc(sa + ks * a_kstep, a_lbo, 1024);
              const uint64_t bd = sdesc(sb + ks * b_kstep, b_lbo, 1024);
              umma_g<ESZ, PAIR>(d_tmem, ad, bd, idesc, (kb > c0 || ks > 0) ? 1u : 0u);
              if constexpr (C_::NMMA == 2) {
                // tile columns [256, 512): this CTA's share of B 16 KB further on,
                // accumulated in TMEM columns 256..511
                const uint64_t bd2 = sdesc(sb + (C_::UMMA_N / PAIR) * 128 + ks * b_kstep, b_lbo, 1024);
                umma_g<ESZ, PAIR>(d_tmem + C_::UMMA_N, ad, bd2, idesc, (kb > c0 || ks > 0) ? 1u : 0u);
              }
              if constexpr (C_::NPART == 2) {
                // 3xTF32: + A_hi B_lo + A_lo B_hi (A_lo B_lo is below fp32 resolution).
                // Both operands are K-major here, so B_lo is one whole B share
                // after B_hi (a half-width unit keeps its b_off into it).
                const uint64_t bd_lo = sdesc(sb + C_::B_BYTES + ks * b_kstep, b_lbo, 1024);
                const uint64_t ad_lo = sdesc(sa + A_BYTES + ks * a_kstep, a_lbo, 1024);
                umma_g<ESZ, PAIR>(d_tmem, ad, bd_lo, idesc, 1u);
                umma_g<ESZ, PAIR>(d_tmem, ad_lo, bd, idesc, 1u);
              }
            }
            issued_any = true;
            umma_commit_g<PAIR>(empty_bar(stage));  // frees this smem stage (in both CTAs) when the MMAs finish
            if (++stage == STAGES) { stage = 0; phase ^= 1u; }
          }
          if (aborted) break;
          umma_commit_g<PAIR>(tfull_bar(abuf));  // accumulators ready for the epilogue(s)
          if (++abuf == C_::NACC) { abuf = 0; aphase ^= 1u; }
        }
        if (aborted) break;
      }
      if (*abort_flag && issued_any) {
        // Drain every MMA this thread issued before TMEM is freed.
        umma_commit_self<PAIR>(drain_bar);
        volatile int no_abort = 0;
        mbar_wait(drain_bar, 0, &no_abort, p.timeout_ns);
      }
    }
  } else {
    // ------------------------------------------------------------ epilogue
    const int ew = warp - 2;              // 0..7
    const int q = warp & 3;               // TMEM lane quarter this warp may access
    const int row = q * 32 + lane;
    const uint32_t stg0 = smem_u32(staging) + (uint32_t)(ew * STAGING_PER_WARP);
    // Hand a drained accumulator back to the (pair leader's) MMA issuer.
    auto release_tmem = [&](int a) {
      if constexpr (PAIR == 2) mbar_arrive_cluster(mapa_shared(tempty_bar(a), 0));
      else mbar_arrive(tempty_bar(a));
    };
    int sbuf = 0;                         // staging buffer to fill next
    int abuf = 0;
    uint32_t aphase = 0;
    UnitIter it = unit_iter(p, pair_id, npairs);
    Unit w;
    while (unit_next(p, it, npairs, w)) {
      if constexpr (C_::NPART == 2) {
        // fp32 (3xTF32): each K chunk's TMEM sum is added to fp32 running sums
        // in registers (IEEE adds), then stored or published as a partial.
        const int m = w.tm * TM_ROWS + (int)rank * BM + row;
        const int ucols = w.half >= 0 ? BN / 2 : BN;
        const int wcols = ucols / 2;
        const int col0 = (ew >> 2) * wcols;
        const int nbase = w.tn * BN + (w.half > 0 ? BN / 2 : 0) + col0;
        float run[C_::RUN];
#pragma unroll
        for (int j = 0; j < C_::RUN; ++j) run[j] = 0.f;
        bool ok = true;
        for (int c0 = w.kb0; c0 < w.kb1; c0 += C_::KCHUNK) {
          if (!wait_x(tfull_bar(abuf), aphase)) { ok = false; break; }
          tc_fence_after();
          const uint32_t tb = tmem_base + ((uint32_t)(q * 32) << 16) + (uint32_t)(abuf * C_::ACC_COLS + col0);
#pragma unroll
          for (int c = 0; c < C_::RUN; c += RCH) {
            if (c < wcols) {
              uint32_t r[32];
              tmem_ld<RCH>(tb + c, r);
              tmem_wait_ld();
#pragma unroll
              for (int j = 0; j < RCH; ++j) run[c + j] += __uint_as_float(r[j]);
            }
          }
          tc_fence_before();
          __syncwarp();
          if (lane == 0) release_tmem(abuf);
          if (++abuf == C_::NACC) { abuf = 0; aphase ^= 1u; }
        }
        if (!ok) break;
        if (!w.split) {
#pragma unroll
          for (int c = 0; c < C_::RUN; c += RCH) {
            if (c < wcols) {
              uint32_t r[32];
#pragma unroll
              for (int j = 0; j < RCH; ++j) r[j] = __float_as_uint(run[c + j]);
              const int n0 = nbase + c;
              if (m < p.M && n0 < p.N) store_row_chunk<T, RCH, PEER>(p, w.b, m, n0, r);
            }
          }
        } else {
          uint4 *part = reinterpret_cast<uint4 *>(reinterpret_cast<uint32_t *>(p.ws) +
                                                  slot_of<PAIR>(p, w.tail, w.s, (int)rank) * ((int64_t)BM * BN) +
                                                  (int64_t)ew * 32 * wcols) + lane;
#pragma unroll
          for (int c = 0; c < C_::RUN; c += 4)
            if (c < wcols)
              __stcg(part + (c >> 2) * 32, make_uint4(__float_as_uint(run[c]), __float_as_uint(run[c + 1]),
                                                      __float_as_uint(run[c + 2]), __float_as_uint(run[c + 3])));
          split_finish<T, BN, RCH, PEER, PAIR>(p, w, ew, lane, m, nbase, wcols, (int)rank);
        }
        continue;
      }
      if (!wait_x(tfull_bar(abuf), aphase)) break;
      tc_fence_after();
      const int m0 = w.tm * TM_ROWS + (int)rank * BM;  // this CTA's first output row of the tile
      const int m = m0 + row;
      // Columns of this unit and of this warp's share (half of the unit).
      const int ucols = w.half >= 0 ? BN / 2 : BN;
      const int wcols = ucols / 2;
      const int ucol0 = w.half > 0 ? BN / 2 : 0;            // unit's first column within the tile
      const int col0 = (ew >> 2) * wcols;                    // warp's first column within the unit
      const uint32_t tbase = tmem_base + ((uint32_t)(q * 32) << 16) + (uint32_t)(abuf * C_::ACC_COLS + col0);
      const int nbase = w.tn * BN + ucol0 + col0;            // global column of tbase
      if (!w.split) {
        if constexpr (C_::TMA_STORE && std::is_same_v<T, TO>) {
          if (p.c_tma) {
            // 64-byte rows staged with the SWIZZLE_64B pattern (16-byte chunk j
            // of row r at chunk j ^ ((r >> 1) & 3)), one TMA store per 32-row
            // box of CC columns, two staging buffers so a store overlaps the
            // next box.  TMEM is read in 32-column sub-chunks, the next one
            // issued before the current one is converted.
            constexpr int SUBS = CC / 32;                // sub-chunks per staged row (1: 16-bit, 2: 8-bit)
            constexpr int V = 32 * ESZ / 16;             // 16-byte pieces per sub-chunk
            const int nsub = wcols / 32;
            uint32_t ra[32];
            tmem_ld_x32(tbase, ra);
            for (int sc = 0; sc < nsub; ++sc) {
              tmem_wait_ld();
              uint32_t rb[32];
#pragma unroll
              for (int j = 0; j < 32; ++j) rb[j] = ra[j];
              if (sc + 1 < nsub) {
                tmem_ld_x32(tbase + (sc + 1) * 32, ra);
              } else {                           // last TMEM read of this unit by this warp
                tc_fence_before();
                __syncwarp();
                if (lane == 0) release_tmem(abuf);
              }
              const int sub = sc % SUBS;
              const uint32_t stg = stg0 + (uint32_t)(sbuf * STAGING_BUF);
              if (sub == 0) {                    // buffer's previous store has read it
                if (lane == 0) asm volatile("cp.async.bulk.wait_group.read 1;" ::: "memory");
                __syncwarp();
              }
              const int n0 = nbase + sc * 32;
              uint32_t pk[32 * ESZ / 4];
              pack32<T>(p, w.b, m, n0, rb, pk);
#pragma unroll
              for (int v = 0; v < V; ++v) {
                const int ci = sub * V + v;
                const uint32_t addr = stg + lane * STAGING_ROW + ((ci ^ ((lane >> 1) & 3)) << 4);
                asm volatile("st.shared.v4.b32 [%0], {%1, %2, %3, %4};" ::"r"(addr), "r"(pk[4 * v]), "r"(pk[4 * v + 1]),
                             "r"(pk[4 * v + 2]), "r"(pk[4 * v + 3])
                             : "memory");
              }
              if (sub == SUBS - 1) {
                fence_proxy_async_smem();
                __syncwarp();
                if (lane == 0) {
                  tma_store_3d(&p.tmC, stg, n0 - (SUBS - 1) * 32, m0 + q * 32, w.b);
                  bulk_commit();
                }
                if constexpr (PEER) {
                  // boxes in pairs (adjacent columns in the two staging
                  // buffers) as 128-byte rows; an unpaired last box alone
                  const int bx = sc / SUBS, nbox = nsub / SUBS;
                  const int bcol0 = n0 - (SUBS - 1) * 32;
                  if (bx & 1)
                    peer_store_box2<T>(p, stg0 + (uint32_t)((sbuf ^ 1) * STAGING_BUF), stg, lane, w.b, m0 + q * 32,
                                       bcol0 - CC);
                  else if (bx == nbox - 1)
                    peer_store_box<T>(p, stg, lane, w.b, m0 + q * 32, bcol0);
                }
                sbuf ^= 1;
              }
            }
            if (++abuf == C_::NACC) { abuf = 0; aphase ^= 1u; }
            continue;
          }
        }
#pragma unroll 1
        for (int c = 0; c < wcols; c += RCHO) {
          uint32_t r[32];
          tmem_ld<RCHO>(tbase + c, r);
          tmem_wait_ld();
          const int n0 = nbase + c;
          if (m < p.M && n0 < p.N) store_row_chunk<TO, RCHO, PEER>(p, w.b, m, n0, r);
        }
        tc_fence_before();
        __syncwarp();
        if (lane == 0) release_tmem(abuf);
      } else if (C_::RED_BYTES > 0 && p.csplit) {
        // Cluster split-K: the same lane-interleaved runs as the workspace
        // partials below, in rank 0's shared memory (slot s - 1 for split s).
        // Ranks 1.. store theirs and arrive on rank 0's reduction barrier
        // (release, cluster scope: each lane orders its own stores); rank 0
        // waits for all of them, adds them to its own accumulator in K order
        // and stores the tile.
        const uint32_t slot_bytes = (uint32_t)(BM * BN * 4);
        const uint32_t off0 = (uint32_t)(ew * 32 * wcols * 4) + (uint32_t)lane * 16u;
        if (w.s > 0) {
          const uint32_t rbase = mapa_shared(red_u32 + (uint32_t)(w.s - 1) * slot_bytes + off0, 0);
#pragma unroll 1
          for (int c = 0; c < wcols; c += RCHO) {
            uint32_t r[32];
            tmem_ld<RCHO>(tbase + c, r);
            tmem_wait_ld();
#pragma unroll
            for (int j = 0; j < RCHO; j += 4)
              st_cluster_v4(rbase + (uint32_t)((c + j) >> 2) * 512u, r[j], r[j + 1], r[j + 2], r[j + 3]);
          }
          tc_fence_before();
          __syncwarp();
          if (lane == 0) release_tmem(abuf);
          mbar_arrive_cluster(mapa_shared(red_bar, 0));
        } else {
          const bool got = mbar_wait_cluster(red_bar, 0, abort_flag, p.timeout_ns);
          if (got) {
#pragma unroll 1
            for (int c = 0; c < wcols; c += RCHO) {
              uint32_t r[32];
              tmem_ld<RCHO>(tbase + c, r);
              tmem_wait_ld();
#pragma unroll 1
              for (int s2 = 1; s2 < w.nparts; ++s2) {
                const uint32_t lb = red_u32 + (uint32_t)(s2 - 1) * slot_bytes + off0 + (uint32_t)(c >> 2) * 512u;
#pragma unroll
                for (int j = 0; j < RCHO; j += 4) {
                  const uint4 v = ld_shared_v4(lb + (uint32_t)(j >> 2) * 512u);
                  if constexpr (Elem<T>::is_int) {
                    r[j] += v.x; r[j + 1] += v.y; r[j + 2] += v.z; r[j + 3] += v.w;
                  } else {
                    r[j] = __float_as_uint(__uint_as_float(r[j]) + __uint_as_float(v.x));
                    r[j + 1] = __float_as_uint(__uint_as_float(r[j + 1]) + __uint_as_float(v.y));
                    r[j + 2] = __float_as_uint(__uint_as_float(r[j + 2]) + __uint_as_float(v.z));
                    r[j + 3] = __float_as_uint(__uint_as_float(r[j + 3]) + __uint_as_float(v.w));
                  }
                }
              }
              const int n0 = nbase + c;
              if (m < p.M && n0 < p.N) store_row_chunk<TO, RCHO, PEER>(p, w.b, m, n0, r);
            }
          }
          tc_fence_before();
          __syncwarp();
          if (lane == 0) release_tmem(abuf);
          if (!got) break;
        }
      } else {
        // Split-K: publish raw accumulators.  Slot (tail, s) holds BM x BN
        // 4-byte values; warp ew's 32 rows x wcols columns are stored as
        // uint4 runs indexed (column / 4) * 32 + lane.
        const int64_t slot_words = (int64_t)BM * BN;
        const int64_t warp_off = (int64_t)ew * 32 * wcols;
        uint4 *part = reinterpret_cast<uint4 *>(reinterpret_cast<uint32_t *>(p.ws) +
                                                slot_of<PAIR>(p, w.tail, w.s, (int)rank) * slot_words + warp_off) + lane;
#pragma unroll 1
        for (int c = 0; c < wcols; c += RCHO) {
          uint32_t r[32];
          tmem_ld<RCHO>(tbase + c, r);
          tmem_wait_ld();
#pragma unroll
          for (int j = 0; j < RCHO; j += 4)
            __stcg(part + ((c + j) >> 2) * 32, make_uint4(r[j], r[j + 1], r[j + 2], r[j + 3]));
        }
        tc_fence_before();
        __syncwarp();
        if (lane == 0) release_tmem(abuf);
        split_finish<TO, BN, RCHO, PEER, PAIR>(p, w, ew, lane, m, nbase, wcols, (int)rank);
      }
      if (++abuf == C_::NACC) { abuf = 0; aphase ^= 1u; }
    }
    if (lane == 0) bulk_wait0();  // every TMA store of this warp has completed
    // peer and multicast stores are performed system-wide before the CTA
    // retires (the alias fence orders the multicast-address stores with later
    // accesses through the unicast addresses of the same memory)
    if constexpr (PEER) {
      asm volatile("fence.proxy.alias;" ::: "memory");
      __threadfence_system();
    }
    __syncwarp();
  }

  tc_fence_before();
  __syncthreads();
  if constexpr (PAIR == 2) cluster_sync_all();  // the pair's MMAs and remote arrivals are done
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc_g<PAIR>(tmem_base, C_::TMEM_COLS);
  }
}

// Debug kernel for the bounded-wait path: waits on a barrier nobody arrives at.
__global__ void wait_timeout_kernel(unsigned long long timeout_ns) {
  __shared__ __align__(8) uint64_t bar;
  __shared__ int abort_flag;
  if (threadIdx.x == 0) {
    mbar_init(smem_u32(&bar), 1);
    abort_flag = 0;
    fence_mbar_init();
  }
  __syncthreads();
  if (threadIdx.x == 0) mbar_wait(smem_u32(&bar), 0, &abort_flag, timeout_ns);
  __syncthreads();
}

}  // namespace tc
}  // namespace mb
