// C ABI of metalblas_b200: validation, the sm_100a plan (tile table), TMA
// descriptor construction and kernel launches.  One translation unit so that
// the device status word has a single definition.
//
// Plan rules (B200 replacement of the reference's planners):
//  * M==1 or N==1 with a unit-stride matrix -> GEMV kernels, oriented like
//    _dispatch_gemv (metalblas/dispatch.py:49-70) and the fast paths of
//    metalblas/float_dispatch.py:745-764;
//  * bf16/fp16/int8/uint8 whose operands TMA can address -> tcgen05 kernel
//    (mpp_tensor_gemm / splitk / gemv_bt / int_gemm-for-8-bit replacement);
//    thin M runs as Cᵀ = Bᵀ·Aᵀ (the reference's flipt/sgpipe/gemv_bt ideas,
//    metalblas/float_dispatch.py:249-366, folded into one kernel);
//    N-tile and split-K come from a wave-quantisation cost model instead of
//    the Apple tile heuristics (metalblas/float_dispatch.py:613-655);
//  * everything else -> CUDA-core kernel (simd_gemm / int_gemm / complex
//    products replacement).
#include <cuda.h>
#include <cudaTypedefs.h>
#include <cuda_runtime.h>

#include <algorithm>
#include <cstdarg>
#include <type_traits>
#include <cmath>
#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <atomic>
#include <mutex>
#include <string>
#include <unordered_map>

#include "../../include/metalblas_b200.h"
#include "mb_common.cuh"
#include "simt_gemm.cuh"
#include "gemv.cuh"
#include "tc_gemm.cuh"
#include "c32.cuh"
#include "peaks.cuh"
#include "pack.cuh"

using namespace mb;

namespace {

thread_local std::string g_err;

int fail(int code, const char *fmt, ...) {
  char buf[512];
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(buf, sizeof(buf), fmt, ap);
  va_end(ap);
  g_err = buf;
  return code;
}

int cuda_check(cudaError_t e, const char *what) {
  if (e == cudaSuccess) return MB_OK;
  return fail(MB_ERR_LAUNCH, "%s: %s", what, cudaGetErrorString(e));
}

int elem_size(int dt) {
  switch (dt) {
    case MB_F32: return 4;
    case MB_F16: case MB_BF16: return 2;
    case MB_C64: return 8;
    case MB_C32: return 4;
    case MB_I8: case MB_U8: return 1;
    case MB_I16: return 2;
    case MB_I32: return 4;
    case MB_I64: return 8;
  }
  return 0;
}
bool acc_is_8byte(int dt) { return dt == MB_C64 || dt == MB_C32 || dt == MB_I64; }
bool is_tc_dtype(int dt) { return dt == MB_BF16 || dt == MB_F16 || dt == MB_I8 || dt == MB_U8; }

int64_t ceil_div(int64_t a, int64_t b) { return (a + b - 1) / b; }
int64_t round_up(int64_t a, int64_t b) { return ceil_div(a, b) * b; }
bool aligned16(const void *p) { return (reinterpret_cast<uintptr_t>(p) & 15) == 0; }

struct DevInfo {
  int sms = 148;
  bool ok = false;
  char name[128] = {0};
};
DevInfo g_dev[64];
std::mutex g_dev_mu;

int current_device(int *dev) {
  return cuda_check(cudaGetDevice(dev), "cudaGetDevice");
}
int num_sms(int dev) {
  std::lock_guard<std::mutex> lk(g_dev_mu);
  if (dev < 0 || dev >= 64) return 148;
  if (!g_dev[dev].ok) {
    int n = 0;
    if (cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev) == cudaSuccess && n > 0) g_dev[dev].sms = n;
    cudaDeviceProp prop;
    if (cudaGetDeviceProperties(&prop, dev) == cudaSuccess) {
      snprintf(g_dev[dev].name, sizeof(g_dev[dev].name), "%s", prop.name);
      for (char *c = g_dev[dev].name; *c; ++c)
        if (*c == '\t' || *c == '\n' || *c == '|') *c = ' ';
    }
    g_dev[dev].ok = true;
  }
  return g_dev[dev].sms;
}
// Device name for autotune keys ("none" without a device).
std::string device_name() {
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) {
    cudaGetLastError();
    return "none";
  }
  num_sms(dev);
  std::lock_guard<std::mutex> lk(g_dev_mu);
  return g_dev[dev].name[0] ? std::string(g_dev[dev].name) : std::string("unknown");
}

// ------------------------------------------------------------ autotune cache
struct Override {
  int keep, backend, tile_n, split_k, swap_ab, cta_pair, stream_k;
};
std::mutex g_tune_mu;
std::unordered_map<std::string, Override> g_tune;
std::atomic<int64_t> g_tune_size{0};

std::string tune_key(const mb_gemm_desc *d) {
  char buf[512];
  const std::string name = device_name();
  auto m8 = [](int64_t v) { return (long long)(((v % 8) + 8) % 8); };
  snprintf(buf, sizeof(buf), "%s|%d|%lld|%lld|%lld|%lld|%d%d|%d%d%d|%lld%lld%lld%lld|%d%d%d|%d", name.c_str(),
           d->dtype, (long long)d->M, (long long)d->N, (long long)d->K, (long long)d->batch, d->sA == 0, d->sB == 0,
           d->a_rs == 1, d->b_rs == 1, d->c_cs == 1, m8(d->a_rs), m8(d->a_cs), m8(d->b_rs), m8(d->b_cs),
           aligned16(d->A), aligned16(d->B), aligned16(d->C), d->epilogue);
  return buf;
}

bool has_overrides(const mb_gemm_desc *d) {
  return d->backend != MB_BACKEND_AUTO || d->tile_n || d->split_k || d->swap_ab || d->cta_pair || d->stream_k;
}

unsigned long long wait_timeout_ns() {
  static unsigned long long v = [] {
    const char *s = getenv("METALBLAS_WAIT_TIMEOUT_MS");
    long long ms = s ? atoll(s) : 2000;
    if (ms <= 0) ms = 2000;
    return (unsigned long long)ms * 1000000ull;
  }();
  return v;
}

// A strided 2-D operand: element (r, c) at base[r*rs + c*cs].  Extent-1
// dimensions get a stride that makes the operand look unit-stride / aligned,
// since that stride never moves the address.
void normalize(int64_t rows, int64_t cols, int64_t &rs, int64_t &cs) {
  if (rows <= 1 && cols <= 1) { rs = std::max<int64_t>(cols, 1); cs = 1; return; }
  if (rows <= 1) { if (cs == 1) rs = round_up(cols, 16); else rs = 1; }
  if (cols <= 1) { if (rs == 1) cs = round_up(rows, 16); else cs = 1; }
}

// --------------------------------------------------------------------------- plan
// Workspace layout, identical for every plan: a fixed region of ticket counters
// at offset 0, then the split-K partials.  Because the ticket region never
// moves, partials written by one plan can never land on the counters another
// plan reads; each kernel returns the counters it used to zero.
constexpr int64_t kTicketBytes = 256 * 1024;
constexpr int64_t kMaxTickets = kTicketBytes / 4;
constexpr int kGemvWarps = 8;         // warps per GEMV CTA
constexpr int kGemvRowsPerWarp = 2;   // staged-x rows kernel
constexpr int64_t kGemvRowsPerCta = kGemvWarps * kGemvRowsPerWarp;

enum PlanKind {
  PK_EMPTY = 0, PK_GEMV_COLS, PK_GEMV_ROWS, PK_TC, PK_SIMT, PK_TC_C32, PK_TC_PACKED, PK_TC_3XTF32, PK_TC_C64X3,
  PK_TC_LIMB
};

struct Plan {
  int kind = PK_EMPTY;
  // GEMV
  GemvParams g{};
  int vec = 1;
  int64_t gemv_ctas_x = 0;
  // TC (operands already swapped when swap == 1)
  int swap = 0, bn = 0, splits = 1;
  double est = 0.0;  // the tile chooser's time estimate (cycles)
  int64_t tiles_m = 0, tiles_n = 0, kb_total = 0, kb_per_split = 0;
  int64_t dp_tiles = 0;  // whole tiles; tiles after them are split `splits` ways along K,
  int tail_half = 0;     // or (tail_half) into two half-width units each
  int pair = 1;          // 2: CTA-pair kernel (cta_group::2, 256-row tiles)
  int sk = 0;            // tail tiles stream-K over sk_ctas CTAs (splits = partial slots per tile)
  int64_t sk_ctas = 0;
  // complex32 as one real fp16 GEMM C' = A' B' (PK_TC_C32); the TC fields above
  // describe that real GEMM
  int c32_pack_a = 0;               // A' is a packed copy (else A's own storage)
  int64_t c32_lda = 0, c32_ldb = 0; // row pitch of packed A' / of B', in half2 pairs
  int64_t c32_a_off = 0, c32_b_off = 0, c32_a_batches = 1, c32_b_batches = 1;
  int a_mn = 0, b_mn = 0;
  // PK_TC_PACKED: operands TMA cannot address are first copied into the
  // workspace as dense row-major matrices (A' M x lda', B' K x ldb')
  int pk_a = 0, pk_b = 0;
  int pk_a_cm = 0, pk_b_cm = 0;  // packed column-major (source column-contiguous): a plain strided copy
  int64_t pk_lda = 0, pk_ldb = 0, pk_a_off = 0, pk_b_off = 0, pk_a_batches = 1, pk_b_batches = 1;
  // PK_TC_3XTF32: fp32 split into tf32 high / low parts, both operands K-major
  // in the workspace (A' M x ldk, B'ᵀ N x ldk)
  int64_t x3_ldk = 0, x3_a_batches = 1, x3_b_batches = 1;
  int64_t x3_ahi = 0, x3_alo = 0, x3_bhi = 0, x3_blo = 0, x3_flag = 0;
  // PK_TC_LIMB: 16/32/64-bit integers as byte planes on the 8-bit tensor cores
  int limb_L = 0;
  int64_t limb_kc = 0, limb_kp = 0, limb_ld = 0, limb_a_off = 0, limb_b_off = 0;
  int64_t limb_a_batches = 1, limb_b_batches = 1;
  // shared
  int64_t ws_bytes = 0;
  std::string why;
};

// Working copy of the descriptor with normalised strides.
struct Op {
  int dt;
  int64_t M, N, K, batch;
  const void *A, *B;
  const void *A2 = nullptr, *B2 = nullptr;  // 3xTF32: low parts, laid out like A / B
  void *C;
  int64_t a_rs, a_cs, sA, b_rs, b_cs, sB, c_rs, c_cs, sC;
  int conj_a, conj_b;
  const void *bias;
  int64_t bias_rs, bias_cs, bias_bs;
};

Op make_op(const mb_gemm_desc *d) {
  Op o{};
  o.dt = d->dtype; o.M = d->M; o.N = d->N; o.K = d->K; o.batch = d->batch;
  o.A = d->A; o.B = d->B; o.C = d->C;
  o.a_rs = d->a_rs; o.a_cs = d->a_cs; o.sA = d->sA;
  o.b_rs = d->b_rs; o.b_cs = d->b_cs; o.sB = d->sB;
  o.c_rs = d->c_rs; o.c_cs = d->c_cs; o.sC = d->sC;
  o.conj_a = d->conj_a; o.conj_b = d->conj_b;
  o.bias = d->bias; o.bias_rs = d->bias_rs; o.bias_cs = d->bias_cs; o.bias_bs = d->bias_bs;
  if (o.batch <= 1) { o.sA = o.sB = o.sC = 0; o.bias_bs = 0; }
  normalize(o.M, o.K, o.a_rs, o.a_cs);
  normalize(o.K, o.N, o.b_rs, o.b_cs);
  return o;
}

Op swapped(const Op &o) {
  Op s = o;
  s.M = o.N; s.N = o.M;
  s.A = o.B; s.B = o.A;
  s.A2 = o.B2; s.B2 = o.A2;
  s.a_rs = o.b_cs; s.a_cs = o.b_rs; s.sA = o.sB;
  s.b_rs = o.a_cs; s.b_cs = o.a_rs; s.sB = o.sA;
  s.c_rs = o.c_cs; s.c_cs = o.c_rs;
  s.bias_rs = o.bias_cs; s.bias_cs = o.bias_rs;
  s.conj_a = o.conj_b; s.conj_b = o.conj_a;
  return s;
}

// Can TMA feed this operand pair?  Sets a_mn / b_mn.
bool tc_layout_ok(const Op &o, int bn, int &a_mn, int &b_mn, std::string *why) {
  const int esz = elem_size(o.dt);
  auto bad = [&](const char *w) { if (why) *why = w; return false; };
  if (o.M >= (1ll << 31) || o.N >= (1ll << 31) || o.K >= (1ll << 31) || o.K < 1) return bad("extent");
  if (!aligned16(o.A) || !aligned16(o.B)) return bad("base not 16B aligned");
  if (o.batch > 1) {
    if ((o.sA * esz) % 16 || (o.sB * esz) % 16) return bad("batch stride not 16B multiple");
    if (o.sA < 0 || o.sB < 0) return bad("negative batch stride");
  }
  if (o.a_cs == 1 && o.a_rs >= o.K && (o.a_rs * esz) % 16 == 0) a_mn = 0;
  else if (o.a_rs == 1 && o.a_cs >= o.M && (o.a_cs * esz) % 16 == 0) a_mn = 1;
  else return bad("A layout");
  if (o.b_rs == 1 && o.b_cs >= o.K && (o.b_cs * esz) % 16 == 0) b_mn = 0;
  else if (o.b_cs == 1 && o.b_rs >= o.N && (o.b_rs * esz) % 16 == 0 && bn * esz >= 128) b_mn = 1;
  else return bad("B layout");
  return true;
}

// Cycles per 128-byte K-block of a 128 x BN tile on one SM.  Measured on the
// B200 (4096^3 .. 8192^3 bf16, warm L2) the mainloop is bounded by operand
// traffic into shared memory at ~45 B/clk/SM rather than by the nominal UMMA
// rate (BN/2 cycles per K=16 step); the model takes the slower of the two.
double kblock_cycles(int bn) { return std::max(2.0 * bn, (128.0 + bn) * 128.0 / 45.0); }
// The same for one SM of a CTA pair (cta_group::2): each SM computes 128 x BN
// per K-block but loads only half of B's columns.  Calibrated on the B200:
// 1.09-1.23x the single-CTA rate at BN=256 (4096^3 .. 8192^3, 2048x14336x4096).
double kblock_cycles_pair(int bn) { return std::max(2.0 * bn, (128.0 + bn / 2.0) * 128.0 / 35.0); }
// The 512-wide pair tile (two N = 256 MMAs per K-step) moves 48 KB per SM per
// K-block for twice the work of the 256-wide one: measured 1.68-1.83x its
// K-block time on the B200 (4096^3, 2048 x 14336 x 4096, 16384^3), i.e. the
// operand stream at ~30.5 B/clk/SM.
double kblock_cycles_pair_wide() { return (128.0 + 256.0) * 128.0 / 30.5; }

// CTA-pair kernels in the tile table (METALBLAS_PAIR=0 leaves them out; they
// can always be requested per call through mb_gemm_desc.cta_pair = 2).
const bool g_pair_enabled = [] {
  const char *s = getenv("METALBLAS_PAIR");
  return !(s && s[0] == '0');
}();
// Stream-K tails on CTA pairs: off in the tile table unless METALBLAS_PAIR_SK=1
// (measured on the B200 they lost to the table's other plans on most shapes
// the cost model would give them: 1024x1024x8192 467 vs 541 TFLOP/s,
// 2048x2048x8192 1035 vs 1337; the fix-up of a piece's partials is exposed).
// stream_k = 2 with cta_pair = 2 still requests one.
const bool g_pair_sk = [] {
  const char *s = getenv("METALBLAS_PAIR_SK");
  return s && s[0] == '1';
}();
// 512-wide CTA-pair tiles in the tile table (METALBLAS_PAIR_WIDE=0 leaves
// them out; tile_n = 512 still requests one).
const bool g_pair_wide = [] {
  const char *s = getenv("METALBLAS_PAIR_WIDE");
  return !(s && s[0] == '0');
}();

// HBM bytes per clock per SM when every SM streams (6537 GB/s / 148 / 1.965 GHz).
constexpr double kHbmBytesPerClkPerSm = 22.4;
// DRAM bytes one SM pulls per clock when its operands stream from HBM rather
// than L2 (B200, thin and split-K shapes on 96-128 busy SMs: 57-61 GB/s each).
constexpr double kSmStreamBytesPerClk = 31.0;

// Stream-K partition of `tail` tiles of kb K-blocks over G CTAs: the most
// pieces any tile is cut into (CTA g owns iterations [g*I/G, (g+1)*I/G)).
int sk_max_parts(int64_t tail, int64_t kb, int64_t G) {
  const int64_t I = tail * kb;
  auto owner = [&](int64_t i) { return ((i + 1) * G - 1) / I; };
  int64_t mx = 0;
  for (int64_t t = 0; t < tail; ++t) mx = std::max(mx, owner((t + 1) * kb - 1) - owner(t * kb) + 1);
  return (int)mx;
}

void choose_tc_tile_uncached(const Op &o, int sms, int force_bn, int force_split, int force_pair, int force_sk,
                             bool have_ws, Plan &pl) {
  const int esz = elem_size(o.dt);
  const int64_t BK = 128 / esz;
  // fp32 runs as 3xTF32: three tf32 MMAs (half the bf16 rate) per K-block and
  // twice the operand bytes (high and low parts)
  const bool s3 = o.dt == MB_F32;
  auto kbc = [&](int bn) { return s3 ? std::max(6.0 * bn, 2.0 * (128.0 + bn) * 128.0 / 45.0) : kblock_cycles(bn); };
  auto kbcp = [&](int bn) {
    if (bn > 256) return kblock_cycles_pair_wide();
    return s3 ? std::max(6.0 * bn, 2.0 * (128.0 + bn / 2.0) * 128.0 / 35.0) : kblock_cycles_pair(bn);
  };
  const int64_t kb_total = ceil_div(o.K, BK);
  static const int bns[] = {16, 32, 64, 128, 256, 512};
  double best = 1e300;
  const double opnd_bytes =
      (double)(o.M * o.K * (o.sA ? o.batch : 1) + o.N * o.K * (o.sB ? o.batch : 1)) * esz +
      (double)(o.M * o.N * o.batch) * esz;
  auto consider = [&](double compute, double units, double waves, double extra_bytes, int bn, int am, int bm,
                      int seff, int64_t kbp, int64_t dp, int half, int pair = 1, int sk = 0) {
    // HBM floor, wave by wave: a wave with n busy SMs streams at the whole
    // chip's bandwidth or at what n SMs can pull from DRAM, whichever is lower
    // (a short last wave streams slowly).  Stream-K CTAs stream B rows at
    // unrelated K offsets at the same time, measured below the same bytes read
    // by K-aligned units: ~15% with wide tiles (skinny 128 x 8192 x 65536),
    // ~8% with narrow ones (thin-M swapped tiles).
    const double full = std::max(0.0, waves - 1.0);
    const double first = std::min<double>(units, sms);
    const double last = std::min<double>(sms, std::max(1.0, units - full * sms));
    const double per_unit = (opnd_bytes + extra_bytes) / std::max(1.0, units);
    auto rate = [&](double n) { return std::min(kHbmBytesPerClkPerSm * sms, kSmStreamBytesPerClk * n); };
    const double mem = (full * first * per_unit / rate(first) + last * per_unit / rate(last)) * (sk ? (bn >= 128 ? 1.15 : 1.08) : 1.0);
    const double t = std::max(compute, mem) * (1.0 + 0.002 * seff);
    if (t < best) {
      best = t;
      pl.est = t;
      pl.bn = bn; pl.splits = seff; pl.a_mn = am; pl.b_mn = bm;
      pl.tiles_m = ceil_div(o.M, 128 * pair); pl.tiles_n = ceil_div(o.N, bn);
      pl.kb_total = kb_total; pl.kb_per_split = kbp;
      pl.dp_tiles = dp; pl.tail_half = half; pl.pair = pair;
      pl.sk = sk; pl.sk_ctas = sk ? sms : 0;
    }
  };
  for (int bn : bns) {
    if (force_bn && bn != force_bn) continue;
    if (s3 && bn > 128) continue;  // 3xTF32: see launch_tc<float>
    // 512 columns: CTA pairs only, whole tiles only (below)
    const bool wide = bn > 256;
    int am, bm;
    if (!tc_layout_ok(o, bn, am, bm, nullptr)) continue;
    if (!force_bn && bn > 16 && round_up(o.N, 16) <= bn / 2) continue;  // a smaller tile already covers N
    const int64_t tiles = o.batch * ceil_div(o.M, 128) * ceil_div(o.N, bn);
    const double unit_full = kb_total * kbc(bn) + 4.0 * bn;
    if (!wide && (!force_split || force_split == 1) && force_pair != 2 && force_sk != 2) {
      // whole tiles
      const int64_t w = ceil_div(tiles, sms);
      consider(w * unit_full, (double)tiles, (double)w, 0.0, bn, am, bm, 1, kb_total, tiles, 0);
      // whole tiles for the full waves, half-width units for the tiles left over
      const bool half_ok = bn >= 128 && (!bm || (bn / 2) * esz >= 128);
      if (half_ok && tiles > sms && tiles % sms) {
        const int64_t dp = (tiles / sms) * sms;
        const int64_t tail_units = 2 * (tiles - dp);
        const double unit_half = kb_total * kbc(bn / 2) + 2.0 * bn;
        const double waves = (double)(dp / sms + ceil_div(tail_units, sms));
        consider((dp / sms) * unit_full + ceil_div(tail_units, sms) * unit_half, (double)(dp + tail_units), waves,
                 0.0, bn, am, bm, 1, kb_total, dp, 1);
      }
    }
    // CTA pairs: 256-row tiles on sms/2 pairs, whole tiles (+ half-width tail)
    // a CTA of the pair loads bn/2 columns of B: an MN-major box is 128 bytes wide
    const bool pair_fits = !bm || (bn / 2) * esz >= 128;
    // Pairs pay a cross-CTA handshake per tile (both epilogues must drain an
    // accumulator before the next MMA): only worth it with enough K per tile.
    // (3xTF32 is bound by its three tf32 MMAs, not by operand traffic: pairs
    // measured no faster at 4096^3 and slower at 8192^3, so only on request)
    const bool want_pair = s3 ? (bn == 128 && force_pair == 2)
                              : (force_pair == 2 || (force_pair == 0 && g_pair_enabled && o.M > 128 && kb_total >= 8));
    if ((bn == 128 || bn == 256 || (wide && (g_pair_wide || force_bn == 512))) && pair_fits && want_pair &&
        (!force_split || force_split == 1)) {
      const int pairs = sms / 2;
      const int64_t ptiles = o.batch * ceil_div(o.M, 256) * ceil_div(o.N, bn);
      // The 512-wide tile's one accumulator leaves its epilogue exposed
      // (about 12 cycles per column): it pays off through its 25% fewer
      // operand bytes per FLOP when there are tiles enough to fill the pairs.
      const double punit = kb_total * kbcp(bn) + (wide ? 12.0 : 4.0) * bn;
      const int64_t w = ceil_div(ptiles, pairs);
      if (force_sk != 2) consider(w * punit, (double)ptiles * 2, (double)w, 0.0, bn, am, bm, 1, kb_total, ptiles, 0, 2);
      if (wide) continue;
      const bool half_ok = bn == 256 && bm && (bn / 4) * esz >= 128 && force_sk != 2;
      if (half_ok && ptiles > pairs && ptiles % pairs) {
        const int64_t dp = (ptiles / pairs) * pairs;
        const int64_t tail_units = 2 * (ptiles - dp);
        const double phalf = kb_total * kbcp(bn / 2) + 2.0 * bn;
        const double waves = (double)(dp / pairs + ceil_div(tail_units, pairs));
        consider((dp / pairs) * punit + ceil_div(tail_units, pairs) * phalf, (double)(dp + tail_units) * 2, waves,
                 0.0, bn, am, bm, 1, kb_total, dp, 1, 2);
      }
      // stream-K tail on pairs: whole 256-row tiles for the full waves, the
      // tiles left over cut into equal K-block ranges, one per pair (each CTA
      // of a pair publishes and reduces its own 128 rows)
      if (have_ws && (g_pair_sk || force_sk == 2) && force_sk != 1 && !force_split && !s3 && ptiles % pairs) {
        const int64_t dp = (ptiles / pairs) * pairs;
        const int64_t tail = ptiles - dp;
        const int64_t iters = tail * kb_total;
        if ((iters >= 4 * (int64_t)pairs || (force_sk == 2 && iters >= pairs)) &&
            tail * 2 * tc::NUM_EPI_WARPS <= kMaxTickets) {
          const int maxp = sk_max_parts(tail, kb_total, pairs);
          const double share = (double)ceil_div(iters, pairs) * kbcp(bn);
          const double fix = maxp > 1 ? 8.0 * 4.0 * bn + 8.0 * maxp * bn : 4.0 * bn;
          const double extra = maxp > 1 ? (double)tail * maxp * 256.0 * bn * 8.0 : 0.0;
          consider((dp / pairs) * punit + share + fix, (double)(dp + pairs) * 2, (double)(dp / pairs + 1), extra,
                   bn, am, bm, maxp, kb_total, dp, 0, 2, 1);
        }
      }
    }
    if (wide) continue;
    // stream-K tail: whole tiles for the full waves, the tiles left over cut
    // into equal K-block ranges, one per CTA (every CTA busy to the end)
    if (have_ws && force_pair != 2 && force_sk != 1 && !force_split && tiles % sms) {
      const int64_t dp = (tiles / sms) * sms;
      const int64_t tail = tiles - dp;
      const int64_t iters = tail * kb_total;
      if (iters >= 4 * (int64_t)sms || (force_sk == 2 && iters >= sms)) {
        const int maxp = sk_max_parts(tail, kb_total, sms);
        if (tail * tc::NUM_EPI_WARPS <= kMaxTickets) {
          const double share = (double)ceil_div(iters, sms) * kbc(bn);
          // the fixup: the last piece of a tile re-reads every partial of it
          const double fix = maxp > 1 ? 8.0 * 4.0 * bn + 8.0 * maxp * bn : 4.0 * bn;
          const double extra = maxp > 1 ? (double)tail * maxp * 128.0 * bn * 8.0 : 0.0;
          consider((dp / sms) * unit_full + share + fix, (double)(dp + sms), (double)(dp / sms + 1), extra, bn, am,
                   bm, maxp, kb_total, dp, 0, 1, 1);
        }
      }
    }
    if (force_sk == 2) continue;
    // every tile split along K (long-K, few tiles: skinny and thin shapes)
    int max_split = have_ws && force_pair != 2 ? (int)std::min<int64_t>(kb_total, 64) : 1;
    if (tiles * tc::NUM_EPI_WARPS > kMaxTickets) max_split = 1;  // ticket counters
    for (int s = 2; s <= max_split; ++s) {
      if (force_split && s != force_split) continue;
      const int64_t kbp = ceil_div(kb_total, s);
      const int64_t seff = ceil_div(kb_total, kbp);
      if (seff != s && !force_split) continue;
      // a split unit writes 128 x BN fp32 partials and the last warp to arrive
      // re-reads all of them before the epilogue: measured far costlier than a
      // whole-tile epilogue, so it is charged per split and per column
      const double unit_split = kbp * kbc(bn) + 4.0 * bn + 16.0 * seff * bn;
      const int64_t units = tiles * seff;
      // splits fill one wave; past that a stream-K tail balances the same work
      // with fewer fix-ups (measured on B200: thin 224-tile shapes, split 3-4
      // at 0.87-0.91x the stream-K time)
      if (!force_split && units > sms) continue;
      const int64_t w = ceil_div(units, sms);
      consider(w * unit_split, (double)units, (double)w, (double)tiles * seff * 128.0 * bn * 8.0, bn, am, bm,
               (int)seff, kbp, 0, 0);
    }
  }
}

// The tile choice is a pure function of the operands' shapes, strides and
// alignment and of the overrides: memoised per thread so that a repeated call
// (the usual case: the same layer every step) skips the cost-model search.
struct TileKey {
  int64_t v[20];
  bool operator==(const TileKey &k) const { return memcmp(v, k.v, sizeof(v)) == 0; }
};
struct TileKeyHash {
  size_t operator()(const TileKey &k) const {
    uint64_t h = 1469598103934665603ull;
    for (int64_t x : k.v) { h ^= (uint64_t)x; h *= 1099511628211ull; }
    return (size_t)h;
  }
};
struct TileChoice {
  int bn, splits, a_mn, b_mn, tail_half, pair, sk;
  int64_t tiles_m, tiles_n, kb_total, kb_per_split, dp_tiles, sk_ctas;
  double est;
};

void choose_tc_tile(const Op &o, int sms, int force_bn, int force_split, int force_pair, int force_sk, bool have_ws,
                    Plan &pl) {
  const int esz = elem_size(o.dt);
  TileKey k;
  int64_t *v = k.v;
  v[0] = o.dt; v[1] = o.M; v[2] = o.N; v[3] = o.K; v[4] = o.batch;
  v[5] = o.a_rs; v[6] = o.a_cs; v[7] = o.b_rs; v[8] = o.b_cs;
  v[9] = o.sA == 0 ? -1 : (o.sA * esz) % 16;  // broadcast, else whether TMA can step batches
  v[10] = o.sB == 0 ? -1 : (o.sB * esz) % 16;
  v[11] = (o.sA < 0) | ((o.sB < 0) << 1);
  v[12] = (int64_t)(reinterpret_cast<uintptr_t>(o.A) & 15) | ((int64_t)(reinterpret_cast<uintptr_t>(o.B) & 15) << 8);
  v[13] = sms; v[14] = force_bn; v[15] = force_split; v[16] = force_pair; v[17] = force_sk; v[18] = have_ws;
  v[19] = 0;
  thread_local std::unordered_map<TileKey, TileChoice, TileKeyHash> cache;
  auto it = cache.find(k);
  if (it == cache.end()) {
    Plan t;
    t.bn = 0;
    choose_tc_tile_uncached(o, sms, force_bn, force_split, force_pair, force_sk, have_ws, t);
    if (cache.size() >= 4096) cache.clear();
    it = cache.emplace(k, TileChoice{t.bn, t.splits, t.a_mn, t.b_mn, t.tail_half, t.pair, t.sk, t.tiles_m, t.tiles_n,
                                     t.kb_total, t.kb_per_split, t.dp_tiles, t.sk_ctas, t.est}).first;
  }
  const TileChoice &c = it->second;
  if (!c.bn) return;  // no tile fits: pl untouched, as the search leaves it
  pl.bn = c.bn; pl.splits = c.splits; pl.a_mn = c.a_mn; pl.b_mn = c.b_mn; pl.tail_half = c.tail_half;
  pl.pair = c.pair; pl.sk = c.sk; pl.tiles_m = c.tiles_m; pl.tiles_n = c.tiles_n; pl.kb_total = c.kb_total;
  pl.kb_per_split = c.kb_per_split; pl.dp_tiles = c.dp_tiles; pl.sk_ctas = c.sk_ctas; pl.est = c.est;
}

// Fill pl for the TC path on operands o (possibly swapped); false if TMA can't.
bool plan_tc(const Op &o, int sms, const mb_gemm_desc *d, bool have_ws, Plan &pl) {
  pl.bn = 0;
  choose_tc_tile(o, sms, d->tile_n, d->split_k, d->cta_pair, d->stream_k, have_ws, pl);
  if (!pl.bn) return false;
  pl.kind = PK_TC;
  const int64_t tiles = o.batch * pl.tiles_m * pl.tiles_n;
  if (pl.splits > 1 && tiles > pl.dp_tiles) {
    // one BM x BN slot per piece and per CTA of a pair
    pl.ws_bytes = kTicketBytes + (tiles - pl.dp_tiles) * pl.splits * pl.pair * 128 * pl.bn * 4;
  } else if (!pl.tail_half) {
    pl.splits = 1;
    pl.dp_tiles = tiles;
    pl.sk = 0;
  }
  return true;
}

// The real fp16 GEMM that computes a complex32 product (see c32.cuh): A' is A's
// storage viewed as M x 2K halves (or a packed copy at `a`), B' the expanded
// 2K x 2N matrix at `b`, C' is C's storage viewed as M x 2N halves.
Op c32_inner(const Op &o, const Plan &pl, const void *a, const void *b) {
  Op r = o;
  r.dt = MB_F16;
  r.N = 2 * o.N;
  r.K = 2 * o.K;
  if (pl.c32_pack_a) {
    r.A = a; r.a_rs = 2 * pl.c32_lda; r.a_cs = 1; r.sA = o.sA ? o.M * 2 * pl.c32_lda : 0;
  } else {
    r.a_rs = 2 * o.a_rs; r.a_cs = 1; r.sA = 2 * o.sA;
  }
  r.B = b; r.b_rs = 2 * pl.c32_ldb; r.b_cs = 1; r.sB = o.sB ? 2 * o.K * 2 * pl.c32_ldb : 0;
  r.c_rs = 2 * o.c_rs; r.c_cs = 1; r.sC = 2 * o.sC;
  r.conj_a = r.conj_b = 0;
  return r;  // bias keeps its complex strides: the epilogue reads half2 pairs
}

bool plan_c32(const Op &o, int sms, const mb_gemm_desc *d, bool have_ws, Plan &pl) {
  if (o.dt != MB_C32 || o.M < 2 || o.N < 2 || o.K < 1 || !have_ws) return false;
  if (o.c_cs != 1 || o.c_rs < o.N) return false;  // C' must be a row-major real view
  if (o.K >= (1ll << 30) || o.N >= (1ll << 30)) return false;
  Plan t;
  t.c32_pack_a = !(o.a_cs == 1 && o.a_rs >= o.K && o.a_rs % 4 == 0 && aligned16(o.A) &&
                   (o.batch <= 1 || o.sA % 4 == 0));
  t.c32_lda = round_up(o.K, 4);
  t.c32_ldb = round_up(o.N, 4);
  t.c32_a_batches = o.sA ? o.batch : 1;
  t.c32_b_batches = o.sB ? o.batch : 1;
  // plan the real GEMM on placeholder (aligned) operand addresses; no swap:
  // the complex epilogue needs both halves of a pair in one thread
  const void *ph = reinterpret_cast<const void *>(uintptr_t(1) << 20);
  Op r = c32_inner(o, t, ph, ph);
  mb_gemm_desc q = *d;
  q.swap_ab = -1;
  if (!plan_tc(r, sms, &q, have_ws, t)) return false;
  // after the ticket region (and any split-K partials): the counters at offset 0
  // are shared by every plan and must never be overwritten
  const int64_t base = std::max<int64_t>(t.ws_bytes, kTicketBytes);
  const int64_t a_bytes = t.c32_pack_a ? t.c32_a_batches * o.M * t.c32_lda * 4 : 0;
  const int64_t b_bytes = t.c32_b_batches * 2 * o.K * t.c32_ldb * 4;
  t.c32_a_off = round_up(base, 256);
  t.c32_b_off = round_up(t.c32_a_off + a_bytes, 256);
  t.ws_bytes = t.c32_b_off + b_bytes;
  t.kind = PK_TC_C32;
  pl = t;
  return true;
}

// TMA can load this operand (rows x cols, strides rs / cs, batch stride bs) in
// place: 16-byte aligned base, a unit stride, and the other stride and the
// batch stride multiples of 16 bytes.
bool operand_tma_ok(const void *ptr, int64_t rows, int64_t cols, int64_t rs, int64_t cs, int64_t bs, int64_t batch,
                    int esz) {
  if (!aligned16(ptr)) return false;
  if (batch > 1 && (bs < 0 || (bs * esz) % 16)) return false;
  if (cs == 1 && rs >= cols && (rs * esz) % 16 == 0) return true;
  if (rs == 1 && cs >= rows && (cs * esz) % 16 == 0) return true;
  return false;
}

// The TC GEMM on operands of which at least one TMA cannot address (the
// reference's "offset" view A[1:, 1:] with lda = K+1, odd pitches, no unit
// stride): those are copied into the workspace first.  The reference copies
// such views with .contiguous() (metalblas/dispatch.py:33-35); here the copy
// goes to aligned scratch and the product still runs on the tensor cores.
Op packed_op(const Op &o, const Plan &t, const void *a, const void *b) {
  Op r = o;
  if (t.pk_a) {
    r.A = a;
    if (t.pk_a_cm) { r.a_rs = 1; r.a_cs = t.pk_lda; r.sA = o.sA ? o.K * t.pk_lda : 0; }
    else { r.a_rs = t.pk_lda; r.a_cs = 1; r.sA = o.sA ? o.M * t.pk_lda : 0; }
  }
  if (t.pk_b) {
    r.B = b;
    if (t.pk_b_cm) { r.b_rs = 1; r.b_cs = t.pk_ldb; r.sB = o.sB ? o.N * t.pk_ldb : 0; }
    else { r.b_rs = t.pk_ldb; r.b_cs = 1; r.sB = o.sB ? o.K * t.pk_ldb : 0; }
  }
  return r;
}

bool plan_tc_any(const Op &o, int sms, const mb_gemm_desc *d, bool have_ws, Plan &pl);

bool plan_packed(const Op &o, int sms, const mb_gemm_desc *d, bool have_ws, Plan &pl) {
  if (!is_tc_dtype(o.dt) || !have_ws || o.M < 1 || o.N < 1 || o.K < 1) return false;
  if (o.M >= (1ll << 31) || o.N >= (1ll << 31) || o.K >= (1ll << 31)) return false;
  const int esz = elem_size(o.dt);
  Plan t;
  t.pk_a = !operand_tma_ok(o.A, o.M, o.K, o.a_rs, o.a_cs, o.sA, o.batch, esz);
  t.pk_b = !operand_tma_ok(o.B, o.K, o.N, o.b_rs, o.b_cs, o.sB, o.batch, esz);
  if (!t.pk_a && !t.pk_b) return false;
  // keep the source's contiguous direction so the copy reads and writes rows
  t.pk_a_cm = o.a_rs == 1 && o.a_cs != 1;
  t.pk_b_cm = o.b_rs == 1 && o.b_cs != 1;
  t.pk_lda = round_up(t.pk_a_cm ? o.M : o.K, 16 / esz);
  t.pk_ldb = round_up(t.pk_b_cm ? o.K : o.N, 16 / esz);
  t.pk_a_batches = o.sA ? o.batch : 1;
  t.pk_b_batches = o.sB ? o.batch : 1;
  const void *ph = reinterpret_cast<const void *>(uintptr_t(1) << 20);  // aligned placeholder
  const Op r = packed_op(o, t, ph, ph);
  if (!plan_tc_any(r, sms, d, have_ws, t)) return false;
  const int64_t base = std::max<int64_t>(t.ws_bytes, kTicketBytes);
  const int64_t a_bytes = t.pk_a ? t.pk_a_batches * (t.pk_a_cm ? o.K : o.M) * t.pk_lda * esz : 0;
  const int64_t b_bytes = t.pk_b ? t.pk_b_batches * (t.pk_b_cm ? o.N : o.K) * t.pk_ldb * esz : 0;
  t.pk_a_off = round_up(base, 256);
  t.pk_b_off = round_up(t.pk_a_off + a_bytes, 256);
  t.ws_bytes = t.pk_b_off + b_bytes;
  t.kind = PK_TC_PACKED;
  pl = t;
  return true;
}

// fp32 on the tensor cores as 3xTF32 (METALBLAS_FP32_TF32X3=0 keeps every fp32
// product on the CUDA-core FFMA kernel).  The split operands live in the
// workspace, K-major: A' = [batch][M][ldk], B'ᵀ = [batch][N][ldk].
const bool g_fp32_tf32x3 = [] {
  const char *s = getenv("METALBLAS_FP32_TF32X3");
  return !(s && s[0] == '0');
}();

Op x3_op(const Op &o, const Plan &t, const void *ahi, const void *alo, const void *bhi, const void *blo) {
  Op r = o;
  r.A = ahi; r.A2 = alo; r.a_rs = t.x3_ldk; r.a_cs = 1; r.sA = o.sA ? o.M * t.x3_ldk : 0;
  r.B = bhi; r.B2 = blo; r.b_rs = 1; r.b_cs = t.x3_ldk; r.sB = o.sB ? o.N * t.x3_ldk : 0;
  return r;
}

bool plan_3xtf32(const Op &o, int sms, const mb_gemm_desc *d, bool have_ws, Plan &pl) {
  if (o.dt != MB_F32 || !have_ws || o.M < 1 || o.N < 1 || o.K < 1) return false;
  if (o.M >= (1ll << 31) || o.N >= (1ll << 31) || o.K >= (1ll << 31)) return false;
  // A product with non-finite inputs is recomputed on the CUDA cores after the
  // tensor-core pass, which must then still see the original bias: an epilogue
  // whose bias is the output itself runs on the CUDA cores from the start.
  if (d->epilogue && d->beta_nz && d->bias == d->C) return false;
  Plan t;
  t.x3_ldk = round_up(o.K, 4);
  t.x3_a_batches = o.sA ? o.batch : 1;
  t.x3_b_batches = o.sB ? o.batch : 1;
  const void *ph = reinterpret_cast<const void *>(uintptr_t(1) << 20);  // aligned placeholder
  if (!plan_tc_any(x3_op(o, t, ph, ph, ph, ph), sms, d, have_ws, t)) return false;
  if (t.a_mn || t.b_mn) return false;
  const int64_t base = std::max<int64_t>(t.ws_bytes, kTicketBytes);
  const int64_t a_bytes = t.x3_a_batches * o.M * t.x3_ldk * 4, b_bytes = t.x3_b_batches * o.N * t.x3_ldk * 4;
  t.x3_ahi = round_up(base, 256);
  t.x3_alo = round_up(t.x3_ahi + a_bytes, 256);
  t.x3_bhi = round_up(t.x3_alo + a_bytes, 256);
  t.x3_blo = round_up(t.x3_bhi + b_bytes, 256);
  t.x3_flag = round_up(t.x3_blo + b_bytes, 256);
  t.ws_bytes = t.x3_flag + 256;
  t.kind = PK_TC_3XTF32;
  pl = t;
  return true;
}

EpiScalars make_epi(const mb_gemm_desc *d);

// complex64 as one real fp32 GEMM on the tensor cores through 3xTF32, in the
// block form of c32.cuh: C' [M x 2N] (C's storage) = A' [M x 2K] B' [2K x 2N].
// The split pass reads the complex operands directly (SplitArgs modes 1 and 2),
// so A and B keep their complex strides here.  The reference computes complex64
// as real products on its fp32 path (metalblas/complex_dispatch.py:69-115).
Op c64_real(const Op &o) {
  Op r = o;
  r.dt = MB_F32;
  r.N = 2 * o.N;
  r.K = 2 * o.K;
  r.c_rs = 2 * o.c_rs; r.c_cs = 1; r.sC = 2 * o.sC;
  r.bias_rs = 2 * o.bias_rs; r.bias_cs = 1; r.bias_bs = 2 * o.bias_bs;
  r.conj_a = r.conj_b = 0;
  return r;
}

bool plan_c64x3(const Op &o, int sms, const mb_gemm_desc *d, bool have_ws, Plan &pl) {
  if (o.dt != MB_C64 || !have_ws || o.M < 1 || o.N < 1 || o.K < 1) return false;
  if (o.c_cs != 1 || o.c_rs < o.N) return false;  // C' must be a row-major real view
  if (o.N >= (1ll << 30) || o.K >= (1ll << 30)) return false;
  // the real epilogue applies alpha / beta per component: real scalars only,
  // and a bias whose components sit next to each other along N
  const EpiScalars e = make_epi(d);
  if (e.enabled && (e.alpha_im != 0.f || e.beta_im != 0.f)) return false;
  if (e.enabled && e.beta_nz && o.bias_cs != 1) return false;
  if (!plan_3xtf32(c64_real(o), sms, d, have_ws, pl)) return false;
  pl.kind = PK_TC_C64X3;
  return true;
}

// ---------------------------------------------------------------------------
// 16/32/64-bit integer products on the 8-bit tensor cores.  An L-byte integer
// is the sum of its unsigned bytes a_l * 2^(8l) modulo 2^(8L) (two's
// complement), so modulo 2^(8L)
//   C = A B = sum over s < L of 2^(8s) * P_s,   P_s = sum over i + j = s of A_i B_j,
// and each P_s is ONE u8 x u8 GEMM over K' = (s+1) kp: A_cat = [A_0 | ... | A_{L-1}]
// (M x L*kp, byte planes side by side along K) and B_rev = [B_{L-1}; ...; B_0]
// (stored transposed, N x L*kp), so P_s = A_cat[:, :(s+1)kp] @ B_rev[(L-1-s)kp:, :].
// P_s lands in C through the epilogue, C = alpha * 2^(8s) * P_s + C with
// wrapping integer arithmetic, the first GEMM with the caller's beta * bias.
// The s32 accumulators stay exact while L * kp * 255^2 < 2^31; a longer K runs
// in chunks.  Bit-exact like the CUDA-core IMAD kernel (metalblas/shaders/
// int_gemm.h:41-154 is the reference's register-tiled integer GEMM).
const bool g_int_limbs = [] {
  const char *s = getenv("METALBLAS_INT_LIMBS");
  return !(s && s[0] == '0');
}();
int limb_planes(int dt) { return dt == MB_I16 ? 2 : dt == MB_I32 ? 4 : dt == MB_I64 ? 8 : 0; }

Op limb_gemm_op(const Op &o, const Plan &t, int s, const void *acat, const void *brev) {
  Op r = o;
  r.dt = MB_U8;
  r.K = (int64_t)(s + 1) * t.limb_kp;
  r.A = acat; r.a_rs = t.limb_ld; r.a_cs = 1; r.sA = o.sA ? o.M * t.limb_ld : 0;
  r.B = static_cast<const uint8_t *>(brev) + (int64_t)(t.limb_L - 1 - s) * t.limb_kp;
  r.b_rs = 1; r.b_cs = t.limb_ld; r.sB = o.sB ? o.N * t.limb_ld : 0;
  r.conj_a = r.conj_b = 0;
  return r;  // C and bias stay the caller's; the epilogue chain sets them per GEMM
}

// Plan of GEMM s of the chain over the tile widths that have integer-output
// kernels; split-K / stream-K tails are allowed (their u32 partial sums are
// exact: the products are summed modulo 2^32, or stay below 2^31 for int64).
bool limb_gemm_plan(const Op &o, const Plan &t, int s, int sms, Plan &g) {
  const void *ph = reinterpret_cast<const void *>(uintptr_t(1) << 20);  // aligned placeholder
  const Op r = limb_gemm_op(o, t, s, ph, ph);
  mb_gemm_desc q;
  mb_gemm_desc_init(&q);
  bool ok = false;
  double best = 1e300;
  for (int bn : {64, 128, 256}) {
    q.tile_n = bn;
    Plan c;
    if (!plan_tc_any(r, sms, &q, true, c)) continue;
    if (c.pair == 2 && c.bn != 128 && c.bn != 256) continue;
    if (c.est < best) { best = c.est; g = c; ok = true; }
  }
  return ok;
}

bool plan_limb(const Op &o, int sms, const mb_gemm_desc *d, bool have_ws, Plan &pl) {
  (void)d;
  const int L = limb_planes(o.dt);
  if (!L || !have_ws || o.M < 1 || o.N < 1 || o.K < 1) return false;
  if (o.M >= (1ll << 31) || o.N >= (1ll << 31)) return false;
  const int64_t kp_max = (33024 / L) / 16 * 16;  // L * kp * 255^2 < 2^31
  Plan t;
  t.limb_L = L;
  t.limb_kc = std::min<int64_t>(o.K, kp_max);
  t.limb_kp = round_up(t.limb_kc, 16);
  t.limb_ld = L * t.limb_kp;
  t.limb_a_batches = o.sA ? o.batch : 1;
  t.limb_b_batches = o.sB ? o.batch : 1;
  // the GEMMs' tickets and split-K partials come first (at the workspace
  // base, as for every plan), then the planes
  int64_t gemm_ws = kTicketBytes;
  Plan g;  // the last (widest) GEMM of the chain, for the plan's description
  for (int s = 0; s < L; ++s) {
    if (!limb_gemm_plan(o, t, s, sms, g)) return false;
    gemm_ws = std::max<int64_t>(gemm_ws, g.ws_bytes);
  }
  const int64_t a_bytes = t.limb_a_batches * o.M * t.limb_ld, b_bytes = t.limb_b_batches * o.N * t.limb_ld;
  t.limb_a_off = round_up(gemm_ws, 256);
  t.limb_b_off = round_up(t.limb_a_off + a_bytes, 256);
  t.ws_bytes = t.limb_b_off + b_bytes;
  t.bn = g.bn; t.pair = g.pair; t.swap = g.swap; t.tiles_m = g.tiles_m; t.tiles_n = g.tiles_n; t.est = g.est;
  t.kind = PK_TC_LIMB;
  pl = t;
  return true;
}

int gemv_cols_per_sm(int dt, int mr);

// Thin products the column GEMV runs with several x rows sharing each load of
// W (the gemv_bt role, metalblas/shaders/gemv_bt.h:47-269): 16/32-bit floats,
// up to kGemvMaxRows rows (fp32: kGemvMaxRowsF32, in blocks of 8).
constexpr int kGemvMaxRows = 4;
constexpr int kGemvMaxRowsF32 = 32;
bool gemv_thin_dtype(int dt) { return dt == MB_BF16 || dt == MB_F16 || dt == MB_F32; }
int64_t gemv_max_rows(int dt) { return dt == MB_F32 ? kGemvMaxRowsF32 : kGemvMaxRows; }
// rows per CTA block (the kernel's MR)
int gemv_mr(int dt, int64_t mrows) {
  if (mrows <= 1) return 1;
  if (mrows == 2) return 2;
  return (dt == MB_F32 && mrows > 4) ? 8 : 4;
}

bool plan_gemv(const Op &o, int sms, const mb_gemm_desc *d, bool have_ws, Plan &pl) {
  GemvParams g{};
  g.mrows = 1;
  int kind = 0;
  if (o.M == 1) {
    // y[n] = sum_k A(0,k) B(k,n): W = B
    g.R = o.N; g.K = o.K; g.W = o.B; g.X = o.A; g.x_s = o.a_cs; g.y_s = o.c_cs; g.bias_s = o.bias_cs;
    g.sW = o.sB; g.sX = o.sA; g.conj_w = o.conj_b; g.conj_x = o.conj_a;
    if (o.b_cs == 1) { kind = PK_GEMV_COLS; g.w_ld = o.b_rs; }
    else if (o.b_rs == 1) { kind = PK_GEMV_ROWS; g.w_ld = o.b_cs; }
  } else if (o.N == 1) {
    // y[m] = sum_k A(m,k) B(k,0): W = A
    g.R = o.M; g.K = o.K; g.W = o.A; g.X = o.B; g.x_s = o.b_rs; g.y_s = o.c_rs; g.bias_s = o.bias_rs;
    g.sW = o.sA; g.sX = o.sB; g.conj_w = o.conj_a; g.conj_x = o.conj_b;
    if (o.a_cs == 1) { kind = PK_GEMV_ROWS; g.w_ld = o.a_rs; }
    else if (o.a_rs == 1) { kind = PK_GEMV_COLS; g.w_ld = o.a_cs; }
  }
  if (!kind && gemv_thin_dtype(o.dt) && o.M <= gemv_max_rows(o.dt) && o.b_cs == 1) {
    // thin M: y[m][n] = sum_k A(m,k) B(k,n), W = B (row-major) read once
    g.R = o.N; g.K = o.K; g.W = o.B; g.X = o.A; g.x_s = o.a_cs; g.y_s = o.c_cs; g.bias_s = o.bias_cs;
    g.sW = o.sB; g.sX = o.sA; g.conj_w = o.conj_b; g.conj_x = o.conj_a;
    g.mrows = (int)o.M; g.x_rs = o.a_rs; g.y_rs = o.c_rs; g.bias_rs = o.bias_rs;
    kind = PK_GEMV_COLS; g.w_ld = o.b_rs;
  } else if (!kind && gemv_thin_dtype(o.dt) && o.N <= gemv_max_rows(o.dt) && o.a_rs == 1) {
    // thin N: the transposed product, W = A (column-major), x rows = B's columns
    g.R = o.M; g.K = o.K; g.W = o.A; g.X = o.B; g.x_s = o.b_rs; g.y_s = o.c_rs; g.bias_s = o.bias_rs;
    g.sW = o.sA; g.sX = o.sB; g.conj_w = o.conj_a; g.conj_x = o.conj_b;
    g.mrows = (int)o.N; g.x_rs = o.b_cs; g.y_rs = o.c_cs; g.bias_rs = o.bias_cs;
    kind = PK_GEMV_COLS; g.w_ld = o.a_cs;
  }
  if (!kind) return false;
  g.Y = o.C; g.bias = o.bias; g.batch = o.batch; g.sY = o.sC; g.sBias = o.bias_bs;
  const int esz = elem_size(o.dt);
  const int vmax = 16 / esz;
  const bool wvec = aligned16(g.W) && (g.w_ld % vmax == 0) && (o.batch <= 1 || (g.sW % vmax == 0));
  pl.vec = wvec ? vmax : 1;
  if (g.mrows > 1 && pl.vec == 1) return false;  // thin kernels are vectorised only
  const int mr = gemv_mr(o.dt, g.mrows);
  g.mrb = (int)ceil_div(g.mrows, mr);

  g.x_vec = (g.x_s == 1 && aligned16(g.X) && (o.batch <= 1 || g.sX % vmax == 0)) ? 1 : 0;
  g.ksplit = 1;
  g.kchunk = std::max<int64_t>(g.K, 1);
  if (kind == PK_GEMV_COLS) {
    const int64_t cols_per_cta = 32 * pl.vec;
    const int64_t ctas_x = ceil_div(g.R, cols_per_cta);
    pl.gemv_ctas_x = ctas_x;
    // K split by wave efficiency: the CTAs (column blocks x row blocks x
    // batches x splits) should fill whole waves of the resident slots; a
    // nearly empty last wave leaves most SMs idle while it streams (672 CTAs
    // on 592 slots measured 0.78 of HBM at N = 28672, 560 CTAs 0.96).  Each
    // extra split costs ~1% (partials, a shorter stream per CTA).
    const int64_t slots = (int64_t)gemv_cols_per_sm(o.dt, mr) * sms;
    const int64_t zb = o.batch * g.mrb;  // CTAs per K chunk: column blocks x row blocks x batches
    // whole unrolled steps per chunk: 8 warps x 8 rows in flight per lane
    auto chunk_of = [&](int64_t k) { return round_up(ceil_div(g.K, k), 64); };
    const int64_t ks_cap = std::min<int64_t>({ceil_div(g.K, 64), 65535, 3 * std::max<int64_t>(1, slots / (ctas_x * zb)) + 2});
    int64_t ks = 1;
    if (d->split_k > 0) {
      ks = std::min<int64_t>(d->split_k, std::min<int64_t>(ceil_div(g.K, 64), 65535));
    } else {
      double best = -1.0;
      for (int64_t k = 1; k <= ks_cap; ++k) {
        const int64_t eff_k = ceil_div(g.K, chunk_of(k));
        if (eff_k != k) continue;
        const double units = (double)(ctas_x * zb * k);
        const double waves = std::ceil(units / (double)slots);
        const double score = units / (waves * slots) * (1.0 - 0.01 * (k - 1));
        if (score > best + 1e-9) { best = score; ks = k; }
      }
    }
    ks = std::max<int64_t>(1, ks);
    if (ks > 1 && !have_ws) ks = 1;
    if (zb * ctas_x > kMaxTickets) ks = 1;  // not enough ticket counters
    if (ks > 1) {
      g.kchunk = chunk_of(ks);
      ks = ceil_div(g.K, g.kchunk);
    }
    g.ksplit = (int)ks;
    if (ks > 1) {
      const int64_t accb = acc_is_8byte(o.dt) ? 8 : 4;
      pl.ws_bytes = kTicketBytes + ks * o.batch * g.mrows * g.R * accb;
    }
  } else if (pl.vec > 1 && g.x_vec) {
    // Staged-x rows kernel: CTAs of kGemvRowsPerCta rows.  A short CTA pays a
    // fixed cost of about two memory round trips (x staging, launch, ticket),
    // so K is split only when rows are long (>= 32 KB) and there are enough
    // row groups to fill the machine; each split CTA then streams 8 KB per
    // row (four unrolled steps of a warp).  Measured on B200 over K in
    // {4096, 8192, 16384} x R in {4096, 14336, 28672} for fp32/fp16/bf16.
    const int64_t rg = ceil_div(g.R, kGemvRowsPerCta);
    const int64_t slots = (int64_t)sms * (acc_is_8byte(o.dt) ? 2 : 3);  // launch-bounds minimum
    const int64_t align = 2048 / esz;  // one unrolled step of a warp: 4 x 32 lanes x 16 bytes
    const int64_t row_bytes = g.K * esz;
    int64_t best_ks = 1;
    if (row_bytes >= 32768 && rg * o.batch >= slots) best_ks = std::min<int64_t>(64, row_bytes / 8192);
    if (!have_ws || o.batch * rg > kMaxTickets) best_ks = 1;
    int64_t ks = best_ks;
    if (d->split_k > 0 && have_ws && o.batch * rg <= kMaxTickets)
      ks = std::min<int64_t>(d->split_k, std::max<int64_t>(1, g.K / align));
    if (ks > 1) {
      g.kchunk = ceil_div(ceil_div(g.K, ks), align) * align;
      ks = ceil_div(g.K, g.kchunk);
    }
    g.ksplit = (int)ks;
    if (ks > 1) {
      const int64_t accb = acc_is_8byte(o.dt) ? 8 : 4;
      pl.ws_bytes = kTicketBytes + ks * o.batch * g.R * accb;
    }
  }
  pl.kind = kind;
  pl.g = g;
  return true;
}

int make_plan(const mb_gemm_desc *d, const Op &o, int sms, bool have_ws, Plan &pl) {
  if (o.M == 0 || o.N == 0 || o.batch == 0) { pl.kind = PK_EMPTY; return MB_OK; }
  const int be = d->backend;
  if (be == MB_BACKEND_GEMV) {
    const bool thin = gemv_thin_dtype(o.dt) && std::min(o.M, o.N) <= gemv_max_rows(o.dt);
    if (!(o.M == 1 || o.N == 1 || thin))
      return fail(MB_ERR_INVALID, "gemv backend requires M==1 or N==1 (or min(M, N) <= 4 for 16-bit floats, "
                                  "<= 32 for fp32)");
    if (o.K == 0) { pl.kind = PK_SIMT; return MB_OK; }
    if (plan_gemv(o, sms, d, have_ws, pl)) return MB_OK;
    pl.kind = PK_SIMT;  // no unit stride: CUDA-core kernel reads it in place
    return MB_OK;
  }
  if (be == MB_BACKEND_SIMT || o.K == 0) { pl.kind = PK_SIMT; return MB_OK; }
  if (be == MB_BACKEND_TC && o.dt == MB_C32) {
    if (plan_c32(o, sms, d, have_ws, pl)) return MB_OK;
    return fail(MB_ERR_UNSUPPORTED, "tensor-core complex32 needs a row-major output and a workspace");
  }
  if (be == MB_BACKEND_TC) {
    if (o.dt == MB_F32) {  // fp32 on the tensor cores is 3xTF32
      if (plan_3xtf32(o, sms, d, have_ws, pl)) return MB_OK;
      return fail(MB_ERR_UNSUPPORTED, "tensor-core fp32 (3xTF32) needs a workspace for the split operands");
    }
    if (o.dt == MB_C64) {  // complex64 on the tensor cores is one real 3xTF32 GEMM
      if (plan_c64x3(o, sms, d, have_ws, pl)) return MB_OK;
      return fail(MB_ERR_UNSUPPORTED, "tensor-core complex64 (3xTF32) needs a row-major output, real alpha/beta, "
                                      "a bias contiguous along N and a workspace");
    }
    if (limb_planes(o.dt)) {  // 16/32/64-bit integers as byte planes on the 8-bit tensor cores
      if (plan_limb(o, sms, d, have_ws, pl)) return MB_OK;
      return fail(MB_ERR_UNSUPPORTED, "tensor-core integer product (byte planes) needs a workspace");
    }
    if (!is_tc_dtype(o.dt))
      return fail(MB_ERR_UNSUPPORTED, "tensor-core backend supports bf16/fp16/fp32/complex32/complex64/8-64-bit "
                                      "integers only");
    if (plan_tc_any(o, sms, d, have_ws, pl)) return MB_OK;
    if (plan_packed(o, sms, d, have_ws, pl)) return MB_OK;
    return fail(MB_ERR_UNSUPPORTED, "tensor-core backend: operands not TMA-addressable (need a unit stride, "
                                    "16-byte aligned base and leading/batch strides) and no workspace to pack them");
  }
  // AUTO
  if ((o.M == 1 || o.N == 1) && plan_gemv(o, sms, d, have_ws, pl)) return MB_OK;
  // fp32 thin products: the column GEMV with the rows sharing W's loads streams
  // W at 0.5-1.0 of HBM where the FFMA tile kernel measured 0.02-0.06 (B200,
  // M = 2..4, K and N 4096..16384); 3xTF32 would move ~5x the bytes.  16-bit
  // floats stay on the tensor cores, measured faster there.
  if (o.dt == MB_F32 && std::min(o.M, o.N) <= kGemvMaxRowsF32 && plan_gemv(o, sms, d, have_ws, pl)) return MB_OK;
  if (o.dt == MB_C32 && plan_c32(o, sms, d, have_ws, pl)) return MB_OK;
  // fp32: 3xTF32 on the tensor cores when its estimated time beats the CUDA-core
  // kernel's.  3xTF32: the split pass moves 12 bytes per operand element and the
  // GEMM reads 8 (measured ~36 B of time per element at ~6 TB/s on thin and
  // small shapes, B200), plus the FLOPs at ~190 TFLOP/s and ~6 us of extra
  // launches.  FFMA: ~40 TFLOP/s on the work of its 128 x 128 tiles (padding
  // included: a thin product wastes most of each tile) when they fill every SM,
  // proportionally less when they do not (it has no split-K).
  if (o.dt == MB_F32 && g_fp32_tf32x3) {
    const double bt = (double)std::max<int64_t>(o.batch, 1);
    const double flops = 2.0 * o.M * o.N * o.K * bt;
    const double opnd = (double)o.M * o.K * (o.sA ? bt : 1.0) + (double)o.K * o.N * (o.sB ? bt : 1.0);
    const double ctas = (double)ceil_div(o.M, 128) * ceil_div(o.N, 128) * bt;
    const double tile_flops = 2.0 * 128.0 * 128.0 * (double)o.K * ctas;
    const double t_simt = tile_flops / (40.0e12 * std::min(1.0, ctas / (double)sms));
    const double t_x3 = 36.0 * opnd / 6.0e12 + flops / 190.0e12 + 6.0e-6;
    if (t_x3 < t_simt && plan_3xtf32(o, sms, d, have_ws, pl)) return MB_OK;
  }
  // complex64: the same estimate on the real form (8MNK real FLOPs; A' is
  // M x 2K, B' 2K x 2N; the FFMA kernel's complex tiles are 64 x 64).
  if (o.dt == MB_C64 && g_fp32_tf32x3) {
    const double bt = (double)std::max<int64_t>(o.batch, 1);
    const double flops = 8.0 * o.M * o.N * o.K * bt;
    const double opnd = 2.0 * o.M * o.K * (o.sA ? bt : 1.0) + 4.0 * o.K * o.N * (o.sB ? bt : 1.0);
    const double ctas = (double)ceil_div(o.M, 64) * ceil_div(o.N, 64) * bt;
    const double tile_flops = 8.0 * 64.0 * 64.0 * (double)o.K * ctas;
    const double t_simt = tile_flops / (40.0e12 * std::min(1.0, ctas / (double)sms));
    const double t_x3 = 36.0 * opnd / 6.0e12 + flops / 190.0e12 + 6.0e-6;
    if (t_x3 < t_simt && plan_c64x3(o, sms, d, have_ws, pl)) return MB_OK;
  }
  // 16/32/64-bit integers: byte planes on the 8-bit tensor cores when the
  // estimate beats the IMAD kernel's.  Planes: L(L+1)/2 u8 GEMM-equivalents at
  // ~2.2 POPS on 128-padded tiles, the plane split and L read-modify-writes of C
  // at ~6 TB/s, ~4 us per launch; IMAD: the measured rates (int16 22.7, int32
  // 26, int64 7.2 Tops on 2048^3) on its 128 x 128 (int64: 64 x 64) tiles.
  if (limb_planes(o.dt) && g_int_limbs && have_ws) {
    const int L = limb_planes(o.dt);
    const int esz = elem_size(o.dt);
    const double bt = (double)std::max<int64_t>(o.batch, 1);
    const int64_t kp_max = (33024 / L) / 16 * 16;
    const double chunks = (double)ceil_div(o.K, kp_max);
    const double kp = (double)round_up(std::min<int64_t>(o.K, kp_max), 16) * chunks;
    const double mp = (double)round_up(o.M, 128), np = (double)round_up(o.N, 128);
    const double t_tc = 2.0 * mp * np * kp * bt * (L * (L + 1) / 2) / 2.2e15;
    const double bytes = ((double)o.M * o.K * (o.sA ? bt : 1.0) + (double)o.N * o.K * (o.sB ? bt : 1.0)) * (esz + L) +
                         2.0 * L * chunks * (double)o.M * o.N * esz * bt;
    const double t_limb = t_tc + bytes / 6.0e12 + (2 + L) * chunks * 4.0e-6;
    const int bm = o.dt == MB_I64 ? 64 : 128;
    const double ctas = (double)ceil_div(o.M, bm) * ceil_div(o.N, bm) * bt;
    const double rate = o.dt == MB_I16 ? 22.7e12 : o.dt == MB_I32 ? 26.0e12 : 7.2e12;
    const double t_simt = 2.0 * bm * bm * (double)o.K * ctas / (rate * std::min(1.0, ctas / (double)sms));
    if (t_limb < t_simt && plan_limb(o, sms, d, have_ws, pl)) return MB_OK;
  }
  if (is_tc_dtype(o.dt)) {
    if (plan_tc_any(o, sms, d, have_ws, pl)) return MB_OK;
    // worth a copy when the product is large enough for the tensor cores to
    // win it back (the CUDA-core kernel reads any layout in place)
    if ((double)o.M * o.N * o.K * std::max<int64_t>(o.batch, 1) >= 1.0e8 && plan_packed(o, sms, d, have_ws, pl))
      return MB_OK;
  }
  pl.kind = PK_SIMT;
  return MB_OK;
}

// The TC plan on o as given or, for thin M, as Cᵀ = Bᵀ·Aᵀ.
bool plan_tc_any(const Op &o, int sms, const mb_gemm_desc *d, bool have_ws, Plan &pl) {
  const bool want_swap = d->swap_ab == 1 || (d->swap_ab == 0 && o.M < 128 && o.N > o.M);
  if (want_swap && d->swap_ab != -1) {
    Op s = swapped(o);
    if (plan_tc(s, sms, d, have_ws, pl)) {
      pl.swap = 1;
      // thin M, free choice: wide unswapped tiles stream B in longer rows and
      // win where they fill the machine (M = 16..100, N = 28672: 112 tiles of
      // 128 x 256 measured 1.05-1.40x the swapped plans on B200; below M = 16
      // they lost at K <= 8192, and split unswapped tiles measured no gain)
      Plan u;
      if (d->swap_ab == 0 && o.M >= 16 && plan_tc(o, sms, d, have_ws, u) && u.splits == 1 && !u.sk &&
          u.est < 0.97 * pl.est) {
        pl = u;
        pl.swap = 0;
      }
      return true;
    }
  }
  if (d->swap_ab != 1 && plan_tc(o, sms, d, have_ws, pl)) { pl.swap = 0; return true; }
  return false;
}

int validate(const mb_gemm_desc *d) {
  if (!d) return fail(MB_ERR_INVALID, "null descriptor");
  if (d->dtype < MB_F32 || d->dtype > MB_I64) return fail(MB_ERR_UNSUPPORTED, "dtype %d not supported", d->dtype);
  if (d->M < 0 || d->N < 0 || d->K < 0 || d->batch < 0) return fail(MB_ERR_INVALID, "negative extent");
  if (d->backend < MB_BACKEND_AUTO || d->backend > MB_BACKEND_SIMT) return fail(MB_ERR_INVALID, "unknown backend %d", d->backend);
  if (d->tile_n && (d->tile_n % 16 || d->tile_n < 16 || d->tile_n > 512 || (d->tile_n & (d->tile_n - 1))))
    return fail(MB_ERR_INVALID, "tile_n must be one of 16, 32, 64, 128, 256 (or 512 on a CTA pair)");
  if (d->split_k < 0 || d->split_k > 65535) return fail(MB_ERR_INVALID, "split_k out of range");
  if (d->cta_pair < 0 || d->cta_pair > 2) return fail(MB_ERR_INVALID, "cta_pair must be 0, 1 or 2");
  const bool empty = d->M == 0 || d->N == 0 || d->batch == 0;
  if (!empty) {
    if (!d->C) return fail(MB_ERR_INVALID, "null C");
    if (d->K > 0 && (!d->A || !d->B)) return fail(MB_ERR_INVALID, "null A or B");
    if (d->epilogue && d->beta_nz && !d->bias) return fail(MB_ERR_INVALID, "beta != 0 needs a bias pointer");
  }
  return MB_OK;
}

EpiScalars make_epi(const mb_gemm_desc *d) {
  EpiScalars e{};
  e.enabled = d->epilogue ? 1 : 0;
  e.alpha_nz = d->epilogue ? (d->alpha_nz ? 1 : 0) : 1;
  e.beta_nz = d->epilogue ? (d->beta_nz ? 1 : 0) : 0;
  e.alpha_re = (float)d->alpha_re; e.alpha_im = (float)d->alpha_im;
  e.beta_re = (float)d->beta_re; e.beta_im = (float)d->beta_im;
  e.ialpha = d->ialpha; e.ibeta = d->ibeta;
  return e;
}

// --------------------------------------------------------------------------- launches
// Programmatic dependent launch for the GEMV and tcgen05 kernels (see
// pdl_trigger / pdl_wait in mb_common.cuh); METALBLAS_PDL=0 launches them
// with plain stream order.
// Split-K of thin tiles reduced inside a thread-block cluster (rank 0's shared
// memory) instead of through the workspace (METALBLAS_CLUSTER_SPLIT=0: off).
const bool g_csplit = [] {
  const char *s = getenv("METALBLAS_CLUSTER_SPLIT");
  return !(s && s[0] == '0');
}();

const bool g_pdl = [] {
  const char *s = getenv("METALBLAS_PDL");
  return !(s && s[0] == '0');
}();

template <class... KArgs, class... Args>
int launch_pdl(void (*kern)(KArgs...), dim3 grid, dim3 block, size_t smem, cudaStream_t st, int cluster_x,
               const char *what, Args &&...args) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = block;
  cfg.dynamicSmemBytes = smem;
  cfg.stream = st;
  cudaLaunchAttribute attr[2];
  int n = 0;
  if (cluster_x > 1) {
    attr[n].id = cudaLaunchAttributeClusterDimension;
    attr[n].val.clusterDim.x = cluster_x;
    attr[n].val.clusterDim.y = 1;
    attr[n].val.clusterDim.z = 1;
    ++n;
  }
  if (g_pdl) {
    attr[n].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[n].val.programmaticStreamSerializationAllowed = 1;
    ++n;
  }
  cfg.attrs = attr;
  cfg.numAttrs = n;
  return cuda_check(cudaLaunchKernelEx(&cfg, kern, std::forward<Args>(args)...), what);
}

template <class T>
int launch_simt(const Op &o, const EpiScalars &e, cudaStream_t st, const int *gate = nullptr) {
  SimtParams p{};
  p.gate = gate;
  p.A = o.A; p.B = o.B; p.C = o.C; p.bias = o.bias;
  p.M = o.M; p.N = o.N; p.K = o.K; p.batch = o.batch;
  p.a_rs = o.a_rs; p.a_cs = o.a_cs; p.sA = o.sA;
  p.b_rs = o.b_rs; p.b_cs = o.b_cs; p.sB = o.sB;
  p.c_rs = o.c_rs; p.c_cs = o.c_cs; p.sC = o.sC;
  p.bias_rs = o.bias_rs; p.bias_cs = o.bias_cs; p.bias_bs = o.bias_bs;
  p.conj_a = o.conj_a; p.conj_b = o.conj_b; p.epi = e;
  // A 4-element run along the contiguous dimension is one aligned vector when
  // the base, the other stride and the batch stride keep 4-element alignment
  // (runs start at multiples of 4 along the contiguous dimension).
  const int64_t run_bytes = 4 * (int64_t)sizeof(T);
  auto vec_ok = [&](const void *base, int64_t rs, int64_t cs, int64_t bs) {
    const int64_t lead = (cs == 1) ? rs : (rs == 1 ? cs : -1);
    if (lead < 0 || reinterpret_cast<uintptr_t>(base) % run_bytes) return 0;
    if (lead % 4 || (o.batch > 1 && bs % 4)) return 0;
    return 1;
  };
  {
    // the kernel's choice of run direction (see simt_gemm_kernel)
    const bool a_kfast = o.a_cs == 1 || (o.a_rs != 1 && std::llabs(o.a_cs) <= std::llabs(o.a_rs));
    const bool b_nfast = o.b_cs == 1 || (o.b_rs != 1 && std::llabs(o.b_cs) <= std::llabs(o.b_rs));
    p.a_vec = (a_kfast ? o.a_cs == 1 : o.a_rs == 1) ? vec_ok(o.A, o.a_rs, o.a_cs, o.sA) : 0;
    p.b_vec = (b_nfast ? o.b_cs == 1 : o.b_rs == 1) ? vec_ok(o.B, o.b_rs, o.b_cs, o.sB) : 0;
  }
  using Acc = typename Elem<T>::acc;
  if constexpr (sizeof(Acc) == 4) {
    constexpr int BM = 128, BN = 128;
    dim3 grid((unsigned)ceil_div(o.N, BN), (unsigned)ceil_div(o.M, BM), (unsigned)std::min<int64_t>(o.batch, 65535));
    if (grid.y > 65535) return fail(MB_ERR_INVALID, "M too large for the CUDA-core kernel");
    simt_gemm_kernel<T, BM, BN, 16, 8, 8><<<grid, 256, 0, st>>>(p);
  } else {
    constexpr int BM = 64, BN = 64;
    dim3 grid((unsigned)ceil_div(o.N, BN), (unsigned)ceil_div(o.M, BM), (unsigned)std::min<int64_t>(o.batch, 65535));
    if (grid.y > 65535) return fail(MB_ERR_INVALID, "M too large for the CUDA-core kernel");
    simt_gemm_kernel<T, BM, BN, 16, 4, 4><<<grid, 256, 0, st>>>(p);
  }
  return cuda_check(cudaGetLastError(), "simt_gemm launch");
}

template <class T>
int launch_gemv(const Plan &pl, const EpiScalars &e, void *ws, cudaStream_t st) {
  GemvParams g = pl.g;
  g.epi = e;
  constexpr int NW = kGemvWarps;
  constexpr int V = 16 / sizeof(T);
  if (g.ksplit > 1) {
    g.tickets = reinterpret_cast<unsigned *>(ws);
    g.ws = reinterpret_cast<char *>(ws) + kTicketBytes;
  }
  const unsigned gz = (unsigned)std::min<int64_t>(g.batch, 65535);
  if (g.batch > 65535) return fail(MB_ERR_INVALID, "batch too large for GEMV");
  auto go = [&](auto kern, dim3 grid) { return launch_pdl(kern, grid, dim3(NW * 32), 0, st, 1, "gemv launch", g); };
  if (pl.kind == PK_GEMV_COLS) {
    dim3 grid((unsigned)(pl.gemv_ctas_x * std::max(g.mrb, 1)), (unsigned)g.ksplit, gz);
    constexpr bool thin = std::is_same<T, __nv_bfloat16>::value || std::is_same<T, __half>::value ||
                          std::is_same<T, float>::value;
    if (pl.vec > 1) {
      if constexpr (thin) {
        const int mr = gemv_mr(std::is_same<T, float>::value ? MB_F32 : MB_BF16, g.mrows);
        if (mr == 8) {
          if constexpr (std::is_same<T, float>::value) return go(gemv_cols_kernel<T, V, NW, 8>, grid);
        } else if (mr == 4) return go(gemv_cols_kernel<T, V, NW, 4>, grid);
        else if (mr == 2) return go(gemv_cols_kernel<T, V, NW, 2>, grid);
        else return go(gemv_cols_kernel<T, V, NW>, grid);
      } else {
        return go(gemv_cols_kernel<T, V, NW>, grid);
      }
    } else {
      return go(gemv_cols_kernel<T, 1, NW>, dim3((unsigned)ceil_div(g.R, 32), (unsigned)g.ksplit, gz));
    }
  } else {
    if (pl.vec > 1 && g.x_vec) {
      constexpr int RPW = kGemvRowsPerWarp;  // x staged in shared memory
      dim3 grid((unsigned)ceil_div(g.R, NW * RPW), (unsigned)g.ksplit, gz);
      return go(gemv_rows_smem_kernel<T, V, NW, RPW>, grid);
    } else {
      dim3 grid((unsigned)ceil_div(g.R, NW), 1, gz);
      if (pl.vec > 1) return go(gemv_rows_kernel<T, V, NW>, grid);
      else return go(gemv_rows_kernel<T, 1, NW>, grid);
    }
  }
  return cuda_check(cudaGetLastError(), "gemv launch");
}

PFN_cuTensorMapEncodeTiled_v12000 get_encode() {
  static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void *p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(p);
  });
  return fn;
}

CUtensorMapDataType tma_dtype(int dt) {
  switch (dt) {
    case MB_BF16: return CU_TENSOR_MAP_DATA_TYPE_BFLOAT16;
    case MB_F16: return CU_TENSOR_MAP_DATA_TYPE_FLOAT16;
    case MB_F32: return CU_TENSOR_MAP_DATA_TYPE_FLOAT32;
    default: return CU_TENSOR_MAP_DATA_TYPE_UINT8;
  }
}

// 3-D tiled map {inner, outer, batch} with SWIZZLE_128B.
int encode_map(CUtensorMap *m, int dt, const void *base, int64_t inner, int64_t outer, int64_t batch,
               int64_t outer_stride_el, int64_t batch_stride_el, int box_inner, int box_outer,
               CUtensorMapSwizzle swz = CU_TENSOR_MAP_SWIZZLE_128B) {
  auto enc = get_encode();
  if (!enc) return fail(MB_ERR_LAUNCH, "cuTensorMapEncodeTiled unavailable");
  const int esz = elem_size(dt);
  cuuint64_t dims[3] = {(cuuint64_t)inner, (cuuint64_t)outer, (cuuint64_t)std::max<int64_t>(batch, 1)};
  int64_t ostr = outer_stride_el * esz;
  int64_t bstr = batch_stride_el * esz;
  if (batch <= 1 || bstr == 0) bstr = round_up(std::max<int64_t>(ostr * outer, 16), 16);
  cuuint64_t strides[2] = {(cuuint64_t)ostr, (cuuint64_t)bstr};
  cuuint32_t box[3] = {(cuuint32_t)box_inner, (cuuint32_t)box_outer, 1};
  cuuint32_t estr[3] = {1, 1, 1};
  CUresult r = enc(m, tma_dtype(dt), 3, const_cast<void *>(base), dims, strides, box, estr,
                   CU_TENSOR_MAP_INTERLEAVE_NONE, swz, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                   CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) return fail(MB_ERR_LAUNCH, "cuTensorMapEncodeTiled failed (%d)", (int)r);
  return MB_OK;
}

template <class T, int BN, int PAIR, class TO = T, bool PEER = false>
int launch_tc_bn(const Op &o, const Plan &pl, const EpiScalars &e, void *ws, int sms, cudaStream_t st,
                 const mb_peer_targets *peers = nullptr) {
  using C_ = tc::Cfg<BN, sizeof(T), PAIR>;
  constexpr int ESZ = sizeof(T);
  constexpr int OSZ = sizeof(TO);
  constexpr int BK = C_::BK;
  tc::TcParams p;
  memset(&p, 0, sizeof(p));
  int rc;
  const int64_t bA = o.sA ? o.batch : 1, bB = o.sB ? o.batch : 1;
  if (!pl.a_mn) rc = encode_map(&p.tmA, o.dt, o.A, o.K, o.M, bA, o.a_rs, o.sA, BK, tc::BM);
  else rc = encode_map(&p.tmA, o.dt, o.A, o.M, o.K, bA, o.a_cs, o.sA, 128 / ESZ, BK);
  if (rc) return rc;
  if constexpr (BN > 256) {
    // the 512-wide pair tile runs whole tiles only
    if (pl.tail_half || pl.splits > 1 || pl.sk) return fail(MB_ERR_INVALID, "512-wide tiles run whole tiles only");
  }
  // K-major B: one box per MMA of this CTA's share of the tile's columns
  if (!pl.b_mn) rc = encode_map(&p.tmB, o.dt, o.B, o.K, o.N, bB, o.b_cs, o.sB, BK, C_::UMMA_N / PAIR);
  else rc = encode_map(&p.tmB, o.dt, o.B, o.N, o.K, bB, o.b_rs, o.sB, 128 / ESZ, BK);
  if (rc) return rc;
  if constexpr (C_::NPART == 2) {
    // 3xTF32 low parts: K-major like the high parts
    if (pl.a_mn || pl.b_mn || !o.A2 || !o.B2) return fail(MB_ERR_INVALID, "3xTF32 operands must be K-major");
    rc = encode_map(&p.tmA2, o.dt, o.A2, o.K, o.M, bA, o.a_rs, o.sA, BK, tc::BM);
    if (!rc) rc = encode_map(&p.tmB2, o.dt, o.B2, o.K, o.N, bB, o.b_cs, o.sB, BK, BN / PAIR);
    if (rc) return rc;
  }
  p.M = (int)o.M; p.N = (int)o.N; p.K = (int)o.K; p.batch = (int)o.batch;
  p.a_mn = pl.a_mn; p.b_mn = pl.b_mn;
  p.a_bcast = o.sA == 0; p.b_bcast = o.sB == 0;
  p.tiles_m = (int)pl.tiles_m; p.tiles_n = (int)pl.tiles_n;
  p.splits = pl.splits; p.kb_total = (int)pl.kb_total; p.kb_per_split = (int)pl.kb_per_split;
  const int64_t tiles = o.batch * pl.tiles_m * pl.tiles_n;
  const int64_t units = pl.dp_tiles + (pl.sk ? 0 : (tiles - pl.dp_tiles) * (pl.tail_half ? 2 : pl.splits));
  if (units >= (1ll << 31)) return fail(MB_ERR_INVALID, "too many tiles");
  p.dp_tiles = (int)pl.dp_tiles;
  p.tail_half = pl.tail_half;
  p.num_units = (int)units;
  if (pl.sk) {
    p.sk = 1;
    p.sk_iters = (long long)(tiles - pl.dp_tiles) * pl.kb_total;
  }
  p.group_m = 16;
  p.C = o.C; p.c_rs = o.c_rs; p.c_cs = o.c_cs; p.sC = o.sC;
  p.bias = o.bias; p.bias_rs = o.bias_rs; p.bias_cs = o.bias_cs; p.bias_bs = o.bias_bs;
  p.epi = e;
  p.c_vec = (o.c_cs == 1 && aligned16(o.C) && (o.c_rs * OSZ) % 16 == 0 && (o.batch <= 1 || (o.sC * OSZ) % 16 == 0)) ? 1 : 0;
  // Row-major output that TMA can address: staged epilogue with TMA stores.
  if (C_::TMA_STORE && std::is_same_v<T, TO> && p.c_vec && o.c_rs >= o.N && o.sC >= 0 && (o.batch <= 1 || o.sC >= o.c_rs * o.M || o.sC == 0) &&
      o.N < (1ll << 31) && o.M < (1ll << 31)) {
    const int64_t bC = o.batch > 1 ? o.batch : 1;
    if (encode_map(&p.tmC, o.dt, o.C, o.N, o.M, bC, o.c_rs, o.sC, C_::CC, 32, CU_TENSOR_MAP_SWIZZLE_64B) == MB_OK)
      p.c_tma = 1;
  }
  if (pl.splits > 1) {
    p.tickets = reinterpret_cast<unsigned *>(ws);
    p.ws = reinterpret_cast<char *>(ws) + kTicketBytes;
  }
  p.timeout_ns = wait_timeout_ns();
  if constexpr (PEER) {
    p.npeers = peers->count;
    for (int i = 0; i < peers->count; ++i) p.peer_C[i] = peers->C[i];
    p.mc_C = peers->mc_C;
  }
  auto kern = tc::tc_gemm_kernel<T, BN, PAIR, TO, PEER>;
  static int attr_done[64] = {0};
  int dev = 0;
  cudaGetDevice(&dev);
  if (dev >= 0 && dev < 64 && !attr_done[dev]) {
    rc = cuda_check(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, C_::SMEM_BYTES),
                    "cudaFuncSetAttribute");
    if (rc) return rc;
    attr_done[dev] = 1;
  }
  if constexpr (PAIR == 1) {
    // stream-K ranges are cut for exactly sk_ctas CTAs
    const int grid = pl.sk ? (int)pl.sk_ctas : (int)std::min<int64_t>(units, sms);
    int cx = 1;
    if constexpr (C_::RED_BYTES > 0 && !PEER && std::is_same_v<T, TO>) {
      // Cluster split-K: one unit per CTA, the `splits` units of a tile in one
      // cluster (units are numbered tile-major, so CTA u holds split u % splits).
      // The CTAs of a cluster are scheduled together, so rank 0 never waits for
      // a peer that cannot start; the occupancy check keeps the one-wave
      // schedule the planner costed (a GPC that cannot hold a whole cluster
      // would push some clusters into a second wave).
      static int max_clusters[64][C_::CSPLIT_MAX + 1] = {};
      if (g_csplit && !pl.sk && !pl.tail_half && pl.dp_tiles == 0 && pl.splits >= 2 &&
          pl.splits <= C_::CSPLIT_MAX && units <= sms && units % pl.splits == 0 && dev >= 0 && dev < 64) {
        int &slot = max_clusters[dev][pl.splits];
        if (slot == 0) {
          cudaLaunchConfig_t cfg = {};
          cfg.gridDim = dim3(pl.splits);
          cfg.blockDim = dim3(tc::NUM_THREADS);
          cfg.dynamicSmemBytes = C_::SMEM_BYTES;
          cudaLaunchAttribute a[1];
          a[0].id = cudaLaunchAttributeClusterDimension;
          a[0].val.clusterDim.x = pl.splits;
          a[0].val.clusterDim.y = 1;
          a[0].val.clusterDim.z = 1;
          cfg.attrs = a;
          cfg.numAttrs = 1;
          int n = 0;
          if (cudaOccupancyMaxActiveClusters(&n, kern, &cfg) != cudaSuccess) {
            (void)cudaGetLastError();
            n = 0;
          }
          slot = n + 1;
        }
        if ((int64_t)(slot - 1) >= units / pl.splits) cx = pl.splits;
      }
    }
    p.csplit = cx > 1 ? 1 : 0;
    return launch_pdl(kern, dim3(grid), dim3(tc::NUM_THREADS), C_::SMEM_BYTES, st, cx, "tc_gemm launch", p);
  } else {
    // one cluster (CTA pair) per unit slot; the pair shares each 256-row tile
    // (stream-K ranges are cut for exactly sk_ctas / 2 pairs)
    const int pairs = pl.sk ? (int)(pl.sk_ctas / 2) : (int)std::min<int64_t>(units, sms / 2);
    return launch_pdl(kern, dim3(2 * pairs), dim3(tc::NUM_THREADS), C_::SMEM_BYTES, st, 2,
                      "tc_gemm (CTA pair) launch", p);
  }
}

template <class T, bool PEER = false>
int launch_tc(const Op &o, const Plan &pl, const EpiScalars &e, void *ws, int sms, cudaStream_t st,
              const mb_peer_targets *peers = nullptr) {
  if constexpr (PEER && !std::is_same_v<T, float>) {
    // the tile shapes the table picks for 16-bit and 8-bit products
    if (pl.pair == 2) {
      switch (pl.bn) {
        case 128: return launch_tc_bn<T, 128, 2, T, true>(o, pl, e, ws, sms, st, peers);
        case 256: return launch_tc_bn<T, 256, 2, T, true>(o, pl, e, ws, sms, st, peers);
        case 512: return launch_tc_bn<T, 512, 2, T, true>(o, pl, e, ws, sms, st, peers);
      }
      return fail(MB_ERR_INVALID, "bad tile_n %d for a CTA pair", pl.bn);
    }
    switch (pl.bn) {
      case 16: return launch_tc_bn<T, 16, 1, T, true>(o, pl, e, ws, sms, st, peers);
      case 32: return launch_tc_bn<T, 32, 1, T, true>(o, pl, e, ws, sms, st, peers);
      case 64: return launch_tc_bn<T, 64, 1, T, true>(o, pl, e, ws, sms, st, peers);
      case 128: return launch_tc_bn<T, 128, 1, T, true>(o, pl, e, ws, sms, st, peers);
      case 256: return launch_tc_bn<T, 256, 1, T, true>(o, pl, e, ws, sms, st, peers);
    }
    return fail(MB_ERR_INVALID, "bad tile_n %d", pl.bn);
  } else if constexpr (PEER) {
    return fail(MB_ERR_UNSUPPORTED, "peer replication is not built for fp32 (3xTF32) products");
  } else if constexpr (std::is_same_v<T, float>) {
    // 3xTF32 keeps BN/2 fp32 running sums per epilogue thread: BN <= 128
    if (pl.pair == 2 && pl.bn == 128) return launch_tc_bn<T, 128, 2>(o, pl, e, ws, sms, st);
    switch (pl.pair == 1 ? pl.bn : 0) {
      case 16: return launch_tc_bn<T, 16, 1>(o, pl, e, ws, sms, st);
      case 32: return launch_tc_bn<T, 32, 1>(o, pl, e, ws, sms, st);
      case 64: return launch_tc_bn<T, 64, 1>(o, pl, e, ws, sms, st);
      case 128: return launch_tc_bn<T, 128, 1>(o, pl, e, ws, sms, st);
    }
    return fail(MB_ERR_INVALID, "3xTF32 plan with tile_n %d pair %d", pl.bn, pl.pair);
  } else {
  if (pl.pair == 2) {
    switch (pl.bn) {
      case 128: return launch_tc_bn<T, 128, 2>(o, pl, e, ws, sms, st);
      case 256: return launch_tc_bn<T, 256, 2>(o, pl, e, ws, sms, st);
      case 512: return launch_tc_bn<T, 512, 2>(o, pl, e, ws, sms, st);
    }
    return fail(MB_ERR_INVALID, "bad tile_n %d for a CTA pair", pl.bn);
  }
  switch (pl.bn) {
    case 16: return launch_tc_bn<T, 16, 1>(o, pl, e, ws, sms, st);
    case 32: return launch_tc_bn<T, 32, 1>(o, pl, e, ws, sms, st);
    case 64: return launch_tc_bn<T, 64, 1>(o, pl, e, ws, sms, st);
    case 128: return launch_tc_bn<T, 128, 1>(o, pl, e, ws, sms, st);
    case 256: return launch_tc_bn<T, 256, 1>(o, pl, e, ws, sms, st);
  }
  return fail(MB_ERR_INVALID, "bad tile_n %d", pl.bn);
  }
}

// complex32 on the tensor cores: build B' (and A' when A is not row-major),
// then one real fp16 GEMM with the complex-pair epilogue.
int launch_c32(const Op &o, const Plan &pl, EpiScalars e, void *ws, int sms, cudaStream_t st) {
  char *w = reinterpret_cast<char *>(ws);
  __half2 *bp = reinterpret_cast<__half2 *>(w + pl.c32_b_off);
  __half2 *ap = reinterpret_cast<__half2 *>(w + pl.c32_a_off);
  const int grid_cap = sms * 16;
  C32Prep pb{};
  pb.src = reinterpret_cast<const __half2 *>(o.B); pb.dst = bp;
  pb.rows = o.K; pb.cols = o.N; pb.rs = o.b_rs; pb.cs = o.b_cs; pb.bs = o.sB;
  pb.batch = pl.c32_b_batches; pb.conj_a = o.conj_a; pb.conj_b = o.conj_b;
  if (pb.batch > 65535) return fail(MB_ERR_INVALID, "batch too large for the complex32 path");
  const dim3 bgrid((unsigned)ceil_div(pb.cols, 1024), (unsigned)std::min<int64_t>(pb.rows, 65535), (unsigned)pb.batch);
  c32_build_b_kernel<<<bgrid, 256, 0, st>>>(pb, pl.c32_ldb);
  int rc = cuda_check(cudaGetLastError(), "complex32 B' build");
  if (rc) return rc;
  if (pl.c32_pack_a) {
    // A' rows = A's rows as half2 pairs (4-byte elements), through the tiled pack
    PackArgs pa{o.A, ap, o.M, o.K, o.a_rs, o.a_cs, o.sA, pl.c32_a_batches, pl.c32_lda};
    const int64_t tiles = pa.batch * ceil_div(o.M, 32) * ceil_div(o.K, 32);
    pack_matrix_kernel<uint32_t><<<(unsigned)std::max<int64_t>(1, std::min<int64_t>(tiles, grid_cap)), dim3(32, 8), 0,
                                   st>>>(pa);
    rc = cuda_check(cudaGetLastError(), "complex32 A' pack");
    if (rc) return rc;
  }
  e.cplx = e.enabled ? 1 : 0;
  return launch_tc<__half>(c32_inner(o, pl, ap, bp), pl, e, ws, sms, st);
}

template <class T>
int launch_packed(const Op &o, const Plan &pl, const EpiScalars &e, void *ws, int sms, cudaStream_t st) {
  char *w = reinterpret_cast<char *>(ws);
  void *ap = w + pl.pk_a_off, *bp = w + pl.pk_b_off;
  using U = std::conditional_t<sizeof(T) == 1, uint8_t, uint16_t>;
  const int grid_cap = sms * 16;
  auto pack = [&](const void *src, void *dst, int64_t rows, int64_t cols, int64_t rs, int64_t cs, int64_t bs,
                  int64_t batches, int64_t ld, const char *what) {
    PackArgs a{src, dst, rows, cols, rs, cs, bs, batches, ld};
    if (cs == 1) {
      const int64_t n = batches * rows * ceil_div(cols, 16 / (int64_t)sizeof(U));
      pack_rows16_kernel<U><<<(unsigned)std::max<int64_t>(1, std::min<int64_t>(ceil_div(n, 256), grid_cap)), 256, 0,
                              st>>>(a);
    } else {
      const int64_t tiles = batches * ceil_div(rows, 32) * ceil_div(cols, 32);
      pack_matrix_kernel<U><<<(unsigned)std::max<int64_t>(1, std::min<int64_t>(tiles, grid_cap)), dim3(32, 8), 0,
                              st>>>(a);
    }
    return cuda_check(cudaGetLastError(), what);
  };
  int rc = MB_OK;
  // a column-major source is copied as the rows of its transpose
  if (pl.pk_a) {
    rc = pl.pk_a_cm ? pack(o.A, ap, o.K, o.M, o.a_cs, o.a_rs, o.sA, pl.pk_a_batches, pl.pk_lda, "pack A")
                    : pack(o.A, ap, o.M, o.K, o.a_rs, o.a_cs, o.sA, pl.pk_a_batches, pl.pk_lda, "pack A");
  }
  if (!rc && pl.pk_b) {
    rc = pl.pk_b_cm ? pack(o.B, bp, o.N, o.K, o.b_cs, o.b_rs, o.sB, pl.pk_b_batches, pl.pk_ldb, "pack B")
                    : pack(o.B, bp, o.K, o.N, o.b_rs, o.b_cs, o.sB, pl.pk_b_batches, pl.pk_ldb, "pack B");
  }
  if (rc) return rc;
  const Op r = packed_op(o, pl, ap, bp);
  return launch_tc<T>(pl.swap ? swapped(r) : r, pl, e, ws, sms, st);
}

int launch_3xtf32(const Op &o, const Plan &pl, const EpiScalars &e, void *ws, int sms, cudaStream_t st) {
  char *w = reinterpret_cast<char *>(ws);
  float *ahi = reinterpret_cast<float *>(w + pl.x3_ahi), *alo = reinterpret_cast<float *>(w + pl.x3_alo);
  float *bhi = reinterpret_cast<float *>(w + pl.x3_bhi), *blo = reinterpret_cast<float *>(w + pl.x3_blo);
  int *flag = reinterpret_cast<int *>(w + pl.x3_flag);
  int rc = cuda_check(cudaMemsetAsync(flag, 0, sizeof(int), st), "3xTF32 clear flag");
  if (rc) return rc;
  auto split = [&](const void *src, float *hi, float *lo, int64_t rows, int64_t cols, int64_t rs, int64_t cs,
                   int64_t bs, int64_t batches, const char *what) {
    SplitArgs a{static_cast<const float *>(src), hi, lo, flag, rows, cols, rs, cs, bs, batches, pl.x3_ldk};
    const int64_t tiles = batches * ceil_div(rows, 32) * ceil_div(cols, 128);
    split_tf32_kernel<<<(unsigned)std::max<int64_t>(1, std::min<int64_t>(tiles, (int64_t)sms * 16)), dim3(32, 8), 0,
                        st>>>(a);
    return cuda_check(cudaGetLastError(), what);
  };
  // A (M x K) and Bᵀ (N x K, element (n, k) = B(k, n))
  rc = split(o.A, ahi, alo, o.M, o.K, o.a_rs, o.a_cs, o.sA, pl.x3_a_batches, "3xTF32 split A");
  if (!rc) rc = split(o.B, bhi, blo, o.N, o.K, o.b_cs, o.b_rs, o.sB, pl.x3_b_batches, "3xTF32 split B");
  if (rc) return rc;
  const Op r = x3_op(o, pl, ahi, alo, bhi, blo);
  rc = launch_tc<float>(pl.swap ? swapped(r) : r, pl, e, ws, sms, st);
  if (rc) return rc;
  // inf / NaN in an input: FFMA recomputes the product (its CTAs exit at once otherwise)
  return launch_simt<float>(o, e, st, flag);
}

// complex64 through 3xTF32: split A' and B'ᵀ straight from the complex
// operands, the real GEMM with the real epilogue, then the gated FFMA
// recompute of the complex product when an input held inf or NaN.
int launch_c64x3(const Op &o, const Plan &pl, const EpiScalars &e, void *ws, int sms, cudaStream_t st) {
  char *w = reinterpret_cast<char *>(ws);
  float *ahi = reinterpret_cast<float *>(w + pl.x3_ahi), *alo = reinterpret_cast<float *>(w + pl.x3_alo);
  float *bhi = reinterpret_cast<float *>(w + pl.x3_bhi), *blo = reinterpret_cast<float *>(w + pl.x3_blo);
  int *flag = reinterpret_cast<int *>(w + pl.x3_flag);
  int rc = cuda_check(cudaMemsetAsync(flag, 0, sizeof(int), st), "complex64 3xTF32 clear flag");
  if (rc) return rc;
  const Op r = c64_real(o);
  auto split = [&](const void *src, float *hi, float *lo, int64_t rows, int64_t cols, int64_t rs, int64_t cs,
                   int64_t bs, int64_t batches, int mode, const char *what) {
    SplitArgs a{static_cast<const float *>(src), hi, lo, flag, rows, cols, rs, cs, bs, batches, pl.x3_ldk,
                mode, o.conj_a, o.conj_b};
    const int64_t tiles = batches * ceil_div(rows, 32) * ceil_div(cols, 128);
    split_tf32_kernel<<<(unsigned)std::max<int64_t>(1, std::min<int64_t>(tiles, (int64_t)sms * 16)), dim3(32, 8), 0,
                        st>>>(a);
    return cuda_check(cudaGetLastError(), what);
  };
  // A' (M x 2K) and B'ᵀ (2N x 2K); complex strides
  rc = split(o.A, ahi, alo, o.M, r.K, o.a_rs, o.a_cs, o.sA, pl.x3_a_batches, 1, "complex64 3xTF32 split A");
  if (!rc) rc = split(o.B, bhi, blo, r.N, r.K, o.b_cs, o.b_rs, o.sB, pl.x3_b_batches, 2, "complex64 3xTF32 split B");
  if (rc) return rc;
  EpiScalars er = e;
  er.cplx = 0;
  const Op x = x3_op(r, pl, ahi, alo, bhi, blo);
  rc = launch_tc<float>(pl.swap ? swapped(x) : x, pl, er, ws, sms, st);
  if (rc) return rc;
  return launch_simt<float2>(o, e, st, flag);
}

template <class TO>
int launch_tc_limb(const Op &o, const Plan &pl, const EpiScalars &e, void *ws, int sms, cudaStream_t st) {
  if (pl.pair == 2) {
    if (pl.bn == 128) return launch_tc_bn<uint8_t, 128, 2, TO>(o, pl, e, ws, sms, st);
    if (pl.bn == 256) return launch_tc_bn<uint8_t, 256, 2, TO>(o, pl, e, ws, sms, st);
  } else {
    if (pl.bn == 64) return launch_tc_bn<uint8_t, 64, 1, TO>(o, pl, e, ws, sms, st);
    if (pl.bn == 128) return launch_tc_bn<uint8_t, 128, 1, TO>(o, pl, e, ws, sms, st);
    if (pl.bn == 256) return launch_tc_bn<uint8_t, 256, 1, TO>(o, pl, e, ws, sms, st);
  }
  return fail(MB_ERR_INVALID, "integer plane GEMM with tile_n %d pair %d", pl.bn, pl.pair);
}

// The byte-plane chain (see plan_limb): per K chunk, split A and B into planes,
// then one u8 GEMM per shift s accumulating into C.
template <class T>
int launch_limb(const Op &o, const Plan &pl, const EpiScalars &e, void *ws, int sms, cudaStream_t st) {
  char *w = reinterpret_cast<char *>(ws);
  uint8_t *acat = reinterpret_cast<uint8_t *>(w + pl.limb_a_off), *brev = reinterpret_cast<uint8_t *>(w + pl.limb_b_off);
  const int L = pl.limb_L;
  const int64_t nchunks = ceil_div(o.K, pl.limb_kc);
  // the caller's alpha (1 without an epilogue); alpha == 0 leaves beta * bias
  const uint64_t alpha = e.enabled ? (e.alpha_nz ? (uint64_t)e.ialpha : 0ull) : 1ull;
  bool first = true;
  for (int64_t ch = 0; ch < nchunks; ++ch) {
    const int64_t k0 = ch * pl.limb_kc, kc = std::min<int64_t>(pl.limb_kc, o.K - k0);
    // A (M x K) and Bᵀ (N x K, element (n, k) = B(k, n)) in one launch
    const LimbArgs la{o.A, acat, o.M, kc, k0, o.a_rs, o.a_cs, o.sA, pl.limb_a_batches, pl.limb_kp, pl.limb_ld, L, 0};
    const LimbArgs lb{o.B, brev, o.N, kc, k0, o.b_cs, o.b_rs, o.sB, pl.limb_b_batches, pl.limb_kp, pl.limb_ld, L, 1};
    const int64_t tiles = limb_tiles(la) + limb_tiles(lb);
    limb_split_kernel<T><<<(unsigned)std::max<int64_t>(1, std::min<int64_t>(tiles, (int64_t)sms * 16)), dim3(32, 8), 0,
                           st>>>(la, lb);
    int rc = cuda_check(cudaGetLastError(), "integer byte planes of A and B");
    if (rc) return rc;
    for (int s = 0; s < L; ++s) {
      Op r = limb_gemm_op(o, pl, s, acat, brev);
      EpiScalars es = e;
      es.cplx = 0;
      if (!first) {
        // C += alpha * 2^(8s) * P_s (wrapping): the running sum is the bias
        r.bias = o.C; r.bias_rs = o.c_rs; r.bias_cs = o.c_cs; r.bias_bs = o.sC;
        es.enabled = 1; es.alpha_nz = 1; es.beta_nz = 1; es.ibeta = 1;
        es.ialpha = (int64_t)(alpha << (8 * s));
      } else if (e.enabled) {
        es.ialpha = (int64_t)(alpha << (8 * s));  // s == 0: the caller's epilogue as given
      }
      Plan g;
      if (!limb_gemm_plan(o, pl, s, sms, g)) return fail(MB_ERR_INVALID, "integer plane GEMM: no tile plan");
      rc = launch_tc_limb<T>(g.swap ? swapped(r) : r, g, es, ws, sms, st);
      if (rc) return rc;
      first = false;
      if (alpha == 0) return MB_OK;  // beta * bias only
    }
  }
  return MB_OK;
}

template <class F>
int by_dtype(int dt, F &&f) {
  switch (dt) {
    case MB_F32: return f((float *)nullptr);
    case MB_F16: return f((__half *)nullptr);
    case MB_BF16: return f((__nv_bfloat16 *)nullptr);
    case MB_C64: return f((float2 *)nullptr);
    case MB_C32: return f((__half2 *)nullptr);
    case MB_I8: return f((int8_t *)nullptr);
    case MB_U8: return f((uint8_t *)nullptr);
    case MB_I16: return f((int16_t *)nullptr);
    case MB_I32: return f((int32_t *)nullptr);
    case MB_I64: return f((int64_t *)nullptr);
  }
  return fail(MB_ERR_UNSUPPORTED, "dtype");
}

// Resident CTAs per SM of the vectorised column GEMV for dtype dt, from the
// occupancy calculator; 4 when no device answers (plan queries on a host).
int gemv_cols_per_sm(int dt, int mr) {
  static std::atomic<int> cache[MB_I64 + 1][4];
  if (dt < 0 || dt > MB_I64) return 4;
  const int mi = mr == 8 ? 3 : mr == 4 ? 2 : mr == 2 ? 1 : 0;
  int v = cache[dt][mi].load(std::memory_order_relaxed);
  if (v > 0) return v;
  auto occ = [](auto kernel) -> int {
    int n = 0;
    if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&n, kernel, kGemvWarps * 32, 0) != cudaSuccess) {
      cudaGetLastError();
      return 0;
    }
    return n;
  };
  v = by_dtype(dt, [&](auto *p) -> int {
    using T = std::remove_pointer_t<decltype(p)>;
    constexpr int V = 16 / sizeof(T);
    if constexpr (std::is_same<T, __nv_bfloat16>::value || std::is_same<T, __half>::value ||
                  std::is_same<T, float>::value) {
      if constexpr (std::is_same<T, float>::value)
        if (mi == 3) return occ(gemv_cols_kernel<T, V, kGemvWarps, 8>);
      if (mi == 2) return occ(gemv_cols_kernel<T, V, kGemvWarps, 4>);
      if (mi == 1) return occ(gemv_cols_kernel<T, V, kGemvWarps, 2>);
    }
    return occ(gemv_cols_kernel<T, V, kGemvWarps>);
  });
  if (v <= 0) return 4;
  cache[dt][mi].store(v, std::memory_order_relaxed);
  return v;
}

template <class T> struct IsTc { static constexpr bool v = false; };
template <> struct IsTc<__half> { static constexpr bool v = true; };
template <> struct IsTc<__nv_bfloat16> { static constexpr bool v = true; };
template <> struct IsTc<int8_t> { static constexpr bool v = true; };
template <> struct IsTc<uint8_t> { static constexpr bool v = true; };

// `query`: plan without a device if none is present (a B200's 148 SMs are
// assumed), so the tile table can be inspected on a host without a GPU.
int plan_for(const mb_gemm_desc *d, Plan &pl, Op &o, int &sms, bool query = false) {
  int rc = validate(d);
  if (rc) return rc;
  int dev = 0;
  rc = current_device(&dev);
  if (rc && !query) return rc;
  sms = rc ? 148 : num_sms(dev);
  if (rc) cudaGetLastError();
  o = make_op(d);
  const bool have_ws = d->workspace != nullptr || d->workspace_bytes < 0;  // <0: size query
  if (g_tune_size.load(std::memory_order_relaxed) > 0 && !has_overrides(d)) {
    Override ov{};
    bool hit = false;
    {
      const std::string key = tune_key(d);
      std::lock_guard<std::mutex> lk(g_tune_mu);
      auto it = g_tune.find(key);
      if (it != g_tune.end()) { ov = it->second; hit = true; }
    }
    if (hit && !ov.keep) {
      mb_gemm_desc q = *d;
      q.backend = ov.backend; q.tile_n = ov.tile_n; q.split_k = ov.split_k; q.swap_ab = ov.swap_ab;
      q.cta_pair = ov.cta_pair; q.stream_k = ov.stream_k;
      if (validate(&q) == MB_OK && make_plan(&q, o, sms, have_ws, pl) == MB_OK) return MB_OK;
      pl = Plan{};  // a stale entry that no longer plans: fall back to the table
    }
  }
  return make_plan(d, o, sms, have_ws, pl);
}

}  // namespace

// =========================================================================== C ABI
extern "C" {

void mb_gemm_desc_init(mb_gemm_desc *d) {
  if (!d) return;
  memset(d, 0, sizeof(*d));
  d->batch = 1;
  d->alpha_re = 1.0; d->beta_re = 1.0;
  d->ialpha = 1; d->ibeta = 1;
  d->alpha_nz = 1; d->beta_nz = 1;
}

int64_t mb_gemm_workspace_size(const mb_gemm_desc *d) {
  if (!d) return 0;
  mb_gemm_desc q = *d;
  q.workspace = nullptr;
  q.workspace_bytes = -1;  // plan as if a workspace were available
  Plan pl; Op o; int sms;
  if (plan_for(&q, pl, o, sms, true)) return 0;
  return pl.ws_bytes;
}

int mb_plan_query(const mb_gemm_desc *d, char *buf, int buflen) {
  Plan pl; Op o; int sms;
  int rc = plan_for(d, pl, o, sms, true);
  if (rc) return -rc;
  char tmp[256];
  switch (pl.kind) {
    case PK_EMPTY: snprintf(tmp, sizeof(tmp), "empty"); break;
    case PK_GEMV_COLS:
      if (pl.g.mrows > 1)
        snprintf(tmp, sizeof(tmp), "gemv_cols vec=%d ksplit=%d rows=%d", pl.vec, pl.g.ksplit, pl.g.mrows);
      else
        snprintf(tmp, sizeof(tmp), "gemv_cols vec=%d ksplit=%d", pl.vec, pl.g.ksplit);
      break;
    case PK_GEMV_ROWS:
      snprintf(tmp, sizeof(tmp), "gemv_rows vec=%d x_smem=%d ksplit=%d", pl.vec, (pl.vec > 1 && pl.g.x_vec) ? 1 : 0,
               pl.g.ksplit);
      break;
    case PK_TC:
      snprintf(tmp, sizeof(tmp),
               "tc bn=%d split=%d dp=%lld half=%d pair=%d sk=%d swap=%d a_mn=%d b_mn=%d tiles=%lldx%lld ws=%lld",
               pl.bn, pl.splits, (long long)pl.dp_tiles, pl.tail_half, pl.pair, pl.sk, pl.swap, pl.a_mn, pl.b_mn,
               (long long)pl.tiles_m, (long long)pl.tiles_n, (long long)pl.ws_bytes);
      break;
    case PK_TC_C32:
      snprintf(tmp, sizeof(tmp), "tc_c32 pack_a=%d bn=%d split=%d pair=%d tiles=%lldx%lld ws=%lld", pl.c32_pack_a,
               pl.bn, pl.splits, pl.pair, (long long)pl.tiles_m, (long long)pl.tiles_n, (long long)pl.ws_bytes);
      break;
    case PK_TC_3XTF32:
    case PK_TC_C64X3:
      snprintf(tmp, sizeof(tmp), "%s bn=%d split=%d dp=%lld half=%d pair=%d sk=%d swap=%d tiles=%lldx%lld ws=%lld",
               pl.kind == PK_TC_C64X3 ? "tc_c64x3" : "tc_3xtf32", pl.bn, pl.splits, (long long)pl.dp_tiles, pl.tail_half, pl.pair, pl.sk, pl.swap, (long long)pl.tiles_m,
               (long long)pl.tiles_n, (long long)pl.ws_bytes);
      break;
    case PK_TC_LIMB:
      snprintf(tmp, sizeof(tmp), "tc_int_planes planes=%d kp=%lld chunks=%lld bn=%d pair=%d swap=%d ws=%lld", pl.limb_L,
               (long long)pl.limb_kp, (long long)ceil_div(o.K, std::max<int64_t>(pl.limb_kc, 1)),
               pl.bn, pl.pair, pl.swap, (long long)pl.ws_bytes);
      break;
    case PK_TC_PACKED:
      snprintf(tmp, sizeof(tmp), "tc_packed pack_a=%d pack_b=%d bn=%d split=%d pair=%d sk=%d swap=%d tiles=%lldx%lld ws=%lld",
               pl.pk_a, pl.pk_b, pl.bn, pl.splits, pl.pair, pl.sk, pl.swap, (long long)pl.tiles_m,
               (long long)pl.tiles_n, (long long)pl.ws_bytes);
      break;
    default: snprintf(tmp, sizeof(tmp), "simt"); break;
  }
  const int n = (int)strlen(tmp);
  if (buf && buflen > 0) {
    strncpy(buf, tmp, (size_t)buflen - 1);
    buf[buflen - 1] = 0;
  }
  return n;
}

int mb_gemm(const mb_gemm_desc *d, void *stream) {
  Plan pl; Op o; int sms;
  int rc = plan_for(d, pl, o, sms);
  if (rc) return rc;
  if (pl.kind == PK_EMPTY) return MB_OK;
  if (pl.ws_bytes > 0 && (d->workspace == nullptr || d->workspace_bytes < pl.ws_bytes))
    return fail(MB_ERR_WORKSPACE, "workspace of %lld bytes required", (long long)pl.ws_bytes);
  cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
  const EpiScalars e = make_epi(d);
  return by_dtype(d->dtype, [&](auto *tag) -> int {
    using T = std::remove_pointer_t<decltype(tag)>;
    switch (pl.kind) {
      case PK_GEMV_COLS:
      case PK_GEMV_ROWS: return launch_gemv<T>(pl, e, d->workspace, st);
      case PK_TC:
        if constexpr (IsTc<T>::v) return launch_tc<T>(pl.swap ? swapped(o) : o, pl, e, d->workspace, sms, st);
        else return fail(MB_ERR_UNSUPPORTED, "tensor-core path for non-TC dtype");
      case PK_TC_C32: return launch_c32(o, pl, e, d->workspace, sms, st);
      case PK_TC_PACKED:
        if constexpr (IsTc<T>::v) return launch_packed<T>(o, pl, e, d->workspace, sms, st);
        else return fail(MB_ERR_UNSUPPORTED, "tensor-core path for non-TC dtype");
      case PK_TC_3XTF32:
        if constexpr (std::is_same_v<T, float>) return launch_3xtf32(o, pl, e, d->workspace, sms, st);
        else return fail(MB_ERR_UNSUPPORTED, "3xTF32 path for a non-fp32 dtype");
      case PK_TC_C64X3:
        if constexpr (std::is_same_v<T, float2>) return launch_c64x3(o, pl, e, d->workspace, sms, st);
        else return fail(MB_ERR_UNSUPPORTED, "complex64 3xTF32 path for a non-complex64 dtype");
      case PK_TC_LIMB:
        if constexpr (std::is_same_v<T, int16_t> || std::is_same_v<T, int32_t> || std::is_same_v<T, int64_t>)
          return launch_limb<T>(o, pl, e, d->workspace, sms, st);
        else return fail(MB_ERR_UNSUPPORTED, "integer plane path for a non 16/32/64-bit integer dtype");
      default: return launch_simt<T>(o, e, st);
    }
  });
}

int mb_gemm_peer(const mb_gemm_desc *d, const mb_peer_targets *peers, void *stream) {
  static_assert(MB_MAX_PEERS == tc::kMaxPeers, "peer table size");
  if (!peers) return fail(MB_ERR_INVALID, "null peer table");
  if (peers->count < 0 || peers->count > MB_MAX_PEERS)
    return fail(MB_ERR_INVALID, "peer count %d outside 0..%d", peers->count, MB_MAX_PEERS);
  for (int i = 0; i < peers->count; ++i)
    if (!peers->C[i]) return fail(MB_ERR_INVALID, "null peer output %d", i);
  if (peers->mc_C && (reinterpret_cast<uintptr_t>(peers->mc_C) & 15) != (reinterpret_cast<uintptr_t>(d->C) & 15))
    return fail(MB_ERR_INVALID, "multicast address of C must have C's 16-byte alignment");
  Plan pl; Op o; int sms;
  int rc = plan_for(d, pl, o, sms);
  if (rc) return rc;
  if (pl.kind == PK_EMPTY) return MB_OK;
  if (pl.kind != PK_TC)
    return fail(MB_ERR_UNSUPPORTED, "peer replication runs on the tensor-core plan only (bf16/fp16/int8/uint8 "
                                    "operands TMA can address); this product plans as kind %d", pl.kind);
  if (pl.bn > 256 && d->tile_n == 0) {
    // The 512-wide tile has one accumulator, so its epilogue (and with it the
    // peer stores) is exposed at each tile's end; the 256-wide tiles hide the
    // epilogue and its peer stores behind the next tile's mainloop.
    mb_gemm_desc q = *d;
    q.tile_n = 256;
    pl = Plan{};
    rc = plan_for(&q, pl, o, sms);
    if (rc) return rc;
  }
  if (pl.ws_bytes > 0 && (d->workspace == nullptr || d->workspace_bytes < pl.ws_bytes))
    return fail(MB_ERR_WORKSPACE, "workspace of %lld bytes required", (long long)pl.ws_bytes);
  cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
  const EpiScalars e = make_epi(d);
  return by_dtype(d->dtype, [&](auto *tag) -> int {
    using T = std::remove_pointer_t<decltype(tag)>;
    if constexpr (IsTc<T>::v)
      return launch_tc<T, true>(pl.swap ? swapped(o) : o, pl, e, d->workspace, sms, st, peers);
    else return fail(MB_ERR_UNSUPPORTED, "tensor-core path for non-TC dtype");
  });
}

int mb_ipc_get_handle(const void *ptr, void *handle, int64_t *offset) {
  static_assert(sizeof(cudaIpcMemHandle_t) == MB_IPC_HANDLE_BYTES, "IPC handle size");
  if (!ptr || !handle || !offset) return fail(MB_ERR_INVALID, "null argument");
  typedef CUresult (*AddrRangeFn)(CUdeviceptr *, size_t *, CUdeviceptr);
  static AddrRangeFn range_fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void *f = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuMemGetAddressRange", &f, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      range_fn = reinterpret_cast<AddrRangeFn>(f);
  });
  if (!range_fn) return fail(MB_ERR_LAUNCH, "cuMemGetAddressRange unavailable");
  CUdeviceptr base = 0;
  size_t size = 0;
  if (range_fn(&base, &size, reinterpret_cast<CUdeviceptr>(ptr)) != CUDA_SUCCESS)
    return fail(MB_ERR_INVALID, "pointer is not a device allocation");
  cudaIpcMemHandle_t h;
  int rc = cuda_check(cudaIpcGetMemHandle(&h, reinterpret_cast<void *>(base)), "cudaIpcGetMemHandle");
  if (rc) return rc;
  memcpy(handle, &h, sizeof(h));
  *offset = (int64_t)(reinterpret_cast<CUdeviceptr>(ptr) - base);
  return MB_OK;
}

int mb_ipc_open(const void *handle, void **base) {
  if (!handle || !base) return fail(MB_ERR_INVALID, "null argument");
  cudaIpcMemHandle_t h;
  memcpy(&h, handle, sizeof(h));
  return cuda_check(cudaIpcOpenMemHandle(base, h, cudaIpcMemLazyEnablePeerAccess), "cudaIpcOpenMemHandle");
}

int mb_ipc_close(void *base) {
  if (!base) return fail(MB_ERR_INVALID, "null argument");
  return cuda_check(cudaIpcCloseMemHandle(base), "cudaIpcCloseMemHandle");
}

int mb_gemv(int32_t dtype, int32_t trans, int64_t rows, int64_t cols, const void *W, int64_t ldw, const void *x,
            int64_t incx, void *y, int64_t incy, void *workspace, int64_t workspace_bytes, void *stream) {
  if (rows < 0 || cols < 0) return fail(MB_ERR_INVALID, "negative extent");
  if (trans != 0 && trans != 1) return fail(MB_ERR_INVALID, "trans must be 0 or 1");
  if (ldw < std::max<int64_t>(cols, 1)) return fail(MB_ERR_INVALID, "ldw %lld < cols %lld", (long long)ldw, (long long)cols);
  mb_gemm_desc d;
  mb_gemm_desc_init(&d);
  d.dtype = dtype;
  d.backend = MB_BACKEND_GEMV;
  d.A = nullptr; d.B = nullptr; d.C = y;
  if (trans == 0) {
    // y (rows x 1) = W (rows x cols) @ x (cols x 1)
    d.M = rows; d.N = 1; d.K = cols;
    d.A = W; d.a_rs = ldw; d.a_cs = 1;
    d.B = x; d.b_rs = incx; d.b_cs = 1;
    d.c_rs = incy; d.c_cs = 1;
  } else {
    // y (1 x cols) = x (1 x rows) @ W (rows x cols)
    d.M = 1; d.N = cols; d.K = rows;
    d.A = x; d.a_rs = 1; d.a_cs = incx;
    d.B = W; d.b_rs = ldw; d.b_cs = 1;
    d.c_rs = 1; d.c_cs = incy;
  }
  d.workspace = workspace;
  d.workspace_bytes = workspace ? workspace_bytes : 0;
  if (!workspace) d.split_k = 1;
  return mb_gemm(&d, stream);
}

int mb_autotune_record(const mb_gemm_desc *d, const mb_plan_override *ov) {
  if (!d || !ov) return fail(MB_ERR_INVALID, "null argument");
  const std::string key = tune_key(d);
  std::lock_guard<std::mutex> lk(g_tune_mu);
  g_tune[key] = Override{ov->keep ? 1 : 0, ov->backend, ov->tile_n, ov->split_k, ov->swap_ab, ov->cta_pair,
                         ov->stream_k};
  g_tune_size.store((int64_t)g_tune.size());
  return MB_OK;
}

int mb_autotune_lookup(const mb_gemm_desc *d, mb_plan_override *ov) {
  if (!d || !ov) return -fail(MB_ERR_INVALID, "null argument");
  const std::string key = tune_key(d);
  std::lock_guard<std::mutex> lk(g_tune_mu);
  auto it = g_tune.find(key);
  if (it == g_tune.end()) return 0;
  const Override &o = it->second;
  ov->keep = o.keep; ov->backend = o.backend; ov->tile_n = o.tile_n; ov->split_k = o.split_k;
  ov->swap_ab = o.swap_ab; ov->cta_pair = o.cta_pair; ov->stream_k = o.stream_k;
  return 1;
}

static const char kTuneHeader[] = "metalblas_b200 autotune v1";

int mb_autotune_cache_load(const char *path) {
  if (!path) return fail(MB_ERR_INVALID, "null path");
  FILE *f = fopen(path, "r");
  if (!f) return fail(MB_ERR_INVALID, "cannot open %s", path);
  std::unordered_map<std::string, Override> add;
  char line[1024];
  bool ok = fgets(line, sizeof(line), f) && strncmp(line, kTuneHeader, sizeof(kTuneHeader) - 1) == 0;
  while (ok && fgets(line, sizeof(line), f)) {
    char *tab = strchr(line, '\t');
    if (!tab) { ok = line[0] == '\n' || line[0] == 0; continue; }
    *tab = 0;
    Override o{};
    if (sscanf(tab + 1, "%d %d %d %d %d %d %d", &o.keep, &o.backend, &o.tile_n, &o.split_k, &o.swap_ab, &o.cta_pair,
               &o.stream_k) != 7) { ok = false; break; }
    add[line] = o;
  }
  fclose(f);
  if (!ok) return fail(MB_ERR_INVALID, "malformed autotune cache %s", path);
  std::lock_guard<std::mutex> lk(g_tune_mu);
  for (auto &kv : add) g_tune[kv.first] = kv.second;
  g_tune_size.store((int64_t)g_tune.size());
  return MB_OK;
}

int mb_autotune_cache_save(const char *path) {
  if (!path) return fail(MB_ERR_INVALID, "null path");
  const std::string tmp = std::string(path) + ".tmp";
  FILE *f = fopen(tmp.c_str(), "w");
  if (!f) return fail(MB_ERR_INVALID, "cannot write %s", tmp.c_str());
  fprintf(f, "%s\n", kTuneHeader);
  {
    std::lock_guard<std::mutex> lk(g_tune_mu);
    for (auto &kv : g_tune) {
      const Override &o = kv.second;
      fprintf(f, "%s\t%d %d %d %d %d %d %d\n", kv.first.c_str(), o.keep, o.backend, o.tile_n, o.split_k, o.swap_ab,
              o.cta_pair, o.stream_k);
    }
  }
  if (fclose(f) != 0 || rename(tmp.c_str(), path) != 0) return fail(MB_ERR_INVALID, "cannot write %s", path);
  return MB_OK;
}

void mb_autotune_cache_clear(void) {
  std::lock_guard<std::mutex> lk(g_tune_mu);
  g_tune.clear();
  g_tune_size.store(0);
}

int64_t mb_autotune_cache_size(void) { return g_tune_size.load(); }

}  // extern "C"

// ---------------------------------------------------------------------------
// Allocation-free variant of mb_gemm.
//
// Some callers of this library cannot call cudaMalloc and have no workspace to
// hand over: inference runtimes that reserve all device memory at start-up and
// forbid allocation on the request path (cudaMalloc may synchronise the device
// and its latency is unbounded), plugin hosts whose per-layer callback passes a
// plugin nothing but its input/output buffers and a stream, and foreign-language
// callers of the C ABI that have no CUDA allocator of their own.  For them the
// split-K scratch lives in this file-scope device array, of fixed size
// MB_NOALLOC_SCRATCH_BYTES, which every GPU that loads the library holds until
// the process exits.
//
// In host code `g_noalloc_scratch` names a host-side stand-in, not a device
// address, so its device address is looked up with cudaGetSymbolAddress once
// per device (with that device current) and that pointer is what the kernels
// get.  Every call on a device shares the array and it keeps the last call's
// contents: the ticket counters, which must start at zero, are cleared on the
// call's stream before each launch that uses them, and calls that overlap on
// the GPU (for example on two streams at once) race on the array.
static __device__ __align__(256) unsigned char g_noalloc_scratch[MB_NOALLOC_SCRATCH_BYTES];

namespace {
std::mutex g_noalloc_mu;
void *g_noalloc_ptr[64] = {nullptr};

// Device address of the scratch array on the current device (set-up on the
// first call for that device).
int noalloc_scratch(void **out) {
  int dev = 0;
  int rc = current_device(&dev);
  if (rc) return rc;
  if (dev < 0 || dev >= 64) return fail(MB_ERR_UNSUPPORTED, "device index %d out of range", dev);
  std::lock_guard<std::mutex> lk(g_noalloc_mu);
  if (!g_noalloc_ptr[dev]) {
    void *p = nullptr;
    rc = cuda_check(cudaGetSymbolAddress(&p, g_noalloc_scratch), "cudaGetSymbolAddress(g_noalloc_scratch)");
    if (rc) return rc;
    g_noalloc_ptr[dev] = p;
  }
  *out = g_noalloc_ptr[dev];
  return MB_OK;
}
}  // namespace

extern "C" {

int mb_gemm_noalloc(const mb_gemm_desc *d, void *stream) {
  if (!d) return fail(MB_ERR_INVALID, "null descriptor");
  // Same plan as mb_gemm given a workspace; d->workspace is ignored.
  mb_gemm_desc q = *d;
  q.workspace = nullptr;
  q.workspace_bytes = -1;
  Plan pl; Op o; int sms;
  int rc = plan_for(&q, pl, o, sms);
  if (rc) return rc;
  if (pl.kind == PK_EMPTY) return MB_OK;
  const int64_t cap = (int64_t)MB_NOALLOC_SCRATCH_BYTES;
  const bool split_forced = d->split_k > 1 || d->stream_k == 2;
  if (pl.ws_bytes > cap && !split_forced) {
    // The planner's first choice needs more scratch than the built-in buffer
    // holds, and the caller did not ask for a K split: plan again as mb_gemm
    // does without a workspace.  Plain tensor-core products then run without a
    // split-K / stream-K tail; complex32, packed operands, 3xTF32 (fp32,
    // complex64) and integer byte planes need scratch for their operand copies,
    // so under AUTO those products move to the CUDA-core kernel (no scratch,
    // any layout), and under an explicit tensor-core backend they are refused.
    mb_gemm_desc r = q;
    r.workspace_bytes = 0;
    pl = Plan{};  // a fresh plan: the planners fill only the fields their kind uses
    rc = plan_for(&r, pl, o, sms);
    if (rc)
      return fail(MB_ERR_WORKSPACE,
                  "mb_gemm_noalloc: this product needs operand scratch beyond the built-in %lld bytes on the "
                  "requested backend; call mb_gemm with a workspace or use backend AUTO",
                  (long long)cap);
  }
  cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
  void *scratch = nullptr;
  if (pl.ws_bytes > 0) {
    if (pl.ws_bytes > cap) {
      if (pl.kind == PK_TC || pl.kind == PK_GEMV_COLS || pl.kind == PK_GEMV_ROWS)
        return fail(MB_ERR_WORKSPACE,
                    "mb_gemm_noalloc: this plan needs %lld bytes of split-K scratch but the built-in scratch "
                    "holds %lld bytes; set split_k=1 (no scratch) or call mb_gemm with a workspace",
                    (long long)pl.ws_bytes, (long long)cap);
      return fail(MB_ERR_WORKSPACE,
                  "mb_gemm_noalloc: this plan needs %lld bytes of scratch but the built-in scratch holds %lld "
                  "bytes; call mb_gemm with a workspace",
                  (long long)pl.ws_bytes, (long long)cap);
    }
    rc = noalloc_scratch(&scratch);
    if (rc) return rc;
    rc = cuda_check(cudaMemsetAsync(scratch, 0, (size_t)kTicketBytes, st), "clear noalloc ticket counters");
    if (rc) return rc;
  }
  const EpiScalars e = make_epi(d);
  return by_dtype(d->dtype, [&](auto *tag) -> int {
    using T = std::remove_pointer_t<decltype(tag)>;
    switch (pl.kind) {
      case PK_GEMV_COLS:
      case PK_GEMV_ROWS: return launch_gemv<T>(pl, e, scratch, st);
      case PK_TC:
        if constexpr (IsTc<T>::v) return launch_tc<T>(pl.swap ? swapped(o) : o, pl, e, scratch, sms, st);
        else return fail(MB_ERR_UNSUPPORTED, "tensor-core path for non-TC dtype");
      case PK_TC_C32: return launch_c32(o, pl, e, scratch, sms, st);
      case PK_TC_PACKED:
        if constexpr (IsTc<T>::v) return launch_packed<T>(o, pl, e, scratch, sms, st);
        else return fail(MB_ERR_UNSUPPORTED, "tensor-core path for non-TC dtype");
      case PK_TC_3XTF32:
        if constexpr (std::is_same_v<T, float>) return launch_3xtf32(o, pl, e, scratch, sms, st);
        else return fail(MB_ERR_UNSUPPORTED, "3xTF32 path for a non-fp32 dtype");
      case PK_TC_C64X3:
        if constexpr (std::is_same_v<T, float2>) return launch_c64x3(o, pl, e, scratch, sms, st);
        else return fail(MB_ERR_UNSUPPORTED, "complex64 3xTF32 path for a non-complex64 dtype");
      case PK_TC_LIMB:
        if constexpr (std::is_same_v<T, int16_t> || std::is_same_v<T, int32_t> || std::is_same_v<T, int64_t>)
          return launch_limb<T>(o, pl, e, scratch, sms, st);
        else return fail(MB_ERR_UNSUPPORTED, "integer plane path for a non 16/32/64-bit integer dtype");
      default: return launch_simt<T>(o, e, st);
    }
  });
}

const char *mb_last_error_string(void) { return g_err.c_str(); }

int mb_device_status(void) {
  int rc = cuda_check(cudaDeviceSynchronize(), "cudaDeviceSynchronize");
  if (rc) return rc;
  int v = 0;
  rc = cuda_check(cudaMemcpyFromSymbol(&v, g_mb_status, sizeof(int)), "read status");
  if (rc) return rc;
  return v;
}

void mb_device_status_clear(void) {
  int z = 0;
  cudaMemcpyToSymbol(g_mb_status, &z, sizeof(int));
}

int mb_debug_wait_timeout(int64_t limit_us, void *stream) {
  if (limit_us <= 0 || limit_us > 10000000) return fail(MB_ERR_INVALID, "limit_us out of range");
  tc::wait_timeout_kernel<<<1, 32, 0, reinterpret_cast<cudaStream_t>(stream)>>>((unsigned long long)limit_us * 1000ull);
  return cuda_check(cudaGetLastError(), "wait_timeout launch");
}

int mb_peak_probe(int32_t kind, double *tops) {
  if (!tops) return fail(MB_ERR_INVALID, "null output");
  if (kind < 0 || kind > 2) return fail(MB_ERR_INVALID, "probe kind must be 0 (fp32), 1 (int32) or 2 (int64)");
  int dev = 0;
  int rc = current_device(&dev);
  if (rc) return rc;
  const int sms = num_sms(dev);
  const dim3 grid((unsigned)(4 * sms)), block(256);
  void *out = nullptr;
  rc = cuda_check(cudaMalloc(&out, (size_t)grid.x * block.x * 8), "probe buffer");
  if (rc) return rc;
  cudaStream_t st = nullptr;
  cudaEvent_t e0 = nullptr, e1 = nullptr;
  float ms = 0.f;
  long long iters = 4096;
  auto launch = [&](long long n) {
    if (kind == 0) peak_mad_kernel<float><<<grid, block, 0, st>>>((float *)out, 1.0001f, n);
    else if (kind == 1) peak_mad_kernel<uint32_t><<<grid, block, 0, st>>>((uint32_t *)out, 3u, n);
    else peak_mad_kernel<unsigned long long><<<grid, block, 0, st>>>((unsigned long long *)out, 3ull, n);
  };
  rc = cuda_check(cudaStreamCreateWithFlags(&st, cudaStreamNonBlocking), "probe stream");
  if (!rc) rc = cuda_check(cudaEventCreate(&e0), "probe event");
  if (!rc) rc = cuda_check(cudaEventCreate(&e1), "probe event");
  if (!rc) {
    launch(64);  // warm-up
    // grow the step count until one launch takes at least 20 ms
    for (int tries = 0; tries < 8 && !rc; ++tries) {
      cudaEventRecord(e0, st);
      launch(iters);
      cudaEventRecord(e1, st);
      rc = cuda_check(cudaEventSynchronize(e1), "probe run");
      if (!rc) rc = cuda_check(cudaEventElapsedTime(&ms, e0, e1), "probe timing");
      if (rc || ms >= 20.f) break;
      iters *= 4;
    }
  }
  if (!rc) rc = cuda_check(cudaGetLastError(), "probe launch");
  if (e0) cudaEventDestroy(e0);
  if (e1) cudaEventDestroy(e1);
  if (st) cudaStreamDestroy(st);
  cudaFree(out);
  if (rc) return rc;
  const double ops = 2.0 * kPeakChains * 16.0 * (double)iters * grid.x * block.x;
  *tops = ops / (ms * 1e-3) / 1e12;
  return MB_OK;
}

int mb_abi_version(void) { return MB_ABI_VERSION; }
int mb_built_sm(void) { return 100; }

}  // extern "C"
