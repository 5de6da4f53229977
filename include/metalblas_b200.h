/*
 * metalblas_b200 — C ABI of the B200 (sm_100a) matmul / addmm / bmm hot path.
 *
 * Every entry point takes plain device pointers, element strides and a CUDA
 * stream (passed as void* so no CUDA header is needed to bind it).  The library
 * never allocates or frees caller memory; scratch space for split-K partials is
 * passed in by the caller (see mb_gemm_workspace_size).  All launches are
 * asynchronous on the given stream.
 *
 * The reference (Isalia20/metalBLAS) has no C ABI: its "FFI" is the set of
 * launchable Metal pipelines returned by metalblas/kernels.py, called as
 *   fn(*buffers, packed_dims, [bias, int2 bstride, float beta, float alpha],
 *      [int4 batch], threads=..., group_size=...)
 * from metalblas/float_dispatch.py:770-775, :945-947, :1087,
 * metalblas/integer_dispatch.py:108-117, :135-146 and
 * metalblas/complex_dispatch.py:60-66, :114.  Each entry point below names the
 * reference interface it replaces.
 */
#ifndef METALBLAS_B200_H
#define METALBLAS_B200_H

#include <stdint.h>
#include <stddef.h>

#ifdef __cplusplus
extern "C" {
#endif

#define MB_ABI_VERSION 1

/* Element types.  Output dtype == input dtype (torch semantics, reference
 * metalblas/dispatch.py:106-114 and integer_dispatch.py:13-19). */
typedef enum mb_dtype {
    MB_F32 = 0, MB_F16 = 1, MB_BF16 = 2,
    MB_C64 = 3,            /* interleaved float2 (torch.complex64)            */
    MB_C32 = 4,            /* interleaved half2  (torch.complex32 / chalf)    */
    MB_I8 = 5, MB_U8 = 6, MB_I16 = 7, MB_I32 = 8, MB_I64 = 9
} mb_dtype;

/* Backend selection; names follow the reference's backend= strings
 * (metalblas/float_dispatch.py:802-852). */
typedef enum mb_backend {
    MB_BACKEND_AUTO = 0,   /* tile table picks                                  */
    MB_BACKEND_GEMV = 1,   /* "gemv": bandwidth kernels, needs M==1 or N==1
                            * (or min(M, N) <= 4 for 16-bit floats, <= 32 fp32) */
    MB_BACKEND_TC   = 2,   /* "mpp_tensor": tcgen05/TMEM tensor-core GEMM; fp32
                            * and complex64 as 3xTF32, 16/32/64-bit integers as
                            * byte planes on the int8 tensor cores (bit-exact)  */
    MB_BACKEND_SIMT = 3    /* "simd" (and "mpp" fallback): CUDA-core FFMA/IMAD  */
} mb_backend;

/* Status codes; the Python layer maps them onto the reference's exception types
 * (AssertionError / ValueError / NotImplementedError / RuntimeError). */
typedef enum mb_status {
    MB_OK = 0,
    MB_ERR_INVALID = 1,        /* bad shape / stride / pointer / tile      -> ValueError/AssertionError */
    MB_ERR_UNSUPPORTED = 2,    /* dtype or layout not handled by the forced backend -> NotImplementedError */
    MB_ERR_LAUNCH = 3,         /* CUDA launch or driver error               -> RuntimeError */
    MB_ERR_DEVICE_TIMEOUT = 4, /* a bounded device-side wait ran out        -> RuntimeError */
    MB_ERR_WORKSPACE = 5       /* workspace missing or too small            -> ValueError */
} mb_status;

/*
 * One (batched) GEMM with optional fused epilogue:
 *   C[b] = alpha * (op(A[b]) @ op(B[b])) + beta * bias[b]          (epilogue)
 *   C[b] = A[b] @ B[b]                                            (no epilogue)
 * Element (m,k) of A[b] is A[b*sA + m*a_rs + k*a_cs]; B(k,n) is
 * B[b*sB + k*b_rs + n*b_cs]; C(m,n) is C[b*sC + m*c_rs + n*c_cs]; bias(m,n) is
 * bias[b*bias_bs + m*bias_rs + n*bias_cs].  All strides are in ELEMENTS and
 * 64-bit (the reference packs int32 offsets, metalblas/dispatch.py:12-16).
 * A batch stride of 0 broadcasts that operand (reference keeps stride 0,
 * metalblas/dispatch.py:96-103, float_dispatch.py:1071-1087).
 * Row-major A is a_cs==1, a_rs==lda; column-major ("trans_a") is a_rs==1,
 * a_cs==lda (reference _unit_lead, metalblas/dispatch.py:23-30).  Other stride
 * pairs are accepted and read in place by the CUDA-core kernel.
 * conj_a / conj_b conjugate a complex operand on load (the reference
 * materialises it, metalblas/complex_dispatch.py:25-30).
 * Epilogue semantics follow metalblas/shaders/mb_epi.h:16-26: with
 * alpha_nz==0 the product is not used, with beta_nz==0 bias is never read
 * (so NaN in bias cannot leak).  Float/complex epilogues compute in fp32
 * (complex: complex multiply, shaders/complex_pack.h:43-55); integer epilogues
 * compute in the accumulator type with two's-complement wrap using ialpha/ibeta.
 */
typedef struct mb_gemm_desc {
    int32_t dtype;          /* mb_dtype */
    int32_t backend;        /* mb_backend */
    int64_t M, N, K, batch;
    const void *A;
    const void *B;
    void *C;
    int64_t a_rs, a_cs, sA;
    int64_t b_rs, b_cs, sB;
    int64_t c_rs, c_cs, sC;
    int32_t conj_a, conj_b;
    /* epilogue */
    int32_t epilogue;       /* 0: plain product; 1: alpha/beta/bias epilogue */
    int32_t alpha_nz, beta_nz;
    int32_t stream_k;       /* plan override, TC: 0 planner decides, 1 no stream-K tail, 2 stream-K tail */
    const void *bias;       /* same dtype as C */
    int64_t bias_rs, bias_cs, bias_bs;
    double alpha_re, alpha_im, beta_re, beta_im;   /* float / complex scalars */
    int64_t ialpha, ibeta;                         /* integer scalars         */
    /* plan overrides (0 = planner decides) */
    int32_t tile_n;         /* TC: N-tile of the tcgen05 kernel (16..256)     */
    int32_t split_k;        /* TC/GEMV: number of K splits                    */
    int32_t swap_ab;        /* TC: -1 never, 0 planner decides, 1 force Cᵀ=BᵀAᵀ */
    int32_t cta_pair;       /* TC: 0 planner decides, 1 one CTA per tile, 2 CTA pair (cta_group::2) */
    /* caller-owned scratch for split-K partials; must be zero-filled before
     * its first use; kernels leave the counter region zeroed again. */
    void *workspace;
    int64_t workspace_bytes;
} mb_gemm_desc;

/* Fill *d with defaults (backend AUTO, alpha=beta=1, no epilogue, batch=1). */
void mb_gemm_desc_init(mb_gemm_desc *d);

/* Launch one (batched) GEMM on `stream` (a cudaStream_t; NULL = legacy default).
 * Replaces the mpp_tensor / mpp / simd / int_gemm / gemv_t / gemv_nt / gemv_bt /
 * splitk_gemm+splitk_reduce / complex split+combine launches of
 * metalblas/float_dispatch.py:745-852, 897-956, 1049-1091,
 * metalblas/integer_dispatch.py:92-150 and metalblas/complex_dispatch.py:33-129. */
int mb_gemm(const mb_gemm_desc *d, void *stream);

/* Allocation-free variant of mb_gemm.  No counterpart in the reference.
 *
 * For callers that cannot call cudaMalloc and have no workspace to pass:
 * inference runtimes that reserve all device memory at start-up and forbid
 * allocation on the request path (cudaMalloc may synchronise the device and its
 * latency is unbounded), plugin hosts whose callbacks hand a plugin only its
 * input/output buffers and a stream, and foreign-language callers without a
 * CUDA allocator.  Same descriptor and plan as mb_gemm, but d->workspace is
 * ignored: split-K scratch comes from a buffer compiled into the library,
 * MB_NOALLOC_SCRATCH_BYTES per GPU, held by every GPU that loads the library
 * until the process exits.  When the planner's first choice needs more
 * scratch than that and the caller forced no K split (split_k <= 1, stream_k
 * != 2), the call is planned again as mb_gemm plans without a workspace:
 * bf16/fp16/int8/uint8 tensor-core products drop their split-K / stream-K
 * tail, and the products whose tensor-core forms need operand copies in
 * scratch (complex32, operands TMA cannot address, fp32 and complex64 as
 * 3xTF32, 16/32/64-bit integers as byte planes) run on the CUDA-core FFMA /
 * IMAD kernel under backend AUTO, several times slower than mb_gemm for large
 * products, and are refused with MB_ERR_WORKSPACE under backend TC.  A forced
 * split (split_k > 1 or stream_k == 2) whose scratch does not fit is refused
 * with MB_ERR_WORKSPACE (split_k = 1 runs a plain tensor-core product without
 * scratch).
 * The call allocates nothing: no cudaMalloc / cudaFree, no allocating library
 * routine.  The first call on a device looks up the buffer's device address
 * (per-device set-up); make that first call before any stream capture.  All
 * calls on a device share the one buffer, which keeps the last call's
 * contents; its counters are cleared on the call's stream before use.  Calls
 * that overlap on the GPU (e.g. on two streams at once) race on the buffer:
 * keep them ordered on one stream. */
#define MB_NOALLOC_SCRATCH_BYTES (16u * 1024u * 1024u)
int mb_gemm_noalloc(const mb_gemm_desc *d, void *stream);

/* ---------------------------------------------------------------------------
 * Multi-GPU: the product fused with its output gather over NVLink.
 *
 * The reference is single-device; its sharded counterpart here splits a large
 * GEMM along N (or a bmm along the batch) over the GPUs of one node, and the
 * north star's "output gathered over NVLink" step is folded into the GEMM's
 * epilogue: every finished output tile is stored into this GPU's C (TMA store)
 * AND into each peer GPU's copy of C at the same element offset (plain 16-byte
 * st.global over NVLink, 64-byte row runs per warp store).  Loads and tensor
 * maps only ever address this GPU's memory; nothing multicasts.
 *
 * mb_gemm_peer computes what mb_gemm computes for `d` and also writes every
 * element of C, at the same offset from peers->C[i], for i < peers->count.
 * peers->C[i] must be device addresses valid in the calling process (a peer
 * buffer mapped with mb_ipc_open) laid out with d's C strides.  Runs on the
 * tensor-core plan only (bf16 / fp16 / int8 / uint8 operands TMA can address):
 * other plans return MB_ERR_UNSUPPORTED.  The peers see complete results only
 * after every GPU's launch has finished: order a cross-GPU barrier (a NCCL
 * all-reduce of one word on the same stream serves) between this call and any
 * reader, and do not start a call that overwrites a peer's C while that peer
 * may still read it (alternate two buffers, or barrier before the call). */
#define MB_MAX_PEERS 7
typedef struct mb_peer_targets {
    int32_t count;                 /* peers that receive the output (0..MB_MAX_PEERS) */
    void *C[MB_MAX_PEERS];         /* each peer's copy of C, same strides as desc->C */
    void *mc_C;                    /* NULL, or the NVSwitch multicast address of C (every
                                    * rank's copy, this one included, bound to one multicast
                                    * object): whole 16-byte chunks are then written once
                                    * with multimem.st and the switch replicates them;
                                    * partial chunks still use C[] */
} mb_peer_targets;
int mb_gemm_peer(const mb_gemm_desc *d, const mb_peer_targets *peers, void *stream);

/* CUDA IPC plumbing for the peer buffers (one process per GPU).
 * mb_ipc_get_handle: the IPC handle (MB_IPC_HANDLE_BYTES opaque bytes) of the
 * device allocation that contains `ptr`, and ptr's byte offset within it.
 * mb_ipc_open: map another process's allocation into this one (peer access
 * enabled on first use); *base receives the mapped base address (add the
 * owner's offset).  mb_ipc_close: unmap a base returned by mb_ipc_open. */
#define MB_IPC_HANDLE_BYTES 64
int mb_ipc_get_handle(const void *ptr, void *handle, int64_t *offset);
int mb_ipc_open(const void *handle, void **base);
int mb_ipc_close(void *base);

/* Bytes of workspace mb_gemm needs for this descriptor's plan (0 if none).
 * Replaces the split-K partial pool of metalblas/float_dispatch.py:183-192. */
int64_t mb_gemm_workspace_size(const mb_gemm_desc *d);

/* Describe the plan mb_gemm would run, as text ("tc bn=256 split=1 swap=0 ...").
 * Replaces the plan/tile lookups of metalblas/float_dispatch.py:484-505 (the
 * tile that _gemm_plan returns). Returns the string length written. */
int mb_plan_query(const mb_gemm_desc *d, char *buf, int buflen);

/* y = op(W) x for a unit-stride matrix W (rows x cols, element (r, c) at
 * W[r*ldw + c]): trans == 0 gives y[r] = sum_c W(r,c) x[c] (rows outputs),
 * trans == 1 gives y[c] = sum_r W(r,c) x[r] (cols outputs).  x and y are
 * strided by incx / incy elements; y has W's dtype.  Replaces the GEMV routing
 * of _dispatch_gemv (metalblas/dispatch.py:49-70) onto the gemv_t / gemv_nt
 * kernels (metalblas/shaders/gemv_t.h:15-99, gemv_nt.h:16-101) and the
 * integer / complex GEMVs (metalblas/integer_dispatch.py:92-105,
 * complex_dispatch.py:33-66).  A workspace (size from mb_gemm_workspace_size
 * of the equivalent mb_gemm descriptor) lets long reductions split across
 * CTAs; with workspace == NULL the reduction stays in one CTA per output
 * block. */
int mb_gemv(int32_t dtype, int32_t trans, int64_t rows, int64_t cols, const void *W, int64_t ldw,
            const void *x, int64_t incx, void *y, int64_t incy, void *workspace, int64_t workspace_bytes,
            void *stream);

/* Per-shape plan overrides: the autotune cache, kept in the library so that
 * every caller of mb_gemm gets tuned plans.  The reference caches autotune
 * winners in module dicts keyed by shape (metalblas/float_dispatch.py:154,
 * 484-505, 977-1045); here the key is the device name, dtype, M, N, K, batch,
 * broadcast flags, layout/alignment class and epilogue flag of a descriptor.
 * mb_gemm consults the table only for descriptors with backend AUTO and no
 * plan override of their own.  keep == 1 records "tuned: the tile table's
 * choice stands".  All functions are thread-safe. */
typedef struct mb_plan_override {
    int32_t keep;
    int32_t backend, tile_n, split_k, swap_ab, cta_pair, stream_k;
} mb_plan_override;
int mb_autotune_record(const mb_gemm_desc *d, const mb_plan_override *ov);
/* 1 and *ov filled on a hit, 0 on a miss, negative mb_status on error. */
int mb_autotune_lookup(const mb_gemm_desc *d, mb_plan_override *ov);
/* Text file, one entry per line; save writes `path` atomically (via a
 * temporary file).  load replaces nothing on a missing or malformed file
 * (returns MB_ERR_INVALID) and otherwise merges the file's entries. */
int mb_autotune_cache_load(const char *path);
int mb_autotune_cache_save(const char *path);
void mb_autotune_cache_clear(void);
int64_t mb_autotune_cache_size(void);

/* Text of the last error raised on this thread. */
const char *mb_last_error_string(void);

/* Device status word of the current device: 0, or MB_ERR_DEVICE_TIMEOUT if a
 * bounded device-side wait ran out since the last mb_device_status_clear.
 * Synchronises the current device.  The reference has no device-side waits. */
int mb_device_status(void);
void mb_device_status_clear(void);

/* Testing hook for the bounded-wait path: launches a kernel that waits on an
 * mbarrier nothing will complete, with the given limit in microseconds; the
 * kernel must give up, record MB_ERR_DEVICE_TIMEOUT and return. */
int mb_debug_wait_timeout(int64_t limit_us, void *stream);

/* Measured CUDA-core multiply-add throughput of the current device, in 1e12
 * operations per second (a multiply-add counts 2, as in 2*M*N*K): kind 0 fp32
 * FFMA, 1 int32 IMAD, 2 int64 multiply-add.  These are the roofline
 * denominators of the CUDA-core GEMM (complex64/fp32, int16/int32, int64),
 * for which no published B200 figure exists; the reference has no
 * counterpart.  Runs for about 20 ms and synchronises its own stream. */
int mb_peak_probe(int32_t kind, double *tops);

/* Library ABI version (MB_ABI_VERSION) and the SM arch it was built for (100). */
int mb_abi_version(void);
int mb_built_sm(void);

#ifdef __cplusplus
}
#endif
#endif /* METALBLAS_B200_H */
