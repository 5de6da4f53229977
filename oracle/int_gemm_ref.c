/*
 * C restatement of the reference's integer GEMM arithmetic — TEST
 * INFRASTRUCTURE ONLY (used by tests/ as a second, independent checker; the
 * product never links it).
 *
 * The reference kernel metalblas/shaders/int_gemm.h:41-154 accumulates every
 * output in ACC_T (int for char/short/int, uint for uchar, long for long;
 * metalblas/integer_dispatch.py:13-19), applies the fused epilogue
 * v = alpha*acc + beta*bias in ACC_T (metalblas/shaders/mb_epi.h:16-26, with
 * alpha_nz / beta_nz switches) and stores with a truncating cast to OUT_T.
 * Signed overflow is undefined in C, so the accumulation below is done in the
 * unsigned type of the same width, which produces the same bits as the
 * two's-complement wrap of the GPU.
 *
 * dtype codes follow include/metalblas_b200.h: 5 int8, 6 uint8, 7 int16,
 * 8 int32, 9 int64.
 */
#include <stdint.h>
#include <stddef.h>

static uint64_t load_u64(int dtype, const void *p, int64_t idx) {
    switch (dtype) {
        case 5: return (uint64_t)(int64_t)((const int8_t *)p)[idx];
        case 6: return (uint64_t)((const uint8_t *)p)[idx];
        case 7: return (uint64_t)(int64_t)((const int16_t *)p)[idx];
        case 8: return (uint64_t)(int64_t)((const int32_t *)p)[idx];
        default: return (uint64_t)((const int64_t *)p)[idx];
    }
}

static void store_trunc(int dtype, void *p, int64_t idx, uint64_t v) {
    switch (dtype) {
        case 5: ((int8_t *)p)[idx] = (int8_t)(uint8_t)v; break;
        case 6: ((uint8_t *)p)[idx] = (uint8_t)v; break;
        case 7: ((int16_t *)p)[idx] = (int16_t)(uint16_t)v; break;
        case 8: ((int32_t *)p)[idx] = (int32_t)(uint32_t)v; break;
        default: ((int64_t *)p)[idx] = (int64_t)v; break;
    }
}

/* ACC_T width in bits: 32 except int64 (64). */
static int acc_bits(int dtype) { return dtype == 9 ? 64 : 32; }

int mb_ref_int_gemm(int dtype, int64_t M, int64_t N, int64_t K,
                    const void *A, int64_t a_rs, int64_t a_cs,
                    const void *B, int64_t b_rs, int64_t b_cs,
                    void *C, int64_t c_rs, int64_t c_cs,
                    int epilogue, const void *bias, int64_t bias_rs, int64_t bias_cs,
                    int64_t alpha, int64_t beta, int alpha_nz, int beta_nz) {
    if (dtype < 5 || dtype > 9) return 1;
    const int wide = acc_bits(dtype) == 64;
    for (int64_t m = 0; m < M; ++m) {
        for (int64_t n = 0; n < N; ++n) {
            uint64_t acc64 = 0;
            uint32_t acc32 = 0;
            for (int64_t k = 0; k < K; ++k) {
                uint64_t a = load_u64(dtype, A, m * a_rs + k * a_cs);
                uint64_t b = load_u64(dtype, B, k * b_rs + n * b_cs);
                if (wide) acc64 += a * b;
                else acc32 += (uint32_t)a * (uint32_t)b;
            }
            uint64_t v = wide ? acc64 : (uint64_t)acc32;
            if (epilogue) {
                uint64_t r = 0;
                if (alpha_nz) r = wide ? (uint64_t)alpha * v : (uint64_t)((uint32_t)alpha * (uint32_t)v);
                if (beta_nz) {
                    uint64_t bv = load_u64(dtype, bias, m * bias_rs + n * bias_cs);
                    r = wide ? r + (uint64_t)beta * bv
                             : (uint64_t)((uint32_t)r + (uint32_t)beta * (uint32_t)bv);
                }
                v = r;
            }
            store_trunc(dtype, C, m * c_rs + n * c_cs, v);
        }
    }
    return 0;
}
