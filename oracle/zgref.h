/*
 * zgref.h -- CPU oracle for the zerograd population-evaluation and
 * factor-replay path.  TEST INFRASTRUCTURE ONLY: the product library
 * (zerograd_b200/libzgb200.so) never links or calls this code; only the
 * tests, the smoke check and the CPU baseline leg of bench.py do.
 *
 * Everything here restates, in plain C, the arithmetic the reference
 * reaches through jax.random / zlib (third-party code that is not part of
 * the reference tree; pinned versions jax 0.10.2 / jaxlib 0.10.2, see the
 * reference's uv.lock):
 *   - zlib CRC-32 (src/zerograd/_keys.py:29-30)
 *   - threefry2x32 with 20 rounds (Salmon et al., SC'11; the Random123
 *     specification), used by jax.random.key / fold_in / split / bits in the
 *     partitionable mode (src/zerograd/_keys.py:30,40,53,58)
 *   - float32 uniform via the mantissa trick and the standard normal as
 *     sqrt(2)*erfinv(u) with Giles' single-precision erfinv
 *     (src/zerograd/_factors.py:43-74)
 *   - the factor layouts of matrix_factors / table_factors / vector_noise
 *   - the exact int8 x int8 -> int32 GEMM + LUT epilogue that defines the
 *     integer QAT linear (no reference counterpart; the semantics are fixed
 *     here and matched by the CUDA kernel).
 */
#ifndef ZGREF_H
#define ZGREF_H
#include <stdint.h>
#include <stddef.h>

#ifdef __cplusplus
extern "C" {
#endif

uint32_t zgo_crc32(const uint8_t* data, size_t n);

/* One threefry2x32-20 block: key (k0,k1), counter (c0,c1) -> out[2]. */
void zgo_threefry2x32(uint32_t k0, uint32_t k1, uint32_t c0, uint32_t c1, uint32_t out[2]);

/* jax.random.fold_in(key, d) for a 32-bit d: threefry(key, (0, d)). */
void zgo_fold_in(const uint32_t key[2], uint32_t d, uint32_t out[2]);

/* jax.random.split(key, n) (partitionable): row i = threefry(key, (0, i)). */
void zgo_split(const uint32_t key[2], int64_t n, uint32_t* out /* [n,2] */);

/* 32-bit random bits of a flat array of n elements (partitionable):
 * element j = o0 ^ o1 with (o0,o1) = threefry(key, (hi32(j), lo32(j))). */
void zgo_random_bits32(const uint32_t key[2], int64_t n, uint32_t* out);

/* Bits -> float32 uniform in [lo, hi): mantissa trick, affine map, clamp. */
float zgo_bits_to_uniform(uint32_t bits, float lo, float hi);

/* Giles' single-precision erfinv (published method), with libm log1pf. */
float zgo_erfinv_f32(float x);

/* Bits -> standard normal exactly as jax.random.normal(float32). */
float zgo_bits_to_normal(uint32_t bits);

/* jax.random.normal(key, (n,), float32), flat order. */
void zgo_normal_f32(const uint32_t key[2], int64_t n, float* out);

/* matrix_factors: A[rows,rank] from split(gk)[0], B[rank,cols] from split(gk)[1]. */
void zgo_matrix_factors(const uint32_t gk[2], int64_t rows, int64_t cols, int rank,
                        float* A, float* B);
/* table_factors: A[rows,rank] from split(gk)[0], B[cols,rank] from split(gk)[1]. */
void zgo_table_factors(const uint32_t gk[2], int64_t rows, int64_t cols, int rank,
                       float* A, float* B);
/* vector_noise: normal(gk, (n,)) with no split. */
void zgo_vector_noise(const uint32_t gk[2], int64_t n, float* out);

/* Population helpers: keys[i] = fold_in(base, ids[i]); then group keys. */
void zgo_candidate_keys(const uint32_t base[2], const int32_t* ids, int64_t n, uint32_t* out);
void zgo_group_keys(const uint32_t* cand_keys, int64_t n, int group, uint32_t* out);

/* Batched factors for P candidate keys (already group keys), f32, the
 * reference layouts with a leading population axis.  layout: 0 MATRIX,
 * 1 TABLE, 2 VECTOR (B unused).  Uses all host threads (pthreads). */
void zgo_population_factors(const uint32_t* group_keys, int64_t P, int layout,
                            int64_t rows, int64_t cols, int rank, float* A, float* B);

/* float32 -> bfloat16 -> float32 round trip (round to nearest even). */
float zgo_round_bf16(float x);

/* Exact int8 GEMM + LUT epilogue for one candidate:
 *   acc[m,n]  = sum_k x[m,k] * W[k,n]                 (int64 accumulate, exact)
 *   y         = acc * x_scale * w_scale[n] + s * sum_j u[m,j] * Bf[j,n]
 *               with u[m,j] = sum_k x[m,k] * A[k,j]    (float32 math, fixed order)
 *   q         = clamp(rint(y / y_scale), -128, 127), 0 when that is NaN
 *   out[m,n]  = lut[q + 128]
 * acc_out (optional, may be NULL) receives the int32 accumulators. */
void zgo_int8_lut_linear(const int8_t* x, const int8_t* W, const float* w_scale,
                         float x_scale, float y_scale, const int8_t* lut,
                         const float* A, const float* Bf, int rank, float s,
                         int64_t M, int64_t K, int64_t N, int8_t* out, int32_t* acc_out);

/* Threads the oracle uses (ZGO_THREADS, else all online cores). */
int zgo_num_threads(void);
void zgo_set_num_threads(int n);

#ifdef __cplusplus
}
#endif
#endif
