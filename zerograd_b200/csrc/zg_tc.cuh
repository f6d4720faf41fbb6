// zg_tc.cuh -- tensor-core (tcgen05 / TMEM / TMA) paths for sm_100a.
#pragma once
#include <cuda.h>

#include "zg_common.cuh"
#include "zg_update.cuh"

namespace zg {

// True on a compute-capability 10.0 device with the TMA descriptor encoder.
bool tc_available();

// bf16 TMA descriptor of `rank` dimensions (innermost first), byte strides of
// dimensions 1.., box extents; 128-byte swizzle or none; out-of-bounds
// elements read as zero.
bool tensor_map_bf16(CUtensorMap* m, const void* base, int rank, const uint64_t* dims, const uint64_t* strides_bytes,
                     const uint32_t* box, bool swizzle128);
// The same with the swizzle span in bytes: 0 (none), 64 or 128.
bool tensor_map_bf16_swz(CUtensorMap* m, const void* base, int rank, const uint64_t* dims,
                         const uint64_t* strides_bytes, const uint32_t* box, int swizzle_bytes);

// Kernel error words of the per-candidate-input and int8 kernels (0 = none).
int batched_error_word(int clear);
int int8_error_word(int clear);
int ce_error_word(int clear);
int attn_error_word(int clear);

// Factor fill transposed to [P r, rows]: out[p*r + j, row] =
// round_dtype(normal(key_p, row*r + j)) (the [rows, r] row-major factor of
// candidate p, stored K-major for the tensor cores); bf16, rank 8 or 16.
int fill_operand_t(const uint32_t* keys, int group, int P, int rank, int64_t rows, int which, void* out,
                   cudaStream_t st, const char* name = "factor_fill");

// Per-candidate-input population forward (bf16, rank 8 or 16):
//   y[p] = x_p @ Wop + s (x_p @ F1_p) @ F2_p^T
// x [P, M, K]; Wop [K, N] (w_mn_major) or [N, K]; F1T [P r, K]; F2 [N, P r].
// The two kernels of that forward:
//   U[p, m, 0:16] = bf16(s * x_p[m] . F1_p) (columns >= rank zero)
//   y[p] = bf16(x_p . Wop + U_p . F2_p^T)
int batched_u_pass(const void* x, const void* F1T, int P, int M, int K, int rank, float s, void* U, cudaStream_t st,
                   bool x_batched = true);
// F2's rows are ld2 elements apart (0: P*rank).  The epilogue rounds to bf16,
// then applies `act` (ZG_ACT_*) and adds the bf16 residual `res` [P, M, N]
// (or null), rounding after each step as the unfused ops do.
int batched_gemm(const void* x, const void* Wop, bool w_mn_major, const void* U, const void* F2, int P, int M, int K,
                 int N, int rank, void* y, cudaStream_t st, int64_t ld2 = 0, int act = 0, const void* res = nullptr);
bool batched_forward_ok(int P, int M, int K, int N, int rank);
size_t batched_forward_workspace(int P, int M, int K, int N, int rank, bool draw);
int batched_forward(const void* x, const void* Wop, bool w_mn_major, const uint32_t* keys, int group, int f1_which,
                    int f2_which, int f2_col_major, bool draw, const void* F1T, const void* F2, int P, int M, int K,
                    int N, int rank, float s, void* y, Carver& cv, cudaStream_t st, int64_t ld2 = 0, int act = 0,
                    const void* res = nullptr);

// D[M,N] = alpha * A[M,K] . B^T; A K-major row-major (lda), B K-major
// [N,K] (ldb) or MN-major [K,N] (ldb); D row-major float32 or bf16 (ldd).
// Rows of A and B must be 16-byte aligned (lda, ldb multiples of 8).
// With `step`, the epilogue also applies that optimizer step to the float32
// result (D may then be null).
int tc_gemm_bf16(const void* A, int64_t lda, const void* B, int64_t ldb, bool b_mn_major, void* D, int64_t ldd,
                 bool out_bf16, int M, int N, int K, float alpha, cudaStream_t st, const char* name = "gemm",
                 const FusedStep* step = nullptr);

// The same GEMM over `splits` equal K ranges of k_split elements (k_split %
// 64 == 0 when splits > 1), each accumulated on its own into the partial
// D + z * d_split (z = the range); no fused step.  The kernel and tile width
// are those of the split_total-range problem, so ranges computed in separate
// launches (or on separate GPUs) give the bits of one launch of all of them.
int tc_gemm_core(const void* A, int64_t lda, const void* B, int64_t ldb, bool b_mn_major, void* D, int64_t ldd,
                 bool out_bf16, int M, int N, int splits, int split_total, int k_split, int64_t d_split, float alpha,
                 cudaStream_t st, const char* name, const FusedStep* step);

// Fixed-order sum of S <= 8 float32 partials (partial s of element e at
// parts + offsets[s] + e): d = alpha * (((p_0 + p_1) + p_2) + ...), then the
// optimizer `step` on d (kind != NONE; param and moments at flat offsets e)
// and/or d -> out (out may be null when there is a step).
constexpr int kMaxSplits = 8;
int split_reduce(const float* parts, const int64_t* offsets, int S, int64_t n, float alpha, const FusedStep* step,
                 float* out, cudaStream_t st);

// Factor fill in GEMM-operand layout: out[row * ld + p*r + j] =
// scale_p * round_dtype(normal(key_p, ctr)), ctr = row*r + j (row-major) or
// j*rows + row (col_major); which = 0 for the A factor key, 1 for B.  ld is
// the row pitch in elements (0: P*r, a buffer of these P candidates alone;
// larger: their column block of a larger population's buffer).
int fill_operand(const uint32_t* keys, int group, int P, int rank, int64_t rows, int which, int col_major,
                 const float* scale, float extra_scale, int dtype, void* out, cudaStream_t st,
                 const char* name = "factor_fill", int64_t ld = 0);

// Rank-8 expansion on the tensor cores: U bf16 [M, P*8], Bq bf16 [N, P*8]
// with rows ldb apart, XW float32 [M, N], y bf16 [P, M, N] written with TMA
// bulk stores.
bool tc_expand_ok(int P, int M, int N, int rank, const void* XW, const void* U, const void* Bq, const void* y);
// y[p, m, n] = bf16(XW[m, n] + s (U_p B_p^T)[m, n]) for rank 8 or 16: U
// [M, P r] bf16, Bq [N, P r] (row pitch ldb), XW [M, N] float32, y [P, M, N].
int tc_expand(const float* XW, const void* U, const void* Bq, int64_t ldb, int P, int M, int N, int rank, float s,
              void* y, cudaStream_t st, const char* name);
int tc_expand_r8(const float* XW, const void* U, const void* Bq, int64_t ldb, int P, int M, int N, float s, void* y,
                 cudaStream_t st);

// y[p, m, n] = XW[m, n] + s * sum_j U[m, p*r + j] * Bq[n, p*r + j].
int lowrank_expand(const float* XW, const float* U, const void* Bq, int P, int M, int N, int rank, float s,
                   int dtype, void* y, cudaStream_t st);

// Shared-input population forward on the tensor cores (bf16).
bool tc_shared_forward_ok(int P, int M, int K, int N, int rank);
size_t tc_shared_forward_workspace(int P, int M, int K, int N, int rank);
int tc_shared_forward(const void* x, const void* Wop, bool w_mn_major, int64_t ldw, const uint32_t* keys, int group,
                      int P, int M, int K, int N, int rank, int f1_which, int f1_col_major, int f2_which,
                      int f2_col_major, float s, void* y, Carver& cv, cudaStream_t st);

// Replay of one MATRIX/TABLE entry as a GEMM over the P*r axis (bf16), split
// into replay_split_count(P, rank) candidate groups summed in group order.
bool tc_replay_ok(int P, int64_t rows, int64_t cols, int rank, int dtype);
int replay_split_count(int P, int rank);
size_t tc_replay_operands_workspace(int P, int64_t rows, int64_t cols, int rank);
size_t tc_replay_workspace(int P, int64_t rows, int64_t cols, int rank);
// Partials of `splits` of `split_total` candidate groups from the factors of
// those groups' P candidates: parts + z * part_stride = unscaled G_z [rows, cols].
int tc_replay_partials(const float* shaped, const void* A, bool a_t, const void* B, bool b_t, int P, int64_t rows,
                       int64_t cols, int rank, int split_total, int splits, float* parts, int64_t part_stride,
                       Carver& cv, cudaStream_t st);
int tc_replay_factors(const float* shaped, const void* A_op, const void* B_op, int P, int64_t rows, int64_t cols,
                      int rank, float inv_sqrt_rank, float* out, Carver& cv, cudaStream_t st,
                      const FusedStep* step = nullptr);
int tc_replay_operands(const float* shaped, const void* A, bool a_t, const void* B, bool b_t, int P, int64_t rows,
                       int64_t cols, int rank, float inv_sqrt_rank, float* out, Carver& cv, cudaStream_t st,
                       const FusedStep* step = nullptr);
int tc_replay_run(const float* shaped, const uint32_t* keys, int group, int P, int layout, int64_t rows, int64_t cols,
                  int rank, float inv_sqrt_rank, float* out, Carver& cv, cudaStream_t st);

}  // namespace zg
