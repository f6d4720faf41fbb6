/*
 * zg_b200.h -- C ABI of libzgb200, the sm_100a kernels behind zerograd's
 * population-evaluation and factor-replay path.
 *
 * Conventions
 *   - Every pointer is a DEVICE pointer unless the comment says "host".
 *   - The caller owns every buffer.  Entry points that need scratch take a
 *     (workspace, workspace_bytes) pair; the matching *_workspace_size()
 *     query returns the bytes required.  No entry point allocates.
 *   - `stream` is a cudaStream_t passed as void*; all work is enqueued on it.
 *   - Return value: ZG_OK (0) or an error code; zg_last_error() returns a
 *     message for the calling host thread.
 *   - Keys are uint32 pairs (jax.random key data) laid out [n, 2].
 *     `group` >= 0: the keys are CANDIDATE keys and the kernel derives the
 *     group key fold(candidate_key, group) itself (split(ck, n)[group] of
 *     the partitionable threefry); `group` == -1: the keys are group keys.
 *   - dtype codes: ZG_F32 or ZG_BF16 for the weights / activations.
 *
 * Each entry point names the reference interface it replaces (paths are
 * relative to the reference project root).
 */
#ifndef ZG_B200_H
#define ZG_B200_H
#include <stddef.h>
#include <stdint.h>

#if defined(__GNUC__)
#define ZG_API __attribute__((visibility("default")))
#else
#define ZG_API
#endif

#ifdef __cplusplus
extern "C" {
#endif

enum {
    ZG_OK = 0,
    ZG_ERR_INVALID = 1,   /* bad argument (shape, dtype, null pointer) */
    ZG_ERR_CUDA = 2,      /* a CUDA runtime call or launch failed */
    ZG_ERR_WORKSPACE = 3, /* workspace missing or too small */
    ZG_ERR_UNSUPPORTED = 4
};
enum { ZG_F32 = 0, ZG_BF16 = 1 };
enum { ZG_MATRIX = 0, ZG_TABLE = 1, ZG_VECTOR = 2 };
/* Element-wise activation applied in a forward GEMM's epilogue. */
enum { ZG_ACT_NONE = 0, ZG_ACT_GELU = 1 };

/* Message of the last failing call on this host thread ("" if none). */
ZG_API const char* zg_last_error(void);
/* Library version string. */
ZG_API const char* zg_version(void);

/* Launch accounting.  zg_launch_count() is the number of kernels this
 * library has launched since load (all threads).  Between
 * zg_profile_begin() and zg_profile_end() every launch is bracketed by CUDA
 * events on its own stream (up to `max_records` launches);
 * zg_profile_summary() (call after the stream work completed) writes one
 * line per kernel name, "name,launches,total_ms", into `buf`.
 * No counterpart in the reference (it has no kernels of its own). */
ZG_API int64_t zg_launch_count(void);
ZG_API int zg_profile_begin(int max_records);
ZG_API int zg_profile_end(void);
ZG_API int zg_profile_summary(char* buf, size_t len);

/* Error code recorded by a tensor-core kernel whose bounded wait expired
 * (0 = none).  Synchronises the current device; `clear` resets it. */
ZG_API int zg_device_error(int clear);

/* Dense bf16 GEMM on the tcgen05 tensor cores, float32 accumulation:
 *   D[M,N] = alpha * A[M,K] . B^T, A row-major [M,K] (lda);
 *   B row-major [N,K] (b_mn_major = 0) or [K,N] (b_mn_major = 1) (ldb);
 *   D row-major (ldd) in float32 (out_dtype ZG_F32) or bf16 (ZG_BF16).
 * lda, ldb multiples of 8; A, B 16-byte aligned.  The contraction the
 * reference expresses with jnp.einsum / @ (src/zerograd/_replay.py:47,51;
 * src/zerograd/_candidate.py:22). */
ZG_API int zg_gemm_bf16(const void* A, int64_t lda, const void* B, int64_t ldb, int b_mn_major, void* D,
                        int64_t ldd, int out_dtype, int M, int N, int K, float alpha, void* stream);

/* ---------------------------------------------------------------- keys -- */

/* Raw threefry2x32-20 blocks: out[i] = threefry(keys[i], ctrs[i]).
 * Replaces jax.random's threefry2x32 primitive (reached from
 * src/zerograd/_keys.py:30,40,53,58). */
ZG_API int zg_threefry2x32(const uint32_t* keys, const uint32_t* ctrs, uint32_t* out, int64_t n,
                    void* stream);

/* out[i] = fold_in(keys[key_stride ? i : 0], data[i]).
 * Replaces candidate_key (src/zerograd/_keys.py:33-53) batched over a
 * candidate-id array, the per-candidate rng fold_in
 * (src/zerograd/_optimizer.py:175) and group_key
 * (src/zerograd/_keys.py:56-58, with data = the group index). */
ZG_API int zg_fold_in(const uint32_t* keys, int key_stride, const uint32_t* data, uint32_t* out,
               int64_t n, void* stream);

/* out[i] = fold_in((k0, k1), data[i]) with the key passed by value (a key
 * computed on the host, like step_key's, needs no host-to-device copy).
 * Replaces candidate_key (src/zerograd/_keys.py:33-53) and the
 * per-candidate rng fold_in (src/zerograd/_optimizer.py:174-175) batched
 * over a candidate-id array. */
ZG_API int zg_candidate_keys(uint32_t k0, uint32_t k1, const uint32_t* data, uint32_t* out, int64_t n,
                             void* stream);

/* Random bits / float32 normals of `n` flat elements for each of `nkeys`
 * keys: out[k, j].  Replaces jax.random.bits / jax.random.normal(float32)
 * as called by src/zerograd/_factors.py:47,53-54,62,65-66,74. */
ZG_API int zg_random_bits(const uint32_t* keys, int64_t nkeys, int64_t n, uint32_t* out, void* stream);
ZG_API int zg_normal(const uint32_t* keys, int64_t nkeys, int64_t n, int dtype, void* out, void* stream);

/* Population factors for one manifest entry, in the reference layouts with
 * a leading population axis: MATRIX A[P,rows,rank], B[P,rank,cols];
 * TABLE A[P,rows,rank], B[P,cols,rank]; VECTOR A[P,rows] (B unused).
 * Values are the float32 draws cast to `dtype`.
 * Replaces matrix_factors / table_factors / vector_noise
 * (src/zerograd/_factors.py:43-74) under jax.vmap over candidates
 * (src/zerograd/_replay.py:45,49,53). */
ZG_API int zg_population_factors(const uint32_t* keys, int group, int P, int layout, int64_t rows,
                          int64_t cols, int rank, int dtype, void* A, void* B, void* stream);

/* Population factors of one MATRIX/TABLE entry in GEMM-operand layout,
 * q = P * rank columns, column p*rank + j = candidate p, rank index j:
 *   A_op[rows, q] = A_p[row, j]                       (counter row*rank + j)
 *   B_op[cols, q] = MATRIX B_p[j, col] (counter j*cols + col) /
 *                   TABLE  B_p[col, j] (counter col*rank + j)
 * Either output may be NULL.  The same two buffers feed the forward pass
 * (zg_forward_factors) and the replay (zg_replay_factors) of one
 * generation, so each factor element is drawn once.  Replaces the
 * matrix_factors / table_factors draws under jax.vmap
 * (src/zerograd/_factors.py:43-67, src/zerograd/_replay.py:45,49). */
ZG_API int zg_factor_operands(const uint32_t* keys, int group, int P, int layout, int64_t rows,
                              int64_t cols, int rank, int dtype, void* A_op, void* B_op,
                              void* stream);

/* The same factors in the per-candidate-input forward's layout (bf16, rank
 * 8 or 16): MATRIX [rows = K, cols = N]: F1T = A^T [P*rank, rows] (row
 * p*rank + j = A_p[:, j]) and F2 = B_op [cols, P*rank]; tied TABLE
 * [rows = V, cols = C]: F1T = B^T [P*rank, cols] and F2 = A_op [rows,
 * P*rank].  F2's rows are ld2 elements apart (0: P*rank).  What
 * zg_batched_forward_ex and zg_tied_logits_ce_ex draw, for drawing a
 * generation's factors ahead of its forward (the matrix_factors /
 * table_factors draws under jax.vmap, src/zerograd/_factors.py:43-67). */
ZG_API int zg_factor_operands_t(const uint32_t* keys, int group, int P, int layout, int64_t rows,
                                int64_t cols, int rank, void* F1T, void* F2, int64_t ld2,
                                void* stream);

/* Shared-input population forward from operand factors (bf16, tcgen05):
 *   y[p] = x @ Wop + s * (x @ F1_p) @ F2_p^T, x [M,K], F1 [K, P*rank],
 *   F2 [N, P*rank], y [P, M, N].
 * w_is_kn = 1: W is a linear weight [K, N] (F1 = A_op, F2 = B_op of its
 * MATRIX entry); w_is_kn = 0: W is a tied table [N, K] (F1 = B_op,
 * F2 = A_op of its TABLE entry).  Requires P*rank, K, N multiples of 8 and
 * rank <= 32.  Replaces perturbed_linear / perturbed_tied_logits under
 * jax.vmap (src/zerograd/_candidate.py:17-22,33-38). */
ZG_API size_t zg_forward_factors_workspace_size(int P, int M, int N, int rank);
ZG_API int zg_forward_factors(const void* x, const void* W, int w_is_kn, const void* F1,
                              const void* F2, int P, int M, int K, int N, int rank, float s,
                              void* y, void* workspace, size_t workspace_bytes, void* stream);

/* zg_forward_factors with F1's and F2's rows ld1 and ld2 elements apart
 * (multiples of 8, at least P*rank): F1 and F2 may be a column block of a
 * larger population's operand factors, such as one process's candidates
 * inside the whole population's factors drawn for the replay, so a
 * population shard's forward reads them instead of drawing its own
 * (src/zerograd/_distributed.py:88-139 evaluates a shard; its factors are
 * those of _factors.py:30-74 for the shard's candidate ids).  A leading
 * dimension above P*rank needs the rank-8 tensor-core expansion (rank 8,
 * N a multiple of 8, 16-byte aligned F2); otherwise ZG_ERR_UNSUPPORTED.
 * Workspace: zg_forward_factors_workspace_size. */
ZG_API int zg_forward_factors_ld(const void* x, const void* W, int w_is_kn, const void* F1, int64_t ld1,
                                 const void* F2, int64_t ld2, int P, int M, int K, int N, int rank, float s,
                                 void* y, void* workspace, size_t workspace_bytes, void* stream);

/* The same forward that also draws its operand factors into F1 / F2
 * (bf16 [K, P*rank] / [N, P*rank], kept by the caller for the replay of the
 * generation): linear (w_is_kn = 1) F1 = A_op, F2 = B_op of the MATRIX
 * entry; tied table (w_is_kn = 0) F1 = B_op, F2 = A_op of the TABLE entry.
 * Internally the factor draws overlap the x @ W GEMM on a second stream
 * joined back before return.  Workspace: zg_forward_factors_workspace_size.
 * Replaces the factor draws plus perturbed_linear / perturbed_tied_logits
 * under jax.vmap (src/zerograd/_candidate.py:17-38, _factors.py:43-67). */
ZG_API int zg_forward_operands(const void* x, const void* W, int w_is_kn, const uint32_t* keys,
                               int group, int P, int M, int K, int N, int rank, float s, void* F1,
                               void* F2, void* y, void* workspace, size_t workspace_bytes,
                               void* stream);

/* Replay from operand factors (bf16, tcgen05):
 *   out[rows, cols] = inv_sqrt_rank * sum_q (w_{q/rank} A_op[:, q]) B_op[:, q]^T
 * (float32).  The sum over the P candidates runs as S =
 * zg_replay_split_count(P, rank) groups of P / S consecutive candidates,
 * each contracted on its own (float32 partial G_z), then added in group
 * order: out = inv_sqrt_rank * (((G_0 + G_1) + G_2) + ...).  The fitness
 * weight is applied to one operand, rounded to bf16 (the input-side factor
 * when it is given transposed, else the smaller of the two).  Replaces
 * replay_entry (src/zerograd/_replay.py:44-51). */
ZG_API size_t zg_replay_factors_workspace_size(int P, int64_t rows, int64_t cols, int rank);
ZG_API int zg_replay_factors(const float* shaped, const void* A_op, const void* B_op, int P,
                             int64_t rows, int64_t cols, int rank, float inv_sqrt_rank, float* out,
                             void* workspace, size_t workspace_bytes, void* stream);

/* The same replay with either operand given transposed: a_transposed = 1
 * takes A as AT [P*rank, rows], b_transposed = 1 takes B as BT [P*rank, cols]
 * (cols a multiple of 8), which is how the per-candidate-input forward keeps
 * its input-side factor.  Replaces replay_entry
 * (src/zerograd/_replay.py:44-51). */
ZG_API size_t zg_replay_operands_workspace_size(int P, int64_t rows, int64_t cols, int rank);
ZG_API int zg_replay_operands(const float* shaped, const void* A, int a_transposed, const void* B,
                              int b_transposed, int P, int64_t rows, int64_t cols, int rank,
                              float inv_sqrt_rank, float* out, void* workspace,
                              size_t workspace_bytes, void* stream);

/* Replay with the optimizer step fused into the replay GEMM's epilogue
 * (bf16 operands as for zg_replay_operands): the descent d of every element
 * of the entry's parameter [rows, cols] is formed in float32 and consumed in
 * place by the step, so it never round-trips through memory:
 *   SGD:   param_out = param + (-lr) * (-d)                (optax.sgd)
 *   AdamW: mu_out, nu_out, param_out as zg_adamw_update   (optax.adamw)
 * on the pseudo-gradient -d, bit-identical to zg_replay_operands followed by
 * zg_sgd_update / zg_adamw_update.  param in `dtype` (float32 or bf16),
 * moments float32, all [rows, cols] row-major; descent_out (optional) also
 * receives d.  The outputs may alias the inputs (param_out == param, and
 * the moments likewise): each element is read and written by one thread.
 * guard (optional, device float): when *guard != 0 nothing is written, so an
 * in-place update of a generation whose losses were rejected leaves the
 * parameters as they were (zg_shape_fitness's non-finite count, metrics[3]);
 * a guarded call takes no descent_out.  bias_corrections (optional, device
 * float[2]): AdamW's [1 - b1^count, 1 - b2^count] read at run time instead
 * of derived from count (zg_adam_bias_corrections gives the same floats),
 * so a captured generation can advance the step count.
 * Workspace: zg_replay_operands_workspace_size.  Replaces
 * replay_entry + transform.update + apply_updates
 * (src/zerograd/_replay.py:44-54, src/zerograd/_optimizer.py:229-234). */
ZG_API int zg_replay_sgd(const float* shaped, const void* A, int a_transposed, const void* B,
                         int b_transposed, int P, int64_t rows, int64_t cols, int rank,
                         float inv_sqrt_rank, const void* param, void* param_out, int dtype,
                         double lr, float* descent_out, const float* guard, void* workspace,
                         size_t workspace_bytes, void* stream);
ZG_API int zg_replay_adamw(const float* shaped, const void* A, int a_transposed, const void* B,
                           int b_transposed, int P, int64_t rows, int64_t cols, int rank,
                           float inv_sqrt_rank, const void* param, void* param_out, int dtype,
                           const float* mu, const float* nu, float* mu_out, float* nu_out, int count,
                           double lr, double b1, double b2, double eps, double weight_decay,
                           float* descent_out, const float* guard, const float* bias_corrections,
                           void* workspace, size_t workspace_bytes, void* stream);

/* The replay split over candidate groups, for a population spread over
 * several GPUs (src/zerograd/_distributed.py:319-366 replays the whole
 * population on every device; here each GPU contracts only the groups whose
 * factors its forward drew, and the partials are exchanged and summed).
 * zg_replay_split_count: S for a population of P candidates at this rank
 * (the largest of 8, 4, 2 whose groups keep >= 4096 contraction columns, a
 * multiple of 64; else 1).
 * zg_replay_partials: `splits` consecutive groups (of the S = split_total
 * groups of the population) from the factors of their P candidates, laid
 * out as for zg_replay_operands, and the candidates' shaped weights:
 * partials + z * partial_stride = G_z [rows, cols] float32 (unscaled), the
 * same bits as the partial zg_replay_operands forms for that group.
 * zg_replay_split_sum: out[e] = alpha * (((p_0 + p_1) + p_2) + ...) over S
 * <= 8 partials, partial s of element e at partials[offsets[s] + e]
 * (offsets: host array of S element offsets).
 * zg_replay_split_sgd: the same sum d, then param_out = param + (-lr)(-d)
 * (optax.sgd), nothing written when *guard != 0.  With the partials of all
 * groups these give exactly the bits of zg_replay_operands / zg_replay_sgd. */
ZG_API int zg_replay_split_count(int P, int rank);
ZG_API size_t zg_replay_partials_workspace_size(int P, int64_t rows, int64_t cols, int rank);
ZG_API int zg_replay_partials(const float* shaped, const void* A, int a_transposed, const void* B,
                              int b_transposed, int P, int64_t rows, int64_t cols, int rank,
                              int split_total, int splits, float* partials, int64_t partial_stride,
                              void* workspace, size_t workspace_bytes, void* stream);
ZG_API int zg_replay_split_sum(const float* partials, const int64_t* offsets, int S, int64_t n,
                               float alpha, float* out, void* stream);
ZG_API int zg_replay_split_sgd(const float* partials, const int64_t* offsets, int S, int64_t n,
                               float alpha, const void* param, void* param_out, int dtype, double lr,
                               const float* guard, void* stream);

/* Tied logits fused with softmax cross-entropy (bf16, tcgen05): for each
 * candidate p and row m
 *   logits = bf16(x_p @ T^T + s * (x_p @ B_p) @ A_p^T)    (perturbed_tied_logits)
 *   loss[p, m] = logsumexp_v logits[m, v] - logits[m, labels[m]]   (float32)
 * without materialising the [P, M, V] logits: a pair of SMs sweeps the whole
 * vocabulary for a 256-row block, keeping each row's running max and sum of
 * exponentials in registers.  T [V, C] (the tied table), x [M, C] shared
 * (x_batched = 0) or [P, M, C]; labels [M] int32 (shared by the candidates);
 * loss [P, M].  A label outside [0, V) gives a NaN loss.  rank 8 or 16; C a
 * multiple of 8; x and T 16-byte aligned.  Replaces perturbed_tied_logits
 * (src/zerograd/_candidate.py:33-38) followed by a cross-entropy over the
 * logits in the loss function. */
ZG_API size_t zg_tied_logits_ce_workspace_size(int P, int M, int V, int C, int rank);
ZG_API int zg_tied_logits_ce(const void* x, int x_batched, const void* T, const uint32_t* keys,
                             int group, const int32_t* labels, int P, int M, int V, int C,
                             int rank, float s, float* loss, void* workspace,
                             size_t workspace_bytes, void* stream);
/* The same with the table factors in caller buffers, F1T = B^T [P*rank, C]
 * and F2 = A_op [V, P*rank] with rows ld2 apart (0: P*rank; larger: these
 * candidates' column block of a population's buffer), drawn first when
 * draw != 0 (keys may be NULL otherwise).  The workspace then holds only the
 * low-rank activations (zg_tied_logits_ce_ex_workspace_size). */
ZG_API size_t zg_tied_logits_ce_ex_workspace_size(int P, int M, int V, int C, int rank);
ZG_API int zg_tied_logits_ce_ex(const void* x, int x_batched, const void* T, const uint32_t* keys,
                                int group, const int32_t* labels, int P, int M, int V, int C,
                                int rank, float s, void* F1T, void* F2, int64_t ld2, int draw,
                                float* loss, void* workspace, size_t workspace_bytes,
                                void* stream);

/* Per-candidate-input population forward (bf16, tcgen05), the hidden-layer
 * case: x [P, M, K] (one input per candidate), y [P, M, N],
 *   y[p] = x_p @ Wop + s * (x_p @ F1_p) @ F2_p^T
 * with F1T [P*rank, K] (each candidate's input-side factor, K-major) and
 * F2 [N, P*rank].  w_is_kn = 1: W is a linear weight [K, N]; F1T rows are
 * A_p^T (A counter k*rank + j), F2 = B_op (counter j*N + n).  w_is_kn = 0:
 * W is a tied table [N, K]; F1T rows are the table B_p^T (counter
 * c*rank + j), F2 = the table A_op (counter v*rank + j).  rank 8 or 16; K, N
 * multiples of 8; all pointers 16-byte aligned.  _operands draws F1T and F2
 * (kept by the caller for the replay, which takes F1T through
 * zg_replay_operands); _factors takes them as given.  Replaces
 * perturbed_linear / perturbed_tied_logits under jax.vmap with a batched x
 * (src/zerograd/_candidate.py:17-22,33-38). */
ZG_API size_t zg_batched_forward_workspace_size(int P, int M, int K, int N, int rank);
ZG_API int zg_batched_forward_factors(const void* x, const void* W, int w_is_kn, const void* F1T,
                                      const void* F2, int P, int M, int K, int N, int rank, float s,
                                      void* y, void* workspace, size_t workspace_bytes,
                                      void* stream);
ZG_API int zg_batched_forward_operands(const void* x, const void* W, int w_is_kn,
                                       const uint32_t* keys, int group, int P, int M, int K, int N,
                                       int rank, float s, void* F1T, void* F2, void* y,
                                       void* workspace, size_t workspace_bytes, void* stream);

/* The per-candidate-input forward with the options a chunked population
 * evaluation and a transformer block need (same workspace size query):
 *   - F2's rows are ld2 elements apart (0: P*rank).  With ld2 > P*rank, F1T
 *     and F2 are these P candidates' block of a larger population's
 *     factors (F1T + c0*rank*K rows, F2 + c0*rank columns), so the
 *     population's factors are drawn once per generation, chunk by chunk,
 *     and the replay reads the whole buffers;
 *   - draw != 0: F1T and F2 are drawn from `keys` first (as
 *     zg_batched_forward_operands), else read as given;
 *   - epilogue: y = bf16(acc); activation ZG_ACT_GELU then gives
 *     y = bf16(gelu(y)) (tanh form, 0.5 y (1 + tanh(sqrt(2/pi)(y + 0.044715 y^3))));
 *     a non-null `residual` [P, M, N] then gives y = bf16(residual + y) --
 *     the roundings of the unfused linear, activation and residual add.
 * A candidate's output does not depend on its position among the P.
 * Replaces perturbed_linear (src/zerograd/_candidate.py:17-22) under
 * jax.vmap followed by the user's element-wise activation and residual add
 * (the transformer block of examples/train_vit_cifar10.py:137-191). */
ZG_API int zg_batched_forward_ex(const void* x, const void* W, int w_is_kn, const uint32_t* keys,
                                 int group, int P, int M, int K, int N, int rank, float s, void* F1T,
                                 void* F2, int64_t ld2, int draw, int activation,
                                 const void* residual, void* y, void* workspace,
                                 size_t workspace_bytes, void* stream);

/* ------------------------------------------------------- forward ops -- */

/* y[p] = x_p @ W + s * (x_p @ A_p) @ B_p for p in [0,P): one population-
 * batched launch sequence.  x is [M,K] shared by all candidates
 * (x_batched = 0) or [P,M,K] (x_batched = 1); W [K,N]; y [P,M,N]; all in
 * `dtype`.  s = scaled_factor (sigma/sqrt(rank) rounded to dtype by the
 * caller).  Replaces perturbed_linear / CandidateContext.linear
 * (src/zerograd/_candidate.py:17-22,61-66) under jax.vmap. */
ZG_API size_t zg_perturbed_linear_workspace_size(int P, int M, int K, int N, int rank, int dtype,
                                          int x_batched);
ZG_API int zg_perturbed_linear(const void* x, int x_batched, const void* W, const uint32_t* keys,
                        int group, int P, int M, int K, int N, int rank, float s, int dtype,
                        void* y, void* workspace, size_t workspace_bytes, void* stream);

/* out[p, t, :] = T[idx[t]] + s * A_p[idx[t]] @ B_p^T, T [rows, cols],
 * idx [n_idx] (int32, shared by all candidates) or [P, n_idx]
 * (idx_batched = 1).  A rows are drawn only at the gathered rows.  bf16
 * with shared ids, rank 8 or 16 and cols a multiple of 8 runs on the
 * tensor cores (the gathered rows and A rows staged in the workspace, one
 * K = 16 MMA per candidate and 128 x 128 tile); otherwise CUDA cores.
 * Replaces perturbed_table_lookup / CandidateContext.table_lookup
 * (src/zerograd/_candidate.py:25-30,68-73). */
ZG_API size_t zg_table_lookup_workspace_size(int P, int64_t n_idx, int64_t rows, int64_t cols, int rank,
                                             int dtype);
ZG_API int zg_table_lookup(const void* T, const int32_t* idx, int idx_batched, int64_t n_idx,
                    const uint32_t* keys, int group, int P, int64_t rows, int64_t cols,
                    int rank, float s, int dtype, void* out, void* workspace,
                    size_t workspace_bytes, void* stream);

/* y[p] = x_p @ T^T + s * (x_p @ B_p) @ A_p^T with T [V, C] (table layout
 * factors A [V,rank], B [C,rank]); x [M,C] or [P,M,C]; y [P,M,V].
 * Replaces perturbed_tied_logits / CandidateContext.tied_logits
 * (src/zerograd/_candidate.py:33-38,75-80). */
ZG_API size_t zg_tied_logits_workspace_size(int P, int M, int V, int C, int rank, int dtype,
                                     int x_batched);
ZG_API int zg_tied_logits(const void* x, int x_batched, const void* T, const uint32_t* keys, int group,
                   int P, int M, int V, int C, int rank, float s, int dtype, void* y,
                   void* workspace, size_t workspace_bytes, void* stream);

/* out[p, i] = v[i] + s * normal(group_key_p)[i]; v [n] or [P, n]
 * (v_batched = 1).  Replaces perturbed_vector / CandidateContext.vector
 * (src/zerograd/_candidate.py:41-45,82-87). */
ZG_API int zg_perturbed_vector(const void* v, int v_batched, const uint32_t* keys, int group, int P,
                        int64_t n, float s, int dtype, void* out, void* stream);

/* --------------------------------------------- fitness / replay / update -- */

/* out[r] = mean(x[r, 0:n]) for r in [0, rows) (float32 in, float64
 * accumulation in a fixed order, float32 out): a candidate's mean loss over
 * its rows, independent of how many candidates one launch holds.  Replaces
 * the loss function's jnp.mean over the per-row cross-entropies
 * (examples/train_cifar10.py:77-78) under jax.vmap. */
ZG_API int zg_row_mean(const float* x, int64_t rows, int64_t n, float* out, void* stream);

/* Validates and shapes the gathered losses [P] (float32):
 *   shaped[p] = -(l[p] - mean(l)) / (P * sigma)
 * metrics (float32[4], device) = {mean, min, max, number of non-finite}.
 * sigma is the Python float the reference divides by (P * sigma is formed
 * in double precision and rounded to float32 once).
 * Replaces shape_centered_loss + validate_losses
 * (src/zerograd/_fitness.py:13-48) and the StepMetrics reductions
 * (src/zerograd/_optimizer.py:237-243). */
ZG_API int zg_shape_fitness(const float* losses, int P, double sigma, float* shaped, float* metrics,
                     void* stream);

/* Pseudo-gradient DESCENT direction of one manifest entry:
 *   MATRIX out[rows,cols] = inv_sqrt_rank * sum_p w_p A_p @ B_p
 *   TABLE  out[rows,cols] = inv_sqrt_rank * sum_p w_p A_p @ B_p^T
 *   VECTOR out[rows]      = sum_p w_p n_p
 * keys [P,2] candidate keys (group >= 0) in candidate-id order, w = the
 * shaped fitness [P] (float32), out float32.  `inv_sqrt_rank` is
 * scaled_factor(rank, 1.0, dtype) computed by the caller.  Factors are drawn
 * in `dtype` exactly as in the forward pass.
 * Replaces replay_entry (src/zerograd/_replay.py:15-54). */
ZG_API size_t zg_replay_workspace_size(int P, int layout, int64_t rows, int64_t cols, int rank,
                                int dtype);
ZG_API int zg_replay(const float* shaped, const uint32_t* keys, int group, int P, int layout,
              int64_t rows, int64_t cols, int rank, float inv_sqrt_rank, int dtype, float* out,
              void* workspace, size_t workspace_bytes, void* stream);

/* zg_replay for callers that cannot allocate device memory where they run
 * the replay (a host that fixes the GPU library's memory at start-up and
 * forbids later cudaMalloc, or a thread that must not call an allocator).
 * Same arguments and result as zg_replay minus the workspace: the scratch
 * is a 16 MiB buffer compiled into this library, which every GPU that loads
 * the library holds until the process exits.  A replay whose
 * zg_replay_workspace_size() exceeds 16 MiB is rejected with
 * ZG_ERR_WORKSPACE.  The first call on a device looks up the buffer's
 * device address (cudaGetSymbolAddress) with that device current; make that
 * first call before any stream capture.  Under lazy module loading (the
 * CUDA default, CUDA_MODULE_LOADING=LAZY) that first call is also when the
 * 16 MiB are taken on the device, so a host that fixes its memory at
 * start-up should make it there.  The looked-up address is kept for the
 * process: cudaDeviceReset (or unloading the library's modules) is not
 * supported between calls.  All calls on a device share the one
 * buffer, so calls that overlap on the GPU (different streams, or host
 * threads racing on one device) corrupt each other's results; serialise
 * them.  The buffer keeps the last call's contents; the replay writes every
 * byte it reads, so nothing needs clearing.  This entry point has no
 * counterpart in the reference. */
ZG_API int zg_replay_noalloc(const float* shaped, const uint32_t* keys, int group, int P, int layout,
                             int64_t rows, int64_t cols, int rank, float inv_sqrt_rank, int dtype,
                             float* out, void* stream);

/* Fused AdamW (optax.adamw: scale_by_adam -> add_decayed_weights ->
 * scale(-lr)) on one leaf, with gradient = -descent (descent may be NULL:
 * a non-manifest leaf, zero gradient, which still receives weight decay).
 * Reads param / mu / nu and writes param_out / mu_out / nu_out (which may
 * alias the inputs).  param is in `dtype`; the moments are float32.
 * `count` is the step count AFTER increment (1 on the first step).  The
 * hyper-parameters are the Python floats given to the transform.
 * bias_corrections (optional, device float[2]) replaces the count's
 * [1 - b1^count, 1 - b2^count] as in zg_replay_adamw.
 * Replaces transform.update + optax.apply_updates
 * (src/zerograd/_optimizer.py:233-234) and _build_pseudo_grad
 * (src/zerograd/_optimizer.py:299-326). */
ZG_API int zg_adamw_update(const void* param, void* param_out, int dtype, const float* descent,
                           const float* mu, const float* nu, float* mu_out, float* nu_out,
                           int64_t n, int count, double lr, double b1, double b2, double eps,
                           double weight_decay, const float* bias_corrections, void* stream);

/* AdamW's bias corrections [1 - b1^count, 1 - b2^count] as the update
 * kernels compute them (float32, on the host), into out[2]. */
ZG_API int zg_adam_bias_corrections(int count, double b1, double b2, float* out);

/* Fused SGD (optax.sgd without momentum): param_out = param + (-lr) * g with
 * g = -descent (zero when descent is NULL). */
ZG_API int zg_sgd_update(const void* param, void* param_out, int dtype, const float* descent,
                         int64_t n, double lr, void* stream);

/* Copy `bytes` from src to dst when *flag == 0 (a float count), else leave
 * dst as it is.  A captured generation writes its update back with this,
 * the flag being the non-finite count that zg_shape_fitness wrote to
 * metrics[3]: losses that are not all finite change no parameter
 * (_fitness.py:37-48 rejects them before any state changes). */
ZG_API int zg_copy_if_zero(void* dst, const void* src, size_t bytes, const float* flag, void* stream);

/* --------------------------------------------- transformer-block ops -- */

/* Population-batched LayerNorm with per-candidate scale and bias (the
 * vectors CandidateContext.vector returns for each candidate):
 *   y[p, m] = (x[m] - mean) / sqrt(var + eps) * scale + bias
 * mean and biased variance in float32 over the last axis (C), y rounded to
 * dtype (ZG_F32 or ZG_BF16).  x [P, M, C] when x_batched, else [M, C] shared
 * by the candidates; scale, bias [P, C] when p_batched, else [C]; bias may be
 * NULL; y [P, M, C].  Replaces layer_norm of the reference's ViT example
 * (examples/train_vit_cifar10.py:76-79) under jax.vmap. */
ZG_API int zg_layer_norm(const void* x, int x_batched, const void* scale, const void* bias, int p_batched,
                         int P, int64_t M, int C, float eps, int dtype, void* y, void* stream);

/* Population-batched RMSNorm (the decoder LM's norm, scale a VECTOR entry):
 *   y[p, m] = x[m] / sqrt(mean(x[m]^2) + eps) * scale
 * layouts and precision as zg_layer_norm. */
ZG_API int zg_rms_norm(const void* x, int x_batched, const void* scale, int p_batched, int P, int64_t M,
                       int C, float eps, int dtype, void* y, void* stream);

/* Softmax attention of every candidate's block, population-batched:
 *   o[z, i, h] = sum_j softmax_j(q[z, i, h] . k[z, j, h] / sqrt(D)) v[z, j, h]
 * q, k, v, o [Z, S, H, D] contiguous (Z = candidates x batch rows; the
 * q/k/v projections' head-interleaved layout); causal != 0 masks keys j > i.
 * bf16 with D = 64 and S <= 256 runs on the tensor cores (scores and P V
 * accumulated in float32, P rounded to bf16, normalised by the float32 sum
 * of P; a persistent kernel holding one CTA per SM); other shapes and
 * float32 run a warp-per-row kernel in float32.
 * D <= 256.  Replaces softmax(einsum(q, k) / sqrt(D)) @ v of the reference's
 * ViT block (examples/train_vit_cifar10.py:166-172) under jax.vmap. */
ZG_API int zg_attention(const void* q, const void* k, const void* v, int Z, int S, int H, int D, int causal,
                        int dtype, void* o, void* stream);
/* The same with q, k and v rows (sequence positions) `ld` elements apart
 * (>= H*D; consecutive z blocks S*ld apart), e.g. three views into one
 * fused [Z, S, 3, H, D] q/k/v projection; o stays [Z, S, H, D] contiguous. */
ZG_API int zg_attention_ex(const void* q, const void* k, const void* v, int64_t ld, int Z, int S, int H,
                           int D, int causal, int dtype, void* o, void* stream);

/* Element-wise GELU (tanh form, as the ZG_ACT_GELU epilogue):
 *   y[i] = round_dtype(gelu(x[i])), x, y [n] of `dtype`.
 * Replaces the activation of the reference examples' MLP blocks
 * (examples/train_vit_cifar10.py:183) applied to a candidate's output. */
ZG_API int zg_gelu(const void* x, void* y, int64_t n, int dtype, void* stream);

/* ------------------------------------------------- integer QAT linear -- */

/* Integer linear with LUT activation for P candidates (no reference
 * counterpart: the reference only has float fake quantisation,
 * examples/train_qat_xor.py:41-50):
 *   acc = x_p @ W (int8 x int8 -> int32, exact)
 *   y   = acc * x_scale * w_scale[n] + s * ((x_p @ A_p) @ B_p)[m,n]   (float32)
 *   q   = clamp(rint(y / y_scale), -128, 127), 0 for NaN;  out = lut[q + 128]   (int8)
 * x [M,K] shared or [P,M,K]; W [K,N] int8; w_scale [N] float32; lut [256]
 * int8; out [P,M,N] int8.  A_p/B_p are matrix factors (float32 draws) of
 * the weight's group.  acc_out (optional, [P,M,N] int32) receives the
 * exact accumulators. */
ZG_API size_t zg_int8_lut_linear_workspace_size(int P, int M, int K, int N, int rank, int x_batched);
ZG_API int zg_int8_lut_linear(const int8_t* x, int x_batched, const int8_t* W, const float* w_scale,
                       float x_scale, float y_scale, const int8_t* lut, const uint32_t* keys,
                       int group, int P, int M, int K, int N, int rank, float s, int8_t* out,
                       int32_t* acc_out, void* workspace, size_t workspace_bytes, void* stream);

#ifdef __cplusplus
}
#endif
#endif
