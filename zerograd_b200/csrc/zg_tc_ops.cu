// zg_tc_ops.cu -- bf16 population paths built on the tcgen05 GEMM:
//
//   factor fill in GEMM-operand layout   out[row, p*r + j]  (bf16)
//   forward, shared x:   U  = x . A_all        (tc_gemm, A_all MN-major)
//                        XW = x . W            (tc_gemm, W MN-major)
//                        y[p] = XW + s * U_p . B_p^T   (HBM-bound expansion)
//   replay:              G = (w . A_all) . B_all^T (one tc_gemm over P*r)
//
// The (candidate, rank) pairs q = p*r + j form the contraction axis of the
// replay and the N axis of U, so every candidate's factors are drawn once per
// call and the tensor cores see ordinary dense operands.
#include "zg_tc.cuh"

namespace {

// ---------------------------------------------------------------------------
// factor fill in operand layout.
// out[row, p*r + j] = scale_p * round_T(normal(key_p, ctr(row, j)))
//   ctr = row * r + j          (row_major: A of MATRIX/TABLE, B of TABLE)
//   ctr = j * rows + row       (col_major: B of MATRIX, B_p[j, n])
// blockDim.x threads = consecutive candidates; each thread derives its
// candidate's key once and walks rows, writing r contiguous values.
// ---------------------------------------------------------------------------
template <typename T>
__global__ void fill_operand_kernel(const uint32_t* __restrict__ keys, int group, int P, int rank, int64_t rows,
                                    int which, int col_major, const float* __restrict__ scale, float extra_scale,
                                    int rows_per_block, T* __restrict__ out) {
    const int p = blockIdx.x * blockDim.x + threadIdx.x;
    if (p >= P) return;
    ZgFactorKeys fk = zg_factor_keys(keys, p, group);
    const ZgKey k = which == 0 ? fk.a : fk.b;
    const float sc = scale ? scale[p] * extra_scale : extra_scale;
    const int64_t ld = (int64_t)P * rank;
    const int64_t r0 = (int64_t)blockIdx.y * rows_per_block;
    const int64_t r1 = r0 + rows_per_block < rows ? r0 + rows_per_block : rows;
    // 16-byte stores of 8 bf16 when the rank and the row pitch allow it.
    const bool vec = sizeof(T) == 2 && (rank % 8) == 0 && ((ld * 2) % 16) == 0 &&
                     (reinterpret_cast<uintptr_t>(out) & 15) == 0;
    for (int64_t row = r0; row < r1; ++row) {
        T* dst = out + row * ld + (int64_t)p * rank;
        for (int j0 = 0; j0 < rank; j0 += 8) {
            float v[8];
#pragma unroll
            for (int i = 0; i < 8; ++i) {
                const int j = j0 + i;
                if (j < rank) {
                    const uint64_t ctr = col_major ? (uint64_t)j * rows + row : (uint64_t)row * rank + j;
                    v[i] = zg_dtype_round<T>(zg_normal(k, ctr));
                    if (scale) v[i] = __fmul_rn(v[i], sc);
                }
            }
            if (vec) {
                uint4 pk;
                __nv_bfloat162* h = reinterpret_cast<__nv_bfloat162*>(&pk);
#pragma unroll
                for (int i = 0; i < 4; ++i) h[i] = __floats2bfloat162_rn(v[2 * i], v[2 * i + 1]);
                *reinterpret_cast<uint4*>(dst + j0) = pk;
            } else {
                for (int i = 0; i < 8 && j0 + i < rank; ++i) dst[j0 + i] = zg_from_float<T>(v[i]);
            }
        }
    }
}

// ---------------------------------------------------------------------------
// Low-rank expansion y[p, m, n] = T(XW[m, n] + s * sum_j U[m, p*r+j] * Bq[n, p*r+j])
// Block tile 64 m x 128 n, 256 threads, each 4 m x 8 n; candidates split
// over gridDim.z; q-chunks of QC columns staged in shared memory.
// ---------------------------------------------------------------------------
constexpr int EX_BM = 64, EX_BN = 128, EX_QC = 64;

__device__ __forceinline__ void bf16x8_to_f32(const uint4& v, float (&f)[8]) {
    const uint32_t w[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
    for (int i = 0; i < 4; ++i) {
        f[2 * i] = __uint_as_float(w[i] << 16);
        f[2 * i + 1] = __uint_as_float(w[i] & 0xFFFF0000u);
    }
}

// bf16 operand, r a multiple of 8 and <= EX_QC, N a multiple of 8.
__global__ void __launch_bounds__(256)
lowrank_expand_bf16_kernel(const float* __restrict__ XW, const float* __restrict__ U,
                           const __nv_bfloat16* __restrict__ Bq, int P, int M, int N, int rank, float s,
                           int p_per_split, __nv_bfloat16* __restrict__ y) {
    __shared__ float Us[EX_BM][EX_QC + 1];
    __shared__ __align__(16) __nv_bfloat16 Bs[EX_QC][EX_BN];  // [q][n]
    const int tid = threadIdx.x;
    const int tm = tid / 16, tn = tid % 16;
    const int m0 = blockIdx.y * EX_BM, n0 = blockIdx.x * EX_BN;
    const int64_t ldq = (int64_t)P * rank;
    const int pc = EX_QC / rank;  // candidates per chunk
    const int qc = pc * rank;
    float xw[4][8];
#pragma unroll
    for (int i = 0; i < 4; ++i) {
        const int m = m0 + tm * 4 + i;
#pragma unroll
        for (int c = 0; c < 8; ++c) {
            const int n = n0 + tn * 8 + c;
            xw[i][c] = (m < M && n < N) ? XW[(int64_t)m * N + n] : 0.f;
        }
    }
    const int pb = blockIdx.z * p_per_split;
    const int pe = min(P, pb + p_per_split);
    for (int p0 = pb; p0 < pe; p0 += pc) {
        const int np = min(pc, pe - p0);
        const int nq = np * rank;
        const int64_t q0 = (int64_t)p0 * rank;
        __syncthreads();
        // U chunk: rows of U are contiguous in q (coalesced), smem rows padded.
        for (int e = tid; e < EX_BM * qc; e += 256) {
            const int mm = e / qc, qq = e % qc;
            const int m = m0 + mm;
            Us[mm][qq] = (m < M && qq < nq) ? U[(int64_t)m * ldq + q0 + qq] : 0.f;
        }
        // B chunk: one 16-byte load of 8 consecutive q per (n, q-group);
        // consecutive threads take consecutive n so the transposed smem
        // stores Bs[q][n] do not conflict.
        for (int e = tid; e < EX_BN * (qc / 8); e += 256) {
            const int nn = e % EX_BN, qg = e / EX_BN;
            const int n = n0 + nn;
            uint4 v = make_uint4(0, 0, 0, 0);
            if (n < N && qg * 8 < nq) v = *reinterpret_cast<const uint4*>(Bq + (int64_t)n * ldq + q0 + qg * 8);
            const __nv_bfloat16* h = reinterpret_cast<const __nv_bfloat16*>(&v);
#pragma unroll
            for (int i = 0; i < 8; ++i) Bs[qg * 8 + i][nn] = h[i];
        }
        __syncthreads();
        for (int pi = 0; pi < np; ++pi) {
            float acc[4][8];
#pragma unroll
            for (int i = 0; i < 4; ++i)
#pragma unroll
                for (int c = 0; c < 8; ++c) acc[i][c] = 0.f;
#pragma unroll 4
            for (int j = 0; j < rank; ++j) {
                const int qq = pi * rank + j;
                float bv[8];
                bf16x8_to_f32(*reinterpret_cast<const uint4*>(&Bs[qq][tn * 8]), bv);
#pragma unroll
                for (int i = 0; i < 4; ++i) {
                    const float u = Us[tm * 4 + i][qq];
#pragma unroll
                    for (int c = 0; c < 8; ++c) acc[i][c] = fmaf(u, bv[c], acc[i][c]);
                }
            }
            const int p = p0 + pi;
#pragma unroll
            for (int i = 0; i < 4; ++i) {
                const int m = m0 + tm * 4 + i;
                const int n = n0 + tn * 8;
                if (m >= M || n >= N) continue;
                __nv_bfloat162 h[4];
#pragma unroll
                for (int c = 0; c < 4; ++c)
                    h[c] = __floats2bfloat162_rn(fmaf(s, acc[i][2 * c], xw[i][2 * c]),
                                                 fmaf(s, acc[i][2 * c + 1], xw[i][2 * c + 1]));
                *reinterpret_cast<uint4*>(y + ((int64_t)p * M + m) * N + n) = *reinterpret_cast<uint4*>(h);
            }
        }
    }
}

// General form (any rank <= 32, any N, float or bf16 operand/output).
constexpr int EXG_QC = 32;

template <typename T>
__global__ void __launch_bounds__(256)
lowrank_expand_kernel(const float* __restrict__ XW, const float* __restrict__ U, const T* __restrict__ Bq, int P,
                      int M, int N, int rank, float s, int p_per_split, T* __restrict__ y) {
    __shared__ float Us[EX_BM][EXG_QC + 1];
    __shared__ __align__(16) float Bs[EXG_QC][EX_BN];
    const int tid = threadIdx.x;
    const int tm = tid / 16, tn = tid % 16;
    const int m0 = blockIdx.y * EX_BM, n0 = blockIdx.x * EX_BN;
    const int64_t ldq = (int64_t)P * rank;
    const int pc = rank <= EXG_QC ? EXG_QC / rank : 1;  // candidates per chunk
    const int qc = pc * rank;
    float xw[4][8];
#pragma unroll
    for (int i = 0; i < 4; ++i) {
        const int m = m0 + tm * 4 + i;
#pragma unroll
        for (int c = 0; c < 8; ++c) {
            const int n = n0 + tn * 8 + c;
            xw[i][c] = (m < M && n < N) ? XW[(int64_t)m * N + n] : 0.f;
        }
    }
    const int pb = blockIdx.z * p_per_split;
    const int pe = min(P, pb + p_per_split);
    for (int p0 = pb; p0 < pe; p0 += pc) {
        const int np = min(pc, pe - p0);
        const int nq = np * rank;
        const int64_t q0 = (int64_t)p0 * rank;
        __syncthreads();
        for (int e = tid; e < EX_BM * qc; e += 256) {
            const int mm = e / qc, qq = e % qc;
            const int m = m0 + mm;
            Us[mm][qq] = (m < M && qq < nq) ? U[(int64_t)m * ldq + q0 + qq] : 0.f;
        }
        for (int e = tid; e < EX_BN * qc; e += 256) {
            const int nn = e % EX_BN, qq = e / EX_BN;
            const int n = n0 + nn;
            Bs[qq][nn] = (n < N && qq < nq) ? zg_to_float(Bq[(int64_t)n * ldq + q0 + qq]) : 0.f;
        }
        __syncthreads();
        for (int pi = 0; pi < np; ++pi) {
            float acc[4][8];
#pragma unroll
            for (int i = 0; i < 4; ++i)
#pragma unroll
                for (int c = 0; c < 8; ++c) acc[i][c] = 0.f;
            for (int j = 0; j < rank; ++j) {
                const int qq = pi * rank + j;
                const float4 b0 = *reinterpret_cast<const float4*>(&Bs[qq][tn * 8]);
                const float4 b1 = *reinterpret_cast<const float4*>(&Bs[qq][tn * 8 + 4]);
                const float bv[8] = {b0.x, b0.y, b0.z, b0.w, b1.x, b1.y, b1.z, b1.w};
#pragma unroll
                for (int i = 0; i < 4; ++i) {
                    const float u = Us[tm * 4 + i][qq];
#pragma unroll
                    for (int c = 0; c < 8; ++c) acc[i][c] = fmaf(u, bv[c], acc[i][c]);
                }
            }
            const int p = p0 + pi;
#pragma unroll
            for (int i = 0; i < 4; ++i) {
                const int m = m0 + tm * 4 + i;
                if (m >= M) continue;
                T* dst = y + ((int64_t)p * M + m) * N + n0 + tn * 8;
                const int nrem = N - (n0 + tn * 8);
                if (nrem <= 0) continue;
                if constexpr (sizeof(T) == 2) {
                    if (nrem >= 8) {
                        __nv_bfloat162 h[4];
#pragma unroll
                        for (int c = 0; c < 4; ++c)
                            h[c] = __floats2bfloat162_rn(fmaf(s, acc[i][2 * c], xw[i][2 * c]),
                                                         fmaf(s, acc[i][2 * c + 1], xw[i][2 * c + 1]));
                        *reinterpret_cast<uint4*>(dst) = *reinterpret_cast<uint4*>(h);
                        continue;
                    }
                }
                for (int c = 0; c < 8 && c < nrem; ++c) dst[c] = zg_from_float<T>(fmaf(s, acc[i][c], xw[i][c]));
            }
        }
    }
}

int sm_count() {
    static int n = 0;
    if (!n) {
        int dev = 0;
        cudaGetDevice(&dev);
        cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev);
        if (n <= 0) n = 148;
    }
    return n;
}

}  // namespace

namespace zg {

int fill_operand(const uint32_t* keys, int group, int P, int rank, int64_t rows, int which, int col_major,
                 const float* scale, float extra_scale, int dtype, void* out, cudaStream_t st, const char* name) {
    const int threads = P >= 128 ? 128 : ((P + 31) / 32) * 32;
    const int pblocks = (P + threads - 1) / threads;
    // enough blocks for ~8 waves of rows, each block >= 4 rows
    int64_t want = (int64_t)sm_count() * 16 / pblocks;
    if (want < 1) want = 1;
    int rows_per_block = (int)((rows + want - 1) / want);
    if (rows_per_block < 8) rows_per_block = 8;  // amortise the per-thread key derivation
    const int64_t yblocks = (rows + rows_per_block - 1) / rows_per_block;
    if (yblocks > 65535) return fail(ZG_ERR_INVALID, "fill_operand: too many rows");
    dim3 grid(pblocks, (unsigned)yblocks);
    zg::LaunchTimer zg_lt_(name, st);
    if (dtype == ZG_BF16)
        fill_operand_kernel<__nv_bfloat16><<<grid, threads, 0, st>>>(keys, group, P, rank, rows, which, col_major,
                                                                     scale, extra_scale, rows_per_block,
                                                                     static_cast<__nv_bfloat16*>(out));
    else
        fill_operand_kernel<float><<<grid, threads, 0, st>>>(keys, group, P, rank, rows, which, col_major, scale,
                                                             extra_scale, rows_per_block, static_cast<float*>(out));
    return check_launch("fill_operand");
}

int lowrank_expand(const float* XW, const float* U, const void* Bq, int P, int M, int N, int rank, float s, int dtype,
                   void* y, cudaStream_t st) {
    const int gx = (N + EX_BN - 1) / EX_BN, gy = (M + EX_BM - 1) / EX_BM;
    int splits = (sm_count() * 4 + gx * gy - 1) / (gx * gy);
    if (splits > P) splits = P;
    if (splits < 1) splits = 1;
    const int per = (P + splits - 1) / splits;
    splits = (P + per - 1) / per;
    dim3 grid(gx, gy, splits);
    zg::LaunchTimer zg_lt_("lowrank_expand", st);
    const int64_t ldq_bytes = (int64_t)P * rank * 2;
    if (dtype == ZG_BF16 && rank % 8 == 0 && rank <= EX_QC && N % 8 == 0 && ldq_bytes % 16 == 0 &&
        (reinterpret_cast<uintptr_t>(Bq) & 15) == 0 && (reinterpret_cast<uintptr_t>(y) & 15) == 0) {
        lowrank_expand_bf16_kernel<<<grid, 256, 0, st>>>(XW, U, static_cast<const __nv_bfloat16*>(Bq), P, M, N, rank,
                                                         s, per, static_cast<__nv_bfloat16*>(y));
        return check_launch("lowrank_expand");
    }
    if (dtype == ZG_BF16)
        lowrank_expand_kernel<__nv_bfloat16><<<grid, 256, 0, st>>>(XW, U, static_cast<const __nv_bfloat16*>(Bq), P, M,
                                                                   N, rank, s, per, static_cast<__nv_bfloat16*>(y));
    else
        lowrank_expand_kernel<float><<<grid, 256, 0, st>>>(XW, U, static_cast<const float*>(Bq), P, M, N, rank, s, per,
                                                           static_cast<float*>(y));
    return check_launch("lowrank_expand");
}

// Shared-x population forward on the tensor cores:
//   y[p] = x @ Wop + s (x @ F1_p) @ F2_p^T
// with F1 drawn as [K, P r] (row-major counter) and F2 as [N, P r]
// (f2_col_major selects the counter order of the second factor).
size_t tc_shared_forward_workspace(int P, int M, int K, int N, int rank) {
    const size_t q = (size_t)P * rank;
    return Carver::need({(size_t)K * q * 2, (size_t)N * q * 2, (size_t)M * q * 4, (size_t)M * N * 4});
}

bool tc_shared_forward_ok(int P, int M, int K, int N, int rank) {
    return tc_available() && ((int64_t)P * rank) % 8 == 0 && K % 8 == 0 && N % 8 == 0 && rank <= 32 && M > 0;
}

int tc_shared_forward(const void* x, const void* Wop, bool w_mn_major, int64_t ldw, const uint32_t* keys, int group,
                      int P, int M, int K, int N, int rank, int f1_which, int f1_col_major, int f2_which,
                      int f2_col_major, float s, void* y, Carver& cv, cudaStream_t st) {
    const int64_t q = (int64_t)P * rank;
    __nv_bfloat16* F1 = cv.take<__nv_bfloat16>((size_t)K * q);
    __nv_bfloat16* F2 = cv.take<__nv_bfloat16>((size_t)N * q);
    float* U = cv.take<float>((size_t)M * q);
    float* XW = cv.take<float>((size_t)M * N);
    if (!F1 || !F2 || !U || !XW) return fail(ZG_ERR_WORKSPACE, "tc forward: workspace too small");
    int rc;
    if ((rc = fill_operand(keys, group, P, rank, K, f1_which, f1_col_major, nullptr, 1.f, ZG_BF16, F1, st,
                           "forward_factor_fill")))
        return rc;
    if ((rc = fill_operand(keys, group, P, rank, N, f2_which, f2_col_major, nullptr, 1.f, ZG_BF16, F2, st,
                           "forward_factor_fill")))
        return rc;
    // U[M, q] = x[M, K] . F1[K, q]   (F1 is MN-major for this product)
    if ((rc = tc_gemm_bf16(x, K, F1, q, true, U, q, false, M, (int)q, K, 1.f, st, "forward_u_gemm"))) return rc;
    if ((rc = tc_gemm_bf16(x, K, Wop, ldw, w_mn_major, XW, N, false, M, N, K, 1.f, st, "forward_xw_gemm")))
        return rc;
    return lowrank_expand(XW, U, F2, P, M, N, rank, s, ZG_BF16, y, st);
}

size_t tc_replay_workspace(int P, int64_t rows, int64_t cols, int rank) {
    const size_t q = (size_t)P * rank;
    return Carver::need({(size_t)rows * q * 2, (size_t)cols * q * 2});
}

bool tc_replay_ok(int P, int64_t rows, int64_t cols, int rank, int dtype) {
    return dtype == ZG_BF16 && tc_available() && ((int64_t)P * rank) % 8 == 0 && rows <= 2147483647 &&
           cols <= 2147483647;
}

int tc_replay_run(const float* shaped, const uint32_t* keys, int group, int P, int layout, int64_t rows, int64_t cols,
                  int rank, float inv_sqrt_rank, float* out, Carver& cv, cudaStream_t st) {
    const int64_t q = (int64_t)P * rank;
    __nv_bfloat16* Aw = cv.take<__nv_bfloat16>((size_t)rows * q);
    __nv_bfloat16* Bq = cv.take<__nv_bfloat16>((size_t)cols * q);
    if (!Aw || !Bq) return fail(ZG_ERR_WORKSPACE, "tc replay: workspace too small");
    int rc;
    // weighted A: w_p * A_p[i, j] (the factor in the leaf dtype times the float32 weight)
    if ((rc = fill_operand(keys, group, P, rank, rows, 0, 0, shaped, 1.f, ZG_BF16, Aw, st, "replay_factor_fill")))
        return rc;
    // B: MATRIX B_p[j, n] (counter j*cols + n), TABLE B_p[n, j] (counter n*r + j)
    if ((rc = fill_operand(keys, group, P, rank, cols, 1, layout == ZG_MATRIX ? 1 : 0, nullptr, 1.f, ZG_BF16, Bq, st,
                           "replay_factor_fill")))
        return rc;
    return tc_gemm_bf16(Aw, q, Bq, q, false, out, cols, false, (int)rows, (int)cols, (int)q, inv_sqrt_rank, st,
                        "replay_gemm");
}

}  // namespace zg
