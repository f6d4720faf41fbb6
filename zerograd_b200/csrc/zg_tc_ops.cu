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
#include <mutex>

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
// Eight independent threefry blocks advanced round by round together, so
// the eight dependency chains interleave (the rounds of one block are a
// serial chain of dependent integer operations).
__device__ __forceinline__ void zg_normal_x8(const ZgKey& k, const uint64_t (&ctr)[8], float (&out)[8]) {
    uint32_t x0[8], x1[8];
#pragma unroll
    for (int i = 0; i < 8; ++i) {
        x0[i] = (uint32_t)(ctr[i] >> 32) + k.k0;
        x1[i] = (uint32_t)ctr[i] + k.k1;
    }
    const uint32_t ks[3] = {k.k0, k.k1, k.k2};
    constexpr int R[8] = {13, 15, 26, 6, 17, 29, 16, 24};
#pragma unroll
    for (int g = 0; g < 5; ++g) {
#pragma unroll
        for (int rr = 0; rr < 4; ++rr) {
#pragma unroll
            for (int i = 0; i < 8; ++i) {
                x0[i] += x1[i];
                x1[i] = __funnelshift_l(x1[i], x1[i], R[(g & 1) * 4 + rr]);
                x1[i] ^= x0[i];
            }
        }
#pragma unroll
        for (int i = 0; i < 8; ++i) {
            x0[i] += ks[(g + 1) % 3];
            x1[i] += ks[(g + 2) % 3] + (uint32_t)(g + 1);
        }
    }
#pragma unroll
    for (int i = 0; i < 8; ++i) out[i] = zg_normal_from_bits(x0[i] ^ x1[i]);
}

// Rank a multiple of 8: eight normals per step, no per-element guards.
template <typename T, int R>
__global__ void fill_operand_r8_kernel(const uint32_t* __restrict__ keys, int group, int P, int64_t rows, int which,
                                       int col_major, const float* __restrict__ scale, int rows_per_block,
                                       int64_t ld, T* __restrict__ out) {
    const int p = blockIdx.x * blockDim.x + threadIdx.x;
    if (p >= P) return;
    ZgFactorKeys fk = zg_factor_keys(keys, p, group);
    const ZgKey k = which == 0 ? fk.a : fk.b;
    const float sc = scale ? scale[p] : 1.f;
    const int64_t r0 = (int64_t)blockIdx.y * rows_per_block;
    const int64_t r1 = r0 + rows_per_block < rows ? r0 + rows_per_block : rows;
    for (int64_t row = r0; row < r1; ++row) {
        T* dst = out + row * ld + (int64_t)p * R;
#pragma unroll
        for (int j0 = 0; j0 < R; j0 += 8) {
            uint64_t ctr[8];
#pragma unroll
            for (int i = 0; i < 8; ++i)
                ctr[i] = col_major ? (uint64_t)(j0 + i) * rows + row : (uint64_t)row * R + j0 + i;
            float v[8];
            zg_normal_x8(k, ctr, v);
#pragma unroll
            for (int i = 0; i < 8; ++i) {
                v[i] = zg_dtype_round<T>(v[i]);
                if (scale) v[i] = __fmul_rn(v[i], sc);
            }
            if constexpr (sizeof(T) == 2) {
                uint4 pk;
                __nv_bfloat162* h = reinterpret_cast<__nv_bfloat162*>(&pk);
#pragma unroll
                for (int i = 0; i < 4; ++i) h[i] = __floats2bfloat162_rn(v[2 * i], v[2 * i + 1]);
                *reinterpret_cast<uint4*>(dst + j0) = pk;
            } else {
#pragma unroll
                for (int i = 0; i < 8; ++i) dst[j0 + i] = v[i];
            }
        }
    }
}

// Small populations (P <= 64): threads are (candidate, row) pairs -- x over
// the P candidates padded to 8/16/32/64, y over rows -- so a row's R-wide
// candidate slices are written by adjacent threads and every lane works;
// the values are fill_operand_r8_kernel's.
template <typename T, int R>
__global__ void fill_operand_small_kernel(const uint32_t* __restrict__ keys, int group, int P, int64_t rows,
                                          int which, int col_major, const float* __restrict__ scale,
                                          int rows_per_thread, int64_t ld, T* __restrict__ out) {
    const int p = threadIdx.x;
    if (p >= P) return;
    ZgFactorKeys fk = zg_factor_keys(keys, p, group);
    const ZgKey k = which == 0 ? fk.a : fk.b;
    const float sc = scale ? scale[p] : 1.f;
    const int64_t r0 = ((int64_t)blockIdx.x * blockDim.y + threadIdx.y) * rows_per_thread;
    for (int64_t row = r0; row < r0 + rows_per_thread && row < rows; ++row) {
        T* dst = out + row * ld + (int64_t)p * R;
#pragma unroll
        for (int j0 = 0; j0 < R; j0 += 8) {
            uint64_t ctr[8];
#pragma unroll
            for (int i = 0; i < 8; ++i)
                ctr[i] = col_major ? (uint64_t)(j0 + i) * rows + row : (uint64_t)row * R + j0 + i;
            float v[8];
            zg_normal_x8(k, ctr, v);
#pragma unroll
            for (int i = 0; i < 8; ++i) {
                v[i] = zg_dtype_round<T>(v[i]);
                if (scale) v[i] = __fmul_rn(v[i], sc);
            }
            if constexpr (sizeof(T) == 2) {
                uint4 pk;
                __nv_bfloat162* h = reinterpret_cast<__nv_bfloat162*>(&pk);
#pragma unroll
                for (int i = 0; i < 4; ++i) h[i] = __floats2bfloat162_rn(v[2 * i], v[2 * i + 1]);
                *reinterpret_cast<uint4*>(dst + j0) = pk;
            } else {
#pragma unroll
                for (int i = 0; i < 8; ++i) dst[j0 + i] = v[i];
            }
        }
    }
}

// Transposed fill: out[(p*R + j) * rows + row] = bf16(normal(key_p, row*R + j)).
// Thread = 8 consecutive rows of one candidate and all R ranks, so each of
// its R stores is 16 bytes and a warp's stores for one j are 512 contiguous
// bytes.  grid (row groups, P).
template <int R>
__global__ void fill_operand_t_kernel(const uint32_t* __restrict__ keys, int group, int64_t rows, int which,
                                      __nv_bfloat16* __restrict__ out) {
    const int p = blockIdx.y;
    const int64_t row0 = ((int64_t)blockIdx.x * blockDim.x + threadIdx.x) * 8;
    if (row0 >= rows) return;
    ZgFactorKeys fk = zg_factor_keys(keys, p, group);
    const ZgKey k = which == 0 ? fk.a : fk.b;
    const bool full = row0 + 8 <= rows && (rows % 8) == 0;
#pragma unroll 1
    for (int j = 0; j < R; ++j) {
        uint64_t ctr[8];
#pragma unroll
        for (int i = 0; i < 8; ++i) ctr[i] = (uint64_t)(row0 + i) * R + j;
        float v[8];
        zg_normal_x8(k, ctr, v);
        __nv_bfloat16* dst = out + ((int64_t)p * R + j) * rows + row0;
        if (full) {
            uint4 pk;
            __nv_bfloat162* h = reinterpret_cast<__nv_bfloat162*>(&pk);
#pragma unroll
            for (int i = 0; i < 4; ++i) h[i] = __floats2bfloat162_rn(v[2 * i], v[2 * i + 1]);
            *reinterpret_cast<uint4*>(dst) = pk;
        } else {
            for (int i = 0; i < 8 && row0 + i < rows; ++i) dst[i] = __float2bfloat16_rn(v[i]);
        }
    }
}

template <typename T>
__global__ void fill_operand_kernel(const uint32_t* __restrict__ keys, int group, int P, int rank, int64_t rows,
                                    int which, int col_major, const float* __restrict__ scale, float extra_scale,
                                    int rows_per_block, int64_t ld, T* __restrict__ out) {
    const int p = blockIdx.x * blockDim.x + threadIdx.x;
    if (p >= P) return;
    ZgFactorKeys fk = zg_factor_keys(keys, p, group);
    const ZgKey k = which == 0 ? fk.a : fk.b;
    const float sc = scale ? scale[p] * extra_scale : extra_scale;
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
constexpr int EX_BM = 64, EX_BN = 128;

// Packed float32 pair FMA (sm_100): d = a * b + c on two lanes at once.
__device__ __forceinline__ float2 ffma2(float2 a, float2 b, float2 c) {
    unsigned long long A = *reinterpret_cast<unsigned long long*>(&a), B = *reinterpret_cast<unsigned long long*>(&b),
                       C = *reinterpret_cast<unsigned long long*>(&c), D;
    asm("fma.rn.f32x2 %0, %1, %2, %3;" : "=l"(D) : "l"(A), "l"(B), "l"(C));
    return *reinterpret_cast<float2*>(&D);
}

// bf16 factors and output, compile-time rank R (8 or 16), N % 8 == 0.
// The factor chunk is converted to float32 once while it is staged, so the
// inner loop is shared-memory loads and packed FMAs only.
template <int R>
__global__ void __launch_bounds__(256, 2)
lowrank_expand_bf16_kernel(const float* __restrict__ XW, const float* __restrict__ U,
                           const __nv_bfloat16* __restrict__ Bq, int P, int M, int N, float s, int p_per_split,
                           __nv_bfloat16* __restrict__ y) {
    constexpr int QC = 32;         // q columns per chunk
    constexpr int PC = QC / R;     // candidates per chunk
    __shared__ __align__(16) float Us[EX_BM][QC + 4];
    __shared__ __align__(16) float Bs[QC][EX_BN + 4];
    const int tid = threadIdx.x;
    const int tm = tid / 16, tn = tid % 16;
    const int m0 = blockIdx.y * EX_BM, n0 = blockIdx.x * EX_BN;
    const int64_t ldq = (int64_t)P * R;
    float2 xw[4][4];
#pragma unroll
    for (int i = 0; i < 4; ++i) {
        const int m = m0 + tm * 4 + i;
#pragma unroll
        for (int c = 0; c < 4; ++c) {
            const int n = n0 + tn * 8 + 2 * c;
            xw[i][c] = (m < M && n < N) ? *reinterpret_cast<const float2*>(XW + (int64_t)m * N + n)
                                        : make_float2(0.f, 0.f);
        }
    }
    const float2 s2 = make_float2(s, s);
    const int pb = blockIdx.z * p_per_split;
    const int pe = min(P, pb + p_per_split);
    for (int p0 = pb; p0 < pe; p0 += PC) {
        const int np = min(PC, pe - p0);
        const int nq = np * R;
        const int64_t q0 = (int64_t)p0 * R;
        __syncthreads();
        // U chunk [64 m x 32 q]: 16-byte loads along q, 2 per thread.
#pragma unroll
        for (int it = 0; it < (EX_BM * QC / 4) / 256; ++it) {
            const int e = tid + it * 256;
            const int mm = e / (QC / 4), c4 = e % (QC / 4);
            const int m = m0 + mm;
            float4 v = make_float4(0.f, 0.f, 0.f, 0.f);
            if (m < M && c4 * 4 < nq) v = *reinterpret_cast<const float4*>(U + (int64_t)m * ldq + q0 + c4 * 4);
            *reinterpret_cast<float4*>(&Us[mm][c4 * 4]) = v;
        }
        // B chunk [128 n x 32 q] bf16 -> Bs[q][n] float32, consecutive threads on consecutive n.
#pragma unroll
        for (int it = 0; it < (EX_BN * QC / 8) / 256; ++it) {
            const int e = tid + it * 256;
            const int nn = e % EX_BN, qg = e / EX_BN;
            const int n = n0 + nn;
            float f[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
            if (n < N && qg * 8 < nq)
                bf16x8_to_f32(*reinterpret_cast<const uint4*>(Bq + (int64_t)n * ldq + q0 + qg * 8), f);
#pragma unroll
            for (int i = 0; i < 8; ++i) Bs[qg * 8 + i][nn] = f[i];
        }
        __syncthreads();
#pragma unroll
        for (int pi = 0; pi < PC; ++pi) {
            if (pi >= np) break;
            float2 acc[4][4];
#pragma unroll
            for (int i = 0; i < 4; ++i)
#pragma unroll
                for (int c = 0; c < 4; ++c) acc[i][c] = make_float2(0.f, 0.f);
#pragma unroll
            for (int j = 0; j < R; ++j) {
                const int qq = pi * R + j;
                const float4 bl = *reinterpret_cast<const float4*>(&Bs[qq][tn * 8]);
                const float4 bh = *reinterpret_cast<const float4*>(&Bs[qq][tn * 8 + 4]);
                const float2 b[4] = {make_float2(bl.x, bl.y), make_float2(bl.z, bl.w), make_float2(bh.x, bh.y),
                                     make_float2(bh.z, bh.w)};
#pragma unroll
                for (int i = 0; i < 4; ++i) {
                    const float u = Us[tm * 4 + i][qq];
                    const float2 u2 = make_float2(u, u);
#pragma unroll
                    for (int c = 0; c < 4; ++c) acc[i][c] = ffma2(u2, b[c], acc[i][c]);
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
                for (int c = 0; c < 4; ++c) {
                    const float2 o = ffma2(s2, acc[i][c], xw[i][c]);
                    h[c] = __floats2bfloat162_rn(o.x, o.y);
                }
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
                 const float* scale, float extra_scale, int dtype, void* out, cudaStream_t st, const char* name,
                 int64_t ld) {
    if (ld == 0) ld = (int64_t)P * rank;
    if (ld < (int64_t)P * rank) return fail(ZG_ERR_INVALID, "fill_operand: row pitch below P*rank");
    const int threads = P >= 128 ? 128 : ((P + 31) / 32) * 32;
    const int pblocks = (P + threads - 1) / threads;
    // enough blocks for ~8 waves of rows, each block >= 4 rows
    int64_t want = (int64_t)sm_count() * 16 / pblocks;
    if (want < 1) want = 1;
    int rows_per_block = (int)((rows + want - 1) / want);
    if (rows_per_block < 4) rows_per_block = 4;  // amortise the per-thread key derivation
    const int64_t yblocks = (rows + rows_per_block - 1) / rows_per_block;
    if (yblocks > 65535) return fail(ZG_ERR_INVALID, "fill_operand: too many rows");
    dim3 grid(pblocks, (unsigned)yblocks);
    zg::LaunchTimer zg_lt_(name, st);
    const size_t esz = dtype == ZG_BF16 ? 2 : 4;
    const bool aligned = (reinterpret_cast<uintptr_t>(out) & 15) == 0 && extra_scale == 1.f && (ld * esz) % 16 == 0;
    if (aligned && (rank == 8 || rank == 16) && P <= 64) {
        const int px = P <= 8 ? 8 : P <= 16 ? 16 : P <= 32 ? 32 : 64;
        const int ry = 128 / px;
        int64_t want_threads = (int64_t)sm_count() * 8 * ry;  // ~8 blocks of 128 threads per SM
        int rpt = (int)((rows + want_threads - 1) / want_threads);
        if (rpt < 2) rpt = 2;  // amortise the per-thread key derivation
        const int64_t gx = (rows + (int64_t)ry * rpt - 1) / ((int64_t)ry * rpt);
        if (gx > 2147483647) return fail(ZG_ERR_INVALID, "fill_operand: too many rows");
        dim3 g2((unsigned)gx), b2(px, ry);
#define ZG_FILL_SMALL(TT, RR)                                                                                      \
    fill_operand_small_kernel<TT, RR><<<g2, b2, 0, st>>>(keys, group, P, rows, which, col_major, scale, rpt, \
                                                          ld, static_cast<TT*>(out))
        if (dtype == ZG_BF16) {
            if (rank == 8) ZG_FILL_SMALL(__nv_bfloat16, 8);
            else ZG_FILL_SMALL(__nv_bfloat16, 16);
        } else {
            if (rank == 8) ZG_FILL_SMALL(float, 8);
            else ZG_FILL_SMALL(float, 16);
        }
#undef ZG_FILL_SMALL
        return check_launch("fill_operand");
    }
    if (aligned && (rank == 8 || rank == 16)) {
        if (dtype == ZG_BF16) {
            if (rank == 8)
                fill_operand_r8_kernel<__nv_bfloat16, 8><<<grid, threads, 0, st>>>(
                    keys, group, P, rows, which, col_major, scale, rows_per_block, ld, static_cast<__nv_bfloat16*>(out));
            else
                fill_operand_r8_kernel<__nv_bfloat16, 16><<<grid, threads, 0, st>>>(
                    keys, group, P, rows, which, col_major, scale, rows_per_block, ld, static_cast<__nv_bfloat16*>(out));
        } else {
            if (rank == 8)
                fill_operand_r8_kernel<float, 8><<<grid, threads, 0, st>>>(keys, group, P, rows, which, col_major,
                                                                           scale, rows_per_block, ld,
                                                                           static_cast<float*>(out));
            else
                fill_operand_r8_kernel<float, 16><<<grid, threads, 0, st>>>(keys, group, P, rows, which, col_major,
                                                                            scale, rows_per_block, ld,
                                                                            static_cast<float*>(out));
        }
        return check_launch("fill_operand");
    }
    if (dtype == ZG_BF16)
        fill_operand_kernel<__nv_bfloat16><<<grid, threads, 0, st>>>(keys, group, P, rank, rows, which, col_major,
                                                                     scale, extra_scale, rows_per_block, ld,
                                                                     static_cast<__nv_bfloat16*>(out));
    else
        fill_operand_kernel<float><<<grid, threads, 0, st>>>(keys, group, P, rank, rows, which, col_major, scale,
                                                             extra_scale, rows_per_block, ld, static_cast<float*>(out));
    return check_launch("fill_operand");
}

int fill_operand_t(const uint32_t* keys, int group, int P, int rank, int64_t rows, int which, void* out,
                   cudaStream_t st, const char* name) {
    if (rank != 8 && rank != 16) return fail(ZG_ERR_INVALID, "fill_operand_t: rank must be 8 or 16");
    if (P < 1 || P > 65535 || rows < 1) return fail(ZG_ERR_INVALID, "fill_operand_t: bad sizes");
    const int64_t gx = ((rows + 7) / 8 + 127) / 128;
    if (gx > 2147483647) return fail(ZG_ERR_INVALID, "fill_operand_t: too many rows");
    dim3 grid((unsigned)gx, (unsigned)P);
    zg::LaunchTimer zg_lt_(name, st);
    auto* o = static_cast<__nv_bfloat16*>(out);
    if (rank == 8)
        fill_operand_t_kernel<8><<<grid, 128, 0, st>>>(keys, group, rows, which, o);
    else
        fill_operand_t_kernel<16><<<grid, 128, 0, st>>>(keys, group, rows, which, o);
    return check_launch("fill_operand_t");
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
    const bool fast = dtype == ZG_BF16 && (rank == 8 || rank == 16) && N % 8 == 0 && ldq_bytes % 16 == 0 &&
                      (reinterpret_cast<uintptr_t>(Bq) & 15) == 0 && (reinterpret_cast<uintptr_t>(y) & 15) == 0 &&
                      (reinterpret_cast<uintptr_t>(U) & 15) == 0 && (reinterpret_cast<uintptr_t>(XW) & 7) == 0;
    if (fast) {
        if (rank == 8)
            lowrank_expand_bf16_kernel<8><<<grid, 256, 0, st>>>(XW, U, static_cast<const __nv_bfloat16*>(Bq), P, M, N,
                                                                s, per, static_cast<__nv_bfloat16*>(y));
        else
            lowrank_expand_bf16_kernel<16><<<grid, 256, 0, st>>>(XW, U, static_cast<const __nv_bfloat16*>(Bq), P, M,
                                                                 N, s, per, static_cast<__nv_bfloat16*>(y));
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

// ---------------------------------------------------------------------------
// Operand factors of one entry: A_op[rows, P r] (A_p, counter row*r + j) and
// B_op[cols, P r] (MATRIX: B_p[j, col], counter j*cols + col; TABLE:
// B_p[col, j], counter col*r + j).  The forward pass and the replay of the
// same generation use the same two buffers, so they are drawn once.
// ---------------------------------------------------------------------------
int factor_operands(const uint32_t* keys, int group, int P, int layout, int64_t rows, int64_t cols, int rank,
                    int dtype, void* A_op, void* B_op, cudaStream_t st) {
    int rc;
    if (A_op && (rc = fill_operand(keys, group, P, rank, rows, 0, 0, nullptr, 1.f, dtype, A_op, st, "factor_fill")))
        return rc;
    if (B_op && (rc = fill_operand(keys, group, P, rank, cols, 1, layout == ZG_MATRIX ? 1 : 0, nullptr, 1.f, dtype,
                                   B_op, st, "factor_fill")))
        return rc;
    return ZG_OK;
}

// Shared-x population forward on the tensor cores from operand factors:
//   y[p] = x @ Wop + s (x @ F1_p) @ F2_p^T,  F1 [K, P r], F2 [N, P r].
size_t tc_forward_factors_workspace(int P, int M, int N, int rank) {
    return Carver::need({(size_t)M * P * rank * 4, (size_t)M * N * 4});
}

bool tc_shared_forward_ok(int P, int M, int K, int N, int rank) {
    return tc_available() && ((int64_t)P * rank) % 8 == 0 && K % 8 == 0 && N % 8 == 0 && rank <= 32 && M > 0;
}

// A second stream per device for fork/join overlap inside one call: work on
// it waits for everything queued on the caller's stream so far, and the
// caller's stream waits for it before the call returns, so to the caller the
// call stays one in-order unit on its own stream.  The enqueue sequence is
// serialised per device so two host threads cannot interleave fork events.
struct SideStream {
    cudaStream_t s = nullptr;
    cudaEvent_t fork = nullptr, join = nullptr;
    std::mutex mu;
};

SideStream* side_stream() {
    static SideStream streams[64];
    static std::mutex init_mu;
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return nullptr;
    SideStream& ss = streams[dev];
    std::lock_guard<std::mutex> lk(init_mu);
    if (!ss.s) {
        if (cudaStreamCreateWithFlags(&ss.s, cudaStreamNonBlocking) != cudaSuccess ||
            cudaEventCreateWithFlags(&ss.fork, cudaEventDisableTiming) != cudaSuccess ||
            cudaEventCreateWithFlags(&ss.join, cudaEventDisableTiming) != cudaSuccess) {
            ss.s = nullptr;
            return nullptr;
        }
    }
    return &ss;
}

// The shared-x forward, with optional factor draws.  Schedule:
//   caller stream: [fill F1] -> U = x F1 --------------------.-> expansion
//   side stream:          XW = x W -> [fill F2] ------------'
// The fills are integer-ALU bound and the GEMMs tensor/L2 bound, so the two
// streams overlap on the same SMs.
// F1's and F2's rows have leading dimensions ld1 and ld2 (P r for buffers of
// this population alone; larger for a column block of a larger population's
// factors, which only the tensor-core expansion reads).
int tc_forward_schedule(const void* x, const void* Wop, bool w_mn_major, int64_t ldw, const uint32_t* keys, int group,
                        int f1_which, int f1_col_major, int f2_which, int f2_col_major, bool draw, const void* F1,
                        int64_t ld1, const void* F2, int64_t ld2, int P, int M, int K, int N, int rank, float s,
                        void* y, Carver& cv, cudaStream_t st) {
    const int64_t q = (int64_t)P * rank;
    float* U = cv.take<float>((size_t)M * q);
    float* XW = cv.take<float>((size_t)M * N);
    if (!U || !XW) return fail(ZG_ERR_WORKSPACE, "tc forward: workspace too small");
    const bool tc_exp = tc_expand_ok(P, M, N, rank, XW, U, F2, y);
    if ((draw && (ld1 != q || ld2 != q)) || (!tc_exp && ld2 != q))
        return fail(ZG_ERR_UNSUPPORTED, "tc forward: strided factors need the rank-8 tensor-core expansion");
    SideStream* ss = side_stream();
    if (!ss) return fail(ZG_ERR_CUDA, "tc forward: side stream");
    int rc = ZG_OK, rc_side = ZG_OK;
    {
        std::lock_guard<std::mutex> lk(ss->mu);
        if (cudaEventRecord(ss->fork, st) != cudaSuccess || cudaStreamWaitEvent(ss->s, ss->fork, 0) != cudaSuccess)
            return fail(ZG_ERR_CUDA, "tc forward: fork");
        rc_side = tc_gemm_bf16(x, K, Wop, ldw, w_mn_major, XW, N, false, M, N, K, 1.f, ss->s, "forward_xw_gemm");
        if (!rc_side && draw)
            rc_side = fill_operand(keys, group, P, rank, N, f2_which, f2_col_major, nullptr, 1.f, ZG_BF16,
                                   const_cast<void*>(F2), ss->s, "factor_fill");
        if (draw)
            rc = fill_operand(keys, group, P, rank, K, f1_which, f1_col_major, nullptr, 1.f, ZG_BF16,
                              const_cast<void*>(F1), st, "factor_fill");
        // U = x F1 (F1 is MN-major for this product); bf16 for the tensor-core
        // expansion (x @ A rounded to the leaf dtype, as the reference's bf16 x @ a is)
        if (!rc) rc = tc_gemm_bf16(x, K, F1, ld1, true, U, q, tc_exp, M, (int)q, K, 1.f, st, "forward_u_gemm");
        // join unconditionally so the side stream never outlives the call
        if (cudaEventRecord(ss->join, ss->s) != cudaSuccess || cudaStreamWaitEvent(st, ss->join, 0) != cudaSuccess)
            return fail(ZG_ERR_CUDA, "tc forward: join");
    }
    if (rc) return rc;
    if (rc_side) return rc_side;
    if (tc_exp) return tc_expand_r8(XW, U, F2, ld2, P, M, N, s, y, st);
    return lowrank_expand(XW, U, F2, P, M, N, rank, s, ZG_BF16, y, st);
}

int tc_forward_factors(const void* x, const void* Wop, bool w_mn_major, int64_t ldw, const void* F1, const void* F2,
                       int P, int M, int K, int N, int rank, float s, void* y, Carver& cv, cudaStream_t st,
                       int64_t ld1 = 0, int64_t ld2 = 0) {
    const int64_t q = (int64_t)P * rank;
    return tc_forward_schedule(x, Wop, w_mn_major, ldw, nullptr, 0, 0, 0, 0, 0, false, F1, ld1 ? ld1 : q, F2,
                               ld2 ? ld2 : q, P, M, K, N, rank, s, y, cv, st);
}

size_t tc_shared_forward_workspace(int P, int M, int K, int N, int rank) {
    const size_t q = (size_t)P * rank;
    return Carver::need({(size_t)K * q * 2, (size_t)N * q * 2}) + tc_forward_factors_workspace(P, M, N, rank) + 256;
}

int tc_shared_forward(const void* x, const void* Wop, bool w_mn_major, int64_t ldw, const uint32_t* keys, int group,
                      int P, int M, int K, int N, int rank, int f1_which, int f1_col_major, int f2_which,
                      int f2_col_major, float s, void* y, Carver& cv, cudaStream_t st) {
    const int64_t q = (int64_t)P * rank;
    __nv_bfloat16* F1 = cv.take<__nv_bfloat16>((size_t)K * q);
    __nv_bfloat16* F2 = cv.take<__nv_bfloat16>((size_t)N * q);
    if (!F1 || !F2) return fail(ZG_ERR_WORKSPACE, "tc forward: workspace too small");
    return tc_forward_schedule(x, Wop, w_mn_major, ldw, keys, group, f1_which, f1_col_major, f2_which, f2_col_major,
                               true, F1, q, F2, q, P, M, K, N, rank, s, y, cv, st);
}

bool batched_forward_ok(int P, int M, int K, int N, int rank) {
    return tc_available() && (rank == 8 || rank == 16) && P > 0 && M > 0 && K % 8 == 0 && N % 8 == 0 &&
           (int64_t)P * ((M + 127) / 128) * ((N + 255) / 256) <= 2147483647LL && (int64_t)P * rank <= 2147483647LL;
}

size_t batched_forward_workspace(int P, int M, int K, int N, int rank, bool draw) {
    const size_t q = (size_t)P * rank;
    size_t need = Carver::need({(size_t)P * M * 16 * 2});
    if (draw) need += Carver::need({q * K * 2, (size_t)N * q * 2});
    return need + 256;
}

// Per-candidate-input forward.  With `draw`, the factors are drawn into F1T /
// F2 (carved from the workspace when null) first:
//   caller stream: [fill F1T] -> u pass --------.-> gemm
//   side stream:   [fill F2] -------------------'
int batched_forward(const void* x, const void* Wop, bool w_mn_major, const uint32_t* keys, int group, int f1_which,
                    int f2_which, int f2_col_major, bool draw, const void* F1T, const void* F2, int P, int M, int K,
                    int N, int rank, float s, void* y, Carver& cv, cudaStream_t st, int64_t ld2, int act,
                    const void* res) {
    const int64_t q = (int64_t)P * rank;
    __nv_bfloat16* U = cv.take<__nv_bfloat16>((size_t)P * M * 16);
    if (draw && !F1T) F1T = cv.take<__nv_bfloat16>((size_t)q * K);
    if (draw && !F2) {
        F2 = cv.take<__nv_bfloat16>((size_t)N * q);
        ld2 = 0;
    }
    if (!U || !F1T || !F2) return fail(ZG_ERR_WORKSPACE, "batched forward: workspace too small");
    auto al = [](const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15) == 0; };
    if (!al(x) || !al(Wop) || !al(F1T) || !al(F2) || !al(y))
        return fail(ZG_ERR_INVALID, "batched forward: operands must be 16-byte aligned");
    int rc = ZG_OK, rc_side = ZG_OK;
    if (draw) {
        SideStream* ss = side_stream();
        if (!ss) return fail(ZG_ERR_CUDA, "batched forward: side stream");
        std::lock_guard<std::mutex> lk(ss->mu);
        if (cudaEventRecord(ss->fork, st) != cudaSuccess || cudaStreamWaitEvent(ss->s, ss->fork, 0) != cudaSuccess)
            return fail(ZG_ERR_CUDA, "batched forward: fork");
        rc_side = fill_operand(keys, group, P, rank, N, f2_which, f2_col_major, nullptr, 1.f, ZG_BF16,
                               const_cast<void*>(F2), ss->s, "factor_fill", ld2);
        rc = fill_operand_t(keys, group, P, rank, K, f1_which, const_cast<void*>(F1T), st, "factor_fill");
        if (!rc) rc = batched_u_pass(x, F1T, P, M, K, rank, s, U, st);
        if (cudaEventRecord(ss->join, ss->s) != cudaSuccess || cudaStreamWaitEvent(st, ss->join, 0) != cudaSuccess)
            return fail(ZG_ERR_CUDA, "batched forward: join");
    } else {
        rc = batched_u_pass(x, F1T, P, M, K, rank, s, U, st);
    }
    if (rc) return rc;
    if (rc_side) return rc_side;
    return batched_gemm(x, Wop, w_mn_major, U, F2, P, M, K, N, rank, y, st, ld2, act, res);
}

// Aw[row, q] = bf16(float(A[row, q]) * w[q / rank]): the reference's
// weighted factor a_pop * shaped (src/zerograd/_replay.py:46) rounded to the
// tensor-core operand type.
// grid (column groups of 8, rows): thread = 8 consecutive columns of one row.
__global__ void scale_operand_kernel(const __nv_bfloat16* __restrict__ A, const float* __restrict__ w, int rank,
                                     int q, int64_t rows, __nv_bfloat16* __restrict__ out) {
    const int col0 = (blockIdx.x * blockDim.x + threadIdx.x) * 8;
    if (col0 >= q) return;
    float wk[8];
    if (rank % 8 == 0) {
        const float wc = w[col0 / rank];
#pragma unroll
        for (int k = 0; k < 8; ++k) wk[k] = wc;
    } else {
#pragma unroll
        for (int k = 0; k < 8; ++k) wk[k] = w[(col0 + k) / rank];
    }
    // four rows per thread per pass, their loads issued together, so enough
    // bytes are in flight per SM to run at HBM rate
    const int64_t gy = gridDim.y;
    for (int64_t r0 = blockIdx.y; r0 < rows; r0 += 4 * gy) {
        uint4 v[4];
#pragma unroll
        for (int u = 0; u < 4; ++u) {
            const int64_t row = r0 + u * gy;
            if (row < rows) v[u] = *reinterpret_cast<const uint4*>(A + row * q + col0);
        }
#pragma unroll
        for (int u = 0; u < 4; ++u) {
            const int64_t row = r0 + u * gy;
            if (row >= rows) break;
            float f[8];
            bf16x8_to_f32(v[u], f);
            uint4 pk;
            __nv_bfloat162* h = reinterpret_cast<__nv_bfloat162*>(&pk);
#pragma unroll
            for (int k = 0; k < 4; ++k)
                h[k] = __floats2bfloat162_rn(__fmul_rn(f[2 * k], wk[2 * k]), __fmul_rn(f[2 * k + 1], wk[2 * k + 1]));
            *reinterpret_cast<uint4*>(out + row * q + col0) = pk;
        }
    }
}

// Grid rows for scale_operand_kernel: about 8 resident blocks per SM, each
// thread covering at least four rows.
int64_t scale_grid_rows(unsigned gx, int64_t rows) {
    int64_t gy = (int64_t)sm_count() * 8 / gx;
    if (gy > (rows + 3) / 4) gy = (rows + 3) / 4;
    if (gy < 1) gy = 1;
    if (gy > 65535) gy = 65535;
    return gy;
}

// Transposing form: Aw[row, q] = bf16(float(AT[q, row]) * w[q / rank]) for
// an input-side factor kept K-major as AT [P r, rows].  64 x 64 tiles through
// shared memory so both the reads and the writes are 16-byte coalesced.
__global__ void __launch_bounds__(256)
scale_operand_t_kernel(const __nv_bfloat16* __restrict__ AT, const float* __restrict__ w, int rank, int q,
                       int64_t rows, __nv_bfloat16* __restrict__ out) {
    __shared__ float tile[64][65];
    const int64_t r0 = (int64_t)blockIdx.x * 64;
    const int q0 = blockIdx.y * 64;
    const int tid = threadIdx.x;
    // read: 64 q rows x 64 row elements, 8 per thread-chunk, 2 chunks per thread
#pragma unroll
    for (int it = 0; it < 2; ++it) {
        const int e = tid + it * 256;
        const int qq = e / 8, c8 = (e % 8) * 8;
        const int qg = q0 + qq;
        float f[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
        if (qg < q) {
            const float wq = w[qg / rank];
            if (r0 + c8 + 8 <= rows) {
                bf16x8_to_f32(*reinterpret_cast<const uint4*>(AT + (int64_t)qg * rows + r0 + c8), f);
            } else {
                for (int i = 0; i < 8; ++i)
                    if (r0 + c8 + i < rows) f[i] = __bfloat162float(AT[(int64_t)qg * rows + r0 + c8 + i]);
            }
#pragma unroll
            for (int i = 0; i < 8; ++i) f[i] = __fmul_rn(f[i], wq);
        }
#pragma unroll
        for (int i = 0; i < 8; ++i) tile[qq][c8 + i] = f[i];
    }
    __syncthreads();
    // write: 64 rows x 64 q, 8 q per thread-chunk
#pragma unroll
    for (int it = 0; it < 2; ++it) {
        const int e = tid + it * 256;
        const int rr = e / 8, c8 = (e % 8) * 8;
        const int64_t row = r0 + rr;
        if (row >= rows || q0 + c8 >= q) continue;
        uint4 pk;
        __nv_bfloat162* h = reinterpret_cast<__nv_bfloat162*>(&pk);
#pragma unroll
        for (int i = 0; i < 4; ++i) h[i] = __floats2bfloat162_rn(tile[c8 + 2 * i][rr], tile[c8 + 2 * i + 1][rr]);
        *reinterpret_cast<uint4*>(out + row * q + q0 + c8) = pk;  // q % 8 == 0
    }
}

// Row form of the weighting, for a factor kept [P r, cols] (the GEMM's
// MN-major operand): out[q, c] = bf16(float(BT[q, c]) * w[q / rank]).
// Thread = 8 consecutive columns of one row (cols % 8 == 0), grid-stride.
__global__ void __launch_bounds__(256)
scale_rows_kernel(const __nv_bfloat16* __restrict__ BT, const float* __restrict__ w, int rank, int64_t q,
                  int64_t cols, __nv_bfloat16* __restrict__ out) {
    const int64_t groups = q * (cols / 8);
    const int64_t stride = (int64_t)gridDim.x * blockDim.x;
    for (int64_t g = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; g < groups; g += stride) {
        const int64_t row = g / (cols / 8);
        const float wr = w[row / rank];
        float f[8];
        bf16x8_to_f32(*reinterpret_cast<const uint4*>(BT + g * 8), f);
        uint4 pk;
        __nv_bfloat162* h = reinterpret_cast<__nv_bfloat162*>(&pk);
#pragma unroll
        for (int k = 0; k < 4; ++k) h[k] = __floats2bfloat162_rn(__fmul_rn(f[2 * k], wr), __fmul_rn(f[2 * k + 1], wr));
        *reinterpret_cast<uint4*>(out + g * 8) = pk;
    }
}

// Number of candidate groups the replay contraction is split into: the
// largest S in {8, 4, 2} whose groups keep at least 4096 of the P r
// contraction columns, a multiple of 64 (else 1).  A function of P and rank
// only, so every entry of a model, on any number of GPUs, splits alike.
int replay_split_count(int P, int rank) {
    const int64_t q = (int64_t)P * rank;
    for (int S = kMaxSplits; S > 1; S /= 2)
        if (q % S == 0 && (q / S) % 64 == 0 && q / S >= 4096) return S;
    return 1;
}

// Bytes of the weighted operand (the side it scales) and of the split partials.
size_t tc_replay_operands_workspace(int P, int64_t rows, int64_t cols, int rank) {
    const size_t q = (size_t)P * rank;
    const int S = replay_split_count(P, rank);
    const size_t side = (size_t)(rows > cols ? rows : cols);
    return Carver::need({side * q * 2, S > 1 ? (size_t)S * rows * cols * 4 : 0}) + 256;
}

namespace {

// The replay's GEMM operands with the shaped fitness applied to one side:
// the input-side factor when it has to be transposed anyway (a_t), else the
// smaller side (the weighting pass then moves the fewest bytes).
int weighted_operands(const float* shaped, const void* A, bool a_t, const void* B, bool b_t, int P, int64_t rows,
                      int64_t cols, int rank, Carver& cv, cudaStream_t st, const void** Aop, const void** Bop) {
    const int64_t q = (int64_t)P * rank;
    if (q % 8 || (reinterpret_cast<uintptr_t>(A) & 15) || (reinterpret_cast<uintptr_t>(B) & 15))
        return fail(ZG_ERR_INVALID, "tc replay: operand alignment");
    if (b_t && cols % 8) return fail(ZG_ERR_INVALID, "tc replay: transposed B needs cols % 8 == 0");
    if (q > 2147483647 || rows > 2147483647 || cols > 2147483647)
        return fail(ZG_ERR_INVALID, "tc replay: sizes too large");
    *Aop = A;
    *Bop = B;
    const bool scale_b = !a_t && cols < rows;
    __nv_bfloat16* W = cv.take<__nv_bfloat16>((size_t)(scale_b ? cols : rows) * q);
    if (!W) return fail(ZG_ERR_WORKSPACE, "tc replay: workspace too small");
    zg::LaunchTimer zg_lt_("replay_scale", st);
    if (a_t) {
        const int64_t gx = (rows + 63) / 64, gy = (q + 63) / 64;
        if (gy > 65535 || gx > 2147483647) return fail(ZG_ERR_INVALID, "tc replay: transposed A too large");
        scale_operand_t_kernel<<<dim3((unsigned)gx, (unsigned)gy), 256, 0, st>>>(
            static_cast<const __nv_bfloat16*>(A), shaped, rank, (int)q, rows, W);
        *Aop = W;
    } else if (scale_b && b_t) {
        const int64_t groups = q * (cols / 8);
        int64_t grid = (groups + 255) / 256;
        if (grid > (int64_t)sm_count() * 8) grid = (int64_t)sm_count() * 8;
        scale_rows_kernel<<<(unsigned)grid, 256, 0, st>>>(static_cast<const __nv_bfloat16*>(B), shaped, rank, q, cols,
                                                          W);
        *Bop = W;
    } else {
        const int64_t n = scale_b ? cols : rows;
        const unsigned gx = (unsigned)((q / 8 + 255) / 256);
        const int64_t gy = scale_grid_rows(gx, n);
        scale_operand_kernel<<<dim3(gx, (unsigned)gy), 256, 0, st>>>(
            static_cast<const __nv_bfloat16*>(scale_b ? B : A), shaped, rank, (int)q, n, W);
        if (scale_b) *Bop = W; else *Aop = W;
    }
    return check_launch("replay_scale");
}

}  // namespace

// Replay from operand factors given in either layout: A [rows, P r] or, with
// a_t, AT [P r, rows]; B [cols, P r] or, with b_t, BT [P r, cols] (then the
// GEMM reads it as its MN-major operand).  The contraction over the P
// candidates runs as S = replay_split_count(P, rank) groups of P / S
// candidates, each accumulated on its own, then summed in group order and
// scaled: d = inv_sqrt_rank * (((G_0 + G_1) + G_2) + ...), so a GPU that
// holds only some of the groups' factors computes the same partials
// (zg_replay_partials) and the sum is the same bits on any number of GPUs.
int tc_replay_operands(const float* shaped, const void* A, bool a_t, const void* B, bool b_t, int P, int64_t rows,
                       int64_t cols, int rank, float inv_sqrt_rank, float* out, Carver& cv, cudaStream_t st,
                       const FusedStep* step) {
    const int64_t q = (int64_t)P * rank;
    const void *Aop, *Bop;
    int rc = weighted_operands(shaped, A, a_t, B, b_t, P, rows, cols, rank, cv, st, &Aop, &Bop);
    if (rc) return rc;
    const int S = replay_split_count(P, rank);
    const int64_t ldb = b_t ? cols : q;
    if (S == 1)
        return tc_gemm_core(Aop, q, Bop, ldb, b_t, out, cols, false, (int)rows, (int)cols, 1, 1, (int)q, 0,
                            inv_sqrt_rank, st, "replay_gemm", step);
    const int64_t n = rows * cols;
    float* parts = cv.take<float>((size_t)S * n);
    if (!parts) return fail(ZG_ERR_WORKSPACE, "tc replay: workspace too small for the split partials");
    rc = tc_gemm_core(Aop, q, Bop, ldb, b_t, parts, cols, false, (int)rows, (int)cols, S, S, (int)(q / S), n, 1.f, st,
                      "replay_gemm", nullptr);
    if (rc) return rc;
    int64_t offs[kMaxSplits];
    for (int s = 0; s < S; ++s) offs[s] = s * n;
    return split_reduce(parts, offs, S, n, inv_sqrt_rank, step, out, st);
}

int tc_replay_partials(const float* shaped, const void* A, bool a_t, const void* B, bool b_t, int P, int64_t rows,
                       int64_t cols, int rank, int split_total, int splits, float* parts, int64_t part_stride,
                       Carver& cv, cudaStream_t st) {
    const int64_t q = (int64_t)P * rank;
    if (splits < 1 || split_total < splits || split_total > kMaxSplits || q % splits || (q / splits) % 64)
        return fail(ZG_ERR_INVALID, "replay partials: each split needs a multiple of 64 contraction columns");
    if (part_stride < rows * cols) return fail(ZG_ERR_INVALID, "replay partials: partials overlap");
    const void *Aop, *Bop;
    int rc = weighted_operands(shaped, A, a_t, B, b_t, P, rows, cols, rank, cv, st, &Aop, &Bop);
    if (rc) return rc;
    return tc_gemm_core(Aop, q, Bop, b_t ? cols : q, b_t, parts, cols, false, (int)rows, (int)cols, splits,
                        split_total, (int)(q / splits), part_stride, 1.f, st, "replay_gemm", nullptr);
}

int tc_replay_factors(const float* shaped, const void* A_op, const void* B_op, int P, int64_t rows, int64_t cols,
                      int rank, float inv_sqrt_rank, float* out, Carver& cv, cudaStream_t st, const FusedStep* step) {
    return tc_replay_operands(shaped, A_op, false, B_op, false, P, rows, cols, rank, inv_sqrt_rank, out, cv, st, step);
}

size_t tc_replay_workspace(int P, int64_t rows, int64_t cols, int rank) {
    const size_t q = (size_t)P * rank;
    return Carver::need({(size_t)rows * q * 2, (size_t)cols * q * 2}) + tc_replay_operands_workspace(P, rows, cols, rank);
}

bool tc_replay_ok(int P, int64_t rows, int64_t cols, int rank, int dtype) {
    return dtype == ZG_BF16 && tc_available() && ((int64_t)P * rank) % 8 == 0 && rows <= 2147483647 &&
           cols <= 2147483647;
}

int tc_replay_run(const float* shaped, const uint32_t* keys, int group, int P, int layout, int64_t rows, int64_t cols,
                  int rank, float inv_sqrt_rank, float* out, Carver& cv, cudaStream_t st) {
    const int64_t q = (int64_t)P * rank;
    __nv_bfloat16* A_op = cv.take<__nv_bfloat16>((size_t)rows * q);
    __nv_bfloat16* B_op = cv.take<__nv_bfloat16>((size_t)cols * q);
    if (!A_op || !B_op) return fail(ZG_ERR_WORKSPACE, "tc replay: workspace too small");
    int rc = factor_operands(keys, group, P, layout, rows, cols, rank, ZG_BF16, A_op, B_op, st);
    if (rc) return rc;
    return tc_replay_factors(shaped, A_op, B_op, P, rows, cols, rank, inv_sqrt_rank, out, cv, st);
}

}  // namespace zg

// ===========================================================================
// C ABI: operand-layout factors, forward and replay from them
// ===========================================================================

extern "C" int zg_factor_operands(const uint32_t* keys, int group, int P, int layout, int64_t rows, int64_t cols,
                                  int rank, int dtype, void* A_op, void* B_op, void* stream) {
    if (P < 1 || P > 65535 || rows < 1 || cols < 1 || rank < 1 || (layout != ZG_MATRIX && layout != ZG_TABLE))
        return zg::fail(ZG_ERR_INVALID, "zg_factor_operands: bad sizes or layout");
    if (!zg::dtype_ok(dtype)) return zg::fail(ZG_ERR_INVALID, "zg_factor_operands: bad dtype");
    if (!keys || (!A_op && !B_op)) return zg::fail(ZG_ERR_INVALID, "zg_factor_operands: null pointer");
    return zg::factor_operands(keys, group, P, layout, rows, cols, rank, dtype, A_op, B_op, zg::as_stream(stream));
}

extern "C" size_t zg_forward_factors_workspace_size(int P, int M, int N, int rank) {
    if (P < 1 || M < 1 || N < 1 || rank < 1) return 0;
    return zg::tc_forward_factors_workspace(P, M, N, rank);
}

extern "C" int zg_forward_factors(const void* x, const void* W, int w_is_kn, const void* F1, const void* F2, int P,
                                  int M, int K, int N, int rank, float s, void* y, void* workspace,
                                  size_t workspace_bytes, void* stream) {
    if (P < 1 || P > 65535 || M < 1 || K < 1 || N < 1 || rank < 1)
        return zg::fail(ZG_ERR_INVALID, "zg_forward_factors: bad sizes");
    if (!x || !W || !F1 || !F2 || !y) return zg::fail(ZG_ERR_INVALID, "zg_forward_factors: null pointer");
    if (!zg::tc_shared_forward_ok(P, M, K, N, rank))
        return zg::fail(ZG_ERR_UNSUPPORTED, "zg_forward_factors: needs sm_100, P*rank, K, N multiples of 8, rank<=32");
    size_t need = zg::tc_forward_factors_workspace(P, M, N, rank);
    if (!workspace || workspace_bytes < need)
        return zg::fail(ZG_ERR_WORKSPACE, "zg_forward_factors: workspace %zu < %zu bytes", workspace_bytes, need);
    zg::Carver cv(workspace, workspace_bytes);
    // W [K, N] (a linear weight) is the MN-major operand; T [N, K] (a tied table) the K-major one.
    return zg::tc_forward_factors(x, W, w_is_kn != 0, w_is_kn ? N : K, F1, F2, P, M, K, N, rank, s, y, cv,
                                  zg::as_stream(stream));
}

extern "C" int zg_forward_factors_ld(const void* x, const void* W, int w_is_kn, const void* F1, int64_t ld1,
                                     const void* F2, int64_t ld2, int P, int M, int K, int N, int rank, float s,
                                     void* y, void* workspace, size_t workspace_bytes, void* stream) {
    if (P < 1 || P > 65535 || M < 1 || K < 1 || N < 1 || rank < 1)
        return zg::fail(ZG_ERR_INVALID, "zg_forward_factors_ld: bad sizes");
    if (!x || !W || !F1 || !F2 || !y) return zg::fail(ZG_ERR_INVALID, "zg_forward_factors_ld: null pointer");
    const int64_t q = (int64_t)P * rank;
    if (ld1 < q || ld2 < q || ld1 % 8 || ld2 % 8)
        return zg::fail(ZG_ERR_INVALID, "zg_forward_factors_ld: leading dimensions must be multiples of 8, >= P*rank");
    if (!zg::tc_shared_forward_ok(P, M, K, N, rank))
        return zg::fail(ZG_ERR_UNSUPPORTED,
                        "zg_forward_factors_ld: needs sm_100, P*rank, K, N multiples of 8, rank<=32");
    size_t need = zg::tc_forward_factors_workspace(P, M, N, rank);
    if (!workspace || workspace_bytes < need)
        return zg::fail(ZG_ERR_WORKSPACE, "zg_forward_factors_ld: workspace %zu < %zu bytes", workspace_bytes, need);
    zg::Carver cv(workspace, workspace_bytes);
    return zg::tc_forward_factors(x, W, w_is_kn != 0, w_is_kn ? N : K, F1, F2, P, M, K, N, rank, s, y, cv,
                                  zg::as_stream(stream), ld1, ld2);
}

extern "C" int zg_forward_operands(const void* x, const void* W, int w_is_kn, const uint32_t* keys, int group, int P,
                                   int M, int K, int N, int rank, float s, void* F1, void* F2, void* y,
                                   void* workspace, size_t workspace_bytes, void* stream) {
    if (P < 1 || P > 65535 || M < 1 || K < 1 || N < 1 || rank < 1)
        return zg::fail(ZG_ERR_INVALID, "zg_forward_operands: bad sizes");
    if (!x || !W || !keys || !F1 || !F2 || !y) return zg::fail(ZG_ERR_INVALID, "zg_forward_operands: null pointer");
    if (!zg::tc_shared_forward_ok(P, M, K, N, rank))
        return zg::fail(ZG_ERR_UNSUPPORTED, "zg_forward_operands: needs sm_100, P*rank, K, N multiples of 8, rank<=32");
    size_t need = zg::tc_forward_factors_workspace(P, M, N, rank);
    if (!workspace || workspace_bytes < need)
        return zg::fail(ZG_ERR_WORKSPACE, "zg_forward_operands: workspace %zu < %zu bytes", workspace_bytes, need);
    zg::Carver cv(workspace, workspace_bytes);
    // linear: F1 = A_op (A, counter k*r + j), F2 = B_op (B, counter j*N + n);
    // tied table: F1 = table B_op (counter c*r + j), F2 = table A_op (counter v*r + j)
    const bool kn = w_is_kn != 0;
    const int64_t q = (int64_t)P * rank;
    return zg::tc_forward_schedule(x, W, kn, kn ? N : K, keys, group, kn ? 0 : 1, 0, kn ? 1 : 0, kn ? 1 : 0, true, F1,
                                   q, F2, q, P, M, K, N, rank, s, y, cv, zg::as_stream(stream));
}

extern "C" size_t zg_replay_factors_workspace_size(int P, int64_t rows, int64_t cols, int rank) {
    if (P < 1 || rows < 1 || cols < 1 || rank < 1) return 0;
    return zg::tc_replay_operands_workspace(P, rows, cols, rank);
}

extern "C" int zg_replay_factors(const float* shaped, const void* A_op, const void* B_op, int P, int64_t rows,
                                 int64_t cols, int rank, float inv_sqrt_rank, float* out, void* workspace,
                                 size_t workspace_bytes, void* stream) {
    if (P < 1 || P > 65535 || rows < 1 || cols < 1 || rank < 1)
        return zg::fail(ZG_ERR_INVALID, "zg_replay_factors: bad sizes");
    if (!shaped || !A_op || !B_op || !out) return zg::fail(ZG_ERR_INVALID, "zg_replay_factors: null pointer");
    if (!zg::tc_replay_ok(P, rows, cols, rank, ZG_BF16))
        return zg::fail(ZG_ERR_UNSUPPORTED, "zg_replay_factors: needs sm_100 and P*rank a multiple of 8");
    size_t need = zg::tc_replay_operands_workspace(P, rows, cols, rank);
    if (!workspace || workspace_bytes < need)
        return zg::fail(ZG_ERR_WORKSPACE, "zg_replay_factors: workspace %zu < %zu bytes", workspace_bytes, need);
    zg::Carver cv(workspace, workspace_bytes);
    return zg::tc_replay_factors(shaped, A_op, B_op, P, rows, cols, rank, inv_sqrt_rank, out, cv,
                                 zg::as_stream(stream));
}

// ===========================================================================
// C ABI: per-candidate-input forward, replay from either factor layout
// ===========================================================================

extern "C" size_t zg_batched_forward_workspace_size(int P, int M, int K, int N, int rank) {
    if (P < 1 || M < 1 || K < 1 || N < 1 || rank < 1) return 0;
    return zg::batched_forward_workspace(P, M, K, N, rank, false);
}

static int batched_args_ok(const char* who, const void* x, const void* W, const void* F1T, const void* F2,
                           const void* y, int P, int M, int K, int N, int rank) {
    if (P < 1 || P > 65535 || M < 1 || K < 1 || N < 1 || rank < 1) return zg::fail(ZG_ERR_INVALID, "%s: bad sizes", who);
    if (!x || !W || !F1T || !F2 || !y) return zg::fail(ZG_ERR_INVALID, "%s: null pointer", who);
    if (!zg::batched_forward_ok(P, M, K, N, rank))
        return zg::fail(ZG_ERR_UNSUPPORTED, "%s: needs sm_100, rank 8 or 16, K and N multiples of 8", who);
    return ZG_OK;
}

extern "C" int zg_batched_forward_factors(const void* x, const void* W, int w_is_kn, const void* F1T, const void* F2,
                                          int P, int M, int K, int N, int rank, float s, void* y, void* workspace,
                                          size_t workspace_bytes, void* stream) {
    int rc = batched_args_ok("zg_batched_forward_factors", x, W, F1T, F2, y, P, M, K, N, rank);
    if (rc) return rc;
    const size_t need = zg::batched_forward_workspace(P, M, K, N, rank, false);
    if (!workspace || workspace_bytes < need)
        return zg::fail(ZG_ERR_WORKSPACE, "zg_batched_forward_factors: workspace %zu < %zu bytes", workspace_bytes,
                        need);
    zg::Carver cv(workspace, workspace_bytes);
    return zg::batched_forward(x, W, w_is_kn != 0, nullptr, 0, 0, 0, 0, false, F1T, F2, P, M, K, N, rank, s, y, cv,
                               zg::as_stream(stream));
}

extern "C" int zg_batched_forward_operands(const void* x, const void* W, int w_is_kn, const uint32_t* keys, int group,
                                           int P, int M, int K, int N, int rank, float s, void* F1T, void* F2,
                                           void* y, void* workspace, size_t workspace_bytes, void* stream) {
    int rc = batched_args_ok("zg_batched_forward_operands", x, W, F1T, F2, y, P, M, K, N, rank);
    if (rc) return rc;
    if (!keys) return zg::fail(ZG_ERR_INVALID, "zg_batched_forward_operands: null keys");
    const size_t need = zg::batched_forward_workspace(P, M, K, N, rank, false);
    if (!workspace || workspace_bytes < need)
        return zg::fail(ZG_ERR_WORKSPACE, "zg_batched_forward_operands: workspace %zu < %zu bytes", workspace_bytes,
                        need);
    zg::Carver cv(workspace, workspace_bytes);
    // linear: F1T = A (counter k*r + j), F2 = B_op (counter j*N + n);
    // tied table: F1T = table B (counter c*r + j), F2 = table A_op (counter v*r + j)
    const bool kn = w_is_kn != 0;
    return zg::batched_forward(x, W, kn, keys, group, kn ? 0 : 1, kn ? 1 : 0, kn ? 1 : 0, true, F1T, F2, P, M, K, N,
                               rank, s, y, cv, zg::as_stream(stream));
}

extern "C" int zg_factor_operands_t(const uint32_t* keys, int group, int P, int layout, int64_t rows, int64_t cols,
                                    int rank, void* F1T, void* F2, int64_t ld2, void* stream) {
    if (P < 1 || P > 65535 || rows < 1 || cols < 1 || (rank != 8 && rank != 16))
        return zg::fail(ZG_ERR_INVALID, "zg_factor_operands_t: bad sizes (rank 8 or 16)");
    if (!keys || !F1T || !F2) return zg::fail(ZG_ERR_INVALID, "zg_factor_operands_t: null pointer");
    if (layout != ZG_MATRIX && layout != ZG_TABLE) return zg::fail(ZG_ERR_INVALID, "zg_factor_operands_t: layout");
    const int64_t q = (int64_t)P * rank;
    if (ld2 != 0 && (ld2 < q || ld2 % 8))
        return zg::fail(ZG_ERR_INVALID, "zg_factor_operands_t: ld2 must be 0 or a multiple of 8 >= P*rank");
    cudaStream_t st = zg::as_stream(stream);
    // MATRIX [K=rows, N=cols]: F1T = A^T [q, rows], F2 = B_op [cols, q] (counter j*cols + n);
    // tied TABLE [V=rows, C=cols]: F1T = B^T [q, cols], F2 = A_op [rows, q] (counter v*r + j)
    const bool mat = layout == ZG_MATRIX;
    int rc = zg::fill_operand_t(keys, group, P, rank, mat ? rows : cols, mat ? 0 : 1, F1T, st, "factor_fill");
    if (!rc)
        rc = zg::fill_operand(keys, group, P, rank, mat ? cols : rows, mat ? 1 : 0, mat ? 1 : 0, nullptr, 1.f, ZG_BF16,
                              F2, st, "factor_fill", ld2);
    return rc;
}

extern "C" int zg_batched_forward_ex(const void* x, const void* W, int w_is_kn, const uint32_t* keys, int group,
                                     int P, int M, int K, int N, int rank, float s, void* F1T, void* F2, int64_t ld2,
                                     int draw, int activation, const void* residual, void* y, void* workspace,
                                     size_t workspace_bytes, void* stream) {
    int rc = batched_args_ok("zg_batched_forward_ex", x, W, F1T, F2, y, P, M, K, N, rank);
    if (rc) return rc;
    if (draw && !keys) return zg::fail(ZG_ERR_INVALID, "zg_batched_forward_ex: null keys");
    if (activation != ZG_ACT_NONE && activation != ZG_ACT_GELU)
        return zg::fail(ZG_ERR_INVALID, "zg_batched_forward_ex: unknown activation %d", activation);
    const int64_t q = (int64_t)P * rank;
    if (ld2 != 0 && (ld2 < q || ld2 % 8))
        return zg::fail(ZG_ERR_INVALID, "zg_batched_forward_ex: ld2 must be 0 or a multiple of 8 >= P*rank");
    if ((reinterpret_cast<uintptr_t>(F2) & 15) || (residual && (reinterpret_cast<uintptr_t>(residual) & 15)))
        return zg::fail(ZG_ERR_INVALID, "zg_batched_forward_ex: F2 and the residual must be 16-byte aligned");
    const size_t need = zg::batched_forward_workspace(P, M, K, N, rank, false);
    if (!workspace || workspace_bytes < need)
        return zg::fail(ZG_ERR_WORKSPACE, "zg_batched_forward_ex: workspace %zu < %zu bytes", workspace_bytes, need);
    zg::Carver cv(workspace, workspace_bytes);
    const bool kn = w_is_kn != 0;
    return zg::batched_forward(x, W, kn, keys, group, kn ? 0 : 1, kn ? 1 : 0, kn ? 1 : 0, draw != 0, F1T, F2, P, M, K,
                               N, rank, s, y, cv, zg::as_stream(stream), ld2, activation, residual);
}

extern "C" size_t zg_replay_operands_workspace_size(int P, int64_t rows, int64_t cols, int rank) {
    if (P < 1 || rows < 1 || cols < 1 || rank < 1) return 0;
    return zg::tc_replay_operands_workspace(P, rows, cols, rank);
}

extern "C" int zg_replay_operands(const float* shaped, const void* A, int a_transposed, const void* B,
                                  int b_transposed, int P, int64_t rows, int64_t cols, int rank, float inv_sqrt_rank,
                                  float* out, void* workspace, size_t workspace_bytes, void* stream) {
    if (P < 1 || P > 65535 || rows < 1 || cols < 1 || rank < 1)
        return zg::fail(ZG_ERR_INVALID, "zg_replay_operands: bad sizes");
    if (!shaped || !A || !B || !out) return zg::fail(ZG_ERR_INVALID, "zg_replay_operands: null pointer");
    if (!zg::tc_replay_ok(P, rows, cols, rank, ZG_BF16))
        return zg::fail(ZG_ERR_UNSUPPORTED, "zg_replay_operands: needs sm_100 and P*rank a multiple of 8");
    size_t need = zg::tc_replay_operands_workspace(P, rows, cols, rank);
    if (!workspace || workspace_bytes < need)
        return zg::fail(ZG_ERR_WORKSPACE, "zg_replay_operands: workspace %zu < %zu bytes", workspace_bytes, need);
    zg::Carver cv(workspace, workspace_bytes);
    return zg::tc_replay_operands(shaped, A, a_transposed != 0, B, b_transposed != 0, P, rows, cols, rank,
                                  inv_sqrt_rank, out, cv, zg::as_stream(stream));
}

// ===========================================================================
// C ABI: replay with the optimizer step fused into its GEMM epilogue
// ===========================================================================

static int replay_step(const char* who, const float* shaped, const void* A, int a_t, const void* B, int b_t, int P,
                       int64_t rows, int64_t cols, int rank, float inv_sqrt_rank, const zg::FusedStep& step,
                       float* descent_out, void* workspace, size_t workspace_bytes, void* stream) {
    if (step.guard && descent_out)
        return zg::fail(ZG_ERR_INVALID, "%s: a guarded step writes no descent", who);
    if (P < 1 || P > 65535 || rows < 1 || cols < 1 || rank < 1) return zg::fail(ZG_ERR_INVALID, "%s: bad sizes", who);
    if (!shaped || !A || !B || !step.param || !step.param_out) return zg::fail(ZG_ERR_INVALID, "%s: null pointer", who);
    if (!zg::tc_replay_ok(P, rows, cols, rank, ZG_BF16))
        return zg::fail(ZG_ERR_UNSUPPORTED, "%s: needs sm_100 and P*rank a multiple of 8", who);
    size_t need = zg::tc_replay_operands_workspace(P, rows, cols, rank);
    if (!workspace || workspace_bytes < need)
        return zg::fail(ZG_ERR_WORKSPACE, "%s: workspace %zu < %zu bytes", who, workspace_bytes, need);
    zg::Carver cv(workspace, workspace_bytes);
    return zg::tc_replay_operands(shaped, A, a_t != 0, B, b_t != 0, P, rows, cols, rank, inv_sqrt_rank, descent_out,
                                  cv, zg::as_stream(stream), &step);
}

extern "C" int zg_replay_sgd(const float* shaped, const void* A, int a_transposed, const void* B, int b_transposed,
                             int P, int64_t rows, int64_t cols, int rank, float inv_sqrt_rank, const void* param,
                             void* param_out, int dtype, double lr, float* descent_out, const float* guard,
                             void* workspace, size_t workspace_bytes, void* stream) {
    if (!zg::dtype_ok(dtype)) return zg::fail(ZG_ERR_INVALID, "zg_replay_sgd: bad dtype");
    zg::FusedStep st{};
    st.kind = zg::ZG_STEP_SGD;
    st.guard = guard;
    st.param_bf16 = dtype == ZG_BF16;
    st.ldp = cols;
    st.param = param;
    st.param_out = param_out;
    st.c.neg_lr = (float)(-lr);
    return replay_step("zg_replay_sgd", shaped, A, a_transposed, B, b_transposed, P, rows, cols, rank, inv_sqrt_rank,
                       st, descent_out, workspace, workspace_bytes, stream);
}

extern "C" int zg_replay_adamw(const float* shaped, const void* A, int a_transposed, const void* B, int b_transposed,
                               int P, int64_t rows, int64_t cols, int rank, float inv_sqrt_rank, const void* param,
                               void* param_out, int dtype, const float* mu, const float* nu, float* mu_out,
                               float* nu_out, int count, double lr, double b1, double b2, double eps,
                               double weight_decay, float* descent_out, const float* guard,
                               const float* bias_corrections, void* workspace, size_t workspace_bytes,
                               void* stream) {
    if (!zg::dtype_ok(dtype)) return zg::fail(ZG_ERR_INVALID, "zg_replay_adamw: bad dtype");
    if (count < 1) return zg::fail(ZG_ERR_INVALID, "zg_replay_adamw: count must be >= 1");
    if (!mu || !nu || !mu_out || !nu_out) return zg::fail(ZG_ERR_INVALID, "zg_replay_adamw: null moment");
    zg::FusedStep st{};
    st.guard = guard;
    st.bc = bias_corrections;
    st.kind = zg::ZG_STEP_ADAMW;
    st.param_bf16 = dtype == ZG_BF16;
    st.ldp = cols;
    st.param = param;
    st.param_out = param_out;
    st.mu = mu;
    st.nu = nu;
    st.mu_out = mu_out;
    st.nu_out = nu_out;
    st.c = zg::adam_consts(count, lr, b1, b2, eps, weight_decay);
    return replay_step("zg_replay_adamw", shaped, A, a_transposed, B, b_transposed, P, rows, cols, rank,
                       inv_sqrt_rank, st, descent_out, workspace, workspace_bytes, stream);
}

// ===========================================================================
// C ABI: the replay split over candidate groups (partials, fixed-order sum)
// ===========================================================================

extern "C" int zg_replay_split_count(int P, int rank) {
    if (P < 1 || rank < 1) return 0;
    return zg::replay_split_count(P, rank);
}

extern "C" size_t zg_replay_partials_workspace_size(int P, int64_t rows, int64_t cols, int rank) {
    if (P < 1 || rows < 1 || cols < 1 || rank < 1) return 0;
    const size_t q = (size_t)P * rank;
    return zg::Carver::need({(size_t)(rows > cols ? rows : cols) * q * 2}) + 256;
}

extern "C" int zg_replay_partials(const float* shaped, const void* A, int a_transposed, const void* B,
                                  int b_transposed, int P, int64_t rows, int64_t cols, int rank, int split_total,
                                  int splits, float* partials, int64_t partial_stride, void* workspace,
                                  size_t workspace_bytes, void* stream) {
    if (P < 1 || P > 65535 || rows < 1 || cols < 1 || rank < 1 || splits < 1 || split_total < splits ||
        split_total > zg::kMaxSplits)
        return zg::fail(ZG_ERR_INVALID, "zg_replay_partials: bad sizes or splits");
    if (!shaped || !A || !B || !partials) return zg::fail(ZG_ERR_INVALID, "zg_replay_partials: null pointer");
    if (!zg::tc_replay_ok(P, rows, cols, rank, ZG_BF16))
        return zg::fail(ZG_ERR_UNSUPPORTED, "zg_replay_partials: needs sm_100 and P*rank a multiple of 8");
    const size_t need = zg_replay_partials_workspace_size(P, rows, cols, rank);
    if (!workspace || workspace_bytes < need)
        return zg::fail(ZG_ERR_WORKSPACE, "zg_replay_partials: workspace %zu < %zu bytes", workspace_bytes, need);
    zg::Carver cv(workspace, workspace_bytes);
    return zg::tc_replay_partials(shaped, A, a_transposed != 0, B, b_transposed != 0, P, rows, cols, rank,
                                  split_total, splits, partials, partial_stride, cv, zg::as_stream(stream));
}

extern "C" int zg_replay_split_sum(const float* partials, const int64_t* offsets, int S, int64_t n, float alpha,
                                   float* out, void* stream) {
    if (!out) return zg::fail(ZG_ERR_INVALID, "zg_replay_split_sum: null output");
    return zg::split_reduce(partials, offsets, S, n, alpha, nullptr, out, zg::as_stream(stream));
}

extern "C" int zg_replay_split_sgd(const float* partials, const int64_t* offsets, int S, int64_t n, float alpha,
                                   const void* param, void* param_out, int dtype, double lr, const float* guard,
                                   void* stream) {
    if (!zg::dtype_ok(dtype)) return zg::fail(ZG_ERR_INVALID, "zg_replay_split_sgd: bad dtype");
    if (!param || !param_out) return zg::fail(ZG_ERR_INVALID, "zg_replay_split_sgd: null parameter");
    zg::FusedStep st{};
    st.kind = zg::ZG_STEP_SGD;
    st.guard = guard;
    st.param_bf16 = dtype == ZG_BF16;
    st.ldp = n;
    st.param = param;
    st.param_out = param_out;
    st.c.neg_lr = (float)(-lr);
    return zg::split_reduce(partials, offsets, S, n, alpha, &st, nullptr, zg::as_stream(stream));
}
