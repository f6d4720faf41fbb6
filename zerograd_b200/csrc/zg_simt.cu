// zg_simt.cu -- CUDA-core GEMM with two-level K and low-rank epilogue.
#include "zg_simt.cuh"

namespace zg {
namespace {

constexpr int BM = 64, BN = 64, BK = 16, THREADS = 256;

template <typename T, typename TO>
__global__ void __launch_bounds__(THREADS) simt_gemm_kernel(const SimtGemm g) {
    __shared__ float As[BK][BM + 4];
    __shared__ float Bs[BK][BN + 4];
    const int b = blockIdx.z;
    const int m0 = blockIdx.y * BM, n0 = blockIdx.x * BN;
    const int tid = threadIdx.x;
    const int tx = tid % 16, ty = tid / 16;
    const T* A = static_cast<const T*>(g.A);
    const T* B = static_cast<const T*>(g.B);
    float acc[4][4] = {};
    const int64_t Ktot = (int64_t)g.Ko * g.Ki;
    for (int64_t k0 = 0; k0 < Ktot; k0 += BK) {
        // A tile: BM x BK (k fastest across threads when A is K-contiguous)
#pragma unroll
        for (int i = 0; i < (BM * BK) / THREADS; ++i) {
            int e = tid + i * THREADS;
            int kk = e % BK, mm = e / BK;
            int64_t k = k0 + kk;
            int m = m0 + mm;
            float v = 0.f;
            if (k < Ktot && m < g.M) {
                int64_t ko = k / g.Ki, ki = k - ko * g.Ki;
                v = zg_to_float(A[b * g.sAb + m * g.sAm + ko * g.sAko + ki * g.sAki]);
                if (g.kscale) v *= g.kscale[ko];
            }
            As[kk][mm] = v;
        }
#pragma unroll
        for (int i = 0; i < (BN * BK) / THREADS; ++i) {
            int e = tid + i * THREADS;
            int nn = e % BN, kk = e / BN;
            int64_t k = k0 + kk;
            int n = n0 + nn;
            float v = 0.f;
            if (k < Ktot && n < g.N) {
                int64_t ko = k / g.Ki, ki = k - ko * g.Ki;
                v = zg_to_float(B[b * g.sBb + ko * g.sBko + ki * g.sBki + n * g.sBn]);
            }
            Bs[kk][nn] = v;
        }
        __syncthreads();
#pragma unroll
        for (int kk = 0; kk < BK; ++kk) {
            float a[4], bb[4];
#pragma unroll
            for (int i = 0; i < 4; ++i) a[i] = As[kk][ty + 16 * i];
#pragma unroll
            for (int j = 0; j < 4; ++j) bb[j] = Bs[kk][tx + 16 * j];
#pragma unroll
            for (int i = 0; i < 4; ++i)
#pragma unroll
                for (int j = 0; j < 4; ++j) acc[i][j] = fmaf(a[i], bb[j], acc[i][j]);
        }
        __syncthreads();
    }
    const T* L = static_cast<const T*>(g.L);
    TO* C = static_cast<TO*>(g.C);
#pragma unroll
    for (int i = 0; i < 4; ++i) {
        int m = m0 + ty + 16 * i;
        if (m >= g.M) continue;
#pragma unroll
        for (int j = 0; j < 4; ++j) {
            int n = n0 + tx + 16 * j;
            if (n >= g.N) continue;
            float v = g.alpha * acc[i][j];
            if (g.Cin) v += g.Cin[b * g.sCinb + m * g.sCinm + n * g.sCinn];
            if (g.U) {
                float lr = 0.f;
                const float* u = g.U + b * g.sUb + m * g.sUm;
                const T* l = L + b * g.sLb + n * g.sLn;
                for (int r = 0; r < g.rank; ++r) lr = fmaf(u[r * g.sUj], zg_to_float(l[r * g.sLj]), lr);
                v = fmaf(g.lr_s, lr, v);
            }
            C[b * g.sCb + (int64_t)m * g.sCm + (int64_t)n * g.sCn] = zg_from_float<TO>(v);
        }
    }
}

// ---- float32 NT replay GEMM ----
constexpr int RS_BM = 128, RS_BN = 128, RS_BK = 16, RS_PAD = 4;

__device__ __forceinline__ float2 fma_f32x2(float2 a, float2 b, float2 c) {
    unsigned long long A = *reinterpret_cast<unsigned long long*>(&a), B = *reinterpret_cast<unsigned long long*>(&b),
                       C = *reinterpret_cast<unsigned long long*>(&c), D;
    asm("fma.rn.f32x2 %0, %1, %2, %3;" : "=l"(D) : "l"(A), "l"(B), "l"(C));
    return *reinterpret_cast<float2*>(&D);
}

__global__ void __launch_bounds__(256, 2) replay_sgemm_kernel(const float* __restrict__ A, const float* __restrict__ B,
                                                           const float* __restrict__ w, int rank, int M, int N,
                                                           int64_t K, float alpha, float* __restrict__ C) {
    __shared__ __align__(16) float As[RS_BK][RS_BM + RS_PAD];
    __shared__ __align__(16) float Bs[RS_BK][RS_BN + RS_PAD];
    const int tid = threadIdx.x, tx = tid % 16, ty = tid / 16;
    const int m0 = blockIdx.y * RS_BM, n0 = blockIdx.x * RS_BN;
    // staging: thread -> (row lr = tid / 4 + 64 i, k chunk kc = tid % 4) for i = 0, 1
    const int lr = tid / 4, kc = (tid % 4) * 4;
    float4 ra[2], rb[2];
    auto fetch = [&](int64_t k0) {
#pragma unroll
        for (int i = 0; i < 2; ++i) {
            const int m = m0 + lr + 64 * i, n = n0 + lr + 64 * i;
            const int64_t k = k0 + kc;
            ra[i] = make_float4(0.f, 0.f, 0.f, 0.f);
            rb[i] = make_float4(0.f, 0.f, 0.f, 0.f);
            if (k < K) {  // K % 4 == 0: a chunk is all in or all out
                if (m < M) {
                    ra[i] = *reinterpret_cast<const float4*>(A + (int64_t)m * K + k);
                    const int64_t q = k / rank;  // the fitness weight of each contraction column
                    if (rank % 4 == 0) {
                        const float wq = w[q];
                        ra[i].x *= wq; ra[i].y *= wq; ra[i].z *= wq; ra[i].w *= wq;
                    } else {
                        ra[i].x *= w[k / rank]; ra[i].y *= w[(k + 1) / rank];
                        ra[i].z *= w[(k + 2) / rank]; ra[i].w *= w[(k + 3) / rank];
                    }
                }
                if (n < N) rb[i] = *reinterpret_cast<const float4*>(B + (int64_t)n * K + k);
            }
        }
    };
    auto stash = [&]() {
#pragma unroll
        for (int i = 0; i < 2; ++i) {
            const int r = lr + 64 * i;
            As[kc][r] = ra[i].x; As[kc + 1][r] = ra[i].y; As[kc + 2][r] = ra[i].z; As[kc + 3][r] = ra[i].w;
            Bs[kc][r] = rb[i].x; Bs[kc + 1][r] = rb[i].y; Bs[kc + 2][r] = rb[i].z; Bs[kc + 3][r] = rb[i].w;
        }
    };
    // acc[i][jj]: outputs (i, 2 jj) and (i, 2 jj + 1), a register pair for
    // the packed float32x2 FMA
    float2 acc[8][4];
#pragma unroll
    for (int i = 0; i < 8; ++i)
#pragma unroll
        for (int jj = 0; jj < 4; ++jj) acc[i][jj] = make_float2(0.f, 0.f);
    fetch(0);
    for (int64_t k0 = 0; k0 < K; k0 += RS_BK) {
        __syncthreads();  // the previous tile's reads are done
        stash();
        __syncthreads();
        if (k0 + RS_BK < K) fetch(k0 + RS_BK);  // in flight during this tile's products
#pragma unroll
        for (int kk = 0; kk < RS_BK; ++kk) {
            const float4 a0 = *reinterpret_cast<const float4*>(&As[kk][ty * 4]);
            const float4 a1 = *reinterpret_cast<const float4*>(&As[kk][64 + ty * 4]);
            const float4 b0 = *reinterpret_cast<const float4*>(&Bs[kk][tx * 4]);
            const float4 b1 = *reinterpret_cast<const float4*>(&Bs[kk][64 + tx * 4]);
            const float a[8] = {a0.x, a0.y, a0.z, a0.w, a1.x, a1.y, a1.z, a1.w};
            const float2 b[4] = {make_float2(b0.x, b0.y), make_float2(b0.z, b0.w), make_float2(b1.x, b1.y),
                                 make_float2(b1.z, b1.w)};
            // two adjacent outputs per packed float32x2 FMA (each lane an
            // IEEE fma: the same value and order as one fmaf per output)
#pragma unroll
            for (int i = 0; i < 8; ++i) {
                const float2 ai = make_float2(a[i], a[i]);
#pragma unroll
                for (int jj = 0; jj < 4; ++jj) acc[i][jj] = fma_f32x2(ai, b[jj], acc[i][jj]);
            }
        }
    }
#pragma unroll
    for (int i = 0; i < 8; ++i) {
        const int m = m0 + (i < 4 ? ty * 4 + i : 64 + ty * 4 + i - 4);
        if (m >= M) continue;
#pragma unroll
        for (int h = 0; h < 2; ++h) {
            const int n = n0 + h * 64 + tx * 4;
            float* c = C + (int64_t)m * N + n;
            const float v0 = alpha * acc[i][2 * h].x, v1 = alpha * acc[i][2 * h].y, v2 = alpha * acc[i][2 * h + 1].x,
                        v3 = alpha * acc[i][2 * h + 1].y;
            if (n + 4 <= N && (N % 4) == 0) {
                *reinterpret_cast<float4*>(c) = make_float4(v0, v1, v2, v3);
            } else {
                if (n < N) c[0] = v0;
                if (n + 1 < N) c[1] = v1;
                if (n + 2 < N) c[2] = v2;
                if (n + 3 < N) c[3] = v3;
            }
        }
    }
}

}  // namespace

int launch_replay_sgemm(const float* A, const float* B, const float* w, int rank, int M, int N, int64_t K, float alpha,
                        float* C, cudaStream_t st, const char* name) {
    if (M <= 0 || N <= 0) return ZG_OK;
    if (K % 4 || rank < 1) return fail(ZG_ERR_INVALID, "replay sgemm: K %% 4 == 0 required");
    auto al = [](const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15) == 0; };
    if (!al(A) || !al(B) || !al(C)) return fail(ZG_ERR_INVALID, "replay sgemm: operands must be 16-byte aligned");
    const int64_t gy = (M + RS_BM - 1) / RS_BM;
    if (gy > 65535) return fail(ZG_ERR_INVALID, "replay sgemm: M too large");
    dim3 grid((unsigned)((N + RS_BN - 1) / RS_BN), (unsigned)gy);
    zg::LaunchTimer zg_lt_(name, st);
    replay_sgemm_kernel<<<grid, 256, 0, st>>>(A, B, w, rank, M, N, K, alpha, C);
    return check_launch("replay_sgemm");
}

template <typename T, typename TO>
int launch_simt_gemm(const SimtGemm& g, cudaStream_t st, const char* name) {
    if (g.M <= 0 || g.N <= 0 || g.batch <= 0) return ZG_OK;
    if (g.batch > 65535) return fail(ZG_ERR_INVALID, "simt gemm: batch %d > 65535", g.batch);
    dim3 grid((g.N + BN - 1) / BN, (g.M + BM - 1) / BM, g.batch);
    if (grid.y > 65535) return fail(ZG_ERR_INVALID, "simt gemm: M too large");
    zg::LaunchTimer zg_lt_(name, st);
    simt_gemm_kernel<T, TO><<<grid, THREADS, 0, st>>>(g);
    return check_launch("simt_gemm");
}

template int launch_simt_gemm<float, float>(const SimtGemm&, cudaStream_t, const char*);
template int launch_simt_gemm<__nv_bfloat16, float>(const SimtGemm&, cudaStream_t, const char*);
template int launch_simt_gemm<__nv_bfloat16, __nv_bfloat16>(const SimtGemm&, cudaStream_t, const char*);

}  // namespace zg
