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

}  // namespace

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
