// zg_int8.cu -- integer QAT linear: int8 x int8 -> int32 GEMM with a
// float32 low-rank perturbation and a 256-entry int8 LUT activation.
//
// There is no reference counterpart (the reference only fake-quantises in
// float, examples/train_qat_xor.py:41-50); the semantics are defined by the
// oracle (oracle/zgref.c zgo_int8_lut_linear) and matched bit for bit:
//   acc = x @ W (exact int32)
//   u[m,j] = sequential float32 FMA over k of x[m,k] * A[k,j]
//   lr = sequential FMA over j of u[m,j] * B[j,n]
//   y = fma(float(acc) * x_scale, w_scale[n], s * lr)
//   q = clamp(rint(y / y_scale), -128, 127); out = lut[q + 128]
#include "zg_common.cuh"
#include "zg_tc.cuh"

namespace zg {
int launch_population_factors(const uint32_t* keys, int group, int P, int layout, int64_t rows,
                              int64_t cols, int rank, int dtype, void* A, void* B,
                              cudaStream_t st);
}

namespace {

// u[p,m,j]: one thread per (m, j), sequential k (the oracle's order).
__global__ void int8_u_kernel(const int8_t* __restrict__ x, int x_batched, const float* __restrict__ A,
                              int M, int K, int rank, float* __restrict__ U) {
    const int p = blockIdx.y;
    const int64_t e = blockIdx.x * (int64_t)blockDim.x + threadIdx.x;
    if (e >= (int64_t)M * rank) return;
    const int m = (int)(e / rank), j = (int)(e % rank);
    const int8_t* xr = x + (x_batched ? (int64_t)p * M * K : 0) + (int64_t)m * K;
    const float* a = A + (int64_t)p * K * rank + j;
    float acc = 0.f;
    for (int k = 0; k < K; ++k) acc = __fmaf_rn((float)xr[k], a[(int64_t)k * rank], acc);
    U[((int64_t)p * M + m) * rank + j] = acc;
}

constexpr int BM = 64, BN = 64, BK = 32, THREADS = 256;

// Exact int32 GEMM tile + LUT epilogue.  grid (N/BN, M/BM, P).
__global__ void __launch_bounds__(THREADS)
int8_lut_simt_kernel(const int8_t* __restrict__ x, int x_batched, const int8_t* __restrict__ W,
                     const float* __restrict__ w_scale, float x_scale, float y_scale,
                     const int8_t* __restrict__ lut, const float* __restrict__ U,
                     const float* __restrict__ Bf, int rank, float s, int M, int K, int N,
                     int8_t* __restrict__ out, int32_t* __restrict__ acc_out) {
    __shared__ int Xs[BK][BM + 1];
    __shared__ int Ws[BK][BN + 1];
    __shared__ int8_t slut[256];
    const int p = blockIdx.z;
    const int m0 = blockIdx.y * BM, n0 = blockIdx.x * BN;
    const int tid = threadIdx.x, tx = tid % 16, ty = tid / 16;
    slut[tid] = lut[tid];
    const int8_t* xp = x + (x_batched ? (int64_t)p * M * K : 0);
    int acc[4][4] = {};
    for (int k0 = 0; k0 < K; k0 += BK) {
#pragma unroll
        for (int i = 0; i < (BM * BK) / THREADS; ++i) {
            int e = tid + i * THREADS;
            int kk = e % BK, mm = e / BK;
            int k = k0 + kk, m = m0 + mm;
            Xs[kk][mm] = (k < K && m < M) ? (int)xp[(int64_t)m * K + k] : 0;
        }
#pragma unroll
        for (int i = 0; i < (BN * BK) / THREADS; ++i) {
            int e = tid + i * THREADS;
            int nn = e % BN, kk = e / BN;
            int k = k0 + kk, n = n0 + nn;
            Ws[kk][nn] = (k < K && n < N) ? (int)W[(int64_t)k * N + n] : 0;
        }
        __syncthreads();
#pragma unroll 8
        for (int kk = 0; kk < BK; ++kk) {
#pragma unroll
            for (int i = 0; i < 4; ++i)
#pragma unroll
                for (int j = 0; j < 4; ++j) acc[i][j] += Xs[kk][ty + 16 * i] * Ws[kk][tx + 16 * j];
        }
        __syncthreads();
    }
#pragma unroll
    for (int i = 0; i < 4; ++i) {
        const int m = m0 + ty + 16 * i;
        if (m >= M) continue;
        const float* u = U + ((int64_t)p * M + m) * rank;
#pragma unroll
        for (int j = 0; j < 4; ++j) {
            const int n = n0 + tx + 16 * j;
            if (n >= N) continue;
            const float* b = Bf + (int64_t)p * rank * N + n;
            float lr = 0.f;
            for (int r = 0; r < rank; ++r) lr = __fmaf_rn(u[r], b[(int64_t)r * N], lr);
            const float y = __fmaf_rn(__fmul_rn((float)acc[i][j], x_scale), w_scale[n], __fmul_rn(s, lr));
            const float qf = rintf(__fdiv_rn(y, y_scale));
            const int q = qf > 127.f ? 127 : (qf < -128.f ? -128 : (int)qf);
            const int64_t o = ((int64_t)p * M + m) * N + n;
            out[o] = slut[q + 128];
            if (acc_out) acc_out[o] = acc[i][j];
        }
    }
}

}  // namespace

extern "C" size_t zg_int8_lut_linear_workspace_size(int P, int M, int K, int N, int rank, int x_batched) {
    (void)x_batched;
    if (P < 1 || M < 1 || K < 1 || N < 1 || rank < 1) return 0;
    return zg::Carver::need({(size_t)P * K * rank * 4, (size_t)P * rank * N * 4, (size_t)P * M * rank * 4});
}

extern "C" int zg_int8_lut_linear(const int8_t* x, int x_batched, const int8_t* W, const float* w_scale,
                                  float x_scale, float y_scale, const int8_t* lut, const uint32_t* keys,
                                  int group, int P, int M, int K, int N, int rank, float s, int8_t* out,
                                  int32_t* acc_out, void* workspace, size_t workspace_bytes, void* stream) {
    if (P < 1 || P > 65535 || M < 1 || K < 1 || N < 1 || rank < 1 || rank > 64)
        return zg::fail(ZG_ERR_INVALID, "zg_int8_lut_linear: bad sizes");
    if (!x || !W || !w_scale || !lut || !keys || !out)
        return zg::fail(ZG_ERR_INVALID, "zg_int8_lut_linear: null pointer");
    if (!(y_scale > 0.f)) return zg::fail(ZG_ERR_INVALID, "zg_int8_lut_linear: y_scale must be positive");
    size_t need = zg_int8_lut_linear_workspace_size(P, M, K, N, rank, x_batched);
    if (!workspace || workspace_bytes < need)
        return zg::fail(ZG_ERR_WORKSPACE, "zg_int8_lut_linear: workspace %zu < %zu bytes", workspace_bytes, need);
    cudaStream_t st = zg::as_stream(stream);
    zg::Carver cv(workspace, workspace_bytes);
    float* fa = cv.take<float>((size_t)P * K * rank);
    float* fb = cv.take<float>((size_t)P * rank * N);
    float* U = cv.take<float>((size_t)P * M * rank);
    int rc = zg::launch_population_factors(keys, group, P, ZG_MATRIX, K, N, rank, ZG_F32, fa, fb, st);
    if (rc) return rc;
    {
        int64_t n = (int64_t)M * rank;
        dim3 grid((unsigned)((n + 127) / 128), P);
        zg::LaunchTimer zg_lt_("int8_u", st);
        int8_u_kernel<<<grid, 128, 0, st>>>(x, x_batched, fa, M, K, rank, U);
        if ((rc = zg::check_launch("int8_u"))) return rc;
    }
    dim3 grid((N + BN - 1) / BN, (M + BM - 1) / BM, P);
    zg::LaunchTimer zg_lt_("int8_lut_gemm", st);
    int8_lut_simt_kernel<<<grid, THREADS, 0, st>>>(x, x_batched, W, w_scale, x_scale, y_scale, lut, U, fb, rank,
                                                   s, M, K, N, out, acc_out);
    return zg::check_launch("zg_int8_lut_linear");
}
