// zg_ops.cu -- population-batched forward ops, fitness shaping, replay and
// fused optimizer updates (C ABI in include/zg_b200.h).
//
// Reference behaviour restated (paths relative to the reference root):
//   perturbed_linear / table_lookup / tied_logits / vector
//                                    src/zerograd/_candidate.py:17-45
//   shape_centered_loss, validate_losses  src/zerograd/_fitness.py:13-48
//   replay_entry                     src/zerograd/_replay.py:15-54
//   _build_pseudo_grad + optax update + apply_updates
//                                    src/zerograd/_optimizer.py:229-234,299-326
#include <cmath>

#include "zg_simt.cuh"
#include "zg_tc.cuh"
#include "zg_update.cuh"

namespace zg {
int launch_population_factors(const uint32_t* keys, int group, int P, int layout, int64_t rows,
                              int64_t cols, int rank, int dtype, void* A, void* B,
                              cudaStream_t st);
int factor_operands(const uint32_t* keys, int group, int P, int layout, int64_t rows, int64_t cols, int rank,
                    int dtype, void* A_op, void* B_op, cudaStream_t st);
}

namespace {

using zg::Carver;
using zg::SimtGemm;

template <typename T, typename TO>
int simt(const SimtGemm& g, cudaStream_t st, const char* name) {
    return zg::launch_simt_gemm<T, TO>(g, st, name);
}

// ---------------------------------------------------------------------------
// perturbed linear / tied logits share one plan:
//   y[p] = x_p @ Wop + s * (x_p @ F1_p) @ F2_p
// linear: Wop = W [K,N] (row-major), F1 = A_p [K,r], F2 = B_p [r,N]
// tied:   Wop = T^T (T [V,C]),       F1 = B_p [C,r], F2 = A_p^T
// ---------------------------------------------------------------------------
struct LowRankPlan {
    int P, M, K, N, rank, dtype, x_batched;
    const void* x;
    const void* Wop;
    int64_t sWk, sWn;          // strides of Wop(k, n)
    const void* F1;            // [P, K, r] contiguous: F1(k, j) at p*K*r + k*r + j
    const void* F2;            // L(j, n) strides within a candidate
    int64_t sF2b, sF2j, sF2n;
    float s;
    void* y;
    float* U;                  // [P, M, r] f32 scratch
    float* XW;                 // [M, N] f32 scratch (shared x only)
};

template <typename T>
int run_low_rank(const LowRankPlan& q, cudaStream_t st) {
    int rc;
    // U[p] = x_p @ F1_p
    {
        SimtGemm g;
        g.A = q.x; g.sAb = q.x_batched ? (int64_t)q.M * q.K : 0; g.sAm = q.K; g.sAko = 0; g.sAki = 1;
        g.B = q.F1; g.sBb = (int64_t)q.K * q.rank; g.sBko = 0; g.sBki = q.rank; g.sBn = 1;
        g.C = q.U; g.sCb = (int64_t)q.M * q.rank; g.sCm = q.rank; g.sCn = 1;
        g.M = q.M; g.N = q.rank; g.Ko = 1; g.Ki = q.K; g.batch = q.P;
        if ((rc = simt<T, float>(g, st, "lowrank_u"))) return rc;
    }
    SimtGemm g;
    g.U = q.U; g.sUb = (int64_t)q.M * q.rank; g.sUm = q.rank; g.sUj = 1;
    g.L = q.F2; g.sLb = q.sF2b; g.sLj = q.sF2j; g.sLn = q.sF2n;
    g.rank = q.rank; g.lr_s = q.s;
    g.C = q.y; g.sCb = (int64_t)q.M * q.N; g.sCm = q.N; g.sCn = 1;
    g.M = q.M; g.N = q.N; g.batch = q.P;
    if (!q.x_batched) {
        // The shared product x @ Wop is computed once (as jax.vmap leaves an
        // unbatched x @ W unbatched) and broadcast into every candidate.
        SimtGemm d;
        d.A = q.x; d.sAm = q.K; d.sAki = 1;
        d.B = q.Wop; d.sBki = q.sWk; d.sBn = q.sWn;
        d.C = q.XW; d.sCm = q.N; d.sCn = 1;
        d.M = q.M; d.N = q.N; d.Ko = 1; d.Ki = q.K; d.batch = 1;
        if ((rc = simt<T, float>(d, st, "shared_xw"))) return rc;
        g.Cin = q.XW; g.sCinb = 0; g.sCinm = q.N; g.sCinn = 1;
        g.Ko = 0; g.Ki = 0;
    } else {
        g.A = q.x; g.sAb = (int64_t)q.M * q.K; g.sAm = q.K; g.sAki = 1;
        g.B = q.Wop; g.sBb = 0; g.sBki = q.sWk; g.sBn = q.sWn;
        g.Ko = 1; g.Ki = q.K;
    }
    return simt<T, T>(g, st, q.x_batched ? "perturbed_gemm" : "lowrank_expand");
}

size_t low_rank_ws(int P, int M, int K, int N, int rank, int dtype, int x_batched, int64_t f1,
                   int64_t f2) {
    size_t es = zg::dtype_size(dtype);
    return Carver::need({(size_t)P * f1 * es, (size_t)P * f2 * es, (size_t)P * M * rank * 4,
                         x_batched ? 0 : (size_t)M * N * 4});
}

bool dims_ok(std::initializer_list<int64_t> v) {
    for (int64_t d : v)
        if (d < 1) return false;
    return true;
}

// ---------------------------------------------------------------------------
// table lookup: out[p,t,c] = T[row,c] + s * sum_j A_p[row,j] * B_p[c,j]
// A rows regenerated in-kernel; B_p from the factor fill.  grid (n_idx, P).
// ---------------------------------------------------------------------------
template <typename T>
__global__ void table_lookup_kernel(const T* __restrict__ table, const int32_t* __restrict__ idx,
                                    int idx_batched, int64_t n_idx, const uint32_t* __restrict__ keys,
                                    int group, int64_t rows, int64_t cols, int rank, float s,
                                    const T* __restrict__ Bf, T* __restrict__ out) {
    extern __shared__ float a_row[];
    const int64_t t = blockIdx.x;
    const int p = blockIdx.y;
    int64_t row = idx[(idx_batched ? (int64_t)p * n_idx : 0) + t];
    if (row < 0) row += rows;                    // numpy-style negative index
    row = row < 0 ? 0 : (row >= rows ? rows - 1 : row);  // jnp gather clamps
    if (threadIdx.x < rank) {
        ZgFactorKeys fk = zg_factor_keys(keys, p, group);
        a_row[threadIdx.x] = zg_dtype_round<T>(zg_normal(fk.a, (uint64_t)row * rank + threadIdx.x));
    }
    __syncthreads();
    const T* bp = Bf + (int64_t)p * cols * rank;
    T* o = out + ((int64_t)p * n_idx + t) * cols;
    const T* trow = table + row * cols;
    for (int64_t c = threadIdx.x; c < cols; c += blockDim.x) {
        float lr = 0.f;
        for (int j = 0; j < rank; ++j) lr = fmaf(a_row[j], zg_to_float(bp[c * rank + j]), lr);
        o[c] = zg_from_float<T>(fmaf(s, lr, zg_to_float(trow[c])));
    }
}

// Rank 8 or 16: a block takes 32 gathered tokens of one candidate, draws
// their A rows into shared memory once, and each thread keeps its column's
// B row in registers across the 32 tokens (the same arithmetic, in the same
// order, as table_lookup_kernel).
template <typename T, int R>
__global__ void table_lookup_tiled_kernel(const T* __restrict__ table, const int32_t* __restrict__ idx,
                                          int idx_batched, int64_t n_idx, const uint32_t* __restrict__ keys,
                                          int group, int64_t rows, int64_t cols, float s, const T* __restrict__ Bf,
                                          T* __restrict__ out) {
    constexpr int TB = 32;
    __shared__ __align__(16) float a_s[TB][R];
    __shared__ int64_t row_s[TB];
    const int p = blockIdx.y;
    const int64_t t0 = (int64_t)blockIdx.x * TB;
    const int nt = n_idx - t0 < TB ? (int)(n_idx - t0) : TB;
    if ((int)threadIdx.x < nt) {
        int64_t row = idx[(idx_batched ? (int64_t)p * n_idx : 0) + t0 + threadIdx.x];
        if (row < 0) row += rows;
        row_s[threadIdx.x] = row < 0 ? 0 : (row >= rows ? rows - 1 : row);
    }
    __syncthreads();
    if ((int)threadIdx.x < nt * R) {
        const ZgFactorKeys fk = zg_factor_keys(keys, p, group);
        for (int i = threadIdx.x; i < nt * R; i += blockDim.x)
            a_s[i / R][i % R] = zg_dtype_round<T>(zg_normal(fk.a, (uint64_t)row_s[i / R] * R + i % R));
    }
    __syncthreads();
    const T* bp = Bf + (int64_t)p * cols * R;
    T* ob = out + ((int64_t)p * n_idx + t0) * cols;
    for (int64_t c = threadIdx.x; c < cols; c += blockDim.x) {
        float b[R];
#pragma unroll
        for (int j = 0; j < R; ++j) b[j] = zg_to_float(bp[c * R + j]);
        for (int tt = 0; tt < nt; ++tt) {
            // the token's A row as 16-byte shared loads (the same value in every lane)
            float a[R];
#pragma unroll
            for (int j = 0; j < R; j += 4) {
                const float4 q = *reinterpret_cast<const float4*>(&a_s[tt][j]);
                a[j] = q.x; a[j + 1] = q.y; a[j + 2] = q.z; a[j + 3] = q.w;
            }
            float lr = 0.f;
#pragma unroll
            for (int j = 0; j < R; ++j) lr = fmaf(a[j], b[j], lr);
            ob[(int64_t)tt * cols + c] = zg_from_float<T>(fmaf(s, lr, zg_to_float(table[row_s[tt] * cols + c])));
        }
    }
}

// Tensor-core lookup (bf16, ids shared by the candidates): the gathered
// table rows once as float32 [n, cols] (the expansion's shared addend) and
// the candidates' A rows at the gathered ids in the expansion's operand
// layout U [n, P R]; then y = bf16(T[idx] + s U_p B_p^T) with one K = 16
// MMA per candidate and tile (tc_expand), so the kernel is bound by its
// output writes.  Ids wrap and clamp as in table_lookup_kernel.
__device__ __forceinline__ int64_t lookup_row(const int32_t* idx, int64_t t, int64_t rows) {
    int64_t row = idx[t];
    if (row < 0) row += rows;
    return row < 0 ? 0 : (row >= rows ? rows - 1 : row);
}

__global__ void gather_rows_f32_kernel(const __nv_bfloat16* __restrict__ T, const int32_t* __restrict__ idx, int64_t n,
                                       int64_t rows, int64_t cols, float* __restrict__ out) {
    const int64_t g8 = cols / 8;
    const int64_t stride = (int64_t)gridDim.x * blockDim.x;
    for (int64_t e = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; e < n * g8; e += stride) {
        const int64_t t = e / g8, c = (e % g8) * 8;
        float f[8];
        bf16x8_to_f32(*reinterpret_cast<const uint4*>(T + lookup_row(idx, t, rows) * cols + c), f);
        float4* o = reinterpret_cast<float4*>(out + t * cols + c);
        o[0] = make_float4(f[0], f[1], f[2], f[3]);
        o[1] = make_float4(f[4], f[5], f[6], f[7]);
    }
}

// U[t, p R + j] = bf16(normal(A key of candidate p, idx_t R + j)): the
// values table_lookup_kernel draws for the same rows.
template <int R>
__global__ void gather_a_rows_kernel(const uint32_t* __restrict__ keys, int group, int P,
                                     const int32_t* __restrict__ idx, int64_t n, int64_t rows,
                                     __nv_bfloat16* __restrict__ U) {
    const int64_t stride = (int64_t)gridDim.x * blockDim.x;
    for (int64_t e = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; e < n * P; e += stride) {
        const int64_t t = e / P;
        const int p = (int)(e % P);
        const uint64_t c0 = (uint64_t)lookup_row(idx, t, rows) * R;
        const ZgFactorKeys fk = zg_factor_keys(keys, p, group);
        uint4 o[R / 8];
        __nv_bfloat16* h = reinterpret_cast<__nv_bfloat16*>(o);
#pragma unroll
        for (int j = 0; j < R; ++j) h[j] = __float2bfloat16_rn(zg_normal(fk.a, c0 + j));
        uint4* dst = reinterpret_cast<uint4*>(U + t * ((int64_t)P * R) + (int64_t)p * R);
#pragma unroll
        for (int i = 0; i < R / 8; ++i) dst[i] = o[i];
    }
}

int sm_count_ops() {
    static int n = 0;
    if (n == 0) {
        int dev = 0;
        cudaGetDevice(&dev);
        if (cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess || n < 1) n = 148;
    }
    return n;
}

inline bool lookup_tc_ok(int P, int64_t n_idx, int64_t cols, int rank, int dtype, int idx_batched, const void* T,
                         const void* out) {
    auto al = [](const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15) == 0; };
    return dtype == ZG_BF16 && !idx_batched && (rank == 8 || rank == 16) && cols % 8 == 0 && n_idx >= 1 &&
           n_idx <= 2147483647 && cols <= 2147483647 && zg::tc_available() && al(T) && al(out);
}

// ---------------------------------------------------------------------------
// vector: out[p,i] = v[i] + s * noise_p[i], with the reference's per-op
// rounding to the leaf dtype (product, then sum).
// ---------------------------------------------------------------------------
template <typename T>
__global__ void vector_kernel(const T* __restrict__ v, int v_batched, const uint32_t* __restrict__ keys,
                              int group, int64_t n, float s, T* __restrict__ out) {
    const int p = blockIdx.y;
    ZgKey gk = zg_group_key(keys, p, group);
    const T* vp = v + (v_batched ? (int64_t)p * n : 0);
    for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < n;
         i += (int64_t)gridDim.x * blockDim.x) {
        float noise = zg_dtype_round<T>(zg_normal(gk, (uint64_t)i));
        float prod = zg_dtype_round<T>(__fmul_rn(s, noise));
        out[(int64_t)p * n + i] = zg_from_float<T>(__fadd_rn(zg_to_float(vp[i]), prod));
    }
}

// ---------------------------------------------------------------------------
// fitness shaping + validation + metrics (one block)
// ---------------------------------------------------------------------------
__global__ void shape_fitness_kernel(const float* __restrict__ losses, int P, float denom,
                                     float* __restrict__ shaped, float* __restrict__ metrics) {
    __shared__ double s_sum[32];
    __shared__ float s_min[32], s_max[32];
    __shared__ int s_bad[32];
    __shared__ float s_mean;
    double sum = 0.0;
    float mn = INFINITY, mx = -INFINITY;
    int bad = 0;
    for (int i = threadIdx.x; i < P; i += blockDim.x) {
        float l = losses[i];
        if (!isfinite(l)) ++bad;
        sum += (double)l;
        mn = fminf(mn, l);
        mx = fmaxf(mx, l);
    }
    for (int o = 16; o > 0; o >>= 1) {
        sum += __shfl_xor_sync(0xffffffffu, sum, o);
        mn = fminf(mn, __shfl_xor_sync(0xffffffffu, mn, o));
        mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, o));
        bad += __shfl_xor_sync(0xffffffffu, bad, o);
    }
    const int w = threadIdx.x / 32, lane = threadIdx.x % 32;
    if (lane == 0) { s_sum[w] = sum; s_min[w] = mn; s_max[w] = mx; s_bad[w] = bad; }
    __syncthreads();
    if (threadIdx.x == 0) {
        double tsum = 0.0;
        float tmn = INFINITY, tmx = -INFINITY;
        int tbad = 0;
        for (int i = 0; i < (int)(blockDim.x + 31) / 32; ++i) {
            tsum += s_sum[i]; tmn = fminf(tmn, s_min[i]); tmx = fmaxf(tmx, s_max[i]); tbad += s_bad[i];
        }
        float mean = (float)(tsum / (double)P);
        s_mean = mean;
        metrics[0] = mean; metrics[1] = tmn; metrics[2] = tmx; metrics[3] = (float)tbad;
    }
    __syncthreads();
    const float mean = s_mean;
    for (int i = threadIdx.x; i < P; i += blockDim.x)
        shaped[i] = __fdiv_rn(-__fsub_rn(losses[i], mean), denom);
}

// ---------------------------------------------------------------------------
// VECTOR replay: out[i] = sum_p w_p * noise_p[i] (noise regenerated).
// Candidates are split into slices of VR_SLICE; block (column tile, slice)
// writes the slice's partial sums, and a second pass adds the slices in
// order.  The split depends only on (P, n), so the result does too.
// ---------------------------------------------------------------------------
constexpr int VR_SLICE = 32, VR_COLS = 128;

inline int vector_replay_slices(int P) { return (P + VR_SLICE - 1) / VR_SLICE; }

template <typename T>
__global__ void vector_replay_partial_kernel(const float* __restrict__ w, const uint32_t* __restrict__ keys, int group,
                                             int P, int64_t n, float* __restrict__ partial) {
    __shared__ uint32_t sk[VR_SLICE][2];
    __shared__ float sw[VR_SLICE];
    const int64_t i = blockIdx.x * (int64_t)VR_COLS + threadIdx.x;
    const int p0 = blockIdx.y * VR_SLICE;
    const int cnt = min(VR_SLICE, P - p0);
    if ((int)threadIdx.x < cnt) {
        const ZgKey gk = zg_group_key(keys, p0 + threadIdx.x, group);
        sk[threadIdx.x][0] = gk.k0;
        sk[threadIdx.x][1] = gk.k1;
        sw[threadIdx.x] = w[p0 + threadIdx.x];
    }
    __syncthreads();
    if (i >= n) return;
    float acc = 0.f;
    for (int q = 0; q < cnt; ++q) {
        const ZgKey gk = zg_make_key(sk[q][0], sk[q][1]);
        acc = fmaf(zg_dtype_round<T>(zg_normal(gk, (uint64_t)i)), sw[q], acc);
    }
    partial[(int64_t)blockIdx.y * n + i] = acc;
}

__global__ void vector_replay_sum_kernel(const float* __restrict__ partial, int slices, int64_t n,
                                         float* __restrict__ out) {
    const int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x;
    if (i >= n) return;
    float acc = 0.f;
    for (int s = 0; s < slices; ++s) acc += partial[(int64_t)s * n + i];
    out[i] = acc;
}

// ---------------------------------------------------------------------------
// fused optimizer updates
// ---------------------------------------------------------------------------
template <typename T>
__global__ void adamw_kernel(const T* __restrict__ param, T* __restrict__ param_out,
                             const float* __restrict__ descent, const float* __restrict__ mu,
                             const float* __restrict__ nu, float* __restrict__ mu_out,
                             float* __restrict__ nu_out, int64_t n, zg::AdamConsts c0,
                             const float* __restrict__ bc) {
    const zg::AdamConsts c = zg::adam_consts_dev(c0, bc);
    for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < n;
         i += (int64_t)gridDim.x * blockDim.x) {
        const float g = descent ? -descent[i] : 0.f;  // pseudo_grad = -descent
        float m, v;
        const float pn = zg::adamw_step(zg_to_float(param[i]), g, mu[i], nu[i], c, m, v);
        mu_out[i] = m;
        nu_out[i] = v;
        param_out[i] = zg_from_float<T>(pn);
    }
}

template <typename T>
__global__ void sgd_kernel(const T* __restrict__ param, T* __restrict__ param_out,
                           const float* __restrict__ descent, int64_t n, float neg_lr) {
    for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < n;
         i += (int64_t)gridDim.x * blockDim.x) {
        const float g = descent ? -descent[i] : 0.f;
        param_out[i] = zg_from_float<T>(zg::sgd_step(zg_to_float(param[i]), g, neg_lr));
    }
}

int ew_grid(int64_t n) {
    int64_t g = (n + 255) / 256;
    return (int)(g < 148 * 8 ? (g < 1 ? 1 : g) : 148 * 8);
}

// dst <- src when *flag == 0 (16-byte words when both are aligned, the tail
// and unaligned buffers bytewise); a NaN or non-zero flag copies nothing.
template <bool VEC>
__global__ void copy_if_zero_kernel(uint8_t* __restrict__ dst, const uint8_t* __restrict__ src, int64_t bytes,
                                    const float* __restrict__ flag) {
    if (!(*flag == 0.f)) return;
    const int64_t tid = (int64_t)blockIdx.x * blockDim.x + threadIdx.x, stride = (int64_t)gridDim.x * blockDim.x;
    int64_t done = 0;
    if (VEC) {
        const int64_t n16 = bytes / 16;
        for (int64_t i = tid; i < n16; i += stride)
            reinterpret_cast<uint4*>(dst)[i] = __ldg(reinterpret_cast<const uint4*>(src) + i);
        done = n16 * 16;
    }
    for (int64_t i = done + tid; i < bytes; i += stride) dst[i] = src[i];
}

}  // namespace

// ===========================================================================
// C ABI
// ===========================================================================

extern "C" size_t zg_perturbed_linear_workspace_size(int P, int M, int K, int N, int rank, int dtype,
                                                     int x_batched) {
    if (P < 1 || M < 1 || K < 1 || N < 1 || rank < 1 || !zg::dtype_ok(dtype)) return 0;
    size_t simt_need = low_rank_ws(P, M, K, N, rank, dtype, x_batched, (int64_t)K * rank, (int64_t)rank * N);
    size_t tc_need = 0;
    if (dtype == ZG_BF16 && !x_batched) tc_need = zg::tc_shared_forward_workspace(P, M, K, N, rank);
    if (dtype == ZG_BF16 && x_batched) tc_need = zg::batched_forward_workspace(P, M, K, N, rank, true);
    return simt_need > tc_need ? simt_need : tc_need;
}

extern "C" int zg_perturbed_linear(const void* x, int x_batched, const void* W, const uint32_t* keys,
                                   int group, int P, int M, int K, int N, int rank, float s, int dtype,
                                   void* y, void* workspace, size_t workspace_bytes, void* stream) {
    if (!dims_ok({P, M, K, N, rank}) || P > 65535)
        return zg::fail(ZG_ERR_INVALID, "zg_perturbed_linear: bad sizes P=%d M=%d K=%d N=%d rank=%d", P, M, K, N, rank);
    if (!zg::dtype_ok(dtype)) return zg::fail(ZG_ERR_INVALID, "zg_perturbed_linear: bad dtype");
    if (!x || !W || !keys || !y) return zg::fail(ZG_ERR_INVALID, "zg_perturbed_linear: null pointer");
    size_t need = zg_perturbed_linear_workspace_size(P, M, K, N, rank, dtype, x_batched);
    if (!workspace || workspace_bytes < need)
        return zg::fail(ZG_ERR_WORKSPACE, "zg_perturbed_linear: workspace %zu < %zu bytes", workspace_bytes, need);
    cudaStream_t st = zg::as_stream(stream);
    Carver cv(workspace, workspace_bytes);
    if (dtype == ZG_BF16 && !x_batched && zg::tc_shared_forward_ok(P, M, K, N, rank))
        // W [K, N] row-major is the MN-major B operand of x @ W.
        return zg::tc_shared_forward(x, W, true, N, keys, group, P, M, K, N, rank, /*f1: A, k*r+j*/ 0, 0,
                                     /*f2: B, j*N+n*/ 1, 1, s, y, cv, st);
    if (dtype == ZG_BF16 && x_batched && zg::batched_forward_ok(P, M, K, N, rank))
        return zg::batched_forward(x, W, true, keys, group, /*f1: A, k*r+j*/ 0, /*f2: B, j*N+n*/ 1, 1, true, nullptr,
                                   nullptr, P, M, K, N, rank, s, y, cv, st);
    size_t es = zg::dtype_size(dtype);
    char* fa = cv.take<char>((size_t)P * K * rank * es);
    char* fb = cv.take<char>((size_t)P * rank * N * es);
    float* U = cv.take<float>((size_t)P * M * rank);
    float* XW = x_batched ? nullptr : cv.take<float>((size_t)M * N);
    int rc = zg::launch_population_factors(keys, group, P, ZG_MATRIX, K, N, rank, dtype, fa, fb, st);
    if (rc) return rc;
    LowRankPlan q{P, M, K, N, rank, dtype, x_batched, x, W, (int64_t)N, 1, fa, fb,
                  (int64_t)rank * N, (int64_t)N, 1, s, y, U, XW};
    return dtype == ZG_BF16 ? run_low_rank<__nv_bfloat16>(q, st) : run_low_rank<float>(q, st);
}

extern "C" size_t zg_tied_logits_workspace_size(int P, int M, int V, int C, int rank, int dtype,
                                                int x_batched) {
    if (P < 1 || M < 1 || V < 1 || C < 1 || rank < 1 || !zg::dtype_ok(dtype)) return 0;
    size_t simt_need = low_rank_ws(P, M, C, V, rank, dtype, x_batched, (int64_t)C * rank, (int64_t)V * rank);
    size_t tc_need = 0;
    if (dtype == ZG_BF16 && !x_batched) tc_need = zg::tc_shared_forward_workspace(P, M, C, V, rank);
    if (dtype == ZG_BF16 && x_batched) tc_need = zg::batched_forward_workspace(P, M, C, V, rank, true);
    return simt_need > tc_need ? simt_need : tc_need;
}

extern "C" int zg_tied_logits(const void* x, int x_batched, const void* T, const uint32_t* keys, int group,
                              int P, int M, int V, int C, int rank, float s, int dtype, void* y,
                              void* workspace, size_t workspace_bytes, void* stream) {
    if (!dims_ok({P, M, V, C, rank}) || P > 65535)
        return zg::fail(ZG_ERR_INVALID, "zg_tied_logits: bad sizes");
    if (!zg::dtype_ok(dtype)) return zg::fail(ZG_ERR_INVALID, "zg_tied_logits: bad dtype");
    if (!x || !T || !keys || !y) return zg::fail(ZG_ERR_INVALID, "zg_tied_logits: null pointer");
    size_t need = zg_tied_logits_workspace_size(P, M, V, C, rank, dtype, x_batched);
    if (!workspace || workspace_bytes < need)
        return zg::fail(ZG_ERR_WORKSPACE, "zg_tied_logits: workspace %zu < %zu bytes", workspace_bytes, need);
    cudaStream_t st = zg::as_stream(stream);
    Carver cv(workspace, workspace_bytes);
    if (dtype == ZG_BF16 && !x_batched && zg::tc_shared_forward_ok(P, M, C, V, rank))
        // T [V, C] is the K-major B operand of x @ T^T; U = x @ B_t (B_t[c, j]:
        // counter c*r + j), expanded through A_t[v, j] (counter v*r + j).
        return zg::tc_shared_forward(x, T, false, C, keys, group, P, M, C, V, rank, /*f1: B*/ 1, 0,
                                     /*f2: A*/ 0, 0, s, y, cv, st);
    if (dtype == ZG_BF16 && x_batched && zg::batched_forward_ok(P, M, C, V, rank))
        return zg::batched_forward(x, T, false, keys, group, /*f1: B*/ 1, /*f2: A*/ 0, 0, true, nullptr, nullptr, P, M,
                                   C, V, rank, s, y, cv, st);
    size_t es = zg::dtype_size(dtype);
    // table factors: A [P, V, r] (rows), B [P, C, r] (cols)
    char* fb = cv.take<char>((size_t)P * C * rank * es);
    char* fa = cv.take<char>((size_t)P * V * rank * es);
    float* U = cv.take<float>((size_t)P * M * rank);
    float* XW = x_batched ? nullptr : cv.take<float>((size_t)M * V);
    int rc = zg::launch_population_factors(keys, group, P, ZG_TABLE, V, C, rank, dtype, fa, fb, st);
    if (rc) return rc;
    // Wop(k=c, n=v) = T[v*C + c];  F1 = B_p [C, r];  F2(j, v) = A_p[v*r + j]
    LowRankPlan q{P, M, C, V, rank, dtype, x_batched, x, T, 1, (int64_t)C, fb, fa,
                  (int64_t)V * rank, 1, (int64_t)rank, s, y, U, XW};
    return dtype == ZG_BF16 ? run_low_rank<__nv_bfloat16>(q, st) : run_low_rank<float>(q, st);
}

extern "C" size_t zg_table_lookup_workspace_size(int P, int64_t n_idx, int64_t rows, int64_t cols, int rank,
                                                 int dtype) {
    if (P < 1 || n_idx < 0 || rows < 1 || cols < 1 || rank < 1 || !zg::dtype_ok(dtype)) return 0;
    // B factors for every candidate; the A factor of the unused slot is tiny.
    const size_t simt = Carver::need({(size_t)P * cols * rank * zg::dtype_size(dtype), 256});
    // tensor-core path: gathered rows (float32), A rows at the ids, B operand
    const size_t q = (size_t)P * rank;
    const size_t tc = Carver::need({(size_t)n_idx * cols * 4, (size_t)n_idx * q * 2, (size_t)cols * q * 2});
    return simt > tc ? simt : tc;
}

extern "C" int zg_table_lookup(const void* T, const int32_t* idx, int idx_batched, int64_t n_idx,
                               const uint32_t* keys, int group, int P, int64_t rows, int64_t cols,
                               int rank, float s, int dtype, void* out, void* workspace,
                               size_t workspace_bytes, void* stream) {
    if (P < 1 || P > 65535 || rows < 1 || cols < 1 || rank < 1 || rank > 1024 || n_idx < 0 || n_idx > 2147483647)
        return zg::fail(ZG_ERR_INVALID, "zg_table_lookup: bad sizes");
    if (!zg::dtype_ok(dtype)) return zg::fail(ZG_ERR_INVALID, "zg_table_lookup: bad dtype");
    if (n_idx == 0) return ZG_OK;
    if (!T || !idx || !keys || !out) return zg::fail(ZG_ERR_INVALID, "zg_table_lookup: null pointer");
    size_t need = zg_table_lookup_workspace_size(P, n_idx, rows, cols, rank, dtype);
    if (!workspace || workspace_bytes < need)
        return zg::fail(ZG_ERR_WORKSPACE, "zg_table_lookup: workspace %zu < %zu bytes", workspace_bytes, need);
    cudaStream_t st = zg::as_stream(stream);
    Carver cv(workspace, workspace_bytes);
    if (lookup_tc_ok(P, n_idx, cols, rank, dtype, idx_batched, T, out)) {
        const int64_t q = (int64_t)P * rank;
        float* Tg = cv.take<float>((size_t)n_idx * cols);
        __nv_bfloat16* U = cv.take<__nv_bfloat16>((size_t)n_idx * q);
        __nv_bfloat16* Bop = cv.take<__nv_bfloat16>((size_t)cols * q);
        if (!Tg || !U || !Bop) return zg::fail(ZG_ERR_WORKSPACE, "zg_table_lookup: workspace too small");
        int rc = zg::factor_operands(keys, group, P, ZG_TABLE, rows, cols, rank, ZG_BF16, nullptr, Bop, st);
        if (rc) return rc;
        const int64_t cap = (int64_t)sm_count_ops() * 8;
        {
            zg::LaunchTimer zg_lt_("table_lookup", st);
            int64_t g1 = (n_idx * (cols / 8) + 255) / 256;
            gather_rows_f32_kernel<<<(unsigned)(g1 < cap ? g1 : cap), 256, 0, st>>>(
                static_cast<const __nv_bfloat16*>(T), idx, n_idx, rows, cols, Tg);
            int64_t g2 = (n_idx * P + 255) / 256;
            if (rank == 8)
                gather_a_rows_kernel<8><<<(unsigned)(g2 < cap ? g2 : cap), 256, 0, st>>>(keys, group, P, idx, n_idx,
                                                                                      rows, U);
            else
                gather_a_rows_kernel<16><<<(unsigned)(g2 < cap ? g2 : cap), 256, 0, st>>>(keys, group, P, idx, n_idx,
                                                                                       rows, U);
            if ((rc = zg::check_launch("zg_table_lookup(gather)"))) return rc;
        }
        return zg::tc_expand(Tg, U, Bop, q, P, (int)n_idx, (int)cols, rank, s, out, st, "table_lookup");
    }
    char* fb = cv.take<char>((size_t)P * cols * rank * zg::dtype_size(dtype));
    // Fill only B_p [cols, rank]; A rows are regenerated at the gathered
    // rows inside the lookup kernel (rows = 0: no A elements are drawn).
    int rc = zg::launch_population_factors(keys, group, P, ZG_TABLE, 0, cols, rank, dtype, nullptr, fb, st);
    if (rc) return rc;
    if (rank == 8 || rank == 16) {
        dim3 grid((unsigned)((n_idx + 31) / 32), P);
        const int threads = cols >= 256 ? 256 : (int)((cols + 31) / 32 * 32);
        zg::LaunchTimer zg_lt_("table_lookup", st);
#define ZG_LOOKUP(TT, R)                                                                                        \
    table_lookup_tiled_kernel<TT, R><<<grid, threads, 0, st>>>((const TT*)T, idx, idx_batched, n_idx, keys, group, \
                                                               rows, cols, s, (const TT*)fb, (TT*)out)
        if (dtype == ZG_BF16) {
            if (rank == 8) ZG_LOOKUP(__nv_bfloat16, 8);
            else ZG_LOOKUP(__nv_bfloat16, 16);
        } else {
            if (rank == 8) ZG_LOOKUP(float, 8);
            else ZG_LOOKUP(float, 16);
        }
#undef ZG_LOOKUP
        return zg::check_launch("zg_table_lookup");
    }
    dim3 grid((unsigned)n_idx, P);
    int threads = cols >= 256 ? 256 : (int)((cols + 31) / 32 * 32);
    if (threads < rank) threads = (rank + 31) / 32 * 32;
    size_t smem = rank * sizeof(float);
    zg::LaunchTimer zg_lt_("table_lookup", st);
    if (dtype == ZG_BF16)
        table_lookup_kernel<__nv_bfloat16><<<grid, threads, smem, st>>>(
            (const __nv_bfloat16*)T, idx, idx_batched, n_idx, keys, group, rows, cols, rank, s,
            (const __nv_bfloat16*)fb, (__nv_bfloat16*)out);
    else
        table_lookup_kernel<float><<<grid, threads, smem, st>>>((const float*)T, idx, idx_batched, n_idx, keys,
                                                                 group, rows, cols, rank, s, (const float*)fb,
                                                                 (float*)out);
    return zg::check_launch("zg_table_lookup");
}

extern "C" int zg_perturbed_vector(const void* v, int v_batched, const uint32_t* keys, int group, int P,
                                   int64_t n, float s, int dtype, void* out, void* stream) {
    if (P < 1 || P > 65535 || n < 1) return zg::fail(ZG_ERR_INVALID, "zg_perturbed_vector: bad sizes");
    if (!zg::dtype_ok(dtype)) return zg::fail(ZG_ERR_INVALID, "zg_perturbed_vector: bad dtype");
    if (!v || !keys || !out) return zg::fail(ZG_ERR_INVALID, "zg_perturbed_vector: null pointer");
    cudaStream_t st = zg::as_stream(stream);
    int chunks = (int)((n + 255) / 256);
    if (chunks > 1024) chunks = 1024;
    dim3 grid(chunks, P);
    zg::LaunchTimer zg_lt_("perturbed_vector", st);
    if (dtype == ZG_BF16)
        vector_kernel<__nv_bfloat16><<<grid, 256, 0, st>>>((const __nv_bfloat16*)v, v_batched, keys, group, n, s,
                                                           (__nv_bfloat16*)out);
    else
        vector_kernel<float><<<grid, 256, 0, st>>>((const float*)v, v_batched, keys, group, n, s, (float*)out);
    return zg::check_launch("zg_perturbed_vector");
}

extern "C" int zg_shape_fitness(const float* losses, int P, double sigma, float* shaped, float* metrics,
                                void* stream) {
    if (P < 2) return zg::fail(ZG_ERR_INVALID, "zg_shape_fitness: at least two candidate losses are required");
    if (!(sigma > 0) || !std::isfinite(sigma)) return zg::fail(ZG_ERR_INVALID, "zg_shape_fitness: bad sigma");
    if (!losses || !shaped || !metrics) return zg::fail(ZG_ERR_INVALID, "zg_shape_fitness: null pointer");
    // population_size * sigma is a Python float (double) converted to the
    // loss dtype at the division (src/zerograd/_fitness.py:34).
    const float denom = (float)((double)P * sigma);
    zg::LaunchTimer zg_lt_("shape_fitness", zg::as_stream(stream));
    shape_fitness_kernel<<<1, 1024, 0, zg::as_stream(stream)>>>(losses, P, denom, shaped, metrics);
    return zg::check_launch("zg_shape_fitness");
}

// out[r] = mean of x[r, 0:n], float64 accumulation in a fixed order (each of
// 256 threads sums a fixed stride of the row, then a fixed tree), so a row's
// mean does not depend on how many rows the launch has.
__global__ void row_mean_kernel(const float* __restrict__ x, int64_t n, float* __restrict__ out) {
    __shared__ double part[256];
    const float* row = x + (int64_t)blockIdx.x * n;
    double acc = 0.0;
    for (int64_t i = threadIdx.x; i < n; i += 256) acc += (double)row[i];
    part[threadIdx.x] = acc;
    __syncthreads();
    for (int w = 128; w > 0; w >>= 1) {
        if ((int)threadIdx.x < w) part[threadIdx.x] += part[threadIdx.x + w];
        __syncthreads();
    }
    if (threadIdx.x == 0) out[blockIdx.x] = (float)(part[0] / (double)n);
}

extern "C" int zg_row_mean(const float* x, int64_t rows, int64_t n, float* out, void* stream) {
    if (rows < 0 || n < 1 || rows > 2147483647LL) return zg::fail(ZG_ERR_INVALID, "zg_row_mean: bad sizes");
    if (rows == 0) return ZG_OK;
    if (!x || !out) return zg::fail(ZG_ERR_INVALID, "zg_row_mean: null pointer");
    zg::LaunchTimer zg_lt_("row_mean", zg::as_stream(stream));
    row_mean_kernel<<<(unsigned)rows, 256, 0, zg::as_stream(stream)>>>(x, n, out);
    return zg::check_launch("zg_row_mean");
}

extern "C" size_t zg_replay_workspace_size(int P, int layout, int64_t rows, int64_t cols, int rank, int dtype) {
    if (P < 1 || rows < 1 || !zg::dtype_ok(dtype)) return 0;
    if (layout == ZG_VECTOR) return Carver::need({(size_t)vector_replay_slices(P) * rows * 4}) + 256;
    if (cols < 1 || rank < 1) return 0;
    size_t es = zg::dtype_size(dtype);
    size_t simt_need = Carver::need({(size_t)P * rows * rank * es, (size_t)P * cols * rank * es});
    size_t tc_need = dtype == ZG_BF16 ? zg::tc_replay_workspace(P, rows, cols, rank) : 0;
    return simt_need > tc_need ? simt_need : tc_need;
}

extern "C" int zg_replay(const float* shaped, const uint32_t* keys, int group, int P, int layout,
                         int64_t rows, int64_t cols, int rank, float inv_sqrt_rank, int dtype, float* out,
                         void* workspace, size_t workspace_bytes, void* stream) {
    if (P < 1 || P > 65535 || rows < 1 || (layout != ZG_VECTOR && (cols < 1 || rank < 1)))
        return zg::fail(ZG_ERR_INVALID, "zg_replay: bad sizes");
    if (layout < ZG_MATRIX || layout > ZG_VECTOR) return zg::fail(ZG_ERR_INVALID, "zg_replay: bad layout");
    if (!zg::dtype_ok(dtype)) return zg::fail(ZG_ERR_INVALID, "zg_replay: bad dtype");
    if (!shaped || !keys || !out) return zg::fail(ZG_ERR_INVALID, "zg_replay: null pointer");
    cudaStream_t st = zg::as_stream(stream);
    size_t need = zg_replay_workspace_size(P, layout, rows, cols, rank, dtype);
    if (!workspace || workspace_bytes < need)
        return zg::fail(ZG_ERR_WORKSPACE, "zg_replay: workspace %zu < %zu bytes", workspace_bytes, need);
    Carver cv(workspace, workspace_bytes);
    if (layout == ZG_VECTOR) {
        const int slices = vector_replay_slices(P);
        float* partial = cv.take<float>((size_t)slices * rows);
        if (!partial) return zg::fail(ZG_ERR_WORKSPACE, "zg_replay: workspace too small");
        const int64_t tiles = (rows + VR_COLS - 1) / VR_COLS;
        if (tiles > 2147483647LL || slices > 65535) return zg::fail(ZG_ERR_INVALID, "zg_replay: vector too long");
        {
            zg::LaunchTimer zg_lt_("replay_vector", st);
            dim3 grid((unsigned)tiles, (unsigned)slices);
            if (dtype == ZG_BF16)
                vector_replay_partial_kernel<__nv_bfloat16><<<grid, VR_COLS, 0, st>>>(shaped, keys, group, P, rows,
                                                                                        partial);
            else
                vector_replay_partial_kernel<float><<<grid, VR_COLS, 0, st>>>(shaped, keys, group, P, rows, partial);
            if (int e = zg::check_launch("zg_replay(vector)")) return e;
        }
        zg::LaunchTimer zg_lt2_("replay_vector_sum", st);
        vector_replay_sum_kernel<<<(unsigned)((rows + 255) / 256), 256, 0, st>>>(partial, slices, rows, out);
        return zg::check_launch("zg_replay(vector sum)");
    }
    if (zg::tc_replay_ok(P, rows, cols, rank, dtype))
        return zg::tc_replay_run(shaped, keys, group, P, layout, rows, cols, rank, inv_sqrt_rank, out, cv, st);
    size_t es = zg::dtype_size(dtype);
    char* fa = cv.take<char>((size_t)P * rows * rank * es);
    char* fb = cv.take<char>((size_t)P * cols * rank * es);
    if (dtype == ZG_F32 && ((int64_t)P * rank) % 4 == 0 && rows <= 2147483647 && cols <= 2147483647) {
        // float32: the factors in operand layout (A_op [rows, P r], B_op
        // [cols, P r], contraction columns contiguous) and one NT GEMM with
        // the fitness weight applied to A as it is staged
        int rc = zg::factor_operands(keys, group, P, layout, rows, cols, rank, ZG_F32, fa, fb, st);
        if (rc) return rc;
        return zg::launch_replay_sgemm(reinterpret_cast<const float*>(fa), reinterpret_cast<const float*>(fb), shaped,
                                       rank, (int)rows, (int)cols, (int64_t)P * rank, inv_sqrt_rank, out, st);
    }
    int rc = zg::launch_population_factors(keys, group, P, layout, rows, cols, rank, dtype, fa, fb, st);
    if (rc) return rc;
    SimtGemm g;
    g.A = fa; g.sAm = rank; g.sAko = rows * (int64_t)rank; g.sAki = 1;
    g.kscale = shaped;
    g.B = fb;
    if (layout == ZG_MATRIX) { g.sBko = (int64_t)rank * cols; g.sBki = cols; g.sBn = 1; }
    else { g.sBko = cols * (int64_t)rank; g.sBki = 1; g.sBn = rank; }
    g.C = out; g.sCm = cols; g.sCn = 1;
    g.M = (int)rows; g.N = (int)cols; g.Ko = P; g.Ki = rank; g.batch = 1; g.alpha = inv_sqrt_rank;
    if (rows > 2147483647 || cols > 2147483647) return zg::fail(ZG_ERR_INVALID, "zg_replay: dims too large");
    return dtype == ZG_BF16 ? simt<__nv_bfloat16, float>(g, st, "replay_gemm") : simt<float, float>(g, st, "replay_gemm");
}

extern "C" int zg_adamw_update(const void* param, void* param_out, int dtype, const float* descent,
                               const float* mu, const float* nu, float* mu_out, float* nu_out, int64_t n,
                               int count, double lr, double b1, double b2, double eps, double weight_decay,
                               const float* bias_corrections, void* stream) {
    if (n < 0 || count < 1) return zg::fail(ZG_ERR_INVALID, "zg_adamw_update: bad sizes");
    if (!zg::dtype_ok(dtype)) return zg::fail(ZG_ERR_INVALID, "zg_adamw_update: bad dtype");
    if (n == 0) return ZG_OK;
    if (!param || !param_out || !mu || !nu || !mu_out || !nu_out)
        return zg::fail(ZG_ERR_INVALID, "zg_adamw_update: null pointer");
    const zg::AdamConsts c = zg::adam_consts(count, lr, b1, b2, eps, weight_decay);
    cudaStream_t st = zg::as_stream(stream);
    zg::LaunchTimer zg_lt_("adamw_update", st);
    if (dtype == ZG_BF16)
        adamw_kernel<__nv_bfloat16><<<ew_grid(n), 256, 0, st>>>((const __nv_bfloat16*)param, (__nv_bfloat16*)param_out,
                                                                descent, mu, nu, mu_out, nu_out, n, c,
                                                                bias_corrections);
    else
        adamw_kernel<float><<<ew_grid(n), 256, 0, st>>>((const float*)param, (float*)param_out, descent, mu, nu,
                                                        mu_out, nu_out, n, c, bias_corrections);
    return zg::check_launch("zg_adamw_update");
}

extern "C" int zg_adam_bias_corrections(int count, double b1, double b2, float* out) {
    if (count < 1 || !out) return zg::fail(ZG_ERR_INVALID, "zg_adam_bias_corrections: count >= 1 and an output");
    const zg::AdamConsts c = zg::adam_consts(count, 0.0, b1, b2, 0.0, 0.0);
    out[0] = c.bc1;
    out[1] = c.bc2;
    return ZG_OK;
}

extern "C" int zg_copy_if_zero(void* dst, const void* src, size_t bytes, const float* flag, void* stream) {
    if (bytes == 0) return ZG_OK;
    if (!dst || !src || !flag) return zg::fail(ZG_ERR_INVALID, "zg_copy_if_zero: null pointer");
    if ((bytes > 0x7fffffffffffffffULL)) return zg::fail(ZG_ERR_INVALID, "zg_copy_if_zero: bad size");
    cudaStream_t st = zg::as_stream(stream);
    const bool vec = ((reinterpret_cast<uintptr_t>(dst) | reinterpret_cast<uintptr_t>(src)) & 15) == 0;
    const int64_t n = (int64_t)bytes;
    zg::LaunchTimer zg_lt_("copy_if_zero", st);
    if (vec)
        copy_if_zero_kernel<true><<<ew_grid(n / 16 + 1), 256, 0, st>>>((uint8_t*)dst, (const uint8_t*)src, n, flag);
    else
        copy_if_zero_kernel<false><<<ew_grid(n), 256, 0, st>>>((uint8_t*)dst, (const uint8_t*)src, n, flag);
    return zg::check_launch("zg_copy_if_zero");
}

extern "C" int zg_sgd_update(const void* param, void* param_out, int dtype, const float* descent, int64_t n,
                             double lr, void* stream) {
    if (n < 0) return zg::fail(ZG_ERR_INVALID, "zg_sgd_update: bad sizes");
    if (!zg::dtype_ok(dtype)) return zg::fail(ZG_ERR_INVALID, "zg_sgd_update: bad dtype");
    if (n == 0) return ZG_OK;
    if (!param || !param_out) return zg::fail(ZG_ERR_INVALID, "zg_sgd_update: null pointer");
    cudaStream_t st = zg::as_stream(stream);
    zg::LaunchTimer zg_lt_("sgd_update", st);
    if (dtype == ZG_BF16)
        sgd_kernel<__nv_bfloat16><<<ew_grid(n), 256, 0, st>>>((const __nv_bfloat16*)param, (__nv_bfloat16*)param_out,
                                                              descent, n, (float)(-lr));
    else
        sgd_kernel<float><<<ew_grid(n), 256, 0, st>>>((const float*)param, (float*)param_out, descent, n,
                                                      (float)(-lr));
    return zg::check_launch("zg_sgd_update");
}
