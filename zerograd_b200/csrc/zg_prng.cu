// zg_prng.cu -- threefry key derivation, bits, normals and population
// factor fills (device restatement of src/zerograd/_keys.py:20-58 and
// src/zerograd/_factors.py:30-74 over jax.random's partitionable threefry).
#include "zg_common.cuh"

namespace {

constexpr int kThreads = 256;

__global__ void threefry_kernel(const uint32_t* __restrict__ keys, const uint32_t* __restrict__ ctrs,
                                uint32_t* __restrict__ out, int64_t n) {
    for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < n;
         i += (int64_t)gridDim.x * blockDim.x) {
        ZgKey k = zg_make_key(keys[2 * i], keys[2 * i + 1]);
        uint2 o = zg_threefry(k, ctrs[2 * i], ctrs[2 * i + 1]);
        out[2 * i] = o.x;
        out[2 * i + 1] = o.y;
    }
}

__global__ void fold_in_kernel(const uint32_t* __restrict__ keys, int key_stride,
                               const uint32_t* __restrict__ data, uint32_t* __restrict__ out,
                               int64_t n) {
    for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < n;
         i += (int64_t)gridDim.x * blockDim.x) {
        int64_t ki = key_stride ? i : 0;
        ZgKey k = zg_make_key(keys[2 * ki], keys[2 * ki + 1]);
        uint2 o = zg_threefry(k, 0u, data[i]);
        out[2 * i] = o.x;
        out[2 * i + 1] = o.y;
    }
}

__global__ void candidate_keys_kernel(uint32_t k0, uint32_t k1, const uint32_t* __restrict__ data,
                                      uint32_t* __restrict__ out, int64_t n) {
    const ZgKey k = zg_make_key(k0, k1);
    for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < n;
         i += (int64_t)gridDim.x * blockDim.x) {
        uint2 o = zg_threefry(k, 0u, data[i]);
        out[2 * i] = o.x;
        out[2 * i + 1] = o.y;
    }
}

// grid: (chunks, nkeys); each thread handles consecutive elements of one key.
template <bool kNormal, typename T>
__global__ void bits_kernel(const uint32_t* __restrict__ keys, int64_t n, void* __restrict__ out) {
    const int64_t kidx = blockIdx.y;
    ZgKey k = zg_make_key(keys[2 * kidx], keys[2 * kidx + 1]);
    for (int64_t j = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; j < n;
         j += (int64_t)gridDim.x * blockDim.x) {
        uint32_t b = zg_bits(k, (uint64_t)j);
        if constexpr (kNormal) {
            static_cast<T*>(out)[kidx * n + j] = zg_from_float<T>(zg_normal_from_bits(b));
        } else {
            static_cast<uint32_t*>(out)[kidx * n + j] = b;
        }
    }
}

// Population factors.  grid: (chunks, P, 2) -- z selects A (0) or B (1).
// Flat element j of a factor is normal(key)[j]; the flat orders of the
// reference layouts are exactly the storage orders used here, so stores are
// contiguous per candidate.
template <typename T>
__global__ void factors_kernel(const uint32_t* __restrict__ keys, int group, int layout,
                               int64_t na, int64_t nb, T* __restrict__ A, T* __restrict__ B) {
    const int p = blockIdx.y;
    const int which = blockIdx.z;
    ZgKey k;
    if (layout == ZG_VECTOR) {
        k = zg_group_key(keys, p, group);
    } else {
        ZgFactorKeys fk = zg_factor_keys(keys, p, group);
        k = which == 0 ? fk.a : fk.b;
    }
    const int64_t n = which == 0 ? na : nb;
    T* dst = (which == 0 ? A + (int64_t)p * na : B + (int64_t)p * nb);
    for (int64_t j = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; j < n;
         j += (int64_t)gridDim.x * blockDim.x) {
        dst[j] = zg_from_float<T>(zg_normal(k, (uint64_t)j));
    }
}

int grid_for(int64_t n, int cap = 148 * 16) {
    int64_t g = (n + kThreads - 1) / kThreads;
    if (g < 1) g = 1;
    return (int)(g < cap ? g : cap);
}

}  // namespace

namespace zg {

// Used by the op files: launch the population factor fill.
int launch_population_factors(const uint32_t* keys, int group, int P, int layout, int64_t rows,
                              int64_t cols, int rank, int dtype, void* A, void* B,
                              cudaStream_t st) {
    const int64_t na = layout == ZG_VECTOR ? rows : rows * (int64_t)rank;
    const int64_t nb = layout == ZG_VECTOR ? 0 : cols * (int64_t)rank;
    const int64_t nmax = na > nb ? na : nb;
    int chunks = grid_for(nmax, 1 << 16);
    int per_cand_cap = (int)((148 * 32 + P - 1) / P);
    if (per_cand_cap < 1) per_cand_cap = 1;
    if (chunks > per_cand_cap) chunks = per_cand_cap;
    dim3 grid(chunks, P, layout == ZG_VECTOR ? 1 : 2);
    zg::LaunchTimer zg_lt_("factor_fill", st);
    if (dtype == ZG_BF16)
        factors_kernel<__nv_bfloat16><<<grid, kThreads, 0, st>>>(
            keys, group, layout, na, nb, static_cast<__nv_bfloat16*>(A), static_cast<__nv_bfloat16*>(B));
    else
        factors_kernel<float><<<grid, kThreads, 0, st>>>(keys, group, layout, na, nb,
                                                         static_cast<float*>(A), static_cast<float*>(B));
    return check_launch("population_factors");
}

}  // namespace zg

extern "C" int zg_threefry2x32(const uint32_t* keys, const uint32_t* ctrs, uint32_t* out, int64_t n,
                               void* stream) {
    if (n < 0) return zg::fail(ZG_ERR_INVALID, "zg_threefry2x32: n < 0");
    if (n == 0) return ZG_OK;
    if (!keys || !ctrs || !out) return zg::fail(ZG_ERR_INVALID, "zg_threefry2x32: null pointer");
    zg::LaunchTimer zg_lt_("threefry", zg::as_stream(stream));
    threefry_kernel<<<grid_for(n), kThreads, 0, zg::as_stream(stream)>>>(keys, ctrs, out, n);
    return zg::check_launch("zg_threefry2x32");
}

extern "C" int zg_fold_in(const uint32_t* keys, int key_stride, const uint32_t* data, uint32_t* out,
                          int64_t n, void* stream) {
    if (n < 0) return zg::fail(ZG_ERR_INVALID, "zg_fold_in: n < 0");
    if (n == 0) return ZG_OK;
    if (!keys || !data || !out) return zg::fail(ZG_ERR_INVALID, "zg_fold_in: null pointer");
    zg::LaunchTimer zg_lt_("fold_in", zg::as_stream(stream));
    fold_in_kernel<<<grid_for(n), kThreads, 0, zg::as_stream(stream)>>>(keys, key_stride, data, out, n);
    return zg::check_launch("zg_fold_in");
}

extern "C" int zg_candidate_keys(uint32_t k0, uint32_t k1, const uint32_t* data, uint32_t* out, int64_t n,
                                 void* stream) {
    if (n < 0) return zg::fail(ZG_ERR_INVALID, "zg_candidate_keys: n < 0");
    if (n == 0) return ZG_OK;
    if (!data || !out) return zg::fail(ZG_ERR_INVALID, "zg_candidate_keys: null pointer");
    zg::LaunchTimer zg_lt_("candidate_keys", zg::as_stream(stream));
    candidate_keys_kernel<<<grid_for(n), kThreads, 0, zg::as_stream(stream)>>>(k0, k1, data, out, n);
    return zg::check_launch("zg_candidate_keys");
}

extern "C" int zg_random_bits(const uint32_t* keys, int64_t nkeys, int64_t n, uint32_t* out,
                              void* stream) {
    if (n < 0 || nkeys < 0 || nkeys > 65535) return zg::fail(ZG_ERR_INVALID, "zg_random_bits: bad sizes");
    if (n == 0 || nkeys == 0) return ZG_OK;
    if (!keys || !out) return zg::fail(ZG_ERR_INVALID, "zg_random_bits: null pointer");
    dim3 grid(grid_for(n), (unsigned)nkeys);
    zg::LaunchTimer zg_lt_("random_bits", zg::as_stream(stream));
    bits_kernel<false, float><<<grid, kThreads, 0, zg::as_stream(stream)>>>(keys, n, out);
    return zg::check_launch("zg_random_bits");
}

extern "C" int zg_normal(const uint32_t* keys, int64_t nkeys, int64_t n, int dtype, void* out,
                         void* stream) {
    if (n < 0 || nkeys < 0 || nkeys > 65535) return zg::fail(ZG_ERR_INVALID, "zg_normal: bad sizes");
    if (!zg::dtype_ok(dtype)) return zg::fail(ZG_ERR_INVALID, "zg_normal: bad dtype %d", dtype);
    if (n == 0 || nkeys == 0) return ZG_OK;
    if (!keys || !out) return zg::fail(ZG_ERR_INVALID, "zg_normal: null pointer");
    dim3 grid(grid_for(n), (unsigned)nkeys);
    zg::LaunchTimer zg_lt_("normal", zg::as_stream(stream));
    if (dtype == ZG_BF16)
        bits_kernel<true, __nv_bfloat16><<<grid, kThreads, 0, zg::as_stream(stream)>>>(keys, n, out);
    else
        bits_kernel<true, float><<<grid, kThreads, 0, zg::as_stream(stream)>>>(keys, n, out);
    return zg::check_launch("zg_normal");
}

extern "C" int zg_population_factors(const uint32_t* keys, int group, int P, int layout, int64_t rows,
                                     int64_t cols, int rank, int dtype, void* A, void* B,
                                     void* stream) {
    if (P < 0 || P > 65535 || rows < 1 || (layout != ZG_VECTOR && (cols < 1 || rank < 1)))
        return zg::fail(ZG_ERR_INVALID, "zg_population_factors: bad sizes");
    if (layout < ZG_MATRIX || layout > ZG_VECTOR) return zg::fail(ZG_ERR_INVALID, "zg_population_factors: bad layout");
    if (!zg::dtype_ok(dtype)) return zg::fail(ZG_ERR_INVALID, "zg_population_factors: bad dtype");
    if (P == 0) return ZG_OK;
    if (!keys || !A || (layout != ZG_VECTOR && !B)) return zg::fail(ZG_ERR_INVALID, "zg_population_factors: null pointer");
    return zg::launch_population_factors(keys, group, P, layout, rows, cols, rank, dtype, A, B,
                                         zg::as_stream(stream));
}
