// zg_norm.cu -- population-batched LayerNorm and RMSNorm with per-candidate
// scale and bias: the normalisations of a candidate's transformer block, fed
// by the vectors CandidateContext.vector returns for every candidate
// (v + sigma * noise_p, src/zerograd/_candidate.py:41-45, 82-87).
//
//   layer_norm: y = (x - mean) / sqrt(var + eps) * scale + bias
//               (biased variance; examples/train_vit_cifar10.py:76-79)
//   rms_norm:   y = x / sqrt(mean(x^2) + eps) * scale
// Per row: the means as sums times 1/C (float32), one reciprocal square
// root (rsqrtf, within 2 ulp), a multiply per element (within a few float32
// ulp of the divisions; the per-row statistics are executed by every lane of
// the row's warp, so their cost weighs most on short rows).
//
// Statistics in float32 over the last axis (C); output rounded to x's dtype.
// x [P, M, C] (x_batched) or [M, C] shared by the candidates; scale, bias
// [P, C] (p_batched) or [C]; y [P, M, C].  One warp per row; HBM-bound.
#include <math.h>

#include "zg_common.cuh"

namespace {

enum { NORM_LAYER = 0, NORM_RMS = 1 };

__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
    return v;
}

template <typename T>
__device__ __forceinline__ void load8(const T* p, float (&v)[8]) {
    if constexpr (sizeof(T) == 2) {
        const uint4 raw = *reinterpret_cast<const uint4*>(p);
        const uint32_t w[4] = {raw.x, raw.y, raw.z, raw.w};
#pragma unroll
        for (int i = 0; i < 4; ++i) {
            v[2 * i] = __uint_as_float(w[i] << 16);
            v[2 * i + 1] = __uint_as_float(w[i] & 0xffff0000u);
        }
    } else {
        const float4 a = *reinterpret_cast<const float4*>(p), b = *reinterpret_cast<const float4*>(p + 4);
        v[0] = a.x; v[1] = a.y; v[2] = a.z; v[3] = a.w; v[4] = b.x; v[5] = b.y; v[6] = b.z; v[7] = b.w;
    }
}

template <typename T>
__device__ __forceinline__ void store8(T* p, const float (&v)[8]) {
    if constexpr (sizeof(T) == 2) {
        uint4 o;
        __nv_bfloat162* h = reinterpret_cast<__nv_bfloat162*>(&o);
#pragma unroll
        for (int i = 0; i < 4; ++i) h[i] = __floats2bfloat162_rn(v[2 * i], v[2 * i + 1]);
        *reinterpret_cast<uint4*>(p) = o;
    } else {
        *reinterpret_cast<float4*>(p) = make_float4(v[0], v[1], v[2], v[3]);
        *reinterpret_cast<float4*>(p + 4) = make_float4(v[4], v[5], v[6], v[7]);
    }
}

struct NormArgs {
    const void* x;
    const void* scale;
    const void* bias;
    void* y;
    int64_t M;
    int P, C, x_batched, p_batched, kind;
    float eps;
    float inv_c;  // 1/C rounded to float32: means are sums times it
};

// Rows held in registers: CH chunks of 8 values per lane (C <= 256 * CH, C a
// multiple of 8, rows 16-byte aligned), R rows per warp per pass with every
// row's loads issued before the first reduction, so a warp keeps R rows of
// HBM reads in flight (a norm is HBM-bound: its rate is the bytes in flight
// per SM over the memory latency).
template <typename T, int CH, int R>
__global__ void __launch_bounds__(256) norm_reg_kernel(const NormArgs a) {
    const int lane = threadIdx.x % 32;
    const int64_t rows = (int64_t)a.P * a.M;
    const int64_t warp0 = ((int64_t)blockIdx.x * blockDim.x + threadIdx.x) / 32;
    const int64_t nwarps = (int64_t)gridDim.x * blockDim.x / 32;
    const int chunks = a.C / 8;
    for (int64_t g0 = warp0 * R; g0 < rows; g0 += nwarps * R) {
        float v[R][CH][8];
        float s1[R], s2[R], mean[R], rinv[R];
#pragma unroll
        for (int q = 0; q < R; ++q) {
            const int64_t g = g0 + q;
            s1[q] = 0.f;
            if (g >= rows) continue;
            const int p = (int)(g / a.M);
            const int64_t m = g % a.M;
            const T* xr = static_cast<const T*>(a.x) + ((a.x_batched ? (int64_t)p : 0) * a.M + m) * a.C;
#pragma unroll
            for (int j = 0; j < CH; ++j) {
                const int c = lane + 32 * j;
                if (c < chunks) load8(xr + 8 * c, v[q][j]);
            }
        }
#pragma unroll
        for (int q = 0; q < R; ++q) {
            mean[q] = 0.f;
            s2[q] = 0.f;
            if (a.kind == NORM_LAYER) {
#pragma unroll
                for (int j = 0; j < CH; ++j)
                    if (lane + 32 * j < chunks)
#pragma unroll
                        for (int i = 0; i < 8; ++i) s1[q] += v[q][j][i];
                mean[q] = warp_sum(s1[q]) * a.inv_c;
#pragma unroll
                for (int j = 0; j < CH; ++j)
                    if (lane + 32 * j < chunks)
#pragma unroll
                        for (int i = 0; i < 8; ++i) {
                            const float d = v[q][j][i] - mean[q];
                            s2[q] = fmaf(d, d, s2[q]);
                        }
            } else {
#pragma unroll
                for (int j = 0; j < CH; ++j)
                    if (lane + 32 * j < chunks)
#pragma unroll
                        for (int i = 0; i < 8; ++i) s2[q] = fmaf(v[q][j][i], v[q][j][i], s2[q]);
            }
            // one division per row
            rinv[q] = rsqrtf(warp_sum(s2[q]) * a.inv_c + a.eps);
        }
#pragma unroll
        for (int q = 0; q < R; ++q) {
            const int64_t g = g0 + q;
            if (g >= rows) continue;
            const int p = (int)(g / a.M);
            const T* sr = static_cast<const T*>(a.scale) + (a.p_batched ? (int64_t)p : 0) * a.C;
            const T* br = a.bias ? static_cast<const T*>(a.bias) + (a.p_batched ? (int64_t)p : 0) * a.C : nullptr;
            T* yr = static_cast<T*>(a.y) + g * a.C;
#pragma unroll
            for (int j = 0; j < CH; ++j) {
                const int c = lane + 32 * j;
                if (c < chunks) {
                    float sc[8], bi[8], o[8];
                    load8(sr + 8 * c, sc);
                    if (br) load8(br + 8 * c, bi);
#pragma unroll
                    for (int i = 0; i < 8; ++i) {
                        o[i] = __fmul_rn(__fmul_rn(v[q][j][i] - mean[q], rinv[q]), sc[i]);
                        if (br) o[i] = __fadd_rn(o[i], bi[i]);
                    }
                    store8(yr + 8 * c, o);
                }
            }
        }
    }
}

// bf16 rows held packed: each lane keeps its chunks of R rows as raw 16-byte
// words (12 registers per row at C = 768 instead of 24) and widens them to
// float32 where the statistics and the output use them, so R = 4 rows per
// warp fit in the registers the float form needs for two: twice the HBM
// reads in flight.  Same per-lane arithmetic, in the same order, as
// norm_reg_kernel (the same bits).
//
// LW = 16 gives each row half a warp (two rows side by side in one warp),
// so each per-row instruction of the statistics (reductions, rsqrtf) serves
// two rows: for short rows (C <= 512) those dominate, and 384 columns split
// evenly over 16 lanes (3 chunks each) where 32 lanes leave half of them
// idle in the second chunk; at C = 768 it still saves a few per cent.
template <int LW>
__device__ __forceinline__ float group_sum(float v) {
#pragma unroll
    for (int o = LW / 2; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
    return v;
}

template <int CH, int R, int LW = 32>
__global__ void __launch_bounds__(256, CH * R >= 16 ? 2 : 3) norm_packed_kernel(const NormArgs a) {
    const int lane = threadIdx.x % LW, slot = (threadIdx.x % 32) / LW;  // lane in the row's group; which row
    constexpr int RW = R * (32 / LW);                                     // rows per warp per pass
    const int64_t rows = (int64_t)a.P * a.M;
    const int64_t warp0 = ((int64_t)blockIdx.x * blockDim.x + threadIdx.x) / 32;
    const int64_t nwarps = (int64_t)gridDim.x * blockDim.x / 32;
    const int chunks = a.C / 8;
    for (int64_t g0 = warp0 * RW; g0 < rows; g0 += nwarps * RW) {
        uint4 raw[R][CH];
        float s2[R], mean[R], rinv[R];
#pragma unroll
        for (int q = 0; q < R; ++q) {
            const int64_t g = g0 + q * (32 / LW) + slot;
#pragma unroll
            for (int j = 0; j < CH; ++j) raw[q][j] = make_uint4(0, 0, 0, 0);
            if (g >= rows) continue;
            const int p = (int)(g / a.M);
            const int64_t m = g % a.M;
            const __nv_bfloat16* xr =
                static_cast<const __nv_bfloat16*>(a.x) + ((a.x_batched ? (int64_t)p : 0) * a.M + m) * a.C;
#pragma unroll
            for (int j = 0; j < CH; ++j) {
                const int c = lane + LW * j;
                if (c < chunks) raw[q][j] = *reinterpret_cast<const uint4*>(xr + 8 * c);
            }
        }
#pragma unroll
        for (int q = 0; q < R; ++q) {
            float s1 = 0.f;
            mean[q] = 0.f;
            s2[q] = 0.f;
            if (a.kind == NORM_LAYER) {
#pragma unroll
                for (int j = 0; j < CH; ++j)
                    if (lane + LW * j < chunks) {
                        float f[8];
                        bf16x8_to_f32(raw[q][j], f);
#pragma unroll
                        for (int i = 0; i < 8; ++i) s1 += f[i];
                    }
                mean[q] = group_sum<LW>(s1) * a.inv_c;
#pragma unroll
                for (int j = 0; j < CH; ++j)
                    if (lane + LW * j < chunks) {
                        float f[8];
                        bf16x8_to_f32(raw[q][j], f);
#pragma unroll
                        for (int i = 0; i < 8; ++i) {
                            const float d = f[i] - mean[q];
                            s2[q] = fmaf(d, d, s2[q]);
                        }
                    }
            } else {
#pragma unroll
                for (int j = 0; j < CH; ++j)
                    if (lane + LW * j < chunks) {
                        float f[8];
                        bf16x8_to_f32(raw[q][j], f);
#pragma unroll
                        for (int i = 0; i < 8; ++i) s2[q] = fmaf(f[i], f[i], s2[q]);
                    }
            }
            rinv[q] = rsqrtf(group_sum<LW>(s2[q]) * a.inv_c + a.eps);
        }
#pragma unroll
        for (int q = 0; q < R; ++q) {
            const int64_t g = g0 + q * (32 / LW) + slot;
            if (g >= rows) continue;
            const int p = (int)(g / a.M);
            const __nv_bfloat16* sr = static_cast<const __nv_bfloat16*>(a.scale) + (a.p_batched ? (int64_t)p : 0) * a.C;
            const __nv_bfloat16* br =
                a.bias ? static_cast<const __nv_bfloat16*>(a.bias) + (a.p_batched ? (int64_t)p : 0) * a.C : nullptr;
            __nv_bfloat16* yr = static_cast<__nv_bfloat16*>(a.y) + g * a.C;
#pragma unroll
            for (int j = 0; j < CH; ++j) {
                const int c = lane + LW * j;
                if (c < chunks) {
                    float f[8], sc[8], bi[8], o[8];
                    bf16x8_to_f32(raw[q][j], f);
                    load8(sr + 8 * c, sc);
                    if (br) load8(br + 8 * c, bi);
#pragma unroll
                    for (int i = 0; i < 8; ++i) {
                        o[i] = __fmul_rn(__fmul_rn(f[i] - mean[q], rinv[q]), sc[i]);
                        if (br) o[i] = __fadd_rn(o[i], bi[i]);
                    }
                    store8(yr + 8 * c, o);
                }
            }
        }
    }
}

// Any C and alignment: three passes over the row in global memory (the
// second and third hit L1/L2).
template <typename T>
__global__ void norm_any_kernel(const NormArgs a) {
    const int lane = threadIdx.x % 32;
    const int64_t rows = (int64_t)a.P * a.M;
    const int64_t warp0 = ((int64_t)blockIdx.x * blockDim.x + threadIdx.x) / 32;
    const int64_t nwarps = (int64_t)gridDim.x * blockDim.x / 32;
    for (int64_t g = warp0; g < rows; g += nwarps) {
        const int p = (int)(g / a.M);
        const int64_t m = g % a.M;
        const T* xr = static_cast<const T*>(a.x) + ((a.x_batched ? (int64_t)p : 0) * a.M + m) * a.C;
        const T* sr = static_cast<const T*>(a.scale) + (a.p_batched ? (int64_t)p : 0) * a.C;
        const T* br = a.bias ? static_cast<const T*>(a.bias) + (a.p_batched ? (int64_t)p : 0) * a.C : nullptr;
        T* yr = static_cast<T*>(a.y) + g * a.C;
        float mean = 0.f, s2 = 0.f;
        if (a.kind == NORM_LAYER) {
            float s1 = 0.f;
            for (int c = lane; c < a.C; c += 32) s1 += zg_to_float(xr[c]);
            mean = warp_sum(s1) * a.inv_c;
            for (int c = lane; c < a.C; c += 32) {
                const float d = zg_to_float(xr[c]) - mean;
                s2 = fmaf(d, d, s2);
            }
        } else {
            for (int c = lane; c < a.C; c += 32) {
                const float xv = zg_to_float(xr[c]);
                s2 = fmaf(xv, xv, s2);
            }
        }
        const float rinv = rsqrtf(warp_sum(s2) * a.inv_c + a.eps);
        for (int c = lane; c < a.C; c += 32) {
            float o = __fmul_rn(__fmul_rn(zg_to_float(xr[c]) - mean, rinv), zg_to_float(sr[c]));
            if (br) o = __fadd_rn(o, zg_to_float(br[c]));
            yr[c] = zg_from_float<T>(o);
        }
    }
}

int sm_count_norm() {
    static int n = 0;
    if (n == 0) {
        int dev = 0;
        cudaGetDevice(&dev);
        if (cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess || n < 1) n = 148;
    }
    return n;
}

template <typename T>
int launch_norm(const NormArgs& a, cudaStream_t st, const char* name) {
    const int64_t rows = (int64_t)a.P * a.M;
    auto al = [](const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15) == 0; };
    const bool vec = a.C % 8 == 0 && al(a.x) && al(a.scale) && (!a.bias || al(a.bias)) && al(a.y);
    // rows per warp pass: two for the register-resident widths up to 1024
    const int R = vec && a.C <= 1024 ? 2 : 1;
    int64_t blocks = (rows + 8 * R - 1) / (8 * R);  // 8 warps per block
    if (blocks > (int64_t)sm_count_norm() * 16) blocks = (int64_t)sm_count_norm() * 16;
    if (blocks < 1) blocks = 1;
    if constexpr (sizeof(T) == 2) {
        if (vec && a.C <= 1024) {
            // bf16 rows held packed: up to C = 768 half a warp per row (four
            // or eight rows per warp), above it a whole warp (four rows)
            int64_t b4 = (rows + 8 * 4 - 1) / (8 * 4);
            if (b4 > (int64_t)sm_count_norm() * 16) b4 = (int64_t)sm_count_norm() * 16;
            if (b4 < 1) b4 = 1;
            zg::LaunchTimer zg_lt_(name, st);
            if (a.C <= 256) norm_packed_kernel<2, 4, 16><<<(unsigned)b4, 256, 0, st>>>(a);
            else if (a.C <= 384) norm_packed_kernel<3, 2, 16><<<(unsigned)b4, 256, 0, st>>>(a);
            else if (a.C <= 512) norm_packed_kernel<4, 2, 16><<<(unsigned)b4, 256, 0, st>>>(a);
            else if (a.C <= 768) norm_packed_kernel<6, 2, 16><<<(unsigned)b4, 256, 0, st>>>(a);
            else norm_packed_kernel<4, 4><<<(unsigned)b4, 256, 0, st>>>(a);
            return zg::check_launch(name);
        }
    }
    zg::LaunchTimer zg_lt_(name, st);
    if (vec && a.C <= 256)
        norm_reg_kernel<T, 1, 2><<<(unsigned)blocks, 256, 0, st>>>(a);
    else if (vec && a.C <= 512)
        norm_reg_kernel<T, 2, 2><<<(unsigned)blocks, 256, 0, st>>>(a);
    else if (vec && a.C <= 768)
        norm_reg_kernel<T, 3, 2><<<(unsigned)blocks, 256, 0, st>>>(a);
    else if (vec && a.C <= 1024)
        norm_reg_kernel<T, 4, 2><<<(unsigned)blocks, 256, 0, st>>>(a);
    else if (vec && a.C <= 2048)
        norm_reg_kernel<T, 8, 1><<<(unsigned)blocks, 256, 0, st>>>(a);
    else
        norm_any_kernel<T><<<(unsigned)blocks, 256, 0, st>>>(a);
    return zg::check_launch(name);
}

int norm_entry(const char* who, int kind, const void* x, int x_batched, const void* scale, const void* bias,
               int p_batched, int P, int64_t M, int C, float eps, int dtype, void* y, void* stream) {
    if (P < 1 || M < 0 || C < 1) return zg::fail(ZG_ERR_INVALID, "%s: bad sizes", who);
    if (!(eps >= 0.f)) return zg::fail(ZG_ERR_INVALID, "%s: eps must be >= 0", who);
    if (!zg::dtype_ok(dtype)) return zg::fail(ZG_ERR_INVALID, "%s: bad dtype", who);
    if (M == 0) return ZG_OK;
    if (!x || !scale || !y) return zg::fail(ZG_ERR_INVALID, "%s: null pointer", who);
    NormArgs a{x, scale, bias, y, M, P, C, x_batched != 0, p_batched != 0, kind, eps, 1.f / (float)C};
    cudaStream_t st = zg::as_stream(stream);
    return dtype == ZG_BF16 ? launch_norm<__nv_bfloat16>(a, st, who) : launch_norm<float>(a, st, who);
}

}  // namespace

extern "C" int zg_layer_norm(const void* x, int x_batched, const void* scale, const void* bias, int p_batched,
                             int P, int64_t M, int C, float eps, int dtype, void* y, void* stream) {
    return norm_entry("layer_norm", NORM_LAYER, x, x_batched, scale, bias, p_batched, P, M, C, eps, dtype, y,
                      stream);
}

extern "C" int zg_rms_norm(const void* x, int x_batched, const void* scale, int p_batched, int P, int64_t M, int C,
                           float eps, int dtype, void* y, void* stream) {
    return norm_entry("rms_norm", NORM_RMS, x, x_batched, scale, nullptr, p_batched, P, M, C, eps, dtype, y, stream);
}

// ---------------------------------------------------------------------------
// Element-wise GELU (tanh form), the unfused twin of the forward GEMM's
// ZG_ACT_GELU epilogue: y = round_dtype(gelu(float(x))), same device function.
// ---------------------------------------------------------------------------
namespace {

__global__ void gelu_bf16x8_kernel(const uint4* __restrict__ x, uint4* __restrict__ y, int64_t n8) {
    for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n8; i += (int64_t)gridDim.x * blockDim.x) {
        uint4 v = x[i];
        __nv_bfloat162* h = reinterpret_cast<__nv_bfloat162*>(&v);
#pragma unroll
        for (int j = 0; j < 4; ++j)
            h[j] = __floats2bfloat162_rn(zg_gelu_tanh(__bfloat162float(h[j].x)), zg_gelu_tanh(__bfloat162float(h[j].y)));
        y[i] = v;
    }
}

template <typename T>
__global__ void gelu_kernel(const T* __restrict__ x, T* __restrict__ y, int64_t n) {
    for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += (int64_t)gridDim.x * blockDim.x)
        y[i] = zg_from_float<T>(zg_gelu_tanh(zg_to_float(x[i])));
}

}  // namespace

extern "C" int zg_gelu(const void* x, void* y, int64_t n, int dtype, void* stream) {
    if (n < 0) return zg::fail(ZG_ERR_INVALID, "zg_gelu: bad size");
    if (!zg::dtype_ok(dtype)) return zg::fail(ZG_ERR_INVALID, "zg_gelu: bad dtype");
    if (n == 0) return ZG_OK;
    if (!x || !y) return zg::fail(ZG_ERR_INVALID, "zg_gelu: null pointer");
    cudaStream_t st = zg::as_stream(stream);
    int dev = 0, sms = 148;
    cudaGetDevice(&dev);
    cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
    auto al = [](const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15) == 0; };
    zg::LaunchTimer zg_lt_("gelu", st);
    if (dtype == ZG_BF16 && n % 8 == 0 && al(x) && al(y)) {
        const int64_t n8 = n / 8;
        int64_t blocks = (n8 + 255) / 256;
        if (blocks > (int64_t)sms * 16) blocks = (int64_t)sms * 16;
        gelu_bf16x8_kernel<<<(unsigned)blocks, 256, 0, st>>>(static_cast<const uint4*>(x), static_cast<uint4*>(y), n8);
        return zg::check_launch("zg_gelu");
    }
    int64_t blocks = (n + 255) / 256;
    if (blocks > (int64_t)sms * 16) blocks = (int64_t)sms * 16;
    if (dtype == ZG_BF16)
        gelu_kernel<__nv_bfloat16><<<(unsigned)blocks, 256, 0, st>>>(static_cast<const __nv_bfloat16*>(x),
                                                                      static_cast<__nv_bfloat16*>(y), n);
    else
        gelu_kernel<float><<<(unsigned)blocks, 256, 0, st>>>(static_cast<const float*>(x), static_cast<float*>(y), n);
    return zg::check_launch("zg_gelu");
}
