// zg_common.cuh -- shared device helpers for libzgb200 (sm_100a).
//
// Device restatement of the key/factor arithmetic of the reference
// (src/zerograd/_keys.py:20-58, src/zerograd/_factors.py:30-74), i.e. of
// jax.random's partitionable threefry2x32 / uniform / normal in float32.
#pragma once
#include <cuda_runtime.h>
#include <cuda_bf16.h>
#include <stdint.h>
#include <stddef.h>

#include "../../include/zg_b200.h"

// ---------------------------------------------------------------------------
// error state (per host thread)
// ---------------------------------------------------------------------------
namespace zg {

void set_error(const char* fmt, ...);
int fail(int code, const char* fmt, ...);
int check_launch(const char* what);

inline cudaStream_t as_stream(void* s) { return reinterpret_cast<cudaStream_t>(s); }

// Counts every launch and, while profiling is on, brackets it with CUDA
// events on the launching stream.  Construct right before a <<<>>> launch.
struct LaunchTimer {
    LaunchTimer(const char* name, cudaStream_t st);
    ~LaunchTimer();
    int slot = -1;
    cudaStream_t stream;
};

// Round a float to bfloat16 (nearest even) and back, on the host.
inline float host_round_bf16(float x) {
    uint32_t u;
    memcpy(&u, &x, 4);
    if ((u & 0x7F800000u) == 0x7F800000u) {
        if (u & 0x007FFFFFu) u |= 0x00400000u;
        u &= 0xFFFF0000u;
    } else {
        u += 0x7FFFu + ((u >> 16) & 1u);
        u &= 0xFFFF0000u;
    }
    float f;
    memcpy(&f, &u, 4);
    return f;
}

inline size_t dtype_size(int dt) { return dt == ZG_BF16 ? 2 : 4; }
inline bool dtype_ok(int dt) { return dt == ZG_F32 || dt == ZG_BF16; }

inline size_t align_up(size_t v, size_t a) { return (v + a - 1) / a * a; }

// Carves sub-buffers out of a caller-provided workspace.
struct Carver {
    char* base;
    size_t cap, used = 0;
    Carver(void* b, size_t c) : base(static_cast<char*>(b)), cap(c) {}
    template <typename T>
    T* take(size_t count) {
        size_t off = align_up(used, 256);
        used = off + count * sizeof(T);
        return used <= cap && base ? reinterpret_cast<T*>(base + off) : nullptr;
    }
    static size_t need(std::initializer_list<size_t> bytes) {
        size_t u = 0;
        for (size_t b : bytes) u = align_up(u, 256) + b;
        return u;
    }
};

}  // namespace zg

// ---------------------------------------------------------------------------
// threefry2x32-20 (Salmon et al., SC'11) in the word order jax uses:
// key (k0,k1), counter (c0,c1); ks2 = k0 ^ k1 ^ 0x1BD11BDA.
// ---------------------------------------------------------------------------
struct ZgKey {
    uint32_t k0, k1, k2;
};

__host__ __device__ __forceinline__ ZgKey zg_make_key(uint32_t k0, uint32_t k1) {
    return ZgKey{k0, k1, k0 ^ k1 ^ 0x1BD11BDAu};
}

#define ZG_TF_ROUND(r)                     \
    x0 += x1;                              \
    x1 = __funnelshift_l(x1, x1, (r));     \
    x1 ^= x0;

__device__ __forceinline__ uint2 zg_threefry(const ZgKey& k, uint32_t c0, uint32_t c1) {
    uint32_t x0 = c0 + k.k0, x1 = c1 + k.k1;
    ZG_TF_ROUND(13) ZG_TF_ROUND(15) ZG_TF_ROUND(26) ZG_TF_ROUND(6)
    x0 += k.k1; x1 += k.k2 + 1u;
    ZG_TF_ROUND(17) ZG_TF_ROUND(29) ZG_TF_ROUND(16) ZG_TF_ROUND(24)
    x0 += k.k2; x1 += k.k0 + 2u;
    ZG_TF_ROUND(13) ZG_TF_ROUND(15) ZG_TF_ROUND(26) ZG_TF_ROUND(6)
    x0 += k.k0; x1 += k.k1 + 3u;
    ZG_TF_ROUND(17) ZG_TF_ROUND(29) ZG_TF_ROUND(16) ZG_TF_ROUND(24)
    x0 += k.k1; x1 += k.k2 + 4u;
    ZG_TF_ROUND(13) ZG_TF_ROUND(15) ZG_TF_ROUND(26) ZG_TF_ROUND(6)
    x0 += k.k2; x1 += k.k0 + 5u;
    return make_uint2(x0, x1);
}

// fold_in(key, d) == split(key, n)[d] under partitionable threefry.
__device__ __forceinline__ ZgKey zg_fold(const ZgKey& k, uint32_t d) {
    uint2 o = zg_threefry(k, 0u, d);
    return zg_make_key(o.x, o.y);
}

// 32 random bits of flat element j.
__device__ __forceinline__ uint32_t zg_bits(const ZgKey& k, uint64_t j) {
    uint2 o = zg_threefry(k, (uint32_t)(j >> 32), (uint32_t)j);
    return o.x ^ o.y;
}

// Giles' single-precision erfinv (published polynomial, explicit FMA Horner
// steps) on CUDA's log1pf / sqrtf.
__device__ __forceinline__ float zg_erfinv(float x) {
    float w = -log1pf(-x * x);
    float p;
    if (w < 5.0f) {
        w = w - 2.5f;
        p = 2.81022636e-08f;
        p = __fmaf_rn(p, w, 3.43273939e-07f);
        p = __fmaf_rn(p, w, -3.5233877e-06f);
        p = __fmaf_rn(p, w, -4.39150654e-06f);
        p = __fmaf_rn(p, w, 0.00021858087f);
        p = __fmaf_rn(p, w, -0.00125372503f);
        p = __fmaf_rn(p, w, -0.00417768164f);
        p = __fmaf_rn(p, w, 0.246640727f);
        p = __fmaf_rn(p, w, 1.50140941f);
    } else {
        w = sqrtf(w) - 3.0f;
        p = -0.000200214257f;
        p = __fmaf_rn(p, w, 0.000100950558f);
        p = __fmaf_rn(p, w, 0.00134934322f);
        p = __fmaf_rn(p, w, -0.00367342844f);
        p = __fmaf_rn(p, w, 0.00573950773f);
        p = __fmaf_rn(p, w, -0.0076224613f);
        p = __fmaf_rn(p, w, 0.00943887047f);
        p = __fmaf_rn(p, w, 1.00167406f);
        p = __fmaf_rn(p, w, 2.83297682f);
    }
    return __fmul_rn(p, x);
}

// Bits -> float32 standard normal: uniform in [nextafter(-1,0), 1) by the
// mantissa trick (span 2.0f after float32 rounding), then sqrt(2)*erfinv.
__device__ __forceinline__ float zg_normal_from_bits(uint32_t bits) {
    const float lo = __uint_as_float(0xBF7FFFFFu);
    float f = __uint_as_float((bits >> 9) | 0x3F800000u) - 1.0f;
    float u = fmaxf(__fmaf_rn(f, 2.0f, lo), lo);
    return __fmul_rn(1.41421356237309504880f, zg_erfinv(u));
}

__device__ __forceinline__ float zg_normal(const ZgKey& k, uint64_t j) {
    return zg_normal_from_bits(zg_bits(k, j));
}
// Storage helpers: the factor value of a bf16 leaf is the float32 draw cast
// to bf16 (src/zerograd/_factors.py:48-55).
template <typename T>
__device__ __forceinline__ T zg_from_float(float v);
template <>
__device__ __forceinline__ float zg_from_float<float>(float v) { return v; }
template <>
__device__ __forceinline__ __nv_bfloat16 zg_from_float<__nv_bfloat16>(float v) { return __float2bfloat16_rn(v); }

__device__ __forceinline__ float zg_to_float(float v) { return v; }
__device__ __forceinline__ float zg_to_float(__nv_bfloat16 v) { return __bfloat162float(v); }

// Round a float draw to the storage dtype and back (value the reference sees).
template <typename T>
__device__ __forceinline__ float zg_dtype_round(float v) { return zg_to_float(zg_from_float<T>(v)); }

// Derives the (A, B) factor keys of one candidate for one manifest group:
// group key = fold(candidate key, group); (ka, kb) = split(group key).
struct ZgFactorKeys {
    ZgKey a, b;
};
__device__ __forceinline__ ZgFactorKeys zg_factor_keys(const uint32_t* cand_keys, int p, int group) {
    ZgKey ck = zg_make_key(cand_keys[2 * p], cand_keys[2 * p + 1]);
    ZgKey gk = group >= 0 ? zg_fold(ck, (uint32_t)group) : ck;
    return ZgFactorKeys{zg_fold(gk, 0u), zg_fold(gk, 1u)};
}
__device__ __forceinline__ ZgKey zg_group_key(const uint32_t* cand_keys, int p, int group) {
    ZgKey ck = zg_make_key(cand_keys[2 * p], cand_keys[2 * p + 1]);
    return group >= 0 ? zg_fold(ck, (uint32_t)group) : ck;
}

// Eight bf16 values (one 16-byte load) as float32.
__device__ __forceinline__ void bf16x8_to_f32(const uint4& v, float (&f)[8]) {
    const uint32_t w[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
    for (int i = 0; i < 4; ++i) {
        f[2 * i] = __uint_as_float(w[i] << 16);
        f[2 * i + 1] = __uint_as_float(w[i] & 0xFFFF0000u);
    }
}

// ---------------------------------------------------------------------------
// Activation and residual epilogue of the population forward.
// ---------------------------------------------------------------------------
// GELU in the tanh form of Hendrycks & Gimpel (arXiv:1606.08415, the form
// GPT-2 uses): 0.5 x (1 + tanh(u)), u = sqrt(2/pi) (x + 0.044715 x^3),
// evaluated as x * sigmoid(2u) = x / (1 + 2^(-2u log2 e)), which keeps its
// relative accuracy on the negative tail where 1 + tanh(u) cancels.
__device__ __forceinline__ float zg_gelu_tanh(float x) {
    const float u = x * fmaf(0.044715f * 0.7978845608028654f, x * x, 0.7978845608028654f);
    float e;
    asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(e) : "f"(u * (-2.f * 1.4426950408889634f)));
    return __fdividef(x, 1.f + e);
}

// One output element: y = bf16(v); with `act` (ZG_ACT_GELU) y = bf16(gelu(y));
// with a residual r, y = bf16(r + y): the roundings of the unfused ops (the
// linear's bf16 output, an element-wise activation of it, a bf16 residual add).
__device__ __forceinline__ float zg_epilogue_value(float v, int act, bool has_res, float r) {
    if (act || has_res) v = __bfloat162float(__float2bfloat16_rn(v));
    if (act == ZG_ACT_GELU) {
        v = zg_gelu_tanh(v);
        if (has_res) v = __bfloat162float(__float2bfloat16_rn(v));
    }
    return has_res ? r + v : v;
}

// Two neighbouring outputs, the same values as zg_epilogue_value on each:
// the intermediate bf16 roundings go through the paired conversion (one
// instruction for both, off the special-function pipe that the single
// conversion and the GELU's exp2 and reciprocal share).
__device__ __forceinline__ float2 zg_round_pair(float a, float b) {
    const __nv_bfloat162 h = __floats2bfloat162_rn(a, b);
    return make_float2(__low2float(h), __high2float(h));
}
__device__ __forceinline__ float2 zg_epilogue_pair(float a, float b, int act, bool has_res, float ra, float rb) {
    float2 v = (act || has_res) ? zg_round_pair(a, b) : make_float2(a, b);
    if (act == ZG_ACT_GELU) {
        v.x = zg_gelu_tanh(v.x);
        v.y = zg_gelu_tanh(v.y);
        if (has_res) v = zg_round_pair(v.x, v.y);
    }
    if (has_res) {
        v.x = ra + v.x;
        v.y = rb + v.y;
    }
    return v;
}

// One thread's 32 consecutive outputs of a row, written straight to global
// memory (zg_epilogue_value per element).  d and r 16-byte aligned; `n`
// valid columns (32 or more take the vector path).
__device__ __forceinline__ void zg_store_row32(const float (&v)[32], __nv_bfloat16* d, const __nv_bfloat16* r,
                                               int act, int n) {
    if (n >= 32) {
        uint4 rv[4];
        if (r) {
#pragma unroll
            for (int i = 0; i < 4; ++i) rv[i] = reinterpret_cast<const uint4*>(r)[i];
        }
#pragma unroll
        for (int i = 0; i < 32; i += 8) {
            __nv_bfloat162 h[4];
#pragma unroll
            for (int j = 0; j < 4; ++j) {
                float r0 = 0.f, r1 = 0.f;
                if (r) {
                    const __nv_bfloat162 rr = reinterpret_cast<const __nv_bfloat162*>(&rv[i / 8])[j];
                    r0 = __bfloat162float(rr.x);
                    r1 = __bfloat162float(rr.y);
                }
                const float2 o = zg_epilogue_pair(v[i + 2 * j], v[i + 2 * j + 1], act, r != nullptr, r0, r1);
                h[j] = __floats2bfloat162_rn(o.x, o.y);
            }
            *reinterpret_cast<uint4*>(d + i) = *reinterpret_cast<uint4*>(h);
        }
        return;
    }
    // ragged end of a row: unrolled with a guard, so v stays in registers
#pragma unroll
    for (int i = 0; i < 32; ++i) {
        if (i >= n) break;
        d[i] = __float2bfloat16_rn(zg_epilogue_value(v[i], act, r != nullptr, r ? __bfloat162float(r[i]) : 0.f));
    }
}
