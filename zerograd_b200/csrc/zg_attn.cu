// zg_attn.cu -- softmax attention of every candidate's transformer block,
// population-batched: for every z (candidate x batch row), head h and query i
//
//   o[z, i, h] = sum_j softmax_j(q[z, i, h] . k[z, j, h] / sqrt(D)) v[z, j, h]
//
// (examples/train_vit_cifar10.py:166-172; causal for the decoder LM: keys
// j > i masked).  q, k, v, o are [Z, S, H, D], the head-interleaved layout
// the q/k/v projections produce, so no transpose is materialised.
//
// Tensor-core path (bf16, D = 64, S <= 256): one CTA per (128-query tile,
// head, z).  TMA brings the query tile and the whole key and value sequence
// (4-D tensor maps over [Z, S, H, D], 128-byte swizzle); one tcgen05 MMA
// chain computes the scores S = Q K^T into TMEM (M=128, N=128 or 256); each
// thread owns one query row, takes its max over the row in TMEM and writes
// p = 2^(s * log2(e)/sqrt(D) - max) as bf16 into shared memory in the MMA's
// K-major swizzled layout (over the finished Q and K tiles); a second MMA
// chain computes O = P V (V as the MN-major operand) into the first 64 TMEM
// columns; the epilogue divides by the row sum of the bf16 p and stores O.
// The whole score row fits (S <= 256), so one pass suffices.
//
// Other shapes (D != 64, S > 256, float32): a warp per query row with an
// online softmax over the keys (float32 arithmetic).
#include <math.h>

#include "zg_ptx.cuh"
#include "zg_tc.cuh"

namespace {

constexpr int AT_THREADS = 256;  // two threads per query row, each half of the key columns
constexpr uint32_t AT_Q = 0;                // 16 KiB: 128 query rows x 128 B
constexpr uint32_t AT_K = 16384;            // 32 KiB: up to 256 key rows
constexpr uint32_t AT_V = 65536;            // 32 KiB: up to 256 value rows
constexpr uint32_t AT_P = 0;                // 64 KiB over Q, K and the gap: P [128, 256] bf16, 4 K-blocks
constexpr uint32_t AT_O = 0;                // 16 KiB over P once P V is done: the output tile [128, 64] bf16
constexpr uint32_t AT_SMEM = 65536 + 32768; // 96 KiB

__device__ __forceinline__ float ex2_approx(float x) {
    float y;
    asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
    return y;
}

struct AttnArgs {
    __nv_bfloat16* o;
    int Z, S, H, s_pad, causal;
    float scale_log2;  // log2(e) / sqrt(D)
};

__global__ void __launch_bounds__(AT_THREADS, 2)
attn_tc_kernel(const __grid_constant__ CUtensorMap tmQ, const __grid_constant__ CUtensorMap tmK,
               const __grid_constant__ CUtensorMap tmV, const __grid_constant__ CUtensorMap tmO, const AttnArgs a) {
    extern __shared__ uint8_t dyn_smem[];
    __shared__ __align__(8) uint64_t load_bar, mma_bar;
    __shared__ uint32_t tmem_base_sh;
    __shared__ float s_red[2][128];  // the two column halves' row max, then row sum
    const uint32_t dyn_base = smem_u32(dyn_smem);
    uint8_t* smem = dyn_smem + (((dyn_base + 1023u) & ~1023u) - dyn_base);
    const int t = threadIdx.x, warp = t / 32, lane = t % 32;
    const int quad = warp % 4, half = warp / 4;  // TMEM lane quadrant; key-column half
    const int r = quad * 32 + lane;              // this thread's query row in the tile
    const int qt = blockIdx.x, h = blockIdx.y, z = blockIdx.z;
    const int q0 = qt * 128;
    // keys this query tile can see: causal tiles stop at their last query
    const int n_keys = a.causal && q0 + 128 < a.s_pad ? q0 + 128 : a.s_pad;
    const int kboxes = n_keys / 128;

    if (t == 0) {
        mbar_init(&load_bar, 1);
        mbar_init(&mma_bar, 1);
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    }
    if (warp == 0) tmem_alloc(&tmem_base_sh, 256);
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = tmem_base_sh;
    bool ok = true;

    if (t == 0) {
        mbar_expect_tx(&load_bar, (1 + 2 * kboxes) * 16384);
        tma_load_4d(smem + AT_Q, &tmQ, &load_bar, 0, h, q0, z);
        for (int b = 0; b < kboxes; ++b) {
            tma_load_4d(smem + AT_K + b * 16384, &tmK, &load_bar, 0, h, b * 128, z);
            tma_load_4d(smem + AT_V + b * 16384, &tmV, &load_bar, 0, h, b * 128, z);
        }
        if (mbar_wait(&load_bar, 0, 81)) {
            tc_fence_after();
            const uint32_t idesc = idesc_bf16(128, n_keys, 0);
            const uint32_t qa = smem_u32(smem + AT_Q), ka = smem_u32(smem + AT_K);
#pragma unroll
            for (int k = 0; k < 4; ++k)
                umma_bf16(tmem, smem_desc(qa + k * 32, 16, 1024), smem_desc(ka + k * 32, 16, 1024), idesc,
                          k > 0 ? 1u : 0u);
            umma_commit(&mma_bar);
        }
    }
    ok = mbar_wait(&mma_bar, 0, 82);
    tc_fence_after();

    // ---- softmax: this thread's row, its half of the key columns ----
    const int qi = q0 + r;
    const uint32_t trow = tmem + ((uint32_t)(quad * 32) << 16);
    // columns [0, vis) are visible to this query: the keys, up to the query when causal
    const int vis = a.causal ? (qi + 1 < a.S ? qi + 1 : a.S) : a.S;
    // the warp's last visible column (its last row sees the most): chunks past it hold no weight
    const int wvis = __reduce_max_sync(0xffffffffu, vis);
    const int hw = n_keys / 2, c_lo = half * hw, c_hi = c_lo + hw;
    const int c_end = wvis < c_hi ? ((wvis - c_lo + 31) / 32) * 32 + c_lo : c_hi;  // chunks to evaluate
    float mx = -INFINITY;
    for (int c = c_lo; c < c_end; c += 32) {
        float v[32];
        tmem_ld32(trow + c, v);
        if (c + 32 <= vis) {
#pragma unroll
            for (int j = 0; j < 32; ++j) mx = fmaxf(mx, v[j]);
        } else {
#pragma unroll
            for (int j = 0; j < 32; ++j)
                if (c + j < vis) mx = fmaxf(mx, v[j]);
        }
    }
    s_red[half][r] = mx;
    __syncthreads();
    mx = fmaxf(s_red[0][r], s_red[1][r]) * a.scale_log2;  // scale_log2 > 0: max(s) * scale = max(s * scale)
    float sum = 0.f;
    for (int c = c_lo; c < c_hi; c += 32) {
        uint32_t pk[16];
        if (c < c_end) {
            float v[32];
            tmem_ld32(trow + c, v);
            const bool full = c + 32 <= vis;
#pragma unroll
            for (int j = 0; j < 16; ++j) {
                float pe[2];
#pragma unroll
                for (int e = 0; e < 2; ++e) {
                    const int col = c + 2 * j + e;
                    pe[e] = full || col < vis ? ex2_approx(fmaf(v[2 * j + e], a.scale_log2, -mx)) : 0.f;
                }
                const __nv_bfloat162 b2 = __floats2bfloat162_rn(pe[0], pe[1]);
                sum += __low2float(b2) + __high2float(b2);  // the weights the PV product uses
                pk[j] = *reinterpret_cast<const uint32_t*>(&b2);
            }
        } else {
#pragma unroll
            for (int j = 0; j < 16; ++j) pk[j] = 0u;  // masked keys: zero weight
        }
        // P is the K-major, 128-byte swizzled A operand: 64-column blocks of
        // [128 rows x 128 B], 16-byte chunk ch of row r at (ch ^ (r & 7)) * 16
        uint8_t* blk = smem + AT_P + (c / 64) * 16384 + r * 128;
#pragma unroll
        for (int i = 0; i < 4; ++i) {
            const int ch = (c % 64) / 8 + i;
            *reinterpret_cast<uint4*>(blk + ((ch ^ (r & 7)) * 16)) =
                make_uint4(pk[4 * i], pk[4 * i + 1], pk[4 * i + 2], pk[4 * i + 3]);
        }
    }
    asm volatile("fence.proxy.async.shared::cta;" ::: "memory");  // P visible to the tensor cores
    tc_fence_before();
    __syncthreads();  // every thread's max is read (s_red reusable), P complete
    tc_fence_after();
    s_red[half][r] = sum;

    if (t == 0 && ok) {
        const uint32_t idesc = idesc_bf16(128, 64, 1);
        const uint32_t pa = smem_u32(smem + AT_P), va = smem_u32(smem + AT_V);
        for (int kk = 0; kk < n_keys / 16; ++kk)
            umma_bf16(tmem, smem_desc(pa + (kk / 4) * 16384 + (kk % 4) * 32, 16, 1024),
                      smem_desc(va + kk * 2048, 64 * 256 * 2, 1024), idesc, kk > 0 ? 1u : 0u);
        umma_commit(&mma_bar);
    }
    ok = ok && mbar_wait(&mma_bar, 1, 83);
    tc_fence_after();
    __syncthreads();  // both halves' sums are in s_red; P is consumed by the MMA
    {
        // O / sum -> bf16 into the staging tile (over P; 128-byte swizzle,
        // the layout of the output box), then one TMA store
        float o[32];
        tmem_ld32(trow + half * 32, o);
        const float inv = 1.f / (s_red[0][r] + s_red[1][r]);
        uint8_t* row = smem + AT_O + r * 128;
#pragma unroll
        for (int i = 0; i < 4; ++i) {
            uint4 pk;
            __nv_bfloat162* hp = reinterpret_cast<__nv_bfloat162*>(&pk);
#pragma unroll
            for (int e = 0; e < 4; ++e) hp[e] = __floats2bfloat162_rn(o[8 * i + 2 * e] * inv, o[8 * i + 2 * e + 1] * inv);
            const int ch = half * 4 + i;
            *reinterpret_cast<uint4*>(row + ((ch ^ (r & 7)) * 16)) = pk;
        }
    }
    asm volatile("fence.proxy.async.shared::cta;" ::: "memory");  // staging visible to the bulk store
    tc_fence_before();
    __syncthreads();
    if (t == 0) {
        if (ok) {
            tma_store_4d(&tmO, smem + AT_O, 0, h, q0, z);  // rows past S are clipped
            asm volatile("cp.async.bulk.commit_group;" ::: "memory");
        }
        asm volatile("cp.async.bulk.wait_group 0;" ::: "memory");
    }
    __syncthreads();
    if (warp == 0) tmem_dealloc(tmem, 256);
}

// Generic path: one warp per (z, query, head); lane d-slices of the head
// dimension, online softmax over the keys, float32 arithmetic.
template <typename T>
__global__ void attn_simt_kernel(const T* __restrict__ q, const T* __restrict__ k, const T* __restrict__ v,
                                 T* __restrict__ o, int Z, int S, int H, int D, int causal, float scale, int64_t ld) {
    const int lane = threadIdx.x % 32;
    const int64_t rows = (int64_t)Z * S * H;
    const int64_t w0 = ((int64_t)blockIdx.x * blockDim.x + threadIdx.x) / 32;
    const int64_t nw = (int64_t)gridDim.x * blockDim.x / 32;
    for (int64_t r = w0; r < rows; r += nw) {
        const int h = (int)(r % H);
        const int qi = (int)((r / H) % S);
        const int64_t z = r / ((int64_t)H * S);
        const T* qr = q + (z * S + qi) * ld + (int64_t)h * D;
        float qv[8], acc[8];
        for (int i = 0; i < 8; ++i) {
            const int d = lane + 32 * i;
            qv[i] = d < D ? zg_to_float(qr[d]) : 0.f;
            acc[i] = 0.f;
        }
        float mx = -INFINITY, den = 0.f;
        const int jend = causal ? qi + 1 : S;
        for (int j = 0; j < jend; ++j) {
            const T* kr = k + (z * S + j) * ld + (int64_t)h * D;
            float s = 0.f;
            for (int i = 0; i < 8; ++i) {
                const int d = lane + 32 * i;
                if (d < D) s = fmaf(qv[i], zg_to_float(kr[d]), s);
            }
#pragma unroll
            for (int off = 16; off > 0; off >>= 1) s += __shfl_xor_sync(0xffffffffu, s, off);
            s *= scale;
            const float m2 = fmaxf(mx, s);
            const float corr = expf(mx - m2), p = expf(s - m2);
            den = den * corr + p;
            const T* vr = v + (z * S + j) * ld + (int64_t)h * D;
            for (int i = 0; i < 8; ++i) {
                const int d = lane + 32 * i;
                if (d < D) acc[i] = fmaf(p, zg_to_float(vr[d]), acc[i] * corr);
            }
            mx = m2;
        }
        T* orow = o + ((z * S + qi) * H + h) * D;
        for (int i = 0; i < 8; ++i) {
            const int d = lane + 32 * i;
            if (d < D) orow[d] = zg_from_float<T>(acc[i] / den);
        }
    }
}

int sm_count_attn() {
    static int n = 0;
    if (n == 0) {
        int dev = 0;
        cudaGetDevice(&dev);
        if (cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess || n < 1) n = 148;
    }
    return n;
}

}  // namespace

namespace zg {

// Timed-out waits of the tensor-core kernel (codes 81-83), 0 = none.
int attn_error_word(int clear) { return ptx_error_word(clear); }

}  // namespace zg

extern "C" int zg_attention(const void* q, const void* k, const void* v, int Z, int S, int H, int D, int causal,
                            int dtype, void* o, void* stream) {
    return zg_attention_ex(q, k, v, (int64_t)H * D, Z, S, H, D, causal, dtype, o, stream);
}

extern "C" int zg_attention_ex(const void* q, const void* k, const void* v, int64_t ld, int Z, int S, int H, int D,
                               int causal, int dtype, void* o, void* stream) {
    if (Z < 0 || S < 0 || H < 1 || D < 1) return zg::fail(ZG_ERR_INVALID, "zg_attention: bad sizes");
    if (ld < (int64_t)H * D) return zg::fail(ZG_ERR_INVALID, "zg_attention: row pitch below H*D");
    if (D > 256) return zg::fail(ZG_ERR_UNSUPPORTED, "zg_attention: head dim above 256");
    if (!zg::dtype_ok(dtype)) return zg::fail(ZG_ERR_INVALID, "zg_attention: bad dtype");
    if (Z == 0 || S == 0) return ZG_OK;
    if (!q || !k || !v || !o) return zg::fail(ZG_ERR_INVALID, "zg_attention: null pointer");
    if ((int64_t)Z * H > 65535LL * 65535LL) return zg::fail(ZG_ERR_INVALID, "zg_attention: too many rows");
    cudaStream_t st = zg::as_stream(stream);
    auto al = [](const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15) == 0; };
    const bool tc = dtype == ZG_BF16 && D == 64 && S <= 256 && Z <= 65535 && H <= 65535 && zg::tc_available() &&
                    al(q) && al(k) && al(v) && al(o) && (ld * 2) % 16 == 0;
    if (tc) {
        static bool attr = false;
        const size_t smem = AT_SMEM + 1024;
        if (!attr) {
            if (cudaFuncSetAttribute(attn_tc_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem) !=
                cudaSuccess)
                return zg::fail(ZG_ERR_CUDA, "zg_attention: shared memory attribute");
            attr = true;
        }
        CUtensorMap tq, tk, tv, to;
        const uint64_t dims[4] = {64, (uint64_t)H, (uint64_t)S, (uint64_t)Z};
        const uint64_t strides[3] = {64 * 2, (uint64_t)ld * 2, (uint64_t)S * ld * 2};
        const uint64_t ostrides[3] = {64 * 2, (uint64_t)H * 64 * 2, (uint64_t)S * H * 64 * 2};
        const uint32_t box[4] = {64, 1, 128, 1};
        if (!zg::tensor_map_bf16(&tq, q, 4, dims, strides, box, true) ||
            !zg::tensor_map_bf16(&tk, k, 4, dims, strides, box, true) ||
            !zg::tensor_map_bf16(&tv, v, 4, dims, strides, box, true) ||
            !zg::tensor_map_bf16(&to, o, 4, dims, ostrides, box, true))
            return zg::fail(ZG_ERR_CUDA, "zg_attention: tensor maps");
        AttnArgs a{static_cast<__nv_bfloat16*>(o), Z, S, H, S <= 128 ? 128 : 256, causal != 0,
                   (float)(1.4426950408889634 / sqrt(64.0))};
        dim3 grid((unsigned)((S + 127) / 128), (unsigned)H, (unsigned)Z);
        zg::LaunchTimer zg_lt_("attention", st);
        attn_tc_kernel<<<grid, AT_THREADS, smem, st>>>(tq, tk, tv, to, a);
        return zg::check_launch("zg_attention");
    }
    const int64_t rows = (int64_t)Z * S * H;
    int64_t blocks = (rows + 7) / 8;
    if (blocks > (int64_t)sm_count_attn() * 16) blocks = (int64_t)sm_count_attn() * 16;
    const float scale = (float)(1.0 / sqrt((double)D));
    zg::LaunchTimer zg_lt_("attention_simt", st);
    if (dtype == ZG_BF16)
        attn_simt_kernel<__nv_bfloat16><<<(unsigned)blocks, 256, 0, st>>>(
            static_cast<const __nv_bfloat16*>(q), static_cast<const __nv_bfloat16*>(k),
            static_cast<const __nv_bfloat16*>(v), static_cast<__nv_bfloat16*>(o), Z, S, H, D, causal != 0, scale, ld);
    else
        attn_simt_kernel<float><<<(unsigned)blocks, 256, 0, st>>>(
            static_cast<const float*>(q), static_cast<const float*>(k), static_cast<const float*>(v),
            static_cast<float*>(o), Z, S, H, D, causal != 0, scale, ld);
    return zg::check_launch("zg_attention");
}
