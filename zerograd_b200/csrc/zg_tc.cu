// zg_tc.cu -- tensor-core GEMM for sm_100a: tcgen05.mma (kind::f16, bf16 in,
// float32 accumulate in TMEM), operands staged by TMA (no multicast) into a
// 4- to 8-stage shared-memory ring (by tile width), persistent CTAs with two
// TMEM accumulators so the epilogue of one tile overlaps the main loop of
// the next.
//
//   D[M,N] = alpha * A[M,K] . B^T           (A K-major, row-major [M, K])
//   B is K-major ([N, K] row-major) or MN-major ([K, N] row-major).
//   D row-major float32 or bf16.
//
// Warp roles (192 threads): warp 0 = TMA producer, warp 1 = TMEM allocator +
// MMA issuer, warps 2..5 = epilogue (TMEM -> registers -> global).  Every
// mbarrier wait is bounded: on expiry the kernel records an error code in
// g_zg_tc_error, drains its own TMA copies, frees its TMEM and returns.
#include <cuda.h>
#include <cudaTypedefs.h>

#include <mutex>

#include "zg_ptx.cuh"
#include "zg_tc.cuh"
#include "zg_update.cuh"

namespace zg {
int launch_population_factors(const uint32_t* keys, int group, int P, int layout, int64_t rows,
                              int64_t cols, int rank, int dtype, void* A, void* B,
                              cudaStream_t st);
}

namespace {

constexpr int BM = 128, BK = 64, THREADS = 192;

// Operand-ring depth for a tile width: as many 64-deep K stages as fit in
// 192 KiB (4 at BN=256, 6 at BN=128, 8 at BN=64), so narrower tiles keep
// more bytes in flight per MMA.
__host__ __device__ constexpr int gemm_stages(int bn) { return (192 * 1024) / (BM * BK * 2 + bn * BK * 2); }


struct TcArgs {
    void* D;
    int64_t ldd;
    int M, N, K;
    float alpha;
    int out_bf16;
    int tiles_m, tiles_n;
    zg::FusedStep step;  // optimizer step on the float32 result (kind 0: none)
    // Split contraction: K is `splits` equal ranges of kb_split 64-deep
    // blocks, each accumulated on its own into the partial output D +
    // z * d_split (z = the range).  splits == 1: one range over all of K.
    int splits, kb_split;
    int64_t d_split;
};

// The optimizer step on d = alpha * v[0..n) of row `row`, columns col0..:
// parameters (and AdamW moments) read and written at the same positions, in
// groups of 8 elements (16-byte bf16 / 2 x 16-byte float32 accesses) when the
// row segment is aligned, element by element at a ragged edge.
__device__ __forceinline__ void tc_step8(const zg::FusedStep& st, int64_t e0, const float* d, int n, bool vec) {
    float p[8], mu[8], nu[8];
    if (vec) {
        if (st.param_bf16) {
            const uint4 raw = *reinterpret_cast<const uint4*>(static_cast<const __nv_bfloat16*>(st.param) + e0);
            const uint32_t w[4] = {raw.x, raw.y, raw.z, raw.w};
#pragma unroll
            for (int i = 0; i < 4; ++i) {
                p[2 * i] = __uint_as_float(w[i] << 16);
                p[2 * i + 1] = __uint_as_float(w[i] & 0xFFFF0000u);
            }
        } else {
            const float4 a = *reinterpret_cast<const float4*>(static_cast<const float*>(st.param) + e0);
            const float4 b = *reinterpret_cast<const float4*>(static_cast<const float*>(st.param) + e0 + 4);
            p[0] = a.x; p[1] = a.y; p[2] = a.z; p[3] = a.w; p[4] = b.x; p[5] = b.y; p[6] = b.z; p[7] = b.w;
        }
        if (st.kind == zg::ZG_STEP_ADAMW) {
            const float4 m0 = *reinterpret_cast<const float4*>(st.mu + e0), m1 = *reinterpret_cast<const float4*>(st.mu + e0 + 4);
            const float4 v0 = *reinterpret_cast<const float4*>(st.nu + e0), v1 = *reinterpret_cast<const float4*>(st.nu + e0 + 4);
            mu[0] = m0.x; mu[1] = m0.y; mu[2] = m0.z; mu[3] = m0.w; mu[4] = m1.x; mu[5] = m1.y; mu[6] = m1.z; mu[7] = m1.w;
            nu[0] = v0.x; nu[1] = v0.y; nu[2] = v0.z; nu[3] = v0.w; nu[4] = v1.x; nu[5] = v1.y; nu[6] = v1.z; nu[7] = v1.w;
        }
    } else {
#pragma unroll
        for (int i = 0; i < 8; ++i) {
            p[i] = 0.f;
            mu[i] = nu[i] = 0.f;
            if (i < n) {
                p[i] = st.param_bf16 ? __bfloat162float(static_cast<const __nv_bfloat16*>(st.param)[e0 + i])
                                     : static_cast<const float*>(st.param)[e0 + i];
                if (st.kind == zg::ZG_STEP_ADAMW) {
                    mu[i] = st.mu[e0 + i];
                    nu[i] = st.nu[e0 + i];
                }
            }
        }
    }
    float pn[8], m[8], vv[8];
    const zg::AdamConsts ac = st.kind == zg::ZG_STEP_ADAMW ? zg::adam_consts_dev(st.c, st.bc) : st.c;
#pragma unroll
    for (int i = 0; i < 8; ++i) {
        const float g = -d[i];  // pseudo-gradient
        if (st.kind == zg::ZG_STEP_SGD) {
            pn[i] = zg::sgd_step(p[i], g, st.c.neg_lr);
        } else {
            pn[i] = zg::adamw_step(p[i], g, mu[i], nu[i], ac, m[i], vv[i]);
        }
    }
    if (vec) {
        if (st.param_bf16) {
            uint4 o;
            __nv_bfloat162* h = reinterpret_cast<__nv_bfloat162*>(&o);
#pragma unroll
            for (int i = 0; i < 4; ++i) h[i] = __floats2bfloat162_rn(pn[2 * i], pn[2 * i + 1]);
            *reinterpret_cast<uint4*>(static_cast<__nv_bfloat16*>(st.param_out) + e0) = o;
        } else {
            float* q = static_cast<float*>(st.param_out) + e0;
            *reinterpret_cast<float4*>(q) = make_float4(pn[0], pn[1], pn[2], pn[3]);
            *reinterpret_cast<float4*>(q + 4) = make_float4(pn[4], pn[5], pn[6], pn[7]);
        }
        if (st.kind == zg::ZG_STEP_ADAMW) {
            *reinterpret_cast<float4*>(st.mu_out + e0) = make_float4(m[0], m[1], m[2], m[3]);
            *reinterpret_cast<float4*>(st.mu_out + e0 + 4) = make_float4(m[4], m[5], m[6], m[7]);
            *reinterpret_cast<float4*>(st.nu_out + e0) = make_float4(vv[0], vv[1], vv[2], vv[3]);
            *reinterpret_cast<float4*>(st.nu_out + e0 + 4) = make_float4(vv[4], vv[5], vv[6], vv[7]);
        }
    } else {
#pragma unroll
        for (int i = 0; i < 8; ++i) {
            if (i < n) {
                if (st.param_bf16)
                    static_cast<__nv_bfloat16*>(st.param_out)[e0 + i] = __float2bfloat16_rn(pn[i]);
                else
                    static_cast<float*>(st.param_out)[e0 + i] = pn[i];
                if (st.kind == zg::ZG_STEP_ADAMW) {
                    st.mu_out[e0 + i] = m[i];
                    st.nu_out[e0 + i] = vv[i];
                }
            }
        }
    }
}

__device__ __forceinline__ void tc_step32(const TcArgs& args, int row, int col0, const float (&v)[32]) {
    const zg::FusedStep& st = args.step;
    const int n = min(32, args.N - col0);
    const int64_t base = (int64_t)row * st.ldp + col0;
    const int esz = st.param_bf16 ? 2 : 4;
    // 16-byte aligned groups of 8 in every array touched
    const bool al = ((reinterpret_cast<uintptr_t>(st.param) + base * esz) & 15) == 0 &&
                    ((reinterpret_cast<uintptr_t>(st.param_out) + base * esz) & 15) == 0 &&
                    (st.kind != zg::ZG_STEP_ADAMW ||
                     (((reinterpret_cast<uintptr_t>(st.mu) | reinterpret_cast<uintptr_t>(st.nu) |
                        reinterpret_cast<uintptr_t>(st.mu_out) | reinterpret_cast<uintptr_t>(st.nu_out)) +
                       base * 4) & 15) == 0);
#pragma unroll
    for (int g = 0; g < 4; ++g) {
        float d[8];
#pragma unroll
        for (int i = 0; i < 8; ++i) d[i] = args.alpha * v[8 * g + i];
        const int ng = n - 8 * g;
        if (ng <= 0) break;
        tc_step8(st, base + 8 * g, d, ng, al && ng >= 8);
    }
}

// alpha * v[0..32) -> D[row, col0 .. col0+32), bounds-checked against M and N.
__device__ __forceinline__ void tc_store32_d(const TcArgs& args, int row, int col0, const float (&v)[32],
                                             int64_t zoff) {
    if (row >= args.M || col0 >= args.N) return;
    if (args.out_bf16) {
        __nv_bfloat16* d = static_cast<__nv_bfloat16*>(args.D) + zoff + (int64_t)row * args.ldd + col0;
        if (col0 + 32 <= args.N && ((reinterpret_cast<uintptr_t>(d) & 15) == 0)) {
#pragma unroll
            for (int i = 0; i < 32; i += 8) {
                __nv_bfloat162 h[4];
#pragma unroll
                for (int j = 0; j < 4; ++j)
                    h[j] = __floats2bfloat162_rn(args.alpha * v[i + 2 * j], args.alpha * v[i + 2 * j + 1]);
                *reinterpret_cast<uint4*>(d + i) = *reinterpret_cast<uint4*>(h);
            }
        } else {
            for (int i = 0; i < 32; ++i)
                if (col0 + i < args.N) d[i] = __float2bfloat16_rn(args.alpha * v[i]);
        }
    } else {
        float* d = static_cast<float*>(args.D) + zoff + (int64_t)row * args.ldd + col0;
        if (col0 + 32 <= args.N && ((reinterpret_cast<uintptr_t>(d) & 15) == 0)) {
#pragma unroll
            for (int i = 0; i < 32; i += 4)
                *reinterpret_cast<float4*>(d + i) = make_float4(args.alpha * v[i], args.alpha * v[i + 1],
                                                                args.alpha * v[i + 2], args.alpha * v[i + 3]);
        } else {
            for (int i = 0; i < 32; ++i)
                if (col0 + i < args.N) d[i] = args.alpha * v[i];
        }
    }
}

// The epilogue's store of 32 columns: the fused optimizer step (if any) and
// D (which may be null when the step consumes the result).
__device__ __forceinline__ void tc_store32(const TcArgs& args, int row, int col0, const float (&v)[32],
                                           int64_t zoff) {
    if (row >= args.M || col0 >= args.N) return;
    if (args.step.kind != zg::ZG_STEP_NONE) tc_step32(args, row, col0, v);
    if (args.D) tc_store32_d(args, row, col0, v, zoff);
}

// One tile row of an epilogue: TMEM columns [0, W) of this thread's lane ->
// D and/or the fused optimizer step.  For an SGD step on an aligned bf16 row
// segment every parameter load of the row is issued before the first TMEM
// read, so their latency is paid once per tile, not once per 32 columns.
template <int W>
__device__ __forceinline__ void tc_epilogue_row(const TcArgs& args, int row, int col_base, uint32_t tacc,
                                                int64_t zoff) {
    const zg::FusedStep& st = args.step;
    // a guarded step writes nothing at all when its guard is set (the same
    // value in every lane, so the warp stays on one path)
    if (st.guard != nullptr && !(*st.guard == 0.f)) return;
    const int64_t base = (int64_t)row * st.ldp + col_base;
    const bool lane_fast = st.kind == zg::ZG_STEP_SGD && st.param_bf16 && row < args.M && col_base + W <= args.N &&
                           ((reinterpret_cast<uintptr_t>(st.param) + base * 2) & 15) == 0 &&
                           ((reinterpret_cast<uintptr_t>(st.param_out) + base * 2) & 15) == 0;
    // tcgen05.ld is warp-collective (.sync.aligned): the whole warp takes one
    // path, so a ragged tile (rows past M in some lanes) uses the general one
    if (__all_sync(0xffffffffu, lane_fast)) {
        uint4 pre[W / 8];
        const uint4* src = reinterpret_cast<const uint4*>(static_cast<const __nv_bfloat16*>(st.param) + base);
#pragma unroll
        for (int i = 0; i < W / 8; ++i) pre[i] = src[i];
        uint4* dst = reinterpret_cast<uint4*>(static_cast<__nv_bfloat16*>(st.param_out) + base);
#pragma unroll
        for (int c = 0; c < W / 32; ++c) {
            float v[32];
            tmem_ld32(tacc + c * 32, v);
            if (args.D) tc_store32_d(args, row, col_base + c * 32, v, zoff);
#pragma unroll
            for (int g = 0; g < 4; ++g) {
                const uint4 raw = pre[c * 4 + g];
                const uint32_t w[4] = {raw.x, raw.y, raw.z, raw.w};
                uint4 o;
                __nv_bfloat162* h = reinterpret_cast<__nv_bfloat162*>(&o);
#pragma unroll
                for (int i = 0; i < 4; ++i) {
                    const float d0 = args.alpha * v[8 * g + 2 * i], d1 = args.alpha * v[8 * g + 2 * i + 1];
                    h[i] = __floats2bfloat162_rn(zg::sgd_step(__uint_as_float(w[i] << 16), -d0, st.c.neg_lr),
                                                 zg::sgd_step(__uint_as_float(w[i] & 0xFFFF0000u), -d1, st.c.neg_lr));
                }
                dst[c * 4 + g] = o;
            }
        }
        return;
    }
#pragma unroll 1
    for (int c0 = 0; c0 < W; c0 += 32) {
        float v[32];
        tmem_ld32(tacc + c0, v);
        tc_store32(args, row, col_base + c0, v, zoff);
    }
}

// Fixed-order sum of split partials and the step on it (split_reduce): one
// thread per 8 consecutive elements, grid-stride; `out` (optional with a
// step) receives the scaled sum.
struct SplitParts {
    const float* p[zg::kMaxSplits];
    int S;
};

__global__ void __launch_bounds__(256)
split_reduce_kernel(const SplitParts parts, int64_t n, float alpha, const zg::FusedStep step, float* out) {
    if (step.guard != nullptr && !(*step.guard == 0.f)) return;
    bool al = true;  // every partial 16-byte aligned: vector loads
#pragma unroll
    for (int s = 0; s < zg::kMaxSplits; ++s)
        if (s < parts.S) al = al && ((reinterpret_cast<uintptr_t>(parts.p[s]) & 15) == 0);
    const bool step_al = step.kind == zg::ZG_STEP_NONE ||
                         ((((reinterpret_cast<uintptr_t>(step.param) | reinterpret_cast<uintptr_t>(step.param_out)) &
                            15) == 0) &&
                          (step.kind != zg::ZG_STEP_ADAMW ||
                           ((reinterpret_cast<uintptr_t>(step.mu) | reinterpret_cast<uintptr_t>(step.nu) |
                             reinterpret_cast<uintptr_t>(step.mu_out) | reinterpret_cast<uintptr_t>(step.nu_out)) &
                            15) == 0));
    const bool out_al = out == nullptr || (reinterpret_cast<uintptr_t>(out) & 15) == 0;
    const int64_t stride = (int64_t)gridDim.x * blockDim.x * 8;
    for (int64_t e0 = ((int64_t)blockIdx.x * blockDim.x + threadIdx.x) * 8; e0 < n; e0 += stride) {
        const int m = n - e0 < 8 ? (int)(n - e0) : 8;
        const bool vec = m == 8 && al;
        float acc[8];
        if (vec) {
            const float4 a = *reinterpret_cast<const float4*>(parts.p[0] + e0);
            const float4 b = *reinterpret_cast<const float4*>(parts.p[0] + e0 + 4);
            acc[0] = a.x; acc[1] = a.y; acc[2] = a.z; acc[3] = a.w; acc[4] = b.x; acc[5] = b.y; acc[6] = b.z;
            acc[7] = b.w;
#pragma unroll
            for (int s = 1; s < zg::kMaxSplits; ++s) {
                if (s >= parts.S) break;
                const float4 c = *reinterpret_cast<const float4*>(parts.p[s] + e0);
                const float4 d = *reinterpret_cast<const float4*>(parts.p[s] + e0 + 4);
                acc[0] = __fadd_rn(acc[0], c.x); acc[1] = __fadd_rn(acc[1], c.y);
                acc[2] = __fadd_rn(acc[2], c.z); acc[3] = __fadd_rn(acc[3], c.w);
                acc[4] = __fadd_rn(acc[4], d.x); acc[5] = __fadd_rn(acc[5], d.y);
                acc[6] = __fadd_rn(acc[6], d.z); acc[7] = __fadd_rn(acc[7], d.w);
            }
        } else {
#pragma unroll
            for (int i = 0; i < 8; ++i) acc[i] = i < m ? parts.p[0][e0 + i] : 0.f;
#pragma unroll
            for (int s = 1; s < zg::kMaxSplits; ++s) {
                if (s >= parts.S) break;
#pragma unroll
                for (int i = 0; i < 8; ++i)
                    if (i < m) acc[i] = __fadd_rn(acc[i], parts.p[s][e0 + i]);
            }
        }
        float d[8];
#pragma unroll
        for (int i = 0; i < 8; ++i) d[i] = __fmul_rn(alpha, acc[i]);
        if (step.kind != zg::ZG_STEP_NONE) tc_step8(step, e0, d, m, m == 8 && step_al);
        if (out == nullptr) continue;
        if (m == 8 && out_al) {
            *reinterpret_cast<float4*>(out + e0) = make_float4(d[0], d[1], d[2], d[3]);
            *reinterpret_cast<float4*>(out + e0 + 4) = make_float4(d[4], d[5], d[6], d[7]);
        } else {
#pragma unroll
            for (int i = 0; i < 8; ++i)
                if (i < m) out[e0 + i] = d[i];
        }
    }
}

template <int BN, bool B_MN>
__global__ void __launch_bounds__(THREADS, 1)
tc_gemm_kernel(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmB, const TcArgs args) {
    constexpr uint32_t A_BYTES = BM * BK * 2;
    constexpr uint32_t B_BYTES = BN * BK * 2;
    constexpr uint32_t STAGE_BYTES = A_BYTES + B_BYTES;
    constexpr uint32_t TMEM_COLS = 2 * BN < 32 ? 32 : 2 * BN;  // power of two for BN in {64,128,256}
    constexpr int STAGES = gemm_stages(BN);
    extern __shared__ uint8_t dyn_smem[];
    __shared__ __align__(8) uint64_t full_bar[STAGES], empty_bar[STAGES], tmem_full[2], tmem_empty[2], mma_done;
    __shared__ uint32_t tmem_base_sh;

    // 1024-byte alignment of the operand ring in the shared window (swizzle atoms)
    const uint32_t dyn_base = smem_u32(dyn_smem);
    uint8_t* smem = dyn_smem + (((dyn_base + 1023u) & ~1023u) - dyn_base);
    const int warp = threadIdx.x / 32, lane = threadIdx.x % 32;
    const int tiles_mn = args.tiles_m * args.tiles_n;
    const int num_tiles = tiles_mn * args.splits;
    const int k_blocks = args.kb_split;  // per tile: one split's K range

    if (threadIdx.x == 0) {
        for (int s = 0; s < STAGES; ++s) {
            mbar_init(&full_bar[s], 1);
            mbar_init(&empty_bar[s], 1);
        }
        for (int a = 0; a < 2; ++a) {
            mbar_init(&tmem_full[a], 1);
            mbar_init(&tmem_empty[a], 4);  // one arrive per epilogue warp
        }
        mbar_init(&mma_done, 1);
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    }
    if (warp == 1) tmem_alloc(&tmem_base_sh, TMEM_COLS);
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem_base = tmem_base_sh;

    if (warp == 0 && lane == 0) {
        // ---------------- TMA producer ----------------
        int stage = 0;
        uint32_t phase = 0;
        uint32_t issued = 0;  // bit s: stage s has an issued load
        uint32_t issue_parity = 0;
        bool ok = true;
        for (int t = blockIdx.x; ok && t < num_tiles; t += gridDim.x) {
            const int z = t / tiles_mn, tt = t % tiles_mn;
            const int tm = tt / args.tiles_n, tn = tt % args.tiles_n;
            // Tiles start their K sweep at different blocks, so CTAs that share
            // an operand tile do not all request the same L2 lines at once.
            // The start depends on the tile's place in its output only, so a
            // split's partial is the same whichever launch computes it.
            const int k_start = tt % k_blocks;
            for (int kb = 0; kb < k_blocks; ++kb) {
                if (!mbar_wait(&empty_bar[stage], phase ^ 1, 1)) { ok = false; break; }
                const int kk = z * k_blocks + (kb + k_start < k_blocks ? kb + k_start : kb + k_start - k_blocks);
                uint8_t* sa = smem + stage * STAGE_BYTES;
                uint8_t* sb = sa + A_BYTES;
                mbar_expect_tx(&full_bar[stage], STAGE_BYTES);
                tma_load_2d(sa, &tmA, &full_bar[stage], kk * BK, tm * BM);
                if constexpr (B_MN) {
#pragma unroll
                    for (int c = 0; c < BN / 64; ++c)
                        tma_load_2d(sb + c * (64 * BK * 2), &tmB, &full_bar[stage], tn * BN + c * 64, kk * BK);
                } else {
                    tma_load_2d(sb, &tmB, &full_bar[stage], kk * BK, tn * BN);
                }
                issued |= 1u << stage;
                issue_parity = (issue_parity & ~(1u << stage)) | (phase << stage);
                if (++stage == STAGES) { stage = 0; phase ^= 1; }
            }
        }
        // Drain: every issued copy has landed before the CTA may exit.
        for (int s = 0; s < STAGES; ++s)
            if (issued & (1u << s)) {
                for (uint32_t i = 0; i < kSpinLimit; ++i)
                    if (mbar_try_wait(&full_bar[s], (issue_parity >> s) & 1)) break;
            }
    } else if (warp == 1 && lane == 0) {
        // ---------------- MMA issuer ----------------
        constexpr uint32_t IDESC = idesc_bf16(BM, BN, B_MN ? 1 : 0);
        int stage = 0;
        uint32_t phase = 0;
        int acc = 0;
        uint32_t acc_phase = 0;
        bool ok = true;
        for (int t = blockIdx.x; ok && t < num_tiles; t += gridDim.x) {
            if (!mbar_wait(&tmem_empty[acc], acc_phase ^ 1, 2)) break;
            tc_fence_after();
            const uint32_t d_tmem = tmem_base + acc * BN;
            for (int kb = 0; kb < k_blocks; ++kb) {
                if (!mbar_wait(&full_bar[stage], phase, 3)) { ok = false; break; }
                tc_fence_after();
                const uint32_t a_addr = smem_u32(smem + stage * STAGE_BYTES);
                const uint32_t b_addr = a_addr + A_BYTES;
#pragma unroll
                for (int k = 0; k < BK / 16; ++k) {
                    // K-major SW128: 16 bf16 of K = 32 bytes along the swizzled row.
                    const uint64_t ad = smem_desc(a_addr + k * 32, 16, 1024);
                    uint64_t bd;
                    if constexpr (B_MN) {
                        // MN-major SW128: 64-wide N blocks 8 KiB apart (LBO), 8-row K groups 1 KiB apart
                        // (SBO); 16 K rows = 2 KiB per step.
                        bd = smem_desc(b_addr + k * 2048, 64 * BK * 2, 1024);
                    } else {
                        bd = smem_desc(b_addr + k * 32, 16, 1024);
                    }
                    umma_bf16(d_tmem, ad, bd, IDESC, (kb > 0 || k > 0) ? 1u : 0u);
                }
                umma_commit(&empty_bar[stage]);  // frees the smem stage once these MMAs complete
                if (++stage == STAGES) { stage = 0; phase ^= 1; }
            }
            if (!ok) break;
            umma_commit(&tmem_full[acc]);
            if (++acc == 2) { acc = 0; acc_phase ^= 1; }
        }
        // No MMA may still be writing TMEM when it is freed.
        umma_commit(&mma_done);
        for (uint32_t i = 0; i < kSpinLimit; ++i)
            if (mbar_try_wait(&mma_done, 0)) break;
    } else if (warp >= 2) {
        // ---------------- epilogue ----------------
        const int quad = warp % 4;  // TMEM lanes 32*quad .. 32*quad+31
        int acc = 0;
        uint32_t acc_phase = 0;
        for (int t = blockIdx.x; t < num_tiles; t += gridDim.x) {
            if (!mbar_wait(&tmem_full[acc], acc_phase, 4)) break;
            tc_fence_after();
            const int z = t / tiles_mn, tt = t % tiles_mn;
            const int tm = tt / args.tiles_n, tn = tt % args.tiles_n;
            const int row = tm * BM + quad * 32 + lane;
            tc_epilogue_row<BN>(args, row, tn * BN, tmem_base + ((uint32_t)(quad * 32) << 16) + acc * BN,
                                z * args.d_split);
            tc_fence_before();
            __syncwarp();
            if (lane == 0) mbar_arrive(&tmem_empty[acc]);
            if (++acc == 2) { acc = 0; acc_phase ^= 1; }
        }
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    if (warp == 1) tmem_dealloc(tmem_base, TMEM_COLS);
}

// ---------------------------------------------------------------------------
// CTA-pair GEMM: 256 x 256 tiles on a cluster of two CTAs (two SMs).  CTA r
// of the pair stages rows [128 r, 128 r + 128) of the A tile and columns
// [128 r, 128 r + 128) of the B tile in its own shared memory; the leader
// (r = 0) issues M=256 N=256 MMAs that read both CTAs' halves, and CTA r's
// TMEM accumulates tile rows [128 r, 128 r + 128).  Per 64-deep K block each
// SM stages 32 KiB instead of the 48 KiB of a one-SM 128 x 256 tile, so the
// L2 -> SM traffic per FLOP drops by a third.
// Barriers: full[s] (leader's; counts both CTAs' bytes), empty[s] (each CTA;
// one commit from the leader), tmem_full[a] (each CTA; one commit),
// tmem_empty[a] (leader's; one arrival per epilogue warp of either CTA).
// ---------------------------------------------------------------------------
constexpr int P2_STAGES = 6;
constexpr uint32_t P2_A = BM * BK * 2;           // this CTA's 128 rows of the A tile
constexpr uint32_t P2_B = 128 * BK * 2;          // this CTA's 128 columns of the B tile
constexpr uint32_t P2_STAGE = P2_A + P2_B;       // 32 KiB
constexpr uint32_t P2_SMEM = P2_STAGES * P2_STAGE;

template <bool B_MN>
__global__ void __cluster_dims__(2, 1, 1) __launch_bounds__(THREADS, 1)
tc_gemm_pair_kernel(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmB,
                    const TcArgs args) {
    extern __shared__ uint8_t dyn_smem[];
    __shared__ __align__(8) uint64_t full_bar[P2_STAGES], empty_bar[P2_STAGES], tmem_full[2], tmem_empty[2],
        mma_done;
    __shared__ uint32_t tmem_base_sh;
    const uint32_t dyn_base = smem_u32(dyn_smem);
    uint8_t* smem = dyn_smem + (((dyn_base + 1023u) & ~1023u) - dyn_base);
    const int warp = threadIdx.x / 32, lane = threadIdx.x % 32;
    const uint32_t rank = cluster_rank();
    const int pair = blockIdx.x / 2, pairs = gridDim.x / 2;
    const int tiles_mn = args.tiles_m * args.tiles_n;
    const int num_tiles = tiles_mn * args.splits;
    const int k_blocks = args.kb_split;  // per tile: one split's K range

    if (threadIdx.x == 0) {
        for (int s = 0; s < P2_STAGES; ++s) {
            mbar_init(&full_bar[s], 1);
            mbar_init(&empty_bar[s], 1);
        }
        for (int a = 0; a < 2; ++a) {
            mbar_init(&tmem_full[a], 1);
            mbar_init(&tmem_empty[a], 8);  // 4 epilogue warps in each CTA
        }
        mbar_init(&mma_done, 1);
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    }
    if (warp == 1) tmem_alloc_pair(&tmem_base_sh, 512);
    tc_fence_before();
    cluster_sync();  // barriers initialised and TMEM allocated in both CTAs
    tc_fence_after();
    const uint32_t tmem_base = tmem_base_sh;

    if (warp == 0 && lane == 0) {
        // ---------------- TMA producer (both CTAs) ----------------
        int stage = 0;
        uint32_t phase = 0, issued = 0, issue_parity = 0;
        bool ok = true;
        for (int t = pair; ok && t < num_tiles; t += pairs) {
            const int z = t / tiles_mn, tt = t % tiles_mn;
            const int tm = tt / args.tiles_n, tn = tt % args.tiles_n;
            const int k_start = tt % k_blocks;
            for (int kb = 0; kb < k_blocks; ++kb) {
                if (!mbar_wait(&empty_bar[stage], phase ^ 1, 21)) { ok = false; break; }
                const int kk = z * k_blocks + (kb + k_start < k_blocks ? kb + k_start : kb + k_start - k_blocks);
                uint8_t* sa = smem + stage * P2_STAGE;
                uint8_t* sb = sa + P2_A;
                if (rank == 0) mbar_expect_tx(&full_bar[stage], 2 * P2_STAGE);
                const uint32_t fb = cluster_addr(&full_bar[stage], 0);
                tma_load_2d_pair(sa, &tmA, fb, kk * BK, tm * 256 + (int)rank * 128);
                if constexpr (B_MN) {
#pragma unroll
                    for (int c = 0; c < 2; ++c)
                        tma_load_2d_pair(sb + c * (64 * BK * 2), &tmB, fb, tn * 256 + (int)rank * 128 + c * 64,
                                         kk * BK);
                } else {
                    tma_load_2d_pair(sb, &tmB, fb, kk * BK, tn * 256 + (int)rank * 128);
                }
                issued |= 1u << stage;
                issue_parity = (issue_parity & ~(1u << stage)) | (phase << stage);
                if (++stage == P2_STAGES) { stage = 0; phase ^= 1; }
            }
        }
        // Drain: the leader sees its stages' bytes land on its full barriers;
        // the peer sees each stage released by the MMAs that consumed it.
        for (int s = 0; s < P2_STAGES; ++s)
            if (issued & (1u << s)) {
                uint64_t* bar = rank == 0 ? &full_bar[s] : &empty_bar[s];
                for (uint32_t i = 0; i < kSpinLimit; ++i)
                    if (mbar_try_wait(bar, (issue_parity >> s) & 1)) break;
            }
    } else if (warp == 1 && lane == 0 && rank == 0) {
        // ---------------- MMA issuer (leader only) ----------------
        constexpr uint32_t IDESC = idesc_bf16(256, 256, B_MN ? 1 : 0);
        int stage = 0, acc = 0;
        uint32_t phase = 0, acc_phase = 0;
        bool ok = true;
        for (int t = pair; ok && t < num_tiles; t += pairs) {
            if (!mbar_wait(&tmem_empty[acc], acc_phase ^ 1, 22)) break;
            tc_fence_after();
            const uint32_t d_tmem = tmem_base + acc * 256;
            for (int kb = 0; kb < k_blocks; ++kb) {
                if (!mbar_wait(&full_bar[stage], phase, 23)) { ok = false; break; }
                tc_fence_after();
                const uint32_t a_addr = smem_u32(smem + stage * P2_STAGE);
                const uint32_t b_addr = a_addr + P2_A;
#pragma unroll
                for (int k = 0; k < BK / 16; ++k) {
                    const uint64_t ad = smem_desc(a_addr + k * 32, 16, 1024);
                    const uint64_t bd = B_MN ? smem_desc(b_addr + k * 2048, 64 * BK * 2, 1024)
                                             : smem_desc(b_addr + k * 32, 16, 1024);
                    umma_bf16_pair(d_tmem, ad, bd, IDESC, (kb > 0 || k > 0) ? 1u : 0u);
                }
                // the stage is free in both CTAs once these MMAs complete
                umma_commit_pair(smem_u32(&empty_bar[stage]));
                umma_commit_pair(cluster_addr(&empty_bar[stage], 1));
                if (++stage == P2_STAGES) { stage = 0; phase ^= 1; }
            }
            if (!ok) break;
            umma_commit_pair(smem_u32(&tmem_full[acc]));
            umma_commit_pair(cluster_addr(&tmem_full[acc], 1));
            if (++acc == 2) { acc = 0; acc_phase ^= 1; }
        }
        umma_commit_pair(smem_u32(&mma_done));
        for (uint32_t i = 0; i < kSpinLimit; ++i)
            if (mbar_try_wait(&mma_done, 0)) break;
    } else if (warp >= 2) {
        // ---------------- epilogue (both CTAs, own TMEM rows) ----------------
        const int quad = warp % 4;
        const uint32_t empty_leader = cluster_addr(&tmem_empty[0], 0);
        int acc = 0;
        uint32_t acc_phase = 0;
        for (int t = pair; t < num_tiles; t += pairs) {
            if (!mbar_wait(&tmem_full[acc], acc_phase, 24)) break;
            tc_fence_after();
            const int z = t / tiles_mn, tt = t % tiles_mn;
            const int tm = tt / args.tiles_n, tn = tt % args.tiles_n;
            const int row = tm * 256 + (int)rank * 128 + quad * 32 + lane;
            tc_epilogue_row<256>(args, row, tn * 256, tmem_base + ((uint32_t)(quad * 32) << 16) + acc * 256,
                                 z * args.d_split);
            tc_fence_before();
            __syncwarp();
            if (lane == 0) mbar_arrive_remote(empty_leader + acc * (uint32_t)sizeof(uint64_t));
            if (++acc == 2) { acc = 0; acc_phase ^= 1; }
        }
    }
    // All pair MMAs have completed (the leader waited on mma_done) and both
    // CTAs' epilogues are done with TMEM before either frees it.
    tc_fence_before();
    cluster_sync();
    tc_fence_after();
    if (warp == 1) tmem_dealloc_pair(tmem_base, 512);
}

// ---------------------------------------------------------------------------
// Low-rank expansion on the tensor cores, rank 8:
//   y[p, m, n] = bf16(XW[m, n] + s * (U_p . B_p^T)[m, n])
// U [M, P*8] bf16 (x @ A_all), B [N, P*8] bf16 (B_nq), XW [M, N] float32.
// One M=128 N=128 K=16 MMA per candidate (the upper 8 K of each operand
// read a zero region through the descriptor's leading byte offset) into one
// of four TMEM accumulators; each epilogue thread keeps its 64-column slice
// of the XW row in registers for the whole tile, adds it with packed FMAs and
// writes bf16 into a 128B-swizzled shared tile that a TMA bulk store copies
// out, so the global writes are full lines and the kernel is bound by HBM
// write bandwidth.  Work item = (m tile, n tile, candidate chunk); each
// persistent CTA takes a contiguous run of items.
// ---------------------------------------------------------------------------
constexpr int EX_STAGES = 4;
constexpr uint32_t EX_OP = 128 * 16;                       // one operand tile: 128 rows x 8 bf16
constexpr uint32_t EX_A = 0, EX_AZ = EX_STAGES * EX_OP;    // A data, A zero half
constexpr uint32_t EX_B = 2 * EX_STAGES * EX_OP, EX_BZ = 3 * EX_STAGES * EX_OP;
constexpr uint32_t EX_LBO = EX_STAGES * EX_OP;             // data -> zero half, same for every stage
constexpr uint32_t EX_STG = 4 * EX_STAGES * EX_OP;        // staging buffers, each 2 x 16 KiB sub-tiles
constexpr uint32_t EX_STG_BYTES = 128 * 128 * 2;
constexpr int EX_NSTG = 4;                                 // staging buffers in flight
constexpr int EX_NACC = 4;                                 // TMEM accumulators of 128 columns (all 512)
constexpr uint32_t EX_SMEM = EX_STG + EX_NSTG * EX_STG_BYTES;  // 160 KiB (+ alignment)

struct ExpandArgs {
    const float* XW;
    int M, N, P;
    float s;
    int tiles_m, tiles_n, chunk, chunks;
};

constexpr int EX_THREADS = 352;  // warp 0 TMA, warp 1 MMA, warps 2..9 epilogue (2 per TMEM lane quadrant),
                                 // warp 10 TMA stores
__device__ __forceinline__ void ex_item_range(int items, int& t0, int& t1) {
    const int per = items / (int)gridDim.x, rem = items % (int)gridDim.x, b = blockIdx.x;
    t0 = b * per + min(b, rem);
    t1 = t0 + per + (b < rem ? 1 : 0);
}

// R = 8: the upper 8 K of each operand read a zero region; R = 16: they
// read the second 8 factor columns, loaded beside the first.
template <int R>
__global__ void __launch_bounds__(EX_THREADS, 1)
expand_tc_kernel(const __grid_constant__ CUtensorMap tmU, const __grid_constant__ CUtensorMap tmB,
                 const __grid_constant__ CUtensorMap tmY, const ExpandArgs a) {
    extern __shared__ uint8_t dyn_smem[];
    __shared__ __align__(8) uint64_t full_bar[EX_STAGES], empty_bar[EX_STAGES], tmem_full[EX_NACC],
        tmem_empty[EX_NACC], stg_full[EX_NSTG], stg_free[EX_NSTG], mma_done;
    __shared__ uint32_t tmem_base_sh;
    const uint32_t dyn_base = smem_u32(dyn_smem);
    uint8_t* smem = dyn_smem + (((dyn_base + 1023u) & ~1023u) - dyn_base);
    const int warp = threadIdx.x / 32, lane = threadIdx.x % 32;
    int t_begin, t_end;
    ex_item_range(a.tiles_m * a.tiles_n * a.chunks, t_begin, t_end);

    if constexpr (R == 8) {
        // zero halves of the K=16 operands (read through the descriptors' LBO)
        for (uint32_t i = threadIdx.x; i < EX_LBO / 16; i += EX_THREADS) {
            reinterpret_cast<uint4*>(smem + EX_AZ)[i] = make_uint4(0, 0, 0, 0);
            reinterpret_cast<uint4*>(smem + EX_BZ)[i] = make_uint4(0, 0, 0, 0);
        }
        asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
    }
    if (threadIdx.x == 0) {
        for (int s = 0; s < EX_STAGES; ++s) {
            mbar_init(&full_bar[s], 1);
            mbar_init(&empty_bar[s], 1);
        }
        for (int b = 0; b < EX_NACC; ++b) {
            mbar_init(&tmem_full[b], 1);
            mbar_init(&tmem_empty[b], 8);   // one arrive per epilogue warp
        }
        for (int b = 0; b < EX_NSTG; ++b) {
            mbar_init(&stg_full[b], 256);   // every epilogue thread
            mbar_init(&stg_free[b], 1);
        }
        mbar_init(&mma_done, 1);
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    }
    if (warp == 1) tmem_alloc(&tmem_base_sh, 512);
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem_base = tmem_base_sh;

    if (warp == 0 && lane == 0) {
        // ---------------- TMA producer: U_p and B_p tiles ----------------
        int stage = 0;
        uint32_t phase = 0, issued = 0, issue_parity = 0;
        bool ok = true;
        for (int t = t_begin; ok && t < t_end; ++t) {
            const int chunk = t % a.chunks, tile = t / a.chunks;
            const int m0 = (tile / a.tiles_n) * 128, n0 = (tile % a.tiles_n) * 128;
            const int p1 = min(a.P, (chunk + 1) * a.chunk);
            for (int p = chunk * a.chunk; p < p1; ++p) {
                if (!mbar_wait(&empty_bar[stage], phase ^ 1, 11)) { ok = false; break; }
                mbar_expect_tx(&full_bar[stage], (R / 8) * 2 * EX_OP);
                tma_load_2d(smem + EX_A + stage * EX_OP, &tmU, &full_bar[stage], p * R, m0);
                tma_load_2d(smem + EX_B + stage * EX_OP, &tmB, &full_bar[stage], p * R, n0);
                if constexpr (R == 16) {
                    tma_load_2d(smem + EX_AZ + stage * EX_OP, &tmU, &full_bar[stage], p * R + 8, m0);
                    tma_load_2d(smem + EX_BZ + stage * EX_OP, &tmB, &full_bar[stage], p * R + 8, n0);
                }
                issued |= 1u << stage;
                issue_parity = (issue_parity & ~(1u << stage)) | (phase << stage);
                if (++stage == EX_STAGES) { stage = 0; phase ^= 1; }
            }
        }
        for (int s = 0; s < EX_STAGES; ++s)
            if (issued & (1u << s))
                for (uint32_t i = 0; i < kSpinLimit; ++i)
                    if (mbar_try_wait(&full_bar[s], (issue_parity >> s) & 1)) break;
    } else if (warp == 1 && lane == 0) {
        // ---------------- MMA issuer: one K=16 MMA per candidate ----------------
        constexpr uint32_t IDESC = idesc_bf16(128, 128, 0);
        int stage = 0, acc = 0;
        uint32_t phase = 0, acc_phase = 0;
        bool ok = true;
        for (int t = t_begin; ok && t < t_end; ++t) {
            const int chunk = t % a.chunks;
            const int p1 = min(a.P, (chunk + 1) * a.chunk);
            for (int p = chunk * a.chunk; p < p1; ++p) {
                if (!mbar_wait(&tmem_empty[acc], acc_phase ^ 1, 12)) { ok = false; break; }
                tc_fence_after();
                if (!mbar_wait(&full_bar[stage], phase, 13)) { ok = false; break; }
                tc_fence_after();
                const uint64_t ad = smem_desc_noswizzle(smem_u32(smem + EX_A + stage * EX_OP), EX_LBO, 128);
                const uint64_t bd = smem_desc_noswizzle(smem_u32(smem + EX_B + stage * EX_OP), EX_LBO, 128);
                umma_bf16(tmem_base + acc * 128, ad, bd, IDESC, 0u);
                umma_commit(&empty_bar[stage]);
                umma_commit(&tmem_full[acc]);
                if (++stage == EX_STAGES) { stage = 0; phase ^= 1; }
                if (++acc == EX_NACC) { acc = 0; acc_phase ^= 1; }
            }
        }
        umma_commit(&mma_done);
        for (uint32_t i = 0; i < kSpinLimit; ++i)
            if (mbar_try_wait(&mma_done, 0)) break;
    } else if (warp == 10) {
        // ---------------- TMA stores: a full staging buffer -> y[p] tile ----------------
        if (lane == 0) {
            int c = 0;
            bool ok = true;
            for (int t = t_begin; ok && t < t_end; ++t) {
                const int chunk = t % a.chunks, tile = t / a.chunks;
                const int m0 = (tile / a.tiles_n) * 128, n0 = (tile % a.tiles_n) * 128;
                const int p1 = min(a.P, (chunk + 1) * a.chunk);
                for (int p = chunk * a.chunk; p < p1; ++p, ++c) {
                    const int sb = c % EX_NSTG;
                    if (!mbar_wait(&stg_full[sb], (uint32_t)(c / EX_NSTG) & 1, 16)) { ok = false; break; }
                    uint8_t* stg = smem + EX_STG + sb * EX_STG_BYTES;
                    tma_store_3d(&tmY, stg, n0, m0, p);
                    tma_store_3d(&tmY, stg + 128 * 128, n0 + 64, m0, p);
                    asm volatile("cp.async.bulk.commit_group;" ::: "memory");
                    // all but the two newest stores have finished reading their buffers
                    asm volatile("cp.async.bulk.wait_group.read 2;" ::: "memory");
                    if (c >= 2) mbar_arrive(&stg_free[(c - 2) % EX_NSTG]);
                }
            }
            asm volatile("cp.async.bulk.wait_group 0;" ::: "memory");
        }
    } else if (warp >= 2) {
        // ---------------- epilogue: TMEM -> bf16 -> swizzled smem (warp 10 stores it) ----------------
        const int quad = warp % 4;             // TMEM lanes 32*quad..32*quad+31
        const int half = (warp - 2) / 4;       // columns 64*half..64*half+63
        const int row = quad * 32 + lane;      // TMEM lane == tile row
        const uint32_t lane_addr = (uint32_t)(quad * 32) << 16;
        const float2 s2 = make_float2(a.s, a.s);
        float2 xw[32];  // this thread's row of the XW tile, its 64 columns (constant within a tile)
        int acc = 0, c = 0, loaded_tile = -1;
        uint32_t acc_phase = 0;
        bool ok = true;
        for (int t = t_begin; ok && t < t_end; ++t) {
            const int chunk = t % a.chunks, tile = t / a.chunks;
            const int m0 = (tile / a.tiles_n) * 128, n0 = (tile % a.tiles_n) * 128;
            if (tile != loaded_tile) {
                const int m = m0 + row;
#pragma unroll
                for (int i = 0; i < 64; i += 4) {
                    const int n = n0 + half * 64 + i;
                    float4 f = make_float4(0.f, 0.f, 0.f, 0.f);
                    if (m < a.M && n + 3 < a.N) f = *reinterpret_cast<const float4*>(a.XW + (int64_t)m * a.N + n);
                    xw[i / 2] = make_float2(f.x, f.y);
                    xw[i / 2 + 1] = make_float2(f.z, f.w);
                }
                loaded_tile = tile;
            }
            const int p1 = min(a.P, (chunk + 1) * a.chunk);
            for (int p = chunk * a.chunk; p < p1; ++p, ++c) {
                const int sb = c % EX_NSTG;
                const uint32_t use = (uint32_t)(c / EX_NSTG);
                if (!mbar_wait(&tmem_full[acc], acc_phase, 14)) { ok = false; break; }
                tc_fence_after();
                if (!mbar_wait(&stg_free[sb], (use & 1) ^ 1, 15)) { ok = false; break; }
                uint8_t* sub = smem + EX_STG + sb * EX_STG_BYTES + half * (128 * 128) + row * 128;
                uint32_t v[64];
                tmem_ld32_nowait(tmem_base + lane_addr + acc * 128 + half * 64, *reinterpret_cast<uint32_t(*)[32]>(v));
                tmem_ld32_nowait(tmem_base + lane_addr + acc * 128 + half * 64 + 32,
                                 *reinterpret_cast<uint32_t(*)[32]>(v + 32));
                asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
                uint32_t pk[32];
#pragma unroll
                for (int i = 0; i < 32; ++i) {
                    const float2 o = ffma2_tc(s2, make_float2(__uint_as_float(v[2 * i]), __uint_as_float(v[2 * i + 1])),
                                              xw[i]);
                    __nv_bfloat162 h = __floats2bfloat162_rn(o.x, o.y);
                    pk[i] = *reinterpret_cast<uint32_t*>(&h);
                }
                // 128B swizzle: 16-byte chunk k of a 128-byte row lives at k ^ (row % 8)
#pragma unroll
                for (int k = 0; k < 8; ++k)
                    *reinterpret_cast<uint4*>(sub + ((k ^ (row & 7)) * 16)) =
                        make_uint4(pk[4 * k], pk[4 * k + 1], pk[4 * k + 2], pk[4 * k + 3]);
                tc_fence_before();
                __syncwarp();
                if (lane == 0) mbar_arrive(&tmem_empty[acc]);
                if (++acc == EX_NACC) { acc = 0; acc_phase ^= 1; }
                asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
                mbar_arrive(&stg_full[sb]);
            }
        }
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    if (warp == 1) tmem_dealloc(tmem_base, 512);
}

// ---------------------------------------------------------------------------
// host side
// ---------------------------------------------------------------------------
PFN_cuTensorMapEncodeTiled_v12000 encode_fn() {
    static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
    static std::once_flag once;
    std::call_once(once, [] {
        void* p = nullptr;
        cudaDriverEntryPointQueryResult q;
        if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) == cudaSuccess &&
            q == cudaDriverEntryPointSuccess)
            fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(p);
    });
    return fn;
}

// 2-D bf16 tensor map over a row-major matrix [rows, inner] with leading
// dimension `ld` elements; box {box_inner, box_rows}, 128-byte swizzle.
bool make_map(CUtensorMap* m, const void* base, uint64_t inner, uint64_t rows, uint64_t ld, uint32_t box_inner,
              uint32_t box_rows) {
    auto fn = encode_fn();
    if (!fn) return false;
    cuuint64_t dims[2] = {inner, rows};
    cuuint64_t strides[1] = {ld * 2};
    cuuint32_t box[2] = {box_inner, box_rows};
    cuuint32_t estr[2] = {1, 1};
    CUresult r = fn(m, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, const_cast<void*>(base), dims, strides, box, estr,
                    CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                    CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    return r == CUDA_SUCCESS;
}

bool make_map_2d(CUtensorMap* m, const void* base, uint64_t inner, uint64_t rows, uint64_t ld, uint32_t box_inner,
                 uint32_t box_rows, CUtensorMapSwizzle swz) {
    auto fn = encode_fn();
    if (!fn) return false;
    cuuint64_t dims[2] = {inner, rows};
    cuuint64_t strides[1] = {ld * 2};
    cuuint32_t box[2] = {box_inner, box_rows};
    cuuint32_t estr[2] = {1, 1};
    return fn(m, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, const_cast<void*>(base), dims, strides, box, estr,
              CU_TENSOR_MAP_INTERLEAVE_NONE, swz, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
              CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

// y [P, M, N] bf16 as a 3-D map so a tile never crosses into the next candidate.
bool make_map_y(CUtensorMap* m, void* base, uint64_t N, uint64_t M, uint64_t P) {
    auto fn = encode_fn();
    if (!fn) return false;
    cuuint64_t dims[3] = {N, M, P};
    cuuint64_t strides[2] = {N * 2, M * N * 2};
    cuuint32_t box[3] = {64, 128, 1};
    cuuint32_t estr[3] = {1, 1, 1};
    return fn(m, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 3, base, dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
              CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_NONE,
              CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

int num_sms() {
    static int n = 0;
    if (!n) {
        int dev = 0;
        cudaGetDevice(&dev);
        cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev);
        if (n <= 0) n = 148;
    }
    return n;
}

template <int BN, bool B_MN>
int launch_tc(const CUtensorMap& ta, const CUtensorMap& tb, const TcArgs& a, cudaStream_t st, const char* name) {
    constexpr size_t smem = (size_t)gemm_stages(BN) * (BM * BK * 2 + BN * BK * 2) + 1024;
    if (cudaFuncSetAttribute(tc_gemm_kernel<BN, B_MN>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem) !=
        cudaSuccess)
        return zg::fail(ZG_ERR_CUDA, "tc_gemm: shared memory attribute");
    int tiles = a.tiles_m * a.tiles_n * a.splits;
    int grid = tiles < num_sms() ? tiles : num_sms();
    zg::LaunchTimer zg_lt_(name, st);
    tc_gemm_kernel<BN, B_MN><<<grid, THREADS, smem, st>>>(ta, tb, a);
    return zg::check_launch("tc_gemm");
}

// CTA pairs that can be resident at once for the pair kernel (0 if unknown).
template <bool B_MN>
int pair_slots() {
    static int n = -1;
    if (n < 0) {
        constexpr size_t smem = (size_t)P2_SMEM + 1024;
        n = 0;
        if (cudaFuncSetAttribute(tc_gemm_pair_kernel<B_MN>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem) ==
            cudaSuccess) {
            cudaLaunchConfig_t cfg = {};
            cfg.gridDim = dim3(2 * 74, 1, 1);
            cfg.blockDim = dim3(THREADS, 1, 1);
            cfg.dynamicSmemBytes = smem;
            int clusters = 0;
            if (cudaOccupancyMaxActiveClusters(&clusters, tc_gemm_pair_kernel<B_MN>, &cfg) == cudaSuccess)
                n = clusters;
        }
        cudaGetLastError();
    }
    return n;
}

template <bool B_MN>
int launch_tc_pair(const CUtensorMap& ta, const CUtensorMap& tb, const TcArgs& a, int slots, cudaStream_t st,
                   const char* name) {
    constexpr size_t smem = (size_t)P2_SMEM + 1024;
    const int tiles = a.tiles_m * a.tiles_n * a.splits;
    const int pairs = tiles < slots ? tiles : slots;
    zg::LaunchTimer zg_lt_(name, st);
    tc_gemm_pair_kernel<B_MN><<<2 * pairs, THREADS, smem, st>>>(ta, tb, a);
    return zg::check_launch("tc_gemm_pair");
}

}  // namespace

namespace zg {

bool tc_available() {
    static int ok = -1;
    if (ok < 0) {
        int dev = 0, major = 0, minor = 0;
        cudaGetDevice(&dev);
        cudaDeviceGetAttribute(&major, cudaDevAttrComputeCapabilityMajor, dev);
        cudaDeviceGetAttribute(&minor, cudaDevAttrComputeCapabilityMinor, dev);
        ok = (major == 10 && minor == 0 && encode_fn() != nullptr) ? 1 : 0;
    }
    return ok == 1;
}

bool tensor_map_bf16(CUtensorMap* m, const void* base, int rank, const uint64_t* dims, const uint64_t* strides_bytes,
                     const uint32_t* box, bool swizzle128) {
    return tensor_map_bf16_swz(m, base, rank, dims, strides_bytes, box, swizzle128 ? 128 : 0);
}

bool tensor_map_bf16_swz(CUtensorMap* m, const void* base, int rank, const uint64_t* dims,
                         const uint64_t* strides_bytes, const uint32_t* box, int swizzle_bytes) {
    auto fn = encode_fn();
    const CUtensorMapSwizzle swz = swizzle_bytes == 128 ? CU_TENSOR_MAP_SWIZZLE_128B
                                   : swizzle_bytes == 64 ? CU_TENSOR_MAP_SWIZZLE_64B
                                                         : CU_TENSOR_MAP_SWIZZLE_NONE;
    if (!fn || rank < 1 || rank > 5) return false;
    cuuint64_t d[5], s[4];
    cuuint32_t b[5], e[5];
    for (int i = 0; i < rank; ++i) {
        d[i] = dims[i];
        b[i] = box[i];
        e[i] = 1;
        if (i + 1 < rank) s[i] = strides_bytes[i];
    }
    return fn(m, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, rank, const_cast<void*>(base), d, s, b, e,
              CU_TENSOR_MAP_INTERLEAVE_NONE, swz, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
              CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

// One GEMM launch: D = alpha * A B^T over `splits` of `split_total` equal K
// ranges of k_split elements each (split z of the launch -> D + z * d_split).
// The kernel and tile width are chosen from the split_total-range problem,
// so a range computed alone (split_total > splits) runs the same kernel and
// tile schedule, and gives the same bits, as in a launch of all of them.
int tc_gemm_core(const void* A, int64_t lda, const void* B, int64_t ldb, bool b_mn_major, void* D, int64_t ldd,
                 bool out_bf16, int M, int N, int splits, int split_total, int k_split, int64_t d_split, float alpha,
                 cudaStream_t st, const char* name, const FusedStep* step) {
    if (M <= 0 || N <= 0 || k_split <= 0 || splits < 1 || split_total < splits)
        return fail(ZG_ERR_INVALID, "tc_gemm: empty problem");
    if (!D && !(step && step->kind != ZG_STEP_NONE)) return fail(ZG_ERR_INVALID, "tc_gemm: no output");
    if (splits > 1 && (k_split % BK || (step && step->kind != ZG_STEP_NONE)))
        return fail(ZG_ERR_INVALID, "tc_gemm: split ranges need K %% 64 == 0 and no fused step");
    const int K = k_split * splits;
    const FusedStep no_step{};
    if ((lda % 8) || (ldb % 8) || (reinterpret_cast<uintptr_t>(A) & 15) || (reinterpret_cast<uintptr_t>(B) & 15))
        return fail(ZG_ERR_INVALID, "tc_gemm: operands need 16-byte aligned rows");
    // Tile width: the persistent grid finishes after ceil(tiles / SMs) tiles
    // per SM, each costing ~BN (narrower tiles re-read A more often, hence
    // the small penalty); take the cheapest.
    auto tiles = [&](int b) { return (int64_t)((M + BM - 1) / BM) * ((N + b - 1) / b) * split_total; };
    auto cost = [&](int b, double pen) {
        return (double)((tiles(b) + num_sms() - 1) / num_sms()) * b * pen;
    };
    int bn = 256;
    double best = cost(256, 1.0);
    if (cost(128, 1.3) < best) { bn = 128; best = cost(128, 1.3); }
    if (cost(64, 1.6) < best) { bn = 64; }
    const int kb_split = (k_split + BK - 1) / BK;
    CUtensorMap ta, tb;
    if (!make_map(&ta, A, K, M, lda, BK, BM)) return fail(ZG_ERR_CUDA, "tc_gemm: tensor map A");
    // At least one full wave of 256 x 256 tiles: CTA pairs (cta_group::2).
    const int64_t pair_tiles = (int64_t)((M + 255) / 256) * ((N + 255) / 256) * split_total;
    const int slots = b_mn_major ? pair_slots<true>() : pair_slots<false>();
    if (slots > 0 && pair_tiles >= slots) {
        bool okp = b_mn_major ? make_map(&tb, B, N, K, ldb, 64, BK) : make_map(&tb, B, K, N, ldb, BK, 128);
        if (!okp) return fail(ZG_ERR_CUDA, "tc_gemm: tensor map B");
        TcArgs a{D, ldd, M, N, K, alpha, out_bf16 ? 1 : 0, (M + 255) / 256, (N + 255) / 256, no_step,
                 splits, kb_split, d_split};
        if (step) a.step = *step;
        return b_mn_major ? launch_tc_pair<true>(ta, tb, a, slots, st, name)
                          : launch_tc_pair<false>(ta, tb, a, slots, st, name);
    }
    bool okb = b_mn_major ? make_map(&tb, B, N, K, ldb, 64, BK) : make_map(&tb, B, K, N, ldb, BK, bn);
    if (!okb) return fail(ZG_ERR_CUDA, "tc_gemm: tensor map B");
    TcArgs a{D, ldd, M, N, K, alpha, out_bf16 ? 1 : 0, (M + BM - 1) / BM, (N + bn - 1) / bn, no_step,
             splits, kb_split, d_split};
    if (step) a.step = *step;
    if (b_mn_major) {
        if (bn == 256) return launch_tc<256, true>(ta, tb, a, st, name);
        if (bn == 128) return launch_tc<128, true>(ta, tb, a, st, name);
        return launch_tc<64, true>(ta, tb, a, st, name);
    }
    if (bn == 256) return launch_tc<256, false>(ta, tb, a, st, name);
    if (bn == 128) return launch_tc<128, false>(ta, tb, a, st, name);
    return launch_tc<64, false>(ta, tb, a, st, name);
}

int split_reduce(const float* parts, const int64_t* offsets, int S, int64_t n, float alpha, const FusedStep* step,
                 float* out, cudaStream_t st) {
    if (S < 1 || S > kMaxSplits || n < 0 || !parts || !offsets) return fail(ZG_ERR_INVALID, "split reduce: bad splits");
    const bool has_step = step && step->kind != ZG_STEP_NONE;
    if (!has_step && !out) return fail(ZG_ERR_INVALID, "split reduce: no output");
    if (n == 0) return ZG_OK;
    SplitParts sp{};
    sp.S = S;
    for (int s = 0; s < S; ++s) sp.p[s] = parts + offsets[s];
    const FusedStep none{};
    const int64_t groups = (n + 7) / 8;
    int64_t grid = (groups + 255) / 256;
    const int64_t cap = (int64_t)num_sms() * 8;
    if (grid > cap) grid = cap;
    zg::LaunchTimer zg_lt_("replay_split_reduce", st);
    split_reduce_kernel<<<(unsigned)grid, 256, 0, st>>>(sp, n, alpha, has_step ? *step : none, out);
    return check_launch("replay_split_reduce");
}

int tc_gemm_bf16(const void* A, int64_t lda, const void* B, int64_t ldb, bool b_mn_major, void* D, int64_t ldd,
                 bool out_bf16, int M, int N, int K, float alpha, cudaStream_t st, const char* name,
                 const FusedStep* step) {
    return tc_gemm_core(A, lda, B, ldb, b_mn_major, D, ldd, out_bf16, M, N, 1, 1, K, 0, alpha, st, name, step);
}

}  // namespace zg

namespace zg {

bool tc_expand_ok(int P, int M, int N, int rank, const void* XW, const void* U, const void* Bq, const void* y) {
    auto al = [](const void* p, uintptr_t a) { return (reinterpret_cast<uintptr_t>(p) & (a - 1)) == 0; };
    return tc_available() && rank == 8 && N % 8 == 0 && M > 0 && P > 0 && al(XW, 16) && al(U, 16) && al(Bq, 16) &&
           al(y, 16);
}

int tc_expand_r8(const float* XW, const void* U, const void* Bq, int64_t ldb, int P, int M, int N, float s, void* y,
                 cudaStream_t st) {
    return tc_expand(XW, U, Bq, ldb, P, M, N, 8, s, y, st, "lowrank_expand");
}

int tc_expand(const float* XW, const void* U, const void* Bq, int64_t ldb, int P, int M, int N, int rank, float s,
              void* y, cudaStream_t st, const char* name) {
    if (rank != 8 && rank != 16) return fail(ZG_ERR_INVALID, "tc_expand: rank 8 or 16");
    CUtensorMap tu, tb, ty;
    const uint64_t q = (uint64_t)P * rank;
    if (!make_map_2d(&tu, U, q, M, q, 8, 128, CU_TENSOR_MAP_SWIZZLE_NONE) ||
        !make_map_2d(&tb, Bq, q, N, (uint64_t)ldb, 8, 128, CU_TENSOR_MAP_SWIZZLE_NONE) || !make_map_y(&ty, y, N, M, P))
        return fail(ZG_ERR_CUDA, "tc_expand: tensor maps");
    ExpandArgs a{XW, M, N, P, s, (M + 127) / 128, (N + 127) / 128, 0, 0};
    const int tiles = a.tiles_m * a.tiles_n;
    // ~8 candidates per item: fine enough that the contiguous per-CTA shares
    // balance to within one item, coarse enough that XW is reloaded rarely.
    int chunks = (P + 7) / 8;
    if (chunks < 1) chunks = 1;
    a.chunk = (P + chunks - 1) / chunks;
    a.chunks = (P + a.chunk - 1) / a.chunk;
    const int items = tiles * a.chunks;
    const int grid = items < num_sms() ? items : num_sms();
    // one CTA (and its 512 TMEM columns) per SM
    const size_t smem = EX_SMEM + 1024;
    if (cudaFuncSetAttribute(rank == 8 ? expand_tc_kernel<8> : expand_tc_kernel<16>,
                             cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem) != cudaSuccess)
        return fail(ZG_ERR_CUDA, "tc_expand: shared memory attribute");
    zg::LaunchTimer zg_lt_(name, st);
    if (rank == 8)
        expand_tc_kernel<8><<<grid, EX_THREADS, smem, st>>>(tu, tb, ty, a);
    else
        expand_tc_kernel<16><<<grid, EX_THREADS, smem, st>>>(tu, tb, ty, a);
    return check_launch("tc_expand");
}

}  // namespace zg

extern "C" int zg_gemm_bf16(const void* A, int64_t lda, const void* B, int64_t ldb, int b_mn_major, void* D,
                            int64_t ldd, int out_dtype, int M, int N, int K, float alpha, void* stream) {
    if (!A || !B || !D) return zg::fail(ZG_ERR_INVALID, "zg_gemm_bf16: null pointer");
    if (M < 1 || N < 1 || K < 1) return zg::fail(ZG_ERR_INVALID, "zg_gemm_bf16: bad sizes");
    if (!zg::dtype_ok(out_dtype)) return zg::fail(ZG_ERR_INVALID, "zg_gemm_bf16: bad output dtype");
    if (!zg::tc_available()) return zg::fail(ZG_ERR_UNSUPPORTED, "zg_gemm_bf16: needs an sm_100 device");
    return zg::tc_gemm_bf16(A, lda, B, ldb, b_mn_major != 0, D, ldd, out_dtype == ZG_BF16, M, N, K, alpha,
                            zg::as_stream(stream));
}

extern "C" int zg_device_error(int clear) {
    // one error word per translation unit with tensor-core kernels
    const int w[5] = {ptx_error_word(clear), zg::batched_error_word(clear), zg::int8_error_word(clear),
                      zg::ce_error_word(clear), zg::attn_error_word(clear)};
    for (int e : w)
        if (e < 0) return -1;
    for (int e : w)
        if (e) return e;
    return 0;
}
