// zg_batched.cu -- population forward with one input per candidate (the
// hidden-layer case of perturbed_linear / perturbed_tied_logits,
// src/zerograd/_candidate.py:17-22,33-38, called under vmap with a batched x)
// on the tcgen05 tensor cores, in two kernels:
//
//   u pass:  U[p, m, 0:16] = bf16(s * x_p[m, :] . F1_p)       columns >= r are 0
//   gemm:    y[p, m, n]    = bf16(x_p[m, :] . Wop[:, n] + U[p, m, :] . F2[n, p r : p r + 16])
//
// F1T [P r, K] holds each candidate's input-side factor K-major (A of a
// MATRIX entry, B of a tied TABLE); F2 [N, P r] is the output-side factor in
// operand layout.  The low-rank term enters the GEMM as one extra
// M=128 N=256 K=16 MMA into the tile's TMEM accumulator after its K loop, so
// every output element is rounded once.
//
// Both kernels: warp 0 = TMA producer, warp 1 = TMEM allocator + MMA issuer,
// warps 2..5 = epilogue; persistent CTAs; two TMEM accumulators so one tile's
// epilogue overlaps the next tile's main loop.  Every mbarrier wait is
// bounded: on expiry the kernel records an error code, drains its own TMA
// copies, frees its TMEM and returns.
#include <climits>

#include "zg_ptx.cuh"
#include "zg_tc.cuh"

namespace {

constexpr int THREADS = 192, BM = 128, BK = 64;

int sm_count_b() {
    static int n = 0;
    if (!n) {
        int dev = 0;
        cudaGetDevice(&dev);
        cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev);
        if (n <= 0) n = 148;
    }
    return n;
}

// ---------------------------------------------------------------------------
// u pass: M=128 N=16 MMAs; the 16 factor rows of a tile are candidate p's r
// rows (and, for r = 8, the next candidate's, whose products the epilogue
// discards).
// ---------------------------------------------------------------------------
constexpr int UP_STAGES = 8;
constexpr uint32_t UP_X = BM * BK * 2;      // 16 KiB input tile
constexpr uint32_t UP_F = 16 * BK * 2;      // 2 KiB factor tile
constexpr uint32_t UP_STAGE = UP_X + UP_F;  // 18 KiB: keeps every tile on a 1 KiB swizzle atom
constexpr uint32_t UP_SMEM = UP_STAGES * UP_STAGE;

struct UPassArgs {
    __nv_bfloat16* U;
    int M, K, P, rank, tiles_m;
    float s;
    int x_batched;  // 0: one input shared by every candidate
};

__global__ void __launch_bounds__(THREADS, 1)
batched_u_kernel(const __grid_constant__ CUtensorMap tmX, const __grid_constant__ CUtensorMap tmF, const UPassArgs a) {
    extern __shared__ uint8_t dyn_smem[];
    __shared__ __align__(8) uint64_t full_bar[UP_STAGES], empty_bar[UP_STAGES], tmem_full[2], tmem_empty[2], mma_done;
    __shared__ uint32_t tmem_base_sh;
    const uint32_t dyn_base = smem_u32(dyn_smem);
    uint8_t* smem = dyn_smem + (((dyn_base + 1023u) & ~1023u) - dyn_base);
    const int warp = threadIdx.x / 32, lane = threadIdx.x % 32;
    const int num_tiles = a.P * a.tiles_m;
    const int k_blocks = (a.K + BK - 1) / BK;

    if (threadIdx.x == 0) {
        for (int s = 0; s < UP_STAGES; ++s) {
            mbar_init(&full_bar[s], 1);
            mbar_init(&empty_bar[s], 1);
        }
        for (int b = 0; b < 2; ++b) {
            mbar_init(&tmem_full[b], 1);
            mbar_init(&tmem_empty[b], 4);
        }
        mbar_init(&mma_done, 1);
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    }
    if (warp == 1) tmem_alloc(&tmem_base_sh, 32);
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem_base = tmem_base_sh;

    if (warp == 0 && lane == 0) {
        int stage = 0;
        uint32_t phase = 0, issued = 0, issue_parity = 0;
        bool ok = true;
        for (int t = blockIdx.x; ok && t < num_tiles; t += gridDim.x) {
            const int p = t / a.tiles_m, tm = t % a.tiles_m;
            for (int kb = 0; kb < k_blocks; ++kb) {
                if (!mbar_wait(&empty_bar[stage], phase ^ 1, 31)) { ok = false; break; }
                uint8_t* sx = smem + stage * UP_STAGE;
                mbar_expect_tx(&full_bar[stage], UP_STAGE);
                tma_load_3d(sx, &tmX, &full_bar[stage], kb * BK, tm * BM, a.x_batched ? p : 0);
                tma_load_2d(sx + UP_X, &tmF, &full_bar[stage], kb * BK, p * a.rank);
                issued |= 1u << stage;
                issue_parity = (issue_parity & ~(1u << stage)) | (phase << stage);
                if (++stage == UP_STAGES) { stage = 0; phase ^= 1; }
            }
        }
        for (int s = 0; s < UP_STAGES; ++s)
            if (issued & (1u << s))
                for (uint32_t i = 0; i < kSpinLimit; ++i)
                    if (mbar_try_wait(&full_bar[s], (issue_parity >> s) & 1)) break;
    } else if (warp == 1 && lane == 0) {
        constexpr uint32_t IDESC = idesc_bf16(BM, 16, 0);
        int stage = 0, acc = 0;
        uint32_t phase = 0, acc_phase = 0;
        bool ok = true;
        for (int t = blockIdx.x; ok && t < num_tiles; t += gridDim.x) {
            if (!mbar_wait(&tmem_empty[acc], acc_phase ^ 1, 32)) break;
            tc_fence_after();
            const uint32_t d_tmem = tmem_base + acc * 16;
            for (int kb = 0; kb < k_blocks; ++kb) {
                if (!mbar_wait(&full_bar[stage], phase, 33)) { ok = false; break; }
                tc_fence_after();
                const uint32_t x_addr = smem_u32(smem + stage * UP_STAGE);
                const uint32_t f_addr = x_addr + UP_X;
#pragma unroll
                for (int k = 0; k < BK / 16; ++k)
                    umma_bf16(d_tmem, smem_desc(x_addr + k * 32, 16, 1024), smem_desc(f_addr + k * 32, 16, 1024),
                              IDESC, (kb > 0 || k > 0) ? 1u : 0u);
                umma_commit(&empty_bar[stage]);
                if (++stage == UP_STAGES) { stage = 0; phase ^= 1; }
            }
            if (!ok) break;
            umma_commit(&tmem_full[acc]);
            if (++acc == 2) { acc = 0; acc_phase ^= 1; }
        }
        umma_commit(&mma_done);
        for (uint32_t i = 0; i < kSpinLimit; ++i)
            if (mbar_try_wait(&mma_done, 0)) break;
    } else if (warp >= 2) {
        const int quad = warp % 4;
        int acc = 0;
        uint32_t acc_phase = 0;
        for (int t = blockIdx.x; t < num_tiles; t += gridDim.x) {
            if (!mbar_wait(&tmem_full[acc], acc_phase, 34)) break;
            tc_fence_after();
            const int p = t / a.tiles_m, tm = t % a.tiles_m;
            const int row = tm * BM + quad * 32 + lane;
            float v[16];
            tmem_ld16(tmem_base + ((uint32_t)(quad * 32) << 16) + acc * 16, v);
            tc_fence_before();
            __syncwarp();
            if (lane == 0) mbar_arrive(&tmem_empty[acc]);
            if (++acc == 2) { acc = 0; acc_phase ^= 1; }
            if (row < a.M) {
                uint4 pk[2];
                __nv_bfloat162* h = reinterpret_cast<__nv_bfloat162*>(pk);
#pragma unroll
                for (int j = 0; j < 8; ++j)
                    h[j] = __floats2bfloat162_rn(2 * j < a.rank ? a.s * v[2 * j] : 0.f,
                                                 2 * j + 1 < a.rank ? a.s * v[2 * j + 1] : 0.f);
                uint4* dst = reinterpret_cast<uint4*>(a.U + ((int64_t)p * a.M + row) * 16);
                dst[0] = pk[0];
                dst[1] = pk[1];
            }
        }
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    if (warp == 1) tmem_dealloc(tmem_base, 32);
}

// ---------------------------------------------------------------------------
// gemm with the low-rank correction: 128 x 256 tiles, 4-stage ring of
// 48 KiB (x tile + Wop tile), plus per accumulator a 12 KiB correction
// buffer (U tile [128, 16] and F2 tile [256, 16], each as two 8-column
// halves in the no-swizzle K-major layout).
// ---------------------------------------------------------------------------
constexpr int BG_BN = 256, BG_STAGES = 4;
constexpr uint32_t BG_A = BM * BK * 2;                            // 16 KiB
constexpr uint32_t BG_B = BG_BN * BK * 2;                         // 32 KiB
constexpr uint32_t BG_STAGE = BG_A + BG_B;                        // 48 KiB
constexpr uint32_t BG_CU = BM * 16;                               // 8 K columns of the U tile
constexpr uint32_t BG_CF = BG_BN * 16;                            // 8 K columns of the F2 tile
constexpr uint32_t BG_CORR = 2 * BG_CU + 2 * BG_CF;               // 12 KiB
constexpr uint32_t BG_SMEM = BG_STAGES * BG_STAGE + 2 * BG_CORR;  // 216 KiB

struct GemmArgs {
    __nv_bfloat16* y;
    int M, N, K, P, rank, tiles_m, tiles_n;
    const __nv_bfloat16* res;  // residual [P, M, N] added after the activation, or null
    int act;                   // ZG_ACT_NONE / ZG_ACT_GELU
};

template <bool B_MN>
__global__ void __launch_bounds__(THREADS, 1)
batched_gemm_kernel(const __grid_constant__ CUtensorMap tmX, const __grid_constant__ CUtensorMap tmW,
                    const __grid_constant__ CUtensorMap tmU, const __grid_constant__ CUtensorMap tmF,
                    const GemmArgs a) {
    extern __shared__ uint8_t dyn_smem[];
    __shared__ __align__(8) uint64_t full_bar[BG_STAGES], empty_bar[BG_STAGES], tmem_full[2], tmem_empty[2],
        corr_full[2], corr_empty[2], mma_done;
    __shared__ uint32_t tmem_base_sh;
    const uint32_t dyn_base = smem_u32(dyn_smem);
    uint8_t* smem = dyn_smem + (((dyn_base + 1023u) & ~1023u) - dyn_base);
    uint8_t* corr = smem + BG_STAGES * BG_STAGE;
    const int warp = threadIdx.x / 32, lane = threadIdx.x % 32;
    const int num_tiles = a.P * a.tiles_m * a.tiles_n;
    const int k_blocks = (a.K + BK - 1) / BK;

    if (threadIdx.x == 0) {
        for (int s = 0; s < BG_STAGES; ++s) {
            mbar_init(&full_bar[s], 1);
            mbar_init(&empty_bar[s], 1);
        }
        for (int b = 0; b < 2; ++b) {
            mbar_init(&tmem_full[b], 1);
            mbar_init(&tmem_empty[b], 4);
            mbar_init(&corr_full[b], 1);
            mbar_init(&corr_empty[b], 1);
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
        // ---------------- TMA producer ----------------
        int stage = 0, acc = 0;
        uint32_t phase = 0, acc_phase = 0;
        uint32_t issued = 0, issue_parity = 0, c_issued = 0, c_parity = 0;
        bool ok = true;
        for (int t = blockIdx.x; ok && t < num_tiles; t += gridDim.x) {
            const int tn = t % a.tiles_n, rest = t / a.tiles_n;
            const int tm = rest % a.tiles_m, p = rest / a.tiles_m;
            // correction operands of this tile
            if (!mbar_wait(&corr_empty[acc], acc_phase ^ 1, 41)) break;
            uint8_t* c = corr + acc * BG_CORR;
            mbar_expect_tx(&corr_full[acc], BG_CORR);
            tma_load_3d(c, &tmU, &corr_full[acc], 0, tm * BM, p);
            tma_load_3d(c + BG_CU, &tmU, &corr_full[acc], 8, tm * BM, p);
            tma_load_2d(c + 2 * BG_CU, &tmF, &corr_full[acc], p * a.rank, tn * BG_BN);
            tma_load_2d(c + 2 * BG_CU + BG_CF, &tmF, &corr_full[acc], p * a.rank + 8, tn * BG_BN);
            c_issued |= 1u << acc;
            c_parity = (c_parity & ~(1u << acc)) | (acc_phase << acc);
            if (++acc == 2) { acc = 0; acc_phase ^= 1; }
            // main loop operands; tiles start their K sweep at different blocks
            // so CTAs sharing an operand tile do not request the same lines at once
            // K sweeps start at different blocks for neighbouring tiles (so CTAs
            // sharing an operand tile do not request the same lines at once),
            // by the tile's place in its candidate's output only: a
            // candidate's result does not depend on its position in the batch
            const int k_start = (tm * a.tiles_n + tn) % k_blocks;
            for (int kb = 0; kb < k_blocks; ++kb) {
                if (!mbar_wait(&empty_bar[stage], phase ^ 1, 42)) { ok = false; break; }
                const int kk = kb + k_start < k_blocks ? kb + k_start : kb + k_start - k_blocks;
                uint8_t* sa = smem + stage * BG_STAGE;
                uint8_t* sb = sa + BG_A;
                mbar_expect_tx(&full_bar[stage], BG_STAGE);
                tma_load_3d(sa, &tmX, &full_bar[stage], kk * BK, tm * BM, p);
                if constexpr (B_MN) {
#pragma unroll
                    for (int cc = 0; cc < BG_BN / 64; ++cc)
                        tma_load_2d(sb + cc * (64 * BK * 2), &tmW, &full_bar[stage], tn * BG_BN + cc * 64, kk * BK);
                } else {
                    tma_load_2d(sb, &tmW, &full_bar[stage], kk * BK, tn * BG_BN);
                }
                issued |= 1u << stage;
                issue_parity = (issue_parity & ~(1u << stage)) | (phase << stage);
                if (++stage == BG_STAGES) { stage = 0; phase ^= 1; }
            }
        }
        for (int s = 0; s < BG_STAGES; ++s)
            if (issued & (1u << s))
                for (uint32_t i = 0; i < kSpinLimit; ++i)
                    if (mbar_try_wait(&full_bar[s], (issue_parity >> s) & 1)) break;
        for (int b = 0; b < 2; ++b)
            if (c_issued & (1u << b))
                for (uint32_t i = 0; i < kSpinLimit; ++i)
                    if (mbar_try_wait(&corr_full[b], (c_parity >> b) & 1)) break;
    } else if (warp == 1 && lane == 0) {
        // ---------------- MMA issuer ----------------
        constexpr uint32_t IDESC = idesc_bf16(BM, BG_BN, B_MN ? 1 : 0);
        constexpr uint32_t IDESC_C = idesc_bf16(BM, BG_BN, 0);
        int stage = 0, acc = 0;
        uint32_t phase = 0, acc_phase = 0;
        bool ok = true;
        for (int t = blockIdx.x; ok && t < num_tiles; t += gridDim.x) {
            if (!mbar_wait(&tmem_empty[acc], acc_phase ^ 1, 43)) break;
            tc_fence_after();
            const uint32_t d_tmem = tmem_base + acc * BG_BN;
            for (int kb = 0; kb < k_blocks; ++kb) {
                if (!mbar_wait(&full_bar[stage], phase, 44)) { ok = false; break; }
                tc_fence_after();
                const uint32_t a_addr = smem_u32(smem + stage * BG_STAGE);
                const uint32_t b_addr = a_addr + BG_A;
#pragma unroll
                for (int k = 0; k < BK / 16; ++k) {
                    const uint64_t ad = smem_desc(a_addr + k * 32, 16, 1024);
                    // MN-major SW128: 64-wide N blocks 8 KiB apart, 8-row K groups 1 KiB apart
                    const uint64_t bd = B_MN ? smem_desc(b_addr + k * 2048, 64 * BK * 2, 1024)
                                             : smem_desc(b_addr + k * 32, 16, 1024);
                    umma_bf16(d_tmem, ad, bd, IDESC, (kb > 0 || k > 0) ? 1u : 0u);
                }
                umma_commit(&empty_bar[stage]);
                if (++stage == BG_STAGES) { stage = 0; phase ^= 1; }
            }
            if (!ok) break;
            // low-rank correction: U tile [128, 16] . F2 tile [256, 16]^T into the same accumulator
            if (!mbar_wait(&corr_full[acc], acc_phase, 45)) break;
            tc_fence_after();
            const uint32_t c_addr = smem_u32(corr + acc * BG_CORR);
            umma_bf16(d_tmem, smem_desc_noswizzle(c_addr, BG_CU, 128),
                      smem_desc_noswizzle(c_addr + 2 * BG_CU, BG_CF, 128), IDESC_C, 1u);
            umma_commit(&corr_empty[acc]);
            umma_commit(&tmem_full[acc]);
            if (++acc == 2) { acc = 0; acc_phase ^= 1; }
        }
        umma_commit(&mma_done);
        for (uint32_t i = 0; i < kSpinLimit; ++i)
            if (mbar_try_wait(&mma_done, 0)) break;
    } else if (warp >= 2) {
        // ---------------- epilogue: TMEM -> bf16 -> global ----------------
        const int quad = warp % 4;
        int acc = 0;
        uint32_t acc_phase = 0;
        for (int t = blockIdx.x; t < num_tiles; t += gridDim.x) {
            if (!mbar_wait(&tmem_full[acc], acc_phase, 46)) break;
            tc_fence_after();
            const int tn = t % a.tiles_n, rest = t / a.tiles_n;
            const int tm = rest % a.tiles_m, p = rest / a.tiles_m;
            const int row = tm * BM + quad * 32 + lane;
            const int64_t row_off = ((int64_t)p * a.M + row) * a.N;
#pragma unroll 1
            for (int c0 = 0; c0 < BG_BN; c0 += 32) {
                float v[32];
                tmem_ld32(tmem_base + ((uint32_t)(quad * 32) << 16) + acc * BG_BN + c0, v);
                const int col0 = tn * BG_BN + c0;
                if (row >= a.M || col0 >= a.N) continue;
                zg_store_row32(v, a.y + row_off + col0, a.res ? a.res + row_off + col0 : nullptr, a.act, a.N - col0);
            }
            tc_fence_before();
            __syncwarp();
            if (lane == 0) mbar_arrive(&tmem_empty[acc]);
            if (++acc == 2) { acc = 0; acc_phase ^= 1; }
        }
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    if (warp == 1) tmem_dealloc(tmem_base, 512);
}

// ---------------------------------------------------------------------------
// The same GEMM on CTA pairs: 256 x 256 tiles, CTA r of the pair stages rows
// [128 r, 128 r + 128) of the x tile and columns [128 r, 128 r + 128) of the
// Wop tile (32 KiB per K block, 5 stages), plus its halves of the correction
// operands (U rows, F2 rows: 8 KiB per accumulator); the leader issues the
// M=256 N=256 MMAs, the correction included, into both CTAs' TMEM.
//
// Epilogue: eight warps per CTA, two per TMEM lane quadrant, each owning 32
// rows and 128 of the tile's 256 columns, in boxes of 32 x 32.  A box goes
// TMEM -> registers -> (activation, residual) -> bf16 -> a 64-byte-swizzled
// staging buffer -> one TMA bulk store issued by the warp's lane 0, so every
// HBM write is a full box of lines (a lane storing its own row straight to
// global memory touches 32 lines per store instruction, and the load/store
// unit then takes a cycle per line).  A residual box is brought into the
// same staging buffer by a TMA load first.  Two staging buffers per warp; a
// buffer is rewritten once the bulk store issued from it two boxes earlier
// has read it.
// ---------------------------------------------------------------------------
constexpr int BP_THREADS = 320;                                    // warp 0 TMA, 1 MMA, 2..9 epilogue
// NB staging boxes per epilogue warp: 2 (double-buffered; the residual's
// TMA load into the next box runs while the last box is stored) or 1 for
// GEMMs without a residual, whose freed 16 KiB buy a sixth operand stage:
// the main loop waits on operand loads for about a third of its time with
// five (the tile's L2 demand, 32 KiB per CTA per 64-deep K block).
__host__ __device__ constexpr int bp_stages(int nb) { return nb == 1 ? 6 : 5; }
constexpr uint32_t BP_A = BM * BK * 2;                             // 16 KiB: 128 rows of x
constexpr uint32_t BP_B = 128 * BK * 2;                            // 16 KiB: 128 columns of Wop
constexpr uint32_t BP_STAGE = BP_A + BP_B;                         // 32 KiB
constexpr uint32_t BP_CU = 128 * 16;                               // 8 K columns of 128 U rows
constexpr uint32_t BP_CF = 128 * 16;                               // 8 K columns of 128 F2 rows
constexpr uint32_t BP_CORR = 2 * BP_CU + 2 * BP_CF;                // 8 KiB per accumulator
constexpr uint32_t BP_BOX = 32 * 32 * 2;                           // 2 KiB: 32 rows x 32 bf16 columns
__host__ __device__ constexpr uint32_t bp_stg(int nb) { return bp_stages(nb) * BP_STAGE + 2 * BP_CORR; }  // staging offset (1 KiB aligned)
__host__ __device__ constexpr uint32_t bp_smem(int nb) { return bp_stg(nb) + 8 * nb * BP_BOX; }            // 208 / 224 KiB

// Byte offset of the 16-byte chunk `c` (0..3) of row `r` (0..31) in a
// 32 x 32 bf16 box with 64-byte swizzle: chunk bits [4,6) ^= address bits [7,9).
__device__ __forceinline__ uint32_t box64_off(int r, int c) { return (uint32_t)(r * 64 + ((c ^ ((r >> 1) & 3)) << 4)); }

template <bool B_MN, int NB>
__global__ void __cluster_dims__(2, 1, 1) __launch_bounds__(BP_THREADS, 1)
batched_gemm_pair_kernel(const __grid_constant__ CUtensorMap tmX, const __grid_constant__ CUtensorMap tmW,
                         const __grid_constant__ CUtensorMap tmU, const __grid_constant__ CUtensorMap tmF,
                         const __grid_constant__ CUtensorMap tmY, const __grid_constant__ CUtensorMap tmR,
                         const GemmArgs a) {
    extern __shared__ uint8_t dyn_smem[];
    constexpr int BP_STAGES = bp_stages(NB);
    constexpr uint32_t BP_STG = bp_stg(NB);
    __shared__ __align__(8) uint64_t full_bar[BP_STAGES], empty_bar[BP_STAGES], tmem_full[2], tmem_empty[2],
        corr_full[2], corr_empty[2], mma_done, res_bar[16];
    __shared__ uint32_t tmem_base_sh;
    const uint32_t dyn_base = smem_u32(dyn_smem);
    uint8_t* smem = dyn_smem + (((dyn_base + 1023u) & ~1023u) - dyn_base);
    uint8_t* corr = smem + BP_STAGES * BP_STAGE;
    const int warp = threadIdx.x / 32, lane = threadIdx.x % 32;
    const uint32_t rank = cluster_rank();
    const int pair = blockIdx.x / 2, pairs = gridDim.x / 2;
    const int num_tiles = a.P * a.tiles_m * a.tiles_n;  // tiles of 256 x 256
    const int k_blocks = (a.K + BK - 1) / BK;

    if (threadIdx.x == 0) {
        for (int s = 0; s < BP_STAGES; ++s) {
            mbar_init(&full_bar[s], 1);
            mbar_init(&empty_bar[s], 1);
        }
        for (int b = 0; b < 2; ++b) {
            mbar_init(&tmem_full[b], 1);
            mbar_init(&tmem_empty[b], 16);  // 8 epilogue warps in each CTA
            mbar_init(&corr_full[b], 1);
            mbar_init(&corr_empty[b], 1);
        }
        for (int b = 0; b < 16; ++b) mbar_init(&res_bar[b], 1);
        mbar_init(&mma_done, 1);
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    }
    if (warp == 1) tmem_alloc_pair(&tmem_base_sh, 512);
    tc_fence_before();
    cluster_sync();
    tc_fence_after();
    const uint32_t tmem_base = tmem_base_sh;

    if (warp == 0 && lane == 0) {
        // ---------------- TMA producer (both CTAs) ----------------
        int stage = 0, acc = 0;
        uint32_t phase = 0, acc_phase = 0;
        uint32_t issued = 0, issue_parity = 0, c_issued = 0, c_parity = 0;
        bool ok = true;
        const int half = (int)rank * 128;
        for (int t = pair; ok && t < num_tiles; t += pairs) {
            const int tn = t % a.tiles_n, rest = t / a.tiles_n;
            const int tm = rest % a.tiles_m, p = rest / a.tiles_m;
            if (!mbar_wait(&corr_empty[acc], acc_phase ^ 1, 51)) break;
            uint8_t* c = corr + acc * BP_CORR;
            if (rank == 0) mbar_expect_tx(&corr_full[acc], 2 * BP_CORR);
            const uint32_t cb = cluster_addr(&corr_full[acc], 0);
            tma_load_3d_pair(c, &tmU, cb, 0, tm * 256 + half, p);
            tma_load_3d_pair(c + BP_CU, &tmU, cb, 8, tm * 256 + half, p);
            tma_load_2d_pair(c + 2 * BP_CU, &tmF, cb, p * a.rank, tn * 256 + half);
            tma_load_2d_pair(c + 2 * BP_CU + BP_CF, &tmF, cb, p * a.rank + 8, tn * 256 + half);
            c_issued |= 1u << acc;
            c_parity = (c_parity & ~(1u << acc)) | (acc_phase << acc);
            if (++acc == 2) { acc = 0; acc_phase ^= 1; }
            // K sweeps start at different blocks for neighbouring tiles, by the
            // tile's place in its candidate's output only (a candidate's result
            // does not depend on its position in the batch)
            const int k_start = (tm * a.tiles_n + tn) % k_blocks;
            for (int kb = 0; kb < k_blocks; ++kb) {
                if (!mbar_wait(&empty_bar[stage], phase ^ 1, 52)) { ok = false; break; }
                const int kk = kb + k_start < k_blocks ? kb + k_start : kb + k_start - k_blocks;
                uint8_t* sa = smem + stage * BP_STAGE;
                uint8_t* sb = sa + BP_A;
                if (rank == 0) mbar_expect_tx(&full_bar[stage], 2 * BP_STAGE);
                const uint32_t fb = cluster_addr(&full_bar[stage], 0);
                tma_load_3d_pair(sa, &tmX, fb, kk * BK, tm * 256 + half, p);
                if constexpr (B_MN) {
#pragma unroll
                    for (int cc = 0; cc < 2; ++cc)
                        tma_load_2d_pair(sb + cc * (64 * BK * 2), &tmW, fb, tn * 256 + half + cc * 64, kk * BK);
                } else {
                    tma_load_2d_pair(sb, &tmW, fb, kk * BK, tn * 256 + half);
                }
                issued |= 1u << stage;
                issue_parity = (issue_parity & ~(1u << stage)) | (phase << stage);
                if (++stage == BP_STAGES) { stage = 0; phase ^= 1; }
            }
        }
        // Drain: the leader sees the bytes land on its full barriers; the peer
        // sees its buffers released by the MMAs that consumed them.
        for (int s = 0; s < BP_STAGES; ++s)
            if (issued & (1u << s)) {
                uint64_t* bar = rank == 0 ? &full_bar[s] : &empty_bar[s];
                for (uint32_t i = 0; i < kSpinLimit; ++i)
                    if (mbar_try_wait(bar, (issue_parity >> s) & 1)) break;
            }
        for (int b = 0; b < 2; ++b)
            if (c_issued & (1u << b)) {
                uint64_t* bar = rank == 0 ? &corr_full[b] : &corr_empty[b];
                for (uint32_t i = 0; i < kSpinLimit; ++i)
                    if (mbar_try_wait(bar, (c_parity >> b) & 1)) break;
            }
    } else if (warp == 1 && lane == 0 && rank == 0) {
        // ---------------- MMA issuer (leader only) ----------------
        constexpr uint32_t IDESC = idesc_bf16(256, 256, B_MN ? 1 : 0);
        constexpr uint32_t IDESC_C = idesc_bf16(256, 256, 0);
        int stage = 0, acc = 0;
        uint32_t phase = 0, acc_phase = 0;
        bool ok = true;
        for (int t = pair; ok && t < num_tiles; t += pairs) {
            if (!mbar_wait(&tmem_empty[acc], acc_phase ^ 1, 53)) break;
            tc_fence_after();
            const uint32_t d_tmem = tmem_base + acc * 256;
            for (int kb = 0; kb < k_blocks; ++kb) {
                if (!mbar_wait(&full_bar[stage], phase, 54)) { ok = false; break; }
                tc_fence_after();
                const uint32_t a_addr = smem_u32(smem + stage * BP_STAGE);
                const uint32_t b_addr = a_addr + BP_A;
#pragma unroll
                for (int k = 0; k < BK / 16; ++k) {
                    const uint64_t ad = smem_desc(a_addr + k * 32, 16, 1024);
                    const uint64_t bd = B_MN ? smem_desc(b_addr + k * 2048, 64 * BK * 2, 1024)
                                             : smem_desc(b_addr + k * 32, 16, 1024);
                    umma_bf16_pair(d_tmem, ad, bd, IDESC, (kb > 0 || k > 0) ? 1u : 0u);
                }
                umma_commit_pair(smem_u32(&empty_bar[stage]));
                umma_commit_pair(cluster_addr(&empty_bar[stage], 1));
                if (++stage == BP_STAGES) { stage = 0; phase ^= 1; }
            }
            if (!ok) break;
            if (!mbar_wait(&corr_full[acc], acc_phase, 55)) break;
            tc_fence_after();
            const uint32_t c_addr = smem_u32(corr + acc * BP_CORR);
            umma_bf16_pair(d_tmem, smem_desc_noswizzle(c_addr, BP_CU, 128),
                           smem_desc_noswizzle(c_addr + 2 * BP_CU, BP_CF, 128), IDESC_C, 1u);
            umma_commit_pair(smem_u32(&corr_empty[acc]));
            umma_commit_pair(cluster_addr(&corr_empty[acc], 1));
            umma_commit_pair(smem_u32(&tmem_full[acc]));
            umma_commit_pair(cluster_addr(&tmem_full[acc], 1));
            if (++acc == 2) { acc = 0; acc_phase ^= 1; }
        }
        umma_commit_pair(smem_u32(&mma_done));
        for (uint32_t i = 0; i < kSpinLimit; ++i)
            if (mbar_try_wait(&mma_done, 0)) break;
    } else if (warp >= 2) {
        // ---------------- epilogue (both CTAs, own TMEM rows) ----------------
        const int ew = warp - 2;               // epilogue warp 0..7
        const int quad = warp % 4;             // TMEM lanes 32*quad .. 32*quad + 31
        const int half = ew / 4;               // tile columns 128*half .. 128*half + 127
        const uint32_t empty_leader = cluster_addr(&tmem_empty[0], 0);
        uint8_t* stg = smem + BP_STG + ew * NB * BP_BOX;
        uint64_t* rbar = &res_bar[ew * 2];
        const bool has_res = a.res != nullptr;
        int acc = 0;
        uint32_t acc_phase = 0, box = 0, rphase = 0;
        bool ok = true;
        for (int t = pair; ok && t < num_tiles; t += pairs) {
            if (!mbar_wait(&tmem_full[acc], acc_phase, 56)) break;
            tc_fence_after();
            const int tn = t % a.tiles_n, rest = t / a.tiles_n;
            const int tm = rest % a.tiles_m, p = rest / a.tiles_m;
            const int row0 = tm * 256 + (int)rank * 128 + quad * 32;  // the box's first row
            const uint32_t t_addr = tmem_base + ((uint32_t)(quad * 32) << 16) + acc * 256 + half * 128;
#pragma unroll 1
            for (int ch = 0; ch < 4; ++ch, ++box) {
                const int b = (int)(box % NB);
                uint8_t* buf = stg + b * BP_BOX;
                const int col0 = tn * 256 + half * 128 + ch * 32;
                const bool active = row0 < a.M && col0 < a.N;  // warp-uniform; TMA clips partial boxes
                if (lane == 0) {
                    // the store issued from this buffer NB boxes ago has read it
                    if constexpr (NB == 2) asm volatile("cp.async.bulk.wait_group.read 1;" ::: "memory");
                    else asm volatile("cp.async.bulk.wait_group.read 0;" ::: "memory");
                    if (has_res && active) {
                        mbar_expect_tx(&rbar[b], BP_BOX);
                        tma_load_3d(buf, &tmR, &rbar[b], col0, row0, p);
                    }
                }
                __syncwarp();
                float v[32];
                tmem_ld32(t_addr + ch * 32, v);
                if (ch == 3) {
                    // the accumulator is read: release it to the MMA issuer
                    tc_fence_before();
                    __syncwarp();
                    if (lane == 0) mbar_arrive_remote(empty_leader + acc * (uint32_t)sizeof(uint64_t));
                }
                if (!active) continue;
                uint4 rv[4];
                if (has_res) {
                    if (!mbar_wait(&rbar[b], (rphase >> b) & 1, 57)) { ok = false; break; }
                    rphase ^= 1u << b;
#pragma unroll
                    for (int c = 0; c < 4; ++c) rv[c] = *reinterpret_cast<const uint4*>(buf + box64_off(lane, c));
                }
#pragma unroll
                for (int c = 0; c < 4; ++c) {
                    __nv_bfloat162 h[4];
#pragma unroll
                    for (int j = 0; j < 4; ++j) {
                        float r0 = 0.f, r1 = 0.f;
                        if (has_res) {
                            const __nv_bfloat162 rr = reinterpret_cast<const __nv_bfloat162*>(&rv[c])[j];
                            r0 = __bfloat162float(rr.x);
                            r1 = __bfloat162float(rr.y);
                        }
                        const float2 o = zg_epilogue_pair(v[8 * c + 2 * j], v[8 * c + 2 * j + 1], a.act, has_res,
                                                          r0, r1);
                        h[j] = __floats2bfloat162_rn(o.x, o.y);
                    }
                    *reinterpret_cast<uint4*>(buf + box64_off(lane, c)) = *reinterpret_cast<uint4*>(h);
                }
                asm volatile("fence.proxy.async.shared::cta;" ::: "memory");  // visible to the bulk store
                __syncwarp();
                if (lane == 0) {
                    tma_store_3d(&tmY, buf, col0, row0, p);
                    asm volatile("cp.async.bulk.commit_group;" ::: "memory");
                }
            }
            if (++acc == 2) { acc = 0; acc_phase ^= 1; }
        }
        if (lane == 0) asm volatile("cp.async.bulk.wait_group 0;" ::: "memory");
        __syncwarp();
    }
    tc_fence_before();
    cluster_sync();
    tc_fence_after();
    if (warp == 1) tmem_dealloc_pair(tmem_base, 512);
}

// CTA pairs that can be resident at once for the pair kernel (0 if unknown).
template <bool B_MN, int NB>
int batched_pair_slots() {
    static int n = -1;
    if (n < 0) {
        constexpr size_t smem = (size_t)bp_smem(NB) + 1024;
        n = 0;
        if (cudaFuncSetAttribute(batched_gemm_pair_kernel<B_MN, NB>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                 (int)smem) == cudaSuccess) {
            cudaLaunchConfig_t cfg = {};
            cfg.gridDim = dim3(2 * 74, 1, 1);
            cfg.blockDim = dim3(BP_THREADS, 1, 1);
            cfg.dynamicSmemBytes = smem;
            int clusters = 0;
            if (cudaOccupancyMaxActiveClusters(&clusters, batched_gemm_pair_kernel<B_MN, NB>, &cfg) == cudaSuccess)
                n = clusters;
        }
        cudaGetLastError();
    }
    return n;
}

}  // namespace

namespace zg {

int batched_error_word(int clear) { return ptx_error_word(clear); }

int batched_u_pass(const void* x, const void* F1T, int P, int M, int K, int rank, float s, void* U, cudaStream_t st,
                   bool x_batched) {
    if ((rank != 8 && rank != 16) || K % 8 || P < 1 || M < 1)
        return fail(ZG_ERR_INVALID, "batched_u_pass: rank 8 or 16 and K a multiple of 8");
    CUtensorMap tx, tf;
    const uint64_t dx[3] = {(uint64_t)K, (uint64_t)M, (uint64_t)(x_batched ? P : 1)};
    const uint64_t sx[2] = {(uint64_t)K * 2, (uint64_t)M * K * 2};
    const uint32_t bx[3] = {BK, BM, 1};
    const uint64_t df[2] = {(uint64_t)K, (uint64_t)P * rank};
    const uint64_t sf[1] = {(uint64_t)K * 2};
    const uint32_t bf[2] = {BK, 16};
    if (!tensor_map_bf16(&tx, x, 3, dx, sx, bx, true) || !tensor_map_bf16(&tf, F1T, 2, df, sf, bf, true))
        return fail(ZG_ERR_CUDA, "batched_u_pass: tensor maps");
    UPassArgs a{static_cast<__nv_bfloat16*>(U), M, K, P, rank, (M + BM - 1) / BM, s, x_batched ? 1 : 0};
    const int64_t tiles = (int64_t)P * a.tiles_m;
    if (tiles > INT_MAX) return fail(ZG_ERR_INVALID, "batched_u_pass: too many tiles");
    const int grid = tiles < sm_count_b() ? (int)tiles : sm_count_b();
    const size_t smem = UP_SMEM + 1024;
    if (cudaFuncSetAttribute(batched_u_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem) != cudaSuccess)
        return fail(ZG_ERR_CUDA, "batched_u_pass: shared memory attribute");
    zg::LaunchTimer zg_lt_("batched_u_pass", st);
    batched_u_kernel<<<grid, THREADS, smem, st>>>(tx, tf, a);
    return check_launch("batched_u_pass");
}

int batched_gemm(const void* x, const void* Wop, bool w_mn_major, const void* U, const void* F2, int P, int M, int K,
                 int N, int rank, void* y, cudaStream_t st, int64_t ld2, int act, const void* res) {
    if ((rank != 8 && rank != 16) || K % 8 || N % 8 || P < 1 || M < 1)
        return fail(ZG_ERR_INVALID, "batched_gemm: rank 8 or 16, K and N multiples of 8");
    if (act != ZG_ACT_NONE && act != ZG_ACT_GELU) return fail(ZG_ERR_INVALID, "batched_gemm: unknown activation");
    if (res && (reinterpret_cast<uintptr_t>(res) & 15)) return fail(ZG_ERR_INVALID, "batched_gemm: residual alignment");
    const uint64_t q = (uint64_t)P * rank;
    // F2's rows are ld2 elements apart (a column block of a larger population's buffer when ld2 > q)
    const uint64_t ldf = ld2 ? (uint64_t)ld2 : q;
    if (ldf < q || ldf % 8) return fail(ZG_ERR_INVALID, "batched_gemm: F2 row pitch");
    const __nv_bfloat16* resb = static_cast<const __nv_bfloat16*>(res);
    CUtensorMap tx, tw, tu, tf;
    const uint64_t dx[3] = {(uint64_t)K, (uint64_t)M, (uint64_t)P};
    const uint64_t sx[2] = {(uint64_t)K * 2, (uint64_t)M * K * 2};
    const uint32_t bx[3] = {BK, BM, 1};
    bool ok = tensor_map_bf16(&tx, x, 3, dx, sx, bx, true);
    if (w_mn_major) {  // Wop [K, N]
        const uint64_t dw[2] = {(uint64_t)N, (uint64_t)K};
        const uint64_t sw[1] = {(uint64_t)N * 2};
        const uint32_t bw[2] = {64, BK};
        ok = ok && tensor_map_bf16(&tw, Wop, 2, dw, sw, bw, true);
    } else {  // Wop [N, K]
        const uint64_t dw[2] = {(uint64_t)K, (uint64_t)N};
        const uint64_t sw[1] = {(uint64_t)K * 2};
        const uint32_t bw[2] = {BK, BG_BN};
        ok = ok && tensor_map_bf16(&tw, Wop, 2, dw, sw, bw, true);
    }
    const uint64_t du[3] = {16, (uint64_t)M, (uint64_t)P};
    const uint64_t su[2] = {32, (uint64_t)M * 32};
    const uint32_t bu[3] = {8, BM, 1};
    const uint64_t df[2] = {q, (uint64_t)N};
    const uint64_t sf[1] = {ldf * 2};
    const uint32_t bf[2] = {8, BG_BN};
    ok = ok && tensor_map_bf16(&tu, U, 3, du, su, bu, false) && tensor_map_bf16(&tf, F2, 2, df, sf, bf, false);
    if (!ok) return fail(ZG_ERR_CUDA, "batched_gemm: tensor maps");
    const bool one_box = resb == nullptr;  // no residual: single-buffered staging, six stages
    const int slots = w_mn_major ? (one_box ? batched_pair_slots<true, 1>() : batched_pair_slots<true, 2>())
                                 : (one_box ? batched_pair_slots<false, 1>() : batched_pair_slots<false, 2>());
    const int64_t pair_tiles = (int64_t)P * ((M + 255) / 256) * ((N + 255) / 256);
    if (slots > 0 && pair_tiles >= slots && pair_tiles <= INT_MAX) {
        // CTA pairs: each CTA loads 128 of the 256 x / U rows and 128 of the 256 Wop / F2 columns
        CUtensorMap tx2, tw2, tu2, tf2;
        const uint32_t bx2[3] = {BK, BM, 1};
        bool ok2 = tensor_map_bf16(&tx2, x, 3, dx, sx, bx2, true);
        if (w_mn_major) {
            const uint64_t dw[2] = {(uint64_t)N, (uint64_t)K};
            const uint64_t sw[1] = {(uint64_t)N * 2};
            const uint32_t bw[2] = {64, BK};
            ok2 = ok2 && tensor_map_bf16(&tw2, Wop, 2, dw, sw, bw, true);
        } else {
            const uint64_t dw[2] = {(uint64_t)K, (uint64_t)N};
            const uint64_t sw[1] = {(uint64_t)K * 2};
            const uint32_t bw[2] = {BK, 128};
            ok2 = ok2 && tensor_map_bf16(&tw2, Wop, 2, dw, sw, bw, true);
        }
        const uint32_t bu2[3] = {8, 128, 1};
        const uint32_t bf2[2] = {8, 128};
        ok2 = ok2 && tensor_map_bf16(&tu2, U, 3, du, su, bu2, false) && tensor_map_bf16(&tf2, F2, 2, df, sf, bf2, false);
        // output and residual [P, M, N] in 32 x 32 boxes, 64-byte swizzle (the epilogue's staging layout)
        CUtensorMap ty, tr;
        const uint64_t dy[3] = {(uint64_t)N, (uint64_t)M, (uint64_t)P};
        const uint64_t sy[2] = {(uint64_t)N * 2, (uint64_t)M * N * 2};
        const uint32_t by[3] = {32, 32, 1};
        ok2 = ok2 && (reinterpret_cast<uintptr_t>(y) & 15) == 0 && tensor_map_bf16_swz(&ty, y, 3, dy, sy, by, 64);
        ok2 = ok2 && tensor_map_bf16_swz(&tr, res ? res : y, 3, dy, sy, by, 64);
        if (!ok2) return fail(ZG_ERR_CUDA, "batched_gemm: tensor maps");
        GemmArgs a2{static_cast<__nv_bfloat16*>(y), M, N, K, P, rank, (M + 255) / 256, (N + 255) / 256, resb, act};
        const int pairs = pair_tiles < slots ? (int)pair_tiles : slots;
        const size_t smem2 = (size_t)bp_smem(one_box ? 1 : 2) + 1024;
        zg::LaunchTimer zg_lt_("batched_gemm", st);
        if (w_mn_major && one_box)
            batched_gemm_pair_kernel<true, 1><<<2 * pairs, BP_THREADS, smem2, st>>>(tx2, tw2, tu2, tf2, ty, tr, a2);
        else if (w_mn_major)
            batched_gemm_pair_kernel<true, 2><<<2 * pairs, BP_THREADS, smem2, st>>>(tx2, tw2, tu2, tf2, ty, tr, a2);
        else if (one_box)
            batched_gemm_pair_kernel<false, 1><<<2 * pairs, BP_THREADS, smem2, st>>>(tx2, tw2, tu2, tf2, ty, tr, a2);
        else
            batched_gemm_pair_kernel<false, 2><<<2 * pairs, BP_THREADS, smem2, st>>>(tx2, tw2, tu2, tf2, ty, tr, a2);
        return check_launch("batched_gemm");
    }
    GemmArgs a{static_cast<__nv_bfloat16*>(y), M, N, K, P, rank, (M + BM - 1) / BM, (N + BG_BN - 1) / BG_BN, resb, act};
    const int64_t tiles = (int64_t)P * a.tiles_m * a.tiles_n;
    if (tiles > INT_MAX) return fail(ZG_ERR_INVALID, "batched_gemm: too many tiles");
    const int grid = tiles < sm_count_b() ? (int)tiles : sm_count_b();
    const size_t smem = BG_SMEM + 1024;
    auto kern = w_mn_major ? batched_gemm_kernel<true> : batched_gemm_kernel<false>;
    if (cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem) != cudaSuccess)
        return fail(ZG_ERR_CUDA, "batched_gemm: shared memory attribute");
    zg::LaunchTimer zg_lt_("batched_gemm", st);
    kern<<<grid, THREADS, smem, st>>>(tx, tw, tu, tf, a);
    return check_launch("batched_gemm");
}

}  // namespace zg
