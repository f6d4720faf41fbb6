// zg_ce.cu -- tied logits fused with softmax cross-entropy, population-batched
// on the tcgen05 tensor cores (CTA pairs, cta_group::2).
//
//   logits_p[m, v] = bf16(x_p[m, :] . T[v, :] + U_p[m, :] . F2[v, p r : p r + 16])
//   loss[p, m]     = logsumexp_v logits_p[m, v] - logits_p[m, label[m]]   (float32)
//
// which is perturbed_tied_logits (src/zerograd/_candidate.py:33-38) followed
// by a float32 cross-entropy over the bf16 logits, without ever writing the
// [P, M, V] logits: a CTA pair owns one (candidate, 256-row block) and sweeps
// every 256-column block of the vocabulary; each epilogue thread owns one row
// and keeps its running max, sum of exponentials and label logit in registers
// (two epilogue warps per TMEM lane quadrant, each over half of every column
// block; the two halves of a row merge through shared memory at the end).
// U_p = bf16(s x_p . B_p) comes from the u pass of the per-candidate-input
// forward (table B kept K-major as F1T); F2 = the table A in operand layout.
// A label outside [0, V) yields a NaN loss.
#include <climits>
#include <math.h>

#include "zg_ptx.cuh"
#include "zg_tc.cuh"

namespace {

constexpr int THREADS = 320, BK = 64;  // warp 0 TMA, warp 1 MMA, warps 2..9 epilogue
constexpr int CE_STAGES = 6;
constexpr uint32_t CE_A = 128 * BK * 2;                            // 16 KiB: this CTA's 128 rows of x
constexpr uint32_t CE_B = 128 * BK * 2;                            // 16 KiB: this CTA's 128 rows of T
constexpr uint32_t CE_STAGE = CE_A + CE_B;                         // 32 KiB
constexpr uint32_t CE_CU = 128 * 16;                               // 8 K columns of 128 U rows
constexpr uint32_t CE_CF = 128 * 16;                               // 8 K columns of 128 F2 rows
constexpr uint32_t CE_CORR = 2 * CE_CU + 2 * CE_CF;                // 8 KiB per accumulator
constexpr uint32_t CE_SMEM = CE_STAGES * CE_STAGE + 2 * CE_CORR;   // 208 KiB

struct CeArgs {
    float* loss;            // [P, M]
    const int32_t* labels;  // [M]
    int M, V, C, P, rank, tiles_m, tiles_n, x_batched;
};

// Schedule of the (unit, 256-column block) tiles over G CTA pairs: whole
// units in rounds, unit k G + g to pair g, so all pairs sweep the vocabulary
// together and each table tile is fetched from DRAM about once per round.
// A unit's columns are always swept in order by one pair, so a candidate's
// loss does not depend on the population size or its place in it.
struct CeSched {
    int g, G, tiles_n, n_units;
    __device__ CeSched(int g_, int G_, int units, int tiles_n_) : g(g_), G(G_), tiles_n(tiles_n_) {
        n_units = units > g ? (units - g + G - 1) / G : 0;
    }
    __device__ int64_t count() const { return (int64_t)n_units * tiles_n; }
    __device__ void at(int64_t j, int& u, int& tn) const {
        u = (int)(j / tiles_n) * G + g;
        tn = (int)(j % tiles_n);
    }
};

// Flags of a row half's record (merged with the other half at a unit's end).
constexpr int kFound = 1, kOk = 2;

constexpr float kLog2e = 1.4426950408889634f;

// 2^x by the hardware approximation (exp(y) is evaluated as 2^(y log2 e)).
__device__ __forceinline__ float ex2_approx(float x) {
    float y;
    asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
    return y;
}

// 32 lanes x 64 columns of float32 accumulators, loaded and waited for in one
// statement so no use of the registers can be scheduled before the wait.
__device__ __forceinline__ void tmem_ld64(uint32_t taddr, float (&v)[64]) {
    uint32_t r[64];
    __syncwarp();
    asm volatile(
        "tcgen05.ld.sync.aligned.32x32b.x64.b32 "
        "{%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,"
        "%16,%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31,"
        "%32,%33,%34,%35,%36,%37,%38,%39,%40,%41,%42,%43,%44,%45,%46,%47,"
        "%48,%49,%50,%51,%52,%53,%54,%55,%56,%57,%58,%59,%60,%61,%62,%63}, [%64];\n\t"
        "tcgen05.wait::ld.sync.aligned;"
        : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
          "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15]),
          "=r"(r[16]), "=r"(r[17]), "=r"(r[18]), "=r"(r[19]), "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]),
          "=r"(r[24]), "=r"(r[25]), "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]), "=r"(r[30]), "=r"(r[31]),
          "=r"(r[32]), "=r"(r[33]), "=r"(r[34]), "=r"(r[35]), "=r"(r[36]), "=r"(r[37]), "=r"(r[38]), "=r"(r[39]),
          "=r"(r[40]), "=r"(r[41]), "=r"(r[42]), "=r"(r[43]), "=r"(r[44]), "=r"(r[45]), "=r"(r[46]), "=r"(r[47]),
          "=r"(r[48]), "=r"(r[49]), "=r"(r[50]), "=r"(r[51]), "=r"(r[52]), "=r"(r[53]), "=r"(r[54]), "=r"(r[55]),
          "=r"(r[56]), "=r"(r[57]), "=r"(r[58]), "=r"(r[59]), "=r"(r[60]), "=r"(r[61]), "=r"(r[62]), "=r"(r[63])
        : "r"(taddr)
        : "memory");
#pragma unroll
    for (int i = 0; i < 64; ++i) v[i] = __uint_as_float(r[i]);
}

// Rounds 64 float32 logits to bf16 in place (round to nearest even, as the
// tied-logits output does) and returns their maximum.
__device__ __forceinline__ float round_bf16_max64(float (&v)[64]) {
    __nv_bfloat162 m[8];
#pragma unroll
    for (int i = 0; i < 32; ++i) {
        const __nv_bfloat162 b = __floats2bfloat162_rn(v[2 * i], v[2 * i + 1]);
        m[i % 8] = i < 8 ? b : __hmax2(m[i % 8], b);
        const uint32_t u = *reinterpret_cast<const uint32_t*>(&b);
        v[2 * i] = __uint_as_float(u << 16);
        v[2 * i + 1] = __uint_as_float(u & 0xffff0000u);
    }
    m[0] = __hmax2(__hmax2(m[0], m[1]), __hmax2(m[2], m[3]));
    m[4] = __hmax2(__hmax2(m[4], m[5]), __hmax2(m[6], m[7]));
    m[0] = __hmax2(m[0], m[4]);
    return fmaxf(__low2float(m[0]), __high2float(m[0]));
}

// sum_i exp(v[i] - vmax) with four independent partial sums.
__device__ __forceinline__ float sum_exp64(const float (&v)[64], float vmax) {
    const float t = vmax * kLog2e;
    float s[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll
    for (int i = 0; i < 64; ++i) s[i % 4] += ex2_approx(fmaf(v[i], kLog2e, -t));
    return (s[0] + s[1]) + (s[2] + s[3]);
}

__device__ __forceinline__ void epi_bar() { asm volatile("bar.sync 1, 256;" ::: "memory"); }

__global__ void __cluster_dims__(2, 1, 1) __launch_bounds__(THREADS, 1)
tied_ce_pair_kernel(const __grid_constant__ CUtensorMap tmX, const __grid_constant__ CUtensorMap tmT,
                    const __grid_constant__ CUtensorMap tmU, const __grid_constant__ CUtensorMap tmF,
                    const CeArgs a) {
    extern __shared__ uint8_t dyn_smem[];
    __shared__ __align__(8) uint64_t full_bar[CE_STAGES], empty_bar[CE_STAGES], tmem_full[2], tmem_empty[2],
        corr_full[2], corr_empty[2], mma_done;
    __shared__ uint32_t tmem_base_sh;
    const uint32_t dyn_base = smem_u32(dyn_smem);
    uint8_t* smem = dyn_smem + (((dyn_base + 1023u) & ~1023u) - dyn_base);
    uint8_t* corr = smem + CE_STAGES * CE_STAGE;
    const int warp = threadIdx.x / 32, lane = threadIdx.x % 32;
    const uint32_t rank = cluster_rank();
    const int pair = blockIdx.x / 2, pairs = gridDim.x / 2;
    const int units = a.P * a.tiles_m;  // (candidate, 256-row block)
    const CeSched sch(pair, pairs, units, a.tiles_n);
    const int64_t n_mine = sch.count();
    const int k_blocks = (a.C + BK - 1) / BK;

    if (threadIdx.x == 0) {
        for (int s = 0; s < CE_STAGES; ++s) {
            mbar_init(&full_bar[s], 1);
            mbar_init(&empty_bar[s], 1);
        }
        for (int b = 0; b < 2; ++b) {
            mbar_init(&tmem_full[b], 1);
            mbar_init(&tmem_empty[b], 16);  // 8 epilogue warps in each CTA
            mbar_init(&corr_full[b], 1);
            mbar_init(&corr_empty[b], 1);
        }
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
        for (int64_t j = 0; ok && j < n_mine; ++j) {
            int u, tn;
            sch.at(j, u, tn);
            const int p = u / a.tiles_m, tm = u % a.tiles_m;
            const int zx = a.x_batched ? p : 0;
            {
                if (!mbar_wait(&corr_empty[acc], acc_phase ^ 1, 71)) { ok = false; break; }
                uint8_t* c = corr + acc * CE_CORR;
                if (rank == 0) mbar_expect_tx(&corr_full[acc], 2 * CE_CORR);
                const uint32_t cb = cluster_addr(&corr_full[acc], 0);
                tma_load_3d_pair(c, &tmU, cb, 0, tm * 256 + half, p);
                tma_load_3d_pair(c + CE_CU, &tmU, cb, 8, tm * 256 + half, p);
                tma_load_2d_pair(c + 2 * CE_CU, &tmF, cb, p * a.rank, tn * 256 + half);
                tma_load_2d_pair(c + 2 * CE_CU + CE_CF, &tmF, cb, p * a.rank + 8, tn * 256 + half);
                c_issued |= 1u << acc;
                c_parity = (c_parity & ~(1u << acc)) | (acc_phase << acc);
                if (++acc == 2) { acc = 0; acc_phase ^= 1; }
                const int k_start = (int)(((int64_t)tm * a.tiles_n + tn) % k_blocks);
                for (int kb = 0; kb < k_blocks; ++kb) {
                    if (!mbar_wait(&empty_bar[stage], phase ^ 1, 72)) { ok = false; break; }
                    const int kk = kb + k_start < k_blocks ? kb + k_start : kb + k_start - k_blocks;
                    uint8_t* sa = smem + stage * CE_STAGE;
                    if (rank == 0) mbar_expect_tx(&full_bar[stage], 2 * CE_STAGE);
                    const uint32_t fb = cluster_addr(&full_bar[stage], 0);
                    tma_load_3d_pair(sa, &tmX, fb, kk * BK, tm * 256 + half, zx);
                    tma_load_2d_pair(sa + CE_A, &tmT, fb, kk * BK, tn * 256 + half);
                    issued |= 1u << stage;
                    issue_parity = (issue_parity & ~(1u << stage)) | (phase << stage);
                    if (++stage == CE_STAGES) { stage = 0; phase ^= 1; }
                }
            }
        }
        // Drain: the leader sees the bytes land on its full barriers; the peer
        // sees its buffers released by the MMAs that consumed them.
        for (int s = 0; s < CE_STAGES; ++s)
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
        constexpr uint32_t IDESC = idesc_bf16(256, 256, 0);
        int stage = 0, acc = 0;
        uint32_t phase = 0, acc_phase = 0;
        bool ok = true;
        for (int64_t j = 0; ok && j < n_mine; ++j) {
            {
                if (!mbar_wait(&tmem_empty[acc], acc_phase ^ 1, 73)) { ok = false; break; }
                tc_fence_after();
                const uint32_t d_tmem = tmem_base + acc * 256;
                for (int kb = 0; kb < k_blocks; ++kb) {
                    if (!mbar_wait(&full_bar[stage], phase, 74)) { ok = false; break; }
                    tc_fence_after();
                    const uint32_t a_addr = smem_u32(smem + stage * CE_STAGE);
                    const uint32_t b_addr = a_addr + CE_A;
#pragma unroll
                    for (int k = 0; k < BK / 16; ++k)
                        umma_bf16_pair(d_tmem, smem_desc(a_addr + k * 32, 16, 1024), smem_desc(b_addr + k * 32, 16, 1024),
                                       IDESC, (kb > 0 || k > 0) ? 1u : 0u);
                    umma_commit_pair(smem_u32(&empty_bar[stage]));
                    umma_commit_pair(cluster_addr(&empty_bar[stage], 1));
                    if (++stage == CE_STAGES) { stage = 0; phase ^= 1; }
                }
                if (!ok) break;
                // low-rank term: U tile [256, 16] . F2 tile [256, 16]^T into the same accumulator
                if (!mbar_wait(&corr_full[acc], acc_phase, 75)) { ok = false; break; }
                tc_fence_after();
                const uint32_t c_addr = smem_u32(corr + acc * CE_CORR);
                umma_bf16_pair(d_tmem, smem_desc_noswizzle(c_addr, CE_CU, 128),
                               smem_desc_noswizzle(c_addr + 2 * CE_CU, CE_CF, 128), IDESC, 1u);
                umma_commit_pair(smem_u32(&corr_empty[acc]));
                umma_commit_pair(cluster_addr(&corr_empty[acc], 1));
                umma_commit_pair(smem_u32(&tmem_full[acc]));
                umma_commit_pair(cluster_addr(&tmem_full[acc], 1));
                if (++acc == 2) { acc = 0; acc_phase ^= 1; }
            }
        }
        umma_commit_pair(smem_u32(&mma_done));
        for (uint32_t i = 0; i < kSpinLimit; ++i)
            if (mbar_try_wait(&mma_done, 0)) break;
    } else if (warp >= 2) {
        // ---------------- epilogue: online log-sum-exp over the vocabulary ----------------
        // Thread = one row of this CTA's 128 and one half (128 columns) of
        // every 256-column block; per 64-column chunk: the chunk's max and sum
        // of exponentials, merged into the running pair of the row half.  At
        // the last tile of a unit the halves merge and the row's loss is written.
        __shared__ float s_half[2][4][128];  // second halves' (max, sum, label logit, flags), by parity
        const int quad = warp % 4, half = (warp - 2) / 4, r = quad * 32 + lane;
        const uint32_t empty_leader = cluster_addr(&tmem_empty[0], 0);
        const uint32_t t_row = tmem_base + ((uint32_t)(quad * 32) << 16) + half * 128;
        int acc = 0, parity = 0, label = -1, row = 0;
        uint32_t acc_phase = 0;
        bool ok = true, found = false;
        float run_max = -INFINITY, run_sum = 0.f, label_logit = 0.f;
        for (int64_t j = 0; j < n_mine; ++j) {
            int u, tn;
            sch.at(j, u, tn);
            if (tn == 0) {
                row = (u % a.tiles_m) * 256 + (int)rank * 128 + r;
                // a label outside [0, V) never matches a column: its loss is NaN
                label = row < a.M ? a.labels[row] : -1;
                if (label >= a.V) label = -1;
                run_max = -INFINITY;
                run_sum = 0.f;
                label_logit = 0.f;
                found = false;
            }
            ok = __all_sync(0xffffffffu, ok && mbar_wait(&tmem_full[acc], acc_phase, 76));
            if (ok) {
                tc_fence_after();
#pragma unroll 1
                for (int c0 = 0; c0 < 128; c0 += 64) {
                    const int col0 = tn * 256 + half * 128 + c0;
                    if (col0 >= a.V) break;  // the rest of this block is past the vocabulary
                    float v[64];
                    tmem_ld64(t_row + acc * 256 + c0, v);
                    float cmax = round_bf16_max64(v);  // v now holds the bf16 logits
                    if (col0 + 64 > a.V) {
                        cmax = -INFINITY;
#pragma unroll
                        for (int i = 0; i < 64; ++i) {
                            if (col0 + i >= a.V) v[i] = -INFINITY;
                            cmax = fmaxf(cmax, v[i]);
                        }
                    }
                    const unsigned li = (unsigned)(label - col0);
                    if (__any_sync(0xffffffffu, li < 64u)) {
#pragma unroll
                        for (int i = 0; i < 64; ++i)
                            if (li == (unsigned)i) {
                                label_logit = v[i];
                                found = true;
                            }
                    }
                    const float csum = sum_exp64(v, cmax);
                    const float m = fmaxf(run_max, cmax);
                    run_sum = run_sum * ex2_approx((run_max - m) * kLog2e) + csum * ex2_approx((cmax - m) * kLog2e);
                    run_max = m;
                }
            }
            tc_fence_before();
            __syncwarp();
            if (lane == 0 && ok) mbar_arrive_remote(empty_leader + acc * (uint32_t)sizeof(uint64_t));
            if (++acc == 2) { acc = 0; acc_phase ^= 1; }
            if (tn == a.tiles_n - 1) {
                if (half == 1) {
                    s_half[parity][0][r] = run_max;
                    s_half[parity][1][r] = run_sum;
                    s_half[parity][2][r] = label_logit;
                    s_half[parity][3][r] = (float)((found ? kFound : 0) | (ok ? kOk : 0));
                }
                epi_bar();
                if (half == 0) {
                    const float m1 = s_half[parity][0][r], s1 = s_half[parity][1][r];
                    const int f1 = (int)s_half[parity][3][r];
                    const int flags = ((found || (f1 & kFound)) ? kFound : 0) | ((ok && (f1 & kOk)) ? kOk : 0);
                    const float m = fmaxf(run_max, m1);
                    const float sum =
                        run_sum * ex2_approx((run_max - m) * kLog2e) + s1 * ex2_approx((m1 - m) * kLog2e);
                    const float lab = found ? label_logit : s_half[parity][2][r];
                    if ((flags & kOk) && row < a.M)
                        a.loss[(int64_t)(u / a.tiles_m) * a.M + row] =
                            (flags & kFound) ? m + logf(sum) - lab : __int_as_float(0x7fc00000);
                }
                parity ^= 1;
            }
        }
    }
    tc_fence_before();
    cluster_sync();
    tc_fence_after();
    if (warp == 1) tmem_dealloc_pair(tmem_base, 512);
}

constexpr int kMaxPairs = 256;  // bound on the pairs of one launch

}  // namespace

namespace zg {

bool tied_ce_ok(int P, int M, int V, int C, int rank) {
    return tc_available() && (rank == 8 || rank == 16) && P > 0 && M > 0 && V > 0 && C % 8 == 0 && C > 0 &&
           (int64_t)P * ((M + 255) / 256) <= INT_MAX;
}

size_t tied_ce_workspace(int P, int M, int V, int C, int rank, bool factors) {
    const size_t q = (size_t)P * rank;
    if (!factors) return Carver::need({(size_t)P * M * 16 * 2}) + 256;
    return Carver::need({(size_t)P * M * 16 * 2, q * C * 2, (size_t)V * q * 2}) + 256;
}

// CTA pairs that can be resident at once (0 if unknown).
static int tied_ce_slots() {
    static int n = -1;
    if (n < 0) {
        const size_t smem = (size_t)CE_SMEM + 1024;
        n = 0;
        if (cudaFuncSetAttribute(tied_ce_pair_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem) ==
            cudaSuccess) {
            cudaLaunchConfig_t cfg = {};
            cfg.gridDim = dim3(2 * 74, 1, 1);
            cfg.blockDim = dim3(THREADS, 1, 1);
            cfg.dynamicSmemBytes = smem;
            int clusters = 0;
            if (cudaOccupancyMaxActiveClusters(&clusters, tied_ce_pair_kernel, &cfg) == cudaSuccess) n = clusters;
        }
        cudaGetLastError();
    }
    return n;
}

// F1T / F2: the caller's table factors (B^T [P r, C], A_op [V, rows ld2
// apart]) drawn first when `draw`; null: drawn into the workspace.
int tied_ce(const void* x, int x_batched, const void* T, const uint32_t* keys, int group, const int32_t* labels,
            int P, int M, int V, int C, int rank, float s, float* loss, Carver& cv, cudaStream_t st, void* F1T_in,
            void* F2_in, int64_t ld2, bool draw) {
    const int64_t q = (int64_t)P * rank;
    __nv_bfloat16* U = cv.take<__nv_bfloat16>((size_t)P * M * 16);
    __nv_bfloat16* F1T = static_cast<__nv_bfloat16*>(F1T_in);
    __nv_bfloat16* F2 = static_cast<__nv_bfloat16*>(F2_in);
    if (!F1T || !F2) {
        F1T = cv.take<__nv_bfloat16>((size_t)q * C);
        F2 = cv.take<__nv_bfloat16>((size_t)V * q);
        ld2 = 0;
        draw = true;
    }
    const uint64_t ldf = ld2 ? (uint64_t)ld2 : (uint64_t)q;
    if (!U || !F1T || !F2) return fail(ZG_ERR_WORKSPACE, "tied_ce: workspace too small");
    auto al = [](const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15) == 0; };
    if (!al(x) || !al(T) || !al(F1T) || !al(F2))
        return fail(ZG_ERR_INVALID, "tied_ce: x, T and the factors must be 16-byte aligned");
    if (ldf < (uint64_t)q || ldf % 8) return fail(ZG_ERR_INVALID, "tied_ce: factor row pitch");
    // table factors: F2 = A_op [V, q] (counter v*r + j), F1T = B^T [q, C] (counter c*r + j)
    int rc = ZG_OK;
    if (draw) {
        rc = fill_operand(keys, group, P, rank, V, 0, 0, nullptr, 1.f, ZG_BF16, F2, st, "factor_fill", (int64_t)ldf);
        if (!rc) rc = fill_operand_t(keys, group, P, rank, C, 1, F1T, st, "factor_fill");
    }
    if (!rc) rc = batched_u_pass(x, F1T, P, M, C, rank, s, U, st, x_batched != 0);
    if (rc) return rc;
    const int slots = tied_ce_slots();
    if (slots <= 0) return fail(ZG_ERR_UNSUPPORTED, "tied_ce: CTA pairs unavailable");
    CUtensorMap tx, tt, tu, tf;
    const uint64_t dx[3] = {(uint64_t)C, (uint64_t)M, (uint64_t)(x_batched ? P : 1)};
    const uint64_t sx[2] = {(uint64_t)C * 2, (uint64_t)M * C * 2};
    const uint32_t bx[3] = {BK, 128, 1};
    const uint64_t dt[2] = {(uint64_t)C, (uint64_t)V};
    const uint64_t stt[1] = {(uint64_t)C * 2};
    const uint32_t bt[2] = {BK, 128};
    const uint64_t du[3] = {16, (uint64_t)M, (uint64_t)P};
    const uint64_t su[2] = {32, (uint64_t)M * 32};
    const uint32_t bu[3] = {8, 128, 1};
    const uint64_t df[2] = {(uint64_t)q, (uint64_t)V};
    const uint64_t sf[1] = {ldf * 2};
    const uint32_t bf[2] = {8, 128};
    if (!tensor_map_bf16(&tx, x, 3, dx, sx, bx, true) || !tensor_map_bf16(&tt, T, 2, dt, stt, bt, true) ||
        !tensor_map_bf16(&tu, U, 3, du, su, bu, false) || !tensor_map_bf16(&tf, F2, 2, df, sf, bf, false))
        return fail(ZG_ERR_CUDA, "tied_ce: tensor maps");
    CeArgs a{loss, labels, M, V, C, P, rank, (M + 255) / 256, (V + 255) / 256, x_batched != 0};
    const int units = P * a.tiles_m;
    int pairs = slots < kMaxPairs ? slots : kMaxPairs;
    if (units < pairs) pairs = units;
    const size_t smem = (size_t)CE_SMEM + 1024;
    zg::LaunchTimer zg_lt_("tied_ce", st);
    tied_ce_pair_kernel<<<2 * pairs, THREADS, smem, st>>>(tx, tt, tu, tf, a);
    return check_launch("tied_ce");
}

int ce_error_word(int clear) { return ptx_error_word(clear); }

}  // namespace zg

extern "C" size_t zg_tied_logits_ce_workspace_size(int P, int M, int V, int C, int rank) {
    if (P < 1 || M < 1 || V < 1 || C < 1 || rank < 1) return 0;
    return zg::tied_ce_workspace(P, M, V, C, rank, true);
}

extern "C" size_t zg_tied_logits_ce_ex_workspace_size(int P, int M, int V, int C, int rank) {
    if (P < 1 || M < 1 || V < 1 || C < 1 || rank < 1) return 0;
    return zg::tied_ce_workspace(P, M, V, C, rank, false);
}

extern "C" int zg_tied_logits_ce_ex(const void* x, int x_batched, const void* T, const uint32_t* keys, int group,
                                    const int32_t* labels, int P, int M, int V, int C, int rank, float s, void* F1T,
                                    void* F2, int64_t ld2, int draw, float* loss, void* workspace,
                                    size_t workspace_bytes, void* stream) {
    if (P < 1 || P > 65535 || M < 1 || V < 1 || C < 1 || rank < 1)
        return zg::fail(ZG_ERR_INVALID, "zg_tied_logits_ce_ex: bad sizes");
    if (!x || !T || !labels || !loss || !F1T || !F2 || (draw && !keys))
        return zg::fail(ZG_ERR_INVALID, "zg_tied_logits_ce_ex: null pointer");
    if (!zg::tied_ce_ok(P, M, V, C, rank))
        return zg::fail(ZG_ERR_UNSUPPORTED, "zg_tied_logits_ce_ex: needs sm_100, rank 8 or 16, C a multiple of 8");
    const int64_t q = (int64_t)P * rank;
    if (ld2 != 0 && (ld2 < q || ld2 % 8))
        return zg::fail(ZG_ERR_INVALID, "zg_tied_logits_ce_ex: ld2 must be 0 or a multiple of 8 >= P*rank");
    const size_t need = zg::tied_ce_workspace(P, M, V, C, rank, false);
    if (!workspace || workspace_bytes < need)
        return zg::fail(ZG_ERR_WORKSPACE, "zg_tied_logits_ce_ex: workspace %zu < %zu bytes", workspace_bytes, need);
    zg::Carver cv(workspace, workspace_bytes);
    return zg::tied_ce(x, x_batched, T, keys, group, labels, P, M, V, C, rank, s, loss, cv, zg::as_stream(stream), F1T,
                       F2, ld2, draw != 0);
}

extern "C" int zg_tied_logits_ce(const void* x, int x_batched, const void* T, const uint32_t* keys, int group,
                                 const int32_t* labels, int P, int M, int V, int C, int rank, float s, float* loss,
                                 void* workspace, size_t workspace_bytes, void* stream) {
    if (P < 1 || P > 65535 || M < 1 || V < 1 || C < 1 || rank < 1)
        return zg::fail(ZG_ERR_INVALID, "zg_tied_logits_ce: bad sizes");
    if (!x || !T || !keys || !labels || !loss) return zg::fail(ZG_ERR_INVALID, "zg_tied_logits_ce: null pointer");
    if (!zg::tied_ce_ok(P, M, V, C, rank))
        return zg::fail(ZG_ERR_UNSUPPORTED, "zg_tied_logits_ce: needs sm_100, rank 8 or 16, C a multiple of 8");
    const size_t need = zg::tied_ce_workspace(P, M, V, C, rank, true);
    if (!workspace || workspace_bytes < need)
        return zg::fail(ZG_ERR_WORKSPACE, "zg_tied_logits_ce: workspace %zu < %zu bytes", workspace_bytes, need);
    zg::Carver cv(workspace, workspace_bytes);
    return zg::tied_ce(x, x_batched, T, keys, group, labels, P, M, V, C, rank, s, loss, cv, zg::as_stream(stream),
                       nullptr, nullptr, 0, true);
}
