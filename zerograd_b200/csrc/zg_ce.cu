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
// and keeps its running max, sum of exponentials and label logit in registers.
// U_p = bf16(s x_p . B_p) comes from the u pass of the per-candidate-input
// forward (table B kept K-major as F1T); F2 = the table A in operand layout.
// A label outside [0, V) yields a NaN loss.
#include <climits>
#include <math.h>

#include "zg_ptx.cuh"
#include "zg_tc.cuh"

namespace {

constexpr int THREADS = 192, BK = 64;
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
    const int k_blocks = (a.C + BK - 1) / BK;

    if (threadIdx.x == 0) {
        for (int s = 0; s < CE_STAGES; ++s) {
            mbar_init(&full_bar[s], 1);
            mbar_init(&empty_bar[s], 1);
        }
        for (int b = 0; b < 2; ++b) {
            mbar_init(&tmem_full[b], 1);
            mbar_init(&tmem_empty[b], 8);  // 4 epilogue warps in each CTA
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
        for (int u = pair; ok && u < units; u += pairs) {
            const int p = u / a.tiles_m, tm = u % a.tiles_m;
            const int zx = a.x_batched ? p : 0;
            for (int tn = 0; ok && tn < a.tiles_n; ++tn) {
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
                const int k_start = (u * a.tiles_n + tn) % k_blocks;
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
        for (int u = pair; ok && u < units; u += pairs) {
            for (int tn = 0; ok && tn < a.tiles_n; ++tn) {
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
        // Thread = one row of this CTA's 128; per 32-column chunk: the chunk's
        // max and sum of exponentials, merged into the row's running pair.
        const int quad = warp % 4;
        const uint32_t empty_leader = cluster_addr(&tmem_empty[0], 0);
        int acc = 0;
        uint32_t acc_phase = 0;
        bool ok = true;
        for (int u = pair; u < units; u += pairs) {
            const int p = u / a.tiles_m, tm = u % a.tiles_m;
            const int row = tm * 256 + (int)rank * 128 + quad * 32 + lane;
            // a label outside [0, V) never matches a column: its loss is NaN
            int label = row < a.M ? a.labels[row] : -1;
            if (label >= a.V) label = -1;
            float run_max = -INFINITY, run_sum = 0.f, label_logit = 0.f;
            bool found = false;
            for (int tn = 0; tn < a.tiles_n; ++tn) {
                ok = ok && mbar_wait(&tmem_full[acc], acc_phase, 76);
                if (ok) {
                    tc_fence_after();
#pragma unroll 1
                    for (int c0 = 0; c0 < 256; c0 += 32) {
                        float v[32];
                        tmem_ld32(tmem_base + ((uint32_t)(quad * 32) << 16) + acc * 256 + c0, v);
                        const int col0 = tn * 256 + c0;
                        float cmax = -INFINITY;
#pragma unroll
                        for (int i = 0; i < 32; ++i) {
                            // the logit tied_logits would return: float32 accumulator rounded to bf16
                            v[i] = col0 + i < a.V ? __bfloat162float(__float2bfloat16_rn(v[i])) : -INFINITY;
                            cmax = fmaxf(cmax, v[i]);
                            if (col0 + i == label) {
                                label_logit = v[i];
                                found = true;
                            }
                        }
                        if (cmax == -INFINITY) continue;  // every column past V
                        float csum = 0.f;
#pragma unroll
                        for (int i = 0; i < 32; ++i) csum += expf(v[i] - cmax);
                        const float m = fmaxf(run_max, cmax);
                        run_sum = run_sum * expf(run_max - m) + csum * expf(cmax - m);
                        run_max = m;
                    }
                }
                tc_fence_before();
                __syncwarp();
                if (lane == 0 && ok) mbar_arrive_remote(empty_leader + acc * (uint32_t)sizeof(uint64_t));
                if (++acc == 2) { acc = 0; acc_phase ^= 1; }
            }
            if (ok && row < a.M)
                a.loss[(int64_t)p * a.M + row] = found ? run_max + logf(run_sum) - label_logit : __int_as_float(0x7fc00000);
        }
    }
    tc_fence_before();
    cluster_sync();
    tc_fence_after();
    if (warp == 1) tmem_dealloc_pair(tmem_base, 512);
}

}  // namespace

namespace zg {

bool tied_ce_ok(int P, int M, int V, int C, int rank) {
    return tc_available() && (rank == 8 || rank == 16) && P > 0 && M > 0 && V > 0 && C % 8 == 0 && C > 0 &&
           (int64_t)P * ((M + 255) / 256) <= INT_MAX;
}

size_t tied_ce_workspace(int P, int M, int V, int C, int rank) {
    const size_t q = (size_t)P * rank;
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

int tied_ce(const void* x, int x_batched, const void* T, const uint32_t* keys, int group, const int32_t* labels,
            int P, int M, int V, int C, int rank, float s, float* loss, Carver& cv, cudaStream_t st) {
    const int64_t q = (int64_t)P * rank;
    __nv_bfloat16* U = cv.take<__nv_bfloat16>((size_t)P * M * 16);
    __nv_bfloat16* F1T = cv.take<__nv_bfloat16>((size_t)q * C);
    __nv_bfloat16* F2 = cv.take<__nv_bfloat16>((size_t)V * q);
    if (!U || !F1T || !F2) return fail(ZG_ERR_WORKSPACE, "tied_ce: workspace too small");
    auto al = [](const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15) == 0; };
    if (!al(x) || !al(T)) return fail(ZG_ERR_INVALID, "tied_ce: x and T must be 16-byte aligned");
    // table factors: F2 = A_op [V, q] (counter v*r + j), F1T = B^T [q, C] (counter c*r + j)
    int rc = fill_operand(keys, group, P, rank, V, 0, 0, nullptr, 1.f, ZG_BF16, F2, st, "factor_fill");
    if (!rc) rc = fill_operand_t(keys, group, P, rank, C, 1, F1T, st, "factor_fill");
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
    const uint64_t sf[1] = {(uint64_t)q * 2};
    const uint32_t bf[2] = {8, 128};
    if (!tensor_map_bf16(&tx, x, 3, dx, sx, bx, true) || !tensor_map_bf16(&tt, T, 2, dt, stt, bt, true) ||
        !tensor_map_bf16(&tu, U, 3, du, su, bu, false) || !tensor_map_bf16(&tf, F2, 2, df, sf, bf, false))
        return fail(ZG_ERR_CUDA, "tied_ce: tensor maps");
    CeArgs a{loss, labels, M, V, C, P, rank, (M + 255) / 256, (V + 255) / 256, x_batched != 0};
    const int64_t units = (int64_t)P * a.tiles_m;
    const int pairs = units < slots ? (int)units : slots;
    const size_t smem = (size_t)CE_SMEM + 1024;
    zg::LaunchTimer zg_lt_("tied_ce", st);
    tied_ce_pair_kernel<<<2 * pairs, THREADS, smem, st>>>(tx, tt, tu, tf, a);
    return check_launch("tied_ce");
}

int ce_error_word(int clear) { return ptx_error_word(clear); }

}  // namespace zg

extern "C" size_t zg_tied_logits_ce_workspace_size(int P, int M, int V, int C, int rank) {
    if (P < 1 || M < 1 || V < 1 || C < 1 || rank < 1) return 0;
    return zg::tied_ce_workspace(P, M, V, C, rank);
}

extern "C" int zg_tied_logits_ce(const void* x, int x_batched, const void* T, const uint32_t* keys, int group,
                                 const int32_t* labels, int P, int M, int V, int C, int rank, float s, float* loss,
                                 void* workspace, size_t workspace_bytes, void* stream) {
    if (P < 1 || P > 65535 || M < 1 || V < 1 || C < 1 || rank < 1)
        return zg::fail(ZG_ERR_INVALID, "zg_tied_logits_ce: bad sizes");
    if (!x || !T || !keys || !labels || !loss) return zg::fail(ZG_ERR_INVALID, "zg_tied_logits_ce: null pointer");
    if (!zg::tied_ce_ok(P, M, V, C, rank))
        return zg::fail(ZG_ERR_UNSUPPORTED, "zg_tied_logits_ce: needs sm_100, rank 8 or 16, C a multiple of 8");
    const size_t need = zg::tied_ce_workspace(P, M, V, C, rank);
    if (!workspace || workspace_bytes < need)
        return zg::fail(ZG_ERR_WORKSPACE, "zg_tied_logits_ce: workspace %zu < %zu bytes", workspace_bytes, need);
    zg::Carver cv(workspace, workspace_bytes);
    return zg::tied_ce(x, x_batched, T, keys, group, labels, P, M, V, C, rank, s, loss, cv, zg::as_stream(stream));
}
