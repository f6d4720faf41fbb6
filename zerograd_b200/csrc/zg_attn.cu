// zg_attn.cu -- softmax attention of every candidate's transformer block,
// population-batched: for every z (candidate x batch row), head h and query i
//
//   o[z, i, h] = sum_j softmax_j(q[z, i, h] . k[z, j, h] / sqrt(D)) v[z, j, h]
//
// (examples/train_vit_cifar10.py:166-172; causal for the decoder LM: keys
// j > i masked).  q, k, v, o are [Z, S, H, D], the head-interleaved layout
// the q/k/v projections produce, so no transpose is materialised.
//
// Tensor-core path (bf16, D = 64, S <= 256): a persistent kernel over the
// (z, head) units.  TMA brings a unit's query tiles and its whole key and
// value sequence (4-D tensor maps over [Z, S, H, D], 128-byte swizzle); one
// tcgen05 MMA chain per 128-query tile computes the scores S = Q K^T into
// TMEM (M=128, N = the keys the tile sees: a causal first tile stops at
// 128); two threads per query row, each over half of the keys, take the
// row's max over the scores in TMEM and write p = 2^(s * log2(e)/sqrt(D) -
// max) as bf16 back into TMEM over them; a second MMA chain computes O = P V
// with P read from TMEM (V the MN-major operand from shared memory); the
// epilogue divides by the row sum of p (float32) and stores O by TMA.  The
// whole score row fits (S <= 256), so one pass suffices.  Two softmax
// groups alternate over the tiles, and the next unit's loads overlap the
// current one's work.
//
// Other shapes (D != 64, S > 256, float32): a warp per query row with an
// online softmax over the keys (float32 arithmetic).
#include <math.h>

#include "zg_ptx.cuh"
#include "zg_tc.cuh"

namespace {

// Persistent CTA (one per SM), 608 threads: warp 0 issues the TMA loads,
// warps 1 and 2 the MMAs of softmax group 0 and 1, warps 3-10 and 11-18 are
// the two softmax groups, two threads per query row (warps w and w + 4: the
// first and second half of the keys).  Work unit = one
// (z, head): its query tiles (one or two of 128 rows), keys and values, in
// one of two shared-memory buffers.  A buffer's queries and keys are loaded
// again as soon as the unit's Q K^T MMAs have read them, its values once the
// P V MMAs have, so the next units' loads run under this unit's softmax.
// Tile j of the CTA's sequence goes to group j % 2, which owns TMEM columns
// [256 g, 256 g + 256): the scores S (up to 256 columns), then P written
// over them in place (each half of the tile's keys at the start of its own
// score columns, key pair (c, c+1) of a half as bf16x2 in its column c/2;
// the P V MMA reads it from TMEM), and O in columns 192..255, which the
// softmax warps divide by their rows' sums of p and stage into their own
// boxes (32 rows x 32 columns) for TMA stores.  A unit's second query tile
// is loaded in reversed 32-row blocks (tile_block).
constexpr int AT_THREADS = 608;
constexpr uint32_t AT_Q = 0;         // 2 x 16 KiB: the unit's query tiles
constexpr uint32_t AT_K = 32768;     // 32 KiB: up to 256 key rows
constexpr uint32_t AT_V = 65536;     // 32 KiB: up to 256 value rows
constexpr uint32_t AT_BUF = 98304;   // one unit
constexpr uint32_t AT_STAGE = 2 * AT_BUF;           // 16 x 2 KiB: each softmax warp's output box
constexpr uint32_t AT_SUM = AT_STAGE + 16 * 2048;   // float [group][half][row]: the halves' sums of p
constexpr uint32_t AT_CTRL = AT_SUM + 2048;         // AttnCtrl
constexpr uint32_t AT_SMEM = AT_CTRL + 256;         // all of the kernel's shared memory (none static)

// mbarriers and the TMEM base, at AT_CTRL.  Per buffer: queries+keys and
// values loaded (full) / read by the MMAs (empty); per softmax group: scores
// ready, weights ready, O ready, O read, MMAs done at exit, the halves'
// maxima passed, the halves' sums passed.
struct AttnCtrl {
    uint64_t qk_full[2], v_full[2], qk_empty[2], v_empty[2], s_full[2], p_full[2], o_full[2], t_empty[2],
        done_bar[2], mx_bar[2], sum_bar[2];
    uint32_t tmem_base;
};
static_assert(sizeof(AttnCtrl) <= 256, "control block");

__device__ __forceinline__ float ex2_approx(float x) {
    float y;
    asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
    return y;
}

struct AttnArgs {
    int Z, S, H, s_pad, causal;
    float scale_log2;  // log2(e) / sqrt(D)
};

// The query tile of the CTA's tile j (unit j / nq): with two tiles per unit
// the order alternates between units, so each softmax group (j % 2) takes
// the short causal tile and the long one in turn.
__device__ __forceinline__ int tile_qt(int j, int nq) { return nq == 2 ? ((j & 1) ^ ((j >> 1) & 1)) : 0; }

// The 32-row block of query tile qt held in TMEM lane quarter `quad` (MMA
// rows 32 quad ..): the first tile in order, the second reversed.  Lane
// quarter q is read only by the warps of SM sub-partition q, and under the
// causal mask a tile's later rows see more keys, so the reversal gives each
// sub-partition one short and one long block of the unit's two tiles.
__device__ __forceinline__ int tile_block(int qt, int quad) { return qt == 1 ? 3 - quad : quad; }

// keys a query tile sees: causal tiles stop at their last query
__device__ __forceinline__ int tile_keys(const AttnArgs& a, int qt) {
    const int q0 = qt * 128;
    return a.causal && q0 + 128 < a.s_pad ? q0 + 128 : a.s_pad;
}

// Running maxima (8 independent chains) over a 32-key chunk of scores; only
// a chunk that crosses the row's last visible key tests each key.
__device__ __forceinline__ void chunk_max(const uint32_t (&r)[32], int c, int vis, float (&mx8)[8]) {
    if (c + 32 <= vis) {
#pragma unroll
        for (int e = 0; e < 32; ++e) mx8[e % 8] = fmaxf(mx8[e % 8], __uint_as_float(r[e]));
    } else {
#pragma unroll
        for (int e = 0; e < 32; ++e)
            if (c + e < vis) mx8[e % 8] = fmaxf(mx8[e % 8], __uint_as_float(r[e]));
    }
}

// bf16 weights p = 2^(s * scale - mx) of a 32-key chunk as 16 packed pairs
// (zero for keys past the row's last visible one, or for a chunk off), and
// their float32 values added pairwise into two running sums (packed f32x2
// adds on the FMA pipe).
__device__ __forceinline__ void chunk_weights(const uint32_t (&r)[32], int c, int vis, bool on, float scale,
                                              float mx, uint32_t (&pk)[16], float2 (&acc)[2]) {
    const float2 one = make_float2(1.f, 1.f);
    if (on && c + 32 <= vis) {
#pragma unroll
        for (int e = 0; e < 16; ++e) {
            const float p0 = ex2_approx(fmaf(__uint_as_float(r[2 * e]), scale, -mx));
            const float p1 = ex2_approx(fmaf(__uint_as_float(r[2 * e + 1]), scale, -mx));
            acc[e & 1] = ffma2_tc(make_float2(p0, p1), one, acc[e & 1]);
            const __nv_bfloat162 b2 = __floats2bfloat162_rn(p0, p1);
            pk[e] = *reinterpret_cast<const uint32_t*>(&b2);
        }
    } else if (on) {
#pragma unroll
        for (int e = 0; e < 16; ++e) {
            const int col = c + 2 * e;
            const float p0 = col < vis ? ex2_approx(fmaf(__uint_as_float(r[2 * e]), scale, -mx)) : 0.f;
            const float p1 = col + 1 < vis ? ex2_approx(fmaf(__uint_as_float(r[2 * e + 1]), scale, -mx)) : 0.f;
            acc[e & 1] = ffma2_tc(make_float2(p0, p1), one, acc[e & 1]);
            const __nv_bfloat162 b2 = __floats2bfloat162_rn(p0, p1);
            pk[e] = *reinterpret_cast<const uint32_t*>(&b2);
        }
    } else {
#pragma unroll
        for (int e = 0; e < 16; ++e) pk[e] = 0u;  // masked keys: zero weight
    }
}

// A bounded wait taken by every lane of a warp, with one outcome for all.
__device__ __forceinline__ bool warp_wait(uint64_t* bar, uint32_t parity, unsigned code) {
    return __all_sync(0xffffffffu, mbar_wait(bar, parity, code));
}

__global__ void __launch_bounds__(AT_THREADS, 1)
attn_tc_kernel(const __grid_constant__ CUtensorMap tmQ, const __grid_constant__ CUtensorMap tmK,
               const __grid_constant__ CUtensorMap tmV, const __grid_constant__ CUtensorMap tmO, const AttnArgs a) {
    // The kernel declares no static shared memory, so the dynamic block
    // starts at the CTA's first shared byte; the 128-byte-swizzled tiles need
    // it 1024-aligned, which is checked (error 90, every thread returns)
    // rather than padded for: the block fills the 227 KiB a CTA may hold.
    extern __shared__ __align__(1024) uint8_t smem[];
    if (smem_u32(smem) & 1023u) {
        if (threadIdx.x == 0) atomicCAS(&g_zg_tc_error, 0u, 90u);
        return;
    }
    AttnCtrl& cs = *reinterpret_cast<AttnCtrl*>(smem + AT_CTRL);
    uint64_t *qk_full = cs.qk_full, *v_full = cs.v_full, *qk_empty = cs.qk_empty, *v_empty = cs.v_empty,
             *s_full = cs.s_full, *p_full = cs.p_full, *o_full = cs.o_full, *t_empty = cs.t_empty,
             *done_bar = cs.done_bar, *mx_bar = cs.mx_bar, *sum_bar = cs.sum_bar;
    float* s_sum = reinterpret_cast<float*>(smem + AT_SUM);
    const int warp = threadIdx.x / 32, lane = threadIdx.x % 32;
    const int nq = a.s_pad / 128;  // query tiles per unit; also the key/value boxes
    const int64_t units = (int64_t)a.Z * a.H;
    const int my_units = units > (int64_t)blockIdx.x ? (int)((units - 1 - blockIdx.x) / gridDim.x + 1) : 0;
    const int tiles = my_units * nq;

    if (threadIdx.x == 0) {
        for (int i = 0; i < 2; ++i) {
            mbar_init(&qk_full[i], 1);
            mbar_init(&v_full[i], 1);
            mbar_init(&qk_empty[i], nq);  // one commit per tile of the unit
            mbar_init(&v_empty[i], nq);
            mbar_init(&s_full[i], 1);
            mbar_init(&p_full[i], 256);
            mbar_init(&o_full[i], 1);
            mbar_init(&t_empty[i], 8);
            mbar_init(&done_bar[i], 1);
            mbar_init(&mx_bar[i], 256);
            mbar_init(&sum_bar[i], 256);
        }
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    }
    if (warp == 1) tmem_alloc(&cs.tmem_base, 512);
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = cs.tmem_base;

    if (warp == 0) {
        if (lane == 0) {
            // unit u's values are loaded before unit u+1's queries and keys.
            // With two tiles per unit, u's buffer has its values freed (P V of
            // unit u-2) before u+1's buffer has its queries and keys freed
            // (Q K^T of unit u-1, issued by each group after its P V of u-2).
            // With one tile per unit those come from different groups, and
            // the fixed order can only delay a load: no P V waits on a later
            // unit's loads.
            uint32_t issued = 0, issue_parity = 0;  // bit b: QK loads of buffer b; bit b+2: V loads
            for (int u = 0; u < my_units; ++u) {
                const int b = u & 1;
                const uint32_t m = (uint32_t)(u >> 1);
                const int64_t U = blockIdx.x + (int64_t)u * gridDim.x;
                const int z = (int)(U / a.H), h = (int)(U % a.H);
                uint8_t* buf = smem + b * AT_BUF;
                if (!mbar_wait(&qk_empty[b], (m & 1) ^ 1, 81)) break;
                mbar_expect_tx(&qk_full[b], (uint32_t)(2 * nq) * 16384u);
                for (int i = 0; i < nq; ++i) {
                    // query tile i as four 32-row blocks, the second tile's in
                    // reverse order (tile_block)
                    for (int blk = 0; blk < 4; ++blk)
                        tma_load_4d(buf + AT_Q + i * 16384 + blk * 4096, &tmQ, &qk_full[b], 0, h,
                                    i * 128 + 32 * tile_block(i, blk), z);
                    tma_load_4d(buf + AT_K + i * 16384, &tmK, &qk_full[b], 0, h, i * 128, z);
                }
                issued |= 1u << b;
                issue_parity = (issue_parity & ~(1u << b)) | ((m & 1) << b);
                if (!mbar_wait(&v_empty[b], (m & 1) ^ 1, 88)) break;
                mbar_expect_tx(&v_full[b], (uint32_t)nq * 16384u);
                for (int i = 0; i < nq; ++i)
                    tma_load_4d(buf + AT_V + i * 16384, &tmV, &v_full[b], 0, h, i * 128, z);
                issued |= 4u << b;
                issue_parity = (issue_parity & ~(4u << b)) | ((m & 1) << (b + 2));
            }
            // loads still in flight (only after an abort) land before the CTA exits
            for (int i = 0; i < 4; ++i)
                if (issued >> i & 1) {
                    uint64_t* bar = i < 2 ? &qk_full[i] : &v_full[i - 2];
                    for (uint32_t t = 0; t < kSpinLimit && !mbar_try_wait(bar, issue_parity >> i & 1); ++t) {
                    }
                }
        }
    } else if (warp <= 2) {
        if (lane == 0) {
            // one MMA issuer per softmax group: S = Q K^T of the group's next
            // tile once it has read the previous tile's O, then P V once its
            // weights are in TMEM
            const int g = warp - 1;
            const uint32_t pt = tmem + g * 256;
            for (int j = g; j < tiles; j += 2) {
                const int u = j / nq, qt = tile_qt(j, nq), b = u & 1;
                const uint32_t n = (uint32_t)(j >> 1), m = (uint32_t)(u >> 1);
                if (!mbar_wait(&qk_full[b], m & 1, 82)) break;
                if (!mbar_wait(&t_empty[g], (n & 1) ^ 1, 83)) break;
                tc_fence_after();
                const uint32_t qa = smem_u32(smem + b * AT_BUF + AT_Q + qt * 16384);
                const uint32_t ka = smem_u32(smem + b * AT_BUF + AT_K);
                const uint32_t idesc_s = idesc_bf16(128, tile_keys(a, qt), 0);
#pragma unroll
                for (int k = 0; k < 4; ++k)
                    umma_bf16(pt, smem_desc(qa + k * 32, 16, 1024), smem_desc(ka + k * 32, 16, 1024), idesc_s,
                              k > 0 ? 1u : 0u);
                umma_commit(&s_full[g]);
                umma_commit(&qk_empty[b]);  // this tile's queries and keys are read

                if (!mbar_wait(&p_full[g], n & 1, 84)) break;
                if (!mbar_wait(&v_full[b], m & 1, 89)) break;
                tc_fence_after();
                const uint32_t idesc = idesc_bf16(128, 64, 1);
                const uint32_t va = smem_u32(smem + b * AT_BUF + AT_V);
                const int hw = tile_keys(a, qt) / 2, hk = hw / 16;  // each half's P at the start of its scores
                for (int kk = 0; kk < 2 * hk; ++kk)
                    umma_bf16_ts(pt + 192, pt + (kk < hk ? kk * 8 : hw + (kk - hk) * 8),
                                 smem_desc(va + kk * 2048, 64 * 256 * 2, 1024), idesc, kk > 0 ? 1u : 0u);
                umma_commit(&o_full[g]);
                umma_commit(&v_empty[b]);  // this tile's values are read
            }
            // every MMA this thread issued has completed before TMEM is freed
            umma_commit(&done_bar[g]);
            for (uint32_t i = 0; i < kSpinLimit && !mbar_try_wait(&done_bar[g], 0); ++i) {
            }
        }
    } else {
        // softmax: two threads per query row, each one half of the tile's keys
        const int g = (warp - 3) / 8, half = ((warp - 3) % 8) / 4, quad = warp % 4;  // quad: TMEM lane quarter
        const uint32_t trow = tmem + ((uint32_t)(quad * 32) << 16) + (uint32_t)(g * 256);
        // this warp's output box (32 rows x 64 B); its first 128 B also pass
        // the rows' partial maxima to the other half's warp (warp -/+ 4)
        uint8_t* stage = smem + AT_STAGE + (warp - 3) * 2048;
        const float* partner_mx = reinterpret_cast<const float*>(stage + (half ? -4 : 4) * 2048);
        for (int j = g; j < tiles; j += 2) {
            const uint32_t n = (uint32_t)(j >> 1);
            const int u = j / nq, qt = tile_qt(j, nq);
            const uint32_t U = blockIdx.x + (uint32_t)u * gridDim.x;
            const int z = (int)(U / (uint32_t)a.H), h = (int)(U % (uint32_t)a.H);
            const int q0 = qt * 128, n_keys = tile_keys(a, qt), hw = n_keys / 2;
            const int k0 = half * hw;  // this thread's keys: [k0, k0 + hw)
            if (!warp_wait(&s_full[g], n & 1, 85)) break;
            tc_fence_after();

            // columns [0, vis) are visible to this query: the keys, up to the query when causal
            const int row0 = q0 + 32 * tile_block(qt, quad);  // the warp's first query row
            const int qi = row0 + lane;
            const int vis = a.causal ? (qi + 1 < a.S ? qi + 1 : a.S) : a.S;
            // the warp's last visible column (its last row sees the most): chunks past it hold no weight
            const int wvis = __reduce_max_sync(0xffffffffu, vis);
            const int c_end = ((wvis + 31) / 32) * 32 < n_keys ? ((wvis + 31) / 32) * 32 : n_keys;
            const int c_stop = k0 + hw < c_end ? k0 + hw : c_end;  // this half's chunks that hold weight
            // the maximum over this half (8 independent chains; only chunks
            // that cross the row's last visible key test each key)
            float mx8[8];
#pragma unroll
            for (int e = 0; e < 8; ++e) mx8[e] = -INFINITY;
#pragma unroll 1
            for (int c = k0; c < c_stop; c += 32) {
                uint32_t rc[32];
                tmem_ld32_nowait(trow + c, rc);
                tmem_wait_ld32(rc);
                chunk_max(rc, c, vis, mx8);
            }
            // the row's maximum over both halves: this half's through the
            // staging box (read out by the last output store before)
            if (lane == 0) asm volatile("cp.async.bulk.wait_group.read 0;" ::: "memory");
            __syncwarp();
            reinterpret_cast<float*>(stage)[lane] = fmaxf(fmaxf(fmaxf(mx8[0], mx8[1]), fmaxf(mx8[2], mx8[3])),
                                                          fmaxf(fmaxf(mx8[4], mx8[5]), fmaxf(mx8[6], mx8[7])));
            mbar_arrive(&mx_bar[g]);
            if (!warp_wait(&mx_bar[g], n & 1, 87)) break;
            // scale_log2 > 0: max(s) * scale = max(s * scale)
            const float mx = fmaxf(reinterpret_cast<const float*>(stage)[lane], partner_mx[lane]) * a.scale_log2;
            // the weights of this half at the start of its own scores, over
            // columns this thread has already read: keys (2e, 2e+1) of chunk
            // i in column 16 i + e of the half
            float2 acc[2] = {make_float2(0.f, 0.f), make_float2(0.f, 0.f)};
#pragma unroll 1
            for (int c = k0; c < k0 + hw; c += 32) {
                const bool on = c < c_stop;
                uint32_t rc[32];
                if (on) {
                    tmem_ld32_nowait(trow + c, rc);
                    tmem_wait_ld32(rc);
                }
                uint32_t pk[16];
                chunk_weights(rc, c, vis, on, a.scale_log2, mx, pk, acc);
                tmem_st16u(trow + k0 + (c - k0) / 2, pk);
            }
            // this half's sum of p for the other half's epilogue
            float* my_sum = s_sum + (g * 2 + half) * 128 + 32 * quad + lane;
            *my_sum = (acc[0].x + acc[0].y) + (acc[1].x + acc[1].y);
            mbar_arrive(&sum_bar[g]);
            tmem_wait_st();
            tc_fence_before();
            mbar_arrive(&p_full[g]);

            if (!warp_wait(&o_full[g], n & 1, 86)) break;
            tc_fence_after();
            // this half's 32 columns of O / sum -> bf16 into the warp's box
            // (64-byte swizzle: 16-byte chunk i of row l at
            // (i ^ ((l >> 1) & 3)) * 16), then one TMA store of the box
            if (!warp_wait(&sum_bar[g], n & 1, 91)) break;
            const float* row_sums = s_sum + g * 256 + 32 * quad + lane;
            const float inv = 1.f / (row_sums[0] + row_sums[128]);  // the halves' sums of p, in half order
            float o[32];
            tmem_ld32(trow + 192 + 32 * half, o);
            tc_fence_before();
            __syncwarp();
            if (lane == 0) mbar_arrive(&t_empty[g]);  // the MMA warp may write this group's columns again
            uint8_t* row = stage + lane * 64;
#pragma unroll
            for (int i = 0; i < 4; ++i) {
                uint4 pk;
                __nv_bfloat162* hp = reinterpret_cast<__nv_bfloat162*>(&pk);
#pragma unroll
                for (int e = 0; e < 4; ++e)
                    hp[e] = __floats2bfloat162_rn(o[8 * i + 2 * e] * inv, o[8 * i + 2 * e + 1] * inv);
                *reinterpret_cast<uint4*>(row + ((i ^ ((lane >> 1) & 3)) * 16)) = pk;
            }
            asm volatile("fence.proxy.async.shared::cta;" ::: "memory");  // staging visible to the bulk store
            __syncwarp();
            if (lane == 0 && row0 < a.S) {  // rows past S are clipped; wholly past S, not stored
                tma_store_4d(&tmO, stage, 32 * half, h, row0, z);
                asm volatile("cp.async.bulk.commit_group;" ::: "memory");
            }
            __syncwarp();
        }
        if (lane == 0) asm volatile("cp.async.bulk.wait_group 0;" ::: "memory");
    }
    tc_fence_before();
    __syncthreads();
    if (warp == 1) {
        tc_fence_after();
        tmem_dealloc(tmem, 512);
    }
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

// Timed-out waits of the tensor-core kernel (codes 81-89, 91) or its shared
// memory not 1024-aligned (90); 0 = none.
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
        const size_t smem = AT_SMEM;
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
        // queries in 32-row boxes (one TMEM lane quarter), keys and values in
        // 128; outputs in boxes of 32 rows x 32 columns (one warp's half rows)
        const uint32_t box[4] = {64, 1, 128, 1}, qbox[4] = {64, 1, 32, 1}, obox[4] = {32, 1, 32, 1};
        if (!zg::tensor_map_bf16(&tq, q, 4, dims, strides, qbox, true) ||
            !zg::tensor_map_bf16(&tk, k, 4, dims, strides, box, true) ||
            !zg::tensor_map_bf16(&tv, v, 4, dims, strides, box, true) ||
            !zg::tensor_map_bf16_swz(&to, o, 4, dims, ostrides, obox, 64))
            return zg::fail(ZG_ERR_CUDA, "zg_attention: tensor maps");
        AttnArgs a{Z, S, H, S <= 128 ? 128 : 256, causal != 0, (float)(1.4426950408889634 / sqrt(64.0))};
        const int64_t units = (int64_t)Z * H;
        const unsigned grid = (unsigned)(units < sm_count_attn() ? units : sm_count_attn());
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
