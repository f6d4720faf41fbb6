// zg_int8.cu -- integer QAT linear: int8 x int8 -> int32 GEMM with a
// float32 low-rank perturbation and a 256-entry int8 LUT activation.
//
// There is no reference counterpart (the reference only fake-quantises in
// float, examples/train_qat_xor.py:41-50); the semantics are defined by the
// oracle (oracle/zgref.c zgo_int8_lut_linear) and matched bit for bit:
//   acc = x @ W (exact int32)
//   u[m,j] = sequential float32 FMA over k of x[m,k] * A[k,j]
//   lr = sequential FMA over j of u[m,j] * B[j,n]
//   y = fma(float(acc) * x_scale, w_scale[n], s * lr)
//   q = clamp(rint(y / y_scale), -128, 127) (0 for NaN); out = lut[q + 128]
//
// Paths: the accumulator GEMM runs on the tcgen05 tensor cores (kind::i8,
// exact int32 accumulators in TMEM) with the scale / low-rank / rint / LUT
// steps fused into its epilogue; a CUDA-core kernel covers shapes the TMA
// layout rules exclude (K or N not a multiple of 16).  u uses one thread per
// (candidate, row) with the oracle's sequential order, its input staged
// through shared memory.
#include <cudaTypedefs.h>

#include <climits>

#include "zg_ptx.cuh"
#include "zg_tc.cuh"

namespace zg {
int launch_population_factors(const uint32_t* keys, int group, int P, int layout, int64_t rows,
                              int64_t cols, int rank, int dtype, void* A, void* B,
                              cudaStream_t st);
}

namespace {

// u[p,m,j]: one thread per (m, j), sequential k (the oracle's order).
__global__ void int8_u_kernel(const int8_t* __restrict__ x, int x_batched, const float* __restrict__ A,
                              int M, int K, int rank, float* __restrict__ U) {
    const int p = blockIdx.y;
    const int64_t e = blockIdx.x * (int64_t)blockDim.x + threadIdx.x;
    if (e >= (int64_t)M * rank) return;
    const int m = (int)(e / rank), j = (int)(e % rank);
    const int8_t* xr = x + (x_batched ? (int64_t)p * M * K : 0) + (int64_t)m * K;
    const float* a = A + (int64_t)p * K * rank + j;
    float acc = 0.f;
    for (int k = 0; k < K; ++k) acc = __fmaf_rn((float)xr[k], a[(int64_t)k * rank], acc);
    U[((int64_t)p * M + m) * rank + j] = acc;
}

// u[p,m,0:R]: one thread per (candidate, row), the R sums advanced together
// in k order (the oracle's order).  A block of 128 rows stages the input in
// 128-byte K slabs through shared memory (coalesced 16-byte loads; rows
// padded to 144 bytes so a quarter-warp's 16-byte reads hit distinct banks)
// together with the slab's A_p rows, read as broadcasts.
constexpr int U_ROWS = 128, U_SLAB = 128, U_PITCH = 144;

// float(b) of a signed byte without the conversion unit (exact).
__device__ __forceinline__ float s8_to_f32(uint32_t word, int byte) {
    const int b = (int)(int8_t)(uint8_t)(word >> (8 * byte));
    return __fsub_rn(__int_as_float(0x4B400000 + b), 12582912.0f);
}

template <int R>
__global__ void __launch_bounds__(U_ROWS)
int8_u_tile_kernel(const int8_t* __restrict__ x, int x_batched, const float* __restrict__ A, int M, int K,
                   float* __restrict__ U) {
    constexpr int XV = U_ROWS * (U_SLAB / 16) / U_ROWS;  // 16-byte pieces of a slab per thread (8)
    __shared__ __align__(16) int8_t xs[U_ROWS][U_PITCH];
    __shared__ __align__(16) float as[U_SLAB][R];
    const int p = blockIdx.y, m0 = blockIdx.x * U_ROWS, tid = threadIdx.x;
    const int8_t* xp = x + (x_batched ? (int64_t)p * M * K : 0);
    const float* ap = A + (int64_t)p * K * R;
    const bool vec = (K % 16) == 0 && (reinterpret_cast<uintptr_t>(x) & 15) == 0;
    const bool avec = R % 4 == 0 && (reinterpret_cast<uintptr_t>(A) & 15) == 0;
    // The next slab is fetched into registers while this one is summed:
    // all of a thread's pieces are requested before any is needed.
    uint4 nx[XV];
    float4 na[R % 4 == 0 ? R / 4 : 1];
    auto fetch = [&](int k0) {
#pragma unroll
        for (int i = 0; i < XV; ++i) {
            const int c = tid + i * U_ROWS;
            const int r = c / (U_SLAB / 16), q = c % (U_SLAB / 16);
            const int m = m0 + r, k = k0 + q * 16;
            uint4 v = make_uint4(0, 0, 0, 0);
            if (m < M) {
                const int8_t* src = xp + (int64_t)m * K + k;
                if (vec && k + 16 <= K) {
                    v = *reinterpret_cast<const uint4*>(src);
                } else {
                    int8_t tmp[16];
#pragma unroll
                    for (int e = 0; e < 16; ++e) tmp[e] = k + e < K ? src[e] : (int8_t)0;
                    v = *reinterpret_cast<const uint4*>(tmp);
                }
            }
            nx[i] = v;
        }
        if (avec) {  // this thread's A row of the slab (k0 + tid), R floats as float4s
#pragma unroll
            for (int i = 0; i < (R % 4 == 0 ? R / 4 : 1); ++i)
                na[i] = k0 + tid < K ? *reinterpret_cast<const float4*>(ap + (int64_t)(k0 + tid) * R + 4 * i)
                                     : make_float4(0.f, 0.f, 0.f, 0.f);
        }
    };
    float acc[R];
#pragma unroll
    for (int j = 0; j < R; ++j) acc[j] = 0.f;
    fetch(0);
    for (int k0 = 0; k0 < K; k0 += U_SLAB) {
        __syncthreads();  // the last slab is summed: its buffers may be overwritten
#pragma unroll
        for (int i = 0; i < XV; ++i) {
            const int c = tid + i * U_ROWS;
            *reinterpret_cast<uint4*>(&xs[c / (U_SLAB / 16)][(c % (U_SLAB / 16)) * 16]) = nx[i];
        }
        if (avec) {
#pragma unroll
            for (int i = 0; i < (R % 4 == 0 ? R / 4 : 1); ++i) *reinterpret_cast<float4*>(&as[tid][4 * i]) = na[i];
        } else {
            for (int e = tid; e < U_SLAB * R; e += U_ROWS) {
                const int kk = e / R, j = e % R;
                as[kk][j] = k0 + kk < K ? ap[(int64_t)(k0 + kk) * R + j] : 0.f;
            }
        }
        __syncthreads();
        if (k0 + U_SLAB < K) fetch(k0 + U_SLAB);
        const int kw = K - k0 < U_SLAB ? K - k0 : U_SLAB;
        if (kw == U_SLAB) {  // a full slab: no per-byte test
#pragma unroll 2
            for (int kk0 = 0; kk0 < U_SLAB; kk0 += 16) {
                const uint4 v = *reinterpret_cast<const uint4*>(&xs[tid][kk0]);
                const uint32_t w[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
                for (int i = 0; i < 16; ++i) {
                    const float xv = s8_to_f32(w[i / 4], i % 4);
#pragma unroll
                    for (int j = 0; j < R; ++j) acc[j] = __fmaf_rn(xv, as[kk0 + i][j], acc[j]);
                }
            }
        } else {
            // zero-padded bytes past K are never folded in: the loop stops at kw
            for (int kk0 = 0; kk0 < kw; kk0 += 16) {
                const uint4 v = *reinterpret_cast<const uint4*>(&xs[tid][kk0]);
                const uint32_t w[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
                for (int i = 0; i < 16; ++i) {
                    if (kk0 + i < kw) {
                        const float xv = s8_to_f32(w[i / 4], i % 4);
#pragma unroll
                        for (int j = 0; j < R; ++j) acc[j] = __fmaf_rn(xv, as[kk0 + i][j], acc[j]);
                    }
                }
            }
        }
    }
    if (m0 + tid < M) {
#pragma unroll
        for (int j = 0; j < R; ++j) U[((int64_t)p * M + m0 + tid) * R + j] = acc[j];
    }
}

constexpr int BM = 64, BN = 64, BK = 32, THREADS = 256;

// Exact int32 GEMM tile + LUT epilogue.  grid (N/BN, M/BM, P).
__global__ void __launch_bounds__(THREADS)
int8_lut_simt_kernel(const int8_t* __restrict__ x, int x_batched, const int8_t* __restrict__ W,
                     const float* __restrict__ w_scale, float x_scale, float y_scale,
                     const int8_t* __restrict__ lut, const float* __restrict__ U,
                     const float* __restrict__ Bf, int rank, float s, int M, int K, int N,
                     int8_t* __restrict__ out, int32_t* __restrict__ acc_out) {
    __shared__ int Xs[BK][BM + 1];
    __shared__ int Ws[BK][BN + 1];
    __shared__ int8_t slut[256];
    const int p = blockIdx.z;
    const int m0 = blockIdx.y * BM, n0 = blockIdx.x * BN;
    const int tid = threadIdx.x, tx = tid % 16, ty = tid / 16;
    slut[tid] = lut[tid];
    const int8_t* xp = x + (x_batched ? (int64_t)p * M * K : 0);
    int acc[4][4] = {};
    for (int k0 = 0; k0 < K; k0 += BK) {
#pragma unroll
        for (int i = 0; i < (BM * BK) / THREADS; ++i) {
            int e = tid + i * THREADS;
            int kk = e % BK, mm = e / BK;
            int k = k0 + kk, m = m0 + mm;
            Xs[kk][mm] = (k < K && m < M) ? (int)xp[(int64_t)m * K + k] : 0;
        }
#pragma unroll
        for (int i = 0; i < (BN * BK) / THREADS; ++i) {
            int e = tid + i * THREADS;
            int nn = e % BN, kk = e / BN;
            int k = k0 + kk, n = n0 + nn;
            Ws[kk][nn] = (k < K && n < N) ? (int)W[(int64_t)k * N + n] : 0;
        }
        __syncthreads();
#pragma unroll 8
        for (int kk = 0; kk < BK; ++kk) {
#pragma unroll
            for (int i = 0; i < 4; ++i)
#pragma unroll
                for (int j = 0; j < 4; ++j) acc[i][j] += Xs[kk][ty + 16 * i] * Ws[kk][tx + 16 * j];
        }
        __syncthreads();
    }
#pragma unroll
    for (int i = 0; i < 4; ++i) {
        const int m = m0 + ty + 16 * i;
        if (m >= M) continue;
        const float* u = U + ((int64_t)p * M + m) * rank;
#pragma unroll
        for (int j = 0; j < 4; ++j) {
            const int n = n0 + tx + 16 * j;
            if (n >= N) continue;
            const float* b = Bf + (int64_t)p * rank * N + n;
            float lr = 0.f;
            for (int r = 0; r < rank; ++r) lr = __fmaf_rn(u[r], b[(int64_t)r * N], lr);
            const float y = __fmaf_rn(__fmul_rn((float)acc[i][j], x_scale), w_scale[n], __fmul_rn(s, lr));
            const float qf = rintf(__fdiv_rn(y, y_scale));
            const int q = qf != qf ? 0 : (qf > 127.f ? 127 : (qf < -128.f ? -128 : (int)qf));
            const int64_t o = ((int64_t)p * M + m) * N + n;
            out[o] = slut[q + 128];
            if (acc_out) acc_out[o] = acc[i][j];
        }
    }
}

// ---------------------------------------------------------------------------
// Tensor-core form: tiles of 128 rows x 256 columns, 128-deep K blocks
// (x K-major, W [K, N] MN-major, both 128B-swizzled), tcgen05.mma kind::i8
// M=128 N=256 K=32 into int32 TMEM accumulators (two, so one tile's epilogue
// overlaps the next tile's K loop).  Work unit = (candidate chunk, m tile,
// n tile): with a per-candidate input the chunk is one candidate; with a
// shared input the exact x.W tile is computed once per chunk and the
// epilogue writes every candidate of the chunk from it.
// ---------------------------------------------------------------------------
constexpr int I8_BM = 128, I8_BN = 256, I8_BK = 128, I8_STAGES = 4, I8_THREADS = 320;  // 2 + 8 warps
constexpr uint32_t I8_A = I8_BM * I8_BK;              // 16 KiB
constexpr uint32_t I8_B = I8_BN * I8_BK;              // 32 KiB: two 128-column blocks
constexpr uint32_t I8_STAGE = I8_A + I8_B;            // 48 KiB
constexpr uint32_t I8_SMEM = I8_STAGES * I8_STAGE;    // 192 KiB

// Instruction descriptor, kind::i8: D s32, A and B signed 8-bit, A K-major,
// B MN-major (b_mn = 1), N >> 3, M >> 4.
__host__ __device__ constexpr uint32_t idesc_s8(int M, int N, int b_mn) {
    return (2u << 4) | (1u << 7) | (1u << 10) | ((uint32_t)b_mn << 16) | ((uint32_t)(N >> 3) << 17) |
           ((uint32_t)(M >> 4) << 24);
}

__device__ __forceinline__ void umma_s8(uint32_t d_tmem, uint64_t a_desc, uint64_t b_desc, uint32_t idesc,
                                        uint32_t accumulate) {
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "setp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::1.kind::i8 [%0], %1, %2, %3, p;\n\t}"
        ::"r"(d_tmem), "l"(a_desc), "l"(b_desc), "r"(idesc), "r"(accumulate));
}

// float(a), correctly rounded, without the conversion unit: a = h*2^16 + l
// with both halves exact in float (magic-number adds), and one FMA rounds
// h*2^16 + l once, which is the round-to-nearest value of a.
__device__ __forceinline__ float s32_to_f32_rn(int a) {
    const int h = a >> 16;      // [-32768, 32767]
    const int l = a & 0xFFFF;   // [0, 65535]
    const float hf = __fsub_rn(__int_as_float(0x4B400000 + h), 12582912.0f);
    const float lf = __fsub_rn(__int_as_float(0x4B000000 | l), 8388608.0f);
    return __fmaf_rn(hf, 65536.0f, lf);
}

// clamp((int)rintf(v), -128, 127) with (int)NaN = 0.  Clamping to the
// integer bounds first commutes with rounding; adding 1.5 * 2^23 then rounds
// to the nearest integer (ties to even) into the low mantissa bits.
__device__ __forceinline__ int rint_clamp_s8(float v) {
    const float c = v != v ? 0.f : fminf(fmaxf(v, -128.f), 127.f);
    return __float_as_int(__fadd_rn(c, 12582912.0f)) - 0x4B400000;
}

struct I8Args {
    int8_t* out;
    int32_t* acc_out;
    const float* w_scale;
    const float* U;
    const float* Bf;
    const int8_t* lut;
    float x_scale, y_scale, s;
    float y_inv;  // 1 / y_scale when y_scale is a power of two (exact), else 0
    int M, N, K, P, rank, tiles_m, tiles_n, chunk, chunks, x_batched;
};

// Named barrier 1 over the eight epilogue warps, and its AND-vote form.
__device__ __forceinline__ void epi8_bar() { asm volatile("bar.sync 1, 256;" ::: "memory"); }
__device__ __forceinline__ bool epi8_all(bool v) {
    uint32_t out;
    asm volatile(
        "{\n\t.reg .pred pi, po;\n\t"
        "setp.ne.u32 pi, %1, 0;\n\t"
        "bar.red.and.pred po, 1, 256, pi;\n\t"
        "selp.u32 %0, 1, 0, po;\n\t}"
        : "=r"(out)
        : "r"((uint32_t)v)
        : "memory");
    return out != 0;
}

// R: the perturbation rank; POW2: y_scale is a power of two, so y / y_scale
// is exactly y * y_inv.
template <int R, bool POW2>
__global__ void __launch_bounds__(I8_THREADS, 1)
int8_lut_tc_kernel(const __grid_constant__ CUtensorMap tmX, const __grid_constant__ CUtensorMap tmW,
                   const I8Args a) {
    extern __shared__ uint8_t dyn_smem[];
    __shared__ __align__(8) uint64_t full_bar[I8_STAGES], empty_bar[I8_STAGES], tmem_full[2], tmem_empty[2],
        mma_done;
    __shared__ uint32_t tmem_base_sh;
    __shared__ int8_t slut[256];
    __shared__ __align__(16) float s_wsc[I8_BN];
    __shared__ __align__(16) float s_b[R][I8_BN];
    const uint32_t dyn_base = smem_u32(dyn_smem);
    uint8_t* smem = dyn_smem + (((dyn_base + 1023u) & ~1023u) - dyn_base);
    const int warp = threadIdx.x / 32, lane = threadIdx.x % 32;
    const int num_tiles = a.chunks * a.tiles_m * a.tiles_n;
    const int k_blocks = (a.K + I8_BK - 1) / I8_BK;

    for (int i = threadIdx.x; i < 256; i += I8_THREADS) slut[i] = a.lut[i];
    if (threadIdx.x == 0) {
        for (int s = 0; s < I8_STAGES; ++s) {
            mbar_init(&full_bar[s], 1);
            mbar_init(&empty_bar[s], 1);
        }
        for (int b = 0; b < 2; ++b) {
            mbar_init(&tmem_full[b], 1);
            mbar_init(&tmem_empty[b], 8);  // one arrive per epilogue warp
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
        int stage = 0;
        uint32_t phase = 0, issued = 0, issue_parity = 0;
        bool ok = true;
        for (int t = blockIdx.x; ok && t < num_tiles; t += gridDim.x) {
            const int tn = t % a.tiles_n, rest = t / a.tiles_n;
            const int tm = rest % a.tiles_m, c = rest / a.tiles_m;
            const int z = a.x_batched ? c : 0;
            const int k_start = t % k_blocks;
            for (int kb = 0; kb < k_blocks; ++kb) {
                if (!mbar_wait(&empty_bar[stage], phase ^ 1, 61)) { ok = false; break; }
                const int kk = kb + k_start < k_blocks ? kb + k_start : kb + k_start - k_blocks;
                uint8_t* sa = smem + stage * I8_STAGE;
                uint8_t* sb = sa + I8_A;
                mbar_expect_tx(&full_bar[stage], I8_STAGE);
                tma_load_3d(sa, &tmX, &full_bar[stage], kk * I8_BK, tm * I8_BM, z);
#pragma unroll
                for (int cc = 0; cc < 2; ++cc)
                    tma_load_2d(sb + cc * (128 * I8_BK), &tmW, &full_bar[stage], tn * I8_BN + cc * 128, kk * I8_BK);
                issued |= 1u << stage;
                issue_parity = (issue_parity & ~(1u << stage)) | (phase << stage);
                if (++stage == I8_STAGES) { stage = 0; phase ^= 1; }
            }
        }
        for (int s = 0; s < I8_STAGES; ++s)
            if (issued & (1u << s))
                for (uint32_t i = 0; i < kSpinLimit; ++i)
                    if (mbar_try_wait(&full_bar[s], (issue_parity >> s) & 1)) break;
    } else if (warp == 1 && lane == 0) {
        // ---------------- MMA issuer ----------------
        constexpr uint32_t IDESC = idesc_s8(I8_BM, I8_BN, 1);
        int stage = 0, acc = 0;
        uint32_t phase = 0, acc_phase = 0;
        bool ok = true;
        for (int t = blockIdx.x; ok && t < num_tiles; t += gridDim.x) {
            if (!mbar_wait(&tmem_empty[acc], acc_phase ^ 1, 62)) break;
            tc_fence_after();
            const uint32_t d_tmem = tmem_base + acc * I8_BN;
            for (int kb = 0; kb < k_blocks; ++kb) {
                if (!mbar_wait(&full_bar[stage], phase, 63)) { ok = false; break; }
                tc_fence_after();
                const uint32_t a_addr = smem_u32(smem + stage * I8_STAGE);
                const uint32_t b_addr = a_addr + I8_A;
#pragma unroll
                for (int k = 0; k < I8_BK / 32; ++k) {
                    // K-major SW128: 32 int8 of K = 32 bytes along the swizzled row;
                    // MN-major SW128: 128-column blocks 16 KiB apart, 8-row K groups
                    // 1 KiB apart, 32 K rows = 4 KiB per step.
                    umma_s8(d_tmem, smem_desc(a_addr + k * 32, 16, 1024),
                            smem_desc(b_addr + k * 4096, 128 * I8_BK, 1024), IDESC, (kb > 0 || k > 0) ? 1u : 0u);
                }
                umma_commit(&empty_bar[stage]);
                if (++stage == I8_STAGES) { stage = 0; phase ^= 1; }
            }
            if (!ok) break;
            umma_commit(&tmem_full[acc]);
            if (++acc == 2) { acc = 0; acc_phase ^= 1; }
        }
        umma_commit(&mma_done);
        for (uint32_t i = 0; i < kSpinLimit; ++i)
            if (mbar_try_wait(&mma_done, 0)) break;
    } else if (warp >= 2) {
        // ---------------- epilogue: scales, low-rank term, rint, LUT ----------------
        // 8 warps: warp w reads TMEM lanes 32 (w % 4) .. +31 (its rows) and
        // columns 128 ((w - 2) / 4) .. +127 of the tile.  Per-column operands
        // (w_scale, B_p rows) are staged in shared memory once per tile /
        // candidate and read as broadcasts.  Every epilogue warp walks every
        // tile, so the named barriers always see all eight.
        const int quad = warp % 4, half = (warp - 2) / 4;
        const int et = threadIdx.x - 64;  // 0..255
        int acc = 0;
        uint32_t acc_phase = 0;
        bool ok = true;
        for (int t = blockIdx.x; t < num_tiles; t += gridDim.x) {
            ok = ok && mbar_wait(&tmem_full[acc], acc_phase, 64);
            ok = epi8_all(ok);
            if (!ok) {
                if (++acc == 2) { acc = 0; acc_phase ^= 1; }
                continue;
            }
            tc_fence_after();
            const int tn = t % a.tiles_n, rest = t / a.tiles_n;
            const int tm = rest % a.tiles_m, c = rest / a.tiles_m;
            const int row = tm * I8_BM + quad * 32 + lane;
            const int n0 = tn * I8_BN;
            const int p0 = c * a.chunk, p1 = min(a.P, p0 + a.chunk);
            const uint32_t tacc = tmem_base + ((uint32_t)(quad * 32) << 16) + acc * I8_BN + half * 128;
            {
                const int n = n0 + et;
                s_wsc[et] = n < a.N ? a.w_scale[n] : 0.f;
            }
            for (int p = p0; p < p1; ++p) {
                epi8_bar();  // previous candidate's reads of s_b are done (and s_wsc written)
                const float* bp = a.Bf + (int64_t)p * a.rank * a.N;
                for (int e = et; e < R * I8_BN; e += 256) {
                    const int j = e / I8_BN, nl = e % I8_BN, n = n0 + nl;
                    s_b[j][nl] = n < a.N ? bp[(int64_t)j * a.N + n] : 0.f;
                }
                float ur[R];
#pragma unroll
                for (int j = 0; j < R; ++j) ur[j] = row < a.M ? a.U[((int64_t)p * a.M + row) * R + j] : 0.f;
                epi8_bar();
#pragma unroll 1
                for (int c0 = 0; c0 < 128; c0 += 32) {
                    float vf[32];
                    __syncwarp();
                    tmem_ld32(tacc + c0, vf);
                    const int nl0 = half * 128 + c0, col0 = n0 + nl0;
                    if (row >= a.M || col0 >= a.N) continue;
                    uint32_t packed[8];
#pragma unroll
                    for (int i4 = 0; i4 < 32; i4 += 4) {
                        const float4 w4 = *reinterpret_cast<const float4*>(&s_wsc[nl0 + i4]);
                        float lr[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll
                        for (int j = 0; j < R; ++j) {
                            const float4 b4 = *reinterpret_cast<const float4*>(&s_b[j][nl0 + i4]);
                            lr[0] = __fmaf_rn(ur[j], b4.x, lr[0]);
                            lr[1] = __fmaf_rn(ur[j], b4.y, lr[1]);
                            lr[2] = __fmaf_rn(ur[j], b4.z, lr[2]);
                            lr[3] = __fmaf_rn(ur[j], b4.w, lr[3]);
                        }
                        const float wv[4] = {w4.x, w4.y, w4.z, w4.w};
                        uint32_t word = 0;
#pragma unroll
                        for (int k = 0; k < 4; ++k) {
                            const float y = __fmaf_rn(__fmul_rn(s32_to_f32_rn(__float_as_int(vf[i4 + k])), a.x_scale),
                                                      wv[k], __fmul_rn(a.s, lr[k]));
                            const float v = POW2 ? __fmul_rn(y, a.y_inv) : __fdiv_rn(y, a.y_scale);
                            word |= (uint32_t)(uint8_t)slut[rint_clamp_s8(v) + 128] << (8 * k);
                        }
                        packed[i4 / 4] = word;
                    }
                    const int64_t o = ((int64_t)p * a.M + row) * a.N + col0;
                    const int ncols = min(32, a.N - col0);
                    // static indices only, so vf and packed stay in registers
                    if (ncols == 32 && (o & 15) == 0) {
                        reinterpret_cast<uint4*>(a.out + o)[0] = make_uint4(packed[0], packed[1], packed[2], packed[3]);
                        reinterpret_cast<uint4*>(a.out + o)[1] = make_uint4(packed[4], packed[5], packed[6], packed[7]);
                    } else {
#pragma unroll
                        for (int i = 0; i < 32; ++i)
                            if (i < ncols) a.out[o + i] = (int8_t)(packed[i / 4] >> (8 * (i & 3)));
                    }
                    if (a.acc_out) {
#pragma unroll
                        for (int i = 0; i < 32; ++i)
                            if (i < ncols) a.acc_out[o + i] = __float_as_int(vf[i]);
                    }
                }
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

int sm_count_i8() {
    static int n = 0;
    if (!n) {
        int dev = 0;
        cudaGetDevice(&dev);
        cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev);
        if (n <= 0) n = 148;
    }
    return n;
}

bool s8_map(CUtensorMap* m, const void* base, int rank, const uint64_t* dims, const uint64_t* strides,
            const uint32_t* box) {
    static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
    if (!fn) {
        void* p = nullptr;
        cudaDriverEntryPointQueryResult q;
        if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) != cudaSuccess ||
            q != cudaDriverEntryPointSuccess)
            return false;
        fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(p);
    }
    cuuint64_t d[3], s[2];
    cuuint32_t b[3], e[3] = {1, 1, 1};
    for (int i = 0; i < rank; ++i) {
        d[i] = dims[i];
        b[i] = box[i];
        if (i + 1 < rank) s[i] = strides[i];
    }
    return fn(m, CU_TENSOR_MAP_DATA_TYPE_UINT8, rank, const_cast<void*>(base), d, s, b, e,
              CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
              CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

int launch_int8_tc(const int8_t* x, int x_batched, const int8_t* W, const I8Args& base, cudaStream_t st) {
    I8Args a = base;
    CUtensorMap tx, tw;
    const uint64_t dx[3] = {(uint64_t)a.K, (uint64_t)a.M, (uint64_t)(x_batched ? a.P : 1)};
    const uint64_t sx[2] = {(uint64_t)a.K, (uint64_t)a.M * a.K};
    const uint32_t bx[3] = {I8_BK, I8_BM, 1};
    const uint64_t dw[2] = {(uint64_t)a.N, (uint64_t)a.K};
    const uint64_t sw[1] = {(uint64_t)a.N};
    const uint32_t bw[2] = {128, I8_BK};
    if (!s8_map(&tx, x, 3, dx, sx, bx) || !s8_map(&tw, W, 2, dw, sw, bw))
        return zg::fail(ZG_ERR_CUDA, "int8 tc: tensor maps");
    a.tiles_m = (a.M + I8_BM - 1) / I8_BM;
    a.tiles_n = (a.N + I8_BN - 1) / I8_BN;
    a.x_batched = x_batched;
    if (x_batched) {
        a.chunk = 1;
        a.chunks = a.P;
    } else {
        // a shared input: x.W once per chunk of 16 candidates (the epilogue,
        // which writes the chunk's outputs, outweighs the recomputed GEMM tile)
        a.chunk = a.P < 16 ? a.P : 16;
        a.chunks = (a.P + a.chunk - 1) / a.chunk;
    }
    const int64_t tiles = (int64_t)a.chunks * a.tiles_m * a.tiles_n;
    if (tiles > INT_MAX) return zg::fail(ZG_ERR_INVALID, "int8 tc: too many tiles");
    const int grid = tiles < sm_count_i8() ? (int)tiles : sm_count_i8();
    const size_t smem = I8_SMEM + 1024;
    using Kern = void (*)(const CUtensorMap, const CUtensorMap, const I8Args);
    Kern kern = nullptr;
    const bool p2 = a.y_inv != 0.f;
    switch (a.rank) {
        case 1: kern = p2 ? int8_lut_tc_kernel<1, true> : int8_lut_tc_kernel<1, false>; break;
        case 2: kern = p2 ? int8_lut_tc_kernel<2, true> : int8_lut_tc_kernel<2, false>; break;
        case 4: kern = p2 ? int8_lut_tc_kernel<4, true> : int8_lut_tc_kernel<4, false>; break;
        case 8: kern = p2 ? int8_lut_tc_kernel<8, true> : int8_lut_tc_kernel<8, false>; break;
        case 16: kern = p2 ? int8_lut_tc_kernel<16, true> : int8_lut_tc_kernel<16, false>; break;
        default: return zg::fail(ZG_ERR_INVALID, "int8 tc: rank %d", a.rank);
    }
    if (cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem) != cudaSuccess)
        return zg::fail(ZG_ERR_CUDA, "int8 tc: shared memory attribute");
    zg::LaunchTimer zg_lt_("int8_lut_gemm", st);
    kern<<<grid, I8_THREADS, smem, st>>>(tx, tw, a);
    return zg::check_launch("int8_lut_tc");
}

}  // namespace

namespace zg {
int int8_error_word(int clear) { return ptx_error_word(clear); }
}  // namespace zg

extern "C" size_t zg_int8_lut_linear_workspace_size(int P, int M, int K, int N, int rank, int x_batched) {
    (void)x_batched;
    if (P < 1 || M < 1 || K < 1 || N < 1 || rank < 1) return 0;
    return zg::Carver::need({(size_t)P * K * rank * 4, (size_t)P * rank * N * 4, (size_t)P * M * rank * 4});
}

extern "C" int zg_int8_lut_linear(const int8_t* x, int x_batched, const int8_t* W, const float* w_scale,
                                  float x_scale, float y_scale, const int8_t* lut, const uint32_t* keys,
                                  int group, int P, int M, int K, int N, int rank, float s, int8_t* out,
                                  int32_t* acc_out, void* workspace, size_t workspace_bytes, void* stream) {
    if (P < 1 || P > 65535 || M < 1 || K < 1 || N < 1 || rank < 1 || rank > 64)
        return zg::fail(ZG_ERR_INVALID, "zg_int8_lut_linear: bad sizes");
    if (!x || !W || !w_scale || !lut || !keys || !out)
        return zg::fail(ZG_ERR_INVALID, "zg_int8_lut_linear: null pointer");
    if (!(y_scale > 0.f)) return zg::fail(ZG_ERR_INVALID, "zg_int8_lut_linear: y_scale must be positive");
    size_t need = zg_int8_lut_linear_workspace_size(P, M, K, N, rank, x_batched);
    if (!workspace || workspace_bytes < need)
        return zg::fail(ZG_ERR_WORKSPACE, "zg_int8_lut_linear: workspace %zu < %zu bytes", workspace_bytes, need);
    cudaStream_t st = zg::as_stream(stream);
    zg::Carver cv(workspace, workspace_bytes);
    float* fa = cv.take<float>((size_t)P * K * rank);
    float* fb = cv.take<float>((size_t)P * rank * N);
    float* U = cv.take<float>((size_t)P * M * rank);
    int rc = zg::launch_population_factors(keys, group, P, ZG_MATRIX, K, N, rank, ZG_F32, fa, fb, st);
    if (rc) return rc;
    {
        zg::LaunchTimer zg_lt_("int8_u", st);
        dim3 rgrid((unsigned)((M + U_ROWS - 1) / U_ROWS), P);
        switch (rank) {
            case 1: int8_u_tile_kernel<1><<<rgrid, U_ROWS, 0, st>>>(x, x_batched, fa, M, K, U); break;
            case 2: int8_u_tile_kernel<2><<<rgrid, U_ROWS, 0, st>>>(x, x_batched, fa, M, K, U); break;
            case 4: int8_u_tile_kernel<4><<<rgrid, U_ROWS, 0, st>>>(x, x_batched, fa, M, K, U); break;
            case 8: int8_u_tile_kernel<8><<<rgrid, U_ROWS, 0, st>>>(x, x_batched, fa, M, K, U); break;
            case 16: int8_u_tile_kernel<16><<<rgrid, U_ROWS, 0, st>>>(x, x_batched, fa, M, K, U); break;
            default: {
                int64_t n = (int64_t)M * rank;
                dim3 grid((unsigned)((n + 127) / 128), P);
                int8_u_kernel<<<grid, 128, 0, st>>>(x, x_batched, fa, M, K, rank, U);
            }
        }
        if ((rc = zg::check_launch("int8_u"))) return rc;
    }
    // tensor cores when the TMA layout rules hold (16-byte aligned rows)
    const bool al = (reinterpret_cast<uintptr_t>(x) & 15) == 0 && (reinterpret_cast<uintptr_t>(W) & 15) == 0;
    const bool tc_rank = rank == 1 || rank == 2 || rank == 4 || rank == 8 || rank == 16;
    if (zg::tc_available() && K % 16 == 0 && N % 16 == 0 && tc_rank && al) {
        int e2 = 0;
        const float mant = frexpf(y_scale, &e2);
        const float y_inv = (mant == 0.5f && e2 > -125 && e2 < 126) ? ldexpf(1.f, 1 - e2) : 0.f;
        I8Args a{out, acc_out, w_scale, U, fb, lut, x_scale, y_scale, s, y_inv, M, N, K, P, rank, 0, 0, 0, 0, 0};
        return launch_int8_tc(x, x_batched, W, a, st);
    }
    dim3 grid((N + BN - 1) / BN, (M + BM - 1) / BM, P);
    zg::LaunchTimer zg_lt_("int8_lut_gemm", st);
    int8_lut_simt_kernel<<<grid, THREADS, 0, st>>>(x, x_batched, W, w_scale, x_scale, y_scale, lut, U, fb, rank,
                                                   s, M, K, N, out, acc_out);
    return zg::check_launch("zg_int8_lut_linear");
}
