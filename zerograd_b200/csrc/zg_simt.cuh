// zg_simt.cuh -- general-stride CUDA-core GEMM with a low-rank epilogue.
//
// Used for the float32 path (the reference's default dtype, where the
// parity bar is rel 1e-5 and tensor-core TF32 would not meet it) and for
// shapes the tensor-core kernels do not cover.
//
//   C[b,m,n] = alpha * sum_{ko<Ko, ki<Ki} A(b,m,ko,ki) * kscale[ko] * B(b,ko,ki,n)
//            + Cin[b,m,n]                                  (optional, float32)
//            + lr_s * sum_{j<rank} U[b,m,j] * L[b,j,n]      (optional)
//
// The two-level K index lets one launch contract over (candidate, rank)
// pairs of the population factor layouts directly (replay), and the
// epilogue adds the low-rank term s * (x A) B of a perturbed linear.
#pragma once
#include "zg_common.cuh"

namespace zg {

struct SimtGemm {
    const void* A = nullptr;
    int64_t sAb = 0, sAm = 0, sAko = 0, sAki = 0;
    const void* B = nullptr;
    int64_t sBb = 0, sBko = 0, sBki = 0, sBn = 0;
    const float* kscale = nullptr;
    const float* Cin = nullptr;
    int64_t sCinb = 0, sCinm = 0, sCinn = 0;
    const float* U = nullptr;
    int64_t sUb = 0, sUm = 0, sUj = 0;
    const void* L = nullptr;
    int64_t sLb = 0, sLj = 0, sLn = 0;
    int rank = 0;
    float lr_s = 0.f;
    void* C = nullptr;
    int64_t sCb = 0, sCm = 0, sCn = 0;
    int M = 0, N = 0, Ko = 0, Ki = 0, batch = 1;
    float alpha = 1.f;
};

// T: storage type of A, B and L (float or bf16).  TO: storage type of C.
template <typename T, typename TO>
int launch_simt_gemm(const SimtGemm& g, cudaStream_t st, const char* name = "simt_gemm");

// Float32 replay contraction on the CUDA cores, operands K-contiguous:
//   C[m, n] = alpha * sum_k (A[m, k] * w[k / rank]) * B[n, k]
// A [M, K] (row pitch K), B [N, K], C [M, N] float32; K % 4 == 0 and the
// operands 16-byte aligned.  128 x 128 tiles, 8 x 8 outputs per thread, the
// next K tile read into registers while the current one is multiplied; each
// output's sum runs over k in order.
int launch_replay_sgemm(const float* A, const float* B, const float* w, int rank, int M, int N, int64_t K, float alpha,
                        float* C, cudaStream_t st, const char* name = "replay_gemm");

}  // namespace zg
