// zg_tc.cuh -- tensor-core (tcgen05 / TMEM / TMA) paths for sm_100a.
//
// Each hook returns true when it handled the call (writing its status to
// *rc), false when the shape/dtype is outside what the tensor-core kernel
// covers, in which case the caller uses the CUDA-core path.
#pragma once
#include "zg_common.cuh"

namespace zg {

struct Carver;

// C[M,N] (float32, row-major) = x[M,K] (row-major) @ Wop where Wop(k,n) is
// at W[k*sWk + n*sWn].
template <typename T>
bool tc_dense_gemm_f32out(const void* x, const void* W, int64_t sWk, int64_t sWn, float* C, int M,
                          int K, int N, cudaStream_t st, int* rc);

// Extra workspace bytes the tensor-core replay needs beyond the factor
// buffers (0 when it is not used for this shape).
size_t tc_replay_extra_workspace(int P, int layout, int64_t rows, int64_t cols, int rank, int dtype);

// Full replay of one MATRIX/TABLE entry on the tensor cores.
bool tc_replay(const float* shaped, const uint32_t* keys, int group, int P, int layout, int64_t rows,
               int64_t cols, int rank, float inv_sqrt_rank, int dtype, float* out, void* fa, void* fb,
               Carver& cv, cudaStream_t st, int* rc);

}  // namespace zg
