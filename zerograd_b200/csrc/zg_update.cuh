// zg_update.cuh -- element-wise optimizer steps (optax 0.2.8 rules on the
// pseudo-gradient g = -descent, src/zerograd/_optimizer.py:229-234), shared
// by the stand-alone update kernels and the replay GEMM epilogue so that a
// fused replay+update produces exactly the bits of replay followed by update.
#pragma once
#include <math.h>

#include "zg_common.cuh"

namespace zg {

// Constants as the traced float32 computation sees them: Python-float
// expressions rounded once to float32; bias corrections 1 - b^count in
// float32 (optax tree_bias_correction).
struct AdamConsts {
    float omb1, b1, omb2, b2, bc1, bc2, eps, wd, neg_lr;
};

inline AdamConsts adam_consts(int count, double lr, double b1, double b2, double eps, double weight_decay) {
    AdamConsts c;
    c.omb1 = (float)(1.0 - b1);
    c.b1 = (float)b1;
    c.omb2 = (float)(1.0 - b2);
    c.b2 = (float)b2;
    c.bc1 = 1.0f - powf((float)b1, (float)count);
    c.bc2 = 1.0f - powf((float)b2, (float)count);
    c.eps = (float)eps;
    c.wd = (float)weight_decay;
    c.neg_lr = (float)(-lr);
    return c;
}

// The constants with the bias corrections [1 - b1^count, 1 - b2^count] read
// from device memory when `bc` is given (a captured generation writes them
// for each step; adam_consts computes the same floats on the host).
__device__ __forceinline__ AdamConsts adam_consts_dev(AdamConsts c, const float* bc) {
    if (bc) {
        c.bc1 = bc[0];
        c.bc2 = bc[1];
    }
    return c;
}

// optax.adamw on one element: new moments (m, v) and the new parameter.
__device__ __forceinline__ float adamw_step(float p, float g, float mu, float nu, const AdamConsts& c, float& m,
                                           float& v) {
    m = __fadd_rn(__fmul_rn(c.omb1, g), __fmul_rn(c.b1, mu));
    v = __fadd_rn(__fmul_rn(c.omb2, __fmul_rn(g, g)), __fmul_rn(c.b2, nu));
    const float mh = __fdiv_rn(m, c.bc1);
    const float vh = __fdiv_rn(v, c.bc2);
    float u = __fdiv_rn(mh, __fadd_rn(__fsqrt_rn(vh), c.eps));
    u = __fadd_rn(u, __fmul_rn(c.wd, p));
    u = __fmul_rn(u, c.neg_lr);
    return __fadd_rn(p, u);
}

// optax.sgd (no momentum) + apply_updates on one element.
__device__ __forceinline__ float sgd_step(float p, float g, float neg_lr) { return __fadd_rn(p, __fmul_rn(g, neg_lr)); }

// An optimizer step applied where the descent is produced (a GEMM
// epilogue): kind 0 = none, 1 = SGD, 2 = AdamW.  Parameters [rows, cols]
// with row pitch ldp (elements), float32 or bf16; moments float32, same pitch.
enum { ZG_STEP_NONE = 0, ZG_STEP_SGD = 1, ZG_STEP_ADAMW = 2 };
struct FusedStep {
    int kind;
    int param_bf16;
    int64_t ldp;
    const void* param;
    void* param_out;
    const float* mu;
    const float* nu;
    float* mu_out;
    float* nu_out;
    AdamConsts c;        // neg_lr is the SGD rate as well
    const float* guard;  // optional: when *guard != 0 the step writes nothing (in-place updates stay intact)
    const float* bc;     // optional: AdamW bias corrections in device memory (replace c.bc1, c.bc2)
};

}  // namespace zg
