"""Integer QAT linear: int8 GEMM + LUT, bit-exact against the oracle."""
import numpy as np
import pytest
import torch

from zerograd_b200 import _ops

pytestmark = pytest.mark.gpu


def _u32(a, dev):
    return torch.tensor(np.asarray(a, np.int64)).to(torch.uint32).to(dev)


@pytest.mark.parametrize("x_batched", [False, True])
@pytest.mark.parametrize("dims", [(8, 64, 48, 4), (33, 100, 70, 3), (128, 256, 192, 4)])
def test_int8_lut_linear_bit_exact(cuda, oracle, x_batched, dims):
    M, K, N, rank = dims
    P, sigma = 3, 0.05
    rng = np.random.default_rng(M + K)
    x = rng.integers(-127, 128, (P, M, K) if x_batched else (M, K), dtype=np.int8)
    W = rng.integers(-127, 128, (K, N), dtype=np.int8)
    w_scale = (rng.uniform(0.5, 1.5, N) / 127).astype(np.float32)
    x_scale, y_scale = 1.0 / 127, 1.0 / 32
    lut = oracle.tanh_lut()
    base = oracle.step_key(0, "qat", 0, 1)
    cks = oracle.candidate_keys(base, range(P))
    gks = oracle.group_keys(cks, 1)
    out, acc = _ops.launch_int8_lut_linear(torch.tensor(x).to(cuda), torch.tensor(W).to(cuda),
                                           torch.tensor(w_scale).to(cuda), x_scale, y_scale,
                                           torch.tensor(lut).to(cuda), _u32(cks, cuda), 1, rank, sigma, x_batched,
                                           return_acc=True)
    s = np.float32(sigma / np.sqrt(rank))
    for p in range(P):
        A, B = oracle.matrix_factors(gks[p], (K, N), rank)
        o, a = oracle.int8_lut_linear(x[p] if x_batched else x, W, w_scale, x_scale, y_scale, lut, A, B, float(s))
        np.testing.assert_array_equal(acc[p].cpu().numpy(), a)
        np.testing.assert_array_equal(out[p].cpu().numpy(), o)
