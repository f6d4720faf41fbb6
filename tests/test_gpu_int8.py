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


def _run_int8(cuda, oracle, P, M, K, N, rank, x_batched, seed, rows=None):
    """Launch on the GPU; compare each candidate (optionally a row subset) with the oracle, bit for bit."""
    from zerograd_b200 import _lib as L

    sigma = 0.05
    rng = np.random.default_rng(seed)
    x = rng.integers(-127, 128, (P, M, K) if x_batched else (M, K), dtype=np.int8)
    W = rng.integers(-127, 128, (K, N), dtype=np.int8)
    w_scale = (rng.uniform(0.5, 1.5, N) / 127).astype(np.float32)
    x_scale, y_scale = 1.0 / 127, 1.0 / 32
    lut = oracle.tanh_lut()
    cks = oracle.candidate_keys(oracle.step_key(seed, "qat", 0, 1), range(P))
    gks = oracle.group_keys(cks, 2)
    L.profile_begin()
    out, acc = _ops.launch_int8_lut_linear(torch.tensor(x).to(cuda), torch.tensor(W).to(cuda),
                                           torch.tensor(w_scale).to(cuda), x_scale, y_scale,
                                           torch.tensor(lut).to(cuda), _u32(cks, cuda), 2, rank, sigma, x_batched,
                                           return_acc=True)
    prof = L.profile_end()
    assert L.load().zg_device_error(1) == 0
    s = np.float32(sigma / np.sqrt(rank))
    sel = slice(None) if rows is None else slice(0, rows)
    for p in range(P):
        A, B = oracle.matrix_factors(gks[p], (K, N), rank)
        xp = (x[p] if x_batched else x)[sel]
        o, a = oracle.int8_lut_linear(xp, W, w_scale, x_scale, y_scale, lut, A, B, float(s))
        np.testing.assert_array_equal(acc[p].cpu().numpy()[sel], a)
        np.testing.assert_array_equal(out[p].cpu().numpy()[sel], o)
    return prof


@pytest.mark.parametrize("P,M,K,N,rank,x_batched", [
    (5, 200, 1024, 528, 4, True),     # several 128-deep K blocks, ragged M and N tiles
    (20, 130, 256, 272, 4, False),    # shared input: candidates in chunks of 16 over one x.W tile
    (3, 64, 512, 256, 8, True),       # rank 8
    (2, 96, 320, 160, 16, False),     # rank 16, K of 2.5 blocks
])
def test_int8_tensor_core_path_bit_exact(cuda, oracle, P, M, K, N, rank, x_batched):
    prof = _run_int8(cuda, oracle, P, M, K, N, rank, x_batched, seed=P + M + K + N)
    assert "int8_lut_gemm" in prof


def test_int8_qat_hidden_layer_size(cuda, oracle):
    """The QAT MLP's 4096 -> 4096 layer with a per-candidate input (batch 512),
    four candidates; the oracle checks the first 48 rows of each bit for bit."""
    _run_int8(cuda, oracle, 4, 512, 4096, 4096, 4, True, seed=7, rows=48)


@pytest.mark.parametrize("y_scale", [1.0 / 32, 0.03, 1e-30])
def test_int8_rounding_and_clamp_edges(cuda, oracle, y_scale):
    """Power-of-two and general output scales, saturation far outside the int8
    range, and non-finite per-channel scales (inf, NaN) quantise exactly as the
    oracle does (a NaN pre-activation maps to 0)."""
    P, M, K, N, rank = 2, 64, 128, 64, 4
    rng = np.random.default_rng(11)
    x = rng.integers(-127, 128, (P, M, K), dtype=np.int8)
    x[:, :, :] = np.where(rng.random((P, M, K)) < 0.05, 0, x)
    W = rng.integers(-127, 128, (K, N), dtype=np.int8)
    W[:, 9] = 0                                          # acc = 0 -> 0 * inf = NaN
    w_scale = (rng.uniform(0.5, 1.5, N) / 127).astype(np.float32)
    w_scale[3], w_scale[5], w_scale[6], w_scale[7], w_scale[9] = np.nan, np.inf, -np.inf, 1e30, np.inf
    lut = oracle.tanh_lut()
    cks = oracle.candidate_keys(oracle.step_key(3, "edges", 0, 1), range(P))
    gks = oracle.group_keys(cks, 0)
    out, acc = _ops.launch_int8_lut_linear(torch.tensor(x).to(cuda), torch.tensor(W).to(cuda),
                                           torch.tensor(w_scale).to(cuda), 1.0 / 127, y_scale,
                                           torch.tensor(lut).to(cuda), _u32(cks, cuda), 0, rank, 0.05, True,
                                           return_acc=True)
    s = np.float32(0.05 / np.sqrt(rank))
    for p in range(P):
        A, B = oracle.matrix_factors(gks[p], (K, N), rank)
        o, a = oracle.int8_lut_linear(x[p], W, w_scale, 1.0 / 127, y_scale, lut, A, B, float(s))
        np.testing.assert_array_equal(acc[p].cpu().numpy(), a)
        np.testing.assert_array_equal(out[p].cpu().numpy(), o)


def test_int8_qat_layer_64_candidates(cuda, oracle):
    """The same layer with 64 candidates (inputs and outputs larger than L2),
    checked on the first 8 rows of candidates 0, 31 and 63."""
    from zerograd_b200 import _lib as L

    P, M, K, N, rank, sigma = 64, 512, 4096, 4096, 4, 0.05
    rng = np.random.default_rng(13)
    x = rng.integers(-127, 128, (P, M, K), dtype=np.int8)
    W = rng.integers(-127, 128, (K, N), dtype=np.int8)
    w_scale = (rng.uniform(0.5, 1.5, N) / 127).astype(np.float32)
    lut = oracle.tanh_lut()
    cks = oracle.candidate_keys(oracle.step_key(13, "qat", 0, 1), range(P))
    gks = oracle.group_keys(cks, 1)
    out = _ops.launch_int8_lut_linear(torch.tensor(x).to(cuda), torch.tensor(W).to(cuda),
                                      torch.tensor(w_scale).to(cuda), 1.0 / 127, 1.0 / 32,
                                      torch.tensor(lut).to(cuda), _u32(cks, cuda), 1, rank, sigma, True)
    assert L.load().zg_device_error(1) == 0
    s = np.float32(sigma / np.sqrt(rank))
    for p in (0, 31, 63):
        A, B = oracle.matrix_factors(gks[p], (K, N), rank)
        o, _ = oracle.int8_lut_linear(x[p][:8], W, w_scale, 1.0 / 127, 1.0 / 32, lut, A, B, float(s))
        np.testing.assert_array_equal(out[p].cpu().numpy()[:8], o)
