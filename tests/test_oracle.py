"""The oracle pinned against published known answers (CPU only)."""
import json
import os
import zlib

import numpy as np
import pytest

GOLDEN = os.path.join(os.path.dirname(__file__), "golden")


def _h(s):
    return int(s, 16)


def test_threefry_known_answers(oracle):
    kat = json.load(open(os.path.join(GOLDEN, "threefry_kat.json")))
    for row in kat["threefry2x32_20"]:
        k = np.array([_h(v) for v in row["key"]], np.uint32)
        out = oracle.threefry(k, _h(row["ctr"][0]), _h(row["ctr"][1]))
        assert [int(v) for v in out] == [_h(v) for v in row["out"]]


def test_partitionable_split_matches_jax(oracle):
    kat = json.load(open(os.path.join(GOLDEN, "threefry_kat.json")))["split_key0"]
    got = oracle.split(np.array(kat["key"], np.uint32), kat["num"])
    assert got.tolist() == kat["out"]


def test_fold_in_is_split_row(oracle):
    k = oracle.key(12345)
    rows = oracle.split(k, 5)
    for i in range(5):
        assert oracle.fold_in(k, i).tolist() == rows[i].tolist()


@pytest.mark.parametrize("payload", [b"", b"a", b"0:bench:1:0", b"42:test:1:0", bytes(range(256))])
def test_crc32_matches_zlib(oracle, payload):
    assert oracle.crc32(payload) == zlib.crc32(payload) & 0xFFFFFFFF


def test_step_key_layout(oracle):
    # jax.random.key(seed) for a 32-bit seed holds the words [0, seed]
    k = oracle.step_key(0, "bench", 0, 1)
    assert int(k[0]) == 0
    assert int(k[1]) == zlib.crc32(b"0:bench:1:0")


def test_bits_are_xor_of_block_words(oracle):
    k = oracle.key(7)
    bits = oracle.random_bits(k, 16)
    for j in range(16):
        o = oracle.threefry(k, 0, j)
        assert int(bits[j]) == int(o[0] ^ o[1])


def test_uniform_edges(oracle):
    L = oracle.lib()
    lo = np.array([0xBF7FFFFF], np.uint32).view(np.float32)[0]
    # bits 0 maps to the lower bound nextafter(-1, 0); all-ones stays below 1
    assert L.zgo_bits_to_normal(0) == pytest.approx(float(np.sqrt(2) * __import__("scipy.special").special.erfinv(float(lo))), rel=1e-5)
    assert np.isfinite(L.zgo_bits_to_normal(0xFFFFFFFF))
    assert abs(L.zgo_bits_to_normal(0x80000000)) < 1e-6


def test_erfinv_accuracy_against_float64(oracle):
    import scipy.special as sp

    xs = np.concatenate([np.linspace(-0.9999, 0.9999, 4001), 1 - np.logspace(-7, -1, 50)]).astype(np.float32)
    f = oracle.lib().zgo_erfinv_f32
    ours = np.array([f(float(x)) for x in xs])
    truth = sp.erfinv(xs.astype(np.float64))
    np.testing.assert_allclose(ours, truth, rtol=1e-5, atol=1e-7)


def test_normal_statistics(oracle):
    n = oracle.normal(oracle.key(0), (1 << 18,))
    assert abs(n.mean()) < 0.01
    assert abs(n.std() - 1.0) < 0.01


def test_golden_oracle_vectors_are_current(oracle):
    g = json.load(open(os.path.join(GOLDEN, "oracle_vectors.json")))
    for row in g["step_keys"]:
        k = oracle.step_key(row["seed"], row["run_id"], row["generation"], row["version"])
        assert [int(v) for v in k] == row["key"]
    for s in g["streams"]:
        k = np.array(s["key"], np.uint32)
        assert oracle.random_bits(k, 64).tolist() == s["bits"]
        assert oracle.normal(k, (64,)).view(np.uint32).tolist() == s["normal_f32_bits"]


def test_factor_layouts(oracle):
    gk = oracle.key(99)
    ka, kb = oracle.split(gk)
    A, B = oracle.matrix_factors(gk, (5, 7), 3)
    assert A.shape == (5, 3) and B.shape == (3, 7)
    np.testing.assert_array_equal(A.ravel(), oracle.normal(ka, (15,)))
    np.testing.assert_array_equal(B.ravel(), oracle.normal(kb, (21,)))
    At, Bt = oracle.table_factors(gk, (5, 7), 3)
    assert At.shape == (5, 3) and Bt.shape == (7, 3)
    np.testing.assert_array_equal(Bt.ravel(), oracle.normal(kb, (21,)))
    # population fill equals per-candidate draws
    gks = np.stack([oracle.key(i) for i in range(4)])
    PA, PB = oracle.population_factors(gks, oracle.MATRIX, (5, 7), 3)
    for i in range(4):
        a, b = oracle.matrix_factors(gks[i], (5, 7), 3)
        np.testing.assert_array_equal(PA[i], a)
        np.testing.assert_array_equal(PB[i], b)


def test_replay_matches_candidate_loop(oracle):
    base = oracle.step_key(42, "test", 0, 1)
    pop, rank, sigma = 8, 2, 0.1
    shaped = oracle.shape_centered_loss(np.arange(pop, dtype=np.float32), sigma)
    got = oracle.replay_entry((8, 4), oracle.MATRIX, base, range(pop), shaped, rank, 0)
    total = np.zeros((8, 4))
    for i in range(pop):
        gk = oracle.fold_in(oracle.fold_in(base, i), 0)
        a, b = oracle.matrix_factors(gk, (8, 4), rank)
        total += shaped[i] * (a.astype(np.float64) @ b)
    np.testing.assert_allclose(got, total * oracle.scaled_factor(rank, 1.0, "float32"), rtol=1e-12)


def test_shaping_sums_to_zero(oracle):
    w = oracle.shape_centered_loss(np.array([1.0, 2.0, 3.0, 10.0]), 0.1)
    assert abs(w.sum()) < 1e-12
    assert w[0] > 0 and w[-1] < 0


def test_int8_oracle_accumulators_exact(oracle):
    rng = np.random.default_rng(0)
    x = rng.integers(-127, 128, (5, 33), dtype=np.int8)
    W = rng.integers(-127, 128, (33, 9), dtype=np.int8)
    A = np.zeros((33, 2), np.float32)
    B = np.zeros((2, 9), np.float32)
    out, acc = oracle.int8_lut_linear(x, W, np.ones(9, np.float32), 1.0, 1.0, oracle.tanh_lut(), A, B, 0.0)
    np.testing.assert_array_equal(acc, x.astype(np.int64) @ W.astype(np.int64))
    q = np.clip(np.rint(acc.astype(np.float32)), -128, 127).astype(np.int64)
    np.testing.assert_array_equal(out, oracle.tanh_lut()[q + 128])
