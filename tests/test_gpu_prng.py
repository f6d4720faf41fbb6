"""Device threefry / bits / normals / factors against the oracle (bit-exact bits)."""
import json
import os

import numpy as np
import pytest
import torch

from zerograd_b200 import _ops
from zerograd_b200 import _lib as L

pytestmark = pytest.mark.gpu
GOLDEN = os.path.join(os.path.dirname(__file__), "golden")


def _u32(a, dev):
    return torch.tensor(np.asarray(a, np.int64), dtype=torch.int64).to(torch.uint32).to(dev)


def _np(t):
    return t.cpu().numpy()


def test_threefry_kats_on_device(cuda):
    kat = json.load(open(os.path.join(GOLDEN, "threefry_kat.json")))["threefry2x32_20"]
    keys = _u32([[int(v, 16) for v in r["key"]] for r in kat], cuda)
    ctrs = _u32([[int(v, 16) for v in r["ctr"]] for r in kat], cuda)
    out = torch.empty_like(keys)
    L.call("zg_threefry2x32", L.ptr(keys), L.ptr(ctrs), L.ptr(out), len(kat), L.stream_ptr(cuda))
    assert _np(out).tolist() == [[int(v, 16) for v in r["out"]] for r in kat]


def test_random_threefry_blocks_bit_exact(cuda, oracle):
    rng = np.random.default_rng(1)
    n = 4096
    keys = rng.integers(0, 2**32, (n, 2), dtype=np.uint64)
    ctrs = rng.integers(0, 2**32, (n, 2), dtype=np.uint64)
    out = torch.empty((n, 2), dtype=torch.uint32, device=cuda)
    kd, cd = _u32(keys, cuda), _u32(ctrs, cuda)
    L.call("zg_threefry2x32", L.ptr(kd), L.ptr(cd), L.ptr(out), n, L.stream_ptr(cuda))
    got = _np(out)
    for i in range(0, n, 97):
        assert got[i].tolist() == oracle.threefry(keys[i].astype(np.uint32), int(ctrs[i, 0]), int(ctrs[i, 1])).tolist()


def test_key_chain_matches_golden(cuda):
    g = json.load(open(os.path.join(GOLDEN, "oracle_vectors.json")))
    for ch in g["chains"]:
        base = _u32(ch["base"], cuda)
        ids = torch.tensor(ch["ids"], dtype=torch.int32, device=cuda)
        cks = _ops.launch_fold_in(base.reshape(1, 2), ids)
        assert _np(cks).tolist() == ch["candidate_keys"]
        gks = _ops.launch_fold_in(cks, torch.full((len(ch["ids"]),), ch["group"], dtype=torch.int32, device=cuda))
        assert _np(gks).tolist() == ch["group_keys"]


def test_bits_and_normals_match_golden(cuda):
    g = json.load(open(os.path.join(GOLDEN, "oracle_vectors.json")))
    for s in g["streams"]:
        k = _u32(s["key"], cuda)
        assert _np(_ops.launch_bits(k, 64))[0].tolist() == s["bits"]
        got = _np(_ops.launch_normal(k, 64))[0]
        want = np.array(s["normal_f32_bits"], np.uint32).view(np.float32)
        np.testing.assert_allclose(got, want, rtol=1e-5, atol=1e-6)


def test_long_streams(cuda, oracle):
    """Large flat index ranges, several keys: bits exact, normals within 1e-5."""
    keys = np.array([[0, 0], [0, 42], [0xDEADBEEF, 0x01234567]], np.uint32)
    n = 1 << 20
    bits = _np(_ops.launch_bits(_u32(keys, cuda), n))
    nrm = _np(_ops.launch_normal(_u32(keys, cuda), n))
    for i, k in enumerate(keys):
        np.testing.assert_array_equal(bits[i], oracle.random_bits(k, n))
        want = oracle.normal(k, (n,))
        np.testing.assert_allclose(nrm[i], want, rtol=1e-5, atol=1e-6)
        assert (nrm[i] == want).mean() > 0.99  # same method: nearly all bit-identical


@pytest.mark.parametrize("layout", [0, 1, 2])
@pytest.mark.parametrize("dtype", [torch.float32, torch.bfloat16])
def test_population_factors(cuda, oracle, layout, dtype):
    base = oracle.step_key(42, "test", 0, 1)
    ids = np.arange(6)
    cks = oracle.candidate_keys(base, ids)
    group = 2
    shape = (37, 19) if layout != 2 else (37,)
    rank = 3
    A, B = _ops.launch_factors(_u32(cks, cuda), group, layout, shape, rank, dtype)
    gks = oracle.group_keys(cks, group)
    dname = "float32" if dtype == torch.float32 else "bfloat16"
    OA, OB = oracle.population_factors(gks, layout, shape, rank, dname)
    np.testing.assert_allclose(A.float().cpu().numpy(), OA.reshape(A.shape), rtol=1e-5, atol=1e-6)
    if layout != 2:
        np.testing.assert_allclose(B.float().cpu().numpy(), OB.reshape(B.shape), rtol=1e-5, atol=1e-6)
