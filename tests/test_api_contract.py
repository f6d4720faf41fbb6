"""Host-side API contract: the reference's validation errors (no GPU).

Mirrors tests/test_keys.py, test_manifest_validation.py,
test_fitness_and_factors.py, test_optimizer_validation.py and
test_distributed.py of the reference.
"""
import math

import pytest
import torch

import zerograd_b200 as zg
from zerograd_b200 import Manifest, ManifestEntry, ParameterLayout


def _manifest():
    return Manifest(version=1, entries=(
        ManifestEntry(("linear", "weight"), ParameterLayout.MATRIX, "linear"),
        ManifestEntry(("table", "embed"), ParameterLayout.TABLE, "embed"),
        ManifestEntry(("vector", "scale"), ParameterLayout.VECTOR, "scale"),
    ))


class TestStepKey:
    @pytest.mark.parametrize("seed", [1.5, True])
    def test_seed_type(self, seed):
        with pytest.raises(TypeError):
            zg.step_key(seed, "run", 0, 1)

    @pytest.mark.parametrize("run_id", ["", None])
    def test_run_id(self, run_id):
        with pytest.raises(ValueError):
            zg.step_key(42, run_id, 0, 1)

    @pytest.mark.parametrize("gen", [-1, 1.5, True])
    def test_generation(self, gen):
        with pytest.raises(ValueError):
            zg.step_key(42, "run", gen, 1)

    @pytest.mark.parametrize("ver", [0, 1.5])
    def test_version(self, ver):
        with pytest.raises(ValueError):
            zg.step_key(42, "run", 0, ver)

    def test_deterministic_and_distinct(self):
        assert torch.equal(zg.step_key(42, "run", 3, 1), zg.step_key(42, "run", 3, 1))
        assert not torch.equal(zg.step_key(42, "run", 0, 1), zg.step_key(42, "run", 1, 1))
        assert not torch.equal(zg.step_key(42, "run-a", 0, 1), zg.step_key(42, "run-b", 0, 1))
        assert not torch.equal(zg.step_key(42, "run", 0, 1), zg.step_key(43, "run", 0, 1))

    def test_matches_oracle(self, oracle):
        for args in [(0, "bench", 0, 1), (42, "test", 0, 1), (-5, "neg", 7, 3)]:
            assert zg.step_key(*args).tolist() == [int(v) for v in oracle.step_key(*args)]


class TestCandidateKey:
    def test_bool_rejected(self):
        with pytest.raises(TypeError):
            zg.candidate_key(zg.step_key(42, "run", 0, 1), True)

    def test_negative_rejected(self):
        with pytest.raises(ValueError):
            zg.candidate_key(zg.step_key(42, "run", 0, 1), -1)

    def test_non_scalar_rejected(self):
        with pytest.raises(TypeError):
            zg.candidate_key(zg.step_key(42, "run", 0, 1), torch.tensor([1, 2]))

    def test_float_rejected(self):
        with pytest.raises(TypeError):
            zg.candidate_key(zg.step_key(42, "run", 0, 1), torch.tensor(1.0))


class TestManifest:
    def test_entry_validation(self):
        with pytest.raises(ValueError):
            ManifestEntry((), ParameterLayout.MATRIX, "g")
        with pytest.raises(ValueError):
            ManifestEntry(("a", ""), ParameterLayout.MATRIX, "g")
        with pytest.raises(TypeError):
            ManifestEntry(("a",), "matrix", "g")
        with pytest.raises(ValueError):
            ManifestEntry(("a",), ParameterLayout.MATRIX, "")

    def test_manifest_validation(self):
        e = ManifestEntry(("a",), ParameterLayout.MATRIX, "g")
        with pytest.raises(ValueError):
            Manifest(0, (e,))
        with pytest.raises(ValueError):
            Manifest(1, ())
        with pytest.raises(TypeError):
            Manifest(1, ("x",))
        with pytest.raises(ValueError):
            Manifest(1, (e, ManifestEntry(("a",), ParameterLayout.MATRIX, "h")))
        with pytest.raises(ValueError):
            Manifest(1, (e, ManifestEntry(("b",), ParameterLayout.MATRIX, "g")))

    def test_lookup_errors(self):
        m = _manifest()
        assert m.group_index("embed") == 1
        with pytest.raises(KeyError):
            m.entry(("nope",))
        with pytest.raises(KeyError):
            m.group_index("nope")
        with pytest.raises(KeyError):
            m.resolve({"linear": torch.zeros(2)}, ("linear", "weight"))
        with pytest.raises(KeyError):
            m.resolve({}, ("linear", "weight"))
        with pytest.raises(TypeError):
            m.resolve({"linear": {"weight": 3.0}}, ("linear", "weight"))

    def test_validate_ndim(self):
        m = _manifest()
        good = {"linear": {"weight": torch.zeros(8, 4)}, "table": {"embed": torch.zeros(16, 4)},
                "vector": {"scale": torch.zeros(4)}}
        m.validate(good)
        bad = dict(good, vector={"scale": torch.zeros(2, 2)})
        with pytest.raises(ValueError):
            m.validate(bad)


class TestFitness:
    def test_shape_validation(self):
        with pytest.raises(ValueError):
            zg.shape_centered_loss(torch.zeros(2, 2), 0.1)
        with pytest.raises(ValueError):
            zg.shape_centered_loss(torch.zeros(1), 0.1)
        for bad in (0.0, -0.1, math.inf, math.nan, 1):
            with pytest.raises(ValueError):
                zg.shape_centered_loss(torch.zeros(4), bad)
        with pytest.raises(TypeError):
            zg.shape_centered_loss(torch.zeros(4, dtype=torch.int32), 0.1)

    def test_validate_losses(self):
        zg.validate_losses(torch.tensor([1.0, 2.0]))
        with pytest.raises(ValueError):
            zg.validate_losses(torch.zeros(2, 2))
        with pytest.raises(ValueError):
            zg.validate_losses(torch.zeros(1))
        with pytest.raises(TypeError):
            zg.validate_losses(torch.zeros(3, dtype=torch.int64))
        with pytest.raises(ValueError):
            zg.validate_losses(torch.tensor([1.0, float("nan")]))
        with pytest.raises(ValueError):
            zg.validate_losses(torch.tensor([1.0, -float("inf")]))


class TestFactorValidation:
    def test_scaled_factor(self):
        v = zg.scaled_factor(4, 0.2, torch.float32)
        assert float(v) == pytest.approx(0.1)
        for rank in (0, True):
            with pytest.raises(ValueError):
                zg.scaled_factor(rank, 0.1, torch.float32)
        for sigma in (0.0, math.inf, True):
            with pytest.raises(ValueError):
                zg.scaled_factor(2, sigma, torch.float32)

    def test_scaled_factor_bf16_is_rounded(self):
        v = zg.scaled_factor(8, 0.01, torch.bfloat16)
        assert v.dtype == torch.bfloat16
        assert float(v) == float(torch.tensor(0.01 / math.sqrt(8), dtype=torch.float32).to(torch.bfloat16))

    def test_shape_and_rank(self):
        k = zg.step_key(0, "r", 0, 1)
        with pytest.raises(ValueError):
            zg.matrix_factors(k, (4,), 2, dtype=torch.float32)
        with pytest.raises(ValueError):
            zg.matrix_factors(k, (4, 0), 2, dtype=torch.float32)
        with pytest.raises(ValueError):
            zg.matrix_factors(k, (4, 4), 0, dtype=torch.float32)
        with pytest.raises(ValueError):
            zg.table_factors(k, (4, 4, 4), 2, dtype=torch.float32)
        with pytest.raises(ValueError):
            zg.vector_noise(k, (4, 4), dtype=torch.float32)


class TestOptimizerValidation:
    def _opt(self, **kw):
        args = dict(manifest=_manifest(), transform=zg.adamw(0.01), population_size=4, rank=2, sigma=0.1, seed=42,
                    run_id="test")
        args.update(kw)
        return zg.ZeroGrad(**args)

    def test_ctor(self):
        with pytest.raises(TypeError):
            self._opt(manifest="m")
        for pop in (1, True, 2.0):
            with pytest.raises(ValueError):
                self._opt(population_size=pop)
        with pytest.raises(ValueError):
            self._opt(rank=0)
        for sigma in (0.0, 1, math.nan):
            with pytest.raises(ValueError):
                self._opt(sigma=sigma)
        with pytest.raises(TypeError):
            self._opt(seed=1.5)
        with pytest.raises(ValueError):
            self._opt(run_id="")

    def test_properties_and_init(self):
        opt = self._opt()
        assert (opt.population_size, opt.rank, opt.sigma, opt.seed, opt.run_id) == (4, 2, 0.1, 42, "test")
        params = {"linear": {"weight": torch.zeros(8, 4)}, "table": {"embed": torch.zeros(16, 4)},
                  "vector": {"scale": torch.zeros(4)}, "extra": torch.zeros(3)}
        state = opt.init(params)
        assert state.generation == 0
        assert state.opt_state.count == 0

    def test_state_type_checked(self):
        opt = self._opt()
        params = {"linear": {"weight": torch.zeros(8, 4)}, "table": {"embed": torch.zeros(16, 4)},
                  "vector": {"scale": torch.zeros(4)}}
        with pytest.raises(TypeError):
            opt.step_from_losses("state", params, torch.zeros(4))
        with pytest.raises(TypeError):
            opt.step("state", params, None, lambda *a: (0.0, None))

    def test_loss_count_checked_before_any_work(self):
        opt = self._opt()
        params = {"linear": {"weight": torch.zeros(8, 4)}, "table": {"embed": torch.zeros(16, 4)},
                  "vector": {"scale": torch.zeros(4)}}
        state = opt.init(params)
        with pytest.raises(ValueError):
            opt.step_from_losses(state, params, torch.zeros(3))
        with pytest.raises(TypeError):
            opt.step_from_losses(state, params, torch.zeros(4, dtype=torch.int32))


class TestPartition:
    def test_largest_remainder(self):
        assert zg.compute_partition_sizes(10, [1, 4]) == [2, 8]
        assert zg.compute_partition_sizes(7, [1, 1]) == [4, 3]
        assert sum(zg.compute_partition_sizes(101, [0.3, 0.3, 0.4])) == 101
        assert zg.compute_partition_sizes(5, [0, 1]) == [0, 5]

    def test_errors(self):
        with pytest.raises(ValueError):
            zg.compute_partition_sizes(0, [1])
        with pytest.raises(ValueError):
            zg.compute_partition_sizes(4, [])
        with pytest.raises(ValueError):
            zg.compute_partition_sizes(4, [-1, 2])
        with pytest.raises(ValueError):
            zg.compute_partition_sizes(4, [0, 0])

    def test_distributed_ctor_errors(self):
        opt = zg.ZeroGrad(_manifest(), zg.sgd(0.1), 4, 2, 0.1, 0, "r")
        with pytest.raises(ValueError):
            zg.DistributedZeroGrad(opt, [], lambda *a: None)
        with pytest.raises(ValueError):
            zg.DistributedZeroGrad(opt, ["cpu", "cpu"], lambda *a: None, weights=[1.0])
        d = zg.DistributedZeroGrad(opt, ["cpu", "cpu"], lambda *a: None, weights=[1, 3])
        assert d.partition_sizes == [1, 3]
        assert [s.num_candidates for s in d.shards] == [1, 3]
        d.shutdown()
        d.shutdown()
        with pytest.raises(RuntimeError):
            d.step(None, {}, None)


def test_cpu_tensors_fail_loudly():
    """The product path has no CPU fallback."""
    from zerograd_b200._lib import ZgLibraryError

    with pytest.raises(ZgLibraryError):
        zg.perturbed_linear(torch.zeros(2, 4), torch.zeros(4, 3), zg.step_key(0, "r", 0, 1), 2, 0.1)


def test_capture_refusals():
    """A captured generation needs the library's sgd or adamw transform
    (their kernels take the per-step values from device buffers) and CUDA
    parameters; shards need a gather."""
    from zerograd_b200._graph import CapturedGeneration
    from zerograd_b200._lib import ZgLibraryError

    m = _manifest()
    params = {"linear": {"weight": torch.zeros(4, 3)}, "table": {"embed": torch.zeros(5, 3)},
              "vector": {"scale": torch.zeros(3)}}
    loss = lambda p, ctx, batch, rng: (torch.zeros(()), None)  # noqa: E731
    class custom:  # an optax-style transform the graph cannot see into
        def init(self, params):
            return ()

        def update(self, grads, state, params=None):
            return grads, state

    with pytest.raises(NotImplementedError):
        zg.ZeroGrad(m, custom(), 4, 2, 0.1, 0, "r").capture(params, loss, torch.zeros(2, 4))
    with pytest.raises(ZgLibraryError):
        zg.ZeroGrad(m, zg.adamw(1e-3), 4, 2, 0.1, 0, "r").capture(params, loss, torch.zeros(2, 4))
    opt = zg.ZeroGrad(m, zg.sgd(0.1), 4, 2, 0.1, 0, "r")
    with pytest.raises(ZgLibraryError):
        opt.capture(params, loss, torch.zeros(2, 4))
    with pytest.raises(ValueError):
        CapturedGeneration(opt, params, loss, torch.zeros(2, 4), candidate_range=(0, 2))
