"""Whole-model generations of the configurations beyond the headline, on
the GPU, against the oracle: the ViT-small workload (the reference
example's ViT, ``examples/train_vit_cifar10.py:137-191``, at reduced size)
and the integer QAT MLP.

Tolerances: losses rel 5e-3 (bf16 activations, float32 cross-entropy);
the int8 path is exact, so its MLP outputs are compared bit for bit."""
import numpy as np
import pytest
import torch

import bench
import zerograd_b200 as zg

pytestmark = pytest.mark.gpu

VIT_SMALL = dict(bench.VIT, layers=2, batch=4, P=4, chunk=2, run_id="vit-test")


def test_vit_generation_matches_oracle(cuda, oracle):
    from oracle import vit as ovit

    cfg = VIT_SMALL
    params = bench.tree_to(bench.vit_params_host(cfg), cuda)
    patches, labels = bench.vit_batch_host(cfg)
    batch = (patches.to(cuda), labels.to(cuda))
    manifest = bench.vit_manifest(cfg)
    opt = zg.ZeroGrad(manifest, zg.sgd(1e-3), cfg["P"], cfg["rank"], cfg["sigma"], 0, cfg["run_id"],
                      chunk_size=cfg["chunk"])
    loss = bench.make_vit_loss(cfg)
    losses = opt.evaluate_shard(params, 2, loss, batch, range(cfg["P"]))

    def host(t):
        return {k: host(v) for k, v in t.items()} if isinstance(t, dict) else t.float().cpu().numpy()

    want = ovit.population_losses(host(params), [e.path for e in manifest.entries],
                                  oracle.step_key(0, cfg["run_id"], 2, 1), range(cfg["P"]), cfg,
                                  patches.float().numpy(), labels.numpy(), cfg["rank"], cfg["sigma"])
    np.testing.assert_allclose(losses.cpu().numpy(), want, rtol=5e-3)
    # the captured generation replays the eager one bit for bit
    cg = opt.capture(params, loss, batch)
    st = opt.init(params)
    got, _, m_c = cg.step(zg.ZeroGradState(5, st.opt_state))
    eager, _, m_e = opt.step(zg.ZeroGradState(5, st.opt_state), params, batch, loss)
    assert m_c.mean_loss == m_e.mean_loss
    for path in [e.path for e in manifest.entries]:
        a, b = got, eager
        for k in path:
            a, b = a[k], b[k]
        assert torch.equal(a, b), path
