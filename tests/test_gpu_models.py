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
from zerograd_b200 import _ops

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


QAT_SMALL = dict(bench.QAT, dims=(256, 512, 512, 128), batch=64, P=6, chunk=4, run_id="qat-test")


def test_qat_mlp_outputs_bit_exact_against_oracle(cuda, oracle):
    """The integer QAT MLP (quantised masters, three int8 LUT layers, identity
    LUT last) evaluated through CandidateContext.int8_lut_linear in chunks:
    every candidate's int8 outputs equal the oracle's bit for bit, and its
    loss is their mean-square error against the targets."""
    from oracle import qat as oqat

    cfg = QAT_SMALL
    params = bench.tree_to(bench.qat_params_host(cfg), cuda)
    x, target = bench.qat_batch_host(cfg)
    luts = bench.qat_luts()
    dluts = tuple(t.to(cuda) for t in luts)
    inner = bench.make_qat_loss(cfg, dluts)
    opt = zg.ZeroGrad(bench.qat_manifest(cfg), zg.sgd(1e-2), cfg["P"], cfg["rank"], cfg["sigma"], 0, cfg["run_id"],
                      chunk_size=cfg["chunk"])
    manifest = bench.qat_manifest(cfg)
    batch = (x.to(cuda), target.to(cuda))
    n = len(cfg["dims"]) - 1

    def outputs(ck):
        # the last layer's int8 outputs of one candidate, as the loss sees them
        ctx = zg.CandidateContext(manifest, ck, cfg["rank"], cfg["sigma"])
        xx = batch[0]
        for i in range(n):
            wq, ws = zg.quantize_int8_columns(params[f"w{i}"])
            xx = ctx.int8_lut_linear(params, (f"w{i}",), xx, wq, ws, bench.QAT_X_SCALE, bench.QAT_Y_SCALE,
                                     dluts[1] if i == n - 1 else dluts[0])
        return xx

    cks = _ops.launch_fold_in(zg.step_key(0, cfg["run_id"], 1, 1),
                              torch.arange(cfg["P"], dtype=torch.int32, device=cuda))
    seen = [torch.func.vmap(outputs)(cks)]
    got = torch.cat(seen).cpu().numpy()
    losses = opt.evaluate_shard(params, 1, inner, batch, range(cfg["P"])).cpu().numpy()
    base = oracle.step_key(0, cfg["run_id"], 1, 1)
    ws = [params[f"w{i}"].cpu().numpy() for i in range(len(cfg["dims"]) - 1)]
    ys = [bench.QAT_Y_SCALE] * len(ws)
    lut_list = [luts[0].numpy()] * (len(ws) - 1) + [luts[1].numpy()]
    for c, ck in enumerate(oracle.candidate_keys(base, range(cfg["P"]))):
        want = oqat.candidate_outputs(ws, ck, x.numpy(), bench.QAT_X_SCALE, ys, lut_list, cfg["rank"], cfg["sigma"])
        np.testing.assert_array_equal(got[c], want)
        mse = np.mean((want.astype(np.float64) * bench.QAT_Y_SCALE - target.numpy()) ** 2)
        assert losses[c] == pytest.approx(mse, rel=1e-6)
