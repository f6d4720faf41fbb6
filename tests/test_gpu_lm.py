"""The decoder-LM workload on the GPU: the ops it adds (fused GELU /
residual epilogues, attention over q/k/v views of one fused projection),
chunked population evaluation, and whole generations against the oracle.

The model is ``bench.py``'s (``make_lm_loss``): tied TABLE embedding read
by ``table_lookup`` and the fused tied-logits cross-entropy, RMSNorm scales
as VECTOR entries, fused q/k/v, causal attention, GELU MLP, residuals.
The oracle (``oracle/lm.py``) restates it in float64 with the CUDA path's
bf16 roundings.  Tolerances: bf16 tensors element-wise rel 2e-2 above a
floor of 1e-2 of the output scale (tests/bf16_tol.py); losses (float32
means of float32 cross-entropies over bf16 logits) rel 5e-3; fused vs
unfused and chunked vs whole evaluation bit for bit.
"""
import numpy as np
import pytest
import torch

import bench
import zerograd_b200 as zg
from bf16_tol import assert_bf16_close
from zerograd_b200 import _block
from zerograd_b200 import _ops

pytestmark = pytest.mark.gpu

SMALL = dict(vocab=2048, width=256, layers=2, heads=4, mlp=1024, seq=128, batch=2, P=8, rank=16, sigma=0.01,
             seed=0, run_id="lm-test", lr=1.0, chunk=4)


def _np(t):
    return t.float().cpu().numpy().astype(np.float64)


def _keys(P, gen=0, run="t"):
    base = zg.step_key(0, run, gen, 1)
    return _ops.launch_fold_in(base, torch.arange(P, dtype=torch.int32, device="cuda"))


@pytest.mark.parametrize("act", [None, "gelu"])
@pytest.mark.parametrize("with_res", [False, True])
@pytest.mark.parametrize("M,N", [(300, 384), (512, 2304)])
def test_linear_epilogue_matches_unfused(cuda, act, with_res, M, N):
    """activation / residual in the GEMM epilogue == the separate ops, bit for
    bit (a ragged row block, and whole 256 x 256 tiles)."""
    P, K, r = 6, 256, 16
    g = torch.Generator(device=cuda).manual_seed(1)
    x = torch.randn(P, M, K, generator=g, device=cuda).to(torch.bfloat16)
    W = (torch.randn(K, N, generator=g, device=cuda) * 0.05).to(torch.bfloat16)
    res = torch.randn(P, M, N, generator=g, device=cuda).to(torch.bfloat16) if with_res else None
    keys = _keys(P)
    fused = _ops.launch_linear(x, W, keys, 3, r, 0.01, True, _ops.ACTIVATIONS[act], res)
    want = _ops.launch_linear(x, W, keys, 3, r, 0.01, True)
    if act == "gelu":
        want = zg.gelu(want)
    if with_res:
        want = res + want
    assert torch.equal(fused, want)


def test_linear_output_independent_of_batch_position(cuda):
    """A candidate's output is the same whatever its position in the launch."""
    P, M, K, N, r = 9, 512, 256, 768, 16
    g = torch.Generator(device=cuda).manual_seed(4)
    x = torch.randn(P, M, K, generator=g, device=cuda).to(torch.bfloat16)
    W = (torch.randn(K, N, generator=g, device=cuda) * 0.05).to(torch.bfloat16)
    keys = _keys(P)
    whole = _ops.launch_linear(x, W, keys, 0, r, 0.01, True)
    part = _ops.launch_linear(x[5:], W, keys[5:], 0, r, 0.01, True)
    assert torch.equal(whole[5:], part)


def test_gelu_matches_oracle(cuda, oracle):
    from oracle import lm as olm

    g = torch.Generator(device=cuda).manual_seed(2)
    x = (torch.randn(4096 * 3 + 5, generator=g, device=cuda) * 3)
    for dt in (torch.float32, torch.bfloat16):
        xs = x.to(dt)
        y = zg.gelu(xs)
        want = olm.gelu_tanh(_np(xs))
        if dt == torch.float32:
            np.testing.assert_allclose(_np(y), want, rtol=1e-5, atol=1e-6)
        else:
            assert_bf16_close(_np(y), want, rel=8e-3, floor=1e-3, what="gelu bf16")
    xb = x.to(torch.bfloat16)  # the unaligned scalar path gives the vector path's values
    assert torch.equal(zg.gelu(xb[1:4097]), zg.gelu(xb[1:4097].clone()))


def test_attention_over_fused_qkv_views(cuda, oracle):
    """q, k, v as strided views of one [Z, S, 3, H, D] projection (no copy) ==
    the same attention on contiguous copies; both against the oracle."""
    Z, S, H, D = 6, 200, 3, 64
    g = torch.Generator(device=cuda).manual_seed(3)
    qkv = torch.randn(Z, S, 3, H, D, generator=g, device=cuda).to(torch.bfloat16)
    q, k, v = qkv[:, :, 0], qkv[:, :, 1], qkv[:, :, 2]
    assert _block._row_pitch(q) == 3 * H * D
    for causal in (False, True):
        o_view = zg.attention(q, k, v, causal=causal)
        o_copy = zg.attention(q.contiguous(), k.contiguous(), v.contiguous(), causal=causal)
        assert torch.equal(o_view, o_copy)
        want = oracle.attention(_np(q), _np(k), _np(v), causal=causal)
        # an output is a weighted mean of V rows whose weights are rounded to
        # bf16 (2^-9 relative each) before the P V product, so its error is
        # bounded by the weights' rounding times the V values it averages, not
        # by the (possibly cancelling) result: rel 2^-7 (two bf16 steps) with
        # a floor of max|V|
        assert_bf16_close(_np(o_view), want, rel=2.0 ** -7, floor=float(v.abs().max()),
                          what=f"attention causal={causal}")


def _lm_setup(cfg, dev):
    params = {k: v.to(dev) for k, v in bench.lm_params_host(cfg, cfg["seed"]).items()}
    tokens, labels = (t.to(dev) for t in bench.lm_batch_host(cfg, cfg["seed"]))
    return bench.lm_manifest(cfg), params, (tokens, labels), bench.make_lm_loss(cfg)


def test_chunked_evaluation_matches_whole(cuda):
    """Chunks of 3 (ragged last chunk) give the losses and the update of one
    whole-population evaluation, bit for bit: the chunks draw the range's
    factor buffers once and the replay reads them."""
    cfg = dict(SMALL, P=11)
    manifest, params, batch, loss = _lm_setup(cfg, cuda)
    outs = []
    for chunk in (None, 3):
        _ops.CACHE.clear()
        opt = zg.ZeroGrad(manifest, zg.sgd(0.5), cfg["P"], cfg["rank"], cfg["sigma"], 0, "chunks", chunk_size=chunk)
        st = opt.init(params)
        losses = opt.evaluate_shard(params, 4, loss, batch, range(cfg["P"]))
        new, _, _ = opt.step_from_losses(zg.ZeroGradState(4, st.opt_state), params, losses)
        outs.append((losses, new))
    (l0, p0), (l1, p1) = outs
    assert torch.equal(l0, l1)
    for k in p0:
        assert torch.equal(p0[k], p1[k]), k


def test_reduced_lm_generation_matches_oracle(cuda, oracle):
    """A reduced decoder-LM generation (2 layers, width 256, vocab 2048, P=8,
    rank 16, chunks of 4): losses against the oracle's forward; the SGD
    update (lr 1, so the update dominates the bf16 weights) against the
    oracle's replay of the same losses."""
    from oracle import lm as olm

    cfg = SMALL
    manifest, params, batch, loss = _lm_setup(cfg, cuda)
    opt = zg.ZeroGrad(manifest, zg.sgd(cfg["lr"]), cfg["P"], cfg["rank"], cfg["sigma"], 0, cfg["run_id"],
                      chunk_size=cfg["chunk"])
    st = opt.init(params)
    gen = 3
    losses = opt.evaluate_shard(params, gen, loss, batch, range(cfg["P"]))
    hp = {k: _np(v).astype(np.float32) for k, v in params.items()}
    tokens, labels = (t.cpu().numpy() for t in batch)
    base = oracle.step_key(0, cfg["run_id"], gen, 1)
    entries = bench.lm_entries(cfg)
    want = olm.population_losses(hp, entries, base, range(cfg["P"]), {"layers": cfg["layers"], "heads": cfg["heads"]},
                                 tokens, labels, cfg["rank"], cfg["sigma"])
    np.testing.assert_allclose(losses.cpu().numpy(), want, rtol=5e-3)
    new, st2, metrics = opt.step_from_losses(zg.ZeroGradState(gen, st.opt_state), params, losses)
    shaped = oracle.shape_centered_loss(losses.cpu().numpy().astype(np.float32), cfg["sigma"])
    layouts = bench.lm_layouts(cfg)
    for g, name in enumerate(entries):
        r = cfg["rank"] if layouts[name] != 2 else 1
        descent = oracle.replay_entry(hp[name].shape, layouts[name], base, range(cfg["P"]), shaped, r, g,
                                      "bfloat16")
        # the update is a sum over P*r rank-one terms whose weighted factors
        # are rounded to bf16, so an element's error scales with the terms
        # (about the update's RMS), not with its possibly cancelling sum:
        # element-wise rel 2e-2 with the RMS as floor, and 5e-3 in Frobenius norm
        want_d = cfg["lr"] * descent
        got_d = _np(new[name]) - hp[name].astype(np.float64)
        rms = float(np.sqrt(np.mean(want_d ** 2)))
        assert_bf16_close(got_d, want_d, floor=rms, what=name)
        assert np.linalg.norm(got_d - want_d) <= 5e-3 * np.linalg.norm(want_d), name
    assert st2.generation == gen + 1 and metrics.population_size == cfg["P"]


def test_captured_lm_generation_matches_eager(cuda):
    """ZeroGrad.capture of the chunked LM generation (factors drawn ahead in
    the per-candidate-input layout) replays bit-identical to eager steps,
    including generations out of sequence."""
    cfg = dict(SMALL, lr=1e-3)
    manifest, params, batch, loss = _lm_setup(cfg, cuda)
    opt = zg.ZeroGrad(manifest, zg.sgd(cfg["lr"]), cfg["P"], cfg["rank"], cfg["sigma"], 0, "cap",
                      chunk_size=cfg["chunk"])
    cg = opt.capture(params, loss, batch)
    assert cg._entries and all(len(e) == 6 for e in cg._entries)  # drawn ahead, per-candidate-input layout
    eager = {k: v.clone() for k, v in params.items()}
    st_c = st_e = opt.init(params)
    for gen in (0, 1, 2, 7, 8):
        got, st_c, m_c = cg.step(zg.ZeroGradState(gen, st_c.opt_state))
        eager, st_e, m_e = opt.step(zg.ZeroGradState(gen, st_e.opt_state), eager, batch, loss)
        assert m_c.mean_loss == m_e.mean_loss
        for k in eager:
            assert torch.equal(got[k], eager[k]), (gen, k)


def test_lm_shapes_one_layer_match_oracle(cuda, oracle):
    """The decoder-LM configuration's shapes (vocab 32000, width 768, 12
    heads, MLP 3072, 256-token sequences), one layer, 4 candidates in chunks
    of 2: losses against the oracle."""
    from oracle import lm as olm

    cfg = dict(bench.LM, layers=1, batch=2, P=4, chunk=2, run_id="lm-shape")
    manifest, params, batch, loss = _lm_setup(cfg, cuda)
    opt = zg.ZeroGrad(manifest, zg.sgd(1e-3), cfg["P"], cfg["rank"], cfg["sigma"], 0, cfg["run_id"],
                      chunk_size=cfg["chunk"])
    losses = opt.evaluate_shard(params, 0, loss, batch, range(cfg["P"]))
    hp = {k: _np(v).astype(np.float32) for k, v in params.items()}
    tokens, labels = (t.cpu().numpy() for t in batch)
    base = oracle.step_key(0, cfg["run_id"], 0, 1)
    want = olm.population_losses(hp, bench.lm_entries(cfg), base, range(cfg["P"]),
                                 {"layers": 1, "heads": cfg["heads"]}, tokens, labels, cfg["rank"], cfg["sigma"])
    np.testing.assert_allclose(losses.cpu().numpy(), want, rtol=5e-3)
