"""Loss-history catch-up and checkpoint resume.

A node that joins late replays the recorded losses generation by generation
(no forward pass) and must hold exactly the parameters of a node that ran
every generation live (the reference's add_node catch-up,
_fault_tolerant.py:148-158); resuming from a checkpoint and catching up the
rest must land on the same bits.
"""
import pytest
import torch

import zerograd_b200 as zg

pytestmark = pytest.mark.gpu


def test_late_node_catches_up_bit_for_bit(cuda, tmp_path):
    P, r, B, K, N = 32, 8, 64, 192, 128
    manifest = zg.Manifest(1, (zg.ManifestEntry(("w",), zg.ParameterLayout.MATRIX, "w"),
                               zg.ManifestEntry(("b",), zg.ParameterLayout.VECTOR, "b")))
    g = torch.Generator().manual_seed(31)
    params0 = {"w": (torch.randn(K, N, generator=g) * 0.05).to(torch.bfloat16).to(cuda),
               "b": torch.zeros(N, dtype=torch.bfloat16, device=cuda)}
    batches = [torch.randn(B, K, generator=g).to(torch.bfloat16).to(cuda) for _ in range(4)]

    def loss_fn(p, ctx, batch, rng):
        y = ctx.linear(p, ("w",), batch) + ctx.vector(p, ("b",))
        return (torch.tanh(y.float()) ** 2).mean(), None

    opt = zg.ZeroGrad(manifest, zg.adamw(3e-3), P, r, 0.02, 5, "catch-up")
    live, state = params0, opt.init(params0)
    history = []
    for gen, batch in enumerate(batches):
        losses = opt.evaluate_shard(live, gen, loss_fn, batch, range(P))
        history.append(losses.cpu())
        live, state, _ = opt.step_from_losses(state, live, losses)
        if gen == 1:
            zg.save_checkpoint(str(tmp_path / "ck.pt"), gen, live, state, extra={"history": list(history)})

    # a node that joins now: seed params + the whole history
    late, late_state, m = opt.catch_up(opt.init(params0), params0, history)
    assert late_state.generation == len(batches) == state.generation
    for k in live:
        assert torch.equal(late[k], live[k]), k
        assert torch.equal(late_state.opt_state.mu[k], state.opt_state.mu[k]), k

    # resume from the generation-1 checkpoint and catch up the remaining generations
    ck = zg.load_checkpoint(str(tmp_path / "ck.pt"))
    resumed, rs, _ = opt.catch_up(ck["state"], ck["params"], history[len(ck["extra"]["history"]):])
    assert rs.generation == state.generation
    for k in live:
        assert torch.equal(resumed[k], live[k]), k
