"""Checkpoint helpers (host side, CPU tensors)."""
import os

import torch

import zerograd_b200 as zg


def test_checkpoint_round_trip_and_atomic_replace(tmp_path):
    path = str(tmp_path / "run" / "ck.pt")
    params = {"w": torch.arange(6.0).reshape(2, 3), "sub": {"b": torch.ones(3, dtype=torch.bfloat16)}}
    state = zg.ZeroGradState(generation=7, opt_state=zg.sgd(0.1).init(params))
    zg.save_checkpoint(path, 7, params, state, extra={"loss_history": [[1.0, 2.0]]})
    zg.save_checkpoint(path, 8, params, state)  # replaces the earlier file
    assert not os.path.exists(path + ".tmp")
    ck = zg.load_checkpoint(path)
    assert ck["step"] == 8 and ck["extra"] is None
    assert ck["state"].generation == 7
    assert torch.equal(ck["params"]["w"], params["w"])
    assert ck["params"]["sub"]["b"].dtype == torch.bfloat16
