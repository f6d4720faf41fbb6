"""The row-sharded update on one GPU: the completion of each rank of a
two-rank group is run in turn, with the exchange of row blocks done by
copying into one assembled tensor instead of NCCL.  The assembled update
equals the replicated one within float tolerance (a block's GEMM tiles
differ from the whole GEMM's, so the float32 sums round differently); a
block computed with the in-place guarded step equals the same block
computed into a new tensor, and writes nothing when a loss is not finite.
"""
import pytest
import torch

import zerograd_b200 as zg
from zerograd_b200 import _lib as L

pytestmark = pytest.mark.gpu


class _LocalRows:
    """A RowShard stand-in that copies this rank's rows into `into`."""

    def __init__(self, rank, world, into):
        self.rank, self.world, self.into = rank, world, into

    def gather(self, t, r0, r1):
        self.into[r0:r1].copy_(t[r0:r1])


def _problem(dev, rows=1024, cols=512, P=64):
    manifest = zg.Manifest(1, (zg.ManifestEntry(("w",), zg.ParameterLayout.MATRIX, "w"),
                               zg.ManifestEntry(("b",), zg.ParameterLayout.VECTOR, "b")))
    g = torch.Generator().manual_seed(rows + cols)
    params = {"w": (torch.randn(rows, cols, generator=g) * 0.05).to(torch.bfloat16).to(dev),
              "b": (torch.randn(cols, generator=g) * 0.01).to(torch.bfloat16).to(dev)}
    opt = zg.ZeroGrad(manifest, zg.sgd(0.5), P, 8, 0.02, 1, "rows")
    losses = torch.randn(P, generator=g).to(dev)
    return opt, params, losses


@pytest.mark.parametrize("world", [2, 4])
def test_row_blocks_assemble_the_replicated_update(cuda, world):
    opt, params, losses = _problem(cuda)
    state = opt.init(params)
    whole, _, m_whole = opt._complete(state, params, losses)
    assembled = torch.full_like(params["w"], float("nan"))
    for rank in range(world):
        new, _, m = opt._complete(state, params, losses, row_shard=_LocalRows(rank, world, assembled))
        assert torch.equal(new["b"], whole["b"])  # VECTOR leaves stay replicated
        assert torch.equal(m, m_whole)
    assert torch.isfinite(assembled.float()).all()
    a, w = assembled.float(), whole["w"].float()
    torch.testing.assert_close(a, w, rtol=1e-2, atol=1e-3)
    assert (a == w).float().mean().item() > 0.99  # nearly every element rounds to the same bf16
    assert L.load().zg_device_error(1) == 0


def test_row_block_in_place_step_is_guarded(cuda):
    opt, params, losses = _problem(cuda)
    state = opt.init(params)
    blocks = torch.full_like(params["w"], float("nan"))
    opt._complete(state, params, losses, row_shard=_LocalRows(1, 2, blocks))
    inplace = {k: v.clone() for k, v in params.items()}
    unused = torch.empty_like(params["w"])
    opt._complete(state, inplace, losses, inplace=True, row_shard=_LocalRows(1, 2, unused))
    assert torch.equal(inplace["w"][512:], blocks[512:])
    assert torch.equal(inplace["w"][:512], params["w"][:512])  # the other rank's rows are not this rank's to write
    bad = losses.clone()
    bad[3] = float("inf")
    before = inplace["w"].clone()
    opt._complete(state, inplace, bad, inplace=True, row_shard=_LocalRows(1, 2, unused))
    assert torch.equal(inplace["w"], before)
    assert L.load().zg_device_error(1) == 0
