"""The factor cache's host logic, on the CPU: entries drawn for a
generation's whole population cover any shard of it (a shard's forward
reads its candidates' columns), entries of other generations, shapes,
layouts or smaller populations do not, and a generation's entries are
dropped together."""
import torch

from zerograd_b200._ops import FactorCache


def _cache():
    return FactorCache(budget_bytes=1 << 30)


def _pair(rows, cols, q):
    return (torch.zeros(rows, q), torch.ones(cols, q))


def test_whole_population_entry_covers_its_shards():
    c = _cache()
    full = _pair(64, 32, 256 * 8)
    c.put(((1, 2), 0, 256, 0, 0, 64, 32, 8), full, torch.device("cpu"))
    tail = (0, 0, 64, 32, 8)
    got = c.covering((1, 2), 128, 64, tail)
    assert got is not None and got[0] == 256 and got[1][0] is full[0]
    assert c.covering((1, 2), 0, 256, tail)[0] == 256
    assert c.covering((1, 2), 200, 64, tail) is None      # past the drawn population
    assert c.covering((9, 9), 0, 64, tail) is None         # another generation
    assert c.covering((1, 2), 0, 64, (1, 0, 64, 32, 8)) is None   # another group
    assert c.covering((1, 2), 0, 64, (0, 1, 64, 32, 8)) is None   # another layout
    assert c.covering((1, 2), 0, 64, (0, 0, 64, 32, 16)) is None  # another rank


def test_shard_entries_and_tagged_entries_do_not_cover():
    c = _cache()
    c.put(((1, 2), 64, 64, 0, 0, 64, 32, 8), _pair(64, 32, 512), torch.device("cpu"))   # a shard's own draws
    c.put(((1, 2), 0, 256, 0, 0, 64, 32, 8, "t"), _pair(64, 32, 2048), torch.device("cpu"))  # transposed layout
    assert c.covering((1, 2), 64, 32, (0, 0, 64, 32, 8)) is None
    c.drop_generation((1, 2))
    assert not c._entries and c._bytes == 0


class _PendingEvent:
    """Stands in for a CUDA event whose draws are still running."""

    def query(self):
        return False


def test_covering_skips_pending_entries_for_a_ready_one():
    c = _cache()
    tail = (0, 0, 64, 32, 8)
    pending = _pair(64, 32, 512 * 8)
    ready = _pair(64, 32, 256 * 8)
    c.put(((1, 2), 0, 512, 0, 0, 64, 32, 8), pending, torch.device("cpu"), ready=_PendingEvent())
    c.put(((1, 2), 0, 256, 0, 0, 64, 32, 8), ready, torch.device("cpu"))
    got = c.covering((1, 2), 0, 64, tail)
    assert got is not None and got[0] == 256 and got[1][0] is ready[0]
    # only a pending entry covers: the shard draws its own
    c2 = _cache()
    c2.put(((1, 2), 0, 512, 0, 0, 64, 32, 8), pending, torch.device("cpu"), ready=_PendingEvent())
    assert c2.covering((1, 2), 0, 64, tail) is None


def test_range_buffers_record_drawn_chunks():
    """The factor buffers of an id range are made once; each chunk records
    its draw, and buffers drawn whole cover every chunk and shard."""
    c = _cache()
    made = []

    def make():
        made.append(1)
        return _pair(64, 32, 16 * 8)

    key = ((1, 2), 0, 16, 0, 0, 64, 32, 8, "t")
    val, drawn = c.range_buffers(key, make, torch.device("cpu"))
    assert (0, 4) not in drawn
    drawn.add((0, 4))
    val2, drawn2 = c.range_buffers(key, make, torch.device("cpu"))
    assert val2 is val and (0, 4) in drawn2 and (4, 4) not in drawn2 and len(made) == 1
    assert c.covering_drawn((1, 2), 4, 4, key[3:]) is None  # not drawn whole
    c.mark_drawn(key)
    assert (12, 4) in c.range_buffers(key, make, torch.device("cpu"))[1]
    got = c.covering_drawn((1, 2), 4, 4, key[3:])
    assert got is not None and got[0] == 16
    c.drop_generation((1, 2))
    assert not c._entries and not c._drawn and c._bytes == 0


def test_range_buffers_over_budget_are_not_kept():
    c = FactorCache(budget_bytes=16)
    val, drawn = c.range_buffers(((1, 2), 0, 16, 0, 0, 64, 32, 8), lambda: _pair(64, 32, 16), torch.device("cpu"))
    assert val[0].shape == (64, 16) and drawn == set() and not c._entries


def test_row_pitch_of_fused_projection_views():
    from zerograd_b200._block import _row_pitch

    qkv = torch.zeros(5, 2, 7, 3, 4, 64)          # [P, B, S, 3, H, D]
    q, k, v = qkv[..., 0, :, :], qkv[..., 1, :, :], qkv[..., 2, :, :]
    assert _row_pitch(q) == _row_pitch(k) == _row_pitch(v) == 3 * 4 * 64
    assert _row_pitch(torch.zeros(2, 7, 4, 64)) == 4 * 64
    assert _row_pitch(q.transpose(0, 1)) is None   # leading axes not one run of blocks
    assert _row_pitch(torch.zeros(7, 64, 4).transpose(1, 2)) is None  # heads not contiguous


def test_chunk_size_validation():
    import pytest

    import zerograd_b200 as zg

    m = zg.Manifest(1, (zg.ManifestEntry(("w",), zg.ParameterLayout.MATRIX, "w"),))
    for bad in (0, -2, 1.5, True):
        with pytest.raises(ValueError):
            zg.ZeroGrad(m, zg.sgd(0.1), 8, 4, 0.01, 0, "r", chunk_size=bad)
    assert zg.ZeroGrad(m, zg.sgd(0.1), 8, 4, 0.01, 0, "r", chunk_size=3).chunk_size == 3
