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
