"""zg_replay_noalloc: the replay for callers that cannot allocate device memory.

Such callers (a host that fixes the library's device memory at start-up, or a
thread that must not call an allocator) get the replay with its scratch taken
from a buffer built into the library.  Its results must equal zg_replay's
with a caller workspace, call after call, although every call reuses the same
buffer; the second call must not allocate any device memory.
"""
import numpy as np
import pytest
import torch

from zerograd_b200 import _lib as L
from zerograd_b200 import _ops

pytestmark = pytest.mark.gpu

# the tolerance of the float32 parity tests (the reference's rtol/atol 1e-5)
RTOL, ATOL = 1e-5, 1e-5
# the scratch the library holds on a device, and the page rounding of free-memory reports
SCRATCH, SLACK = 16 << 20, 4 << 20
_first_call_done = []


def _keys(oracle, P, dev):
    cks = oracle.candidate_keys(oracle.step_key(3, "noalloc", 0, 1), range(P))
    return torch.tensor(np.asarray(cks, np.int64)).to(torch.uint32).to(dev)


def _noalloc(shaped, cks, group, layout, shape, rank, dtype, out=None):
    dev = shaped.device
    P = cks.shape[0]
    rows, cols = shape[0], (shape[1] if layout != L.ZG_VECTOR else 1)
    r = rank if layout != L.ZG_VECTOR else 1
    if out is None:
        out = torch.empty(tuple(shape), dtype=torch.float32, device=dev)
    inv = _ops.scaled_factor_value(r, 1.0, dtype)
    L.call("zg_replay_noalloc", L.ptr(shaped), L.ptr(cks), group, P, layout, rows, cols, r, inv, L.dtype_code(dtype),
           L.ptr(out), L.stream_ptr(dev))
    return out


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float32])
@pytest.mark.parametrize("layout,shape", [(L.ZG_MATRIX, (512, 384)), (L.ZG_TABLE, (300, 256)), (L.ZG_VECTOR, (999,))])
def test_noalloc_replay_matches_workspace_replay(cuda, oracle, dtype, layout, shape):
    P, rank = 64, 8
    cks = _keys(oracle, P, cuda)
    g = torch.Generator().manual_seed(11)
    for call in range(2):  # two calls in a row share the built-in scratch
        w = torch.randn(P, generator=g).to(cuda)
        want = _ops.launch_replay(w, cks, 2, layout, shape, rank, dtype)  # zg_replay, caller workspace
        got = torch.empty(tuple(shape), dtype=torch.float32, device=cuda)
        torch.cuda.synchronize()
        free_before = torch.cuda.mem_get_info(cuda)[0]
        _noalloc(w, cks, 2, layout, shape, rank, dtype, out=got)
        torch.cuda.synchronize()
        if call == 1:
            assert torch.cuda.mem_get_info(cuda)[0] == free_before
        elif not _first_call_done:
            # the process's first call may load the buffer's module (lazy
            # loading) and so take the built-in scratch, and no more
            assert free_before - torch.cuda.mem_get_info(cuda)[0] <= SCRATCH + SLACK
            _first_call_done.append(True)
        np.testing.assert_allclose(got.cpu().numpy(), want.cpu().numpy(), rtol=RTOL, atol=ATOL)
    assert L.load().zg_device_error(1) == 0


def test_noalloc_rejects_replays_larger_than_its_scratch(cuda, oracle):
    P, rank = 256, 8
    cks = _keys(oracle, P, cuda)
    w = torch.ones(P, device=cuda)
    with pytest.raises(L.ZgLibraryError, match="bytes of scratch"):
        _noalloc(w, cks, 0, L.ZG_MATRIX, (4096, 4096), rank, torch.bfloat16)
