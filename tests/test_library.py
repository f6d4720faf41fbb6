"""The C-ABI library loads and exports every symbol include/zg_b200.h declares."""
import ctypes
import os
import re
import subprocess

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def _declared():
    text = open(os.path.join(ROOT, "include", "zg_b200.h")).read()
    return sorted(set(re.findall(r"ZG_API\s+[\w\s\*]+?\b(zg_\w+)\s*\(", text)))


def test_header_declares_entry_points():
    names = _declared()
    assert "zg_perturbed_linear" in names and "zg_replay" in names and len(names) >= 20


def test_library_exports_every_declared_symbol():
    from zerograd_b200 import _lib

    lib = _lib.load()
    for name in _declared():
        assert hasattr(lib, name), name
    out = subprocess.run(["nm", "-D", "--defined-only", _lib.LIB_PATH], capture_output=True, text=True).stdout
    exported = set(re.findall(r" T (zg_\w+)", out))
    assert set(_declared()) <= exported
    # the Python binding covers the whole header
    assert set(_declared()) == set(_lib.SIGNATURES)


def test_library_is_built_for_sm100a():
    from zerograd_b200 import _lib

    out = subprocess.run(["cuobjdump", "--list-elf", _lib.LIB_PATH], capture_output=True, text=True)
    if out.returncode != 0:
        pytest.skip("cuobjdump unavailable")
    assert "sm_100a" in out.stdout


def test_argument_errors_need_no_gpu():
    """Validation happens on the host before any launch."""
    from zerograd_b200 import _lib

    lib = _lib.load()
    assert lib.zg_fold_in(None, 0, None, None, -1, None) == _lib.ZG_ERR_INVALID
    assert b"n < 0" in lib.zg_last_error()
    assert lib.zg_shape_fitness(None, 1, 0.1, None, None, None) == _lib.ZG_ERR_INVALID
    assert lib.zg_perturbed_linear(None, 0, None, None, 0, 0, 1, 1, 1, 1, 0.1, 0, None, None, 0, None) == \
        _lib.ZG_ERR_INVALID
    assert lib.zg_replay(None, None, 0, 4, 7, 4, 4, 2, 1.0, 0, None, None, 0, None) == _lib.ZG_ERR_INVALID
    # block ops: sizes, eps, head dim and row pitch are checked before any launch
    bf = _lib.ZG_BF16
    assert lib.zg_rms_norm(None, 1, None, 1, 0, 1, 8, 1e-6, bf, None, None) == _lib.ZG_ERR_INVALID
    assert b"bad sizes" in lib.zg_last_error()
    assert lib.zg_layer_norm(None, 1, None, None, 1, 1, 1, 8, -1.0, bf, None, None) == _lib.ZG_ERR_INVALID
    assert b"eps" in lib.zg_last_error()
    assert lib.zg_rms_norm(None, 1, None, 1, 2, 0, 8, 1e-6, bf, None, None) == _lib.ZG_OK  # no rows: no work
    assert lib.zg_attention(None, None, None, -1, 4, 2, 64, 1, bf, None, None) == _lib.ZG_ERR_INVALID
    assert lib.zg_attention(None, None, None, 1, 4, 2, 300, 1, bf, None, None) == _lib.ZG_ERR_UNSUPPORTED
    assert lib.zg_attention_ex(None, None, None, 100, 1, 4, 2, 64, 1, bf, None, None) == _lib.ZG_ERR_INVALID
    assert b"row pitch" in lib.zg_last_error()
    assert lib.zg_attention(None, None, None, 0, 4, 2, 64, 1, bf, None, None) == _lib.ZG_OK  # no rows


def test_workspace_queries():
    from zerograd_b200 import _lib

    lib = _lib.load()
    P, M, K, N, r = 256, 256, 4096, 4096, 8
    ws = lib.zg_perturbed_linear_workspace_size(P, M, K, N, r, _lib.ZG_BF16, 0)
    # bf16 factors (A and B) + float32 x@A + float32 shared x@W
    assert ws >= P * r * (K + N) * 2 + P * M * r * 4 + M * N * 4
    assert lib.zg_replay_workspace_size(P, _lib.ZG_MATRIX, K, N, r, _lib.ZG_BF16) >= P * r * (K + N) * 2
    assert lib.zg_perturbed_linear_workspace_size(0, M, K, N, r, 0, 0) == 0
