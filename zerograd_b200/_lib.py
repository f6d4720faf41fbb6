"""ctypes binding of libzgb200 (the C ABI declared in include/zg_b200.h).

The library is the only compute path: if it is missing or a call fails the
error is raised, never papered over with a host fallback.
"""
from __future__ import annotations

import ctypes
import os
import threading

import torch

from ._build import LIB_PATH

ZG_OK, ZG_ERR_INVALID, ZG_ERR_CUDA, ZG_ERR_WORKSPACE, ZG_ERR_UNSUPPORTED = 0, 1, 2, 3, 4
ZG_F32, ZG_BF16 = 0, 1
ZG_MATRIX, ZG_TABLE, ZG_VECTOR = 0, 1, 2
ZG_ACT_NONE, ZG_ACT_GELU = 0, 1

_c = ctypes
_vp, _i32, _i64, _f32, _f64, _sz = _c.c_void_p, _c.c_int, _c.c_int64, _c.c_float, _c.c_double, _c.c_size_t

# name -> (restype, argtypes)
SIGNATURES = {
    "zg_last_error": (_c.c_char_p, []),
    "zg_version": (_c.c_char_p, []),
    "zg_launch_count": (_i64, []),
    "zg_profile_begin": (_i32, [_i32]),
    "zg_profile_end": (_i32, []),
    "zg_profile_summary": (_i32, [_c.c_char_p, _sz]),
    "zg_device_error": (_i32, [_i32]),
    "zg_gemm_bf16": (_i32, [_vp, _i64, _vp, _i64, _i32, _vp, _i64, _i32, _i32, _i32, _i32, _f32, _vp]),
    "zg_threefry2x32": (_i32, [_vp, _vp, _vp, _i64, _vp]),
    "zg_fold_in": (_i32, [_vp, _i32, _vp, _vp, _i64, _vp]),
    "zg_candidate_keys": (_i32, [_c.c_uint32, _c.c_uint32, _vp, _vp, _i64, _vp]),
    "zg_random_bits": (_i32, [_vp, _i64, _i64, _vp, _vp]),
    "zg_normal": (_i32, [_vp, _i64, _i64, _i32, _vp, _vp]),
    "zg_population_factors": (_i32, [_vp, _i32, _i32, _i32, _i64, _i64, _i32, _i32, _vp, _vp, _vp]),
    "zg_factor_operands": (_i32, [_vp, _i32, _i32, _i32, _i64, _i64, _i32, _i32, _vp, _vp, _vp]),
    "zg_factor_operands_t": (_i32, [_vp, _i32, _i32, _i32, _i64, _i64, _i32, _vp, _vp, _i64, _vp]),
    "zg_forward_factors_workspace_size": (_sz, [_i32, _i32, _i32, _i32]),
    "zg_forward_factors_ld": (_i32, [_vp, _vp, _i32, _vp, _i64, _vp, _i64, _i32, _i32, _i32, _i32, _i32, _f32, _vp,
                                     _vp, _sz, _vp]),
    "zg_forward_factors": (_i32, [_vp, _vp, _i32, _vp, _vp, _i32, _i32, _i32, _i32, _i32, _f32, _vp, _vp, _sz,
                                  _vp]),
    "zg_forward_operands": (_i32, [_vp, _vp, _i32, _vp, _i32, _i32, _i32, _i32, _i32, _i32, _f32, _vp, _vp, _vp,
                                   _vp, _sz, _vp]),
    "zg_replay_factors_workspace_size": (_sz, [_i32, _i64, _i64, _i32]),
    "zg_replay_factors": (_i32, [_vp, _vp, _vp, _i32, _i64, _i64, _i32, _f32, _vp, _vp, _sz, _vp]),
    "zg_replay_operands_workspace_size": (_sz, [_i32, _i64, _i64, _i32]),
    "zg_replay_operands": (_i32, [_vp, _vp, _i32, _vp, _i32, _i32, _i64, _i64, _i32, _f32, _vp, _vp, _sz, _vp]),
    "zg_replay_sgd": (_i32, [_vp, _vp, _i32, _vp, _i32, _i32, _i64, _i64, _i32, _f32, _vp, _vp, _i32, _f64, _vp,
                             _vp, _vp, _sz, _vp]),
    "zg_replay_adamw": (_i32, [_vp, _vp, _i32, _vp, _i32, _i32, _i64, _i64, _i32, _f32, _vp, _vp, _i32, _vp, _vp,
                               _vp, _vp, _i32, _f64, _f64, _f64, _f64, _f64, _vp, _vp, _vp, _vp, _sz, _vp]),
    "zg_replay_split_count": (_i32, [_i32, _i32]),
    "zg_replay_partials_workspace_size": (_sz, [_i32, _i64, _i64, _i32]),
    "zg_replay_partials": (_i32, [_vp, _vp, _i32, _vp, _i32, _i32, _i64, _i64, _i32, _i32, _i32, _vp, _i64, _vp, _sz,
                                  _vp]),
    "zg_replay_split_sum": (_i32, [_vp, _vp, _i32, _i64, _f32, _vp, _vp]),
    "zg_replay_split_sgd": (_i32, [_vp, _vp, _i32, _i64, _f32, _vp, _vp, _i32, _f64, _vp, _vp]),
    "zg_tied_logits_ce_workspace_size": (_sz, [_i32, _i32, _i32, _i32, _i32]),
    "zg_tied_logits_ce": (_i32, [_vp, _i32, _vp, _vp, _i32, _vp, _i32, _i32, _i32, _i32, _i32, _f32, _vp, _vp, _sz,
                                 _vp]),
    "zg_batched_forward_workspace_size": (_sz, [_i32, _i32, _i32, _i32, _i32]),
    "zg_batched_forward_factors": (_i32, [_vp, _vp, _i32, _vp, _vp, _i32, _i32, _i32, _i32, _i32, _f32, _vp, _vp,
                                          _sz, _vp]),
    "zg_batched_forward_operands": (_i32, [_vp, _vp, _i32, _vp, _i32, _i32, _i32, _i32, _i32, _i32, _f32, _vp, _vp,
                                           _vp, _vp, _sz, _vp]),
    "zg_batched_forward_ex": (_i32, [_vp, _vp, _i32, _vp, _i32, _i32, _i32, _i32, _i32, _i32, _f32, _vp, _vp, _i64,
                                     _i32, _i32, _vp, _vp, _vp, _sz, _vp]),
    "zg_tied_logits_ce_ex_workspace_size": (_sz, [_i32, _i32, _i32, _i32, _i32]),
    "zg_tied_logits_ce_ex": (_i32, [_vp, _i32, _vp, _vp, _i32, _vp, _i32, _i32, _i32, _i32, _i32, _f32, _vp, _vp,
                                    _i64, _i32, _vp, _vp, _sz, _vp]),
    "zg_attention_ex": (_i32, [_vp, _vp, _vp, _i64, _i32, _i32, _i32, _i32, _i32, _i32, _vp, _vp]),
    "zg_gelu": (_i32, [_vp, _vp, _i64, _i32, _vp]),
    "zg_perturbed_linear_workspace_size":(_sz, [_i32, _i32, _i32, _i32, _i32, _i32, _i32]),
    "zg_perturbed_linear": (_i32, [_vp, _i32, _vp, _vp, _i32, _i32, _i32, _i32, _i32, _i32, _f32, _i32,
                                   _vp, _vp, _sz, _vp]),
    "zg_table_lookup_workspace_size": (_sz, [_i32, _i64, _i64, _i64, _i32, _i32]),
    "zg_table_lookup": (_i32, [_vp, _vp, _i32, _i64, _vp, _i32, _i32, _i64, _i64, _i32, _f32, _i32, _vp,
                               _vp, _sz, _vp]),
    "zg_tied_logits_workspace_size": (_sz, [_i32, _i32, _i32, _i32, _i32, _i32, _i32]),
    "zg_tied_logits": (_i32, [_vp, _i32, _vp, _vp, _i32, _i32, _i32, _i32, _i32, _i32, _f32, _i32, _vp,
                              _vp, _sz, _vp]),
    "zg_perturbed_vector": (_i32, [_vp, _i32, _vp, _i32, _i32, _i64, _f32, _i32, _vp, _vp]),
    "zg_shape_fitness": (_i32, [_vp, _i32, _f64, _vp, _vp, _vp]),
    "zg_row_mean": (_i32, [_vp, _i64, _i64, _vp, _vp]),
    "zg_replay_workspace_size": (_sz, [_i32, _i32, _i64, _i64, _i32, _i32]),
    "zg_replay": (_i32, [_vp, _vp, _i32, _i32, _i32, _i64, _i64, _i32, _f32, _i32, _vp, _vp, _sz, _vp]),
    "zg_replay_noalloc": (_i32, [_vp, _vp, _i32, _i32, _i32, _i64, _i64, _i32, _f32, _i32, _vp, _vp]),
    "zg_adamw_update": (_i32, [_vp, _vp, _i32, _vp, _vp, _vp, _vp, _vp, _i64, _i32, _f64, _f64, _f64, _f64,
                               _f64, _vp, _vp]),
    "zg_adam_bias_corrections": (_i32, [_i32, _f64, _f64, _vp]),
    "zg_sgd_update": (_i32, [_vp, _vp, _i32, _vp, _i64, _f64, _vp]),
    "zg_copy_if_zero": (_i32, [_vp, _vp, _sz, _vp, _vp]),
    "zg_layer_norm": (_i32, [_vp, _i32, _vp, _vp, _i32, _i32, _i64, _i32, _f32, _i32, _vp, _vp]),
    "zg_rms_norm": (_i32, [_vp, _i32, _vp, _i32, _i32, _i64, _i32, _f32, _i32, _vp, _vp]),
    "zg_attention": (_i32, [_vp, _vp, _vp, _i32, _i32, _i32, _i32, _i32, _i32, _vp, _vp]),
    "zg_int8_lut_linear_workspace_size": (_sz, [_i32, _i32, _i32, _i32, _i32, _i32]),
    "zg_int8_lut_linear": (_i32, [_vp, _i32, _vp, _vp, _f32, _f32, _vp, _vp, _i32, _i32, _i32, _i32, _i32,
                                  _i32, _f32, _vp, _vp, _vp, _sz, _vp]),
}

_lock = threading.Lock()
_lib = None


class ZgLibraryError(RuntimeError):
    """libzgb200 is missing, failed to load, or a kernel launch failed."""


def load():
    """Load libzgb200.so (built in-tree by zerograd_b200._build)."""
    global _lib
    if _lib is not None:
        return _lib
    with _lock:
        if _lib is None:
            if not os.path.exists(LIB_PATH):
                raise ZgLibraryError(
                    f"{LIB_PATH} is not built; run `python -m zerograd_b200._build` "
                    "(nvcc for sm_100a). There is no CPU fallback.")
            lib = ctypes.CDLL(LIB_PATH)
            for name, (res, args) in SIGNATURES.items():
                fn = getattr(lib, name)
                fn.restype = res
                fn.argtypes = args
            _lib = lib
    return _lib


def call(name: str, *args):
    """Call an int-returning entry point and raise on a non-zero status."""
    lib = load()
    rc = getattr(lib, name)(*args)
    if rc != ZG_OK:
        msg = lib.zg_last_error().decode(errors="replace")
        if rc == ZG_ERR_INVALID:
            raise ValueError(msg)
        raise ZgLibraryError(f"{name} failed ({rc}): {msg}")


def launch_count() -> int:
    """Kernels this library has launched since it was loaded."""
    return int(load().zg_launch_count())


def profile_begin(max_records: int = 65536) -> None:
    call("zg_profile_begin", max_records)


def profile_end() -> dict:
    """Stops profiling; returns {kernel name: (launches, total_ms)} (synchronises on the events)."""
    call("zg_profile_end")
    buf = ctypes.create_string_buffer(1 << 16)
    call("zg_profile_summary", buf, len(buf))
    out = {}
    for line in buf.value.decode().splitlines():
        name, n, ms = line.rsplit(",", 2)
        out[name] = (int(n), float(ms))
    return out


def query(name: str, *args) -> int:
    return int(getattr(load(), name)(*args))


def ptr(t: torch.Tensor | None):
    return None if t is None else ctypes.c_void_p(t.data_ptr())


_raw_stream = getattr(torch._C, "_cuda_getCurrentRawStream", None)


def stream_ptr(device: torch.device) -> ctypes.c_void_p:
    """The current CUDA stream of `device` (raw handle)."""
    if _raw_stream is not None:
        idx = device.index if device.index is not None else torch.cuda.current_device()
        return ctypes.c_void_p(_raw_stream(idx))
    return ctypes.c_void_p(torch.cuda.current_stream(device).cuda_stream)


def dtype_code(dtype: torch.dtype) -> int:
    if dtype == torch.float32:
        return ZG_F32
    if dtype == torch.bfloat16:
        return ZG_BF16
    raise TypeError(f"unsupported dtype {dtype}: the kernels take float32 or bfloat16 leaves")


def require_cuda(*tensors: torch.Tensor) -> torch.device:
    dev = None
    for t in tensors:
        if t is None:
            continue
        if not t.is_cuda:
            raise ZgLibraryError(
                "zerograd_b200 runs on CUDA devices only (got a tensor on "
                f"{t.device}); there is no CPU fallback")
        if dev is None:
            dev = t.device
        elif t.device != dev:
            raise ValueError(f"tensors are on different devices: {dev} and {t.device}")
    return dev


def workspace(nbytes: int, device: torch.device) -> torch.Tensor:
    return torch.empty(max(int(nbytes), 256), dtype=torch.uint8, device=device)
