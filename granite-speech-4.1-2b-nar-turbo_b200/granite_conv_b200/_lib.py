"""ctypes binding of libgsn_conv.so (the C ABI declared in include/gsn_conv.h).

The library is built ahead of time into ``granite_conv_b200/lib/`` (``granite_conv_b200.build``).  There is no
fallback: if the library is missing or a call returns a non-zero status, a RuntimeError carrying the library's own
message is raised, the way the reference's JIT harness turns CUDA errors into RuntimeError
(``script/cuda_kernels/jit.py:78-92``).
"""
from __future__ import annotations

import ctypes
import os
import threading

from . import build as _build

_vp = ctypes.c_void_p
_i32 = ctypes.c_int
_i64 = ctypes.c_int64
_f32 = ctypes.c_float
_u64 = ctypes.c_uint64
_sz = ctypes.c_size_t
_fp = ctypes.c_void_p     # float* passed as an address

# name -> (restype, argtypes); must list every function of include/gsn_conv.h
SIGNATURES = {
    "gsn_version": (_i32, []),
    "gsn_last_error_string": (ctypes.c_char_p, []),
    "gsn_dwconv_silu_bf16": (_i32, [_vp, _vp, _vp, _vp, _i32, _i32, _i32, _i32,
                                    _i64, _i64, _i64, _i64, _i64, _i64, _vp, _vp]),
    "gsn_dwconv_silu_glu_bf16": (_i32, [_vp, _vp, _vp, _vp, _i32, _i32, _i32, _i32,
                                        _i64, _i64, _i64, _i64, _i64, _i64, _vp, _vp]),
    "gsn_layernorm_bf16": (_i32, [_vp, _i64, _vp, _vp, _vp, _i64, _i32, _i32, _f32, _vp, _i32, _vp]),
    "gsn_gemm1_glu_bf16": (_i32, [_vp, _vp, _fp, _vp, _i32, _i32, _i32, _vp, _i32, _vp]),
    "gsn_gemm1_glu_i8w": (_i32, [_vp, _vp, _fp, _fp, _vp, _i32, _i32, _i32, _vp, _i32, _vp]),
    "gsn_gemm2_residual_bf16": (_i32, [_vp, _vp, _fp, _vp, _i64, _vp, _i64, _i32, _i32, _i32, _vp, _i32, _vp]),
    "gsn_gemm2_residual_i8w": (_i32, [_vp, _vp, _fp, _fp, _vp, _i64, _vp, _i64, _i32, _i32, _i32, _vp, _i32,
                                      _vp]),
    "gsn_gemm1_glu_dwconv_bf16": (_i32, [_vp, _vp, _fp, _fp, _vp, _vp, _vp, _i32, _i32, _i32, _i32, _vp, _vp]),
    "gsn_fold_layernorm_bf16": (_i32, [_vp, _fp, _vp, _vp, _vp, _fp, _fp, _i32, _i32, _vp]),
    "gsn_layernorm_stats_bf16": (_i32, [_vp, _i64, _fp, _i32, _i32, _f32, _vp, _i32, _vp]),
    "gsn_gemm1_lnfold_glu_dwconv_bf16": (_i32, [_vp, _vp, _fp, _fp, _fp, _vp, _vp, _vp, _i32, _i32, _i32, _i32, _vp,
                                                _vp]),
    "gsn_conv_module_lnfold_bf16": (_i32, [_vp, _vp, _fp, _fp, _vp, _vp, _vp, _fp, _vp, _i32, _vp, _i32, _i32, _i32,
                                           _i32, _f32, _vp, _sz, _vp]),
    "gsn_gemm2_residual_stats_bf16": (_i32, [_vp, _vp, _fp, _vp, _i64, _vp, _i64, _i32, _i32, _i32, _vp, _i32, _fp,
                                             _vp]),
    "gsn_gemm1_lnfold_partials_glu_dwconv_bf16": (_i32, [_vp, _vp, _fp, _fp, _fp, _f32, _vp, _vp, _vp, _i32, _i32,
                                                         _i32, _i32, _vp, _vp]),
    "gsn_conv_module_lnfold_chain_bf16": (_i32, [_vp, _vp, _fp, _fp, _vp, _vp, _vp, _fp, _vp, _i32, _vp, _i32, _i32,
                                                 _i32, _i32, _f32, _fp, _fp, _vp, _sz, _vp]),
    "gsn_gemm_silu_bf16": (_i32, [_vp, _vp, _fp, _vp, _i32, _i32, _i32, _vp, _i32, _vp]),
    "gsn_gemm_residual_scaled_bf16": (_i32, [_vp, _vp, _fp, _vp, _i64, _vp, _i64, _i32, _i32, _i32, _f32, _vp, _i32,
                                             _vp]),
    "gsn_ff_half_workspace_bytes": (_sz, [_i32, _i32, _i32, _i32]),
    "gsn_ff_half_bf16": (_i32, [_vp, _vp, _vp, _vp, _fp, _vp, _fp, _vp, _vp, _i32, _i32, _i32, _i32, _f32, _vp, _sz,
                                _vp]),
    "gsn_widen_i8_bf16": (_i32, [_vp, _vp, _i64, _vp, _vp, _i64, _vp]),
    "gsn_attention_core_bf16": (_i32, [_vp, _i64, _vp, _i32, _vp, _i64, _vp, _i32, _i32, _i32, _i32, _i32, _i32,
                                       _f32, _vp]),
    "gsn_attention_block_workspace_bytes": (_sz, [_i32, _i32, _i32, _i32, _i32]),
    "gsn_gemm_linear_bf16": (_i32, [_vp, _vp, _fp, _vp, _i64, _i32, _i32, _i32, _vp, _i32, _vp]),
    "gsn_ctc_selfcond_workspace_bytes": (_sz, [_i32, _i32, _i32]),
    "gsn_ctc_selfcond_bf16": (_i32, [_vp, _vp, _fp, _i32, _vp, _fp, _vp, _vp, _fp, _i32, _i32, _i32, _vp, _sz,
                                     _vp]),
    "gsn_bpe_pool_bf16": (_i32, [_vp, _fp, _vp, _vp, _vp, _i32, _i32, _i32, _i32, _i32, _vp]),
    "gsn_bpe_head_workspace_bytes": (_sz, [_i32, _i32]),
    "gsn_bpe_head_ctc_bf16": (_i32, [_vp, _vp, _vp, _fp, _i32, _i32, _vp, _vp, _vp, _i32, _i32, _i32, _vp, _sz,
                                     _vp]),
    "gsn_attention_block_bf16": (_i32, [_vp, _vp, _vp, _f32, _vp, _fp, _vp, _fp, _vp, _i32, _vp, _vp, _i32, _i32,
                                        _i32, _i32, _i32, _i32, _i32, _vp, _sz, _vp]),
    "gsn_gemm1_glu_bf16s": (_i32, [_vp, _vp, _fp, _fp, _vp, _i32, _i32, _i32, _vp, _i32, _vp]),
    "gsn_gemm2_residual_bf16s": (_i32, [_vp, _vp, _fp, _fp, _vp, _i64, _vp, _i64, _i32, _i32, _i32, _vp, _i32,
                                        _vp]),
    "gsn_conv_module_workspace_bytes": (_sz, [_i32, _i32, _i32, _i32]),
    "gsn_conv_module_i8w_workspace_bytes": (_sz, [_i32, _i32, _i32, _i32]),
    "gsn_conv_module_bf16": (_i32, [_vp, _vp, _vp, _vp, _fp, _vp, _vp, _vp, _fp, _vp, _i32, _vp, _i32,
                                    _i32, _i32, _i32, _f32, _vp, _sz, _vp]),
    "gsn_conv_module_i8w": (_i32, [_vp, _vp, _vp, _vp, _fp, _fp, _vp, _vp, _vp, _fp, _fp, _vp, _i32, _vp,
                                   _i32, _i32, _i32, _i32, _f32, _vp, _sz, _vp]),
    "gsn_conv_module_i8w_widened": (_i32, [_vp, _vp, _vp, _vp, _fp, _fp, _vp, _vp, _vp, _fp, _fp, _vp, _i32, _vp,
                                           _i32, _i32, _i32, _i32, _f32, _vp, _sz, _vp]),
    "gsn_conv_module_w8a8_workspace_bytes": (_sz, [_i32, _i32, _i32, _i32]),
    "gsn_conv_module_w8a8": (_i32, [_vp, _vp, _vp, _vp, _fp, _fp, _vp, _vp, _vp, _fp, _fp, _vp, _i32, _vp,
                                    _i32, _i32, _i32, _i32, _f32, _vp, _sz, _vp]),
    "gsn_quant_rows_bf16": (_i32, [_vp, _i64, _vp, _fp, _i32, _i32, _vp, _i32, _vp]),
    "gsn_conv_module_bf16_noalloc": (_i32, [_vp, _vp, _vp, _vp, _fp, _vp, _vp, _vp, _fp, _vp, _i32, _vp, _i32,
                                            _i32, _i32, _i32, _f32, _vp]),
    "gsn_interleave_glu_rows": (_i32, [_vp, _vp, _i32, _i64, _vp]),
    "gsn_device_status": (_i32, [ctypes.POINTER(_i32), _i32, _vp]),
    "gsn_selftest_bounded_wait": (_i32, [_u64, _vp]),
    "gsn_selftest_gemm_withheld_bf16": (_i32, [_vp, _vp, _fp, _vp, _vp, _i32, _i32, _i32, _vp]),
    "gsn_selftest_dwconv_withheld_bf16": (_i32, [_vp, _vp, _vp, _vp, _i32, _i32, _i32, _i64, _i64, _i64, _i64, _i64,
                                                 _i64, _vp]),
}

_LIB = None
_LOCK = threading.Lock()


def library_path() -> str:
    return os.environ.get("GSN_CONV_LIB", _build.LIB_PATH)


def lib() -> ctypes.CDLL:
    """Load the shared library once and attach the signatures."""
    global _LIB
    if _LIB is not None:
        return _LIB
    with _LOCK:
        if _LIB is None:
            path = library_path()
            if not os.path.exists(path):
                raise RuntimeError(
                    f"libgsn_conv.so is not built ({path}); run `python -m granite_conv_b200.build` "
                    "(there is no CPU or JIT fallback for the conv-module kernels)")
            handle = ctypes.CDLL(path)
            for name, (res, args) in SIGNATURES.items():
                fn = getattr(handle, name)
                fn.restype = res
                fn.argtypes = args
            _LIB = handle
    return _LIB


def last_error() -> str:
    msg = lib().gsn_last_error_string()
    return msg.decode() if msg else ""


def check(rc: int, what: str) -> None:
    if rc != 0:
        raise RuntimeError(f"{what} failed with status {rc}: {last_error()}")


def call(name: str, *args) -> None:
    """Call an int-returning entry point and raise on a non-zero status."""
    check(getattr(lib(), name)(*args), name)


def device_status(stream: int = 0, clear: bool = True) -> int:
    v = _i32(0)
    check(lib().gsn_device_status(ctypes.byref(v), 1 if clear else 0, stream), "gsn_device_status")
    return int(v.value)
