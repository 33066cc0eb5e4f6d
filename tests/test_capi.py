"""The C ABI without a GPU: the library loads, exports every function include/gsn_conv.h declares (and the ctypes
table binds exactly those), and argument validation rejects bad calls before any CUDA work."""
import ctypes
import os
import re
import subprocess

import pytest

from granite_conv_b200 import _lib, build

HEADER = os.path.join(os.path.dirname(os.path.dirname(os.path.abspath(__file__))), "include", "gsn_conv.h")


def _declared():
    src = open(HEADER).read()
    src = re.sub(r"/\*.*?\*/", "", src, flags=re.S)
    return sorted(set(re.findall(r"\b(gsn_[a-z0-9_]+)\s*\(", src)))


def test_library_exports_every_declared_symbol():
    names = _declared()
    assert len(names) >= 15
    L = _lib.lib()
    for n in names:
        assert hasattr(L, n), f"{n} declared in gsn_conv.h but not exported"
    assert sorted(_lib.SIGNATURES) == names
    out = subprocess.run(["nm", "-D", "--defined-only", _lib.library_path()], capture_output=True, text=True).stdout
    exported = set(re.findall(r"\sT\s(gsn_[a-z0-9_]+)", out))
    assert set(names) <= exported


def test_version_and_workspace():
    L = _lib.lib()
    assert L.gsn_version() == 10000
    assert L.gsn_conv_module_workspace_bytes(48, 1536, 1024, 2048) == 48 * 1536 * (2048 * 2 + 2048 * 2)
    assert L.gsn_conv_module_workspace_bytes(0, 10, 1024, 2048) == 0


def test_validation_without_gpu():
    L = _lib.lib()
    p = ctypes.c_void_p(16)
    # kernel size other than 15
    rc = L.gsn_dwconv_silu_bf16(p, p, p, p, 1, 8, 8, 14, 64, 8, 1, 64, 8, 1, None, None)
    assert rc == 2 and "kernel size 14" in _lib.last_error()
    # GEMM shape constraints
    assert L.gsn_gemm1_glu_bf16(p, p, p, p, 128, 100, 4096, None, 0, None) == 2
    assert "multiple of 8" in _lib.last_error()
    assert L.gsn_gemm2_residual_bf16(p, p, p, None, 0, p, 1024, 128, 2048, 1000, None, 0, None) == 2
    assert L.gsn_layernorm_bf16(p, 768, p, p, p, 768, 4, 768, 1e-5, None, 0, None) == 2
    # lengths need T on the 128-frame grid dividing M
    assert L.gsn_gemm1_glu_bf16(p, p, p, p, 200, 1024, 4096, p, 100, None) == 2
    assert "multiple of 128" in _lib.last_error()
    # empty problems succeed without touching the device
    assert L.gsn_dwconv_silu_bf16(None, None, None, None, 0, 8, 8, 15, 0, 0, 0, 0, 0, 0, None, None) == 0
    assert L.gsn_gemm1_glu_bf16(None, None, None, None, 0, 1024, 4096, None, 0, None) == 0
    assert L.gsn_conv_module_bf16(*([None] * 10), 1, None, 0, 16, 1024, 2048, 1e-5, None, 0, None) == 0
    # workspace too small
    rc = L.gsn_conv_module_bf16(*([p] * 10), 1, p, 2, 16, 1024, 2048, 1e-5, p, 100, None)
    assert rc == 5 and "workspace" in _lib.last_error()
    assert L.gsn_interleave_glu_rows(p, p, 100, 8, None) == 2
    assert L.gsn_selftest_bounded_wait(0, None) == 1


def test_ops_refuse_cpu_tensors():
    import torch
    x = torch.zeros(1, 8, 10, dtype=torch.bfloat16)
    w = torch.zeros(8, 1, 15, dtype=torch.bfloat16)
    b = torch.zeros(8, dtype=torch.bfloat16)
    with pytest.raises(Exception):
        torch.ops.granite.dwconv_silu(x, w, b)


def test_build_is_current():
    assert not build.needs_build()


def test_validation_of_fused_and_block_entry_points():
    """The fused up_conv + depthwise kernel, the LayerNorm fold, the feed-forward half and the int8 widening
    reject bad shapes and pointers before any CUDA work; empty problems succeed."""
    L = _lib.lib()
    p = ctypes.c_void_p(256)
    # fused kernel: T must sit on the 128-frame grid, N on the 256-column tile
    assert L.gsn_gemm1_glu_dwconv_bf16(p, p, None, p, p, p, p, 2, 100, 1024, 4096, None, None) == 2
    assert "T % 128" in _lib.last_error()
    assert L.gsn_gemm1_glu_dwconv_bf16(p, p, None, p, p, p, p, 2, 128, 1024, 4000, None, None) == 2
    assert L.gsn_gemm1_glu_dwconv_bf16(None, None, None, None, None, None, None, 0, 128, 1024, 4096, None,
                                       None) == 0
    assert L.gsn_gemm1_glu_dwconv_bf16(None, p, None, p, p, p, p, 2, 128, 1024, 4096, None, None) == 1
    # LayerNorm fold and statistics
    assert L.gsn_fold_layernorm_bf16(p, p, p, p, p, p, p, 4096, 1000, None) == 2
    assert "multiple of 256" in _lib.last_error()
    assert L.gsn_layernorm_stats_bf16(p, 768, p, 4, 768, 1e-5, None, 0, None) == 2
    assert L.gsn_gemm1_lnfold_glu_dwconv_bf16(p, p, p, p, None, p, p, p, 2, 128, 1024, 4096, None, None) == 1
    assert L.gsn_conv_module_lnfold_bf16(*([p] * 8), None, 1, p, 2, 100, 1024, 2048, 1e-5, p, 1 << 30, None) == 2
    assert "multiple of 128" in _lib.last_error()
    # feed-forward half
    assert L.gsn_ff_half_workspace_bytes(2, 128, 1024, 4096) == 2 * 128 * (1024 * 2 + 4096 * 2)
    assert L.gsn_ff_half_bf16(*([p] * 7), None, p, 2, 128, 1024, 4000, 1e-5, p, 1 << 30, None) == 2
    rc = L.gsn_ff_half_bf16(*([p] * 7), None, p, 2, 128, 1024, 4096, 1e-5, p, 100, None)
    assert rc == 5 and "workspace" in _lib.last_error()
    assert L.gsn_gemm_silu_bf16(p, p, p, p, 128, 1001, 4096, None, 0, None) == 2
    assert L.gsn_gemm_residual_scaled_bf16(p, p, p, None, 0, p, 1024, 128, 4096, 1000, 0.5, None, 0, None) == 2
    # int8 widening: sizes must be multiples of 16
    assert L.gsn_widen_i8_bf16(p, p, 17, None, None, 0, None) == 1
    assert L.gsn_widen_i8_bf16(None, None, 0, None, None, 0, None) == 0
    assert L.gsn_conv_module_i8w_workspace_bytes(2, 128, 1024, 2048) == (
        L.gsn_conv_module_workspace_bytes(2, 128, 1024, 2048) + 2 * 2048 * 1024 * 2 + 1024 * 2048 * 2)


def test_validation_of_attention_entry_points():
    """The attention core and the whole attention step reject unsupported shapes (dim_head, context, heads,
    the relative-position table, strides) and small workspaces before any CUDA work; empty problems succeed."""
    L = _lib.lib()
    p = ctypes.c_void_p(256)
    core = L.gsn_attention_core_bf16
    assert core(p, 3072, p, 1025, p, 1024, None, 2, 200, 8, 64, 200, 512, 0.125, None) == 2
    assert "dim_head=64" in _lib.last_error()
    assert core(p, 3072, p, 1025, p, 1024, None, 2, 200, 8, 128, 100, 512, 0.125, None) == 2
    assert core(p, 3072, p, 1025, p, 1024, None, 2, 200, 0, 128, 200, 512, 0.125, None) == 1
    assert core(p, 3072, p, 300, p, 1024, None, 2, 200, 8, 128, 200, 512, 0.125, None) == 1
    assert "n_rel" in _lib.last_error()
    assert core(p, 3071, p, 1025, p, 1024, None, 2, 200, 8, 128, 200, 512, 0.125, None) == 2
    assert core(p, 3072, p, 1025, p, 1000, None, 2, 200, 8, 128, 200, 512, 0.125, None) == 2
    assert core(None, 3072, None, 1025, None, 1024, None, 0, 200, 8, 128, 200, 512, 0.125, None) == 0
    assert core(None, 3072, p, 1025, p, 1024, None, 2, 200, 8, 128, 200, 512, 0.125, None) == 1
    ws = L.gsn_attention_block_workspace_bytes(2, 256, 1024, 8, 128)
    assert ws == 2 * 256 * (1024 * 2 + 3072 * 2 + 1024 * 2)
    blk = L.gsn_attention_block_bf16
    assert blk(p, p, p, 1e-5, p, p, p, p, p, 1025, None, p, 2, 256, 1024, 8, 128, 200, 512, p, 100, None) == 5
    assert "workspace" in _lib.last_error()
    assert blk(p, p, p, 1e-5, p, p, p, p, p, 1025, None, p, 2, 256, 1024, 7, 128, 200, 512, p, ws, None) == 2
    assert blk(p, p, p, 1e-5, p, p, p, p, p, 1025, None, p, 2, 256, 768, 8, 128, 200, 512, p, ws, None) == 2
    assert blk(*([None] * 3), 1e-5, *([None] * 5), 1025, None, None, 0, 256, 1024, 8, 128, 200, 512, None, 0,
               None) == 0


def test_validation_of_ctc_head_entry_points():
    L = _lib.lib()
    p = ctypes.c_void_p(256)
    ws = L.gsn_ctc_selfcond_workspace_bytes(2, 128, 348)
    assert ws == 2 * 128 * (512 * 2 + 384 * 2)
    assert L.gsn_ctc_selfcond_bf16(p, p, p, 600, p, p, None, p, p, 2, 128, 1024, p, ws, None) == 2
    assert L.gsn_ctc_selfcond_bf16(p, p, p, 348, p, p, None, p, p, 2, 128, 1000, p, ws, None) == 2
    assert L.gsn_ctc_selfcond_bf16(p, p, p, 348, p, p, None, p, p, 2, 128, 1024, p, 100, None) == 5
    assert L.gsn_ctc_selfcond_bf16(*([None] * 3), 348, None, None, None, None, None, 0, 128, 1024, None, 0, None) == 0
    assert L.gsn_bpe_pool_bf16(p, p, None, p, p, 2, 128, 1024, 16, 4, None) == 1       # Pp < ceil(T / 4)
    assert L.gsn_bpe_pool_bf16(p, p, None, p, p, 2, 128, 1024, 32, 9, None) == 1       # window too large
    assert L.gsn_bpe_head_workspace_bytes(2, 128) == 2 * 128 * 8
    head = L.gsn_bpe_head_ctc_bf16
    assert head(p, p, p, p, 1000, 7, p, p, p, 2, 128, 1024, p, 4096, None) == 2         # V % 256
    assert head(p, p, p, p, 1024, 7, p, p, p, 2, 100, 1024, p, 4096, None) == 2         # Pp % 128
    assert head(p, p, p, p, 1024, 7, p, p, p, 2, 128, 1024, p, 100, None) == 5
    assert head(None, None, None, None, 1024, 7, None, None, None, 0, 128, 1024, None, 0, None) == 0


def test_selftest_withheld_validation_without_gpu():
    """The unwind-path test entry points check their operands like the entry points they mirror."""
    L = _lib.lib()
    p = ctypes.c_void_p(16)
    assert L.gsn_selftest_gemm_withheld_bf16(p, p, p, p, p, 128, 64, 256, None) == 2
    assert "K=64" in _lib.last_error()
    assert L.gsn_selftest_gemm_withheld_bf16(p, p, p, p, p, 128, 1024, 100, None) == 2     # N % 256
    assert L.gsn_selftest_dwconv_withheld_bf16(p, p, p, p, -1, 8, 8, 64, 8, 1, 64, 8, 1, None) == 1
    assert L.gsn_selftest_gemm_withheld_bf16(None, None, None, None, None, 0, 1024, 1024, None) == 0   # empty


def test_chain_entry_points_validate_without_gpu():
    """The chained-stack entry points reject bad arguments before any CUDA work."""
    L = _lib.lib()
    p = ctypes.c_void_p(256)
    odd = ctypes.c_void_p(260)                     # 4-byte aligned only
    # residual GEMM with row statistics: N must be a multiple of 256, the statistics 8-byte aligned
    assert L.gsn_gemm2_residual_stats_bf16(p, p, p, p, 1024, p, 1024, 128, 2048, 1024, None, 0, None, None) == 1
    assert "null row_partials" in _lib.last_error()
    assert L.gsn_gemm2_residual_stats_bf16(p, p, p, p, 1024, p, 1024, 128, 2048, 1024, None, 0, odd, None) == 2
    assert "8-byte" in _lib.last_error()
    # fused kernel with merged statistics: K % 256 == 0 and K <= 2048
    assert L.gsn_gemm1_lnfold_partials_glu_dwconv_bf16(p, p, p, p, p, 1e-5, p, p, p, 1, 128, 640, 4096, None,
                                                         None) == 2
    assert L.gsn_gemm1_lnfold_partials_glu_dwconv_bf16(p, p, p, p, p, 1e-5, p, p, p, 1, 128, 4096, 4096, None,
                                                         None) == 2
    assert "K <= 2048" in _lib.last_error()
    assert L.gsn_gemm1_lnfold_partials_glu_dwconv_bf16(p, p, p, p, None, 1e-5, p, p, p, 1, 128, 1024, 4096, None,
                                                         None) == 1
    # one chained layer: misaligned statistics, T off the 128 grid, empty problems
    nb = L.gsn_conv_module_workspace_bytes(1, 128, 1024, 2048)
    rc = L.gsn_conv_module_lnfold_chain_bf16(*([p] * 8), None, 1, p, 1, 128, 1024, 2048, 1e-5, odd, None, p, nb,
                                             None)
    assert rc == 2 and "8-byte" in _lib.last_error()
    rc = L.gsn_conv_module_lnfold_chain_bf16(*([p] * 8), None, 1, p, 1, 100, 1024, 2048, 1e-5, None, None, p, nb,
                                             None)
    assert rc == 2 and "multiple of 128" in _lib.last_error()
    assert L.gsn_conv_module_lnfold_chain_bf16(*([None] * 8), None, 1, None, 0, 128, 1024, 2048, 1e-5, None, None,
                                               None, 0, None) == 0
