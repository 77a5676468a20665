"""The C-ABI library loads without a GPU and exports every function that
include/mtp_b200.h declares; host-side argument checks reject bad calls
before any kernel launch.  CPU only (no compute calls)."""

import ctypes
import os
import re

import pytest

from conftest import REPO


def header_functions():
    src = open(os.path.join(REPO, "include", "mtp_b200.h")).read()
    src = re.sub(r"/\*.*?\*/", "", src, flags=re.S)
    return sorted(set(re.findall(r"\b(mtp_[a-z0-9_]+)\s*\(", src)))


def test_header_matches_binding():
    import _mtp_native as N
    assert header_functions() == sorted(N.exported_symbols())


def test_library_exports_all():
    import _mtp_native as N
    lib = N.lib()
    for name in header_functions():
        assert hasattr(lib, name), name
    assert lib.mtp_abi_version() == 1


def test_workspace_sizes():
    import _mtp_native as N
    L = N.lib()
    assert L.mtp_verify_workspace(384) >= 384 * 8 + 8
    assert L.mtp_rmsnorm_linear_workspace(512, 4096, 0) >= 512 * 4
    assert L.mtp_rmsnorm_linear_workspace(512, 4096, 1) >= 512 * 4 + 512 * 4096 * 2
    assert L.mtp_rmsnorm_linear_fp8_workspace(1024, 8192) >= 1024 * 4 + 1024 * 8192


def test_argument_errors_without_launch():
    import _mtp_native as N
    L = N.lib()
    before = L.mtp_launch_count()
    # K = 0, bad dtype, missing workspace, S = 0: all rejected on the host
    st = L.mtp_rmsnorm_linear(None, 1, None, 1, None, 0, None, 0, None, 1, 4, 4, 0, 1e-6, 1.0, None, 0, None)
    assert st == 1 and b"K" in L.mtp_last_error()
    st = L.mtp_rmsnorm_linear(None, 9, None, 1, None, 0, None, 0, None, 1, 4, 4, 4, 1e-6, 1.0, None, 0, None)
    assert st == 2
    st = L.mtp_rmsnorm_linear(ctypes.c_void_p(16), 1, ctypes.c_void_p(16), 1, None, 0, None, 0,
                              ctypes.c_void_p(16), 1, 4, 4, 4, 1e-6, 1.0, None, 0, None)
    assert st == 6
    st = L.mtp_fused_multi_verify(None, 1, None, 1, None, 0, None, None, None, None, 2, 0, 8, 8, None, 0, None)
    assert st == 1
    st = L.mtp_tree_attention_paged(None, None, None, None, 4, 4, None, None, None, None, 1, 1, 2, 6, 4, 8,
                                    4, 4, 1.0, None, 0, None)
    assert st == 1  # Hq not a multiple of Hkv
    assert L.mtp_launch_count() == before


def test_cpu_tensors_rejected():
    torch = pytest.importorskip("torch")
    import mtp_fused_verify
    import mtp_kernels
    with pytest.raises(ValueError, match="CUDA"):
        mtp_kernels.fused_rmsnorm_linear(torch.randn(2, 8), torch.randn(4, 8))
    with pytest.raises(ValueError, match="CUDA"):
        mtp_fused_verify.fused_multi_verify(torch.randn(1, 3, 8), torch.randn(5, 8),
                                            torch.zeros(1, 2, dtype=torch.int32))


def test_out_of_scope_names():
    import mtp_kernels
    with pytest.raises(AttributeError, match="not part of the B200 hot path"):
        mtp_kernels.fused_causal_attention_autotuned  # noqa: B018
    assert mtp_kernels._HAS_TRITON is False


def test_attn_kernel_switch_roundtrip():
    import _mtp_native as N
    before = N.attn_kernel()
    assert before in (1, 2)
    try:
        N.set_attn_kernel(2)
        assert N.attn_kernel() == 2
        N.set_attn_kernel(1)
        assert N.attn_kernel() == 1
        assert N.lib().mtp_set_attn_kernel(3) == 8  # MTP_ERR_ARG
    finally:
        N.set_attn_kernel(before)
