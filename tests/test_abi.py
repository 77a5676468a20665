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
    assert lib.mtp_abi_version() == 2


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


def test_new_entry_points_checks_without_launch():
    """Empty sizes return MTP_OK and bad arguments their status, all on the
    host before any CUDA call (this machine has no GPU: a CUDA call would
    surface as MTP_ERR_CUDA) and without launching anything."""
    import _mtp_native as N
    L = N.lib()
    p = ctypes.c_void_p(256)  # never dereferenced: every call below returns before a launch
    before = L.mtp_launch_count()
    OK, SHAPE, DTYPE, ARG = 0, 1, 2, 8
    # tree attention -> RMSNorm -> linear
    assert L.mtp_tree_attn_rmsnorm_linear(p, p, p, 1, None, None, p, 1, None, 0, None, p, 0, 4, 8, 64, 16, 0.1,
                                          1e-6, None, 0, None) == OK
    assert L.mtp_tree_attn_rmsnorm_linear(p, p, p, 1, None, None, p, 1, None, 0, None, p, 2, 4, 8, 9000, 16,
                                          0.1, 1e-6, None, 0, None) == SHAPE  # D above 8192
    assert L.mtp_tree_attn_rmsnorm_linear(p, p, p, 3, None, None, p, 1, None, 0, None, p, 2, 4, 8, 64, 16, 0.1,
                                          1e-6, None, 0, None) == DTYPE  # E4M3 queries
    assert L.mtp_tree_attn_rmsnorm_linear(None, p, p, 1, None, None, p, 1, None, 0, None, p, 2, 4, 8, 64, 16,
                                          0.1, 1e-6, None, 0, None) == ARG
    # paged KV write
    assert L.mtp_paged_kv_write(p, p, 1, p, 64, 8, 16, p, p, 1, 4, None, None, 2, 2, 64, 0, 0, None) == OK
    assert L.mtp_paged_kv_write(p, p, 1, p, 64, 8, 16, p, p, 1, 4, None, None, 2, 2, 64, 62, 4, None) == SHAPE
    assert L.mtp_paged_kv_write(p, p, 1, p, 64, 8, 16, p, p, 1, 4, None, None, 2, 2, 64, 0, 5, None) == SHAPE
    assert L.mtp_paged_kv_write(p, p, 3, p, 64, 8, 16, p, p, 1, 4, None, None, 2, 2, 64, 0, 4, None) == DTYPE
    assert L.mtp_paged_kv_write(None, p, 1, p, 64, 8, 16, p, p, 1, 4, None, None, 2, 2, 64, 0, 4, None) == ARG
    # verify step
    assert L.mtp_verify_step(p, p, p, 0, 4, p, 5, p, None) == OK
    assert L.mtp_verify_step(p, p, p, 2, 4, p, 3, p, None) == SHAPE  # ld < D
    assert L.mtp_verify_step(p, None, p, 2, 4, p, 5, p, None) == ARG
    # FP8-KV attention and INT4 matmul
    assert L.mtp_causal_attention_scaled(p, 1, p, p, 3, None, None, p, 0, 4, 8, 64, 0.1, None) == OK
    assert L.mtp_causal_attention_scaled(p, 3, p, p, 3, None, None, p, 2, 4, 8, 64, 0.1, None) == DTYPE
    assert L.mtp_int4_matmul(p, 1, p, p, 32, p, 1, 0, 16, 64, None) == OK
    assert L.mtp_int4_matmul(p, 1, p, p, 32, p, 1, 2, 16, 63, None) == SHAPE  # K odd
    assert L.mtp_int4_matmul(p, 1, p, p, 0, p, 1, 2, 16, 64, None) == SHAPE  # group 0
    assert L.mtp_int4_matmul(p, 1, None, p, 32, p, 1, 2, 16, 64, None) == ARG
    # fused vocab-parallel verify and the exchange
    assert L.mtp_verify_shard_fused(p, 1, p, 1, None, 0, p, 0, 2, p, p, p, p, 0, 6, 64, 128, 0, p, 256,
                                    None) == OK
    assert L.mtp_verify_shard_fused(p, 1, p, 1, None, 0, p, 2, 2, p, p, p, p, 4, 6, 64, 128, 0, p, 256,
                                    None) == ARG  # rank out of range
    assert L.mtp_verify_fused_bytes(384, 8) >= 2 * 384 * 8 + 2 * 8 * 8 + 8
    assert L.mtp_verify_exchange_bytes(384, 8) == 2 * 8 * 384 * 8 + 2 * 8 * 8
    assert L.mtp_launch_count() == before


def test_key_packing_matches_oracle():
    """The kernels' own key packing (run on the host) equals the oracle's,
    bit for bit, and max over keys is torch.argmax's rule."""
    import numpy as np
    import _mtp_native as N
    from oracle import mtp_oracle as O
    special = np.array([0.0, -0.0, 1.0, -1.0, np.inf, -np.inf, 1e-45, -1e-45, 1.17e-38, -1.17e-38,
                        3.4028235e38, -3.4028235e38, 0.5, 0.5, 2.0, -2.0], dtype=np.float32)
    rng = np.random.default_rng(0)
    vals = np.concatenate([special, rng.standard_normal(5000).astype(np.float32) * 100,
                           rng.integers(-3, 4, 2000).astype(np.float32)])
    idx = rng.integers(0, 2 ** 31, vals.size).astype(np.uint32)
    idx[:16] = np.arange(16, dtype=np.uint32)
    keys = np.empty(vals.size, np.int64)
    assert N.lib().mtp_keys_pack_host(vals.ctypes.data, idx.ctypes.data, keys.ctypes.data, vals.size) == 0
    assert np.array_equal(keys, O.pack_key(vals, idx))
    back = np.empty(vals.size, np.int32)
    assert N.lib().mtp_keys_index_host(keys.ctypes.data, back.ctypes.data, vals.size) == 0
    assert np.array_equal(back, idx.astype(np.int32))
    # argmax rule on a row with ties: the first (lowest-index) maximum wins
    row = rng.integers(-3, 4, 1000).astype(np.float32)
    k = O.pack_key(row, np.arange(row.size, dtype=np.uint32))
    assert int(O.key_index(k.max())) == int(np.argmax(row))
    # value order: keys order like the values (distinct values)
    v = np.unique(rng.standard_normal(300).astype(np.float32))
    kk = O.pack_key(v, np.zeros(v.size, np.uint32))
    assert np.all(np.diff(kk) > 0)


def test_decode_kernel_switch_roundtrip():
    import _mtp_native as N
    before = N.decode_kernel()
    assert before in (1, 2)
    try:
        N.set_decode_kernel(2)
        assert N.decode_kernel() == 2
        N.set_decode_kernel(1)
        assert N.decode_kernel() == 1
        assert N.lib().mtp_set_decode_kernel(0) == 8  # MTP_ERR_ARG
    finally:
        N.set_decode_kernel(before)


def test_c_host_program(tmp_path):
    """A plain C99 program compiled against include/mtp_b200.h alone links
    libmtp_b200.so and drives the entry points that need no GPU
    (tests/c_host/abi_host.c): the header is valid C and the boundary is
    usable without Python."""
    import shutil
    import subprocess
    import _mtp_native as N
    cc = shutil.which("gcc") or shutil.which("cc")
    if cc is None:
        pytest.skip("no C compiler")
    repo = REPO
    N.lib()  # builds the library when it is missing
    libdir = os.path.join(repo, "mtp-engine_b200")
    exe = str(tmp_path / "abi_host")
    r = subprocess.run([cc, "-std=c99", "-Wall", "-Wextra", "-Werror", "-I", os.path.join(repo, "include"),
                        os.path.join(repo, "tests", "c_host", "abi_host.c"), "-L", libdir, "-lmtp_b200",
                        f"-Wl,-rpath,{libdir}", "-o", exe], capture_output=True, text=True, timeout=120)
    assert r.returncode == 0, r.stderr
    r = subprocess.run([exe], capture_output=True, text=True, timeout=120)
    assert r.returncode == 0 and r.stdout.strip() == "ok", r.stdout + r.stderr
