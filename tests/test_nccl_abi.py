"""The C-ABI NCCL communicator and one-call vocab-parallel verify
(mtp_nccl_*, mtp_vocab_parallel_multi_verify), without a GPU: NCCL is
opened at run time, the process's own NCCL is reused, a missing library is
reported as MTP_ERR_NCCL without affecting the rest of the library, and
arguments are checked before anything is launched.  The collective itself
runs in tests/test_gpu_nccl_abi.py and tests/test_gpu_multi.py.  CPU only."""

import ctypes
import os
import subprocess
import sys

import pytest

import _mtp_native as N

REPO = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
ERR_NCCL, ERR_ARG, ERR_SHAPE, ERR_WS, ERR_ALIGN = 9, 8, 1, 6, 3


def test_status_name_and_id_size():
    assert N.STATUS_NAMES[ERR_NCCL] == "MTP_ERR_NCCL"
    assert N.NCCL_ID_BYTES == 128


def test_nccl_loads_and_reuses_the_process_copy():
    import torch  # noqa: F401  (torch brings its NCCL into the process first)
    v = ctypes.c_int(0)
    st = N.lib().mtp_nccl_version(ctypes.byref(v))
    if st == ERR_NCCL:
        pytest.skip("no NCCL in this image: " + N.lib().mtp_last_error().decode())
    assert st == 0 and v.value >= 21000
    if hasattr(torch.cuda, "nccl") and hasattr(torch.cuda.nccl, "version"):
        try:
            tv = torch.cuda.nccl.version()
        except Exception:  # torch built without NCCL
            tv = None
        if tv is not None:
            code = tv[0] * 10000 + tv[1] * 100 + tv[2] if isinstance(tv, tuple) else int(tv)
            assert v.value == code  # the copy torch loaded, not a second NCCL


def test_unique_id_is_128_fresh_bytes():
    import mtp_parallel as mp
    try:
        a, b = mp.NcclCommunicator.unique_id(), mp.NcclCommunicator.unique_id()
    except RuntimeError as e:
        if "MTP_ERR_NCCL" in str(e):
            pytest.skip(str(e))
        raise
    assert len(a) == 128 and len(b) == 128 and a != b


def test_comm_init_argument_errors():
    L = N.lib()
    c = ctypes.c_void_p()
    uid = ctypes.create_string_buffer(128)
    for rank, world in ((2, 2), (-1, 2), (0, 0)):
        assert L.mtp_nccl_comm_init(ctypes.byref(c), uid, rank, world) == ERR_ARG
        assert not c.value
    assert L.mtp_nccl_comm_init(None, uid, 0, 1) == ERR_ARG
    assert L.mtp_nccl_comm_init(ctypes.byref(c), None, 0, 1) == ERR_ARG
    assert L.mtp_nccl_unique_id(None) == ERR_ARG
    assert L.mtp_nccl_version(None) == ERR_ARG
    assert L.mtp_nccl_comm_status(None) == ERR_ARG
    assert L.mtp_nccl_comm_destroy(None) == 0 and L.mtp_nccl_comm_abort(None) == 0


def test_communicator_rejects_short_id():
    import mtp_parallel as mp
    with pytest.raises(ValueError):
        mp.NcclCommunicator(b"\0" * 64, 0, 1)


def test_workspace_size():
    L = N.lib()
    # no device here, so no stream-K region: the keys alone, in 256-byte units
    assert L.mtp_vocab_parallel_workspace(64, 6, 16032, 4096, N.DT_BF16) == 3072
    assert L.mtp_vocab_parallel_workspace(1, 1, 10, 16, N.DT_BF16) == 256
    assert L.mtp_vocab_parallel_workspace(0, 6, 10, 16, N.DT_BF16) == 256
    assert L.mtp_vocab_parallel_workspace(-1, 6, 10, 16, N.DT_BF16) == 0
    assert L.mtp_vocab_parallel_workspace(4, 0, 10, 16, N.DT_BF16) == 0


def test_verify_checks_before_launch():
    L = N.lib()
    f = L.mtp_vocab_parallel_multi_verify
    ws = ctypes.create_string_buffer(4096 + 16)
    ws_ptr = (ctypes.addressof(ws) + 15) // 16 * 16
    args = lambda B, S, wsp, nbytes, comm=None: (None, N.DT_BF16, None, N.DT_BF16, None, 0, None, None, None, None,
                                                  B, S, 64, 100, 0, comm, wsp, nbytes, None)
    assert f(*args(2, 0, ws_ptr, 4096)) == ERR_SHAPE           # S >= 1
    assert f(*args(0, 6, None, 0)) == 0                        # empty batch: nothing to do
    assert f(*args(64, 6, ws_ptr, 1024)) == ERR_WS             # keys need 3072 bytes
    assert f(*args(2, 6, None, 0)) == ERR_WS
    assert f(*args(2, 6, ws_ptr + 8, 256)) == ERR_ALIGN


def test_missing_library_is_reported_not_fatal():
    """MTP_NCCL_LIBRARY naming a file that does not exist: every NCCL entry
    answers MTP_ERR_NCCL with the loader's reason, and the rest of the
    library still works (a fresh process, since NCCL is opened once)."""
    code = r"""
import ctypes, sys
sys.path.insert(0, sys.argv[1])
import _mtp_native as N
L = N.lib()
v = ctypes.c_int(0)
assert L.mtp_nccl_version(ctypes.byref(v)) == 9, L.mtp_last_error()
msg = L.mtp_last_error().decode()
assert "cannot open NCCL" in msg and "no-such-nccl" in msg, msg
assert L.mtp_nccl_unique_id(ctypes.create_string_buffer(128)) == 9
assert L.mtp_abi_version() >= 1 and L.mtp_gemm_schedule() in (0, 1)
print("ok")
"""
    env = dict(os.environ, MTP_NCCL_LIBRARY="/nonexistent/no-such-nccl.so.2")
    r = subprocess.run([sys.executable, "-c", code, os.path.join(REPO, "mtp-engine_b200")], env=env,
                       capture_output=True, text=True, timeout=300)
    assert r.returncode == 0 and r.stdout.strip().endswith("ok"), r.stdout + r.stderr
