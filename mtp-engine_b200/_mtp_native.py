"""ctypes binding of libmtp_b200.so (include/mtp_b200.h) plus the host-side
plumbing shared by the drop-in modules: dtype codes, stream handles, cached
per-(device, stream) workspaces and status -> exception mapping.

There is no fallback: if the library is missing or a tensor is not on a CUDA
device, the call raises.
"""

from __future__ import annotations

import ctypes
import os
import threading
from typing import Dict, Optional, Tuple

import torch

_HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(_HERE, "libmtp_b200.so")

DT_F32, DT_BF16, DT_F16, DT_E4M3 = 0, 1, 2, 3
_DTYPE_CODES = {torch.float32: DT_F32, torch.bfloat16: DT_BF16, torch.float16: DT_F16}
if hasattr(torch, "float8_e4m3fn"):
    _DTYPE_CODES[torch.float8_e4m3fn] = DT_E4M3

STATUS_NAMES = {0: "OK", 1: "MTP_ERR_SHAPE", 2: "MTP_ERR_DTYPE", 3: "MTP_ERR_ALIGN", 4: "MTP_ERR_CUDA",
                5: "MTP_ERR_TIMEOUT", 6: "MTP_ERR_WORKSPACE", 7: "MTP_ERR_DEVICE", 8: "MTP_ERR_ARG",
                9: "MTP_ERR_NCCL"}
NCCL_ID_BYTES = 128

_vp, _i, _i64, _f, _sz = ctypes.c_void_p, ctypes.c_int, ctypes.c_int64, ctypes.c_float, ctypes.c_size_t

# name -> (restype, argtypes); mirrors include/mtp_b200.h
SIGNATURES = {
    "mtp_abi_version": (_i, []),
    "mtp_last_error": (ctypes.c_char_p, []),
    "mtp_device_status": (_i, [_vp, ctypes.POINTER(_i), _i]),
    "mtp_rmsnorm_linear_workspace": (_sz, [_i64, _i64, _i]),
    "mtp_rmsnorm_linear": (_i, [_vp, _i, _vp, _i, _vp, _i, _vp, _i, _vp, _i, _i64, _i64, _i64, _f, _f,
                                _vp, _sz, _vp]),
    "mtp_rmsnorm_linear_fp8_workspace": (_sz, [_i64, _i64]),
    "mtp_rmsnorm_linear_fp8": (_i, [_vp, _i, _vp, _vp, _i, _vp, _vp, _i, _vp, _i, _i64, _i64, _i64, _f,
                                    _vp, _sz, _vp]),
    "mtp_tree_attention": (_i, [_vp, _vp, _vp, _vp, _vp, _i, _i64, _i64, _i64, _i64, _f, _vp]),
    "mtp_paged_attention": (_i, [_vp, _vp, _vp, _vp, _vp, _i, _i64, _i64, _i64, _i64, _i64, _i64, _f, _vp]),
    "mtp_causal_attention_scaled": (_i, [_vp, _i, _vp, _vp, _i, _vp, _vp, _vp, _i64, _i64, _i64, _i64, _f, _vp]),
    "mtp_int4_matmul": (_i, [_vp, _i, _vp, _vp, _i64, _vp, _i, _i64, _i64, _i64, _vp]),
    "mtp_tree_attention_paged_workspace": (_sz, [_i64, _i64, _i64, _i64, _i64, _i64]),
    "mtp_tree_attention_paged": (_i, [_vp, _vp, _vp, _vp, _i64, _i64, _vp, _vp, _vp, _vp, _i, _i64, _i64, _i64,
                                      _i64, _i64, _i64, _i64, _f, _vp, _sz, _vp]),
    "mtp_tree_attn_rmsnorm_linear_workspace": (_sz, [_i64, _i64, _i64, _i, _i]),
    "mtp_tree_attn_rmsnorm_linear": (_i, [_vp, _vp, _vp, _i, _vp, _vp, _vp, _i, _vp, _i, _vp, _vp, _i64, _i64,
                                          _i64, _i64, _i64, _f, _f, _vp, _sz, _vp]),
    "mtp_paged_kv_write": (_i, [_vp, _vp, _i, _vp, _i64, _i64, _i64, _vp, _vp, _i, _i64, _vp, _vp, _i64, _i64,
                                _i64, _i64, _i64, _vp]),
    "mtp_verify_workspace": (_sz, [_i64]),
    "mtp_verify_workspace_init": (_i, [_vp, _sz, _vp]),
    "mtp_fused_verify": (_i, [_vp, _i, _vp, _i, _vp, _i, _vp, _vp, _vp, _i64, _i64, _i64, _vp, _sz, _vp]),
    "mtp_fused_multi_verify": (_i, [_vp, _i, _vp, _i, _vp, _i, _vp, _vp, _vp, _vp, _i64, _i64, _i64, _i64,
                                    _vp, _sz, _vp]),
    "mtp_verify_shard_keys": (_i, [_vp, _i, _vp, _i, _vp, _i, _vp, _i64, _i64, _i64, _i64, _vp]),
    "mtp_verify_shard_keys_ws": (_i, [_vp, _i, _vp, _i, _vp, _i, _vp, _i64, _i64, _i64, _i64, _vp, _sz, _vp]),
    "mtp_verify_chain_from_keys": (_i, [_vp, _vp, _vp, _vp, _vp, _i64, _i64, _vp]),
    "mtp_keys_fill": (_i, [_vp, _i64, _vp]),
    "mtp_gemm_tile_plan": (_i, [_i64, _i64, _i, ctypes.POINTER(_i)]),
    "mtp_gemm_tile_check": (_i, [_i64, _i64, _i, ctypes.POINTER(_i64)]),
    "mtp_nccl_version": (_i, [ctypes.POINTER(_i)]),
    "mtp_nccl_unique_id": (_i, [_vp]),
    "mtp_nccl_comm_init": (_i, [ctypes.POINTER(_vp), _vp, _i, _i]),
    "mtp_nccl_comm_destroy": (_i, [_vp]),
    "mtp_nccl_comm_abort": (_i, [_vp]),
    "mtp_nccl_comm_status": (_i, [_vp]),
    "mtp_vocab_parallel_workspace": (_sz, [_i64, _i64, _i64, _i64, _i]),
    "mtp_vocab_parallel_multi_verify": (_i, [_vp, _i, _vp, _i, _vp, _i, _vp, _vp, _vp, _vp, _i64, _i64, _i64,
                                             _i64, _i64, _vp, _vp, _sz, _vp]),
    "mtp_verify_step": (_i, [_vp, _vp, _vp, _i64, _i64, _vp, _i64, _vp, _vp]),
    "mtp_verify_fused_bytes": (_sz, [_i64, _i]),
    "mtp_verify_fused_init": (_i, [_vp, _i64, _i, _vp]),
    "mtp_verify_shard_fused": (_i, [_vp, _i, _vp, _i, _vp, _i, _vp, _i, _i, _vp, _vp, _vp, _vp, _i64, _i64, _i64,
                                    _i64, _i64, _vp, _sz, _vp]),
    "mtp_verify_exchange_bytes": (_sz, [_i64, _i]),
    "mtp_verify_exchange_chain": (_i, [_vp, _vp, _i, _i, _vp, _vp, _vp, _vp, _vp, _i64, _i64, _vp]),
    "mtp_set_gemm_schedule": (_i, [_i]),
    "mtp_gemm_schedule": (_i, []),
    "mtp_set_decode_kernel": (_i, [_i]),
    "mtp_decode_kernel": (_i, []),
    "mtp_gemm_streamk_bytes": (_sz, [_i64, _i64, _i64, _i]),
    "mtp_gemm_streamk_plan": (_i, [_i64, _i64, _i64, _i, _i, _i, ctypes.POINTER(_i64)]),
    "mtp_gemm_streamk_check": (_i, [_i64, _i64, _i64, _i, _i, _i]),
    "mtp_gemm_test_streamk": (_i, [_vp, _vp, _i, _vp, _i64, _i64, _i64, _i, _vp, _sz, _vp]),
    "mtp_keys_pack_host": (_i, [_vp, _vp, _vp, _i64]),
    "mtp_keys_index_host": (_i, [_vp, _vp, _i64]),
    "mtp_launch_count": (ctypes.c_uint64, []),
    "mtp_gemm_test": (_i, [_vp, _vp, _i, _vp, _i64, _i64, _i64, _i, _vp]),
    "mtp_fused_multi_verify_noalloc": (_i, [_vp, _i, _vp, _i, _vp, _i, _vp, _vp, _vp, _vp, _i64, _i64, _i64,
                                            _i64, _vp]),
}

_lib = None
_lib_lock = threading.Lock()


def lib() -> ctypes.CDLL:
    """Load libmtp_b200.so (once).  Raises if it was not built."""
    global _lib
    if _lib is None:
        with _lib_lock:
            if _lib is None:
                if not os.path.exists(LIB_PATH):
                    raise RuntimeError(
                        f"{LIB_PATH} is missing: build it with `python mtp-engine_b200/_build.py` "
                        "(this package has no CPU or Triton fallback)")
                L = ctypes.CDLL(LIB_PATH)
                for name, (res, args) in SIGNATURES.items():
                    fn = getattr(L, name)
                    fn.restype = res
                    fn.argtypes = args
                if os.environ.get("MTP_GEMM_STREAMK") == "1":  # before any workspace exists
                    L.mtp_set_gemm_schedule(1)
                _lib = L
    return _lib


class MTPError(RuntimeError):
    pass


def check(status: int, what: str) -> None:
    if status != 0:
        msg = lib().mtp_last_error().decode(errors="replace")
        raise MTPError(f"{what} failed with {STATUS_NAMES.get(status, status)}: {msg}")


def dtype_code(t: torch.Tensor) -> int:
    try:
        return _DTYPE_CODES[t.dtype]
    except KeyError:
        raise TypeError(f"unsupported dtype {t.dtype}") from None


def ptr(t: Optional[torch.Tensor]):
    """Device address of t (None for NULL); the bound argtypes take plain ints."""
    return None if t is None else t.data_ptr()


def require_cuda(*tensors: Optional[torch.Tensor]) -> torch.device:
    dev = None
    for t in tensors:
        if t is None:
            continue
        if not t.is_cuda:
            raise ValueError("mtp-engine-b200 operators run on CUDA tensors only "
                             f"(got a tensor on {t.device}); there is no CPU fallback")
        if dev is None:
            dev = t.device
        elif t.device != dev:
            raise ValueError(f"tensors on different devices: {dev} vs {t.device}")
    if dev is None:
        raise ValueError("no tensor given")
    return dev


_raw_stream = getattr(torch._C, "_cuda_getCurrentRawStream", None)


def stream_handle(device: torch.device):
    """The current torch stream of `device` as a cudaStream_t value (without
    building a torch Stream object on every call)."""
    idx = device.index if device.index is not None else torch.cuda.current_device()
    if _raw_stream is not None:
        return _raw_stream(idx)
    return torch.cuda.current_stream(device).cuda_stream


# --------------------------------------------------------------------------- #
# workspaces: one set per (device, stream); calls on one stream are ordered,
# so reusing the buffer across calls on that stream is race-free.
# --------------------------------------------------------------------------- #
_ws: Dict[Tuple[int, int, str], torch.Tensor] = {}
_ws_lock = threading.Lock()


def workspace(device: torch.device, name: str, nbytes: int, init=None) -> torch.Tensor:
    """Cached uint8 device buffer of at least `nbytes`.  `init(buf)` runs
    (on the current stream) whenever a new buffer is allocated."""
    nbytes = max(int(nbytes), 256)
    stream = torch.cuda.current_stream(device).cuda_stream
    key = (device.index if device.index is not None else torch.cuda.current_device(), stream, name)
    with _ws_lock:
        buf = _ws.get(key)
        if buf is None or buf.numel() < nbytes:
            buf = torch.empty(nbytes, dtype=torch.uint8, device=device)
            if init is not None:
                init(buf)
            _ws[key] = buf
    return buf


def drop_workspace(device: torch.device, name: str) -> None:
    stream = torch.cuda.current_stream(device).cuda_stream
    key = (device.index if device.index is not None else torch.cuda.current_device(), stream, name)
    with _ws_lock:
        _ws.pop(key, None)


# --------------------------------------------------------------------------- #
# GEMM schedule (stream-K needs room in the workspace, see include/mtp_b200.h)
# --------------------------------------------------------------------------- #
STREAMK_TAIL = 16640  # MTP_STREAMK_TAIL_BYTES: counters + the final 256 bytes
_GEMM_WS = ("rmsnorm_linear", "rmsnorm_linear_fp8", "tree_attn_rmsnorm_linear")


def _rest_fill(device: torch.device):
    """Workspace init: every 8-byte word INT64_MIN (the stream-K counters'
    resting value; the rest of an RMSNorm-linear workspace is overwritten by
    every call)."""
    def _init(buf):
        check(lib().mtp_keys_fill(ptr(buf), buf.numel() // 8, stream_handle(device)), "mtp_keys_fill")
    return _init


def gemm_schedule() -> int:
    return int(lib().mtp_gemm_schedule())


def set_gemm_schedule(mode: int) -> None:
    """0 = data-parallel tiles, 1 = stream-K where it is faster.  Cached
    RMSNorm-linear workspaces are dropped: one used under schedule 0 may have
    overwritten the counter tail."""
    check(lib().mtp_set_gemm_schedule(int(mode)), "mtp_set_gemm_schedule")
    with _ws_lock:
        for key in [k for k in _ws if k[2] in _GEMM_WS]:
            del _ws[key]


def decode_kernel() -> int:
    return int(lib().mtp_decode_kernel())


def set_decode_kernel(version: int) -> None:
    """Single-query attention kernel: 1 = one warp per key, 2 = 16-byte loads
    with several keys in flight (16-bit K/V, power-of-two head size <= 256)."""
    check(lib().mtp_set_decode_kernel(int(version)), "mtp_set_decode_kernel")


def streamk_bytes(M: int, N: int, K: int, ab_code: int) -> int:
    if gemm_schedule() != 1:
        return 0
    return int(lib().mtp_gemm_streamk_bytes(int(M), int(N), int(K), int(ab_code)))


def gemm_workspace(device: torch.device, name: str, base: int, M: int, N: int, K: int,
                   ab_code: int) -> torch.Tensor:
    """Operator workspace of `base` bytes; under schedule 1 followed by the
    stream-K slots and counters (at least the counter tail, so no call of
    another size ever writes over the counters)."""
    if gemm_schedule() != 1:
        return workspace(device, name, base, _rest_fill(device))
    extra = streamk_bytes(M, N, K, ab_code) or STREAMK_TAIL
    return workspace(device, name, int(base) + extra, _rest_fill(device))


def verify_workspace(device: torch.device, rows: int, N: int = 0, K: int = 0, ab_code: int = DT_BF16) -> torch.Tensor:
    """Keys + ticket counter for the fused verify kernels (+ the stream-K
    region for an [rows, K] x [N, K] GEMM under schedule 1).  Initialised
    once; every verify call leaves it initialised again."""
    need = lib().mtp_verify_workspace(int(rows))
    if N > 0 and K > 0:
        need += streamk_bytes(rows, N, K, ab_code)

    def _init(buf):
        check(lib().mtp_verify_workspace_init(ptr(buf), buf.numel(), stream_handle(device)),
              "mtp_verify_workspace_init")

    return workspace(device, "verify", need, _init)


MTP_ERR_TIMEOUT = 5
_timeout_hooks = []


def on_timeout(fn) -> None:
    """Register fn(device), called when device_status() reports that a
    bounded wait ran out on `device` (mtp_parallel invalidates its peer
    exchanges this way)."""
    _timeout_hooks.append(fn)


def _reset_after_timeout(device: torch.device) -> None:
    """A kernel on `device` gave up on a bounded wait: drop every cached
    workspace of the device, so the next call allocates it again and fills
    it at rest (the stream-K counters of schedule 1 may have been left
    mid-count), then tell the registered owners of other device state."""
    idx = device.index if device.index is not None else torch.cuda.current_device()
    with _ws_lock:
        for key in [k for k in _ws if k[0] == idx]:
            del _ws[key]
    for fn in list(_timeout_hooks):
        fn(device)


def device_status(device: torch.device, clear: bool = True) -> int:
    """Synchronise the current stream of `device` and return its error word
    (0 = clean, else an MTP_ERR_* code a kernel recorded).  On
    MTP_ERR_TIMEOUT the device's cached workspaces are dropped, so later
    calls start from workspaces at rest."""
    code = ctypes.c_int(0)
    with torch.cuda.device(device):
        check(lib().mtp_device_status(stream_handle(device), ctypes.byref(code), int(clear)),
              "mtp_device_status")
    if code.value == MTP_ERR_TIMEOUT:
        _reset_after_timeout(device)
    return code.value


def exported_symbols():
    return list(SIGNATURES)
