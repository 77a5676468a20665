"""Vocab-parallel verification for the reference's ``mtp_parallel`` module.

The lm_head W [V, K] is split into contiguous row blocks, one per rank,
exactly as ``torch.chunk(W, tp, dim=0)`` splits it (the scatter of
ParallelPrimitives, mtp_parallel.py:62-66; RowParallelLinear holds
out_features // tp rows per rank, mtp_parallel.py:96-101).  Instead of
gathering [B, S, V/tp] fp32 logits from every rank (RowParallelLinear with
gather_output, mtp_parallel.py:114-118), each rank reduces its block to one
packed int64 key per logit row,

    key = (signed-ordered fp32 max logit << 32) | (0xFFFFFFFF - global index),

so a single all-reduce(MAX) of B*S int64 keys (3 KB at B=64, S=6) yields
the global argmax with torch.argmax's lowest-index tie rule, after which
every rank decodes identical (accept, accepted_n, corrected).  The
collective is torch.distributed (NCCL over NVLink on a B200 node, gloo on
CPU test ranks).

Also provided for drop-in compatibility: ParallelPrimitives /
get_parallel_primitives (same properties and collectives as
mtp_parallel.py:12-81), RowParallelLinear (vocab-sharded linear,
mtp_parallel.py:84-118) with an added ``verify`` method, and
ColumnParallelLinear (mtp_parallel.py:121-156).
"""

from __future__ import annotations

import ctypes
import importlib.util
import math
import os
import sys
from typing import List, Optional, Tuple

import torch
import torch.nn as nn
import torch.nn.functional as F

import _mtp_native as _N


class ParallelPrimitives:
    """World/rank lookup and the three collectives of the reference
    (sum all-reduce, all-gather + concat, local chunk), mtp_parallel.py:12-66."""

    def __init__(self, group: Optional[object] = None):
        self._group = group

    @property
    def dist(self):
        d = torch.distributed
        return d if d.is_available() and d.is_initialized() else None

    @property
    def initialized(self) -> bool:
        return self.dist is not None

    @property
    def world_size(self) -> int:
        return int(self.dist.get_world_size(self._group)) if self.initialized else 1

    @property
    def rank(self) -> int:
        return int(self.dist.get_rank(self._group)) if self.initialized else 0

    @property
    def tp_size(self) -> int:
        return self.world_size

    @property
    def group(self):
        return self._group

    def all_reduce(self, x: torch.Tensor, op=None) -> torch.Tensor:
        if self.tp_size > 1:
            if op is None:
                self.dist.all_reduce(x, group=self._group)
            else:
                self.dist.all_reduce(x, op=op, group=self._group)
        return x

    def all_gather(self, x: torch.Tensor, dim: int) -> torch.Tensor:
        if self.tp_size <= 1:
            return x
        parts = [torch.empty_like(x) for _ in range(self.tp_size)]
        self.dist.all_gather(parts, x, group=self._group)
        return torch.cat(parts, dim=dim)

    def scatter(self, x: torch.Tensor, dim: int, shard_size: Optional[int] = None) -> torch.Tensor:
        if self.tp_size <= 1:
            return x
        return torch.chunk(x, self.tp_size, dim=dim)[self.rank].contiguous()


_PRIMITIVES: Optional[ParallelPrimitives] = None


def get_parallel_primitives(group: Optional[object] = None) -> ParallelPrimitives:
    global _PRIMITIVES
    if _PRIMITIVES is None:
        _PRIMITIVES = ParallelPrimitives(group)
    return _PRIMITIVES


def _reset_parallel_primitives() -> None:
    global _PRIMITIVES
    _PRIMITIVES = None


def vocab_shard_range(vocab_size: int, world: int, rank: int) -> Tuple[int, int]:
    """[lo, hi) rows of rank `rank` under torch.chunk(W, world, dim=0)."""
    step = -(-vocab_size // world)
    lo = min(rank * step, vocab_size)
    return lo, min(lo + step, vocab_size)


def key_index(keys: torch.Tensor) -> torch.Tensor:
    """Global vocabulary index carried in the low 32 bits of packed row keys
    (int64 -> int32, on the keys' device)."""
    return (0xFFFFFFFF - (keys & 0xFFFFFFFF)).to(torch.int32)


def shard_lm_head(weight: torch.Tensor, world: int, rank: int) -> Tuple[torch.Tensor, int]:
    """This rank's contiguous vocabulary block of a full lm_head and its offset."""
    lo, hi = vocab_shard_range(weight.shape[0], world, rank)
    return weight[lo:hi].contiguous(), lo


_KEYS_WS = "vocab_parallel_keys"


def _keys_buffer(dev: torch.device, rows: int, sk_bytes: int = 0):
    """This rank's keys [rows] int64, followed (under GEMM schedule 1) by the
    stream-K region of the shard GEMM; the whole buffer rests at INT64_MIN.
    Returns (keys, region, region_bytes)."""
    L = _N.lib()

    def _init(buf):
        _N.check(L.mtp_keys_fill(_N.ptr(buf), buf.numel() // 8, _N.stream_handle(dev)), "mtp_keys_fill")

    keys_bytes = (rows * 8 + 255) // 256 * 256
    buf = _N.workspace(dev, _KEYS_WS, keys_bytes + sk_bytes, _init)
    region = buf[keys_bytes:] if sk_bytes > 0 else None
    return buf[: rows * 8].view(torch.int64), region, (buf.numel() - keys_bytes) if sk_bytes > 0 else 0


class _PeerExchange:
    """Symmetric-memory buffers for the peer-memory key exchange
    (mtp_verify_exchange_chain): one buffer per rank, mapped into every rank,
    plus this rank's device-side call counter.  Every rank must build it at the
    same point and then make the same sequence of verify calls."""

    def __init__(self, dev: torch.device, rows: int, prim: "ParallelPrimitives"):
        import torch.distributed._symmetric_memory as symm

        group = prim.group if prim.group is not None else torch.distributed.group.WORLD
        if hasattr(symm, "enable_symm_mem_for_group"):
            symm.enable_symm_mem_for_group(group.group_name)
        self.rows = rows
        nbytes = _N.lib().mtp_verify_exchange_bytes(rows, prim.tp_size)
        self.buf = symm.empty(-(-nbytes // 8), dtype=torch.int64, device=dev)
        self.buf.zero_()
        self.handle = symm.rendezvous(self.buf, group)
        self.peers = int(self.handle.buffer_ptrs_dev)
        self.epoch = torch.zeros(1, dtype=torch.int64, device=dev)
        torch.cuda.synchronize(dev)
        torch.distributed.barrier(group=group)  # every buffer zeroed before any rank writes


_EXCHANGES = {}


def _invalidate_exchanges(device: torch.device) -> None:
    """A bounded wait ran out on `device` (seen by _mtp_native.device_status):
    its peer exchanges may be one call out of step with the other ranks'."""
    for key, ex in _EXCHANGES.items():
        if key[1] == device.index:
            ex.stale = True


_N.on_timeout(_invalidate_exchanges)


def reset_exchanges() -> None:
    """Forget this rank's peer-exchange buffers; the next p2p / fused
    vocab-parallel verify builds new ones at rest (a collective step).  After
    a timeout every rank must call it, between the same two verify calls:
    a rank that gave up on a wait is one call out of step with its peers."""
    _EXCHANGES.clear()


def _check_fresh(ex) -> None:
    if getattr(ex, "stale", False):
        raise _N.MTPError("a bounded wait ran out in an earlier peer-exchange verify on this device; call "
                          "mtp_parallel.reset_exchanges() on every rank before the next vocab-parallel verify")


def _peer_exchange(dev: torch.device, rows: int, prim: "ParallelPrimitives") -> _PeerExchange:
    # the buffer layout depends on rows (flags follow the keys), so a buffer is
    # used for exactly one row count; every rank makes the same calls, so all
    # ranks rebuild together
    key = ("p2p", dev.index, id(prim.group), prim.tp_size)
    ex = _EXCHANGES.get(key)
    if ex is not None:
        _check_fresh(ex)
    if ex is None or ex.rows != rows:
        ex = _PeerExchange(dev, rows, prim)
        _EXCHANGES[key] = ex
    return ex


class _FusedExchange:
    """Symmetric-memory buffers of the fused shard GEMM + exchange
    (mtp_verify_shard_fused): per rank keys [2][rows] at rest INT64_MIN,
    flags [2][world] and the call counter at 0, mapped into every rank."""

    def __init__(self, dev: torch.device, rows: int, prim: "ParallelPrimitives"):
        import torch.distributed._symmetric_memory as symm

        group = prim.group if prim.group is not None else torch.distributed.group.WORLD
        if hasattr(symm, "enable_symm_mem_for_group"):
            symm.enable_symm_mem_for_group(group.group_name)
        self.rows = rows
        L = _N.lib()
        nbytes = L.mtp_verify_fused_bytes(rows, prim.tp_size)
        self.buf = symm.empty(-(-nbytes // 8), dtype=torch.int64, device=dev)
        _N.check(L.mtp_verify_fused_init(_N.ptr(self.buf), rows, prim.tp_size, _N.stream_handle(dev)),
                 "mtp_verify_fused_init")
        self.handle = symm.rendezvous(self.buf, group)
        self.peers = int(self.handle.buffer_ptrs_dev)
        torch.cuda.synchronize(dev)
        torch.distributed.barrier(group=group)  # every buffer at rest before any rank writes


def _fused_exchange(dev: torch.device, rows: int, prim: "ParallelPrimitives") -> _FusedExchange:
    key = ("fused", dev.index, id(prim.group), prim.tp_size)
    ex = _EXCHANGES.get(key)
    if ex is not None:
        _check_fresh(ex)
    if ex is None or ex.rows != rows:
        ex = _FusedExchange(dev, rows, prim)
        _EXCHANGES[key] = ex
    return ex


def vocab_parallel_multi_verify(
    hidden: torch.Tensor,
    weight_shard: torch.Tensor,
    draft: torch.Tensor,
    bias_shard: Optional[torch.Tensor] = None,
    vocab_offset: Optional[int] = None,
    prim: Optional[ParallelPrimitives] = None,
    exchange: str = "nccl",
) -> Tuple[torch.Tensor, torch.Tensor, torch.Tensor]:
    """``fused_multi_verify`` with the lm_head split over the ranks of `prim`.

    hidden [B,S,K] and draft [B,S-1] are replicated; weight_shard
    [V_r, K] / bias_shard [V_r] are this rank's rows, starting at global row
    `vocab_offset` (default: the torch.chunk offset of this rank, assuming
    equal shards).  Every rank returns the same (accept, accepted_n,
    corrected) as single-device ``fused_multi_verify`` on the full weight.

    exchange: "nccl" -- all-reduce(MAX) of the keys through torch.distributed,
    then the acceptance scan; "p2p" -- one kernel pushes the keys to every
    peer over NVLink through symmetric memory, waits for the peers' keys and
    runs the scan (no collective library call; every rank must use it for the
    same sequence of calls); "fused" -- one kernel per rank: the shard GEMM
    sends every tile's keys to every rank's buffer (atomic max over NVLink)
    and its last CTA waits for the peers and runs the scan (tensor-core
    dtypes only; same rule on the sequence of calls).
    """
    if exchange not in ("nccl", "p2p", "fused"):
        raise ValueError(f"exchange must be 'nccl', 'p2p' or 'fused', got {exchange!r}")
    prim = prim or get_parallel_primitives()
    hidden = hidden.contiguous()
    weight_shard = weight_shard.contiguous()
    draft = draft.contiguous().to(torch.int32)
    dev = _N.require_cuda(hidden, weight_shard, draft, bias_shard)
    if bias_shard is not None:
        bias_shard = bias_shard.contiguous()
    B, S, K = hidden.shape
    D = draft.shape[1]
    assert S == D + 1, f"expected S == D + 1, got S={S} D={D}"
    Vr = weight_shard.shape[0]
    if vocab_offset is None:
        vocab_offset = prim.rank * Vr
    rows = B * S
    accept = torch.empty((B, D), dtype=torch.int8, device=hidden.device)
    accepted_n = torch.empty((B,), dtype=torch.int32, device=hidden.device)
    corrected = torch.empty((B,), dtype=torch.int32, device=hidden.device)
    L = _N.lib()
    stream = _N.stream_handle(dev)
    if prim.tp_size > 1 and exchange == "fused":
        ex = _fused_exchange(dev, rows, prim)
        ws = _N.verify_workspace(dev, 0, Vr, K, _N.dtype_code(hidden))  # ticket (+ stream-K region)
        _N.check(L.mtp_verify_shard_fused(
            _N.ptr(hidden), _N.dtype_code(hidden), _N.ptr(weight_shard), _N.dtype_code(weight_shard),
            _N.ptr(bias_shard), _N.dtype_code(bias_shard) if bias_shard is not None else 0,
            ctypes.c_void_p(ex.peers), prim.rank, prim.tp_size, _N.ptr(draft), _N.ptr(accept),
            _N.ptr(accepted_n), _N.ptr(corrected), B, S, K, Vr, int(vocab_offset), _N.ptr(ws), ws.numel(),
            stream), "mtp_verify_shard_fused")
        return accept, accepted_n, corrected
    sk = _N.streamk_bytes(rows, Vr, K, _N.dtype_code(hidden))
    keys, region, region_bytes = _keys_buffer(dev, rows, sk)  # at rest: every word is INT64_MIN
    try:
        _N.check(L.mtp_verify_shard_keys_ws(
            _N.ptr(hidden), _N.dtype_code(hidden), _N.ptr(weight_shard), _N.dtype_code(weight_shard),
            _N.ptr(bias_shard), _N.dtype_code(bias_shard) if bias_shard is not None else 0,
            _N.ptr(keys), rows, K, Vr, int(vocab_offset), _N.ptr(region), region_bytes, stream),
            "mtp_verify_shard_keys_ws")
        if prim.tp_size > 1 and exchange == "p2p":
            ex = _peer_exchange(dev, rows, prim)
            _N.check(L.mtp_verify_exchange_chain(
                _N.ptr(keys), ctypes.c_void_p(ex.peers), prim.rank, prim.tp_size, _N.ptr(ex.epoch),
                _N.ptr(draft), _N.ptr(accept), _N.ptr(accepted_n), _N.ptr(corrected), B, S, stream),
                "mtp_verify_exchange_chain")  # also puts the keys back to rest
        else:
            if prim.tp_size > 1:
                prim.all_reduce(keys, op=torch.distributed.ReduceOp.MAX)
            _N.check(L.mtp_verify_chain_from_keys(
                _N.ptr(keys), _N.ptr(draft), _N.ptr(accept), _N.ptr(accepted_n), _N.ptr(corrected), B, S,
                stream), "mtp_verify_chain_from_keys")  # also puts the keys back to rest
    except Exception:
        _N.drop_workspace(dev, _KEYS_WS)  # never reuse keys left mid-reduction
        raise
    return accept, accepted_n, corrected


class NcclCommunicator:
    """One rank's NCCL communicator made through the C ABI
    (mtp_nccl_comm_init), for processes that run the vocab-parallel verify
    without a torch.distributed process group.  Rank 0 calls ``unique_id()``
    and the host sends those bytes to every rank (any transport); each rank
    then builds ``NcclCommunicator(uid, rank, world)`` with its own GPU
    current.  The constructor returns once every rank has joined."""

    def __init__(self, uid: bytes, rank: int, world: int, device: Optional[torch.device] = None):
        if len(uid) != _N.NCCL_ID_BYTES:
            raise ValueError(f"unique id must be {_N.NCCL_ID_BYTES} bytes, got {len(uid)}")
        self.rank, self.world = int(rank), int(world)
        self.device = torch.device("cuda", torch.cuda.current_device()) if device is None else device
        self._h = ctypes.c_void_p()
        with torch.cuda.device(self.device):
            _N.check(_N.lib().mtp_nccl_comm_init(ctypes.byref(self._h), ctypes.create_string_buffer(uid, len(uid)),
                                                 self.rank, self.world), "mtp_nccl_comm_init")

    @staticmethod
    def unique_id() -> bytes:
        buf = ctypes.create_string_buffer(_N.NCCL_ID_BYTES)
        _N.check(_N.lib().mtp_nccl_unique_id(buf), "mtp_nccl_unique_id")
        return buf.raw

    @staticmethod
    def version() -> int:
        v = ctypes.c_int(0)
        _N.check(_N.lib().mtp_nccl_version(ctypes.byref(v)), "mtp_nccl_version")
        return v.value

    @property
    def handle(self) -> ctypes.c_void_p:
        if not self._h:
            raise RuntimeError("communicator is closed")
        return self._h

    def status(self) -> None:
        """Raises RuntimeError when NCCL reports an asynchronous error."""
        _N.check(_N.lib().mtp_nccl_comm_status(self.handle), "mtp_nccl_comm_status")

    def abort(self) -> None:
        """End the communicator without waiting for its collectives (a rank
        died); the communicator cannot be used afterwards."""
        if self._h:
            h, self._h = self._h, ctypes.c_void_p()
            _N.check(_N.lib().mtp_nccl_comm_abort(h), "mtp_nccl_comm_abort")

    def close(self) -> None:
        if self._h:
            h, self._h = self._h, ctypes.c_void_p()
            _N.check(_N.lib().mtp_nccl_comm_destroy(h), "mtp_nccl_comm_destroy")

    def __enter__(self):
        return self

    def __exit__(self, *exc):
        self.close()


_ABI_WS = "vocab_parallel_abi"


def vocab_parallel_multi_verify_nccl(
    hidden: torch.Tensor, weight_shard: torch.Tensor, draft: torch.Tensor, vocab_offset: int,
    comm: Optional[NcclCommunicator], bias_shard: Optional[torch.Tensor] = None,
) -> Tuple[torch.Tensor, torch.Tensor, torch.Tensor]:
    """vocab_parallel_multi_verify over a C-ABI NCCL communicator: one call
    of mtp_vocab_parallel_multi_verify (shard GEMM to argmax keys, NCCL
    all-reduce(MAX) of the keys, acceptance scan).  ``comm=None`` is a
    single-rank run.  Returns the replicated (accept, accepted_n, corrected)
    of fused_multi_verify on the whole lm_head."""
    if hidden.dim() != 3 or draft.dim() != 2:
        raise ValueError("hidden must be [B, S, K] and draft [B, S-1]")
    B, S, K = hidden.shape
    assert S == draft.shape[1] + 1, "hidden.shape[1] must equal draft.shape[1] + 1"
    assert weight_shard.shape[1] == K, "weight_shard must be [V_shard, K]"
    dev = _N.require_cuda(hidden, weight_shard, draft, bias_shard)
    hidden = hidden.contiguous()
    weight_shard = weight_shard.contiguous()
    draft = draft.contiguous().to(torch.int32)
    if bias_shard is not None:
        bias_shard = bias_shard.contiguous()
    Vr = weight_shard.shape[0]
    accept = torch.empty((B, S - 1), dtype=torch.int8, device=dev)
    accepted_n = torch.empty((B,), dtype=torch.int32, device=dev)
    corrected = torch.empty((B,), dtype=torch.int32, device=dev)
    L = _N.lib()
    need = L.mtp_vocab_parallel_workspace(B, S, Vr, K, _N.dtype_code(hidden))
    ws = _N.workspace(dev, _ABI_WS, need, _N._rest_fill(dev))  # every word INT64_MIN
    try:
        _N.check(L.mtp_vocab_parallel_multi_verify(
            _N.ptr(hidden), _N.dtype_code(hidden), _N.ptr(weight_shard), _N.dtype_code(weight_shard),
            _N.ptr(bias_shard), _N.dtype_code(bias_shard) if bias_shard is not None else 0, _N.ptr(draft),
            _N.ptr(accept), _N.ptr(accepted_n), _N.ptr(corrected), B, S, K, Vr, int(vocab_offset),
            comm.handle if comm is not None else None, _N.ptr(ws), ws.numel(), _N.stream_handle(dev)),
            "mtp_vocab_parallel_multi_verify")
    except Exception:
        _N.drop_workspace(dev, _ABI_WS)  # never reuse keys left mid-reduction
        raise
    return accept, accepted_n, corrected


class VocabParallelVerify:
    """Callable holding one rank's lm_head shard: ``__call__(hidden, draft)``
    returns the replicated (accept, accepted_n, corrected)."""

    def __init__(self, weight_shard: torch.Tensor, vocab_offset: Optional[int] = None,
                 bias_shard: Optional[torch.Tensor] = None, prim: Optional[ParallelPrimitives] = None,
                 exchange: str = "nccl"):
        self.prim = prim or get_parallel_primitives()
        self.exchange = exchange
        self.weight_shard = weight_shard.contiguous()
        self.bias_shard = None if bias_shard is None else bias_shard.contiguous()
        self.vocab_offset = self.prim.rank * self.weight_shard.shape[0] if vocab_offset is None else vocab_offset

    @classmethod
    def from_full(cls, weight: torch.Tensor, bias: Optional[torch.Tensor] = None,
                  prim: Optional[ParallelPrimitives] = None, exchange: str = "nccl") -> "VocabParallelVerify":
        prim = prim or get_parallel_primitives()
        w, off = shard_lm_head(weight, prim.tp_size, prim.rank)
        b = None if bias is None else bias[off:off + w.shape[0]]
        return cls(w, off, b, prim, exchange)

    def __call__(self, hidden: torch.Tensor, draft: torch.Tensor,
                 bias_shard: Optional[torch.Tensor] = None):
        b = self.bias_shard if bias_shard is None else bias_shard
        return vocab_parallel_multi_verify(hidden, self.weight_shard, draft, b, self.vocab_offset, self.prim,
                                           self.exchange)


class RowParallelLinear(nn.Module):
    """Linear layer whose out_features (the vocabulary) are split over the
    ranks, as in mtp_parallel.py:84-118: forward() returns this rank's
    logits, all-gathered when gather_output else sum-all-reduced (the
    reference's default).  ``verify`` runs the fused vocab-parallel
    verification on the shard without materialising logits."""

    def __init__(self, in_features: int, out_features: int, bias: bool = True, gather_output: bool = False,
                 prim: Optional[ParallelPrimitives] = None):
        super().__init__()
        self.prim = prim if prim is not None else get_parallel_primitives()
        tp = self.prim.tp_size
        assert out_features % tp == 0
        self.in_features = in_features
        self.out_features = out_features
        self.out_features_per_rank = out_features // tp
        self.gather_output = gather_output
        self.weight = nn.Parameter(torch.empty(self.out_features_per_rank, in_features))
        self.bias = nn.Parameter(torch.empty(self.out_features_per_rank)) if bias else None
        self.reset_parameters()

    def reset_parameters(self) -> None:
        nn.init.kaiming_uniform_(self.weight, a=math.sqrt(5))
        if self.bias is not None:
            bound = 1.0 / math.sqrt(self.in_features)
            nn.init.uniform_(self.bias, -bound, bound)

    def forward(self, x: torch.Tensor) -> torch.Tensor:
        y = F.linear(x, self.weight, self.bias)
        return self.prim.all_gather(y, dim=-1) if self.gather_output else self.prim.all_reduce(y)

    @torch.no_grad()
    def verify(self, hidden: torch.Tensor, draft: torch.Tensor):
        off = self.prim.rank * self.out_features_per_rank
        return vocab_parallel_multi_verify(hidden, self.weight, draft, self.bias, off, self.prim)


class ColumnParallelLinear(nn.Module):
    """Linear layer whose in_features are split over the ranks, as in
    mtp_parallel.py:121-156: forward() takes this rank's torch.chunk slice
    of x along the last dim and returns its partial product (plus the full
    bias), all-gathered along the last dim when gather_output.  Kept for
    drop-in compatibility; it is not on the verify path (the verify splits the
    vocabulary, RowParallelLinear / vocab_parallel_multi_verify)."""

    def __init__(self, in_features: int, out_features: int, bias: bool = True, gather_output: bool = False,
                 prim: Optional[ParallelPrimitives] = None):
        super().__init__()
        self.prim = prim if prim is not None else get_parallel_primitives()
        tp = self.prim.tp_size
        assert in_features % tp == 0
        self.in_features = in_features
        self.in_features_per_rank = in_features // tp
        self.out_features = out_features
        self.gather_output = gather_output
        self.weight = nn.Parameter(torch.empty(out_features, self.in_features_per_rank))
        self.bias = nn.Parameter(torch.empty(out_features)) if bias else None
        self.reset_parameters()

    def reset_parameters(self) -> None:
        nn.init.kaiming_uniform_(self.weight, a=math.sqrt(5))
        if self.bias is not None:
            bound = 1.0 / math.sqrt(self.in_features_per_rank)
            nn.init.uniform_(self.bias, -bound, bound)

    def forward(self, x: torch.Tensor) -> torch.Tensor:
        y = F.linear(self.prim.scatter(x, dim=-1, shard_size=self.in_features_per_rank), self.weight, self.bias)
        return self.prim.all_gather(y, dim=-1) if self.gather_output else y


# --------------------------------------------------------------------------- #
# names outside the hot path (SegmentedGraphRunner, GraphSegment, ...)
# --------------------------------------------------------------------------- #
_reference_module = None


def _load_reference():
    global _reference_module
    if _reference_module is None:
        root = os.environ.get("MTP_REFERENCE_PATH")
        if not root:
            return None
        spec = importlib.util.spec_from_file_location("_mtp_reference_parallel", os.path.join(root, "mtp_parallel.py"))
        mod = importlib.util.module_from_spec(spec)
        sys.modules["_mtp_reference_parallel"] = mod
        spec.loader.exec_module(mod)
        _reference_module = mod
    return _reference_module


def __getattr__(name: str):
    if name.startswith("__"):
        raise AttributeError(name)
    ref = _load_reference()
    if ref is not None and hasattr(ref, name):
        return getattr(ref, name)
    raise AttributeError(
        f"mtp_parallel.{name} is not part of the B200 hot path implemented by mtp-engine-b200; "
        "set MTP_REFERENCE_PATH to the reference checkout to resolve it there")


__all__ = [
    "ParallelPrimitives", "get_parallel_primitives", "vocab_shard_range", "shard_lm_head",
    "vocab_parallel_multi_verify", "VocabParallelVerify", "RowParallelLinear", "ColumnParallelLinear",
    "key_index", "NcclCommunicator", "vocab_parallel_multi_verify_nccl", "reset_exchanges",
]
