"""The two peer-memory exchanges on one GPU: the exchange kernel
(mtp_verify_exchange_chain) and the shard GEMM with the exchange fused in
(mtp_verify_shard_fused).  With world = 1 each must reproduce
fused_multi_verify (keys to its own buffer, flag itself, decode) call after
call.  With world = 2 and a second buffer that no rank ever signals -- a
flag that nothing sets -- the bounded wait must run out (2 s), the kernel
must return with MTP_ERR_TIMEOUT in the device status and its keys back at
rest, and the context must stay usable for the next operator.  No second
kernel waits on these.  GPU only; runs in a child process
(tests/test_gpu_isolated.py)."""

import time

import pytest
import torch

pytestmark = [pytest.mark.gpu, pytest.mark.isolated]

INT64_MIN = -(2 ** 63)
ERR_TIMEOUT = 5


@pytest.fixture(scope="module")
def mods():
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    import _mtp_native as N
    import mtp_fused_verify as mv
    torch.cuda.set_device(0)
    return N, mv


def inputs(seed, B=8, S=6, K=512, V=10007):
    d = torch.device("cuda", 0)
    g = torch.Generator(device=d).manual_seed(seed)
    hid = torch.randn(B, S, K, generator=g, device=d).to(torch.bfloat16)
    w = (0.05 * torch.randn(V, K, generator=g, device=d)).to(torch.bfloat16)
    draft = torch.randint(0, V, (B, S - 1), generator=g, device=d, dtype=torch.int32)
    return hid, w, draft


def shard_keys(N, hid, w):
    B, S, K = hid.shape
    keys = torch.full((B * S,), INT64_MIN, dtype=torch.int64, device=hid.device)
    N.check(N.lib().mtp_verify_shard_keys(N.ptr(hid), N.DT_BF16, N.ptr(w), N.DT_BF16, None, 0, N.ptr(keys), B * S,
                                          K, w.shape[0], 0, N.stream_handle(hid.device)), "shard keys")
    return keys


def exchange(N, keys, peers, rank, world, epoch, draft, B, S):
    d = keys.device
    acc = torch.full((B, S - 1), -1, dtype=torch.int8, device=d)
    n = torch.full((B,), -1, dtype=torch.int32, device=d)
    c = torch.full((B,), -1, dtype=torch.int32, device=d)
    N.check(N.lib().mtp_verify_exchange_chain(N.ptr(keys), N.ptr(peers), rank, world, N.ptr(epoch), N.ptr(draft),
                                              N.ptr(acc), N.ptr(n), N.ptr(c), B, S, N.stream_handle(d)),
            "mtp_verify_exchange_chain")
    return acc, n, c


def exchange_buffers(N, rows, world, count):
    d = torch.device("cuda", 0)
    nbytes = N.lib().mtp_verify_exchange_bytes(rows, world)
    bufs = [torch.zeros(-(-nbytes // 8), dtype=torch.int64, device=d) for _ in range(count)]
    peers = torch.tensor([b.data_ptr() for b in bufs], dtype=torch.int64, device=d)
    return bufs, peers


def test_single_rank_exchange_matches_verify(mods):
    N, mv = mods
    hid, w, draft = inputs(1)
    B, S, _ = hid.shape
    ref = mv.fused_multi_verify(hid, w, draft)
    bufs, peers = exchange_buffers(N, B * S, 1, 1)
    epoch = torch.zeros(1, dtype=torch.int64, device=hid.device)
    for _ in range(3):  # both key parities, then the first again
        keys = shard_keys(N, hid, w)
        got = exchange(N, keys, peers, 0, 1, epoch, draft, B, S)
        torch.cuda.synchronize()
        for a, b in zip(got, ref):
            assert torch.equal(a, b)
        assert bool((keys == INT64_MIN).all())  # decoded keys are back at rest
    assert int(epoch.item()) == 3
    assert N.device_status(hid.device) == 0


def test_missing_peer_times_out_and_context_survives(mods):
    N, mv = mods
    hid, w, draft = inputs(2)
    B, S, _ = hid.shape
    dev = hid.device
    N.device_status(dev)  # clear
    bufs, peers = exchange_buffers(N, B * S, 2, 2)  # rank 1's buffer: nobody ever signals it
    epoch = torch.zeros(1, dtype=torch.int64, device=dev)
    keys = shard_keys(N, hid, w)
    t0 = time.perf_counter()
    exchange(N, keys, peers, 0, 2, epoch, draft, B, S)
    torch.cuda.synchronize()
    waited = time.perf_counter() - t0
    assert N.device_status(dev) == ERR_TIMEOUT
    assert 1.0 < waited < 30.0
    assert bool((keys == INT64_MIN).all())  # the failed call put its keys back at rest
    # the context is still usable
    ref = mv.fused_multi_verify(hid, w, draft)
    torch.cuda.synchronize()
    assert N.device_status(dev) == 0
    assert int(ref[1].min()) >= 0


def fused_buffers(N, rows, world, count):
    d = torch.device("cuda", 0)
    nbytes = N.lib().mtp_verify_fused_bytes(rows, world)
    bufs = [torch.empty(-(-nbytes // 8), dtype=torch.int64, device=d) for _ in range(count)]
    for b in bufs:
        N.check(N.lib().mtp_verify_fused_init(N.ptr(b), rows, world, N.stream_handle(d)), "fused init")
    peers = torch.tensor([b.data_ptr() for b in bufs], dtype=torch.int64, device=d)
    return bufs, peers


def shard_fused(N, hid, w, draft, peers, rank, world):
    B, S, K = hid.shape
    d = hid.device
    ws = N.verify_workspace(d, 0, w.shape[0], K, N.DT_BF16)
    acc = torch.full((B, S - 1), -1, dtype=torch.int8, device=d)
    n = torch.full((B,), -1, dtype=torch.int32, device=d)
    c = torch.full((B,), -1, dtype=torch.int32, device=d)
    N.check(N.lib().mtp_verify_shard_fused(N.ptr(hid), N.DT_BF16, N.ptr(w), N.DT_BF16, None, 0, N.ptr(peers), rank,
                                           world, N.ptr(draft), N.ptr(acc), N.ptr(n), N.ptr(c), B, S, K, w.shape[0],
                                           0, N.ptr(ws), ws.numel(), N.stream_handle(d)), "mtp_verify_shard_fused")
    return acc, n, c


def test_fused_exchange_single_rank_matches_verify(mods):
    """The GEMM with the exchange fused in, world = 1: every tile's keys go
    to this rank's own buffer, the last CTA flags itself and decodes."""
    N, mv = mods
    hid, w, draft = inputs(3)
    B, S, _ = hid.shape
    ref = mv.fused_multi_verify(hid, w, draft)
    bufs, peers = fused_buffers(N, B * S, 1, 1)
    for _ in range(3):  # both key parities, then the first again
        got = shard_fused(N, hid, w, draft, peers, 0, 1)
        torch.cuda.synchronize()
        for a, b in zip(got, ref):
            assert torch.equal(a, b)
    assert N.device_status(hid.device) == 0


def test_fused_exchange_missing_peer_times_out(mods):
    """After the fused exchange gives up on a peer, the verify that shares
    its workspace (ticket) gives exactly its earlier result -- first without
    anyone reading the device status, then after device_status() has reported
    the timeout and dropped the cached workspaces."""
    N, mv = mods
    hid, w, draft = inputs(4)
    B, S, _ = hid.shape
    dev = hid.device
    ref = mv.fused_multi_verify(hid, w, draft)
    torch.cuda.synchronize()
    N.device_status(dev)
    bufs, peers = fused_buffers(N, B * S, 2, 2)  # rank 1 never runs
    t0 = time.perf_counter()
    shard_fused(N, hid, w, draft, peers, 0, 2)
    torch.cuda.synchronize()
    waited = time.perf_counter() - t0
    after = mv.fused_multi_verify(hid, w, draft)  # same workspace, status not read yet
    torch.cuda.synchronize()
    for a, b in zip(after, ref):
        assert torch.equal(a, b)
    assert N.device_status(dev) == ERR_TIMEOUT
    assert 1.0 < waited < 30.0
    # this rank's keys of the failed call are back at rest, and the context works
    rows = B * S
    assert bool((bufs[0][:2 * rows] == INT64_MIN).all())
    again = mv.fused_multi_verify(hid, w, draft)  # new workspace after the reset
    torch.cuda.synchronize()
    for a, b in zip(again, ref):
        assert torch.equal(a, b)
    assert N.device_status(dev) == 0


def test_fused_exchange_streamk_single_rank(mods):
    """The fused GEMM+exchange under the stream-K schedule at the shape of
    one rank of an 8-way verify (384 x 16032 x 4096, where the cost model
    takes stream-K).  Integer-valued operands keep every split-K sum exact,
    so the outputs must equal the data-parallel schedule's bit for bit,
    ties included (lowest index)."""
    N, mv = mods
    d = torch.device("cuda", 0)
    g = torch.Generator(device=d).manual_seed(5)
    B, S, K, V = 64, 6, 4096, 16032
    hid = torch.randint(-2, 3, (B, S, K), generator=g, device=d).to(torch.bfloat16)
    w = torch.randint(-2, 3, (V, K), generator=g, device=d).to(torch.bfloat16)
    draft = torch.randint(0, V, (B, S - 1), generator=g, device=d, dtype=torch.int32)
    before = N.gemm_schedule()
    try:
        N.set_gemm_schedule(0)
        ref = mv.fused_multi_verify(hid, w, draft)
        N.set_gemm_schedule(1)
        bufs, peers = fused_buffers(N, B * S, 1, 1)
        for _ in range(2):
            got = shard_fused(N, hid, w, draft, peers, 0, 1)
            torch.cuda.synchronize()
            for a, b in zip(got, ref):
                assert torch.equal(a, b)
    finally:
        N.set_gemm_schedule(before)
    assert N.device_status(d) == 0
