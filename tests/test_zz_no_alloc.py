"""mtp_fused_multi_verify_noalloc: the chain-verification entry point for
hosts that cannot give the library any device scratch memory (their HBM is
already reserved by another allocator, or they are plain C / FFI callers
that only own their inputs and outputs and must not call cudaMalloc mid-step).

It is called through the C ABI and must return exactly what the regular
mtp_fused_multi_verify returns (integer tokens and counts: bit-exact), on two
calls in a row -- the second call reuses the library's fixed scratch array
after the first one left its contents there.  This file is collected last
and passes both alone in a fresh process and after the rest of the suite.
"""

import ctypes

import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu

MAX_ROWS = 8192  # MTP_NOALLOC_MAX_ROWS in include/mtp_b200.h


@pytest.fixture(scope="module")
def N():
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    import _mtp_native
    _mtp_native.lib()
    return _mtp_native


def _inputs(seed, B, S, K, V, dtype, dev):
    g = torch.Generator(device=dev).manual_seed(seed)
    hid = torch.randn(B, S, K, generator=g, device=dev).to(dtype)
    w = (0.05 * torch.randn(V, K, generator=g, device=dev)).to(dtype)
    bias = 0.1 * torch.randn(V, generator=g, device=dev)
    top = (hid.float().reshape(B * S, K) @ w.float().T + bias).argmax(-1).reshape(B, S).cpu().numpy()
    rng = np.random.default_rng(seed)
    draft = rng.integers(0, V, size=(B, S - 1))
    for b in range(B):  # accept prefixes of every length
        a = b % S
        draft[b, :a] = top[b, 1:a + 1]
    return hid, w, bias, torch.tensor(draft, dtype=torch.int32, device=dev)


def _outputs(B, D, dev):
    return (torch.full((B, D), 7, dtype=torch.int8, device=dev), torch.full((B,), -5, dtype=torch.int32, device=dev),
            torch.full((B,), -5, dtype=torch.int32, device=dev))


def _regular(N, hid, w, bias, draft):
    dev = hid.device
    B, S, K = hid.shape
    a, n, c = _outputs(B, S - 1, dev)
    ws = torch.empty(N.lib().mtp_verify_workspace(B * S), dtype=torch.uint8, device=dev)
    st = N.stream_handle(dev)
    N.check(N.lib().mtp_verify_workspace_init(N.ptr(ws), ws.numel(), st), "init")
    N.check(N.lib().mtp_fused_multi_verify(N.ptr(hid), N.dtype_code(hid), N.ptr(w), N.dtype_code(w), N.ptr(bias),
                                           N.dtype_code(bias), N.ptr(draft), N.ptr(a), N.ptr(n), N.ptr(c), B, S, K,
                                           w.shape[0], N.ptr(ws), ws.numel(), st), "mtp_fused_multi_verify")
    return a, n, c


def _noalloc(N, hid, w, bias, draft):
    dev = hid.device
    B, S, K = hid.shape
    a, n, c = _outputs(B, S - 1, dev)
    status = N.lib().mtp_fused_multi_verify_noalloc(
        N.ptr(hid), N.dtype_code(hid), N.ptr(w), N.dtype_code(w), N.ptr(bias), N.dtype_code(bias), N.ptr(draft),
        N.ptr(a), N.ptr(n), N.ptr(c), B, S, K, w.shape[0], N.stream_handle(dev))
    N.check(status, "mtp_fused_multi_verify_noalloc")
    return a, n, c


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float32])
def test_noalloc_matches_regular_twice(N, dtype):
    dev = torch.device("cuda", 0)
    cases = [_inputs(11, 16, 6, 1024, 30011, dtype, dev), _inputs(12, 5, 4, 512, 7001, dtype, dev)]
    for hid, w, bias, draft in cases:  # two calls in a row on the shared scratch array
        ref = _regular(N, hid, w, bias, draft)
        got = _noalloc(N, hid, w, bias, draft)
        torch.cuda.synchronize()
        for x, y in zip(got, ref):
            assert torch.equal(x, y)
    assert N.device_status(dev) == 0


def test_noalloc_single_position(N):
    """S == 1 (no drafts: draft and accept may be NULL): only corrected and
    accepted_n = 0 come out, equal to the regular entry's, twice in a row."""
    dev = torch.device("cuda", 0)
    for seed in (13, 14):
        hid, w, bias, draft = _inputs(seed, 24, 1, 768, 5003, torch.bfloat16, dev)
        ref = _regular(N, hid, w, bias, draft)
        got = _noalloc(N, hid, w, bias, draft)
        torch.cuda.synchronize()
        for x, y in zip(got, ref):
            assert torch.equal(x, y)
        assert int(got[1].abs().max()) == 0
    assert N.device_status(dev) == 0


def test_noalloc_rejects_oversized(N):
    dev = torch.device("cuda", 0)
    before = N.lib().mtp_launch_count()
    B, S = MAX_ROWS // 4 + 1, 4  # B*S just above the limit
    st = N.lib().mtp_fused_multi_verify_noalloc(None, 1, None, 1, None, 0, None, None, None, None, B, S, 64, 128,
                                                N.stream_handle(dev))
    assert st == 1  # MTP_ERR_SHAPE
    assert b"exceeds" in N.lib().mtp_last_error()
    # B * S past INT64_MAX must not wrap into the accepted range
    st = N.lib().mtp_fused_multi_verify_noalloc(None, 1, None, 1, None, 0, None, None, None, None, 2 ** 62 + 1, 4,
                                                64, 128, N.stream_handle(dev))
    assert st == 1
    assert N.lib().mtp_launch_count() == before
