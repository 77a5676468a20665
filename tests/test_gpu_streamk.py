"""The stream-K GEMM kernel on the GPU.  Integer-valued operands make every
summation order exact, so the stream-K result must equal the float64 product
bit for bit whatever the split; the operators under schedule 1 must then
match schedule 0 exactly, and leave their workspaces at rest.  GPU only."""

import numpy as np
import pytest
import torch

pytestmark = [pytest.mark.gpu, pytest.mark.isolated]

INT64_MIN = -(2 ** 63)


@pytest.fixture(scope="module")
def N():
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    import _mtp_native
    _mtp_native.lib()
    return _mtp_native


def sms():
    return torch.cuda.get_device_properties(0).multi_processor_count


def int_operands(M, Nn, K, dt, seed):
    d = torch.device("cuda", 0)
    g = torch.Generator(device=d).manual_seed(seed)
    A = torch.randint(-3, 4, (M, K), generator=g, device=d).float()
    B = torch.randint(-3, 4, (Nn, K), generator=g, device=d).float()
    return A.to(dt), B.to(dt), (A.double() @ B.double().T).float()


def streamk_workspace(N, M, Nn, K, code, grid):
    import ctypes
    info = (ctypes.c_int64 * 9)()
    N.check(N.lib().mtp_gemm_streamk_plan(M, Nn, K, code, sms(), grid, info), "plan")
    ws = torch.empty(int(info[8]), dtype=torch.uint8, device="cuda")
    N.check(N.lib().mtp_keys_fill(N.ptr(ws), ws.numel() // 8, N.stream_handle(ws.device)), "fill")
    return ws


def gemm_sk(N, A, B, grid, ws):
    M, K = A.shape
    C = torch.full((M, B.shape[0]), float("nan"), dtype=torch.float32, device=A.device)
    N.check(N.lib().mtp_gemm_test_streamk(N.ptr(A), N.ptr(B), N.dtype_code(A), N.ptr(C), M, B.shape[0], K, grid,
                                          N.ptr(ws), ws.numel(), N.stream_handle(A.device)), "mtp_gemm_test_streamk")
    torch.cuda.synchronize()
    return C


def counters_at_rest(ws, N):
    tail = ws[ws.numel() - N.STREAMK_TAIL: ws.numel() - 256].view(torch.int64)
    return bool((tail == INT64_MIN).all())


@pytest.mark.parametrize("dt", [torch.bfloat16, torch.float16, torch.float8_e4m3fn])
@pytest.mark.parametrize("M,Nn,K", [(384, 3000, 1024), (129, 257, 4096), (512, 1792, 512), (1, 300, 128)])
@pytest.mark.parametrize("grid", [0, 7, 37])
def test_exact_any_split(N, dt, M, Nn, K, grid):
    A, B, ref = int_operands(M, Nn, K, dt, seed=M * 7 + Nn + K + grid)
    code = N.dtype_code(A)
    ws = streamk_workspace(N, M, Nn, K, code, grid if grid > 0 else sms())
    for _ in range(2):  # the counters must be back at rest for the second call
        C = gemm_sk(N, A, B, grid, ws)
        assert torch.equal(C, ref)
        assert counters_at_rest(ws, N)
    assert N.device_status(A.device) == 0


def test_random_close_to_data_parallel(N):
    d = torch.device("cuda", 0)
    g = torch.Generator(device=d).manual_seed(5)
    M, Nn, K = 384, 20000, 4096
    A = torch.randn(M, K, generator=g, device=d).to(torch.bfloat16)
    B = torch.randn(Nn, K, generator=g, device=d).to(torch.bfloat16)
    ws = streamk_workspace(N, M, Nn, K, N.DT_BF16, sms())
    C = gemm_sk(N, A, B, 0, ws).double()
    ref = A.double() @ B.double().T
    bound = 1e-5 * (A.double().abs() @ B.double().abs().T) + 1e-6
    assert bool(((C - ref).abs() <= bound).all())


def _verify_inputs(B, S, K, V, seed):
    d = torch.device("cuda", 0)
    g = torch.Generator(device=d).manual_seed(seed)
    hid = torch.randint(-3, 4, (B, S, K), generator=g, device=d).to(torch.bfloat16)
    w = torch.randint(-3, 4, (V, K), generator=g, device=d).to(torch.bfloat16)
    draft = torch.randint(0, V, (B, S - 1), generator=g, device=d, dtype=torch.int32)
    return hid, w, draft


def test_multi_verify_schedules_agree_and_workspace_rests(N):
    import mtp_fused_verify as mv
    B, S, K, V = 64, 6, 4096, 16032  # one rank of an 8-way verify: 189 tiles, stream-K on 148 SMs
    hid, w, draft = _verify_inputs(B, S, K, V, seed=11)
    before = N.gemm_schedule()
    try:
        N.set_gemm_schedule(0)
        ref = mv.fused_multi_verify(hid, w, draft)
        N.set_gemm_schedule(1)
        assert N.streamk_bytes(B * S, V, K, N.DT_BF16) > 0
        for _ in range(3):
            got = mv.fused_multi_verify(hid, w, draft)
            torch.cuda.synchronize()
            assert all(torch.equal(a, b) for a, b in zip(got, ref))
        ws = N.verify_workspace(hid.device, B * S, V, K, N.DT_BF16)
        body = ws[: ws.numel() - 256].view(torch.int64)
        assert bool((body == INT64_MIN).all()), "verify workspace not at rest after stream-K calls"
        assert int(ws[ws.numel() - 256:].view(torch.int32)[0]) == 0
    finally:
        N.set_gemm_schedule(before)
    assert N.device_status(hid.device) == 0


def test_rmsnorm_linear_schedules_agree(N):
    import mtp_kernels as mk
    d = torch.device("cuda", 0)
    g = torch.Generator(device=d).manual_seed(3)
    M, Nn, K = 512, 14336, 4096  # config 2: 224 tiles, all stream-K
    x = torch.randint(-3, 4, (M, K), generator=g, device=d).to(torch.bfloat16)
    W = torch.randint(-3, 4, (Nn, K), generator=g, device=d).to(torch.bfloat16)
    before = N.gemm_schedule()
    try:
        N.set_gemm_schedule(0)
        ref = mk.fused_rmsnorm_linear(x, W, eps=1e-6)
        N.set_gemm_schedule(1)
        for _ in range(2):
            got = mk.fused_rmsnorm_linear(x, W, eps=1e-6)
            torch.cuda.synchronize()
            assert torch.equal(got, ref)
    finally:
        N.set_gemm_schedule(before)
    assert N.device_status(d) == 0


def test_fp8_schedules_agree(N):
    import mtp_kernels as mk
    d = torch.device("cuda", 0)
    g = torch.Generator(device=d).manual_seed(4)
    M, Nn, K = 1024, 14336, 4096  # config 3 sizes
    x = torch.randn(M, K, generator=g, device=d).to(torch.bfloat16)
    wq = torch.randint(-3, 4, (Nn, K), generator=g, device=d).float().to(torch.float8_e4m3fn)
    ws = torch.rand(Nn, generator=g, device=d) * 0.01 + 0.001
    before = N.gemm_schedule()
    try:
        N.set_gemm_schedule(0)
        ref = mk.fused_rmsnorm_linear_fp8(x, wq, ws).float()
        N.set_gemm_schedule(1)
        got = mk.fused_rmsnorm_linear_fp8(x, wq, ws).float()
        torch.cuda.synchronize()
    finally:
        N.set_gemm_schedule(before)
    # E4M3 activations are not integers: only the fp32 summation order differs
    assert torch.allclose(got, ref, rtol=2e-2, atol=1e-3)
    assert N.device_status(d) == 0


def test_shard_keys_streamk_matches(N):
    import mtp_parallel as mp
    B, S, K, V = 64, 6, 4096, 16032  # one rank of an 8-way config-5 verify: 189 tiles
    hid, w, _ = _verify_inputs(B, S, K, V, seed=13)
    rows = B * S
    L = N.lib()
    st = N.stream_handle(hid.device)
    ref = torch.full((rows,), INT64_MIN, dtype=torch.int64, device=hid.device)
    N.check(L.mtp_verify_shard_keys(N.ptr(hid), N.DT_BF16, N.ptr(w), N.DT_BF16, None, 0, N.ptr(ref), rows, K, V,
                                    1000, st), "mtp_verify_shard_keys")
    before = N.gemm_schedule()
    try:
        N.set_gemm_schedule(1)
        sk = N.streamk_bytes(rows, V, K, N.DT_BF16)
        assert sk > 0
        for _ in range(2):
            keys, region, region_bytes = mp._keys_buffer(hid.device, rows, sk)
            N.check(L.mtp_verify_shard_keys_ws(N.ptr(hid), N.DT_BF16, N.ptr(w), N.DT_BF16, None, 0, N.ptr(keys),
                                               rows, K, V, 1000, N.ptr(region), region_bytes, st),
                    "mtp_verify_shard_keys_ws")
            torch.cuda.synchronize()
            assert torch.equal(keys, ref)
            keys.fill_(INT64_MIN)  # what the decode step does
            assert bool((region[: region_bytes - 256].view(torch.int64) == INT64_MIN).all())
    finally:
        N.set_gemm_schedule(before)
    assert N.device_status(hid.device) == 0
