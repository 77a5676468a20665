"""The 256-row tiles of the tensor-core GEMM (mtp_set_gemm_tile_rows): two
M=128 MMAs per K step sharing one weight stage, a single TMEM accumulator
per tile, row tiles rotated by round, and a half tile whose second half is
skipped.  Integer-valued operands make every summation order exact, so
mtp_gemm_test must equal the float64 product bit for bit; the operators
(RMSNorm-linear store epilogue, verify argmax epilogue) must then give what
the 128-row tiles give, and write nothing outside their outputs.  GPU only;
runs in a child process (tests/test_gpu_isolated.py)."""

import ctypes

import pytest
import torch

pytestmark = [pytest.mark.gpu, pytest.mark.isolated]

PAD = 8192
CANARY = 0x5A


@pytest.fixture(scope="module")
def N():
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    import _mtp_native
    _mtp_native.lib()
    before = _mtp_native.gemm_tile_rows()
    yield _mtp_native
    _mtp_native.set_gemm_tile_rows(before)


def int_operands(M, Nn, K, dt, seed):
    d = torch.device("cuda", 0)
    g = torch.Generator(device=d).manual_seed(seed)
    A = torch.randint(-3, 4, (M, K), generator=g, device=d).float()
    B = torch.randint(-3, 4, (Nn, K), generator=g, device=d).float()
    return A.to(dt), B.to(dt), (A.double() @ B.double().T).float()


def gemm_guarded(N, A, B):
    """C through mtp_gemm_test, inside canary bytes; returns (C, intact)."""
    M, K = A.shape
    Nn = B.shape[0]
    raw = torch.full((M * Nn * 4 + 2 * PAD,), CANARY, dtype=torch.uint8, device=A.device)
    N.check(N.lib().mtp_gemm_test(N.ptr(A), N.ptr(B), N.dtype_code(A), ctypes.c_void_p(raw.data_ptr() + PAD), M,
                                  Nn, K, 0, N.stream_handle(A.device)), "mtp_gemm_test")
    torch.cuda.synchronize()
    intact = bool((raw[:PAD] == CANARY).all()) and bool((raw[PAD + M * Nn * 4:] == CANARY).all())
    return raw[PAD:PAD + M * Nn * 4].view(torch.float32).view(M, Nn), intact


# M: full 256-row tiles, a half tile (384 = 256 + 128), a second half that is
# partly (130, 300) or wholly (257 -> 256 + 1) inside M, one row tile only
SHAPES = [(384, 1000, 512), (256, 256, 64), (130, 300, 264), (257, 513, 128), (300, 4096, 192),
          (512, 777, 1024), (1000, 700, 320), (129, 64, 4096)]


@pytest.mark.parametrize("dt", [torch.bfloat16, torch.float16, torch.float8_e4m3fn])
@pytest.mark.parametrize("M,Nn,K", SHAPES)
def test_exact_integer_gemm(N, dt, M, Nn, K):
    A, B, ref = int_operands(M, Nn, K, dt, M + Nn + K)
    N.set_gemm_tile_rows(2)
    C, intact = gemm_guarded(N, A, B)
    assert intact, "write outside C"
    assert torch.equal(C, ref)
    assert N.device_status(A.device) == 0


def test_many_rounds_rotation(N):
    """More tiles than SMs, grid a multiple of the row-tile count: every CTA
    walks through both row tiles (the rotated order must still cover each
    tile exactly once)."""
    sms = torch.cuda.get_device_properties(0).multi_processor_count
    M, K = 384, 128
    Nn = 256 * (2 * sms + 7)  # > 2 rounds of 256 x 256 tiles, last round ragged
    A, B, ref = int_operands(M, Nn, K, torch.bfloat16, 5)
    for mode in (1, 2):
        N.set_gemm_tile_rows(mode)
        C, intact = gemm_guarded(N, A, B)
        assert intact and torch.equal(C, ref)


def test_operators_match_128_row_tiles(N):
    import mtp_fused_verify as mv
    import mtp_kernels as mk
    d = torch.device("cuda", 0)
    g = torch.Generator(device=d).manual_seed(9)
    # RMSNorm-linear (store epilogue, rstd and gamma)
    x = torch.randn(384, 1024, generator=g, device=d).to(torch.bfloat16)
    W = (0.02 * torch.randn(3000, 1024, generator=g, device=d)).to(torch.bfloat16)
    gam = 1.0 + 0.1 * torch.randn(1024, generator=g, device=d)
    N.set_gemm_tile_rows(0)
    y0 = mk.fused_rmsnorm_linear(x, W, None, 1e-5, norm_weight=gam)
    N.set_gemm_tile_rows(2)
    y1 = mk.fused_rmsnorm_linear(x, W, None, 1e-5, norm_weight=gam)
    torch.cuda.synchronize()
    # same products, same K order per element; allow for a different tile width
    assert (y1.float() - y0.float()).abs().max().item() <= 1e-2 * y0.float().abs().max().item()
    # verify (argmax epilogue + acceptance scan): tokens exactly
    B, S, K, V = 64, 6, 1024, 40000
    hid = torch.randn(B, S, K, generator=g, device=d).to(torch.bfloat16)
    lm = (0.05 * torch.randn(V, K, generator=g, device=d)).to(torch.bfloat16)
    draft = torch.randint(0, V, (B, S - 1), generator=g, device=d, dtype=torch.int32)
    N.set_gemm_tile_rows(0)
    ref = mv.fused_multi_verify(hid, lm, draft)
    for mode in (1, 2):
        N.set_gemm_tile_rows(mode)
        for _ in range(2):  # the verify workspace is back at rest after each call
            got = mv.fused_multi_verify(hid, lm, draft)
            torch.cuda.synchronize()
            for a, b in zip(got, ref):
                assert torch.equal(a, b)
    assert N.device_status(d) == 0


def test_switch_roundtrip(N):
    L = N.lib()
    for m in (0, 1, 2):
        N.set_gemm_tile_rows(m)
        assert L.mtp_gemm_tile_rows() == m
    assert L.mtp_set_gemm_tile_rows(3) == 8  # MTP_ERR_ARG


def test_config5_verify_and_config2_shapes(N):
    """At the benchmark sizes the cost model sends to 256-row tiles (mode 1):
    the 1-GPU verify (384 x 128256 x 4096, a half row tile) must give the
    128-row tiles' tokens exactly, and config 2 (512 x 14336 x 4096) the
    same outputs within the bf16 bound."""
    import mtp_fused_verify as mv
    import mtp_kernels as mk
    d = torch.device("cuda", 0)
    g = torch.Generator(device=d).manual_seed(4)
    hid = torch.randn(64, 6, 4096, generator=g, device=d).to(torch.bfloat16)
    lm = (0.02 * torch.randn(128256, 4096, generator=g, device=d)).to(torch.bfloat16)
    draft = torch.randint(0, 128256, (64, 5), generator=g, device=d, dtype=torch.int32)
    N.set_gemm_tile_rows(0)
    ref = mv.fused_multi_verify(hid, lm, draft)
    N.set_gemm_tile_rows(1)
    got = mv.fused_multi_verify(hid, lm, draft)
    torch.cuda.synchronize()
    for a, b in zip(got, ref):
        assert torch.equal(a, b)
    del lm
    x = torch.randn(512, 4096, generator=g, device=d).to(torch.bfloat16)
    W = (0.02 * torch.randn(14336, 4096, generator=g, device=d)).to(torch.bfloat16)
    gam = 1.0 + 0.1 * torch.randn(4096, generator=g, device=d)
    N.set_gemm_tile_rows(0)
    y0 = mk.fused_rmsnorm_linear(x, W, None, 1e-5, norm_weight=gam)
    N.set_gemm_tile_rows(1)
    y1 = mk.fused_rmsnorm_linear(x, W, None, 1e-5, norm_weight=gam)
    torch.cuda.synchronize()
    assert (y1.float() - y0.float()).abs().max().item() <= 2e-2 * y0.float().abs().max().item()
    assert N.device_status(d) == 0
