"""The tcgen05 GEMM mainloop in isolation (mtp_gemm_test): structured
operands pin the TMEM row/column mapping and the swizzled K order, random
operands check accumulation, for bf16, f16 and E4M3.  GPU only."""

import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def N():
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    import _mtp_native
    _mtp_native.lib()
    return _mtp_native


def gemm(N, A, B, simt=0):
    M, K = A.shape
    C = torch.zeros(M, B.shape[0], dtype=torch.float32, device=A.device)
    N.check(N.lib().mtp_gemm_test(N.ptr(A), N.ptr(B), N.dtype_code(A), N.ptr(C), M, B.shape[0], K, simt,
                                  N.stream_handle(A.device)), "mtp_gemm_test")
    torch.cuda.synchronize()
    return C


def test_structured_mapping(N):
    d = torch.device("cuda", 0)
    bf = torch.bfloat16
    for Nn in (128, 256):
        M, K = 128, 64
        # rows: C[m, n] = m % 64 + 1
        A = torch.zeros(M, K, device=d); A[:, 0] = torch.arange(M, device=d) % 64 + 1
        B = torch.zeros(Nn, K, device=d); B[:, 0] = 1
        assert torch.equal(gemm(N, A.to(bf), B.to(bf)), A @ B.T)
        # columns: C[m, n] = n % 200 + 1
        A = torch.zeros(M, K, device=d); A[:, 0] = 1
        B = torch.zeros(Nn, K, device=d); B[:, 0] = torch.arange(Nn, device=d) % 200 + 1
        assert torch.equal(gemm(N, A.to(bf), B.to(bf)), A @ B.T)
        # K order through the 128-byte swizzle, A side and B side
        A = torch.zeros(M, K, device=d); A[torch.arange(M), torch.arange(M) % 64] = 1
        B = (torch.arange(K, device=d) + 1).float().repeat(Nn, 1)
        assert torch.equal(gemm(N, A.to(bf), B.to(bf)), A @ B.T)
        assert torch.equal(gemm(N, B.to(bf)[:M], A.to(bf)[: min(Nn, M)]), B[:M] @ A[: min(Nn, M)].T)


@pytest.mark.parametrize("dt", [torch.bfloat16, torch.float16, torch.float8_e4m3fn])
@pytest.mark.parametrize("M,Nn,K", [(128, 128, 64), (48, 384, 512), (300, 1000, 1024), (129, 257, 4096)])
def test_random(N, dt, M, Nn, K):
    d = torch.device("cuda", 0)
    g = torch.Generator(device=d).manual_seed(M + Nn + K)
    A = torch.randn(M, K, generator=g, device=d).to(dt)
    B = torch.randn(Nn, K, generator=g, device=d).to(dt)
    ref = A.float().cpu().double() @ B.float().cpu().double().T
    C = gemm(N, A, B).cpu().double()
    # products are exact in fp32; only the summation order differs
    bound = 1e-5 * (A.float().abs().cpu().double() @ B.float().abs().cpu().double().T) + 1e-6
    assert ((C - ref).abs() <= bound).all()
    Cs = gemm(N, A, B, simt=1).cpu().double()
    assert ((Cs - ref).abs() <= bound).all()
