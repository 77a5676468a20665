"""fused_tree_attn_rmsnorm_linear on the GPU against the reference's golden
vectors and the CPU oracle (_eager_tree_attn_rmsnorm_linear,
mtp_kernels.py:881-905).  Tolerances: fp32 operands 1e-4 of max|ref|
(only the summation order differs); 16-bit operands the hot-path bar,
max|y - ref| <= 2e-2 max|ref| (the normalised attention output is rounded
once to the operand dtype).  GPU only."""

import math

import numpy as np
import pytest
import torch

from oracle import mtp_oracle as O

pytestmark = [pytest.mark.gpu, pytest.mark.isolated]


@pytest.fixture(scope="module")
def mk():
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    import mtp_kernels
    return mtp_kernels


def f32(t):
    return None if t is None else t.detach().float().cpu().numpy()


def rel_err(y, ref):
    y, ref = np.asarray(y, np.float64), np.asarray(ref, np.float64)
    return np.max(np.abs(y - ref)) / max(np.max(np.abs(ref)), 1e-30)


def test_golden_fp32(mk, golden):
    g = golden("tree_attn_rmsnorm_linear.npz")
    d = torch.device("cuda", 0)
    T = lambda n: torch.tensor(g[n], device=d)
    s = float(g["scale"][0])
    y = mk.fused_tree_attn_rmsnorm_linear(T("q"), T("k"), T("v"), T("mask"), T("proj_w"), rms_w=T("rms_w"),
                                          proj_bias=T("proj_b"), wscale=T("wscale"), scale=s, eps=1e-6)
    assert rel_err(f32(y), g["out"]) <= 1e-4
    y = mk.fused_tree_attn_rmsnorm_linear(T("q"), T("k"), T("v"), T("mask"), T("proj_w"), scale=0.3, eps=1e-5)
    assert rel_err(f32(y), g["out_bare"]) <= 1e-4
    z = torch.zeros_like(T("mask"))
    y = mk.fused_tree_attn_rmsnorm_linear(T("q")[:1], T("k")[:1], T("v")[:1], z, T("proj_w"), rms_w=T("rms_w"),
                                          proj_bias=T("proj_b"), scale=s)
    assert torch.isnan(y).all() and np.isnan(g["out_nan"]).all()


def test_golden_bf16(mk, golden):
    g = golden("tree_attn_rmsnorm_linear.npz")
    d = torch.device("cuda", 0)
    B16 = lambda n: torch.tensor(g[n].view(np.int16), device=d).view(torch.bfloat16)
    y = mk.fused_tree_attn_rmsnorm_linear(B16("q_bits"), B16("k_bits"), B16("v_bits"),
                                          torch.tensor(g["mask"], device=d), B16("w_bits"),
                                          rms_w=torch.tensor(g["rms_w"], device=d),
                                          proj_bias=torch.tensor(g["proj_b"], device=d),
                                          scale=float(g["scale"][0]), eps=1e-6)
    assert y.dtype == torch.bfloat16
    assert rel_err(f32(y), O.bf16_bits_to_f32(g["out_b_bits"])) <= 2e-2


CASES = [
    # B, H, D, L, N, dtype, weight dtype
    (64, 1, 4096, 64, 32000, torch.bfloat16, torch.bfloat16),   # engine draft head: tensor-core projection
    (4, 4, 200, 40, 300, torch.bfloat16, torch.bfloat16),       # 25 chunks of 8: padded q copy
    (3, 2, 100, 17, 129, torch.float16, torch.float16),         # D % 8 != 0: scalar path
    (2, 3, 128, 700, 96, torch.float32, torch.float32),         # kept-key compaction over 3 blocks
    (2, 2, 512, 33, 640, torch.bfloat16, torch.float32),        # fp32 weight: fp32 operand, CUDA-core GEMM
    (2, 2, 256, 24, 320, torch.float32, torch.float8_e4m3fn),   # E4M3 weight with wscale
]


@pytest.mark.parametrize("B,H,D,L,N,dt,wdt", CASES)
def test_against_oracle(mk, B, H, D, L, N, dt, wdt):
    d = torch.device("cuda", 0)
    g = torch.Generator(device=d).manual_seed(B * 1000 + D + L)
    q = torch.randn(B, H, D, generator=g, device=d).to(dt)
    k = torch.randn(B, H, L, D, generator=g, device=d).to(dt)
    v = torch.randn(B, H, L, D, generator=g, device=d).to(dt)
    mask = (torch.rand(L, generator=g, device=d) > 0.3).float()
    mask[0] = 1.0
    rms_w = 1.0 + 0.1 * torch.randn(D, generator=g, device=d)
    w = 0.05 * torch.randn(N, D, generator=g, device=d)
    wscale = None
    if wdt == torch.float8_e4m3fn:
        amax = w.abs().amax(dim=1)
        wscale = amax / 448.0
        w = (w / wscale[:, None]).clamp(-448, 448)
    w = w.to(wdt)
    bias = torch.randn(N, generator=g, device=d)
    scale = 1.0 / math.sqrt(D)
    y = mk.fused_tree_attn_rmsnorm_linear(q, k, v, mask, w, rms_w=rms_w, proj_bias=bias, wscale=wscale,
                                          scale=scale, eps=1e-6)
    torch.cuda.synchronize()
    assert y.shape == (B, H, N) and y.dtype == dt
    ref = O.tree_attn_rmsnorm_linear(f32(q), f32(k), f32(v), f32(mask), f32(rms_w), f32(w), f32(bias),
                                     f32(wscale), scale, 1e-6)
    tol = 1e-4 if (dt == torch.float32 and wdt in (torch.float32, torch.float8_e4m3fn)) else 2e-2
    assert rel_err(f32(y), ref) <= tol
    import _mtp_native as N_
    assert N_.device_status(d) == 0


def test_no_kept_key_and_no_keys(mk):
    d = torch.device("cuda", 0)
    q = torch.randn(2, 2, 64, device=d)
    w = torch.randn(50, 64, device=d)
    k = torch.randn(2, 2, 5, 64, device=d)
    y = mk.fused_tree_attn_rmsnorm_linear(q, k, k, torch.zeros(5, device=d), w)
    assert torch.isnan(y).all()
    e = torch.empty(2, 2, 0, 64, device=d)
    y = mk.fused_tree_attn_rmsnorm_linear(q, e, e, torch.empty(0, device=d), w)
    assert torch.isnan(y).all()
