"""FP8-KV causal attention, plain causal attention and the INT4 matmul
((f)4), against golden vectors from the reference's eager functions
(tests/golden/quant_attention_int4.npz).  CPU: the oracle and the
host-side int4 helpers (torch) are bit-identical to the reference's.  GPU:
the kernels within fp32 summation-order tolerance (1e-5 of max|ref| for
the int4 matmul, 1e-5 for attention)."""

import math

import numpy as np
import pytest
import torch

from oracle import mtp_oracle as O


def rel_err(y, ref):
    y, ref = np.asarray(y, np.float64), np.asarray(ref, np.float64)
    return np.max(np.abs(y - ref)) / max(np.max(np.abs(ref)), 1e-30)


def test_oracle(golden):
    g = golden("quant_attention_int4.npz")
    k8, v8 = O.e4m3_bits_to_f32(g["k_bits"]), O.e4m3_bits_to_f32(g["v_bits"])
    D = g["q"].shape[-1]
    att8 = O.causal_attention_scaled(g["q"], k8, v8, g["kscale"], g["vscale"], 1.0 / math.sqrt(D))
    assert rel_err(att8, g["att8"]) <= 1e-5
    assert rel_err(O.causal_attention_scaled(g["q"], g["kf"], g["vf"], None, None, 0.2), g["att"]) <= 1e-5
    pk, sc = O.quantize_int4(g["w"], 32)
    assert np.array_equal(pk, g["packed"]) and np.array_equal(sc, g["scales"])
    assert np.array_equal(O.dequantize_int4(pk, sc, 96, 32), g["w_deq"])
    assert rel_err(O.int4_matmul(g["x"], pk, sc, 96, 32), g["y"]) <= 1e-5
    pk2, sc2 = O.quantize_int4(g["w2"], 32)
    assert np.array_equal(pk2, g["packed2"]) and np.array_equal(sc2, g["scales2"])
    assert rel_err(O.int4_matmul(g["x2"], pk2, sc2, 40, 32), g["y2"]) <= 1e-5


def test_torch_int4_helpers(golden):
    import mtp_kernels as mk
    g = golden("quant_attention_int4.npz")
    pk, sc = mk.quantize_int4(torch.tensor(g["w"]), group=32)
    assert np.array_equal(pk.numpy(), g["packed"]) and np.array_equal(sc.numpy(), g["scales"])
    assert np.array_equal(mk.dequantize_int4(pk, sc, 96, 32).numpy(), g["w_deq"])


@pytest.fixture(scope="module")
def mk():
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    import mtp_kernels
    return mtp_kernels


@pytest.mark.gpu
@pytest.mark.isolated
def test_device_attention(mk, golden):
    g = golden("quant_attention_int4.npz")
    d = torch.device("cuda", 0)
    q = torch.tensor(g["q"], device=d)
    k8 = torch.tensor(g["k_bits"], device=d).view(torch.float8_e4m3fn)
    v8 = torch.tensor(g["v_bits"], device=d).view(torch.float8_e4m3fn)
    out = mk.fused_causal_attention_fp8(q, k8, v8, torch.tensor(g["kscale"], device=d),
                                        torch.tensor(g["vscale"], device=d))
    assert rel_err(out.cpu().numpy(), g["att8"]) <= 1e-5
    out = mk.fused_causal_attention(q, torch.tensor(g["kf"], device=d), torch.tensor(g["vf"], device=d), 0.2)
    assert rel_err(out.cpu().numpy(), g["att"]) <= 1e-5
    # bf16 queries over an fp8 cache: the bf16 bar
    qb = q.to(torch.bfloat16)
    out = mk.fused_causal_attention_fp8(qb, k8, v8, torch.tensor(g["kscale"], device=d),
                                        torch.tensor(g["vscale"], device=d))
    ref = O.causal_attention_scaled(qb.float().cpu().numpy(), O.e4m3_bits_to_f32(g["k_bits"]),
                                    O.e4m3_bits_to_f32(g["v_bits"]), g["kscale"], g["vscale"], 1.0 / 8.0)
    assert rel_err(out.float().cpu().numpy(), ref) <= 2e-2


@pytest.mark.gpu
@pytest.mark.isolated
def test_device_int4(mk, golden):
    g = golden("quant_attention_int4.npz")
    d = torch.device("cuda", 0)
    y = mk.fused_int4_matmul(torch.tensor(g["x"], device=d), torch.tensor(g["packed"], device=d),
                             torch.tensor(g["scales"], device=d), 96, 32)
    assert rel_err(y.cpu().numpy(), g["y"]) <= 1e-5
    y = mk.fused_int4_matmul(torch.tensor(g["x2"], device=d), torch.tensor(g["packed2"], device=d),
                             torch.tensor(g["scales2"], device=d), 40, 32)
    assert rel_err(y.cpu().numpy(), g["y2"]) <= 1e-5


@pytest.mark.gpu
@pytest.mark.isolated
@pytest.mark.parametrize("M,N,K,group,dt", [
    (1, 4096, 4096, 128, torch.bfloat16),   # decode-sized: streamed GEMV kernel, one row of x
    (2, 1000, 1024, 32, torch.float32),
    (3, 777, 2048, 16, torch.float32),      # group 16: a scale per code pair of groups
    (5, 300, 4096, 64, torch.float16),
    (8, 14336, 4096, 128, torch.bfloat16),
    (130, 300, 1000, 32, torch.float32),    # tile kernel (K not a multiple of 32)
    (16, 14336, 4096, 64, torch.float16),   # tile kernel
])
def test_device_int4_sizes(mk, M, N, K, group, dt):
    d = torch.device("cuda", 0)
    gen = torch.Generator(device=d).manual_seed(M + N)
    W = torch.randn(N, K, generator=gen, device=d)
    pk, sc = mk.quantize_int4(W, group=group)
    x = torch.randn(M, K, generator=gen, device=d).to(dt)
    y = mk.fused_int4_matmul(x, pk, sc, K, group)
    ref = O.int4_matmul(x.float().cpu().numpy(), pk.cpu().numpy(), sc.cpu().numpy(), K, group)
    assert rel_err(y.float().cpu().numpy(), ref) <= (1e-5 if dt == torch.float32 else 1e-2)
