"""The second single-query attention kernel (mtp_set_decode_kernel(2)) behind
fused_tree_attention and fused_paged_attention, against the CPU oracle
(_eager_tree_attention, mtp_kernels.py:859-872; _eager_paged_attention,
832-856) and against the first kernel.  Tolerance: the bf16/f16 bar,
max|out - ref| <= 2e-2 max|ref| (outputs are rounded to the input dtype).
GPU only; runs in a child process (tests/test_gpu_isolated.py)."""

import math

import numpy as np
import pytest
import torch

from oracle import mtp_oracle as O

pytestmark = [pytest.mark.gpu, pytest.mark.isolated]


@pytest.fixture(scope="module")
def mods():
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    import _mtp_native as N
    import mtp_kernels as mk
    before = N.decode_kernel()
    yield N, mk
    N.set_decode_kernel(before)


def f32(t):
    return t.detach().float().cpu().numpy()


def rel_err(y, ref):
    y, ref = np.asarray(y, np.float64), np.asarray(ref, np.float64)
    return np.max(np.abs(y - ref)) / max(np.max(np.abs(ref)), 1e-30)


@pytest.mark.parametrize("B,H,L,D,dt,p_keep", [
    (2, 3, 37, 128, torch.bfloat16, 0.7),
    (4, 8, 4096, 128, torch.bfloat16, 0.9),   # more keys than one pass of the CTA
    (3, 2, 300, 64, torch.float16, 0.5),
    (2, 2, 129, 256, torch.bfloat16, 1.0),
    (1, 4, 1, 32, torch.bfloat16, 1.0),
    (2, 2, 50, 8, torch.float16, 0.6),
])
def test_tree_attention(mods, B, H, L, D, dt, p_keep):
    N, mk = mods
    d = torch.device("cuda", 0)
    g = torch.Generator(device=d).manual_seed(B + L + D)
    q = torch.randn(B, H, D, generator=g, device=d).to(dt)
    k = torch.randn(B, H, L, D, generator=g, device=d).to(dt)
    v = torch.randn(B, H, L, D, generator=g, device=d).to(dt)
    mask = (torch.rand(L, generator=g, device=d) < p_keep).float()
    mask[0] = 1.0
    N.set_decode_kernel(1)
    o1 = mk.fused_tree_attention(q, k, v, mask)
    N.set_decode_kernel(2)
    o2 = mk.fused_tree_attention(q, k, v, mask)
    torch.cuda.synchronize()
    ref = O.tree_attention(f32(q), f32(k), f32(v), f32(mask), 1.0 / math.sqrt(D))
    assert rel_err(f32(o2), ref) <= 2e-2
    assert rel_err(f32(o2), f32(o1)) <= 2e-2
    assert N.device_status(d) == 0


@pytest.mark.parametrize("B,H,L,D,ps", [(2, 4, 1000, 128, 16), (3, 2, 64, 64, 8), (1, 8, 4096, 128, 64)])
def test_paged_attention(mods, B, H, L, D, ps):
    N, mk = mods
    d = torch.device("cuda", 0)
    g = torch.Generator(device=d).manual_seed(B * 7 + L)
    per = -(-L // ps)
    P = B * per + 3
    kp = torch.randn(P, B, H, ps, D, generator=g, device=d).to(torch.bfloat16)
    vp = torch.randn(P, B, H, ps, D, generator=g, device=d).to(torch.bfloat16)
    perm = torch.randperm(P, generator=torch.Generator().manual_seed(L))
    table = torch.stack([perm[b * per:(b + 1) * per].repeat_interleave(ps)[:L] for b in range(B)]).to(torch.int32)
    q = torch.randn(B, H, D, generator=g, device=d).to(torch.bfloat16)
    N.set_decode_kernel(2)
    out = mk.fused_paged_attention(q, kp, vp, table.to(d), ps)
    torch.cuda.synchronize()
    ref = O.paged_attention(f32(q), f32(kp), f32(vp), table.numpy(), ps, 1.0 / math.sqrt(D))
    assert rel_err(f32(out), ref) <= 2e-2
    assert N.device_status(d) == 0


def test_empty_and_masked_rows(mods):
    N, mk = mods
    d = torch.device("cuda", 0)
    N.set_decode_kernel(2)
    q = torch.randn(2, 2, 128, device=d).to(torch.bfloat16)
    k = torch.randn(2, 2, 9, 128, device=d).to(torch.bfloat16)
    out = mk.fused_tree_attention(q, k, k, torch.zeros(9, device=d))
    assert torch.isnan(out.float()).all()
    e = torch.empty(2, 2, 0, 128, device=d, dtype=torch.bfloat16)
    out = mk.fused_tree_attention(q, e, e, torch.empty(0, device=d))
    assert torch.isnan(out.float()).all()
    assert N.device_status(d) == 0


def test_bad_page_recorded(mods):
    N, mk = mods
    d = torch.device("cuda", 0)
    N.set_decode_kernel(2)
    kp = torch.randn(2, 1, 1, 4, 64, device=d).to(torch.bfloat16)
    table = torch.tensor([[0, 0, 0, 0, 9, 9, 9, 9]], dtype=torch.int32, device=d)  # page 9 is outside the pool
    q = torch.randn(1, 1, 64, device=d).to(torch.bfloat16)
    N.device_status(d)
    out = mk.fused_paged_attention(q, kp, kp, table, 4)
    assert N.device_status(d) == 7  # MTP_ERR_DEVICE; the bad keys are skipped
    kk = f32(kp[0, 0, 0])[None, None]  # the four valid keys: page 0, slots 0..3
    ref = O.tree_attention(f32(q), kk, kk, np.ones(4, np.float32), 1 / 8.0)
    assert rel_err(f32(out), ref) <= 2e-2
