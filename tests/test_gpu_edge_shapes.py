"""More shapes for the validated default kernels, against the CPU oracle:
output widths that end inside a 32-column store group, f16 with a bias and a
scale, single rows, the single-row verify (fused_verify) over a vocabulary
that is not a multiple of any tile, bf16 biases, and paged tree attention
with 1 and 8 query heads per KV head, 32-token pages, a context that ends
inside a page and a chunk, and one-node and odd-sized trees.  Tolerances as
in tests/test_gpu_parity.py (bf16/f16: inf-norm relative 2e-2; tokens
bit-exact on rows whose fp32 top-2 margin exceeds 1e-3).  GPU only; runs in
a child process (tests/test_gpu_isolated.py)."""

import math

import numpy as np
import pytest
import torch

from oracle import mtp_oracle as O

pytestmark = [pytest.mark.gpu, pytest.mark.isolated]

REL_TOL = 2e-2
MARGIN = 1e-3


@pytest.fixture(scope="module")
def mods():
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    import _mtp_native as N
    import mtp_fused_verify as mv
    import mtp_kernels as mk
    from mtp_draft_tree import SpeculativeDraftTree
    N.lib()
    return N, mk, mv, SpeculativeDraftTree


def dev():
    return torch.device("cuda", 0)


def np32(t):
    return t.detach().float().cpu().numpy()


def rel_err(y, ref):
    y, ref = np.asarray(y, np.float64), np.asarray(ref, np.float64)
    return np.abs(y - ref).max() / max(np.abs(ref).max(), 1e-30)


@pytest.mark.parametrize("M,N,K,dt,bias,scale", [
    (7, 1000, 256, torch.float16, True, 0.5),      # N ends inside a 32-column group
    (1, 333, 512, torch.bfloat16, True, 1.0),      # one row
    (129, 4104, 1024, torch.bfloat16, False, 2.0),
    (64, 14336, 4096, torch.bfloat16, False, 1.0),  # the M=64 line of the config-2 sweep
])
def test_rmsnorm_linear_shapes(mods, M, N, K, dt, bias, scale):
    _, mk, _, _ = mods
    g = torch.Generator(device=dev()).manual_seed(M + N)
    x = torch.randn(M, K, generator=g, device=dev()).to(dt)
    w = (0.02 * torch.randn(N, K, generator=g, device=dev())).to(dt)
    b = (0.1 * torch.randn(N, generator=g, device=dev())).to(dt) if bias else None
    gam = 1.0 + 0.1 * torch.randn(K, generator=g, device=dev())
    y = mk.fused_rmsnorm_linear(x, w, b, 1e-5, scale, norm_weight=gam)
    assert y.dtype == dt and y.shape == (M, N)
    rows = list(range(min(M, 8)))
    ref = O.rmsnorm_linear(np32(x[rows]), np32(w) * np32(gam)[None, :], np32(b) if bias else None, 1e-5, scale)
    assert rel_err(np32(y[rows]), ref) <= REL_TOL


@pytest.mark.parametrize("M,K,V,bias_dt", [(5, 256, 50021, torch.bfloat16), (33, 512, 7, None),
                                           (1, 4096, 128256, torch.float32)])
def test_fused_verify_single_row(mods, M, K, V, bias_dt):
    N, _, mv, _ = mods
    g = torch.Generator(device=dev()).manual_seed(M + V)
    h = torch.randn(M, K, generator=g, device=dev()).to(torch.bfloat16)
    w = (0.05 * torch.randn(V, K, generator=g, device=dev())).to(torch.bfloat16)
    b = (0.1 * torch.randn(V, generator=g, device=dev())).to(bias_dt) if bias_dt is not None else None
    top = O.logits_f32(np32(h), np32(w), np32(b) if b is not None else None).argmax(-1)
    draft = torch.tensor(top, dtype=torch.int32, device=dev())
    draft[::2] = (draft[::2] + 1) % V  # every other row rejected
    accept, got_top = mv.fused_verify(h, w, draft, b)
    margin = O.top2_margin(np32(h)[:, None, :], np32(w), np32(b) if b is not None else None).reshape(-1)
    ok = margin > MARGIN
    assert ok.mean() >= 0.9
    np.testing.assert_array_equal(got_top.cpu().numpy()[ok], top[ok])
    want_accept = (draft.cpu().numpy() == top).astype(np.int8)
    np.testing.assert_array_equal(accept.cpu().numpy()[ok], want_accept[ok])
    assert N.device_status(dev()) == 0


@pytest.mark.parametrize("B,Hq,Hkv,ps,ctx,depth,br", [
    (3, 8, 8, 32, 1000, 1, 1),    # G = 1, one-node tree, context ends inside a page
    (2, 32, 4, 16, 777, 3, 7),    # G = 8, 21-node tree
    (4, 16, 4, 8, 130, 4, 2),     # 8-token pages, context just past one chunk
])
def test_tree_attention_paged_shapes(mods, B, Hq, Hkv, ps, ctx, depth, br):
    N, mk, _, Tree = mods
    D = 128
    tm = Tree(depth, br, "tree").tree_mask.numpy()
    T = tm.shape[0]
    per = -(-ctx // ps)
    P = B * per + 2
    g = torch.Generator(device=dev()).manual_seed(B * 100 + ctx)
    kp = torch.randn(P, B, Hkv, ps, D, generator=g, device=dev()).to(torch.bfloat16)
    vp = torch.randn(P, B, Hkv, ps, D, generator=g, device=dev()).to(torch.bfloat16)
    perm = torch.randperm(P, generator=torch.Generator().manual_seed(ctx))
    table = torch.stack([perm[b * per:(b + 1) * per].repeat_interleave(ps)[:ctx] for b in range(B)]).to(torch.int32)
    q = torch.randn(B, T, Hq, D, generator=g, device=dev()).to(torch.bfloat16)
    tk = torch.randn(B, Hkv, T, D, generator=g, device=dev()).to(torch.bfloat16)
    tv = torch.randn(B, Hkv, T, D, generator=g, device=dev()).to(torch.bfloat16)
    out = mk.fused_tree_attention_paged(q, kp, vp, table.to(dev()), tk, tv, torch.tensor(tm, device=dev()))
    torch.cuda.synchronize()
    ref = O.tree_attention_paged(np32(q), np32(kp), np32(vp), table.numpy(), ctx, ps, np32(tk), np32(tv), tm,
                                 1.0 / math.sqrt(D))
    assert rel_err(np32(out), ref) <= REL_TOL
    assert N.device_status(dev()) == 0


@pytest.mark.parametrize("M,N,K,bias", [(1, 300, 512, True), (70, 1000, 256, False), (256, 520, 4096, True)])
def test_rmsnorm_linear_fp8_shapes(mods, M, N, K, bias):
    """E4M3 weight with per-channel scales, activations quantised per token
    in the row pre-pass: against the oracle on the dequantised operands
    (the activation codes are recomputed from x as the kernel does)."""
    _, mk, _, _ = mods
    g = torch.Generator(device=dev()).manual_seed(M + N + K)
    x = torch.randn(M, K, generator=g, device=dev()).to(torch.bfloat16)
    wq, sw = mk.quantize_fp8_rows(0.05 * torch.randn(N, K, generator=g, device=dev()))
    b = (0.1 * torch.randn(N, generator=g, device=dev())).to(torch.bfloat16) if bias else None
    y = mk.fused_rmsnorm_linear_fp8(x, wq, sw, b, 1e-6)
    assert y.dtype == torch.bfloat16 and y.shape == (M, N)
    xq, sx = mk.quantize_fp8_rows(x)
    rows = list(range(min(M, 6)))
    xd = O.e4m3_bits_to_f32(xq[rows].view(torch.uint8).cpu().numpy()) * np32(sx)[rows, None]
    wd = O.e4m3_bits_to_f32(wq.view(torch.uint8).cpu().numpy())
    ref = O.rmsnorm_linear_fp8(xd, wd, np32(sw), np32(b) if bias else None, 1e-6)
    assert rel_err(np32(y[rows]), ref) <= REL_TOL


@pytest.mark.parametrize("B,H,L,D,dt", [(2, 3, 1, 72, torch.bfloat16), (1, 2, 300, 200, torch.float16),
                                        (4, 1, 2049, 256, torch.bfloat16), (2, 2, 17, 40, torch.float32)])
def test_single_query_tree_attention_shapes(mods, B, H, L, D, dt):
    """fused_tree_attention (default single-query kernel) for head sizes
    that are not powers of two, one key, fp32, and a context past 2048."""
    N, mk, _, _ = mods
    g = torch.Generator(device=dev()).manual_seed(B + H + L + D)
    q = torch.randn(B, H, D, generator=g, device=dev()).to(dt)
    k = torch.randn(B, H, L, D, generator=g, device=dev()).to(dt)
    v = torch.randn(B, H, L, D, generator=g, device=dev()).to(dt)
    mask = (torch.rand(L, generator=g, device=dev()) < 0.8).float()
    mask[0] = 1.0
    out = mk.fused_tree_attention(q, k, v, mask)
    ref = O.tree_attention(np32(q), np32(k), np32(v), np32(mask), 1.0 / math.sqrt(D))
    assert rel_err(np32(out), ref) <= (1e-4 if dt == torch.float32 else REL_TOL)
    assert N.device_status(dev()) == 0
