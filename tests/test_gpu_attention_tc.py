"""Tensor-core paged tree attention against the oracle over the shapes it
accepts: GQA group sizes, one or two 128-row query tiles, ragged context
lengths (partial pages and chunks), no context at all, several page sizes,
and few (sequence, KV head) units so the key range is split over CTAs and
merged.  bf16 tolerance: ||out - ref||_inf / ||ref||_inf <= 2e-2.  GPU only."""

import math

import numpy as np
import pytest
import torch

from oracle import mtp_oracle as O

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def mk():
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    import mtp_kernels
    return mtp_kernels


def f32(t):
    return t.detach().float().cpu().numpy()


def run_case(mk, B, Hq, Hkv, T_depth, T_br, ctx, ps, P=None, dtype=torch.bfloat16, seed=0, causal_only=False):
    dev = torch.device("cuda", 0)
    _, tmask = O.draft_tree(T_depth, T_br, "trunk" if causal_only else "tree")
    T = tmask.shape[0]
    D = 128
    pages_per_seq = max(1, -(-ctx // ps))
    P = P or pages_per_seq * B + 3
    g = torch.Generator(device=dev).manual_seed(seed)
    kp = torch.randn(P, B, Hkv, ps, D, generator=g, device=dev).to(dtype)
    vp = torch.randn(P, B, Hkv, ps, D, generator=g, device=dev).to(dtype)
    perm = torch.randperm(P, generator=torch.Generator().manual_seed(seed))
    width = pages_per_seq * ps
    table = torch.stack([perm[b * pages_per_seq:(b + 1) * pages_per_seq].repeat_interleave(ps)
                         for b in range(B)]).to(torch.int32) if ctx > 0 else torch.zeros(B, 1, dtype=torch.int32)
    q = torch.randn(B, T, Hq, D, generator=g, device=dev).to(dtype)
    tk = torch.randn(B, Hkv, T, D, generator=g, device=dev).to(dtype)
    tv = torch.randn(B, Hkv, T, D, generator=g, device=dev).to(dtype)
    out = mk.fused_tree_attention_paged(q, kp, vp, table.to(dev), tk, tv, torch.tensor(tmask, device=dev),
                                        ctx_len=ctx)
    ref = O.tree_attention_paged_fast(f32(q), f32(kp), f32(vp), table.numpy()[:, :max(ctx, 1)], ctx, ps,
                                      f32(tk), f32(tv), tmask, 1.0 / math.sqrt(D))
    got = f32(out)
    rel = np.abs(got - ref).max() / np.abs(ref).max()
    assert rel <= 2e-2, f"rel err {rel:.3e}"
    return rel


@pytest.mark.parametrize("B,Hq,Hkv,depth,br,ctx,ps", [
    (2, 8, 2, 4, 2, 64, 16),       # G=4, one tile, partial chunk, split + merge
    (3, 32, 8, 16, 4, 300, 16),    # config-4 head geometry, 64 nodes x 4 = 256 rows (2 tiles), ragged ctx
    (1, 16, 2, 8, 4, 1000, 8),     # G=8, ctx not a multiple of the page, page 8
    (2, 4, 4, 4, 8, 513, 32),      # G=1, 32 nodes, page 32
    (2, 8, 1, 8, 4, 0, 16),        # no context: tree keys only
    (4, 64, 8, 16, 2, 2048, 64),   # G=8 x 32 nodes = 256 rows, page 64
])
def test_tree_attention_tc_shapes(mk, B, Hq, Hkv, depth, br, ctx, ps):
    run_case(mk, B, Hq, Hkv, depth, br, ctx, ps)


def test_tree_attention_tc_f16_trunk(mk):
    run_case(mk, 2, 16, 4, 12, 1, 777, 16, dtype=torch.float16, causal_only=True)


def test_tree_attention_tc_large_scores(mk):
    """Scores far above the lazy-rescale threshold: the running max jumps
    between chunks, so O must be rescaled in TMEM."""
    dev = torch.device("cuda", 0)
    B, Hq, Hkv, ps, ctx = 1, 8, 2, 16, 700
    _, tmask = O.draft_tree(4, 2, "tree")
    T = tmask.shape[0]
    pages = -(-ctx // ps)
    g = torch.Generator(device=dev).manual_seed(5)
    kp = torch.randn(pages, B, Hkv, ps, 128, generator=g, device=dev)
    kp[pages // 2] *= 6.0  # a late page with much larger scores
    kp = kp.to(torch.bfloat16)
    vp = torch.randn(pages, B, Hkv, ps, 128, generator=g, device=dev).to(torch.bfloat16)
    table = torch.arange(pages, dtype=torch.int32).repeat_interleave(ps)[None, :ctx]
    q = (3.0 * torch.randn(B, T, Hq, 128, generator=g, device=dev)).to(torch.bfloat16)
    tk = torch.randn(B, Hkv, T, 128, generator=g, device=dev).to(torch.bfloat16)
    tv = torch.randn(B, Hkv, T, 128, generator=g, device=dev).to(torch.bfloat16)
    out = mk.fused_tree_attention_paged(q, kp, vp, table.to(dev), tk, tv, torch.tensor(tmask, device=dev))
    ref = O.tree_attention_paged_fast(f32(q), f32(kp), f32(vp), table.numpy(), ctx, ps, f32(tk), f32(tv), tmask,
                                      1.0 / math.sqrt(128))
    rel = np.abs(f32(out) - ref).max() / np.abs(ref).max()
    assert rel <= 2e-2, rel
    import _mtp_native
    assert _mtp_native.device_status(dev) == 0
