"""CUDA-graph capture and replay of the operators (the reference checks
graph == sync for its own path, mtp_engine.py:1836-1855): every replay must
give bit-for-bit the eager result -- the kernels are deterministic, launch on
the caller's stream, allocate nothing and leave their workspaces at rest, so
the verify's keys and ticket are ready again for the next replay.  GPU only;
runs in a child process (tests/test_gpu_isolated.py)."""

import numpy as np
import pytest
import torch

from oracle import mtp_oracle as O

pytestmark = [pytest.mark.gpu, pytest.mark.isolated]


@pytest.fixture(scope="module")
def mods():
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    import mtp_fused_verify as mv
    import mtp_kernels as mk
    return mk, mv


def replay_matches(fn, outs_eager, replays=3):
    """Warm up on a side stream (workspaces get allocated there first), capture
    fn, replay it and compare every output with the eager run."""
    s = torch.cuda.Stream()
    s.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(s):
        fn()
    torch.cuda.current_stream().wait_stream(s)
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g, stream=s):
        outs = fn()
    outs = outs if isinstance(outs, tuple) else (outs,)
    for _ in range(replays):
        g.replay()
        torch.cuda.synchronize()
        for a, b in zip(outs, outs_eager):
            assert torch.equal(a, b)
    del g


def test_rmsnorm_linear_graph(mods):
    mk, _ = mods
    d = torch.device("cuda", 0)
    gen = torch.Generator(device=d).manual_seed(1)
    x = torch.randn(256, 1024, generator=gen, device=d).to(torch.bfloat16)
    w = (0.02 * torch.randn(2048, 1024, generator=gen, device=d)).to(torch.bfloat16)
    gam = 1.0 + 0.1 * torch.randn(1024, generator=gen, device=d)
    fn = lambda: mk.fused_rmsnorm_linear(x, w, None, 1e-5, norm_weight=gam)
    ref = fn()
    torch.cuda.synchronize()
    assert torch.equal(fn(), ref)  # deterministic
    replay_matches(fn, (ref,))


def test_tree_attention_paged_graph(mods):
    mk, _ = mods
    d = torch.device("cuda", 0)
    gen = torch.Generator(device=d).manual_seed(2)
    B, Hq, Hkv, D, ps, ctx = 3, 16, 4, 128, 16, 512
    _, tm = O.draft_tree(8, 4, "tree")
    T = tm.shape[0]
    P = B * ctx // ps + 2
    kp = torch.randn(P, B, Hkv, ps, D, generator=gen, device=d).to(torch.bfloat16)
    vp = torch.randn(P, B, Hkv, ps, D, generator=gen, device=d).to(torch.bfloat16)
    perm = torch.randperm(P, generator=torch.Generator().manual_seed(2))
    per = ctx // ps
    table = torch.stack([perm[b * per:(b + 1) * per].repeat_interleave(ps) for b in range(B)]).to(torch.int32).to(d)
    q = torch.randn(B, T, Hq, D, generator=gen, device=d).to(torch.bfloat16)
    tk = torch.randn(B, Hkv, T, D, generator=gen, device=d).to(torch.bfloat16)
    tv = torch.randn(B, Hkv, T, D, generator=gen, device=d).to(torch.bfloat16)
    tmd = torch.tensor(tm, device=d)
    fn = lambda: mk.fused_tree_attention_paged(q, kp, vp, table, tk, tv, tmd)
    ref = fn()
    torch.cuda.synchronize()
    assert torch.equal(fn(), ref)
    replay_matches(fn, (ref,))


def test_multi_verify_and_step_graph(mods):
    _, mv = mods
    d = torch.device("cuda", 0)
    gen = torch.Generator(device=d).manual_seed(3)
    B, S, K, V = 8, 6, 1024, 20000
    hid = torch.randn(B, S, K, generator=gen, device=d).to(torch.bfloat16)
    w = (0.02 * torch.randn(V, K, generator=gen, device=d)).to(torch.bfloat16)
    draft = torch.randint(0, V, (B, S - 1), generator=gen, device=d, dtype=torch.int32)
    ref = mv.fused_multi_verify(hid, w, draft)
    torch.cuda.synchronize()
    replay_matches(lambda: mv.fused_multi_verify(hid, w, draft), ref)
    step_ref = mv.fused_multi_verify_step(hid, w, draft)
    torch.cuda.synchronize()
    replay_matches(lambda: mv.fused_multi_verify_step(hid, w, draft), step_ref)
    np.testing.assert_array_equal(step_ref[0].cpu().numpy(), ref[0].cpu().numpy())
