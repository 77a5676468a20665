"""Parity of the sm_100a kernels (through the drop-in modules and the C ABI)
against the CPU oracle on the same seeded inputs.  GPU only.

Tolerances (the benchmark specification's):
  * fp32 paths: max abs error <= 1e-4 (the reference's own bound,
    test_engine.py:5, mtp_engine.py:1644-1651);
  * bf16 GEMM outputs: ||y - ref||_inf / ||ref||_inf <= 2e-2 and
    allclose(rtol=2e-2, atol=2e-2 * rms(ref));
  * FP8: against the oracle evaluated on the dequantised operands, same bound;
  * argmax tokens / accept / accepted_n / corrected: bit-exact for every row
    whose fp32 top-2 logit margin exceeds MARGIN (rows inside it are
    reported, not failed).
"""

import math
import os

import numpy as np
import pytest
import torch

from oracle import mtp_oracle as O

pytestmark = pytest.mark.gpu

REL_TOL = 2e-2
MARGIN = 1e-3


@pytest.fixture(scope="module")
def mods():
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    import _mtp_native
    import mtp_fused_verify
    import mtp_kernels
    import mtp_parallel
    _mtp_native.lib()
    return mtp_kernels, mtp_fused_verify, mtp_parallel


def dev():
    return torch.device("cuda", 0)


def np32(t):
    return t.detach().float().cpu().numpy()


def check_rel(y, ref, tol=REL_TOL):
    y = np.asarray(y, np.float64)
    ref = np.asarray(ref, np.float64)
    rel = np.abs(y - ref).max() / max(np.abs(ref).max(), 1e-30)
    rms = math.sqrt(float((ref ** 2).mean()))
    assert rel <= tol, f"relative inf-norm error {rel:.3e} > {tol}"
    np.testing.assert_allclose(y, ref, rtol=tol, atol=tol * rms)
    return rel


def chain_rows_confident(hidden_np, w_np, bias_np, B, S):
    margin = O.top2_margin(hidden_np, w_np, bias_np).reshape(B, S)
    return (margin > MARGIN).all(axis=1), margin


# --------------------------------------------------------------------------- #
# golden fixtures (reference shapes, fp32 -> CUDA-core fp32 path)
# --------------------------------------------------------------------------- #
def test_rmsnorm_linear_fp32_golden(mods, golden):
    mk, _, _ = mods
    g = golden("rmsnorm_linear_fp32.npz")
    y = mk.fused_rmsnorm_linear(torch.tensor(g["x"], device=dev()), torch.tensor(g["w"], device=dev()),
                                torch.tensor(g["b"], device=dev()), 1e-6)
    assert y.dtype == torch.float32 and y.shape == (5, 128)
    assert np.abs(np32(y) - g["y"]).max() < 1e-4
    y2 = mk.fused_rmsnorm_linear(torch.tensor(g["x2"], device=dev()), torch.tensor(g["w2"], device=dev()),
                                 None, 1e-5, 0.5)
    assert np.abs(np32(y2) - g["y2"]).max() < 1e-4


def test_rmsnorm_linear_bf16_golden(mods, golden):
    mk, _, _ = mods
    g = golden("rmsnorm_linear_bf16.npz")
    x = torch.tensor(g["x_bits"].view(np.int16), device=dev()).view(torch.bfloat16)
    w = torch.tensor(g["w_bits"].view(np.int16), device=dev()).view(torch.bfloat16)
    y = mk.fused_rmsnorm_linear(x, w, None, 1e-5)
    assert y.dtype == torch.bfloat16
    check_rel(np32(y), O.bf16_bits_to_f32(g["y_bits"]))
    gam = torch.tensor(g["gamma"], device=dev())
    yg = mk.fused_rmsnorm_linear(x, w, None, 1e-5, norm_weight=gam)
    check_rel(np32(yg), g["y_gamma_f32"])


def test_rmsnorm_linear_fp8_golden(mods, golden):
    mk, _, _ = mods
    g = golden("rmsnorm_linear_fp8.npz")
    # the reference's self-check: fp32-valued clamped weight (no quantisation)
    y = mk.fused_rmsnorm_linear_fp8(torch.tensor(g["x"], device=dev()), torch.tensor(g["w_vals"], device=dev()),
                                    torch.tensor(g["wscale"], device=dev()))
    assert np.abs(np32(y) - g["y_selfcheck"]).max() < 1e-4
    # a genuine e4m3 weight: activations quantised per token in-kernel
    wq = torch.tensor(g["wq_bits"], device=dev()).view(torch.float8_e4m3fn)
    y = mk.fused_rmsnorm_linear_fp8(torch.tensor(g["xa"], device=dev()), wq, torch.tensor(g["wscale"], device=dev()),
                                    torch.tensor(g["bias"], device=dev()))
    assert np.abs(np32(y) - g["y_real"]).max() < 1e-4 * max(1.0, np.abs(g["y_real"]).max())


def test_verify_golden(mods, golden):
    _, mv, _ = mods
    g = golden("verify.npz")
    t = lambda a: torch.tensor(a, device=dev())
    acc, top = mv.fused_verify(t(g["h"]), t(g["w"]), t(g["d"]), t(g["b"]))
    assert acc.dtype == torch.int8 and top.dtype == torch.int32
    np.testing.assert_array_equal(acc.cpu().numpy(), g["accept1"])
    np.testing.assert_array_equal(top.cpu().numpy(), g["top1"])
    a, n, c = mv.fused_multi_verify(t(g["hm"]), t(g["wm"]), t(g["dm"]), t(g["bm"]))
    np.testing.assert_array_equal(a.cpu().numpy(), g["accept_m"])
    np.testing.assert_array_equal(n.cpu().numpy(), g["n_m"])
    np.testing.assert_array_equal(c.cpu().numpy(), g["corr_m"])
    # ties (duplicated lm_head rows) and every accept length 0..5
    a, n, c = mv.fused_multi_verify(t(g["h3"]), t(g["w3"]), t(g["d3"]))
    np.testing.assert_array_equal(a.cpu().numpy(), g["accept3"])
    np.testing.assert_array_equal(n.cpu().numpy(), g["n3"])
    np.testing.assert_array_equal(c.cpu().numpy(), g["corr3"])


def test_config1_chain(mods, golden):
    """benchmark config 1: rmsnorm_linear (gamma) -> fused_multi_verify, fp32."""
    mk, mv, _ = mods
    g = golden("config1.npz")
    gen = torch.Generator().manual_seed(0)
    x = torch.randn(1, 5, 256, generator=gen)
    gamma = 1.0 + 0.1 * torch.randn(256, generator=gen)
    w = 0.02 * torch.randn(256, 256, generator=gen)
    lm = 0.02 * torch.randn(4096, 256, generator=gen)
    y = mk.fused_rmsnorm_linear(x[0].to(dev()), w.to(dev()), None, 1e-6, norm_weight=gamma.to(dev()))
    assert np.abs(np32(y) - g["y"]).max() < 1e-4
    a, n, c = mv.fused_multi_verify(y[None], lm.to(dev()), torch.tensor(g["draft"], device=dev()))
    np.testing.assert_array_equal(a.cpu().numpy(), g["accept"])
    np.testing.assert_array_equal(n.cpu().numpy(), g["accepted_n"])
    np.testing.assert_array_equal(c.cpu().numpy(), g["corrected"])
    assert int(n[0]) == 2


def test_attention_golden(mods, golden):
    mk, _, _ = mods
    t = lambda a: torch.tensor(a, device=dev())
    g = golden("tree_attention.npz")
    s = 1.0 / math.sqrt(32)
    o = mk.fused_tree_attention(t(g["q"]), t(g["k"]), t(g["v"]), torch.ones(8, device=dev()))
    assert np.abs(np32(o) - g["o_ones"]).max() < 1e-4
    o = mk.fused_tree_attention(t(g["q"]), t(g["k"]), t(g["v"]), t(g["mask_part"]))
    assert np.abs(np32(o) - g["o_part"]).max() < 1e-4
    o = mk.fused_tree_attention(t(g["qL"]), t(g["kL"]), t(g["vL"]), t(g["mL"]), 0.125)
    assert np.abs(np32(o) - g["oL"]).max() < 1e-4
    g = golden("paged_attention.npz")
    o = mk.fused_paged_attention(t(g["q"]), t(g["k_pages"]), t(g["v_pages"]), t(g["page_table"]),
                                 int(g["page_size"][0]))
    assert np.abs(np32(o) - g["out"]).max() < 1e-4
    g = golden("tree_paged.npz")
    ctx, ps = (int(v) for v in g["meta"])
    o = mk.fused_tree_attention_paged(t(g["q"]), t(g["k_pages"]), t(g["v_pages"]), t(g["page_table"]),
                                      t(g["tree_k"]), t(g["tree_v"]), t(g["tree_mask"]), ctx_len=ctx)
    assert np.abs(np32(o) - g["out"]).max() < 1e-4


def test_tree_paged_reserve_built_table(mods, golden):
    """Page table from the reference's own PagedKVCache after reserve() of
    5, 1, 1, 16, 7, ... tokens and swap_logical_pages(): every context chunk
    is gathered token by token by the tensor-core kernel (and -1 entries read
    page P-1, as torch indexing does); the single-query operator on the same
    table through both decode kernels."""
    import _mtp_native as N
    mk, _, _ = mods
    g = golden("tree_paged_reserve.npz")
    ctx, ps = (int(v) for v in g["meta"])
    bf = lambda a: torch.tensor(a.view(np.int16), device=dev()).view(torch.bfloat16)
    N.device_status(dev())
    o = mk.fused_tree_attention_paged(bf(g["q_bits"]), bf(g["k_pages_bits"]), bf(g["v_pages_bits"]),
                                      torch.tensor(g["page_table"], device=dev()), bf(g["tree_k_bits"]),
                                      bf(g["tree_v_bits"]), torch.tensor(g["tree_mask"], device=dev()), ctx_len=ctx)
    check_rel(np32(o), g["out"])
    assert N.device_status(dev()) == 0
    table = torch.tensor(g["page_table"][:, :ctx], device=dev())
    prev = N.decode_kernel()
    for ver in (1, 2):
        N.set_decode_kernel(ver)
        try:
            o1 = mk.fused_paged_attention(bf(g["q1_bits"]), bf(g["k_pages_bits"]), bf(g["v_pages_bits"]), table, ps)
        finally:
            N.set_decode_kernel(prev)
        check_rel(np32(o1), g["out1"])
        assert N.device_status(dev()) == 0


@pytest.mark.parametrize("mode", ["per_token", "mixed"])
def test_tree_paged_per_token_tables(mods, mode):
    """Tables that are not page-granular at a config-4-like shape (GQA 4,
    64 tree nodes, 16-token pages): every token's page drawn on its own in
    [-P, P) ("per_token"), or page-granular chunks with one token moved in
    every other 128-token chunk ("mixed"), so both gathers of the
    tensor-core kernel run in one launch."""
    import _mtp_native as N
    mk, _, _ = mods
    B, Hq, Hkv, D, ps, ctx, P = 2, 32, 8, 128, 16, 1000, 128
    g = torch.Generator(device=dev()).manual_seed(31)
    rnd = lambda *shape: torch.randn(*shape, generator=g, device=dev()).to(torch.bfloat16)
    kp, vp = rnd(P, B, Hkv, ps, D), rnd(P, B, Hkv, ps, D)
    rng = np.random.default_rng(31)
    if mode == "per_token":
        table = rng.integers(-P, P, size=(B, ctx))
    else:
        pages = rng.permutation(P)[: (ctx + ps - 1) // ps * B].reshape(B, -1)
        table = np.repeat(pages, ps, axis=1)[:, :ctx]
        for c in range(0, ctx, 256):
            table[:, c + 5] = rng.integers(-P, P, size=B)
    table = np.ascontiguousarray(table, dtype=np.int32)
    _, tm = O.draft_tree(16, 4, "tree")
    T = tm.shape[0]
    q, tk, tv = rnd(B, T, Hq, D), rnd(B, Hkv, T, D), rnd(B, Hkv, T, D)
    N.device_status(dev())
    o = mk.fused_tree_attention_paged(q, kp, vp, torch.tensor(table, device=dev()), tk, tv,
                                      torch.tensor(tm, device=dev()), ctx_len=ctx)
    ref = O.tree_attention_paged_fast(np32(q), np32(kp), np32(vp), table, ctx, ps, np32(tk), np32(tv), tm,
                                      1.0 / math.sqrt(D))
    check_rel(np32(o), ref)
    assert N.device_status(dev()) == 0


# --------------------------------------------------------------------------- #
# bf16 / fp8 tensor-core paths
# --------------------------------------------------------------------------- #
@pytest.mark.parametrize("M,N,K", [(1, 40, 64), (100, 300, 192), (128, 256, 4096), (257, 1000, 520),
                                   (64, 14336, 4096)])
def test_rmsnorm_linear_bf16_shapes(mods, M, N, K):
    mk, _, _ = mods
    g = torch.Generator(device=dev()).manual_seed(M * 7 + N)
    x = torch.randn(M, K, generator=g, device=dev()).to(torch.bfloat16)
    w = (0.02 * torch.randn(N, K, generator=g, device=dev())).to(torch.bfloat16)
    b = torch.randn(N, generator=g, device=dev()).to(torch.bfloat16)
    gam = 1.0 + 0.1 * torch.randn(K, generator=g, device=dev())
    y = mk.fused_rmsnorm_linear(x, w, b, 1e-5, 0.75)
    ref = O.rmsnorm_linear(np32(x), np32(w), np32(b), 1e-5, 0.75)
    check_rel(np32(y), ref)
    yg = mk.fused_rmsnorm_linear(x, w, None, 1e-5, norm_weight=gam)
    refg = O.rmsnorm_linear(np32(x), np32(w) * np32(gam)[None, :], None, 1e-5, 1.0)
    check_rel(np32(yg), refg)


def test_config2_rmsnorm_linear_bf16(mods):
    """benchmark config 2 (seed 1): M=512, K=4096, N=14336, gamma 1+N(0,0.1), eps 1e-5."""
    mk, _, _ = mods
    M, K, N = 512, 4096, 14336
    g = torch.Generator(device=dev()).manual_seed(1)
    x = torch.randn(M, K, generator=g, device=dev()).to(torch.bfloat16)
    gam = 1.0 + 0.1 * torch.randn(K, generator=g, device=dev())
    w = (0.02 * torch.randn(N, K, generator=g, device=dev())).to(torch.bfloat16)
    y = mk.fused_rmsnorm_linear(x, w, None, 1e-5, norm_weight=gam)
    rows = np.r_[0:64, 448:512]
    ref = O.rmsnorm_linear(np32(x)[rows], np32(w) * np32(gam)[None, :], None, 1e-5, 1.0)
    check_rel(np32(y)[rows], ref)


def test_config3_fp8(mods):
    """benchmark config 3 (seed 2): M=1024, K=8192, N=28672 e4m3, rows scaled to amax 448,
    per-channel weight scales stored through pack_scales, bf16 out."""
    mk, _, _ = mods
    M, K, N = 1024, 8192, 28672
    g = torch.Generator(device=dev()).manual_seed(2)
    x = torch.randn(M, K, generator=g, device=dev())
    x = x * (448.0 / x.abs().amax(dim=1, keepdim=True))
    xq, sx = mk.quantize_fp8_rows(x)
    wq, sw = mk.quantize_fp8_rows(0.02 * torch.randn(N, K, generator=g, device=dev()))
    flat, offs = mk.pack_scales([sw])
    sw_view = mk.unpack_scale_tensor(flat, offs, 0, (N,))
    y = mk.fused_rmsnorm_linear_fp8(xq, wq, sw_view, x_scale=sx, out_dtype=torch.bfloat16)
    assert y.dtype == torch.bfloat16
    # in-kernel per-token quantisation of a bf16 input
    xb = x.to(torch.bfloat16)
    y2 = mk.fused_rmsnorm_linear_fp8(xb, wq, sw_view)
    rows = np.r_[0:32, 992:1024]
    w_deq = O.e4m3_bits_to_f32(wq.view(torch.uint8).cpu().numpy())
    x_deq = O.e4m3_bits_to_f32(xq.view(torch.uint8).cpu().numpy()[rows]) * np32(sx)[rows, None]
    check_rel(np32(y)[rows], O.rmsnorm_linear_fp8(x_deq, w_deq, np32(sw), None, 1e-6))
    # its own dequantised reference: the oracle quantises the same bf16 rows
    qb, sb = O.quantize_rows_e4m3(np32(xb)[rows])
    check_rel(np32(y2)[rows], O.rmsnorm_linear_fp8(O.e4m3_bits_to_f32(qb) * sb[:, None], w_deq, np32(sw),
                                                   None, 1e-6))


def test_fp8_quantisation_bits(mods):
    mk, _, _ = mods
    g = torch.Generator(device=dev()).manual_seed(5)
    x = (3.0 * torch.randn(37, 272, generator=g, device=dev()))
    wq, sw = mk.quantize_fp8_rows(0.05 * torch.randn(64, 272, generator=g, device=dev()))
    y = mk.fused_rmsnorm_linear_fp8(x, wq, sw, eps=1e-6)
    xb, sxb = O.quantize_rows_e4m3(np32(x))
    ref = O.rmsnorm_linear_fp8(O.e4m3_bits_to_f32(xb) * sxb[:, None],
                               O.e4m3_bits_to_f32(wq.view(torch.uint8).cpu().numpy()), np32(sw), None, 1e-6)
    assert np.abs(np32(y) - ref).max() <= 1e-4 * np.abs(ref).max() + 1e-5


@pytest.mark.parametrize("B,S,K,V,bias", [(2, 5, 64, 256, True), (8, 6, 512, 5003, False), (3, 1, 256, 300, True),
                                          (64, 6, 4096, 32064, False)])
def test_multi_verify_bf16(mods, B, S, K, V, bias):
    _, mv, _ = mods
    g = torch.Generator(device=dev()).manual_seed(B * 131 + V)
    hid = torch.randn(B, S, K, generator=g, device=dev()).to(torch.bfloat16)
    w = (0.02 * torch.randn(V, K, generator=g, device=dev())).to(torch.bfloat16)
    bvec = torch.randn(V, generator=g, device=dev()) * 0.1 if bias else None
    h_np, w_np = np32(hid), np32(w)
    b_np = None if bvec is None else np32(bvec)
    top = O.logits_f32(h_np.reshape(B * S, K), w_np, b_np).argmax(-1).reshape(B, S)
    rng = np.random.default_rng(B + V)
    draft = rng.integers(0, V, size=(B, S - 1))
    for b in range(B):
        a = b % S
        draft[b, :a] = top[b, 1:a + 1]
        if a < S - 1 and draft[b, a] == top[b, a + 1]:
            draft[b, a] = (draft[b, a] + 1) % V
    ref = O.chain_accept(top, draft)
    a, n, c = mv.fused_multi_verify(hid, w, torch.tensor(draft, device=dev()), bvec)
    ok, _ = chain_rows_confident(h_np, w_np, b_np, B, S)
    assert ok.mean() > 0.9
    np.testing.assert_array_equal(a.cpu().numpy()[ok], ref[0][ok])
    np.testing.assert_array_equal(n.cpu().numpy()[ok], ref[1][ok])
    np.testing.assert_array_equal(c.cpu().numpy()[ok], ref[2][ok])
    # the workspace is left at rest: a second call gives the same answer
    a2, n2, c2 = mv.fused_multi_verify(hid, w, torch.tensor(draft, device=dev()), bvec)
    assert torch.equal(a, a2) and torch.equal(n, n2) and torch.equal(c, c2)


def test_config5_verify_full(mods):
    """benchmark config 5 at tp=1 (seed 4): B=64, S=6, K=4096, V=128256 bf16, no bias."""
    _, mv, mp = mods
    B, S, K, V = 64, 6, 4096, 128256
    g = torch.Generator(device=dev()).manual_seed(4)
    hid = torch.randn(B, S, K, generator=g, device=dev()).to(torch.bfloat16)
    w = (0.02 * torch.randn(V, K, generator=g, device=dev())).to(torch.bfloat16)
    h_np, w_np = np32(hid), np32(w)
    logits = O.logits_f32(h_np.reshape(B * S, K), w_np, None)
    top = logits.argmax(-1).reshape(B, S)
    rng = np.random.default_rng(4)
    draft = rng.integers(0, V, size=(B, S - 1))
    for b in range(B):
        a = int(rng.integers(0, S))
        draft[b, :a] = top[b, 1:a + 1]
        if a < S - 1:
            while draft[b, a] == top[b, a + 1]:
                draft[b, a] = rng.integers(0, V)
    ref = O.chain_accept(top, draft)
    part = np.partition(logits, -2, axis=-1)
    ok = ((part[:, -1] - part[:, -2]) > MARGIN).reshape(B, S).all(axis=1)
    d_t = torch.tensor(draft, device=dev())
    a, n, c = mv.fused_multi_verify(hid, w, d_t)
    np.testing.assert_array_equal(a.cpu().numpy()[ok], ref[0][ok])
    np.testing.assert_array_equal(n.cpu().numpy()[ok], ref[1][ok])
    np.testing.assert_array_equal(c.cpu().numpy()[ok], ref[2][ok])
    # the vocab-sharded pieces on one device: 4 shards folded into one key buffer
    import _mtp_native as N
    keys = torch.full((B * S,), -(2 ** 63), dtype=torch.int64, device=dev())
    for r in range(4):
        ws, off = mp.shard_lm_head(w, 4, r)
        N.check(N.lib().mtp_verify_shard_keys(N.ptr(hid), N.DT_BF16, N.ptr(ws), N.DT_BF16, None, 0, N.ptr(keys),
                                              B * S, K, ws.shape[0], off, N.stream_handle(dev())), "shard")
    a4 = torch.empty_like(a)
    n4 = torch.empty_like(n)
    c4 = torch.empty_like(c)
    N.check(N.lib().mtp_verify_chain_from_keys(N.ptr(keys), N.ptr(d_t.to(torch.int32)), N.ptr(a4), N.ptr(n4),
                                               N.ptr(c4), B, S, N.stream_handle(dev())), "chain")
    assert torch.equal(a4, a) and torch.equal(n4, n) and torch.equal(c4, c)
    assert int(keys.max()) == -(2 ** 63)  # reset to rest


def test_fused_verify_single_bf16(mods):
    _, mv, _ = mods
    g = torch.Generator(device=dev()).manual_seed(9)
    M, K, V = 77, 1024, 7777
    h = torch.randn(M, K, generator=g, device=dev()).to(torch.bfloat16)
    w = (0.02 * torch.randn(V, K, generator=g, device=dev())).to(torch.bfloat16)
    top_ref = O.logits_f32(np32(h), np32(w), None).argmax(-1).astype(np.int32)
    draft = top_ref.copy()
    draft[::3] = (draft[::3] + 1) % V
    acc, top = mv.fused_verify(h, w, torch.tensor(draft, device=dev()))
    ok = O.top2_margin(np32(h), np32(w), None) > MARGIN
    np.testing.assert_array_equal(top.cpu().numpy()[ok], top_ref[ok])
    np.testing.assert_array_equal(acc.cpu().numpy()[ok], (top_ref == draft).astype(np.int8)[ok])


def test_config4_tree_attention_paged(mods):
    """benchmark config 4 (seed 3): B=16, Hq=32, Hkv=8, D=128, page 16, ctx 4096 over a
    randomly permuted 4096-page pool, 64-node tree (depth 16, 4 branches), bf16."""
    mk, _, _ = mods
    B, Hq, Hkv, D, ps, ctx, P = 16, 32, 8, 128, 16, 4096, 4096
    _, tmask = O.draft_tree(16, 4, "tree")
    T = tmask.shape[0]
    g = torch.Generator(device=dev()).manual_seed(3)
    kp = torch.randn(P, B, Hkv, ps, D, generator=g, device=dev()).to(torch.bfloat16)
    vp = torch.randn(P, B, Hkv, ps, D, generator=g, device=dev()).to(torch.bfloat16)
    perm = torch.randperm(P, generator=torch.Generator().manual_seed(3))
    pages_per_seq = ctx // ps
    table = torch.empty(B, ctx, dtype=torch.int32)
    for b in range(B):
        table[b] = perm[b * pages_per_seq:(b + 1) * pages_per_seq].repeat_interleave(ps).to(torch.int32)
    q = torch.randn(B, T, Hq, D, generator=g, device=dev()).to(torch.bfloat16)
    tk = torch.randn(B, Hkv, T, D, generator=g, device=dev()).to(torch.bfloat16)
    tv = torch.randn(B, Hkv, T, D, generator=g, device=dev()).to(torch.bfloat16)
    out = mk.fused_tree_attention_paged(q, kp, vp, table.to(dev()), tk, tv, torch.tensor(tmask, device=dev()))
    assert out.shape == (B, T, Hq, D) and out.dtype == torch.bfloat16
    # oracle on a subset of sequences and nodes
    bs = [0, 15]
    nodes = [0, 1, 5, 21, 63]
    sub_pages = table[bs].unique().long()
    remap = torch.full((P,), -1, dtype=torch.int64)
    remap[sub_pages] = torch.arange(sub_pages.numel())
    kp_s = np32(kp[sub_pages.to(dev())][:, bs])
    vp_s = np32(vp[sub_pages.to(dev())][:, bs])
    tab_s = remap[table[bs].long()].numpy()
    ref = O.tree_attention_paged(np32(q[bs][:, nodes]), kp_s, vp_s, tab_s, ctx, ps, np32(tk[bs]), np32(tv[bs]),
                                 tmask[np.ix_(nodes, list(range(T)))], 1.0 / math.sqrt(D))
    # the oracle got only the selected query nodes but every tree key: select the rows
    check_rel(np32(out[bs][:, nodes]), ref)


def test_edge_cases(mods):
    mk, mv, _ = mods
    d = dev()
    # empty batch
    a, n, c = mv.fused_multi_verify(torch.zeros(0, 3, 64, device=d), torch.randn(10, 64, device=d),
                                    torch.zeros(0, 2, dtype=torch.int32, device=d))
    assert a.shape == (0, 2) and n.shape == (0,)
    # no drafts (S = 1): only the anchor
    h = torch.randn(4, 1, 32, device=d)
    w = torch.randn(50, 32, device=d)
    a, n, c = mv.fused_multi_verify(h, w, torch.zeros(4, 0, dtype=torch.int32, device=d))
    assert a.shape == (4, 0) and int(n.abs().sum()) == 0
    np.testing.assert_array_equal(c.cpu().numpy(), O.logits_f32(np32(h[:, 0]), np32(w), None).argmax(-1))
    # K not a multiple of 8 -> CUDA-core path for bf16
    x = torch.randn(33, 65, device=d).to(torch.bfloat16)
    wt = torch.randn(70, 65, device=d).to(torch.bfloat16)
    check_rel(np32(mk.fused_rmsnorm_linear(x, wt)), O.rmsnorm_linear(np32(x), np32(wt), None, 1e-6, 1.0))
    # shape errors are assertions, like the reference's
    with pytest.raises(AssertionError):
        mv.fused_multi_verify(torch.randn(2, 4, 8, device=d), torch.randn(9, 8, device=d),
                              torch.zeros(2, 2, dtype=torch.int32, device=d))
    with pytest.raises(ValueError):
        mk.fused_rmsnorm_linear(torch.randn(2, 8), torch.randn(4, 8))
    # all-masked tree row -> NaN like the reference's eager softmax
    q = torch.randn(1, 1, 16, device=d)
    k = torch.randn(1, 1, 4, 16, device=d)
    o = mk.fused_tree_attention(q, k, k, torch.zeros(4, device=d))
    assert torch.isnan(o).all()


def test_device_status_clean(mods):
    import _mtp_native as N
    assert N.device_status(dev()) == 0
