"""Pin the CPU oracle against golden vectors produced by the reference's own
eager functions (tests/golden/make_golden.py).  CPU only."""

import math

import numpy as np
import pytest

from oracle import mtp_oracle as O


def test_rmsnorm_linear_fp32(golden):
    g = golden("rmsnorm_linear_fp32.npz")
    y = O.rmsnorm_linear(g["x"], g["w"], g["b"], 1e-6, 1.0)
    np.testing.assert_allclose(y, g["y"], rtol=1e-5, atol=1e-5)
    y2 = O.rmsnorm_linear(g["x2"], g["w2"], None, 1e-5, 0.5)
    np.testing.assert_allclose(y2, g["y2"], rtol=1e-5, atol=1e-5)


def test_rmsnorm_linear_bf16(golden):
    g = golden("rmsnorm_linear_bf16.npz")
    x = O.bf16_bits_to_f32(g["x_bits"])
    w = O.bf16_bits_to_f32(g["w_bits"])
    y = O.f32_to_bf16_bits(O.rmsnorm_linear(x, w, None, 1e-5, 1.0))
    ref = g["y_bits"]
    # identical up to one bf16 ulp (fp32 summation order differs from torch's)
    diff = np.abs(y.astype(np.int32) - ref.astype(np.int32))
    assert diff.max() <= 1
    yg = O.f32_to_bf16_bits(O.rmsnorm_linear(x, w * g["gamma"][None, :], None, 1e-5, 1.0))
    ref_g = O.f32_to_bf16_bits(g["y_gamma_f32"])  # the reference returns x.dtype (bf16)
    assert np.abs(yg.astype(np.int32) - ref_g.astype(np.int32)).max() <= 1


def test_rmsnorm_linear_fp8(golden):
    g = golden("rmsnorm_linear_fp8.npz")
    y = O.rmsnorm_linear_fp8(g["x"], g["w_vals"], g["wscale"], None, 1e-6)
    np.testing.assert_allclose(y, g["y_selfcheck"], rtol=1e-5, atol=1e-5)
    # genuine e4m3 weight and per-token quantised activations
    wq = O.e4m3_bits_to_f32(g["wq_bits"])
    xq_bits, sx = O.quantize_rows_e4m3(g["xa"])
    np.testing.assert_array_equal(xq_bits, g["xa_q_bits"])
    np.testing.assert_allclose(sx, g["sx"], rtol=0, atol=0)
    x_deq = O.e4m3_bits_to_f32(xq_bits) * sx[:, None]
    y = O.rmsnorm_linear_fp8(x_deq, wq, g["wscale"], g["bias"], 1e-6)
    np.testing.assert_allclose(y, g["y_real"], rtol=1e-5, atol=1e-5)


def test_e4m3_codec(golden):
    g = golden("quant_fp8.npz")
    codes = O.f32_to_e4m3_bits(g["vals"])
    np.testing.assert_array_equal(codes, g["codes"])
    np.testing.assert_array_equal(O.e4m3_bits_to_f32(g["codes"]), g["decoded"])
    qb, qs = O.quantize_fp8_e4m3(g["xt"])
    np.testing.assert_array_equal(qb, g["q_bits"])
    assert qs == g["q_scale"][0]


def test_pack_scales(golden):
    g = golden("pack_scales.npz")
    flat, offs = O.pack_scales([g["s0"], g["s1"]], [g["s2"]])
    np.testing.assert_array_equal(flat, g["flat"])
    np.testing.assert_array_equal(offs, g["offsets"])
    np.testing.assert_array_equal(O.unpack_scale_tensor(flat, offs, 1, (64, 2)), g["unpack1"])


def test_fused_verify(golden):
    g = golden("verify.npz")
    acc, top = O.fused_verify(g["h"], g["w"], g["b"], g["d"])
    np.testing.assert_array_equal(acc, g["accept1"])
    np.testing.assert_array_equal(top, g["top1"])


def test_fused_multi_verify(golden):
    g = golden("verify.npz")
    a, n, c = O.fused_multi_verify(g["hm"], g["wm"], g["bm"], g["dm"])
    np.testing.assert_array_equal(a, g["accept_m"])
    np.testing.assert_array_equal(n, g["n_m"])
    np.testing.assert_array_equal(c, g["corr_m"])
    a, n, c = O.fused_multi_verify(g["h3"], g["w3"], None, g["d3"])
    np.testing.assert_array_equal(a, g["accept3"])
    np.testing.assert_array_equal(n, g["n3"])
    np.testing.assert_array_equal(c, g["corr3"])
    # every accept-prefix length 0..5 is represented, and the duplicated
    # rows really tie (lowest index wins)
    assert sorted(set(g["n3"].tolist())) == [0, 1, 2, 3, 4, 5]


def test_vocab_sharded_equals_full(golden):
    g = golden("verify.npz")
    full = O.fused_multi_verify(g["h3"], g["w3"], None, g["d3"])
    for world in (1, 2, 3, 4, 8):
        sh = O.vocab_sharded_multi_verify(g["h3"], g["w3"], None, g["d3"], world)
        for x, y in zip(full, sh):
            np.testing.assert_array_equal(x, y)


def test_key_order_and_ties():
    vals = np.array([-np.inf, -3.0, -0.0, 0.0, 1e-30, 2.5, 2.5, np.float32(3.4e38)], np.float32)
    idx = np.array([7, 6, 5, 4, 3, 9, 2, 1])
    keys = O.pack_key(vals, idx)
    # value order dominates
    assert np.all(np.diff(keys[[0, 1, 4, 5, 7]]) > 0)
    # equal values: the smaller index has the larger key
    assert O.pack_key(np.float32([2.5]), np.array([2]))[0] > O.pack_key(np.float32([2.5]), np.array([9]))[0]
    np.testing.assert_array_equal(O.key_index(keys), idx)
    # the sentinel used to initialise key buffers is below every real key
    assert np.all(keys > np.iinfo(np.int64).min)


def test_config1_chain(golden):
    torch = pytest.importorskip("torch")
    g = golden("config1.npz")
    gen = torch.Generator().manual_seed(0)
    x = torch.randn(1, 5, 256, generator=gen)
    gamma = 1.0 + 0.1 * torch.randn(256, generator=gen)
    w = 0.02 * torch.randn(256, 256, generator=gen)
    lm = 0.02 * torch.randn(4096, 256, generator=gen)
    np.testing.assert_array_equal(x.numpy(), g["x"])
    np.testing.assert_array_equal(w.numpy(), g["w"])
    probe = g["lm_probe"]
    assert lm[0, 0].item() == probe[1] and lm[4095, 255].item() == probe[2]
    y = O.rmsnorm_linear(g["x"][0], g["w"] * g["gamma"][None, :], None, 1e-6, 1.0)
    np.testing.assert_allclose(y, g["y"], rtol=1e-5, atol=1e-6)
    a, n, c = O.fused_multi_verify(y[None], lm.numpy(), None, g["draft"])
    np.testing.assert_array_equal(a, g["accept"])
    np.testing.assert_array_equal(n, g["accepted_n"])
    np.testing.assert_array_equal(c, g["corrected"])
    assert int(n[0]) == 2


def test_tree_attention(golden):
    g = golden("tree_attention.npz")
    s = 1.0 / math.sqrt(32)
    np.testing.assert_allclose(O.tree_attention(g["q"], g["k"], g["v"], np.ones(8, np.float32), s),
                               g["o_ones"], rtol=1e-5, atol=1e-5)
    np.testing.assert_allclose(O.tree_attention(g["q"], g["k"], g["v"], g["mask_part"], s),
                               g["o_part"], rtol=1e-5, atol=1e-5)
    # the reference's own check: all-ones tree mask == causal attention (mtp_engine.py:1821-1824)
    np.testing.assert_allclose(g["o_ones"], g["causal"], atol=1e-2)
    np.testing.assert_allclose(O.tree_attention(g["qL"], g["kL"], g["vL"], g["mL"], 0.125),
                               g["oL"], rtol=1e-5, atol=1e-5)


def test_tree_attn_rmsnorm_linear(golden):
    g = golden("tree_attn_rmsnorm_linear.npz")
    s = float(g["scale"][0])
    o = O.tree_attn_rmsnorm_linear(g["q"], g["k"], g["v"], g["mask"], g["rms_w"], g["proj_w"], g["proj_b"],
                                   g["wscale"], s, 1e-6)
    np.testing.assert_allclose(o, g["out"], rtol=1e-4, atol=1e-4)
    o = O.tree_attn_rmsnorm_linear(g["q"], g["k"], g["v"], g["mask"], None, g["proj_w"], None, None, 0.3, 1e-5)
    np.testing.assert_allclose(o, g["out_bare"], rtol=1e-4, atol=1e-4)
    # bf16 operands widened to fp32, result rounded once to bf16
    qb, kb, vb, wb = (O.bf16_bits_to_f32(g[n]) for n in ("q_bits", "k_bits", "v_bits", "w_bits"))
    o = O.tree_attn_rmsnorm_linear(qb, kb, vb, g["mask"], g["rms_w"], wb, g["proj_b"], None, s, 1e-6)
    ref = O.bf16_bits_to_f32(g["out_b_bits"])
    assert np.max(np.abs(O.round_to_bf16(o) - ref)) <= 2.0 ** -7 * np.max(np.abs(ref))
    # every key masked: NaN rows, as the reference's softmax gives
    o = O.tree_attn_rmsnorm_linear(g["q"][:1], g["k"][:1], g["v"][:1], np.zeros(g["mask"].shape, np.float32),
                                   g["rms_w"], g["proj_w"], g["proj_b"], None, s, 1e-6)
    assert np.isnan(g["out_nan"]).all() and np.isnan(o).all()


def test_paged_attention(golden):
    g = golden("paged_attention.npz")
    ps = int(g["page_size"][0])
    o = O.paged_attention(g["q"], g["k_pages"], g["v_pages"], g["page_table"], ps,
                          1.0 / math.sqrt(g["q"].shape[-1]))
    np.testing.assert_allclose(o, g["out"], rtol=1e-5, atol=1e-5)


def test_tree_paged_attention(golden):
    g = golden("tree_paged.npz")
    ctx, ps = (int(v) for v in g["meta"])
    o = O.tree_attention_paged(g["q"], g["k_pages"], g["v_pages"], g["page_table"], ctx, ps,
                               g["tree_k"], g["tree_v"], g["tree_mask"],
                               1.0 / math.sqrt(g["q"].shape[-1]))
    np.testing.assert_allclose(o, g["out"], rtol=1e-5, atol=1e-5)
    of = O.tree_attention_paged_fast(g["q"], g["k_pages"], g["v_pages"], g["page_table"], ctx, ps,
                                     g["tree_k"], g["tree_v"], g["tree_mask"],
                                     1.0 / math.sqrt(g["q"].shape[-1]))
    np.testing.assert_allclose(of, g["out"], rtol=1e-5, atol=1e-5)


def test_tree_paged_attention_reserve_built_table(golden):
    """A page table from the reference's own PagedKVCache after unaligned
    reserve() calls and swap_logical_pages(): not page-granular, with -1
    entries inside the context that index page P-1 as torch does."""
    g = golden("tree_paged_reserve.npz")
    ctx, ps = (int(v) for v in g["meta"])
    bf = O.bf16_bits_to_f32
    args = (bf(g["q_bits"]), bf(g["k_pages_bits"]), bf(g["v_pages_bits"]), g["page_table"], ctx, ps,
            bf(g["tree_k_bits"]), bf(g["tree_v_bits"]), g["tree_mask"], 1.0 / math.sqrt(128))
    assert (g["page_table"][:, :ctx] < 0).any()  # the wrap is exercised
    np.testing.assert_allclose(O.tree_attention_paged(*args), g["out"], rtol=1e-5, atol=1e-5)
    np.testing.assert_allclose(O.tree_attention_paged_fast(*args), g["out"], rtol=1e-5, atol=1e-5)
    o1 = O.paged_attention(bf(g["q1_bits"]), bf(g["k_pages_bits"]), bf(g["v_pages_bits"]),
                           g["page_table"][:, :ctx], ps, 1.0 / math.sqrt(128))
    np.testing.assert_allclose(o1, g["out1"], rtol=1e-5, atol=1e-5)


@pytest.mark.parametrize("key,args", [("tree_16_4", (16, 4, "tree")), ("tree_4_8", (4, 8, "tree")),
                                      ("trunk_4_8", (4, 8, "trunk")), ("tree_4_2", (4, 2, "tree"))])
def test_draft_tree(golden, key, args):
    g = golden("draft_tree.npz")
    parent, mask = O.draft_tree(*args)
    np.testing.assert_array_equal(parent, g[key + "_parent"])
    np.testing.assert_array_equal(mask, g[key + "_mask"])


def test_config4_tree_shape():
    parent, mask = O.draft_tree(16, 4, "tree")
    assert mask.shape == (64, 64)
    depth = np.zeros(64, int)
    for n in range(1, 64):
        depth[n] = depth[parent[n]] + 1
    assert np.bincount(depth).tolist() == [1, 4, 16, 43]


def test_bf16_roundtrip():
    x = np.array([1.0, -2.5, 3.14159, 1e-20, -7e30, 0.0], np.float32)
    b = O.f32_to_bf16_bits(x)
    y = O.bf16_bits_to_f32(b)
    np.testing.assert_allclose(y, x, rtol=2 ** -8)
    np.testing.assert_array_equal(O.f32_to_bf16_bits(y), b)
