"""Generate the golden vectors in tests/golden/*.npz from the reference itself.

Run (in a container that has the reference checkout):

    python tests/golden/make_golden.py --reference /path/to/mtp-engine

The script imports the reference's own modules and calls its eager PyTorch
functions (``_eager_*``, mtp_kernels.py:778-907, mtp_fused_verify.py:159-196)
plus ``pack_scales`` / ``quantize_fp8_e4m3`` / ``SpeculativeDraftTree``
directly.  Inputs and outputs are written side by side, so the tests need
neither the reference nor torch's RNG to replay a case (except config 1,
whose 4 MB lm_head is regenerated from its torch.Generator seed and checked
against stored probes).  bf16 tensors are
stored as uint16 bit patterns, float8_e4m3fn tensors as uint8 bit patterns.

Shapes follow the reference's own tests where one exists (test_engine.py:5,
test_new_features.py:18-56, test_tree.py:37-44, mtp_engine.py:1792-1800,
mtp_engine.py:1821-1824, test_perf_hardening.py:75-80); the remaining cases
(paged attention values, partial tree masks, GQA composite, bf16, real fp8
weights, ties, config 1) are not pinned by any reference test and are
computed here from the same eager functions.
"""

from __future__ import annotations

import argparse
import math
import os
import sys

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))


def bits16(t):
    import torch
    return t.contiguous().view(torch.int16).numpy().view(np.uint16)


def bits8(t):
    import torch
    return t.contiguous().view(torch.uint8).numpy()


def f32(t):
    import torch
    return t.detach().to(torch.float32).numpy()


def save(name, **arrays):
    path = os.path.join(HERE, name)
    np.savez_compressed(path, **arrays)
    print(f"wrote {name}: " + ", ".join(f"{k}{tuple(v.shape)}" for k, v in arrays.items()))


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--reference", default=os.environ.get("MTP_REFERENCE"),
                    help="checkout of the reference project (or set MTP_REFERENCE)")
    ap.add_argument("--only", default="", help="write only this fixture (e.g. tree_attn_rmsnorm_linear)")
    args = ap.parse_args()
    if not args.reference:
        ap.error("give --reference or set MTP_REFERENCE")
    sys.path.insert(0, args.reference)
    os.environ.setdefault("TRITON_INTERPRET", "1")
    import torch
    import mtp_kernels as mk
    import mtp_fused_verify as mv
    from mtp_engine import SpeculativeDraftTree

    if args.only == "tree_attn_rmsnorm_linear":
        make_tree_attn_rmsnorm_linear(torch, mk)
        return
    if args.only == "quant_attention_int4":
        make_quant_attention_int4(torch, mk)
        return
    if args.only == "draft_tree":
        make_draft_trees(SpeculativeDraftTree)
        return
    if args.only == "paged_kv_write":
        import mtp_engine
        make_paged_kv_write(torch, mtp_engine)
        return
    if args.only == "api_signatures":
        make_api_signatures()
        return
    if args.only == "tree_paged_reserve":
        import mtp_engine
        make_tree_paged_reserve(torch, mk, mtp_engine)
        return

    # ---------------------------------------------------------------- rmsnorm_linear fp32
    torch.manual_seed(1)  # test_engine.py:5
    x = torch.randn(5, 64)
    W = torch.randn(128, 64)
    b = torch.randn(128)
    y = mk._eager_rmsnorm_linear(x, W, b, 1e-6, 1.0)
    torch.manual_seed(11)
    x2 = torch.randn(7, 96)
    W2 = torch.randn(40, 96)
    y2 = mk._eager_rmsnorm_linear(x2, W2, None, 1e-5, 0.5)
    save("rmsnorm_linear_fp32.npz", x=f32(x), w=f32(W), b=f32(b), y=f32(y),
         x2=f32(x2), w2=f32(W2), y2=f32(y2))

    # ---------------------------------------------------------------- rmsnorm_linear bf16
    torch.manual_seed(12)
    xb = torch.randn(9, 128).to(torch.bfloat16)
    Wb = (0.02 * torch.randn(72, 128)).to(torch.bfloat16)
    gam = 1.0 + 0.1 * torch.randn(128)
    yb = mk._eager_rmsnorm_linear(xb, Wb, None, 1e-5, 1.0)
    # gamma folded along K (exact algebra): rmsnorm(x)*gamma @ W^T == rmsnorm(x) @ (W*gamma)^T
    yg = mk._eager_rmsnorm_linear(xb, Wb.float() * gam[None, :], None, 1e-5, 1.0)
    save("rmsnorm_linear_bf16.npz", x_bits=bits16(xb), w_bits=bits16(Wb), gamma=f32(gam),
         y_bits=bits16(yb), y_gamma_f32=f32(yg))

    # ---------------------------------------------------------------- fp8
    torch.manual_seed(13)  # mtp_engine.py:1792-1800 shapes
    Wsw = torch.randn(32, 64)
    row_scale = Wsw.abs().max(dim=-1, keepdim=True).values.squeeze(-1) / 448.0
    Wf8 = (Wsw / row_scale[:, None]).clamp(-448, 448)
    xq = torch.randn(4, 64)
    y_selfcheck = mk._eager_rmsnorm_linear_fp8(xq, Wf8.contiguous(), row_scale, None, 1e-6)
    # genuine float8_e4m3fn weight + per-token-quantised activations
    Wq = Wf8.to(torch.float8_e4m3fn)
    xa = 3.0 * torch.randn(6, 64)
    amax = xa.abs().max(dim=-1).values
    sx = torch.where(amax > 0, amax / 448.0, torch.ones_like(amax))
    xa_q = (xa / sx[:, None]).clamp(-448, 448).to(torch.float8_e4m3fn)
    xa_deq = xa_q.float() * sx[:, None]
    bias8 = torch.randn(32)
    y_real = mk._eager_rmsnorm_linear_fp8(xa_deq, Wq, row_scale, bias8, 1e-6)
    save("rmsnorm_linear_fp8.npz", w_vals=f32(Wf8), wscale=f32(row_scale), x=f32(xq),
         y_selfcheck=f32(y_selfcheck), wq_bits=bits8(Wq), xa=f32(xa), xa_q_bits=bits8(xa_q),
         sx=f32(sx), bias=f32(bias8), y_real=f32(y_real))

    # ---------------------------------------------------------------- e4m3 rounding + per-tensor quant
    grid = torch.tensor([0.0, -0.0, 1e-9, 0.0009765625, 0.001953125, 0.0029296875, 0.015625,
                         0.0146484375, 1.0625, 1.1875, 3.25, 7.5, 15.0, 239.0, 240.0, 248.0,
                         256.0, 272.0, 440.0, 447.9, 448.0, -448.0, -0.3, 0.33, 1.0 / 3.0])
    rnd = torch.randn(4096) * 50.0
    vals = torch.cat([grid, -grid, rnd]).clamp(-448, 448)
    codes = vals.to(torch.float8_e4m3fn)
    torch.manual_seed(14)
    xt = torch.randn(16, 32) * 7.0
    qb, qs = mk.quantize_fp8_e4m3(xt)
    save("quant_fp8.npz", vals=f32(vals), codes=bits8(codes), decoded=f32(codes.float()),
         xt=f32(xt), q_bits=bits8(qb), q_scale=np.float32(qs.item()).reshape(1))

    # ---------------------------------------------------------------- packed scales
    torch.manual_seed(15)  # test_perf_hardening.py:75-80 style
    s0, s1, s2 = torch.rand(128), torch.rand(64, 2), torch.rand(3)
    flat, offs = mk.pack_scales([s0, s1], [s2])
    save("pack_scales.npz", s0=f32(s0), s1=f32(s1), s2=f32(s2), flat=f32(flat),
         offsets=offs.numpy().astype(np.int64),
         unpack1=f32(mk.unpack_scale_tensor(flat, offs, 1, (64, 2))))

    # ---------------------------------------------------------------- verify
    torch.manual_seed(0)  # test_new_features.py:18-33
    M, K, V = 4, 64, 256
    h = torch.randn(M, K)
    Wv = torch.randn(V, K)
    bv = torch.randn(V)
    d = torch.randint(0, V, (M,))
    acc1, top1 = mv._eager_fused_verify(h, Wv, bv, d.to(torch.int32))
    torch.manual_seed(1)  # test_new_features.py:36-55
    B, S, K2, V2, D = 2, 5, 64, 256, 4
    hm = torch.randn(B, S, K2)
    Wm = torch.randn(V2, K2)
    bm = torch.randn(V2)
    dm = torch.randint(0, V2, (B, D))
    am, nm, cm = mv._eager_fused_multi_verify(hm, Wm, bm, dm.to(torch.int32))
    # designed prefixes, no bias, ragged V, duplicated rows for exact ties
    torch.manual_seed(16)
    B3, S3, K3, V3 = 6, 6, 48, 333
    h3 = torch.randn(B3, S3, K3)
    W3 = torch.randn(V3, K3)
    W3[200] = W3[17]  # identical rows -> identical logits; argmax must pick 17
    W3[300] = W3[5]
    top3 = torch.nn.functional.linear(h3, W3).argmax(-1)
    d3 = torch.randint(0, V3, (B3, S3 - 1))
    for bb in range(B3):
        a = bb % S3  # accept prefix length 0..5
        d3[bb, :a] = top3[bb, 1:a + 1]
        if a < S3 - 1:
            d3[bb, a] = (top3[bb, a + 1] + 1) % V3
    a3, n3, c3 = mv._eager_fused_multi_verify(h3, W3, None, d3.to(torch.int32))
    save("verify.npz", h=f32(h), w=f32(Wv), b=f32(bv), d=d.numpy().astype(np.int64),
         accept1=acc1.numpy(), top1=top1.numpy(),
         hm=f32(hm), wm=f32(Wm), bm=f32(bm), dm=dm.numpy().astype(np.int64),
         accept_m=am.numpy(), n_m=nm.numpy(), corr_m=cm.numpy(),
         h3=f32(h3), w3=f32(W3), d3=d3.numpy().astype(np.int64), top3=top3.numpy().astype(np.int32),
         accept3=a3.numpy(), n3=n3.numpy(), corr3=c3.numpy())

    # ---------------------------------------------------------------- config 1 (tiny chain, fp32)
    g = torch.Generator().manual_seed(0)
    xc = torch.randn(1, 5, 256, generator=g)
    gamma = 1.0 + 0.1 * torch.randn(256, generator=g)
    Wc = 0.02 * torch.randn(256, 256, generator=g)
    LM = 0.02 * torch.randn(4096, 256, generator=g)
    draft_c = torch.randint(0, 4096, (1, 4), generator=g)
    yc = mk._eager_rmsnorm_linear(xc[0], Wc * gamma[None, :], None, 1e-6, 1.0)
    topc = torch.nn.functional.linear(yc, LM).argmax(-1)
    draft_c[0, :2] = topc[1:3]
    if draft_c[0, 2] == topc[3]:
        draft_c[0, 2] = (topc[3] + 1) % 4096
    ac, nc, cc = mv._eager_fused_multi_verify(yc[None], LM, None, draft_c.to(torch.int32))
    # the lm_head (4 MB) is not stored: tests replay the same torch.Generator
    # sequence and check it against these probes
    lm_probe = np.array([LM.sum().item(), LM[0, 0].item(), LM[4095, 255].item()], dtype=np.float64)
    save("config1.npz", x=f32(xc), gamma=f32(gamma), w=f32(Wc), lm_probe=lm_probe,
         draft=draft_c.numpy().astype(np.int64), y=f32(yc), accept=ac.numpy(),
         accepted_n=nc.numpy(), corrected=cc.numpy())

    # ---------------------------------------------------------------- tree attention
    torch.manual_seed(1)  # test_tree.py:37-44 shapes
    q = torch.randn(2, 2, 32)
    k = torch.randn(2, 2, 8, 32)
    v = torch.randn(2, 2, 8, 32)
    ones = torch.ones(8)
    part = torch.tensor([1.0, 0.0, 1.0, 0.7, 0.2, 0.0, 1.0, 0.51])
    o_ones = mk._eager_tree_attention(q, k, v, ones, 1.0 / math.sqrt(32))
    o_part = mk._eager_tree_attention(q, k, v, part, 1.0 / math.sqrt(32))
    causal = mk._eager_causal_attention(q, k, v, 1.0 / math.sqrt(32))
    torch.manual_seed(17)
    qL = torch.randn(3, 4, 64)
    kL = torch.randn(3, 4, 70, 64)
    vL = torch.randn(3, 4, 70, 64)
    mL = (torch.rand(70) > 0.4).float()
    mL[3] = 1.0
    oL = mk._eager_tree_attention(qL, kL, vL, mL, 0.125)
    save("tree_attention.npz", q=f32(q), k=f32(k), v=f32(v), mask_part=f32(part),
         o_ones=f32(o_ones), o_part=f32(o_part), causal=f32(causal),
         qL=f32(qL), kL=f32(kL), vL=f32(vL), mL=f32(mL), oL=f32(oL))

    # ---------------------------------------------------------------- paged attention
    torch.manual_seed(18)
    Bp, Hp, Dp, ps, P, L = 2, 2, 16, 4, 6, 12
    kp = torch.randn(P, Bp, Hp, ps, Dp)
    vp = torch.randn(P, Bp, Hp, ps, Dp)
    pt = torch.empty(Bp, L, dtype=torch.int32)
    for bb in range(Bp):
        perm = torch.randperm(P)[: L // ps]
        for t in range(L):
            pt[bb, t] = perm[t // ps]
    qp = torch.randn(Bp, Hp, Dp)
    op = mk._eager_paged_attention(qp, kp, vp, pt, ps, 1.0 / math.sqrt(Dp))
    save("paged_attention.npz", q=f32(qp), k_pages=f32(kp), v_pages=f32(vp),
         page_table=pt.numpy(), page_size=np.int64(ps).reshape(1), out=f32(op))

    # ---------------------------------------------------------------- paged tree attention (composite, GQA)
    torch.manual_seed(19)
    tree = SpeculativeDraftTree(depth=4, max_branches=2, mode="tree")
    T = tree.max_nodes
    Bt, Hq, Hkv, Dt, pst, Pt, ctx = 2, 4, 2, 32, 4, 8, 10
    G = Hq // Hkv
    kpt = torch.randn(Pt, Bt, Hkv, pst, Dt)
    vpt = torch.randn(Pt, Bt, Hkv, pst, Dt)
    ptt = torch.full((Bt, 16), -1, dtype=torch.int32)
    for bb in range(Bt):
        perm = torch.randperm(Pt)
        for t in range(16):
            ptt[bb, t] = perm[t // pst]
    qt = torch.randn(Bt, T, Hq, Dt)
    tk = torch.randn(Bt, Hkv, T, Dt)
    tv = torch.randn(Bt, Hkv, T, Dt)
    scale = 1.0 / math.sqrt(Dt)
    # gather with the index math of _eager_paged_attention (mtp_kernels.py:839-848)
    page = ptt[:, :ctx].long()
    slot = torch.arange(ctx) % pst
    bi = torch.arange(Bt)[:, None, None].expand(Bt, Hkv, ctx)
    hi = torch.arange(Hkv)[None, :, None].expand(Bt, Hkv, ctx)
    kc = kpt[page.unsqueeze(1).expand(Bt, Hkv, ctx), bi, hi, slot[None, None].expand(Bt, Hkv, ctx)]
    vc = vpt[page.unsqueeze(1).expand(Bt, Hkv, ctx), bi, hi, slot[None, None].expand(Bt, Hkv, ctx)]
    Kall = torch.cat([kc, tk], dim=2).repeat_interleave(G, dim=1)
    Vall = torch.cat([vc, tv], dim=2).repeat_interleave(G, dim=1)
    out_t = torch.empty(Bt, T, Hq, Dt)
    for n in range(T):
        mask_n = torch.cat([torch.ones(ctx), tree.tree_mask[n]])
        out_t[:, n] = mk._eager_tree_attention(qt[:, n], Kall, Vall, mask_n, scale)
    save("tree_paged.npz", q=f32(qt), k_pages=f32(kpt), v_pages=f32(vpt), page_table=ptt.numpy(),
         tree_k=f32(tk), tree_v=f32(tv), tree_mask=f32(tree.tree_mask),
         meta=np.array([ctx, pst], dtype=np.int64), out=f32(out_t))

    make_draft_trees(SpeculativeDraftTree)
    make_tree_attn_rmsnorm_linear(torch, mk)
    import mtp_engine
    make_paged_kv_write(torch, mtp_engine)
    make_tree_paged_reserve(torch, mk, mtp_engine)
    make_quant_attention_int4(torch, mk)
    make_api_signatures()


# (depth, max_branches, mode): the config-4 tree, small trees, trees whose
# node budget runs out inside a level (3*8: level 2 gets 15 of 64 children),
# chains, and single-branch trees
DRAFT_TREES = [(16, 4, "tree"), (4, 8, "tree"), (4, 8, "trunk"), (4, 2, "tree"), (3, 8, "tree"),
               (5, 3, "tree"), (8, 4, "tree"), (1, 4, "tree"), (1, 1, "trunk"), (6, 1, "tree"),
               (7, 2, "trunk"), (2, 3, "tree")]


def make_draft_trees(SpeculativeDraftTree):
    """SpeculativeDraftTree (mtp_engine.py:635-719): parent index, ancestor
    mask, linear layout and active node count."""
    arrs = {}
    for (dep, br, mode) in DRAFT_TREES:
        t = SpeculativeDraftTree(depth=dep, max_branches=br, mode=mode)
        key = f"{mode}_{dep}_{br}"
        arrs[key + "_parent"] = t.parent.numpy()
        arrs[key + "_mask"] = t.tree_mask.numpy()
        do, bo = t.build_linear_layout()
        arrs[key + "_depth_offsets"] = do.numpy()
        arrs[key + "_branch_offsets"] = bo.numpy()
        arrs[key + "_active"] = np.array(t.active_node_count(), dtype=np.int64)
    save("draft_tree.npz", **arrs)


def make_quant_attention_int4(torch, mk):
    """fused_causal_attention_fp8 / fused_causal_attention / fused_int4_matmul
    through their eager bodies (mtp_kernels.py:817-830, 790-802, 875-878) and
    the int4 host helpers quantize_int4 / dequantize_int4 (730-767).  The fp8
    case uses genuine float8_e4m3fn K/V with per-head scales != 1 (the
    reference's own self-check, mtp_engine.py:1802-1809, uses fp32 K/V and
    unit scales); the int4 case follows mtp_engine.py:1812-1818 plus a
    partial last group."""
    torch.manual_seed(23)
    B, H, L, D = 2, 3, 40, 64
    q = torch.randn(B, H, D)
    kf = torch.randn(B, H, L, D) * 3
    vf = torch.randn(B, H, L, D) * 3
    ks = torch.tensor([0.5, 1.25, 2.0])
    vs = torch.tensor([1.5, 0.75, 1.0])
    k8, v8 = kf.clamp(-448, 448).to(torch.float8_e4m3fn), vf.clamp(-448, 448).to(torch.float8_e4m3fn)
    att8 = mk._eager_causal_attention_fp8(q, k8, v8, ks, vs, 1.0 / math.sqrt(D))
    att = mk._eager_causal_attention(q, kf, vf, 0.2)
    W = torch.randn(48, 96) * 2
    W[3, :32] = 0.0
    pk, sc = mk.quantize_int4(W, group=32)
    Wd = mk.dequantize_int4(pk, sc, 96, 32)
    x = torch.randn(5, 96)
    y = mk._eager_int4_matmul(x, pk, sc, 96, 32)
    W2 = torch.randn(20, 40)
    pk2, sc2 = mk.quantize_int4(W2, group=32)  # last group holds 8 columns
    x2 = torch.randn(3, 40)
    y2 = mk._eager_int4_matmul(x2, pk2, sc2, 40, 32)
    save("quant_attention_int4.npz", q=f32(q), k_bits=bits8(k8), v_bits=bits8(v8), kscale=f32(ks),
         vscale=f32(vs), att8=f32(att8), kf=f32(kf), vf=f32(vf), att=f32(att), w=f32(W),
         packed=pk.numpy(), scales=f32(sc), w_deq=f32(Wd), x=f32(x), y=f32(y), w2=f32(W2), packed2=pk2.numpy(),
         scales2=f32(sc2), x2=f32(x2), y2=f32(y2))


def make_paged_kv_write(torch, mtp_engine):
    """The reference's own PagedKVCache (mtp_engine.py:523-610) on the CPU:
    reserve() builds the page table, write_inplace() (582-586) writes one
    token of one head at a time.  A float32 pool and a bf16 pool written
    from float32 rows (write_inplace casts with .to(self.dtype))."""
    torch.manual_seed(22)
    B, H, D, P, ps = 2, 3, 16, 8, 4
    out = {}
    for name, dt in (("f32", torch.float32), ("bf16", torch.bfloat16)):
        kv = mtp_engine.PagedKVCache(batch=B, num_heads=H, head_dim=D, num_pages=P, page_size=ps,
                                     device=torch.device("cpu"), dtype=dt)
        kv.k_pages.normal_()
        kv.v_pages.normal_()
        before_k, before_v = kv.k_pages.clone(), kv.v_pages.clone()
        start = kv.reserve(3)   # positions 0..2 (not written)
        start = kv.reserve(9)   # positions 3..11 -> written below
        n = 9
        k_new = torch.randn(B, H, n, D)
        v_new = torch.randn(B, H, n, D)
        for t in range(n):
            for b in range(B):
                for h in range(H):
                    kv.write_inplace(start + t, b, h, k_new[b, h, t], v_new[b, h, t])
        conv = (lambda t_: f32(t_)) if dt == torch.float32 else (lambda t_: bits16(t_))
        out.update({f"{name}_k_before": conv(before_k), f"{name}_v_before": conv(before_v),
                    f"{name}_k_after": conv(kv.k_pages), f"{name}_v_after": conv(kv.v_pages),
                    f"{name}_page_table": kv.page_table.numpy(), f"{name}_k_new": f32(k_new),
                    f"{name}_v_new": f32(v_new), f"{name}_start": np.array([start], np.int64)})
    save("paged_kv_write.npz", **out)


# the reference's public functions on the hot path (and around it) whose
# signatures the drop-in must keep: module -> names ("Class.method" for
# methods)
API = {
    "mtp_kernels": ["fused_rmsnorm_linear", "fused_rmsnorm_linear_fp8", "fused_tree_attention",
                    "fused_paged_attention", "fused_tree_attn_rmsnorm_linear", "fused_causal_attention",
                    "fused_causal_attention_fp8", "fused_int4_matmul", "pack_scales", "unpack_scale_tensor",
                    "quantize_fp8_e4m3", "dequantize_fp8", "quantize_int4", "dequantize_int4",
                    "build_tuning_config", "KernelTuningConfig.__init__"],
    "mtp_fused_verify": ["fused_verify", "fused_multi_verify"],
    "mtp_parallel": ["ParallelPrimitives.__init__", "get_parallel_primitives", "RowParallelLinear.__init__",
                     "RowParallelLinear.forward", "ColumnParallelLinear.__init__", "ColumnParallelLinear.forward"],
}


def make_api_signatures():
    """The parameters (name, kind, default) of every function in API, read
    from the reference's own modules with inspect, as the drop-in contract
    that tests/test_dropin_api.py checks the modules here against."""
    import importlib
    import inspect
    import json
    out = {}
    for mod_name, names in API.items():
        mod = importlib.import_module(mod_name)
        for name in names:
            obj = mod
            for part in name.split("."):
                obj = getattr(obj, part)
            params = []
            for p_ in inspect.signature(obj).parameters.values():
                default = None if p_.default is inspect.Parameter.empty else repr(p_.default)
                params.append([p_.name, p_.kind.name, default])
            out[f"{mod_name}.{name}"] = params
    path = os.path.join(HERE, "reference_api.json")
    with open(path, "w") as f:
        json.dump(out, f, indent=1, sort_keys=True)
        f.write("\n")
    print(f"wrote reference_api.json: {len(out)} signatures")


# token counts passed to PagedKVCache.reserve, then the logical columns swapped
RESERVES = (5, 1, 1, 16, 7, 40, 3, 50, 30, 9)
SWAPS = ((3, 100), (20, 21), (0, 140), (64, 65), (17, 161))


def make_tree_paged_reserve(torch, mk, mtp_engine):
    """Paged tree attention over a page table that the reference's own
    PagedKVCache built (mtp_engine.py:523-610): reserve() with token counts
    that are not multiples of page_size, then swap_logical_pages().  The
    table is then not page-granular (one page slot's 16 tokens come from
    several pages), and the columns that reserve() never reaches keep -1,
    which torch indexing reads as page P-1.  Output: the composite of the
    reference's eager functions -- the gather of _eager_paged_attention
    (mtp_kernels.py:839-848), then _eager_tree_attention per tree node
    (859-872), GQA by repeat_interleave -- with head_dim 128 and page_size
    16, the shapes the tensor-core kernel takes; plus _eager_paged_attention
    itself (the single-query operator) on the same table.  K/V/Q values are
    bf16-representable (stored as bf16 bits)."""
    torch.manual_seed(23)
    B, Hq, Hkv, D, ps, P = 2, 8, 2, 128, 16, 24
    G = Hq // Hkv
    bf = lambda t: t.to(torch.bfloat16).to(torch.float32)
    kv = mtp_engine.PagedKVCache(batch=B, num_heads=Hkv, head_dim=D, num_pages=P, page_size=ps,
                                 device=torch.device("cpu"), dtype=torch.float32)
    kv.k_pages.copy_(bf(torch.randn(kv.k_pages.shape)))
    kv.v_pages.copy_(bf(torch.randn(kv.v_pages.shape)))
    for n in RESERVES:
        kv.reserve(n)
    ctx = kv._next_logical
    for a, b_ in SWAPS:
        kv.swap_logical_pages(a, b_)
    tree = mtp_engine.SpeculativeDraftTree(depth=4, max_branches=2, mode="tree")
    T = tree.max_nodes
    qt = bf(torch.randn(B, T, Hq, D))
    tk = bf(torch.randn(B, Hkv, T, D))
    tv = bf(torch.randn(B, Hkv, T, D))
    scale = 1.0 / math.sqrt(D)
    page = kv.page_table[:, :ctx].long()
    slot = torch.arange(ctx) % ps
    bi = torch.arange(B)[:, None, None].expand(B, Hkv, ctx)
    hi = torch.arange(Hkv)[None, :, None].expand(B, Hkv, ctx)
    kc = kv.k_pages[page.unsqueeze(1).expand(B, Hkv, ctx), bi, hi, slot[None, None].expand(B, Hkv, ctx)]
    vc = kv.v_pages[page.unsqueeze(1).expand(B, Hkv, ctx), bi, hi, slot[None, None].expand(B, Hkv, ctx)]
    Kall = torch.cat([kc, tk], dim=2).repeat_interleave(G, dim=1)
    Vall = torch.cat([vc, tv], dim=2).repeat_interleave(G, dim=1)
    out_t = torch.empty(B, T, Hq, D)
    for n in range(T):
        mask_n = torch.cat([torch.ones(ctx), tree.tree_mask[n]])
        out_t[:, n] = mk._eager_tree_attention(qt[:, n], Kall, Vall, mask_n, scale)
    q1 = bf(torch.randn(B, Hkv, D))
    out1 = mk._eager_paged_attention(q1, kv.k_pages, kv.v_pages, kv.page_table[:, :ctx].contiguous(), ps, scale)
    save("tree_paged_reserve.npz", q_bits=bits16(qt.to(torch.bfloat16)),
         k_pages_bits=bits16(kv.k_pages.to(torch.bfloat16)), v_pages_bits=bits16(kv.v_pages.to(torch.bfloat16)),
         page_table=kv.page_table.numpy(), tree_k_bits=bits16(tk.to(torch.bfloat16)),
         tree_v_bits=bits16(tv.to(torch.bfloat16)), tree_mask=f32(tree.tree_mask),
         meta=np.array([ctx, ps], dtype=np.int64), out=f32(out_t),
         q1_bits=bits16(q1.to(torch.bfloat16)), out1=f32(out1))


def make_tree_attn_rmsnorm_linear(torch, mk):
    """``_eager_tree_attn_rmsnorm_linear`` (mtp_kernels.py:881-905), the body
    of ``fused_tree_attn_rmsnorm_linear`` (1222-1250).  Shapes: the
    reference's memory bench geometry (bench_memory.py:96, H=4 D=64 L=32
    N=256) with a partial mask, rms_w, bias and wscale; a bare case (no
    rms_w / bias / wscale); a bf16 case; and an all-masked case (NaN rows)."""
    torch.manual_seed(21)
    B, H, D, L, N = 3, 4, 64, 32, 256
    q = torch.randn(B, H, D)
    k = torch.randn(B, H, L, D)
    v = torch.randn(B, H, L, D)
    mask = (torch.rand(L) > 0.4).float()
    mask[0] = 1.0
    rms_w = 1.0 + 0.1 * torch.randn(D)
    proj_w = 0.05 * torch.randn(N, D)
    proj_b = torch.randn(N)
    wscale = 0.5 + torch.rand(N)
    scale = 1.0 / math.sqrt(D)
    out = mk._eager_tree_attn_rmsnorm_linear(q, k, v, mask, rms_w, proj_w, proj_b, wscale, scale, 1e-6)
    out_bare = mk._eager_tree_attn_rmsnorm_linear(q, k, v, mask, None, proj_w, None, None, 0.3, 1e-5)
    # bf16 operands (the reference widens everything to fp32 and rounds the result once)
    qb, kb, vb = (t.to(torch.bfloat16) for t in (q, k, v))
    wb = proj_w.to(torch.bfloat16)
    out_b = mk._eager_tree_attn_rmsnorm_linear(qb, kb, vb, mask, rms_w, wb, proj_b, None, scale, 1e-6)
    out_nan = mk._eager_tree_attn_rmsnorm_linear(q[:1], k[:1], v[:1], torch.zeros(L), rms_w, proj_w, proj_b,
                                                 None, scale, 1e-6)
    save("tree_attn_rmsnorm_linear.npz", q=f32(q), k=f32(k), v=f32(v), mask=f32(mask), rms_w=f32(rms_w),
         proj_w=f32(proj_w), proj_b=f32(proj_b), wscale=f32(wscale), scale=np.float32(scale).reshape(1),
         out=f32(out), out_bare=f32(out_bare), q_bits=bits16(qb), k_bits=bits16(kb), v_bits=bits16(vb),
         w_bits=bits16(wb), out_b_bits=bits16(out_b), out_nan=f32(out_nan))


if __name__ == "__main__":
    main()
