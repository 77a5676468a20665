"""CPU oracle for the tree-verification hot path -- TEST INFRASTRUCTURE ONLY.

This module restates, in numpy, the eager PyTorch reference functions of
Dahacker444/mtp-engine that define the semantics of the hot path.  It is the
checker used by ``tests/``, by ``__graft_entry__.smoke()`` and by the
``cpu_baseline`` / ``--impl reference`` legs of ``bench.py``.  Nothing in the
product package (``mtp-engine_b200/``) imports it, and the product never
falls back to it.

Parity pin: every function below is checked against golden vectors that were
produced by running the reference's own eager functions
(``tests/golden/make_golden.py`` imports the reference and writes
``tests/golden/*.npz``; ``tests/test_oracle_golden.py`` compares), except
``verify_step``: the reference has that step only inline in its generate
loops, so it is restated from both loops and the two restatements are
checked against each other (``tests/test_verify_step.py``).

All citations are ``file:line`` within the reference project.

Numeric conventions (same as the reference's eager path): every input is
widened to float32 before any arithmetic (mtp_kernels.py:782, 809,
mtp_fused_verify.py:180-182); argmax picks the lowest index among equal
maxima (torch.argmax semantics); bf16 values are carried as uint16 bit
patterns and fp8-E4M3 values as uint8 bit patterns.
"""

from __future__ import annotations

import math
from typing import List, Optional, Sequence, Tuple

import numpy as np

MAX_FP8 = 448.0  # mtp_kernels.py:66

# --------------------------------------------------------------------------- #
# dtype helpers (bf16 / e4m3 bit patterns <-> float32)
# --------------------------------------------------------------------------- #


def bf16_bits_to_f32(bits: np.ndarray) -> np.ndarray:
    """bf16 bit patterns (uint16) -> float32 (exact)."""
    b = np.asarray(bits, dtype=np.uint16).astype(np.uint32) << 16
    return b.view(np.float32)


def f32_to_bf16_bits(x: np.ndarray) -> np.ndarray:
    """float32 -> bf16 bit patterns, round-to-nearest-even (NaN kept NaN)."""
    x = np.ascontiguousarray(x, dtype=np.float32)
    u = x.view(np.uint32).astype(np.uint64)
    rounding = ((u >> 16) & 1) + 0x7FFF
    out = ((u + rounding) >> 16).astype(np.uint16)
    nan = np.isnan(x)
    if nan.any():
        out = np.where(nan, np.uint16(0x7FC0), out)
    return out


def round_to_bf16(x: np.ndarray) -> np.ndarray:
    """float32 -> nearest bf16 value, returned as float32."""
    return bf16_bits_to_f32(f32_to_bf16_bits(x))


def _e4m3_table() -> np.ndarray:
    t = np.zeros(256, dtype=np.float32)
    for code in range(256):
        s = -1.0 if code & 0x80 else 1.0
        e = (code >> 3) & 0xF
        m = code & 0x7
        if e == 0xF and m == 0x7:
            t[code] = np.nan  # e4m3fn has no inf; S.1111.111 is NaN
        elif e == 0:
            t[code] = s * (m / 8.0) * 2.0 ** -6
        else:
            t[code] = s * (1.0 + m / 8.0) * 2.0 ** (e - 7)
    return t


E4M3_TABLE = _e4m3_table()
_E4M3_POS = E4M3_TABLE[:127].astype(np.float64)  # codes 0..126 ascending, +0 .. 448


def e4m3_bits_to_f32(bits: np.ndarray) -> np.ndarray:
    return E4M3_TABLE[np.asarray(bits, dtype=np.uint8)]


def f32_to_e4m3_bits(x: np.ndarray) -> np.ndarray:
    """float32 -> float8_e4m3fn bit patterns, round-to-nearest-even.

    Inputs are expected already clamped to [-448, 448] (the reference clamps
    before casting, mtp_kernels.py:708); larger magnitudes saturate to 448.
    """
    x = np.asarray(x, dtype=np.float32)
    a = np.minimum(np.abs(x).astype(np.float64), MAX_FP8)
    idx = np.searchsorted(_E4M3_POS, a, side="left")
    idx = np.clip(idx, 0, 126)
    lo = np.clip(idx - 1, 0, 126)
    d_hi = _E4M3_POS[idx] - a
    d_lo = a - _E4M3_POS[lo]
    pick_lo = (d_lo < d_hi) | ((d_lo == d_hi) & (lo % 2 == 0) & (lo != idx))
    code = np.where(pick_lo, lo, idx).astype(np.uint8)
    neg = np.signbit(x)  # the sign survives rounding to zero (IEEE -0)
    return (code | (neg.astype(np.uint8) << 7)).astype(np.uint8)


# --------------------------------------------------------------------------- #
# FP8 quantisation helpers and the packed scale layout
# --------------------------------------------------------------------------- #


def quantize_fp8_e4m3(x: np.ndarray) -> Tuple[np.ndarray, np.float32]:
    """Per-tensor E4M3 quantisation, mtp_kernels.py:704-713.

    scale = amax / 448 (1.0 when amax == 0); q = e4m3(clamp(x / scale)).
    Returns (uint8 bit patterns, float32 scale).
    """
    xf = np.asarray(x, dtype=np.float32)
    amax = np.float32(np.abs(xf).max()) if xf.size else np.float32(0)
    scale = np.float32(amax / np.float32(MAX_FP8)) if amax > 0 else np.float32(1.0)
    scaled = np.clip(xf / scale, -MAX_FP8, MAX_FP8).astype(np.float32)
    return f32_to_e4m3_bits(scaled), scale


def dequantize_fp8(bits: np.ndarray, scale) -> np.ndarray:
    """mtp_kernels.py:726-727."""
    return e4m3_bits_to_f32(bits) * np.float32(scale)


def quantize_rows_e4m3(x: np.ndarray) -> Tuple[np.ndarray, np.ndarray]:
    """Per-row (per-token / per-output-channel) E4M3 quantisation.

    Row scale = amax_row / 448 (1.0 for an all-zero row), the convention of
    QuantScaleState.update_weight_scales (mtp_engine.py:617-622) and of the
    FP8 self-check (mtp_engine.py:1793-1794).  Returns (bits, scales[rows]).
    """
    xf = np.asarray(x, dtype=np.float32)
    amax = np.abs(xf).max(axis=-1)
    scale = np.where(amax > 0, amax / np.float32(MAX_FP8), np.float32(1.0)).astype(np.float32)
    scaled = np.clip(xf / scale[..., None], -MAX_FP8, MAX_FP8).astype(np.float32)
    return f32_to_e4m3_bits(scaled), scale


def pack_scales(weight_scales: Sequence[np.ndarray],
                kv_scales: Optional[Sequence[np.ndarray]] = None) -> Tuple[np.ndarray, np.ndarray]:
    """Flat fp32 concatenation plus int64 offsets, mtp_kernels.py:1336-1346."""
    all_scales = list(weight_scales) + list(kv_scales or [])
    offsets = [0]
    for s in all_scales:
        offsets.append(offsets[-1] + int(np.asarray(s).size))
    if all_scales:
        flat = np.concatenate([np.asarray(s, dtype=np.float32).reshape(-1) for s in all_scales])
    else:
        flat = np.zeros(0, dtype=np.float32)
    return flat.astype(np.float32), np.asarray(offsets, dtype=np.int64)


def unpack_scale_tensor(flat: np.ndarray, offsets: np.ndarray, idx: int,
                        shape: Tuple[int, ...]) -> np.ndarray:
    """mtp_kernels.py:1349-1353."""
    start, end = int(offsets[idx]), int(offsets[idx + 1])
    return flat[start:end].reshape(shape)


# --------------------------------------------------------------------------- #
# RMSNorm -> linear
# --------------------------------------------------------------------------- #


def rms_rstd(xf: np.ndarray, eps: float) -> np.ndarray:
    """rstd = 1/sqrt(mean(x^2) + eps) per row, mtp_kernels.py:783-784."""
    xf = np.asarray(xf, dtype=np.float32)
    ms = (xf * xf).mean(axis=-1, keepdims=True, dtype=np.float32)
    return (np.float32(1.0) / np.sqrt(ms + np.float32(eps))).astype(np.float32)


def rmsnorm_linear(x: np.ndarray, w: np.ndarray, bias: Optional[np.ndarray], eps: float,
                   scale: float) -> np.ndarray:
    """``_eager_rmsnorm_linear``, mtp_kernels.py:778-787 (float32 result).

    y = (linear(x * rstd, W) + b) * scale, all in float32.  The caller casts
    to the output dtype (the reference casts to x.dtype, line 787).
    """
    xf = np.asarray(x, dtype=np.float32)
    x_norm = xf * rms_rstd(xf, eps)
    y = x_norm @ np.asarray(w, dtype=np.float32).T
    if bias is not None:
        y = y + np.asarray(bias, dtype=np.float32)
    return (y * np.float32(scale)).astype(np.float32)


def rmsnorm_linear_fp8(x: np.ndarray, w_vals: np.ndarray, wscale: np.ndarray,
                       bias: Optional[np.ndarray], eps: float) -> np.ndarray:
    """``_eager_rmsnorm_linear_fp8``, mtp_kernels.py:804-814 (float32 result).

    ``w_vals`` are the stored weight values as float32 (decoded e4m3, or the
    fp32-valued clamped weight the reference's own self-check passes,
    mtp_engine.py:1792-1800); W = w_vals * wscale[:, None].
    """
    w = np.asarray(w_vals, dtype=np.float32) * np.asarray(wscale, dtype=np.float32)[:, None]
    return rmsnorm_linear(x, w, bias, eps, 1.0)


# --------------------------------------------------------------------------- #
# attention
# --------------------------------------------------------------------------- #


def _softmax_rows(scores: np.ndarray) -> np.ndarray:
    m = scores.max(axis=-1, keepdims=True)
    p = np.exp(scores - m)
    return p / p.sum(axis=-1, keepdims=True)


def tree_attention(q: np.ndarray, k: np.ndarray, v: np.ndarray, mask: np.ndarray,
                   scale: float) -> np.ndarray:
    """``_eager_tree_attention``, mtp_kernels.py:859-872.

    q [B,H,D], k/v [B,H,L,D], mask [L] float (key j kept iff mask[j] > 0.5,
    shared by every b, h).  Float32 result.
    """
    qf, kf, vf = (np.asarray(a, dtype=np.float32) for a in (q, k, v))
    scores = np.einsum("bhd,bhld->bhl", qf, kf) * np.float32(scale)
    keep = np.asarray(mask, dtype=np.float32)[None, None, :] > 0.5
    scores = np.where(keep, scores, np.float32(-np.inf))
    with np.errstate(invalid="ignore"):
        p = _softmax_rows(scores)
    return np.einsum("bhl,bhld->bhd", p, vf).astype(np.float32)


def tree_attn_rmsnorm_linear(q: np.ndarray, k: np.ndarray, v: np.ndarray, mask: np.ndarray,
                             rms_w: Optional[np.ndarray], proj_w: np.ndarray,
                             proj_bias: Optional[np.ndarray], wscale: Optional[np.ndarray],
                             scale: float, eps: float) -> np.ndarray:
    """``_eager_tree_attn_rmsnorm_linear``, mtp_kernels.py:881-905, which the
    public ``fused_tree_attn_rmsnorm_linear`` (mtp_kernels.py:1222-1250)
    calls unconditionally.

    q [B,H,D], k/v [B,H,L,D], mask [L] (shared by every b, h); the attention
    output stays float32 (no rounding to q.dtype, 884-895), then
    ``attn * rsqrt(mean(attn**2) + eps) * rms_w`` (896-899; rms_w None = ones),
    then ``attn @ (proj_w * wscale[:, None])^T + proj_bias`` (900-904).
    A row whose keys are all masked is NaN, as in the reference.  Float32
    result [B,H,N].
    """
    attn = tree_attention(q, k, v, mask, scale)  # the same softmax(q k^T) v, float32
    D = attn.shape[-1]
    rw = np.ones(D, np.float32) if rms_w is None else np.asarray(rms_w, dtype=np.float32)
    with np.errstate(invalid="ignore"):
        ms = (attn * attn).mean(axis=-1, keepdims=True)
        attn = attn * (np.float32(1.0) / np.sqrt(ms + np.float32(eps))) * rw
    w = np.asarray(proj_w, dtype=np.float32)
    if wscale is not None:
        w = w * np.asarray(wscale, dtype=np.float32)[:, None]
    out = np.einsum("bhd,nd->bhn", attn, w)
    if proj_bias is not None:
        out = out + np.asarray(proj_bias, dtype=np.float32)
    return out.astype(np.float32)


def causal_attention_scaled(q: np.ndarray, k: np.ndarray, v: np.ndarray,
                            kscale: Optional[np.ndarray], vscale: Optional[np.ndarray],
                            scale: float) -> np.ndarray:
    """``_eager_causal_attention_fp8``, mtp_kernels.py:817-830 (k * kscale[h],
    v * vscale[h], every key kept); with no scales ``_eager_causal_attention``,
    790-802.  k/v given as float32 values (decoded E4M3 for the fp8 cache).
    Float32 result [B,H,D]."""
    kf = np.asarray(k, dtype=np.float32)
    vf = np.asarray(v, dtype=np.float32)
    if kscale is not None:
        kf = kf * np.asarray(kscale, dtype=np.float32)[None, :, None, None]
        vf = vf * np.asarray(vscale, dtype=np.float32)[None, :, None, None]
    return tree_attention(q, kf, vf, np.ones(kf.shape[2], np.float32), scale)


def quantize_int4(x: np.ndarray, group: int = 32) -> Tuple[np.ndarray, np.ndarray]:
    """mtp_kernels.py:730-751: per row and group s = amax / 7 (1 if amax == 0),
    q = clamp(round_half_even(x / s), -8, 7), packed as the low nibble of q's
    two's-complement byte, two per byte, low nibble first."""
    xf = np.asarray(x, dtype=np.float32)
    N, K = xf.shape
    G = (K + group - 1) // group
    scales = np.empty((N, G), np.float32)
    q = np.empty((N, K), np.int32)
    for g in range(G):
        c0, c1 = g * group, min((g + 1) * group, K)
        amax = np.abs(xf[:, c0:c1]).max(axis=1)
        s = np.where(amax > 0, amax / np.float32(7.0), np.float32(1.0)).astype(np.float32)
        scales[:, g] = s
        q[:, c0:c1] = np.clip(np.round(xf[:, c0:c1] / s[:, None]), -8, 7).astype(np.int32)
    nib = q & 0x0F
    packed = (nib[:, 0:K - K % 2:2] | (nib[:, 1:K:2] << 4)).astype(np.uint8)
    return packed, scales


def dequantize_int4(packed: np.ndarray, scales: np.ndarray, K: int, group: int) -> np.ndarray:
    """mtp_kernels.py:754-767: code - 8 from each nibble (low first), times
    scales[n, k // group]; float32 [N, K]."""
    b = np.asarray(packed, dtype=np.int32)
    w = np.stack([(b & 0x0F) - 8, ((b >> 4) & 0x0F) - 8], axis=-1).reshape(b.shape[0], -1)[:, :K]
    g = np.arange(K) // group
    return w.astype(np.float32) * np.asarray(scales, dtype=np.float32)[:, g]


def int4_matmul(x: np.ndarray, packed: np.ndarray, scales: np.ndarray, K: int, group: int) -> np.ndarray:
    """``_eager_int4_matmul``, mtp_kernels.py:875-878: linear(x, dequant(W)),
    float32."""
    return (np.asarray(x, dtype=np.float32) @ dequantize_int4(packed, scales, K, group).T).astype(np.float32)


def gather_paged_kv(pages: np.ndarray, page_table: np.ndarray, page_size: int,
                    L: Optional[int] = None) -> np.ndarray:
    """Per-token page gather of ``_eager_paged_attention``, mtp_kernels.py:839-848.

    pages [P,B,H,page_size,D], page_table [B,Lmax] int (page id per token);
    token t of sequence b lives at pages[page_table[b,t], b, :, t % page_size].
    Returns [B,H,L,D].
    """
    B, Lmax = page_table.shape
    L = Lmax if L is None else L
    t = np.arange(L)
    slot = t % page_size
    page = np.asarray(page_table[:, :L], dtype=np.int64)  # [B, L]
    b_idx = np.arange(B)[:, None]
    g = pages[page, b_idx, :, slot[None, :], :]  # [B, L, H, D]
    return np.ascontiguousarray(np.transpose(g, (0, 2, 1, 3)))


def paged_attention(q: np.ndarray, k_pages: np.ndarray, v_pages: np.ndarray,
                    page_table: np.ndarray, page_size: int, scale: float) -> np.ndarray:
    """``_eager_paged_attention``, mtp_kernels.py:832-856 (float32 result)."""
    k = gather_paged_kv(k_pages, page_table, page_size)
    v = gather_paged_kv(v_pages, page_table, page_size)
    L = k.shape[2]
    return tree_attention(q, k, v, np.ones(L, dtype=np.float32), scale)


def paged_kv_write(k_pages: np.ndarray, v_pages: np.ndarray, page_table: np.ndarray, start: int,
                   k_new: np.ndarray, v_new: np.ndarray, node_idx: Optional[np.ndarray] = None,
                   count: Optional[np.ndarray] = None) -> Tuple[np.ndarray, np.ndarray]:
    """Batched ``PagedKVCache.write_inplace``, mtp_engine.py:582-586: for each
    token t, sequence b and head h, pid = page_table[b, start + t],
    slot = (start + t) % page_size, pages[pid, b, h, slot] = new[b, h, node].
    node = node_idx[b, t] or t; count[b] limits the tokens of sequence b.
    Returns updated copies (values converted to the pool dtype by the caller)."""
    kp, vp = np.array(k_pages, copy=True), np.array(v_pages, copy=True)
    P, B, H, ps, D = kp.shape
    n = node_idx.shape[1] if node_idx is not None else k_new.shape[2]
    for b in range(B):
        nb = n if count is None else min(n, int(count[b]))
        for t in range(nb):
            logical = start + t
            pid = int(page_table[b, logical])
            node = int(node_idx[b, t]) if node_idx is not None else t
            for h in range(H):
                kp[pid, b, h, logical % ps] = k_new[b, h, node]
                vp[pid, b, h, logical % ps] = v_new[b, h, node]
    return kp, vp


def tree_attention_paged(q: np.ndarray, k_pages: np.ndarray, v_pages: np.ndarray,
                         page_table: np.ndarray, ctx_len: int, page_size: int,
                         tree_k: np.ndarray, tree_v: np.ndarray, tree_mask: np.ndarray,
                         scale: float) -> np.ndarray:
    """Paged tree attention with GQA -- the composite operator.

    The reference has no single function for it; it is the composition of
    ``_eager_paged_attention`` (context keys, page gather of
    mtp_kernels.py:839-848) and ``_eager_tree_attention`` (tree keys under a
    mask, mtp_kernels.py:859-872).  For tree node n and query head h (KV head
    h // (Hq/Hkv)) the keys are all ``ctx_len`` context tokens of sequence b
    followed by the tree nodes m with tree_mask[n, m] > 0.5 (the static
    ancestor mask of SpeculativeDraftTree, mtp_engine.py:671-680).

    q [B,T,Hq,D]; pages [P,B,Hkv,page_size,D]; page_table [B,>=ctx_len];
    tree_k/tree_v [B,Hkv,T,D]; tree_mask [T,T].  Returns [B,T,Hq,D] float32.
    """
    qf = np.asarray(q, dtype=np.float32)
    B, T, Hq, D = qf.shape
    Hkv = tree_k.shape[1]
    G = Hq // Hkv
    kc = gather_paged_kv(k_pages, page_table, page_size, ctx_len).astype(np.float32)
    vc = gather_paged_kv(v_pages, page_table, page_size, ctx_len).astype(np.float32)
    K = np.concatenate([kc, np.asarray(tree_k, dtype=np.float32)], axis=2)  # [B,Hkv,L+T,D]
    V = np.concatenate([vc, np.asarray(tree_v, dtype=np.float32)], axis=2)
    K = np.repeat(K, G, axis=1)  # GQA: q head h uses kv head h // G
    V = np.repeat(V, G, axis=1)
    out = np.empty((B, T, Hq, D), dtype=np.float32)
    tm = np.asarray(tree_mask, dtype=np.float32)
    for n in range(T):
        mask = np.concatenate([np.ones(ctx_len, dtype=np.float32), tm[n]])
        out[:, n] = tree_attention(qf[:, n], K, V, mask, scale)
    return out


def tree_attention_paged_fast(q: np.ndarray, k_pages: np.ndarray, v_pages: np.ndarray,
                              page_table: np.ndarray, ctx_len: int, page_size: int,
                              tree_k: np.ndarray, tree_v: np.ndarray, tree_mask: np.ndarray,
                              scale: float) -> np.ndarray:
    """Same result as ``tree_attention_paged`` (checked by the CPU tests),
    computed per (b, kv head) with one BLAS matmul over all T*G query rows --
    the form the CPU baseline of bench.py times."""
    qf = np.asarray(q, dtype=np.float32)
    B, T, Hq, D = qf.shape
    Hkv = tree_k.shape[1]
    G = Hq // Hkv
    Tk = tree_k.shape[2]
    kc = gather_paged_kv(k_pages, page_table, page_size, ctx_len).astype(np.float32)
    vc = gather_paged_kv(v_pages, page_table, page_size, ctx_len).astype(np.float32)
    keep = np.concatenate([np.ones((T, ctx_len), bool), np.asarray(tree_mask)[:, :Tk] > 0.5], axis=1)
    out = np.empty((B, T, Hq, D), dtype=np.float32)
    for b in range(B):
        for h in range(Hkv):
            K = np.concatenate([kc[b, h], np.asarray(tree_k[b, h], np.float32)], axis=0)  # [L+T, D]
            V = np.concatenate([vc[b, h], np.asarray(tree_v[b, h], np.float32)], axis=0)
            Q = qf[b, :, h * G:(h + 1) * G, :].reshape(T * G, D)  # rows (t, g)
            s = (Q @ K.T) * np.float32(scale)
            s = np.where(np.repeat(keep, G, axis=0), s, np.float32(-np.inf))
            with np.errstate(invalid="ignore"):
                p = _softmax_rows(s)
            out[b, :, h * G:(h + 1) * G, :] = (p @ V).reshape(T, G, D)
    return out


# --------------------------------------------------------------------------- #
# speculative draft tree (mask contract)
# --------------------------------------------------------------------------- #


def draft_tree(depth: int, max_branches: int = 8, mode: str = "tree") -> Tuple[np.ndarray, np.ndarray]:
    """Parent index and ancestor mask of SpeculativeDraftTree, mtp_engine.py:635-680."""
    max_nodes = depth * max_branches
    parent = np.full(max_nodes, -1, dtype=np.int32)
    if mode == "trunk":
        for i in range(1, depth):
            parent[i] = i - 1
    else:
        frontier, idx = [0], 1
        for _ in range(1, depth):
            nxt = []
            for p in frontier:
                for _ in range(max_branches):
                    if idx < max_nodes:
                        parent[idx] = p
                        nxt.append(idx)
                        idx += 1
            frontier = nxt
    mask = np.zeros((max_nodes, max_nodes), dtype=np.float32)
    for n in range(1, max_nodes):
        p = int(parent[n])
        while p >= 0:
            mask[n, p] = 1.0
            p = int(parent[p])
        mask[n, n] = 1.0
    mask[0, 0] = 1.0
    return parent, mask


# --------------------------------------------------------------------------- #
# verification
# --------------------------------------------------------------------------- #


def logits_f32(hidden: np.ndarray, w: np.ndarray, bias: Optional[np.ndarray]) -> np.ndarray:
    """F.linear(hidden.float(), W.float(), bias), mtp_fused_verify.py:163, 179-181."""
    lg = np.asarray(hidden, dtype=np.float32) @ np.asarray(w, dtype=np.float32).T
    if bias is not None:
        lg = lg + np.asarray(bias, dtype=np.float32)
    return lg.astype(np.float32)


def fused_verify(hidden: np.ndarray, w: np.ndarray, bias: Optional[np.ndarray],
                 draft: np.ndarray) -> Tuple[np.ndarray, np.ndarray]:
    """``_eager_fused_verify``, mtp_fused_verify.py:159-166 -> (accept int8, top int32)."""
    top = logits_f32(hidden, w, bias).argmax(axis=-1).astype(np.int32)
    accept = (top == np.asarray(draft).astype(np.int32)).astype(np.int8)
    return accept, top


def chain_accept(top: np.ndarray, draft: np.ndarray) -> Tuple[np.ndarray, np.ndarray, np.ndarray]:
    """Prefix-gated acceptance scan, mtp_fused_verify.py:184-195.

    top [B,S] argmax tokens, draft [B,D], S == D+1.  accept[b,d] is 1 only if
    draft d matches top[b,d+1] and every earlier draft matched (the loop
    breaks at the first reject, leaving later entries 0); accepted_n is the
    accepted prefix length; corrected is the anchor argmax top[b,0].
    """
    top = np.asarray(top, dtype=np.int32)
    draft = np.asarray(draft).astype(np.int32)
    B, S = top.shape
    D = draft.shape[1]
    accept = np.zeros((B, D), dtype=np.int8)
    accepted_n = np.zeros((B,), dtype=np.int32)
    for b in range(B):
        n = 0
        for d in range(D):
            if top[b, d + 1] == draft[b, d]:
                accept[b, d] = 1
                n = d + 1
            else:
                break
        accepted_n[b] = n
    corrected = (top[:, 0] if S > 0 else np.zeros((B,), np.int32)).astype(np.int32)
    return accept, accepted_n, corrected


def fused_multi_verify(hidden: np.ndarray, w: np.ndarray, bias: Optional[np.ndarray],
                       draft: np.ndarray) -> Tuple[np.ndarray, np.ndarray, np.ndarray]:
    """``_eager_fused_multi_verify``, mtp_fused_verify.py:169-196.

    hidden [B,S,K], W [V,K], draft [B,D], S == D+1 (asserted by the wrapper,
    mtp_fused_verify.py:262).  Returns (accept [B,D] int8, accepted_n [B]
    int32, corrected [B] int32).
    """
    B, S, K = hidden.shape
    assert S == draft.shape[1] + 1
    top = logits_f32(hidden, w, bias).argmax(axis=-1).astype(np.int32).reshape(B, S)
    return chain_accept(top, draft)


def verify_step(draft: np.ndarray, accepted_n: np.ndarray, corrected: np.ndarray,
                variant: str = "optimized") -> Tuple[np.ndarray, int]:
    """The host step after fused_multi_verify, restated from the reference's
    inline code (no function of its own there):
    ``generate_optimized`` (mtp_engine.py:1326-1337): n = min(accepted_n);
    n == depth -> draft; n == 0 -> corrected[:, None]; else
    cat(draft[:, :n], corrected[:, None]).
    ``generate_fused`` (mtp_engine.py:1244-1258): a_n = min(accepted_n);
    has_reject = sum(accept) < depth * batch (equivalently a_n < depth);
    cat(draft[:, :a_n], corrected[:, None]) if has_reject else draft.
    Returns (new_tokens [B, width] int32, n)."""
    draft = np.asarray(draft, dtype=np.int32)
    B, depth = draft.shape
    corr = np.asarray(corrected, dtype=np.int32)
    n = int(np.asarray(accepted_n).min())
    if variant == "optimized":
        if n == depth:
            return draft.copy(), n
        if n == 0:
            return corr[:, None].copy(), n
        return np.concatenate([draft[:, :n], corr[:, None]], axis=1), n
    has_reject = n < depth
    if has_reject:
        return np.concatenate([draft[:, :n], corr[:, None]], axis=1), n
    return draft.copy(), n


def top2_margin(hidden: np.ndarray, w: np.ndarray, bias: Optional[np.ndarray]) -> np.ndarray:
    """Gap between the largest and second-largest fp32 logit per row."""
    lg = logits_f32(hidden.reshape(-1, hidden.shape[-1]), w, bias)
    part = np.partition(lg, -2, axis=-1)
    return (part[:, -1] - part[:, -2]).astype(np.float32)


# --------------------------------------------------------------------------- #
# vocab-sharded verify: packed (max logit, index) keys
# --------------------------------------------------------------------------- #


def ordered_i32(x: np.ndarray) -> np.ndarray:
    """float32 -> int32 whose signed order equals the float order."""
    i = np.ascontiguousarray(x, dtype=np.float32).view(np.int32)
    return np.where(i < 0, i ^ np.int32(0x7FFFFFFF), i).astype(np.int32)


def pack_key(value: np.ndarray, index: np.ndarray) -> np.ndarray:
    """int64 key: signed-ordered value in the high word, 0xFFFFFFFF - index low.

    max(key) over a set of (value, index) pairs selects the largest value and,
    among equal values, the smallest index -- torch.argmax's tie rule.
    """
    hi = ordered_i32(value).astype(np.int64) << 32
    lo = (np.uint32(0xFFFFFFFF) - np.asarray(index, dtype=np.uint32)).astype(np.int64)
    return hi | lo


def key_index(key: np.ndarray) -> np.ndarray:
    lo = (np.asarray(key, dtype=np.int64) & np.int64(0xFFFFFFFF)).astype(np.uint32)
    return (np.uint32(0xFFFFFFFF) - lo).astype(np.int32)


def shard_argmax_keys(hidden2d: np.ndarray, w_shard: np.ndarray, bias_shard: Optional[np.ndarray],
                      vocab_offset: int) -> np.ndarray:
    """Per-rank row keys for a contiguous vocabulary block [offset, offset+V_r)."""
    lg = logits_f32(hidden2d, w_shard, bias_shard)
    idx = lg.argmax(axis=-1)
    val = lg[np.arange(lg.shape[0]), idx]
    return pack_key(val, idx + vocab_offset)


def vocab_shard_bounds(V: int, world: int) -> List[Tuple[int, int]]:
    """Contiguous row blocks of torch.chunk(W, world, dim=0) (mtp_parallel.py:62-66)."""
    step = -(-V // world)
    return [(min(r * step, V), min((r + 1) * step, V)) for r in range(world)]


def vocab_sharded_multi_verify(hidden: np.ndarray, w: np.ndarray, bias: Optional[np.ndarray],
                               draft: np.ndarray, world: int):
    """Vocab-parallel verify: per-shard keys, max-combine, chain scan.

    Must equal ``fused_multi_verify`` on the full weight (exact, since each
    logit is computed identically and the combine is an exact max).
    """
    B, S, K = hidden.shape
    h2 = hidden.reshape(B * S, K)
    keys = None
    for lo, hi in vocab_shard_bounds(w.shape[0], world):
        if hi <= lo:
            continue
        kb = shard_argmax_keys(h2, w[lo:hi], None if bias is None else bias[lo:hi], lo)
        keys = kb if keys is None else np.maximum(keys, kb)
    top = key_index(keys).reshape(B, S)
    return chain_accept(top, draft)


__all__ = [n for n in dir() if not n.startswith("_")]
