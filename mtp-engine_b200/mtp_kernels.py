"""B200-native drop-in for the hot-path operators of the reference's
``mtp_kernels`` module (Dahacker444/mtp-engine).

Same function names, positional order, defaults and return dtypes as the
reference; every call validates on the host, allocates its outputs with
torch on the input's device and launches hand-written sm_100a kernels from
``libmtp_b200.so`` on the current CUDA stream (no host synchronisation, no
cudaMalloc: safe inside ``torch.cuda.graph`` capture, which is how the
reference calls ``fused_rmsnorm_linear``, mtp_engine.py:1053-1058).

Operators provided here (reference file:line):
  fused_rmsnorm_linear       mtp_kernels.py:936-977   (+ keyword norm_weight)
  fused_rmsnorm_linear_fp8   mtp_kernels.py:1014-1044 (+ keywords x_scale, out_dtype)
  fused_tree_attention       mtp_kernels.py:1165-1191
  fused_paged_attention      mtp_kernels.py:1136-1162
  fused_tree_attention_paged (new: paged context + tree nodes, GQA)
  fused_tree_attn_rmsnorm_linear
                             mtp_kernels.py:1222-1250
  fused_causal_attention     mtp_kernels.py:980-1006
  fused_causal_attention_fp8 mtp_kernels.py:1105-1133
  fused_int4_matmul          mtp_kernels.py:1194-1219
  paged_kv_write             (new: batched PagedKVCache.write_inplace, mtp_engine.py:582-586)
  quantize_fp8_e4m3 / dequantize_fp8 / quantize_int4 / dequantize_int4 /
  pack_scales / unpack_scale_tensor
                             mtp_kernels.py:704-767, 1336-1353
  TUNING / KernelTuningConfig / MAX_FP8 / build_tuning_config (API compatibility)

Operators of the reference module that are not on the verification path
(bitmask attention, add-rmsnorm, autotuning wrappers, ...) are not
reimplemented.
If MTP_REFERENCE_PATH names a checkout of the reference, such names resolve
to the reference's own implementation (so ``from mtp_kernels import ...`` in
the reference's engine keeps working); otherwise they raise AttributeError.
"""

from __future__ import annotations

import importlib.util
import math
import os
import sys
from dataclasses import dataclass
from typing import List, Optional, Tuple

import torch

import _mtp_native as _N

# This package contains no Triton code.  Reference modules that branch on
# this flag (mtp_fused_verify.py:30, mtp_pipeline.py:7) take their eager path.
_HAS_TRITON = False

MAX_FP8 = 448.0  # largest finite float8_e4m3fn value

# Importing the reference module turns TF32 off for torch's own fp32 matmuls
# (mtp_kernels.py:14-16), so a caller's F.linear comparisons run in full
# fp32; the drop-in keeps that side effect.  It does not touch these kernels.
if torch.cuda.is_available():
    torch.backends.cuda.matmul.allow_tf32 = False
    torch.backends.cudnn.allow_tf32 = False


@dataclass(frozen=True)
class KernelTuningConfig:
    """Kept for API compatibility, with the reference's fields and defaults
    (mtp_kernels.py:54-62).  Tiling of the sm_100a kernels is fixed at
    compile time; only ``fp8_scale`` is read (the default ``scale`` of
    fused_rmsnorm_linear, mtp_kernels.py:943-944)."""

    BLOCK_M: int = 64
    BLOCK_N: int = 64
    BLOCK_K: int = 32
    BLOCK_DHEAD: int = 64
    num_warps: int = 4
    num_stages: int = 2
    fp8_scale: float = 1.0


TUNING = KernelTuningConfig()


def build_tuning_config() -> KernelTuningConfig:
    """The values the reference's build_tuning_config returns for the
    current device (mtp_kernels.py:91-103); informational only here."""
    if torch.cuda.is_available():
        major = torch.cuda.get_device_capability(0)[0]
        if major >= 9:
            return KernelTuningConfig(BLOCK_M=128, BLOCK_N=128, BLOCK_K=64, BLOCK_DHEAD=128, num_warps=8,
                                      num_stages=3)
        if major == 8:
            return KernelTuningConfig(BLOCK_M=128, BLOCK_N=64, BLOCK_K=32, BLOCK_DHEAD=64, num_warps=4,
                                      num_stages=2)
    return KernelTuningConfig()


# --------------------------------------------------------------------------- #
# RMSNorm -> linear
# --------------------------------------------------------------------------- #
def fused_rmsnorm_linear(
    x: torch.Tensor,
    weight: torch.Tensor,
    bias: Optional[torch.Tensor] = None,
    eps: float = 1e-6,
    scale: Optional[float] = None,
    *,
    norm_weight: Optional[torch.Tensor] = None,
) -> torch.Tensor:
    """``y = ((x * rsqrt(mean(x^2) + eps)) * norm_weight) @ weight.T + bias) * scale``.

    x [M, K], weight [N, K], bias [N] or None; returns [M, N] in x.dtype.
    ``norm_weight`` (the RMSNorm gamma, [K]) is an addition to the
    reference's signature, which has none (mtp_kernels.py:936-942).
    bf16/f16 inputs run a tcgen05 tensor-core GEMM with fp32 accumulation;
    fp32 inputs run an IEEE fp32 CUDA-core GEMM.
    """
    if scale is None:
        scale = TUNING.fp8_scale
    x = x.contiguous()
    weight = weight.contiguous()
    M, K = x.shape
    N, K2 = weight.shape
    assert K == K2, f"x has K={K}, weight has K={K2}"
    dev = _N.require_cuda(x, weight, bias, norm_weight)
    if bias is not None:
        bias = bias.contiguous().to(dtype=x.dtype, device=x.device)  # mtp_kernels.py:952-953
    if norm_weight is not None:
        norm_weight = norm_weight.contiguous()
        assert norm_weight.shape == (K,), "norm_weight must have shape [K]"
    y = torch.empty((M, N), dtype=x.dtype, device=x.device)
    L = _N.lib()
    ws = _N.gemm_workspace(dev, "rmsnorm_linear", L.mtp_rmsnorm_linear_workspace(M, K, int(norm_weight is not None)),
                           M, N, K, _N.dtype_code(x))
    _N.check(L.mtp_rmsnorm_linear(
        _N.ptr(x), _N.dtype_code(x), _N.ptr(weight), _N.dtype_code(weight),
        _N.ptr(bias), _N.dtype_code(bias) if bias is not None else 0,
        _N.ptr(norm_weight), _N.dtype_code(norm_weight) if norm_weight is not None else 0,
        _N.ptr(y), _N.dtype_code(y), M, N, K, float(eps), float(scale),
        _N.ptr(ws), ws.numel(), _N.stream_handle(dev)), "fused_rmsnorm_linear")
    return y


def fused_rmsnorm_linear_fp8(
    x: torch.Tensor,
    weight_fp8: torch.Tensor,
    wscale: torch.Tensor,
    bias: Optional[torch.Tensor] = None,
    eps: float = 1e-6,
    *,
    x_scale: Optional[torch.Tensor] = None,
    out_dtype: Optional[torch.dtype] = None,
) -> torch.Tensor:
    """``y = rmsnorm(x) @ (weight_fp8 * wscale[:, None]).T + bias``.

    weight_fp8 [N, K]; wscale [N] fp32 per output channel -- typically a
    view into the flat buffer of ``pack_scales`` (``unpack_scale_tensor``).
    With a float8_e4m3fn weight the activations are quantised per token
    (scale amax/448) and the GEMM runs on the FP8 tensor cores; the result
    equals the reference evaluated on the dequantised activations.  Pass
    pre-quantised activations as an e4m3 ``x`` plus ``x_scale`` [M].
    Any other weight dtype (the reference's fp32-valued self-check weight,
    mtp_engine.py:1792-1800) runs unquantised in fp32.
    Output dtype: x.dtype (reference), or ``out_dtype`` / bf16 for e4m3 x.
    """
    x = x.contiguous()
    weight_fp8 = weight_fp8.contiguous()
    wscale = wscale.contiguous().to(torch.float32)
    M, K = x.shape
    N = weight_fp8.shape[0]
    assert weight_fp8.shape[1] == K and wscale.numel() == N
    dev = _N.require_cuda(x, weight_fp8, wscale, bias, x_scale)
    x_is_fp8 = _N.dtype_code(x) == _N.DT_E4M3
    if x_is_fp8:
        if x_scale is None:
            raise ValueError("pre-quantised e4m3 activations need x_scale [M]")
        x_scale = x_scale.contiguous().to(torch.float32)
    if out_dtype is None:
        out_dtype = torch.bfloat16 if x_is_fp8 else x.dtype
    if bias is not None:
        bias = bias.contiguous()
    y = torch.empty((M, N), dtype=out_dtype, device=x.device)
    L = _N.lib()
    ws = _N.gemm_workspace(dev, "rmsnorm_linear_fp8", L.mtp_rmsnorm_linear_fp8_workspace(M, K), M, N, K,
                           _N.DT_E4M3)
    _N.check(L.mtp_rmsnorm_linear_fp8(
        _N.ptr(x), _N.dtype_code(x), _N.ptr(x_scale), _N.ptr(weight_fp8), _N.dtype_code(weight_fp8),
        _N.ptr(wscale), _N.ptr(bias), _N.dtype_code(bias) if bias is not None else 0,
        _N.ptr(y), _N.dtype_code(y), M, N, K, float(eps), _N.ptr(ws), ws.numel(),
        _N.stream_handle(dev)), "fused_rmsnorm_linear_fp8")
    return y


# --------------------------------------------------------------------------- #
# attention
# --------------------------------------------------------------------------- #
def fused_tree_attention(
    q: torch.Tensor, k: torch.Tensor, v: torch.Tensor, mask: torch.Tensor,
    scale: Optional[float] = None,
) -> torch.Tensor:
    """Single-query attention per (b, h) over L contiguous keys; key j is
    used iff mask[j] > 0.5 (mask [L] shared by every b, h).
    q [B,H,D], k/v [B,H,L,D] -> [B,H,D] in q.dtype."""
    q, k, v = q.contiguous(), k.contiguous(), v.contiguous()
    B, H, D = q.shape
    L = k.shape[2]
    assert k.shape == (B, H, L, D) and v.shape == (B, H, L, D)
    if scale is None:
        scale = 1.0 / math.sqrt(D)
    dev = _N.require_cuda(q, k, v, mask)
    mask = mask.contiguous().to(torch.float32)
    assert mask.numel() == L
    k, v = k.to(q.dtype), v.to(q.dtype)
    out = torch.empty_like(q)
    _N.check(_N.lib().mtp_tree_attention(
        _N.ptr(q), _N.ptr(k), _N.ptr(v), _N.ptr(mask), _N.ptr(out), _N.dtype_code(q),
        B, H, L, D, float(scale), _N.stream_handle(dev)), "fused_tree_attention")
    return out


def fused_causal_attention(
    q: torch.Tensor, k: torch.Tensor, v: torch.Tensor, scale: Optional[float] = None,
) -> torch.Tensor:
    """Single-query attention per (b, h) over all L keys (mtp_kernels.py:980-1006;
    eager 790-802).  q [B,H,D], k/v [B,H,L,D] -> [B,H,D] in q.dtype."""
    return _scaled_attention(q, k, v, None, None, scale, "fused_causal_attention")


def fused_causal_attention_fp8(
    q: torch.Tensor, k_fp8: torch.Tensor, v_fp8: torch.Tensor,
    kscale: torch.Tensor, vscale: torch.Tensor, scale: Optional[float] = None,
) -> torch.Tensor:
    """Single-query attention with an FP8 (or any-dtype) KV cache scaled per
    head: k = k_fp8 * kscale[h], v = v_fp8 * vscale[h] (mtp_kernels.py:1105-1133;
    eager 817-830).  q [B,H,D], k_fp8/v_fp8 [B,H,L,D], kscale/vscale [H]."""
    return _scaled_attention(q, k_fp8, v_fp8, kscale, vscale, scale, "fused_causal_attention_fp8")


def _scaled_attention(q, k, v, kscale, vscale, scale, what):
    q, k, v = q.contiguous(), k.contiguous(), v.contiguous()
    B, H, D = q.shape
    _B, _H, L, _D = k.shape
    assert (B, H, D) == (_B, _H, _D) and v.shape == k.shape  # mtp_kernels.py:1116
    if scale is None:
        scale = 1.0 / math.sqrt(D)
    dev = _N.require_cuda(q, k, v, kscale, vscale)
    v = v.to(k.dtype)
    if kscale is not None:
        kscale = kscale.contiguous().to(torch.float32)
        vscale = vscale.contiguous().to(torch.float32)
        assert kscale.numel() == H and vscale.numel() == H
    out = torch.empty_like(q)
    _N.check(_N.lib().mtp_causal_attention_scaled(
        _N.ptr(q), _N.dtype_code(q), _N.ptr(k), _N.ptr(v), _N.dtype_code(k), _N.ptr(kscale), _N.ptr(vscale),
        _N.ptr(out), B, H, L, D, float(scale), _N.stream_handle(dev)), what)
    return out


def fused_paged_attention(
    q: torch.Tensor, k_pages: torch.Tensor, v_pages: torch.Tensor,
    page_table: torch.Tensor, page_size: int, scale: Optional[float] = None,
) -> torch.Tensor:
    """Single-query attention over a PagedKVCache pool (mtp_engine.py:523-610).
    q [B,H,D]; k/v_pages [P,B,H,page_size,D]; page_table [B,L] int (page id
    per token; token t sits in slot t % page_size) -> [B,H,D]."""
    q, k_pages, v_pages = q.contiguous(), k_pages.contiguous(), v_pages.contiguous()
    page_table = page_table.contiguous().to(torch.int32)
    B, H, D = q.shape
    L = page_table.shape[-1]
    P = k_pages.shape[0]
    assert k_pages.shape == (P, B, H, page_size, D) and v_pages.shape == k_pages.shape
    if scale is None:
        scale = 1.0 / math.sqrt(D)
    dev = _N.require_cuda(q, k_pages, v_pages, page_table)
    k_pages, v_pages = k_pages.to(q.dtype), v_pages.to(q.dtype)
    out = torch.empty_like(q)
    _N.check(_N.lib().mtp_paged_attention(
        _N.ptr(q), _N.ptr(k_pages), _N.ptr(v_pages), _N.ptr(page_table), _N.ptr(out), _N.dtype_code(q),
        B, H, L, D, P, int(page_size), float(scale), _N.stream_handle(dev)), "fused_paged_attention")
    return out


def fused_tree_attention_paged(
    q: torch.Tensor, k_pages: torch.Tensor, v_pages: torch.Tensor, page_table: torch.Tensor,
    tree_k: torch.Tensor, tree_v: torch.Tensor, tree_mask: torch.Tensor,
    ctx_len: Optional[int] = None, scale: Optional[float] = None,
) -> torch.Tensor:
    """Tree attention over paged context (composite of fused_paged_attention
    and fused_tree_attention, with grouped-query heads).

    q [B,T,Hq,D] (T tree nodes); k/v_pages [P,B,Hkv,page_size,D];
    page_table [B, >=ctx_len] int32 per-token page ids; tree_k/tree_v
    [B,Hkv,T,D]; tree_mask [T,T] (SpeculativeDraftTree.tree_mask: node n
    sees node m iff tree_mask[n,m] > 0.5).  Node n, query head h attends to
    the ctx_len context tokens and its visible tree nodes through kv head
    h // (Hq // Hkv).  Returns [B,T,Hq,D] in q.dtype.
    """
    q = q.contiguous()
    k_pages, v_pages = k_pages.contiguous(), v_pages.contiguous()
    page_table = page_table.contiguous().to(torch.int32)
    tree_k, tree_v = tree_k.contiguous(), tree_v.contiguous()
    B, T, Hq, D = q.shape
    P, B2, Hkv, page_size, D2 = k_pages.shape
    assert B2 == B and D2 == D and v_pages.shape == k_pages.shape
    assert tree_k.shape == (B, Hkv, T, D) and tree_v.shape == tree_k.shape
    assert Hq % Hkv == 0
    if ctx_len is None:
        ctx_len = page_table.shape[-1]
    assert page_table.shape[0] == B and page_table.shape[-1] >= ctx_len
    if scale is None:
        scale = 1.0 / math.sqrt(D)
    dev = _N.require_cuda(q, k_pages, v_pages, page_table, tree_k, tree_v, tree_mask)
    tree_mask = tree_mask.contiguous().to(torch.float32)
    assert tree_mask.shape == (T, T)
    out = torch.empty_like(q)
    L = _N.lib()
    ws = _N.workspace(dev, "tree_attention_paged",
                      L.mtp_tree_attention_paged_workspace(B, T, Hq, Hkv, D, int(ctx_len)))
    _N.check(L.mtp_tree_attention_paged(
        _N.ptr(q), _N.ptr(k_pages), _N.ptr(v_pages), _N.ptr(page_table), page_table.shape[-1], int(ctx_len),
        _N.ptr(tree_k), _N.ptr(tree_v), _N.ptr(tree_mask), _N.ptr(out), _N.dtype_code(q),
        B, T, Hq, Hkv, D, P, page_size, float(scale), _N.ptr(ws), ws.numel(), _N.stream_handle(dev)),
        "fused_tree_attention_paged")
    return out


def fused_tree_attn_rmsnorm_linear(
    q: torch.Tensor, k: torch.Tensor, v: torch.Tensor, mask: torch.Tensor,
    proj_w: torch.Tensor,
    rms_w: Optional[torch.Tensor] = None,
    proj_bias: Optional[torch.Tensor] = None,
    wscale: Optional[torch.Tensor] = None,
    scale: Optional[float] = None,
    eps: float = 1e-6,
) -> torch.Tensor:
    """Tree attention -> RMSNorm -> linear in one call (mtp_kernels.py:1222-1250;
    eager semantics _eager_tree_attn_rmsnorm_linear, 881-905).

    q [B,H,D], k/v [B,H,L,D], mask [L] (key j kept iff mask[j] > 0.5, shared
    by every b, h); proj_w [N,D]; rms_w [D], proj_bias [N], wscale [N]
    optional.  Returns [B,H,N] in q.dtype.  The attention output is
    normalised in fp32 (not rounded to q.dtype first, as in the reference)
    and rounded once as the projection's operand; a row whose keys are all
    masked is NaN."""
    q, k, v = q.contiguous(), k.contiguous(), v.contiguous()
    proj_w = proj_w.contiguous()
    B, H, D = q.shape
    L = k.shape[2]
    N = proj_w.shape[0]
    assert k.shape == (B, H, L, D) and v.shape == (B, H, L, D)
    assert proj_w.shape == (N, D)
    if scale is None:
        scale = 1.0 / math.sqrt(D)  # mtp_kernels.py:1238-1239
    dev = _N.require_cuda(q, k, v, mask, proj_w, rms_w, proj_bias, wscale)
    mask = mask.contiguous().to(torch.float32)
    assert mask.numel() == L
    k, v = k.to(q.dtype), v.to(q.dtype)
    if rms_w is not None:
        rms_w = rms_w.contiguous().to(torch.float32)
        assert rms_w.shape == (D,)
    if wscale is not None:
        wscale = wscale.contiguous().to(torch.float32)
        assert wscale.numel() == N
    if proj_bias is not None:
        proj_bias = proj_bias.contiguous()
        assert proj_bias.numel() == N
    out = torch.empty((B, H, N), dtype=q.dtype, device=q.device)
    Lib = _N.lib()
    qc, wc = _N.dtype_code(q), _N.dtype_code(proj_w)
    operand = qc if (wc == qc and wc in (_N.DT_BF16, _N.DT_F16)) else _N.DT_F32
    ws = _N.gemm_workspace(dev, "tree_attn_rmsnorm_linear",
                           Lib.mtp_tree_attn_rmsnorm_linear_workspace(B, H, D, qc, wc), B * H, N, D, operand)
    _N.check(Lib.mtp_tree_attn_rmsnorm_linear(
        _N.ptr(q), _N.ptr(k), _N.ptr(v), qc, _N.ptr(mask), _N.ptr(rms_w), _N.ptr(proj_w), wc,
        _N.ptr(proj_bias), _N.dtype_code(proj_bias) if proj_bias is not None else 0, _N.ptr(wscale),
        _N.ptr(out), B, H, L, D, N, float(scale), float(eps), _N.ptr(ws), ws.numel(), _N.stream_handle(dev)),
        "fused_tree_attn_rmsnorm_linear")
    return out


def paged_kv_write(
    k_pages: torch.Tensor, v_pages: torch.Tensor, page_table: torch.Tensor, start: int,
    k_new: torch.Tensor, v_new: torch.Tensor,
    node_idx: Optional[torch.Tensor] = None, count: Optional[torch.Tensor] = None,
) -> None:
    """Write new K/V rows into a PagedKVCache pool in one launch (the batched
    form of PagedKVCache.write_inplace, mtp_engine.py:582-586, without its
    per-token .item()).

    k_pages/v_pages [P,B,H,page_size,D] (written in place, must be
    contiguous); page_table [B, L] int32 (PagedKVCache.page_table);
    k_new/v_new [B,H,src_len,D]; row t of sequence b goes to logical position
    start + t and comes from source row node_idx[b, t] ([B, n], e.g. the
    accepted path of a draft tree) or t; count [B] (e.g. accepted_n + 1)
    limits how many rows each sequence writes."""
    assert k_pages.is_contiguous() and v_pages.is_contiguous(), "page pools are written in place"
    P, B, H, page_size, D = k_pages.shape
    assert v_pages.shape == k_pages.shape and v_pages.dtype == k_pages.dtype
    page_table = page_table.contiguous().to(torch.int32)
    k_new, v_new = k_new.contiguous(), v_new.to(k_new.dtype).contiguous()
    assert k_new.shape[:2] == (B, H) and k_new.shape[3] == D and v_new.shape == k_new.shape
    src_len = k_new.shape[2]
    if node_idx is not None:
        node_idx = node_idx.contiguous().to(torch.int32)
        assert node_idx.dim() == 2 and node_idx.shape[0] == B
        n = node_idx.shape[1]
    else:
        n = src_len
    if count is not None:
        count = count.contiguous().to(torch.int32)
        assert count.shape == (B,)
    dev = _N.require_cuda(k_pages, v_pages, page_table, k_new, v_new, node_idx, count)
    _N.check(_N.lib().mtp_paged_kv_write(
        _N.ptr(k_pages), _N.ptr(v_pages), _N.dtype_code(k_pages), _N.ptr(page_table), page_table.shape[-1], P,
        page_size, _N.ptr(k_new), _N.ptr(v_new), _N.dtype_code(k_new), src_len, _N.ptr(node_idx), _N.ptr(count),
        B, H, D, int(start), n, _N.stream_handle(dev)), "paged_kv_write")


def fused_int4_matmul(
    x: torch.Tensor, packed: torch.Tensor, scales: torch.Tensor, K: int, group: int = 32,
) -> torch.Tensor:
    """y = x @ dequantize_int4(packed, scales, K, group)^T in one kernel
    (mtp_kernels.py:1194-1219): x [M,K], packed [N,K/2] uint8 (two codes per
    byte, low nibble first, decoded as code - 8), scales [N, ceil(K/group)].
    Returns [M,N] in x.dtype; fp32 products and sums."""
    x, packed, scales = x.contiguous(), packed.contiguous(), scales.contiguous().to(torch.float32)
    M, _K = x.shape
    assert _K == K  # mtp_kernels.py:1201
    N = packed.shape[0]
    assert packed.dtype == torch.uint8 and packed.shape == (N, K // 2)
    assert scales.shape == (N, (K + group - 1) // group)
    dev = _N.require_cuda(x, packed, scales)
    y = torch.empty((M, N), dtype=x.dtype, device=x.device)
    _N.check(_N.lib().mtp_int4_matmul(_N.ptr(x), _N.dtype_code(x), _N.ptr(packed), _N.ptr(scales), int(group),
                                      _N.ptr(y), _N.dtype_code(y), M, N, K, _N.stream_handle(dev)),
             "fused_int4_matmul")
    return y


def quantize_int4(x: torch.Tensor, group: int = 32) -> Tuple[torch.Tensor, torch.Tensor]:
    """Group-wise 4-bit quantisation, as mtp_kernels.py:730-751 (host-side
    preparation): per row and group of `group` columns s = amax / 7 (1 when
    amax == 0), q = clamp(round(x / s), -8, 7), stored as the low nibble of
    q's two's-complement byte, two per byte (low nibble first).  Note that
    the reference decodes these nibbles as code - 8 (dequantize_int4), and so
    does fused_int4_matmul."""
    N, K = x.shape
    xf = x.to(torch.float32)
    G = (K + group - 1) // group
    pad = G * group - K
    xg = torch.nn.functional.pad(xf, (0, pad)).view(N, G, group)
    amax = xg.abs().amax(dim=-1)
    s = torch.where(amax > 0, amax / 7.0, torch.ones_like(amax))
    q = torch.round(xg / s[..., None]).clamp(-8, 7).to(torch.int8).view(N, G * group)[:, :K]
    nib = q.to(torch.int32) & 0x0F
    if K % 2:
        nib = torch.nn.functional.pad(nib, (0, 1))
    packed = (nib[:, 0::2] | (nib[:, 1::2] << 4)).to(torch.uint8)[:, : K // 2]
    return packed.contiguous(), s.contiguous()


def dequantize_int4(packed: torch.Tensor, scales: torch.Tensor, K: int, group: int) -> torch.Tensor:
    """mtp_kernels.py:754-767: w[n, 2j] = (low nibble - 8), w[n, 2j+1] =
    (high nibble - 8), times scales[n, k // group]; float32 [N, K]."""
    b = packed.to(torch.int32)
    w = torch.stack([(b & 0x0F) - 8, ((b >> 4) & 0x0F) - 8], dim=-1).view(packed.shape[0], -1)[:, :K]
    g = torch.arange(K, device=packed.device) // group
    return w.to(torch.float32) * scales.to(torch.float32)[:, g]


# --------------------------------------------------------------------------- #
# FP8 helpers and the packed scale layout (host-side preparation, torch ops)
# --------------------------------------------------------------------------- #
def quantize_fp8_e4m3(x: torch.Tensor) -> Tuple[torch.Tensor, torch.Tensor]:
    """Per-tensor E4M3: scale = amax/448 (1 if amax == 0), q = e4m3(clamp(x/scale)).
    Same contract as mtp_kernels.py:704-713."""
    xf = x.to(torch.float32)
    amax = xf.abs().max()
    one = torch.ones((), dtype=torch.float32, device=x.device)
    s = torch.where(amax > 0, amax / MAX_FP8, one)
    q = (xf / s).clamp(-MAX_FP8, MAX_FP8).to(torch.float8_e4m3fn)
    return q, s.to(torch.float32)


def quantize_fp8_rows(x: torch.Tensor) -> Tuple[torch.Tensor, torch.Tensor]:
    """Per-row E4M3 (per output channel for a weight [N,K], per token for
    activations [M,K]): scale[r] = amax_r/448 (1 for a zero row), the
    convention of QuantScaleState.update_weight_scales (mtp_engine.py:617-622)."""
    xf = x.to(torch.float32)
    amax = xf.abs().amax(dim=-1)
    s = torch.where(amax > 0, amax / MAX_FP8, torch.ones_like(amax))
    q = (xf / s.unsqueeze(-1)).clamp(-MAX_FP8, MAX_FP8).to(torch.float8_e4m3fn)
    return q, s


def dequantize_fp8(x_fp8: torch.Tensor, scale: torch.Tensor) -> torch.Tensor:
    return x_fp8.to(torch.float32) * scale.to(torch.float32)


def pack_scales(weight_scales: List[torch.Tensor],
                kv_scales: Optional[List[torch.Tensor]] = None) -> Tuple[torch.Tensor, torch.Tensor]:
    """Concatenate scale tensors into one flat fp32 buffer plus int64 offsets
    [n+1] (layout of mtp_kernels.py:1336-1346).  Kernels take
    ``flat[offsets[i]:offsets[i+1]]`` as a plain pointer."""
    tensors = list(weight_scales) + list(kv_scales or [])
    sizes = [int(t.numel()) for t in tensors]
    offsets = [0]
    for n in sizes:
        offsets.append(offsets[-1] + n)
    flat = torch.cat([t.reshape(-1).to(torch.float32) for t in tensors]) if tensors else torch.zeros(0)
    return flat, torch.tensor(offsets, dtype=torch.int64, device=flat.device)


def unpack_scale_tensor(flat: torch.Tensor, offsets: torch.Tensor, idx: int,
                        shape: Tuple[int, ...]) -> torch.Tensor:
    """View of the idx-th scale tensor inside the flat buffer (no copy)."""
    lo, hi = int(offsets[idx]), int(offsets[idx + 1])
    return flat[lo:hi].view(*shape)


# --------------------------------------------------------------------------- #
# names outside the hot path
# --------------------------------------------------------------------------- #
_reference_module = None


def _load_reference():
    global _reference_module
    if _reference_module is None:
        root = os.environ.get("MTP_REFERENCE_PATH")
        if not root:
            return None
        spec = importlib.util.spec_from_file_location("_mtp_reference_kernels", os.path.join(root, "mtp_kernels.py"))
        mod = importlib.util.module_from_spec(spec)
        sys.modules["_mtp_reference_kernels"] = mod
        spec.loader.exec_module(mod)
        _reference_module = mod
    return _reference_module


def __getattr__(name: str):
    if name.startswith("__"):
        raise AttributeError(name)
    ref = _load_reference()
    if ref is not None and hasattr(ref, name):
        return getattr(ref, name)
    raise AttributeError(
        f"mtp_kernels.{name} is not part of the B200 hot path implemented by mtp-engine-b200; "
        "set MTP_REFERENCE_PATH to the reference checkout to resolve it there")


__all__ = [
    "KernelTuningConfig", "TUNING", "MAX_FP8", "build_tuning_config",
    "fused_rmsnorm_linear", "fused_rmsnorm_linear_fp8",
    "fused_tree_attention", "fused_paged_attention", "fused_tree_attention_paged",
    "fused_tree_attn_rmsnorm_linear", "paged_kv_write",
    "fused_causal_attention", "fused_causal_attention_fp8", "fused_int4_matmul", "quantize_int4", "dequantize_int4",
    "quantize_fp8_e4m3", "quantize_fp8_rows", "dequantize_fp8", "pack_scales", "unpack_scale_tensor",
    "_HAS_TRITON",
]
