"""B200-native drop-in for the reference's ``mtp_fused_verify`` module.

``fused_verify`` (mtp_fused_verify.py:199-234) and ``fused_multi_verify``
(mtp_fused_verify.py:237-290) keep their signatures and return tuples.
One kernel launch per call: a tcgen05 lm_head GEMM whose epilogue reduces
every logit row to a packed (value, index) argmax key -- no logits tensor
is ever written -- and whose last CTA decodes the keys into the acceptance
outputs.  bf16/f16 hidden + weight run on the tensor cores with fp32
accumulation; fp32 inputs run an IEEE fp32 CUDA-core GEMM, matching the
reference's fp32 logits (mtp_fused_verify.py:179-181).

Also ``verify_step`` / ``fused_multi_verify_step``: the host step the
reference's generate loops run after the verify (batch-min rollback index
and the step's tokens, mtp_engine.py:1244-1258, 1326-1337), on the device.
"""

from __future__ import annotations

from typing import Optional, Tuple

import torch

import _mtp_native as _N


def _prep(hidden, weight, draft, bias):
    hidden = hidden.contiguous()
    weight = weight.contiguous()
    draft = draft.contiguous().to(torch.int32)
    dev = _N.require_cuda(hidden, weight, draft, bias)
    if bias is not None:
        bias = bias.contiguous()
        assert bias.numel() == weight.shape[0]
    return hidden, weight, draft, bias, dev


def fused_verify(
    hidden: torch.Tensor,
    weight: torch.Tensor,
    draft: torch.Tensor,
    bias: Optional[torch.Tensor] = None,
) -> Tuple[torch.Tensor, torch.Tensor]:
    """top[m] = argmax(hidden[m] @ weight.T + bias); accept[m] = top[m] == draft[m].
    hidden [M,K], weight [V,K], draft [M] -> (accept int8 [M], top int32 [M])."""
    hidden, weight, draft, bias, dev = _prep(hidden, weight, draft, bias)
    M, K = hidden.shape
    V = weight.shape[0]
    assert weight.shape[1] == K and draft.numel() == M
    accept = torch.empty(M, dtype=torch.int8, device=hidden.device)
    top = torch.empty(M, dtype=torch.int32, device=hidden.device)
    if M == 0:
        return accept, top
    ws = _N.verify_workspace(dev, M, V, K, _N.dtype_code(hidden))
    _N.check(_N.lib().mtp_fused_verify(
        _N.ptr(hidden), _N.dtype_code(hidden), _N.ptr(weight), _N.dtype_code(weight),
        _N.ptr(bias), _N.dtype_code(bias) if bias is not None else 0,
        _N.ptr(draft), _N.ptr(accept), _N.ptr(top), M, K, V, _N.ptr(ws), ws.numel(),
        _N.stream_handle(dev)), "fused_verify")
    return accept, top


def fused_multi_verify(
    hidden: torch.Tensor,
    weight: torch.Tensor,
    draft: torch.Tensor,
    bias: Optional[torch.Tensor] = None,
) -> Tuple[torch.Tensor, torch.Tensor, torch.Tensor]:
    """Linear -> argmax -> prefix-gated chain acceptance for a draft chain.

    hidden [B,S,K] (anchor + D drafts, S == D + 1); weight [V,K];
    draft [B,D]; bias [V] or None.  Returns
      accept     [B,D] int8  (1 while every earlier draft was accepted too)
      accepted_n [B]   int32 (accepted prefix length = rollback index)
      corrected  [B]   int32 (argmax at the anchor position 0)
    """
    hidden, weight, draft, bias, dev = _prep(hidden, weight, draft, bias)
    B, S, K = hidden.shape
    V = weight.shape[0]
    D = draft.shape[1]
    assert S == D + 1, f"expected S == D + 1, got S={S} D={D}"
    assert weight.shape[1] == K and draft.shape[0] == B
    accept = torch.empty((B, D), dtype=torch.int8, device=hidden.device)  # fully written
    accepted_n = torch.empty((B,), dtype=torch.int32, device=hidden.device)
    corrected = torch.empty((B,), dtype=torch.int32, device=hidden.device)
    if B == 0:
        return accept, accepted_n, corrected
    ws = _N.verify_workspace(dev, B * S, V, K, _N.dtype_code(hidden))
    _N.check(_N.lib().mtp_fused_multi_verify(
        _N.ptr(hidden), _N.dtype_code(hidden), _N.ptr(weight), _N.dtype_code(weight),
        _N.ptr(bias), _N.dtype_code(bias) if bias is not None else 0,
        _N.ptr(draft), _N.ptr(accept), _N.ptr(accepted_n), _N.ptr(corrected),
        B, S, K, V, _N.ptr(ws), ws.numel(), _N.stream_handle(dev)), "fused_multi_verify")
    return accept, accepted_n, corrected


def verify_step(draft: torch.Tensor, accepted_n: torch.Tensor,
                corrected: torch.Tensor) -> Tuple[torch.Tensor, torch.Tensor]:
    """The host step that follows fused_multi_verify in generate_fused /
    generate_optimized (mtp_engine.py:1244-1258, 1326-1337), on the device.

    n = accepted_n.min() (one rollback index for the batch); the step's new
    tokens are draft[:, :n] followed by corrected when n < D, else draft.
    Returns (step_tokens [B, D+1] int32, info [2] int32 = (n, width)); the new
    tokens are step_tokens[:, :width] and the columns after them hold -1 (no
    token).  Nothing is read back to the host, so
    a loop can stay on the device (or read the 8 bytes of info once)."""
    dev = _N.require_cuda(draft, accepted_n, corrected)
    draft = draft.contiguous().to(torch.int32)
    accepted_n = accepted_n.contiguous().to(torch.int32)
    corrected = corrected.contiguous().to(torch.int32)
    B, D = draft.shape
    assert accepted_n.shape == (B,) and corrected.shape == (B,)
    step_tokens = torch.empty((B, D + 1), dtype=torch.int32, device=draft.device)
    info = torch.zeros(2, dtype=torch.int32, device=draft.device)
    if B == 0:
        return step_tokens, info
    _N.check(_N.lib().mtp_verify_step(_N.ptr(draft), _N.ptr(accepted_n), _N.ptr(corrected), B, D,
                                      _N.ptr(step_tokens), D + 1, _N.ptr(info), _N.stream_handle(dev)),
             "verify_step")
    return step_tokens, info


def fused_multi_verify_step(hidden: torch.Tensor, weight: torch.Tensor, draft: torch.Tensor,
                            bias: Optional[torch.Tensor] = None):
    """fused_multi_verify followed by verify_step: (accept, accepted_n,
    corrected, step_tokens, info), all on the device, two launches."""
    accept, accepted_n, corrected = fused_multi_verify(hidden, weight, draft, bias)
    step_tokens, info = verify_step(draft, accepted_n, corrected)
    return accept, accepted_n, corrected, step_tokens, info


__all__ = ["fused_verify", "fused_multi_verify", "verify_step", "fused_multi_verify_step"]
