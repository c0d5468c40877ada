"""Causal FlashAttention forward on B200 tensor cores (c3cu_flash_attn_fwd). The reference
has no attention kernel; this is the attention engine the hot path adds."""
from __future__ import annotations

import math

import torch

from . import _lib
from .linear import _p, _require, _stream


@_lib.on_tensor_device
def flash_attn_fwd(Q: torch.Tensor, K: torch.Tensor, V: torch.Tensor, causal: bool = True,
                   scale: float | None = None, out: torch.Tensor | None = None,
                   lse: torch.Tensor | None = None):
    """Q, K, V: [B, H, S, 128] bf16 contiguous CUDA tensors. Returns (O bf16, LSE fp32 [B, H, S])."""
    _require(Q, "Q", torch.bfloat16, 4)
    B, H, S, D = Q.shape
    _require(K, "K", torch.bfloat16, 4, Q.shape)
    _require(V, "V", torch.bfloat16, 4, Q.shape)
    if scale is None:
        scale = 1.0 / math.sqrt(D)
    if out is None:
        out = torch.empty_like(Q)
    _require(out, "out", torch.bfloat16, 4, Q.shape)
    if lse is None:
        lse = torch.empty((B, H, S), dtype=torch.float32, device=Q.device)
    _require(lse, "lse", torch.float32, 3, (B, H, S))
    rc = _lib.load().c3cu_flash_attn_fwd(_p(Q), _p(K), _p(V), _p(out), _p(lse), B, H, S, D, scale,
                                         int(causal), _stream(Q.device))
    _lib.check(rc, "c3cu_flash_attn_fwd")
    return out, lse
