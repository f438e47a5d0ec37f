"""flash-attn-compatible attention entry points backed by the sm_100a kernel.

The reference calls flash-attn 2 from Attention.apply_attn
(stable_audio_3/models/transformer.py:620-666) through module globals imported
at transformer.py:22-40:

    flash_attn_func(q, k, v, causal=..., window_size=(wl, wr))                   # q,k,v [B, N, H, d]
    flash_attn_varlen_func(q, k, v, cu_q, cu_k, max_q, max_k, causal=..., window_size=...)  # [total, H, d]
    index_first_axis(x, indices), pad_input(x, indices, batch, seqlen)           # flash_attn.bert_padding

This module provides the same callables; install() swaps them into
stable_audio_3.models.transformer so the reference's own modules (and the
sampler above them) run on the B200 kernel unchanged. Arguments the kernel
does not implement (dropout, softcap, ALiBi, returning probabilities) raise.
"""
from __future__ import annotations

import sys
from typing import Optional

import torch

from . import ops


def _check_unsupported(dropout_p, softcap, alibi_slopes, return_attn_probs):
    if dropout_p:
        raise NotImplementedError("dropout is not supported (inference path)")
    if softcap:
        raise NotImplementedError("softcap is not supported")
    if alibi_slopes is not None:
        raise NotImplementedError("ALiBi is not supported")
    if return_attn_probs:
        raise NotImplementedError("return_attn_probs is not supported")


def _window(causal: bool, window_size) -> tuple:
    wl, wr = (int(window_size[0]), int(window_size[1])) if window_size is not None else (-1, -1)
    if causal:  # bottom-right aligned causal mask == right window 0 (flash-attn convention)
        wr = 0 if wr < 0 else min(wr, 0)
    return wl, wr


def _dtype_ok(t: torch.Tensor):
    if t.dtype not in (torch.bfloat16, torch.float16):
        raise RuntimeError("flash_attn_func expects fp16 or bf16 inputs (as flash-attn does)")


def flash_attn_func(q, k, v, dropout_p=0.0, softmax_scale=None, causal=False, window_size=(-1, -1), softcap=0.0,
                    alibi_slopes=None, deterministic=False, return_attn_probs=False):
    """q [B, Nq, H, d], k/v [B, Nk, H, d] (d = 64) -> [B, Nq, H, d]."""
    _check_unsupported(dropout_p, softcap, alibi_slopes, return_attn_probs)
    _dtype_ok(q)
    B, Nq, H, d = q.shape
    Nk = k.shape[1]
    if d != 64:
        raise NotImplementedError("head_dim must be 64")
    if k.shape[2] != H:
        raise NotImplementedError("grouped-query attention: repeat k/v heads first (apply_attn does)")
    q, k, v = (t.contiguous() for t in (q, k, v))
    out = torch.empty_like(q)
    ops.attention(q.view(B * Nq, H * d), k.view(B * Nk, H * d), v.view(B * Nk, H * d), heads=H, batch=B,
                  max_seqlen_q=Nq, max_seqlen_k=Nk, window=_window(causal, window_size), softmax_scale=softmax_scale,
                  out=out.view(B * Nq, H * d))
    return out


def flash_attn_varlen_func(q, k, v, cu_seqlens_q, cu_seqlens_k, max_seqlen_q, max_seqlen_k, dropout_p=0.0,
                           softmax_scale=None, causal=False, window_size=(-1, -1), softcap=0.0, alibi_slopes=None,
                           deterministic=False, return_attn_probs=False, block_table=None):
    """Packed q [total_q, H, d], k/v [total_k, H, d]; cu_seqlens int32 [batch + 1] on the device."""
    _check_unsupported(dropout_p, softcap, alibi_slopes, return_attn_probs)
    if block_table is not None:
        raise NotImplementedError("paged KV is not supported")
    _dtype_ok(q)
    tq, H, d = q.shape
    tk = k.shape[0]
    if d != 64:
        raise NotImplementedError("head_dim must be 64")
    q, k, v = (t.contiguous() for t in (q, k, v))
    out = torch.empty_like(q)
    ops.attention(q.view(tq, H * d), k.view(tk, H * d), v.view(tk, H * d), heads=H,
                  cu_seqlens_q=cu_seqlens_q.to(torch.int32), cu_seqlens_k=cu_seqlens_k.to(torch.int32),
                  max_seqlen_q=int(max_seqlen_q), max_seqlen_k=int(max_seqlen_k),
                  window=_window(causal, window_size), softmax_scale=softmax_scale, out=out.view(tq, H * d))
    return out


def index_first_axis(x: torch.Tensor, indices: torch.Tensor) -> torch.Tensor:
    """flash_attn.bert_padding.index_first_axis: x[indices] over the flattened first axis."""
    return x.reshape(x.shape[0], -1)[indices].reshape(indices.shape[0], *x.shape[1:])


def pad_input(hidden: torch.Tensor, indices: torch.Tensor, batch: int, seqlen: int) -> torch.Tensor:
    """flash_attn.bert_padding.pad_input: scatter packed rows back to [batch, seqlen, ...] (zeros elsewhere)."""
    out = torch.zeros(batch * seqlen, *hidden.shape[1:], device=hidden.device, dtype=hidden.dtype)
    out[indices] = hidden
    return out.view(batch, seqlen, *hidden.shape[1:])


def unpad_input(hidden: torch.Tensor, attention_mask: torch.Tensor):
    """flash_attn.bert_padding.unpad_input (first four results)."""
    seqlens = attention_mask.sum(dim=-1, dtype=torch.int32)
    indices = torch.nonzero(attention_mask.flatten(), as_tuple=False).flatten()
    cu = torch.nn.functional.pad(torch.cumsum(seqlens, 0, dtype=torch.int32), (1, 0))
    return index_first_axis(hidden, indices), indices, cu, int(seqlens.max().item())


def install(transformer_module=None) -> None:
    """Point the reference's attention globals at this module's kernels.

    transformer_module defaults to the imported stable_audio_3.models.transformer.
    """
    mod = transformer_module or sys.modules.get("stable_audio_3.models.transformer")
    if mod is None:
        raise RuntimeError("import stable_audio_3.models.transformer first (or pass the module)")
    mod.flash_attn_func = flash_attn_func
    mod.flash_attn_varlen_func = flash_attn_varlen_func
    mod.index_first_axis = index_first_axis
    mod.pad_input = pad_input
    mod.unpad_input = unpad_input
