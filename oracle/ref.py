"""fp32 CPU restatement of the reference DiT denoiser math (oracle; test infrastructure).

Every function cites the reference lines (paths relative to the
Stability-AI/stable-audio-3 project) whose computation it restates.
Tensors are torch.float32 on CPU.
"""
from __future__ import annotations

import math
from typing import Optional

import torch
import torch.nn.functional as F


# --------------------------------------------------------------------------- norms
def rms_norm(x: torch.Tensor, gamma: Optional[torch.Tensor], eps: float) -> torch.Tensor:
    """RMSNorm.forward -> F.rms_norm over the last dim (stable_audio_3/models/transformer.py:392-410)."""
    y = x * torch.rsqrt(x.pow(2).mean(-1, keepdim=True) + eps)
    return y * gamma if gamma is not None else y


def modulate(x: torch.Tensor, scale: torch.Tensor, shift: torch.Tensor) -> torch.Tensor:
    """adaLN modulation x * (1 + scale) + shift (transformer.py:1023-1024, 1044-1045)."""
    return x * (1 + scale) + shift


def gate_residual(h: torch.Tensor, gate: torch.Tensor, residual: torch.Tensor) -> torch.Tensor:
    """x * sigmoid(1 - gate) + residual (transformer.py:1026-1029, 1047-1049)."""
    return h * torch.sigmoid(1 - gate) + residual


# --------------------------------------------------------------------------- rotary
def rotary_inv_freq(dim: int = 32, base: float = 10000.0) -> torch.Tensor:
    """RotaryEmbedding.__init__ inv_freq (transformer.py:252-256)."""
    return 1.0 / (base ** (torch.arange(0, dim, 2).float() / dim))


def rotary_freqs(seq_len: int, dim: int = 32) -> torch.Tensor:
    """RotaryEmbedding.forward_from_seq_len / forward (transformer.py:269-285): [N, dim] = cat(f, f)."""
    t = torch.arange(seq_len, dtype=torch.float32)
    f = torch.einsum("i,j->ij", t, rotary_inv_freq(dim))
    return torch.cat((f, f), dim=-1)


def rotate_half(x: torch.Tensor) -> torch.Tensor:
    """rotate_half (transformer.py:296-299): split the last dim in two halves, (x1, x2) -> (-x2, x1)."""
    x1, x2 = x.chunk(2, dim=-1)
    return torch.cat((-x2, x1), dim=-1)


def apply_rotary(t: torch.Tensor, freqs: torch.Tensor) -> torch.Tensor:
    """apply_rotary_pos_emb (transformer.py:302-322): rotate the first rot_dim dims, pass the rest through."""
    rot = freqs.shape[-1]
    freqs = freqs[-t.shape[-2]:, :]
    tr, tp = t[..., :rot], t[..., rot:]
    tr = tr * freqs.cos() + rotate_half(tr) * freqs.sin()
    return torch.cat((tr, tp), dim=-1)


# --------------------------------------------------------------------------- attention
def band_mask(lq: int, lk: int, wl: int, wr: int) -> torch.Tensor:
    """Boolean visibility of key j to query i: -wl <= j - i - (lk - lq) <= wr; negative = unbounded.

    Matches _sliding_window_additive_mask (transformer.py:118-127) for lq == lk and the
    flash-attn window_size convention used at transformer.py:641-666.
    """
    i = torch.arange(lq)[:, None]
    j = torch.arange(lk)[None, :]
    d = j - i - (lk - lq)
    ok = torch.ones(lq, lk, dtype=torch.bool)
    if wl >= 0:
        ok &= d >= -wl
    if wr >= 0:
        ok &= d <= wr
    return ok


def attention(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor, wl: int = -1, wr: int = -1,
              scale: Optional[float] = None) -> torch.Tensor:
    """softmax(q k^T * scale + band) v for [..., N, d] (masked SDPA path, transformer.py:696-699).

    Rows with no visible key produce zeros (flash-attn convention).
    """
    d = q.shape[-1]
    if (scale is None and wl >= 0 and wr >= 0 and q.shape[-2] == k.shape[-2] and q.shape[-2] > 2048
            and wl + wr < q.shape[-2]):
        # long windowed self-attention: the reference's own chunked-halo formulation (same values,
        # no N x N score matrix)
        return chunked_halo_attention(q, k, v, wl, wr)
    scale = 1.0 / math.sqrt(d) if scale is None else scale
    s = torch.matmul(q, k.transpose(-1, -2)) * scale
    m = band_mask(q.shape[-2], k.shape[-2], wl, wr)
    s = s.masked_fill(~m, float("-inf"))
    p = torch.softmax(s, dim=-1)
    p = torch.nan_to_num(p, nan=0.0)
    return torch.matmul(p, v)


def chunked_halo_attention(q, k, v, wl: int, wr: int, chunk: int = 1024):
    """_sliding_window_chunked_halo_sdpa (transformer.py:143-159): same result as attention()
    computed over 1024-query chunks with a (wl, wr) halo of keys — used for long sequences."""
    n = q.shape[-2]
    outs = []
    for q0 in range(0, n, chunk):
        q1 = min(q0 + chunk, n)
        k0, k1 = max(0, q0 - wl), min(n, q1 + wr)
        qi = torch.arange(q0, q1)[:, None]
        kj = torch.arange(k0, k1)[None, :]
        dd = kj - qi
        ok = (dd >= -wl) & (dd <= wr)
        s = torch.matmul(q[..., q0:q1, :], k[..., k0:k1, :].transpose(-1, -2)) / math.sqrt(q.shape[-1])
        s = s.masked_fill(~ok, float("-inf"))
        outs.append(torch.matmul(torch.softmax(s, -1), v[..., k0:k1, :]))
    return torch.cat(outs, dim=-2)


def differential_attention(q, k, v, q2, k2, wl=-1, wr=-1, scale=None):
    """attn(q, k, v) - attn(q_diff, k_diff, v) (transformer.py:790-795)."""
    return attention(q, k, v, wl, wr, scale) - attention(q2, k2, v, wl, wr, scale)


# --------------------------------------------------------------------------- misc
def silu(x):
    return x * torch.sigmoid(x)


def swiglu(h: torch.Tensor) -> torch.Tensor:
    """GLU.forward with SiLU (transformer.py:421-444): x, gate = chunk(2); x * silu(gate)."""
    x, g = h.chunk(2, dim=-1)
    return x * silu(g)
