"""FP8-e4m3 and GPTQ-int4 definitions of the quantized linears (oracle; test infrastructure).

The reference has no quantized path (every projection in
stable_audio_3/models/transformer.py:547-560, 421-444, 485 is a plain
nn.Linear), so this module DEFINES the quantized computation the CUDA path
must reproduce: the reference F.linear applied to the dequantized weight and,
for FP8, the fake-quantized activation, in fp32.

FP8 (e4m3, OCP "fn" variant, finite max 448):
  weight:     s_w[n] = max(absmax(W[n, :]), 1e-12) / 448 ; Wq = e4m3(W / s_w[n])
  activation: s_x    = max(absmax(X), 1e-12) / 448 (per tensor, dynamic) ; Xq = e4m3(X * r_x),
              r_x    = 448 / max(absmax(X), 1e-12)  (a reciprocal computed once, then one multiply per element)
  y = (Xq * s_x) @ (Wq * s_w)^T + bias
  Rounding is round-to-nearest-even with saturation to +-448.

GPTQ int4 (asymmetric, group size g, act-order), layout declared here:
  qweight int32 [K/8, N]  : word (kk, n) holds q[k, n] for k = 8*kk + j in bits [4j, 4j+4) (LSB first)
  qzeros  int32 [G, N/8]  : word (gi, nn) holds z[gi, n] for n = 8*nn + j in bits [4j, 4j+4) (no +1 offset)
  scales  fp16  [G, N]
  g_idx   int32 [K]       : group of input channel k (arbitrary order = act-order)
  W[n, k] = (q[k, n] - z[g_idx[k], n]) * s[g_idx[k], n]
"""
from __future__ import annotations

import numpy as np
import torch
import torch.nn.functional as F

E4M3_MAX = 448.0


# --------------------------------------------------------------------------- FP8
def e4m3_round(x: torch.Tensor) -> torch.Tensor:
    """Round fp32 to the e4m3 grid (RNE, saturating) and return it as fp32."""
    return x.clamp(-E4M3_MAX, E4M3_MAX).to(torch.float8_e4m3fn).to(torch.float32)


def act_scale(x: torch.Tensor) -> torch.Tensor:
    return torch.clamp(x.abs().max(), min=1e-12) / E4M3_MAX


def act_inv_scale(x: torch.Tensor) -> torch.Tensor:
    return E4M3_MAX / torch.clamp(x.abs().max(), min=1e-12)


def quantize_weight_e4m3(w: torch.Tensor):
    """Per-output-channel scale absmax/448 -> (Wq as float8_e4m3fn, s_w fp32 [N])."""
    w = w.float()
    s = torch.clamp(w.abs().amax(dim=1), min=1e-12) / E4M3_MAX
    wq = (w / s[:, None]).clamp(-E4M3_MAX, E4M3_MAX).to(torch.float8_e4m3fn)
    return wq, s


def fake_quant_act(x: torch.Tensor) -> torch.Tensor:
    return e4m3_round(x * act_inv_scale(x)) * act_scale(x)


def fp8_linear(x: torch.Tensor, wq: torch.Tensor, s_w: torch.Tensor, bias=None) -> torch.Tensor:
    """F.linear(fake_quant(x), dequant(Wq)) + bias, all fp32 (the FP8 linear's definition)."""
    w = wq.float() * s_w[:, None]
    return F.linear(fake_quant_act(x.float()), w, None if bias is None else bias.float())


# --------------------------------------------------------------------------- GPTQ
def gptq_pack(q: np.ndarray, z: np.ndarray, s: np.ndarray, g_idx: np.ndarray):
    """Pack integer weights q [K, N] in 0..15, zeros z [G, N] in 0..15, scales s [G, N], g_idx [K].

    Returns (qweight int32 [K/8, N], qzeros int32 [G, N/8], scales fp16 [G, N], g_idx int32 [K]).
    """
    K, N = q.shape
    assert K % 8 == 0 and N % 8 == 0
    q = q.astype(np.uint32)
    qw = np.zeros((K // 8, N), dtype=np.uint32)
    for j in range(8):
        qw |= q[j::8, :] << np.uint32(4 * j)
    z = z.astype(np.uint32)
    qz = np.zeros((z.shape[0], N // 8), dtype=np.uint32)
    for j in range(8):
        qz |= z[:, j::8] << np.uint32(4 * j)
    return qw.view(np.int32), qz.view(np.int32), s.astype(np.float16), g_idx.astype(np.int32)


def gptq_unpack(qweight: np.ndarray, qzeros: np.ndarray):
    """Inverse of gptq_pack for the integer fields: (q [K, N], z [G, N]) as int32."""
    qw = qweight.view(np.uint32)
    K8, N = qw.shape
    q = np.zeros((K8 * 8, N), dtype=np.int32)
    for j in range(8):
        q[j::8, :] = ((qw >> np.uint32(4 * j)) & np.uint32(0xF)).astype(np.int32)
    qz = qzeros.view(np.uint32)
    G, N8 = qz.shape
    z = np.zeros((G, N8 * 8), dtype=np.int32)
    for j in range(8):
        z[:, j::8] = ((qz >> np.uint32(4 * j)) & np.uint32(0xF)).astype(np.int32)
    return q, z


def gptq_dequant(qweight, qzeros, scales, g_idx) -> np.ndarray:
    """W [N, K] fp32 = (q[k, n] - z[g_idx[k], n]) * s[g_idx[k], n]."""
    q, z = gptq_unpack(np.asarray(qweight), np.asarray(qzeros))
    g = np.asarray(g_idx).astype(np.int64)
    s = np.asarray(scales).astype(np.float32)
    w = (q - z[g, :]).astype(np.float32) * s[g, :]
    return np.ascontiguousarray(w.T)


def gptq_linear(x: torch.Tensor, qweight, qzeros, scales, g_idx, bias=None) -> torch.Tensor:
    """F.linear(x, dequant(W)) + bias in fp32 (the GPTQ linear's definition; activations unquantized)."""
    w = torch.from_numpy(gptq_dequant(qweight, qzeros, scales, g_idx))
    return F.linear(x.float(), w, None if bias is None else bias.float())


def random_gptq_layer(N: int, K: int, group: int = 128, seed: int = 0, act_order: bool = True):
    """Synthetic GPTQ layer with the distributions of the GPTQ benchmark config:
    packed values U{0..15}, zeros U{0..15}, fp16 scales U(0.001, 0.02), g_idx = perm(k) // group."""
    rng = np.random.default_rng(seed)
    G = K // group
    q = rng.integers(0, 16, size=(K, N))
    z = rng.integers(0, 16, size=(G, N))
    s = rng.uniform(0.001, 0.02, size=(G, N))
    if act_order:
        g_idx = rng.permutation(K) // group
    else:
        g_idx = np.arange(K) // group
    return gptq_pack(q, z, s, g_idx)
