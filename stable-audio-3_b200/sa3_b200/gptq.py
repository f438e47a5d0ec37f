"""GPTQ int4 weight-only linears on the sm_100a kernel.

The reference has no quantized code (every projection is an nn.Linear,
stable_audio_3/models/transformer.py:547-560, 432, 485). GPTQ checkpoints
come as the usual tensors
    qweight int32 [K/8, N] : word (kk, n) holds q[k, n], k = 8*kk + j, in bits [4j, 4j+4) (LSB first)
    qzeros  int32 [G, N/8] : word (g, nn) holds z[g, n], n = 8*nn + j, in bits [4j, 4j+4) (stored as is)
    scales  fp16  [G, N]
    g_idx   int32 [K]      : group of input channel k (act-order: any order, gs channels per group)
with W[n, k] = (q[k, n] - z[g_idx[k], n]) * s[g_idx[k], n].

repack() turns them into the kernel layout of sa3_gptq_gemm: input channels
sorted by group (stable argsort of g_idx, so each 64-wide K tile lies in one
group), 4-bit values packed along K per output row, and fp32 (s, z*s) rows per
group. The GEMM's A operand is x[:, perm] (sa3_permute_cols). inv_perm (the
inverse permutation) lets sa3_gptq_dequant_orig write the dense weight in the
original channel order, which is how large batches run (dequantise once per
call, then the bf16 GEMM on the unpermuted activations).
"""
from __future__ import annotations

from typing import Optional

import numpy as np
import torch
from torch import nn

from . import ops


def unpack(qweight: np.ndarray, qzeros: np.ndarray):
    """(q [K, N], z [G, N]) as int32 from the GPTQ packed fields."""
    qw = np.asarray(qweight).view(np.uint32)
    K8, N = qw.shape
    q = np.empty((K8 * 8, N), dtype=np.int32)
    for j in range(8):
        q[j::8, :] = (qw >> np.uint32(4 * j)) & np.uint32(0xF)
    qz = np.asarray(qzeros).view(np.uint32)
    G, N8 = qz.shape
    z = np.empty((G, N8 * 8), dtype=np.int32)
    for j in range(8):
        z[:, j::8] = (qz >> np.uint32(4 * j)) & np.uint32(0xF)
    return q, z


def repack(qweight, qzeros, scales, g_idx, group_size: int = 128) -> dict:
    """GPTQ tensors -> dict(perm int32 [K], qw int32 [N, K/8], sz fp32 [G, 2N], n, k, group_size)."""
    q, z = unpack(qweight, qzeros)
    K, N = q.shape
    g_idx = np.asarray(g_idx).astype(np.int64)
    perm = np.argsort(g_idx, kind="stable")
    if not np.array_equal(g_idx[perm], np.arange(K) // group_size):
        raise ValueError("g_idx must assign exactly group_size channels to every group")
    qt = np.ascontiguousarray(q[perm, :].T).astype(np.uint32)  # [N, K] in sorted channel order
    words = np.zeros((N, K // 8), dtype=np.uint32)
    for j in range(8):
        words |= qt[:, j::8] << np.uint32(4 * j)
    s = np.asarray(scales).astype(np.float32)
    zs = z.astype(np.float32) * s  # exact: 4-bit integer times an fp16 value
    return dict(perm=torch.from_numpy(perm.astype(np.int32)), inv_perm=torch.from_numpy(np.argsort(perm).astype(np.int32)),
                qw=torch.from_numpy(words.view(np.int32)), sz=torch.from_numpy(np.concatenate([s, zs], axis=1)),
                n=N, k=K, group_size=group_size)


def reorder_rows(packed: dict, idx: torch.Tensor) -> dict:
    """Permute the output rows (n) of a repacked layer, e.g. the SwiGLU [x | gate] interleave."""
    n = packed["n"]
    idx = idx.to(packed["qw"].device)
    sz = packed["sz"]
    return dict(packed, qw=packed["qw"][idx].contiguous(),
                sz=torch.cat([sz[:, :n][:, idx], sz[:, n:][:, idx]], dim=1).contiguous())


def random_layer(n: int, k: int, group_size: int = 128, generator: Optional[torch.Generator] = None,
                 device="cuda") -> dict:
    """Synthetic GPTQ layer directly in kernel layout (GPTQ benchmark distributions): values and zeros
    uniform in 0..15, fp16 scales U(0.001, 0.02), act-order = a random channel permutation."""
    g = generator
    G = k // group_size
    words = torch.randint(-2**31, 2**31 - 1, (n, k // 8), generator=g, dtype=torch.int64).to(torch.int32)
    s = (torch.rand(G, n, generator=g) * 0.019 + 0.001).half().float()
    z = torch.randint(0, 16, (G, n), generator=g).float()
    perm = torch.randperm(k, generator=g).to(torch.int32)
    inv = torch.argsort(perm).to(torch.int32)
    return dict(perm=perm.to(device), inv_perm=inv.to(device), qw=words.to(device),
                sz=torch.cat([s, z * s], dim=1).contiguous().to(device), n=n, k=k, group_size=group_size)


def to_device(packed: dict, device) -> dict:
    return {key: (v.to(device).contiguous() if isinstance(v, torch.Tensor) else v) for key, v in packed.items()}


class QuantLinearGPTQ(nn.Module):
    """GPTQ int4 drop-in for nn.Linear: forward(x[..., in]) -> [..., out] (bf16). Each call gathers x's
    channels into act-order (sa3_permute_cols) and runs the dequantising tcgen05 GEMM."""

    def __init__(self, packed: dict, bias: Optional[torch.Tensor] = None, device="cuda"):
        super().__init__()
        p = to_device(packed, device)
        self.in_features, self.out_features, self.group_size = p["k"], p["n"], p["group_size"]
        self.register_buffer("perm", p["perm"])
        self.register_buffer("qw", p["qw"])
        self.register_buffer("sz", p["sz"])
        self.register_buffer("bias", None if bias is None else bias.detach().float().to(device).contiguous())

    @classmethod
    def from_gptq(cls, qweight, qzeros, scales, g_idx, bias=None, group_size: int = 128, device="cuda"):
        return cls(repack(qweight, qzeros, scales, g_idx, group_size), bias, device)

    def forward(self, x: torch.Tensor) -> torch.Tensor:
        shape = x.shape
        x2 = x.reshape(-1, shape[-1]).to(torch.bfloat16).contiguous()
        xp = ops.permute_cols(x2, self.perm)
        y = ops.gptq_gemm(xp, self.qw, self.sz, self.out_features, group_size=self.group_size, bias=self.bias)
        return y.reshape(*shape[:-1], self.out_features)

    def extra_repr(self) -> str:
        return f"in_features={self.in_features}, out_features={self.out_features}, int4 gs={self.group_size}"


QUANT_SUFFIXES = ("self_attn.to_qkv", "self_attn.to_out", "cross_attn.to_q", "cross_attn.to_kv",
                  "cross_attn.to_out", "ff.ff.0.proj", "ff.ff.2")


def random_model_layers(model: nn.Module, group_size: int = 128, seed: int = 0, device="cuda") -> dict:
    """Synthetic GPTQ layers (random_layer) for every attention / FF linear of a reference-shaped DiT,
    keyed by the reference module names."""
    g = torch.Generator().manual_seed(seed)
    out = {}
    for name, mod in model.named_modules():
        if isinstance(mod, nn.Linear) and name.endswith(QUANT_SUFFIXES):
            out[name] = random_layer(mod.out_features, mod.in_features, group_size, g, device)
    return out
