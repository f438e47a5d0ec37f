"""Reference-shaped DiT module tree (parameter names identical to the reference).

The classes mirror stable_audio_3/models/dit.py DiffusionTransformer and
stable_audio_3/models/transformer.py ContinuousTransformer / TransformerBlock /
Attention / FeedForward / GLU / RMSNorm / RotaryEmbedding attribute for
attribute, so a reference checkpoint (or a reference module's state_dict())
loads with load_state_dict(strict=True). They hold parameters only; the
forward pass runs on the B200 kernels through sa3_b200.engine.DiTEngine.
"""
from __future__ import annotations

import math
from dataclasses import dataclass, replace
from typing import Optional

import torch
from torch import nn


@dataclass(frozen=True)
class DiTConfig:
    """Shape of a DiffusionTransformer with adaLN global conditioning and an rf_denoiser objective."""

    io_channels: int = 256
    embed_dim: int = 1536
    depth: int = 24
    num_heads: int = 24
    cond_token_dim: int = 768
    global_cond_dim: int = 768
    local_add_cond_dim: int = 257
    num_memory_tokens: int = 64
    sliding_window: Optional[tuple] = (256, 256)
    differential: bool = True
    ff_mult: int = 4
    timestep_features_dim: int = 256
    norm_eps: float = 1e-5
    qk_norm_eps: float = 1e-6

    @property
    def head_dim(self) -> int:
        return self.embed_dim // self.num_heads

    @property
    def ff_inner(self) -> int:
        return self.embed_dim * self.ff_mult


# sa3 "medium": 1536-wide, 24 blocks, 24 heads of 64, differential attention (1453 M params).
MEDIUM = DiTConfig()
# sa3 "small" at 24 blocks: 1024-wide, 16 heads of 64, standard attention.
SMALL = DiTConfig(embed_dim=1024, num_heads=16, differential=False)


class RMSNorm(nn.Module):
    """transformer.py:392-410 (gamma only)."""

    def __init__(self, dim: int, eps: float = 1e-5):
        super().__init__()
        self.gamma = nn.Parameter(torch.ones(dim))
        self.eps = eps


class RotaryEmbedding(nn.Module):
    """transformer.py:239-263: persistent inv_freq buffer."""

    def __init__(self, dim: int, base: float = 10000.0):
        super().__init__()
        self.register_buffer("inv_freq", 1.0 / (base ** (torch.arange(0, dim, 2).float() / dim)))


class Attention(nn.Module):
    """transformer.py:523-570: fused to_qkv (self) or to_q / to_kv (cross), to_out, q_norm / k_norm."""

    def __init__(self, dim: int, dim_heads: int = 64, dim_context: Optional[int] = None, differential: bool = False,
                 qk_norm_eps: float = 1e-6):
        super().__init__()
        self.dim, self.dim_heads, self.differential = dim, dim_heads, differential
        self.num_heads = dim // dim_heads
        if dim_context is not None:
            self.to_q = nn.Linear(dim, dim * (2 if differential else 1), bias=False)
            self.to_kv = nn.Linear(dim_context, dim_context * (3 if differential else 2), bias=False)
        else:
            self.to_qkv = nn.Linear(dim, dim * (5 if differential else 3), bias=False)
        self.to_out = nn.Linear(dim, dim, bias=False)
        self.q_norm = RMSNorm(dim_heads, eps=qk_norm_eps)
        self.k_norm = RMSNorm(dim_heads, eps=qk_norm_eps)


class GLU(nn.Module):
    """transformer.py:421-444 (SiLU gate)."""

    def __init__(self, dim_in: int, dim_out: int):
        super().__init__()
        self.proj = nn.Linear(dim_in, dim_out * 2)


class FeedForward(nn.Module):
    """transformer.py:453-500: ff = Sequential(GLU, Identity, Linear, Identity)."""

    def __init__(self, dim: int, mult: int = 4):
        super().__init__()
        inner = dim * mult
        self.ff = nn.Sequential(GLU(dim, inner), nn.Identity(), nn.Linear(inner, dim), nn.Identity())


class TransformerBlock(nn.Module):
    """transformer.py:859-957 with adaLN (global_cond_dim), cross-attention and local additive conditioning."""

    def __init__(self, cfg: DiTConfig, cross_attend: bool = True):
        super().__init__()
        dim = cfg.embed_dim
        self.pre_norm = RMSNorm(dim, cfg.norm_eps)
        self.self_attn = Attention(dim, cfg.head_dim, differential=cfg.differential, qk_norm_eps=cfg.qk_norm_eps)
        if cross_attend:
            self.cross_attend_norm = RMSNorm(dim, cfg.norm_eps)
            self.cross_attn = Attention(dim, cfg.head_dim, dim_context=dim, differential=cfg.differential,
                                        qk_norm_eps=cfg.qk_norm_eps)
        self.ff_norm = RMSNorm(dim, cfg.norm_eps)
        self.ff = FeedForward(dim, cfg.ff_mult)
        self.to_scale_shift_gate = nn.Parameter(torch.randn(6 * dim) / dim ** 0.5)
        if cfg.local_add_cond_dim:
            self.to_local_embed = nn.Sequential(nn.Linear(cfg.local_add_cond_dim, dim), nn.SiLU(), nn.Linear(dim, dim))


class ContinuousTransformer(nn.Module):
    """transformer.py:1070-1159."""

    def __init__(self, cfg: DiTConfig):
        super().__init__()
        dim = cfg.embed_dim
        self.project_in = nn.Linear(cfg.io_channels, dim, bias=False)
        self.project_out = nn.Linear(dim, cfg.io_channels, bias=False)
        self.rotary_pos_emb = RotaryEmbedding(max(cfg.head_dim // 2, 32))
        if cfg.num_memory_tokens:
            self.memory_tokens = nn.Parameter(torch.randn(cfg.num_memory_tokens, dim))
        self.global_cond_embedder = nn.Sequential(nn.Linear(dim, dim), nn.SiLU(), nn.Linear(dim, dim * 6))
        self.layers = nn.ModuleList([TransformerBlock(cfg, cross_attend=cfg.cond_token_dim > 0)
                                     for _ in range(cfg.depth)])


class DiffusionTransformer(nn.Module):
    """dit.py:13-139 (continuous_transformer, adaLN global cond, expo timestep features, rf_denoiser).

    forward() mirrors DiffusionTransformer.forward (dit.py:345-643) for the arguments the
    sampler passes; it runs on the sm_100a kernels (see sa3_b200.engine). Use quantize()
    to select the FP8 or GPTQ linear path before the first call.
    """

    def __init__(self, cfg: DiTConfig = MEDIUM):
        super().__init__()
        self.cfg = cfg
        D = cfg.embed_dim
        self.to_timestep_embed = nn.Sequential(nn.Linear(cfg.timestep_features_dim, D), nn.SiLU(), nn.Linear(D, D))
        if cfg.cond_token_dim:
            self.to_cond_embed = nn.Sequential(nn.Linear(cfg.cond_token_dim, D, bias=False), nn.SiLU(),
                                               nn.Linear(D, D, bias=False))
        if cfg.global_cond_dim:
            self.to_global_embed = nn.Sequential(nn.Linear(cfg.global_cond_dim, D, bias=False), nn.SiLU(),
                                                 nn.Linear(D, D, bias=False))
        self.transformer = ContinuousTransformer(cfg)
        self.preprocess_conv = nn.Conv1d(cfg.io_channels, cfg.io_channels, 1, bias=False)
        self.postprocess_conv = nn.Conv1d(cfg.io_channels, cfg.io_channels, 1, bias=False)
        self._engine = None
        self._mode = "bf16"
        self._gptq = None
        self._stream = "fp16"
        self._graphs = None

    def quantize(self, mode: str = "fp8", gptq_layers: Optional[dict] = None,
                 stream: str = "fp16") -> "DiffusionTransformer":
        """Select the linear path: 'bf16', 'fp8' (e4m3 weights, per-channel scales, dynamic
        per-tensor activation scale) or 'gptq' (int4 weight-only; gptq_layers maps reference
        linear names to packed (qweight, qzeros, scales, g_idx)), and the precision of the residual
        stream between the blocks: 'fp16' (the precision of the reference's half-precision GPU
        deployment, StableAudioModel.from_pretrained(model_half=True) -> model.to(torch.float16),
        stable_audio_3/loading_utils.py:69-70) or 'fp32'."""
        if mode not in ("bf16", "fp8", "gptq"):
            raise ValueError(mode)
        if stream not in ("fp16", "fp32"):
            raise ValueError(stream)
        self._mode, self._gptq, self._stream, self._engine = mode, gptq_layers, stream, None
        return self

    def enable_cuda_graph(self, enabled: bool = True) -> "DiffusionTransformer":
        """Replay each distinct call signature (shapes, cfg_scale, apg_scale) from a captured CUDA graph.
        The first call per signature runs eagerly twice and captures; later calls copy the inputs
        (host or device) into static buffers and replay."""
        self._graphs = {} if enabled else None
        return self

    def engine(self):
        from .engine import DiTEngine

        if self._engine is None:
            self._engine = DiTEngine(self, mode=self._mode, gptq_layers=self._gptq,
                                     stream_dtype=torch.float16 if self._stream == "fp16" else torch.float32)
        return self._engine

    def forward(self, x, t, cross_attn_cond=None, cross_attn_cond_mask=None, negative_cross_attn_cond=None,
                negative_cross_attn_mask=None, input_concat_cond=None, local_add_cond=None, global_embed=None,
                cfg_scale: float = 1.0, apg_scale: float = 1.0, padding_mask=None, **kwargs):
        cfg_interval = kwargs.pop("cfg_interval", (0, 1))
        unsupported = {k: v for k, v in dict(negative_cross_attn_cond=negative_cross_attn_cond,
                                             input_concat_cond=input_concat_cond, **kwargs).items()
                       if v is not None and v is not False}
        for k in ("cfg_dropout_prob", "scale_phi", "cfg_norm_threshold"):
            if unsupported.get(k, 0) in (0, 0.0):
                unsupported.pop(k, None)
        if unsupported:
            raise NotImplementedError(f"arguments not supported on the B200 path: {sorted(unsupported)}")
        if cfg_scale != 1.0 and tuple(cfg_interval) != (0, 1):
            # CFG applies only while cfg_interval[0] <= sigma[0] <= cfg_interval[1] (dit.py:479), sigma = t
            s0 = float(t.reshape(-1)[0])
            if not (cfg_interval[0] <= s0 <= cfg_interval[1]):
                cfg_scale = 1.0
        if padding_mask is not None:
            padding_mask = padding_mask.bool()
        if self._graphs is not None:
            args = (x, t, cross_attn_cond, global_embed, local_add_cond)
            mkey = None if padding_mask is None else padding_mask.cpu().numpy().tobytes()
            key = (tuple(None if a is None else tuple(a.shape) for a in args), float(cfg_scale), float(apg_scale),
                   mkey)
            g = self._graphs.get(key)
            if g is None:
                g = self._graphs[key] = self.engine().graphed(*args, cfg_scale=cfg_scale, apg_scale=apg_scale,
                                                              padding_mask=padding_mask)
            return g(*args).clone()
        return self.engine().forward(x, t, cross_attn_cond=cross_attn_cond, global_embed=global_embed,
                                     local_add_cond=local_add_cond, cfg_scale=cfg_scale, apg_scale=apg_scale,
                                     padding_mask=padding_mask)


def init_synthetic_(module: nn.Module, seed: int = 0, std: float = 0.02) -> nn.Module:
    """Deterministic synthetic weights (no checkpoints offline): every parameter ~ N(0, std^2),
    RMSNorm gammas ~ 1 + N(0, std^2), to_scale_shift_gate ~ N(0,1)/sqrt(dim) and memory tokens
    ~ N(0,1) as the reference initialises them (transformer.py:942, 1117-1120). Parameters are
    visited in sorted-name order with one CPU generator, so any module with the reference's
    names and shapes gets identical values."""
    g = torch.Generator().manual_seed(seed)
    params = dict(module.named_parameters())
    with torch.no_grad():
        for name in sorted(params):
            p = params[name]
            if name.endswith("gamma"):
                v = 1 + std * torch.randn(p.shape, generator=g)
            elif name.endswith("to_scale_shift_gate"):
                v = torch.randn(p.shape, generator=g) / math.sqrt(p.shape[0] // 6)
            elif name.endswith("memory_tokens"):
                v = torch.randn(p.shape, generator=g)
            else:
                v = std * torch.randn(p.shape, generator=g)
            p.copy_(v.to(p.dtype))
    return module


def with_depth(cfg: DiTConfig, depth: int) -> DiTConfig:
    return replace(cfg, depth=depth)
