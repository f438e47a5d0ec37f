"""fp32 CPU restatement of the reference DiT denoiser forward (oracle; test infrastructure).

Driven by a state dict with the reference's own key names
(stable_audio_3/models/dit.py DiffusionTransformer + transformer.py
ContinuousTransformer / TransformerBlock / Attention / FeedForward), so the
same weights can be loaded into the reference module, this oracle, and the
CUDA path. Linears listed in `quant` are replaced by the FP8 or GPTQ
definitions of oracle.quant (the reference has no quantized path).
"""
from __future__ import annotations

import math
from dataclasses import dataclass, field
from typing import Dict, Optional

import torch
import torch.nn.functional as F

from . import quant as oq
from . import ref as R


@dataclass
class Cfg:
    io_channels: int = 256
    embed_dim: int = 1536
    depth: int = 24
    num_heads: int = 24
    cond_token_dim: int = 768
    global_cond_dim: int = 768
    local_add_cond_dim: int = 257
    num_memory_tokens: int = 64
    sliding_window: tuple = (256, 256)
    differential: bool = True
    ff_mult: int = 4
    timestep_features_dim: int = 256
    norm_eps: float = 1e-5
    qk_norm_eps: float = 1e-6


# Linears the quantized variants replace (suffixes of the reference key names).
QUANT_LINEARS = ("self_attn.to_qkv", "self_attn.to_out", "cross_attn.to_q", "cross_attn.to_kv",
                 "cross_attn.to_out", "ff.ff.0.proj", "ff.ff.2")


class Linears:
    """Linear dispatcher: plain fp32 F.linear, or the FP8 / GPTQ definition for QUANT_LINEARS."""

    def __init__(self, sd: Dict[str, torch.Tensor], mode: str = "fp32", gptq: Optional[dict] = None):
        self.sd = sd
        self.mode = mode
        self.gptq = gptq or {}
        self._fp8 = {}

    def __call__(self, name: str, x: torch.Tensor) -> torch.Tensor:
        w = self.sd[name + ".weight"]
        b = self.sd.get(name + ".bias")
        quantized = any(name.endswith(s) for s in QUANT_LINEARS)
        if quantized and self.mode == "fp8":
            if name not in self._fp8:
                self._fp8[name] = oq.quantize_weight_e4m3(w)
            wq, sw = self._fp8[name]
            return oq.fp8_linear(x, wq, sw, b)
        if quantized and self.mode == "gptq":
            qw, qz, sc, gi = self.gptq[name]
            return oq.gptq_linear(x, qw, qz, sc, gi, b)
        return F.linear(x, w.float(), None if b is None else b.float())


def expo_fourier_features(t: torch.Tensor, dim: int = 256, min_freq: float = 0.5, max_freq: float = 10000.0):
    """ExpoFourierFeatures.forward (stable_audio_3/models/blocks.py:50-82), fp32."""
    t = t.float()[:, None]
    half = dim // 2
    ramp = torch.linspace(0, 1, half, dtype=torch.float32)
    freqs = torch.exp(ramp * (math.log(max_freq) - math.log(min_freq)) + math.log(min_freq))
    args = t * freqs * 2 * math.pi
    return torch.cat([torch.cos(args), torch.sin(args)], dim=-1)


def mlp3(lin: Linears, prefix: str, x: torch.Tensor) -> torch.Tensor:
    """nn.Sequential(Linear, SiLU, Linear) as used by to_timestep_embed / to_cond_embed /
    to_global_embed / global_cond_embedder / to_local_embed (dit.py:57-93, transformer.py:944-957, 1131-1136)."""
    return lin(prefix + ".2", R.silu(lin(prefix + ".0", x)))


def _heads(t: torch.Tensor, h: int) -> torch.Tensor:
    b, n, _ = t.shape
    return t.view(b, n, h, -1).permute(0, 2, 1, 3)


def _merge(t: torch.Tensor) -> torch.Tensor:
    b, h, n, d = t.shape
    return t.permute(0, 2, 1, 3).reshape(b, n, h * d)


def self_attention(lin: Linears, sd, p: str, x: torch.Tensor, cfg: Cfg, freqs: torch.Tensor) -> torch.Tensor:
    """Attention.forward, fused to_qkv branch (transformer.py:704-820): qk RMSNorm, fp32 RoPE,
    windowed attention (apply_attn, :598-700), differential combine (:790-795), to_out."""
    h = cfg.num_heads
    qkv = lin(p + ".to_qkv", x)
    gq, gk = sd[p + ".q_norm.gamma"].float(), sd[p + ".k_norm.gamma"].float()
    wl, wr = cfg.sliding_window if cfg.sliding_window is not None else (-1, -1)
    if cfg.differential:
        q, k, v, q2, k2 = (_heads(t, h) for t in qkv.chunk(5, dim=-1))
        q, q2 = (R.apply_rotary(R.rms_norm(t, gq, cfg.qk_norm_eps), freqs) for t in (q, q2))
        k, k2 = (R.apply_rotary(R.rms_norm(t, gk, cfg.qk_norm_eps), freqs) for t in (k, k2))
        out = R.differential_attention(q, k, v, q2, k2, wl, wr)
    else:
        q, k, v = (_heads(t, h) for t in qkv.chunk(3, dim=-1))
        q = R.apply_rotary(R.rms_norm(q, gq, cfg.qk_norm_eps), freqs)
        k = R.apply_rotary(R.rms_norm(k, gk, cfg.qk_norm_eps), freqs)
        out = R.attention(q, k, v, wl, wr)
    return lin(p + ".to_out", _merge(out))


def cross_attention(lin: Linears, sd, p: str, x: torch.Tensor, ctx: torch.Tensor, cfg: Cfg) -> torch.Tensor:
    """Attention.forward with context (transformer.py:721-745): separate to_q / to_kv, qk RMSNorm,
    no RoPE, full attention, differential combine, to_out."""
    h = cfg.num_heads
    gq, gk = sd[p + ".q_norm.gamma"].float(), sd[p + ".k_norm.gamma"].float()
    if cfg.differential:
        q, q2 = (_heads(t, h) for t in lin(p + ".to_q", x).chunk(2, dim=-1))
        k, k2, v = (_heads(t, h) for t in lin(p + ".to_kv", ctx).chunk(3, dim=-1))
        q, q2 = (R.rms_norm(t, gq, cfg.qk_norm_eps) for t in (q, q2))
        k, k2 = (R.rms_norm(t, gk, cfg.qk_norm_eps) for t in (k, k2))
        out = R.differential_attention(q, k, v, q2, k2)
    else:
        q = R.rms_norm(_heads(lin(p + ".to_q", x), h), gq, cfg.qk_norm_eps)
        k, v = (_heads(t, h) for t in lin(p + ".to_kv", ctx).chunk(2, dim=-1))
        k = R.rms_norm(k, gk, cfg.qk_norm_eps)
        out = R.attention(q, k, v)
    return lin(p + ".to_out", _merge(out))


def block_forward(lin: Linears, sd, p: str, x, cfg: Cfg, global_cond6, freqs, context=None, local_add_cond=None):
    """TransformerBlock.forward, adaLN branch (transformer.py:996-1049).

    global_cond6 is the [B, 6*dim] output of global_cond_embedder."""
    D = cfg.embed_dim
    ss = sd[p + ".to_scale_shift_gate"].float() + global_cond6
    sc_s, sh_s, g_s, sc_f, sh_f, g_f = ss[:, None, :].chunk(6, dim=-1)
    res = x
    y = R.modulate(R.rms_norm(x, sd[p + ".pre_norm.gamma"].float(), cfg.norm_eps), sc_s, sh_s)
    y = self_attention(lin, sd, p + ".self_attn", y, cfg, freqs)
    x = R.gate_residual(y, g_s, res)
    if context is not None and (p + ".cross_attn.to_q.weight") in sd:
        c = R.rms_norm(x, sd[p + ".cross_attend_norm.gamma"].float(), cfg.norm_eps)
        x = x + cross_attention(lin, sd, p + ".cross_attn", c, context, cfg)
    if local_add_cond is not None and (p + ".to_local_embed.0.weight") in sd:
        emb = mlp3(lin, p + ".to_local_embed", local_add_cond)
        pad = x.shape[1] - emb.shape[1]   # _left_pad_to_match (transformer.py:77-88)
        emb = F.pad(emb, (0, 0, pad, 0)) if pad > 0 else emb[:, -x.shape[1]:]
        x = x + emb
    res = x
    y = R.modulate(R.rms_norm(x, sd[p + ".ff_norm.gamma"].float(), cfg.norm_eps), sc_f, sh_f)
    y = lin(p + ".ff.ff.2", R.swiglu(lin(p + ".ff.ff.0.proj", y)))
    return R.gate_residual(y, g_f, res)


def dit_inner_forward(lin: Linears, sd, cfg: Cfg, x, t, cross_attn_cond=None, global_embed=None,
                      local_add_cond=None):
    """DiffusionTransformer._forward (dit.py:179-309) + ContinuousTransformer.forward (transformer.py:1161-1272)."""
    ctx = mlp3(lin, "to_cond_embed", cross_attn_cond.float()) if cross_attn_cond is not None else None
    g = mlp3(lin, "to_global_embed", global_embed.float()) if global_embed is not None else None
    temb = mlp3(lin, "to_timestep_embed", expo_fourier_features(t, cfg.timestep_features_dim))
    g = temb if g is None else g + temb
    loc = local_add_cond.float().transpose(1, 2) if local_add_cond is not None else None
    wpre = sd["preprocess_conv.weight"].float()[:, :, 0]
    x = x.float()
    x = torch.einsum("oc,bct->bot", wpre, x) + x
    h = lin("transformer.project_in", x.transpose(1, 2))
    B = h.shape[0]
    if cfg.num_memory_tokens:
        h = torch.cat([sd["transformer.memory_tokens"].float().expand(B, -1, -1), h], dim=1)
    freqs = R.rotary_freqs(h.shape[1], max(cfg.embed_dim // cfg.num_heads // 2, 32))
    g6 = mlp3(lin, "transformer.global_cond_embedder", g)
    for i in range(cfg.depth):
        h = block_forward(lin, sd, f"transformer.layers.{i}", h, cfg, g6, freqs, ctx, loc)
    h = h[:, cfg.num_memory_tokens:]
    out = lin("transformer.project_out", h).transpose(1, 2)
    wpost = sd["postprocess_conv.weight"].float()[:, :, 0]
    return torch.einsum("oc,bct->bot", wpost, out) + out


def apg_project(v0, v1):
    """DiffusionTransformer.apg_project without padding mask (dit.py:311-343), fp32."""
    v1n = F.normalize(v1, dim=[-1, -2])
    par = (v0 * v1n).sum(dim=[-1, -2], keepdim=True) * v1n
    return par, v0 - par


def dit_forward(sd, cfg: Cfg, x, t, cross_attn_cond=None, global_embed=None, local_add_cond=None,
                cfg_scale: float = 1.0, apg_scale: float = 1.0, mode: str = "fp32", gptq: Optional[dict] = None):
    """DiffusionTransformer.forward for the rf_denoiser objective (dit.py:345-643): CFG batch doubling
    with a zero cross-attention cond for the unconditional half, then the APG-projected combine."""
    lin = Linears(sd, mode, gptq)
    t = t.float()
    if cfg_scale == 1.0 or cross_attn_cond is None:
        return dit_inner_forward(lin, sd, cfg, x, t, cross_attn_cond, global_embed, local_add_cond)
    bx = torch.cat([x, x])
    bt = torch.cat([t, t])
    bc = torch.cat([cross_attn_cond, torch.zeros_like(cross_attn_cond)])
    bg = torch.cat([global_embed, global_embed]) if global_embed is not None else None
    bl = torch.cat([local_add_cond, local_add_cond]) if local_add_cond is not None else None
    out = dit_inner_forward(lin, sd, cfg, bx, bt, bc, bg, bl)
    return cfg_combine(x, t, out, cfg_scale, apg_scale)


def cfg_batch(x, t, cross_attn_cond, global_embed=None, local_add_cond=None):
    """CFG batch doubling of DiffusionTransformer.forward (dit.py:479-568): cond half, then an
    unconditional half with a zero cross-attention cond."""
    return (torch.cat([x, x]), torch.cat([t, t]), torch.cat([cross_attn_cond, torch.zeros_like(cross_attn_cond)]),
            None if global_embed is None else torch.cat([global_embed, global_embed]),
            None if local_add_cond is None else torch.cat([local_add_cond, local_add_cond]))


def cfg_combine(x, t, out, cfg_scale: float, apg_scale: float):
    """rf_denoiser CFG + APG combine of the batched network output (dit.py:571-625), fp32."""
    cond_out, uncond_out = out.float().chunk(2)
    sigma = t.float()[:, None, None]
    x = x.float()
    cond_den = x - cond_out * sigma
    uncond_den = x - uncond_out * sigma
    diff = cond_den - uncond_den
    if apg_scale == 0.0:
        cfg_diff = diff
    else:
        par, orth = apg_project(diff, cond_den)
        cfg_diff = orth if apg_scale == 1.0 else apg_scale * orth + (1 - apg_scale) * diff
    cfg_den = cond_den + (cfg_scale - 1) * cfg_diff
    return (x - cfg_den) / sigma


def block_only(sd, prefix: str, cfg: Cfg, x, global_cond6, mode="fp32"):
    """One TransformerBlock with global_cond fed directly as [B, 6*dim] and RoPE over x's length."""
    lin = Linears(sd, mode)
    freqs = R.rotary_freqs(x.shape[1], max(cfg.embed_dim // cfg.num_heads // 2, 32))
    return block_forward(lin, sd, prefix, x.float(), cfg, global_cond6.float(), freqs)
