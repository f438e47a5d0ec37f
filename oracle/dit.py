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
    # Attention.apply_attn casts fp32 q/k/v to fp16 before a flash-attn call and the fp16 output back
    # (transformer.py:632-633, 650, 659-660, 666); True reproduces those two roundings (used to pin the oracle
    # to the reference run through its flash call sites on CPU).
    flash_fp16: bool = False
    # Precision of the model's bf16 deployment: the activations a bf16 model stores between layers are
    # rounded to bf16 (attention q/k/v and outputs, the SwiGLU hidden, the conditioning embeddings, the
    # latent input and the rows handed to project_out; the norm outputs too unless they feed an FP8
    # linear, which quantizes them from fp32). The residual stream stays fp32. With FP8 linears this is the
    # FP8 definition evaluated at the activations a bf16 model actually quantizes: e4m3 rounding is
    # discontinuous, so the fp32-activation definition is itself ~2-3e-2 away from it at these shapes.
    act_bf16: bool = False
    # The residual stream held in fp16 between the layers (the precision of the reference's half-precision GPU
    # deployment, loading_utils.py:69-70): project_in's output and the memory tokens are stored in fp16, and every
    # residual update adds the fp16-rounded branch to the fp16 stream and rounds the sum to fp16.
    stream_f16: bool = False


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


def _fp16(t: torch.Tensor) -> torch.Tensor:
    return t.to(torch.float16).to(torch.float32)


def _b(cfg: Cfg, t: torch.Tensor) -> torch.Tensor:
    """A tensor the bf16 deployment stores in bf16 (Cfg.act_bf16); unchanged otherwise."""
    return t.bfloat16().float() if cfg.act_bf16 else t


def _s(cfg: Cfg, t: torch.Tensor) -> torch.Tensor:
    """A value the residual stream stores (Cfg.stream_f16: rounded to fp16)."""
    return t.half().float() if cfg.stream_f16 else t


def _add(cfg: Cfg, res: torch.Tensor, delta: torch.Tensor) -> torch.Tensor:
    """A residual update of the stream: res + delta, with fp16 rounding of both the branch and the sum when the
    stream is fp16."""
    return _s(cfg, res + _s(cfg, delta))


def _bn(cfg: Cfg, lin: "Linears", t: torch.Tensor) -> torch.Tensor:
    """A norm output: bf16 in the bf16 deployment unless the FP8 linear it feeds quantizes it from fp32."""
    return t if lin.mode == "fp8" else _b(cfg, t)


def mlp3b(cfg: Cfg, lin: "Linears", prefix: str, x: torch.Tensor) -> torch.Tensor:
    """mlp3 with the bf16 deployment's input, hidden and output roundings (Cfg.act_bf16)."""
    return _b(cfg, lin(prefix + ".2", _b(cfg, R.silu(lin(prefix + ".0", _b(cfg, x))))))


def _segment_attn(cfg: Cfg, q, k, v, segs, wl=-1, wr=-1, kv_segs=None):
    """Attention of packed rows [1, H, M, d]: the rows of segment (s0, s1) attend only among themselves
    (or, with kv_segs, to the key rows of the matching key segment), as flash_attn_varlen_func does with
    cu_seqlens (transformer.py:641-647)."""
    out = torch.zeros_like(q)
    for i, (s0, s1) in enumerate(segs):
        k0, k1 = kv_segs[i] if kv_segs is not None else (s0, s1)
        out[:, :, s0:s1] = _attn(cfg, q[:, :, s0:s1], k[:, :, k0:k1], v[:, :, k0:k1], wl, wr)
    return out


def _attn(cfg: Cfg, q, k, v, wl=-1, wr=-1, valid=None):
    """Attention.apply_attn (transformer.py:598-700) for [B, H, N, d]: without `valid`, windowed or full
    attention; with `valid` ([B, N] bool, True = token attends and is attended), the flash-varlen path
    (:620-651): each sequence's valid tokens are packed in order, attend among themselves with the window
    counted in packed positions, and padded rows get a zero output (pad_input)."""
    if cfg.flash_fp16:
        q, k, v = _fp16(q), _fp16(k), _fp16(v)
    if valid is None:
        out = R.attention(q, k, v, wl, wr)
    else:
        out = torch.zeros_like(q)
        for b in range(q.shape[0]):
            idx = valid[b].nonzero().flatten()
            if idx.numel():
                out[b, :, idx] = R.attention(q[b][:, idx], k[b][:, idx], v[b][:, idx], wl, wr)
    return _fp16(out) if cfg.flash_fp16 else out


def self_attention(lin: Linears, sd, p: str, x: torch.Tensor, cfg: Cfg, freqs: torch.Tensor,
                   valid: Optional[torch.Tensor] = None, segs=None) -> torch.Tensor:
    """Attention.forward, fused to_qkv branch (transformer.py:704-820): qk RMSNorm, fp32 RoPE,
    windowed attention (apply_attn, :598-700), differential combine (:790-795), to_out.
    `valid` is the memory-extended padding mask (varlen attention; padded rows attend to nothing);
    `segs` lists the row ranges of packed sequences (x is [1, M, D]; freqs is then per row)."""
    h = cfg.num_heads
    qkv = lin(p + ".to_qkv", x)
    gq, gk = sd[p + ".q_norm.gamma"].float(), sd[p + ".k_norm.gamma"].float()
    wl, wr = cfg.sliding_window if cfg.sliding_window is not None else (-1, -1)

    def attn(q, k, v):
        if segs is not None:
            return _segment_attn(cfg, q, k, v, segs, wl, wr)
        return _attn(cfg, q, k, v, wl, wr, valid)

    if cfg.differential:
        q, k, v, q2, k2 = (_heads(t, h) for t in qkv.chunk(5, dim=-1))
        q, q2 = (_b(cfg, R.apply_rotary(R.rms_norm(t, gq, cfg.qk_norm_eps), freqs)) for t in (q, q2))
        k, k2 = (_b(cfg, R.apply_rotary(R.rms_norm(t, gk, cfg.qk_norm_eps), freqs)) for t in (k, k2))
        v = _b(cfg, v)
        out = _b(cfg, _b(cfg, attn(q, k, v)) - attn(q2, k2, v))
    else:
        q, k, v = (_heads(t, h) for t in qkv.chunk(3, dim=-1))
        q = _b(cfg, R.apply_rotary(R.rms_norm(q, gq, cfg.qk_norm_eps), freqs))
        k = _b(cfg, R.apply_rotary(R.rms_norm(k, gk, cfg.qk_norm_eps), freqs))
        out = _b(cfg, attn(q, k, _b(cfg, v)))
    return lin(p + ".to_out", _merge(out))


def cross_attention(lin: Linears, sd, p: str, x: torch.Tensor, ctx: torch.Tensor, cfg: Cfg, segs=None) -> torch.Tensor:
    """Attention.forward with context (transformer.py:721-745): separate to_q / to_kv, qk RMSNorm,
    no RoPE, full attention, differential combine, to_out. With `segs` (packed rows, x [1, M, D]),
    ctx is [B, Tc, D] and the rows of segment b attend to context b."""
    h = cfg.num_heads
    gq, gk = sd[p + ".q_norm.gamma"].float(), sd[p + ".k_norm.gamma"].float()
    kv_segs = None
    if segs is not None:
        tc = ctx.shape[1]
        kv_segs = [(b * tc, (b + 1) * tc) for b in range(len(segs))]
        ctx = ctx.reshape(1, -1, ctx.shape[-1])

    def attn(q, k, v):
        return _attn(cfg, q, k, v) if segs is None else _segment_attn(cfg, q, k, v, segs, kv_segs=kv_segs)

    if cfg.differential:
        q, q2 = (_heads(t, h) for t in lin(p + ".to_q", x).chunk(2, dim=-1))
        k, k2, v = (_heads(t, h) for t in lin(p + ".to_kv", ctx).chunk(3, dim=-1))
        q, q2 = (_b(cfg, R.rms_norm(t, gq, cfg.qk_norm_eps)) for t in (q, q2))
        k, k2 = (_b(cfg, R.rms_norm(t, gk, cfg.qk_norm_eps)) for t in (k, k2))
        v = _b(cfg, v)
        out = _b(cfg, _b(cfg, attn(q, k, v)) - attn(q2, k2, v))
    else:
        q = _b(cfg, R.rms_norm(_heads(lin(p + ".to_q", x), h), gq, cfg.qk_norm_eps))
        k, v = (_heads(t, h) for t in lin(p + ".to_kv", ctx).chunk(2, dim=-1))
        k = _b(cfg, R.rms_norm(k, gk, cfg.qk_norm_eps))
        out = _b(cfg, attn(q, k, _b(cfg, v)))
    return lin(p + ".to_out", _merge(out))


def block_forward(lin: Linears, sd, p: str, x, cfg: Cfg, global_cond6, freqs, context=None, local_add_cond=None,
                  valid: Optional[torch.Tensor] = None, segs=None, row_batch=None):
    """TransformerBlock.forward, adaLN branch (transformer.py:996-1049).

    global_cond6 is the [B, 6*dim] output of global_cond_embedder. With `valid` (the padding mask extended
    over the memory tokens, transformer.py:1213-1232) self-attention takes the varlen path and the
    feed-forward runs on the valid rows only, packed across the batch; padded rows get a zero FF branch
    (FeedForward.forward with varlen_metadata, transformer.py:500-519). Cross-attention and the local
    conditioning are unmasked, as in the reference.

    Packed sequences (`segs` = row ranges, x [1, M, D], `row_batch` = sequence of each row, local_add_cond
    a list of [L_b, C] per sequence): every row-wise op runs over all rows at once, attention within each
    sequence, the adaLN coefficients per row from its sequence."""
    D = cfg.embed_dim
    ss = sd[p + ".to_scale_shift_gate"].float() + global_cond6
    ss = ss[row_batch][None] if segs is not None else ss[:, None, :]
    sc_s, sh_s, g_s, sc_f, sh_f, g_f = ss.chunk(6, dim=-1)
    res = x
    y = _bn(cfg, lin, R.modulate(R.rms_norm(x, sd[p + ".pre_norm.gamma"].float(), cfg.norm_eps), sc_s, sh_s))
    y = self_attention(lin, sd, p + ".self_attn", y, cfg, freqs, valid, segs)
    x = _add(cfg, res, R.gate_residual(y, g_s, torch.zeros_like(res)))
    if context is not None and (p + ".cross_attn.to_q.weight") in sd:
        c = _bn(cfg, lin, R.rms_norm(x, sd[p + ".cross_attend_norm.gamma"].float(), cfg.norm_eps))
        x = _add(cfg, x, cross_attention(lin, sd, p + ".cross_attn", c, context, cfg, segs))
    if local_add_cond is not None and (p + ".to_local_embed.0.weight") in sd:
        def emb_of(lc, n):
            e = lin(p + ".to_local_embed.2", _b(cfg, R.silu(lin(p + ".to_local_embed.0", _b(cfg, lc)))))
            pad = n - e.shape[-2]   # _left_pad_to_match (transformer.py:77-88)
            return F.pad(e, (0, 0, pad, 0)) if pad > 0 else e[..., -n:, :]
        if segs is None:
            x = _add(cfg, x, emb_of(local_add_cond, x.shape[1]))
        else:
            x = _add(cfg, x, torch.cat([emb_of(lc, s1 - s0) for lc, (s0, s1) in zip(local_add_cond, segs)])[None])
    res = x
    y = _bn(cfg, lin, R.modulate(R.rms_norm(x, sd[p + ".ff_norm.gamma"].float(), cfg.norm_eps), sc_f, sh_f))
    if valid is None:
        y = lin(p + ".ff.ff.2", _b(cfg, R.swiglu(lin(p + ".ff.ff.0.proj", y))))
    else:
        packed = lin(p + ".ff.ff.2", _b(cfg, R.swiglu(lin(p + ".ff.ff.0.proj", y[valid]))))
        y = torch.zeros_like(y)
        y[valid] = packed
    return _add(cfg, res, R.gate_residual(y, g_f, torch.zeros_like(res)))


def dit_inner_forward(lin: Linears, sd, cfg: Cfg, x, t, cross_attn_cond=None, global_embed=None,
                      local_add_cond=None, padding_mask=None):
    """DiffusionTransformer._forward (dit.py:179-309) + ContinuousTransformer.forward (transformer.py:1161-1272).

    padding_mask [B, L] bool (True = valid latent) is extended by always-valid memory tokens
    (transformer.py:1213-1232) and handed to every block."""
    ctx = mlp3b(cfg, lin, "to_cond_embed", cross_attn_cond.float()) if cross_attn_cond is not None else None
    g6 = _global_cond6(lin, cfg, t, global_embed)
    loc = local_add_cond.float().transpose(1, 2) if local_add_cond is not None else None
    wpre = sd["preprocess_conv.weight"].float()[:, :, 0]
    x = _b(cfg, x.float())
    x = torch.einsum("oc,bct->bot", wpre, x) + x
    h = _s(cfg, lin("transformer.project_in", x.transpose(1, 2)))
    B = h.shape[0]
    if cfg.num_memory_tokens:
        h = torch.cat([_s(cfg, sd["transformer.memory_tokens"].float()).expand(B, -1, -1), h], dim=1)
    freqs = R.rotary_freqs(h.shape[1], max(cfg.embed_dim // cfg.num_heads // 2, 32))
    valid = None
    if padding_mask is not None:
        valid = torch.cat([torch.ones(B, cfg.num_memory_tokens, dtype=torch.bool), padding_mask.bool()], dim=1)
    for i in range(cfg.depth):
        h = block_forward(lin, sd, f"transformer.layers.{i}", h, cfg, g6, freqs, ctx, loc, valid)
    h = _b(cfg, h[:, cfg.num_memory_tokens:])
    out = lin("transformer.project_out", h).transpose(1, 2)
    wpost = sd["postprocess_conv.weight"].float()[:, :, 0]
    return torch.einsum("oc,bct->bot", wpost, out) + out


def _global_cond6(lin: Linears, cfg: Cfg, t, global_embed):
    """Timestep embedding + global embedding -> global_cond_embedder: the [B, 6*dim] adaLN conditioning
    (dit.py:197-262, transformer.py:1210-1211)."""
    g = mlp3b(cfg, lin, "to_global_embed", global_embed.float()) if global_embed is not None else None
    temb = mlp3b(cfg, lin, "to_timestep_embed", expo_fourier_features(t, cfg.timestep_features_dim))
    g = temb if g is None else _b(cfg, g + temb)
    return mlp3b(cfg, lin, "transformer.global_cond_embedder", g)


def dit_inner_forward_packed(lin: Linears, sd, cfg: Cfg, xs, t, cross_attn_cond=None, global_embed=None,
                             local_add_conds=None):
    """The network on sequences of different lengths packed back to back (no padding): xs is a list of [C, L_b]
    latents, t [B], cross_attn_cond [B, Tc, cond_dim], global_embed [B, global_dim], local_add_conds a list of
    [local_dim, L_b]. Every row-wise op (the linears included, so an FP8 activation scale spans all packed rows)
    sees the packed [1, sum(L_b + memory), D] rows; attention stays within each sequence, RoPE positions restart
    per sequence. This is flash_attn_varlen_func's packing (transformer.py:620-651) applied to whole prompts.
    Returns a list of [C, L_b]."""
    nm = cfg.num_memory_tokens
    B = len(xs)
    ctx = mlp3b(cfg, lin, "to_cond_embed", cross_attn_cond.float()) if cross_attn_cond is not None else None
    g6 = _global_cond6(lin, cfg, t, global_embed)
    wpre = sd["preprocess_conv.weight"].float()[:, :, 0]
    rows, segs, pos, rb, r0 = [], [], [], [], 0
    for b, x in enumerate(xs):
        x = _b(cfg, x.float())
        hb = _s(cfg, lin("transformer.project_in", (wpre @ x + x).transpose(0, 1)))
        if nm:
            hb = torch.cat([_s(cfg, sd["transformer.memory_tokens"].float()).reshape(nm, -1), hb])
        rows.append(hb)
        segs.append((r0, r0 + hb.shape[0]))
        pos.append(torch.arange(hb.shape[0]))
        rb.append(torch.full((hb.shape[0],), b, dtype=torch.long))
        r0 += hb.shape[0]
    h = torch.cat(rows)[None]
    row_batch = torch.cat(rb)
    rot = max(cfg.embed_dim // cfg.num_heads // 2, 32)
    freqs = R.rotary_freqs(max(s1 - s0 for s0, s1 in segs), rot)[torch.cat(pos)]
    locs = None if local_add_conds is None else [lc.float().transpose(0, 1) for lc in local_add_conds]
    for i in range(cfg.depth):
        h = block_forward(lin, sd, f"transformer.layers.{i}", h, cfg, g6, freqs, ctx, locs, segs=segs,
                          row_batch=row_batch)
    wpost = sd["postprocess_conv.weight"].float()[:, :, 0]
    outs = []
    for s0, s1 in segs:
        o = lin("transformer.project_out", _b(cfg, h[0, s0 + nm:s1])).transpose(0, 1)
        outs.append(wpost @ o + o)
    return outs


def apg_project(v0, v1, padding_mask=None):
    """DiffusionTransformer.apg_project (dit.py:311-343), fp32. With padding_mask [B, T] (True = valid) the
    direction is v1 restricted to valid positions, normalised with a 1e-8 floor, and the orthogonal part is
    zeroed on padded positions."""
    if padding_mask is None:
        v1n = F.normalize(v1, dim=[-1, -2])
        par = (v0 * v1n).sum(dim=[-1, -2], keepdim=True) * v1n
        return par, v0 - par
    mask = padding_mask[:, None, :].float()
    v1m = v1 * mask
    v1n = v1m / v1m.norm(dim=[-1, -2], keepdim=True).clamp(min=1e-8)
    proj = (v0 * v1n).sum(dim=[-1, -2], keepdim=True) * v1n
    return (v0 * mask * v1n).sum(dim=[-1, -2], keepdim=True) * v1n, (v0 - proj) * mask


def dit_forward(sd, cfg: Cfg, x, t, cross_attn_cond=None, global_embed=None, local_add_cond=None,
                cfg_scale: float = 1.0, apg_scale: float = 1.0, mode: str = "fp32", gptq: Optional[dict] = None,
                padding_mask=None):
    """DiffusionTransformer.forward for the rf_denoiser objective (dit.py:345-643): CFG batch doubling
    with a zero cross-attention cond for the unconditional half (both halves share the padding mask,
    dit.py:549-550), then the APG-projected combine."""
    lin = Linears(sd, mode, gptq)
    t = t.float()
    if cfg_scale == 1.0 or cross_attn_cond is None:
        return dit_inner_forward(lin, sd, cfg, x, t, cross_attn_cond, global_embed, local_add_cond, padding_mask)
    bx = torch.cat([x, x])
    bt = torch.cat([t, t])
    bc = torch.cat([cross_attn_cond, torch.zeros_like(cross_attn_cond)])
    bg = torch.cat([global_embed, global_embed]) if global_embed is not None else None
    bl = torch.cat([local_add_cond, local_add_cond]) if local_add_cond is not None else None
    bm = torch.cat([padding_mask, padding_mask]) if padding_mask is not None else None
    out = dit_inner_forward(lin, sd, cfg, bx, bt, bc, bg, bl, bm)
    return cfg_combine(x, t, out, cfg_scale, apg_scale, padding_mask)


def cfg_batch(x, t, cross_attn_cond, global_embed=None, local_add_cond=None):
    """CFG batch doubling of DiffusionTransformer.forward (dit.py:479-568): cond half, then an
    unconditional half with a zero cross-attention cond."""
    return (torch.cat([x, x]), torch.cat([t, t]), torch.cat([cross_attn_cond, torch.zeros_like(cross_attn_cond)]),
            None if global_embed is None else torch.cat([global_embed, global_embed]),
            None if local_add_cond is None else torch.cat([local_add_cond, local_add_cond]))


def cfg_combine(x, t, out, cfg_scale: float, apg_scale: float, padding_mask=None):
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
        par, orth = apg_project(diff, cond_den, padding_mask)
        cfg_diff = orth if apg_scale == 1.0 else apg_scale * orth + (1 - apg_scale) * diff
    cfg_den = cond_den + (cfg_scale - 1) * cfg_diff
    return (x - cfg_den) / sigma


def block_only(sd, prefix: str, cfg: Cfg, x, global_cond6, mode="fp32"):
    """One TransformerBlock with global_cond fed directly as [B, 6*dim] and RoPE over x's length."""
    lin = Linears(sd, mode)
    freqs = R.rotary_freqs(x.shape[1], max(cfg.embed_dim // cfg.num_heads // 2, 32))
    return block_forward(lin, sd, prefix, x.float(), cfg, global_cond6.float(), freqs)
