"""Generate golden fixtures by running the REFERENCE modules (Stability-AI/stable-audio-3) on CPU in fp32.

Usage:  python tests/golden/make_golden.py /path/to/stable-audio-3     (or SA3_REFERENCE=/path/to/stable-audio-3)

Weights come from sa3_b200.modules.init_synthetic_ applied to this project's
reference-shaped module tree and are loaded into the reference module with
load_state_dict(strict=True), so the fixtures also prove that the parameter
names and shapes match. flash-attn and flex-attention are disabled so the
reference takes its CPU chunked-halo SDPA path (transformer.py:686-699).

The padding-mask cases ("dit_mask") run the reference through its flash-attn
call sites instead, because that is the path whose semantics the B200 kernels
implement (packed valid tokens, transformer.py:620-651; FF on valid rows,
:500-519). flash-attn has no CPU build, so its four entry points are replaced
by CPU functions computing what they are documented to compute (windowed
softmax attention per packed sequence, gather / scatter of token rows). The
reference casts fp32 q/k/v to fp16 around those calls; the oracle reproduces
that with Cfg.flash_fp16 when it is compared with these fixtures.

Inputs are regenerated from the seeds stored in each fixture; the fixture holds
the reference output (full for small cases, a fixed row subsample otherwise).
DiT fixtures also hold `ref_bf16_rel`: the relative L2 distance between the
reference module run in bf16 and in fp32 on the same case, which measures how
much the CFG/APG combine amplifies low-precision arithmetic there.
"""
import contextlib
import math
import os
import sys

import numpy as np
import torch

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(os.path.dirname(HERE))
sys.path.insert(0, os.path.join(ROOT, "stable-audio-3_b200"))
sys.path.insert(0, ROOT)

from sa3_b200.modules import DiTConfig, DiffusionTransformer, TransformerBlock, init_synthetic_  # noqa: E402
from tests.golden.cases import CASES, block_inputs, dit_inputs, dit_padding_mask, attn_inputs  # noqa: E402


def load_reference(ref_root):
    sys.path.insert(0, ref_root)
    import stable_audio_3.models.transformer as T
    T.flash_attn_func = None
    T.flash_attn_varlen_func = None
    T.flex_attention_available = False
    from stable_audio_3.models import dit as Dm
    return T, Dm


def _band_softmax(q, k, v, wl, wr):
    """[H, n, d] fp32 windowed attention over one sequence (key j visible to query i iff -wl <= j - i <= wr,
    a negative bound meaning unbounded)."""
    n = q.shape[1]
    d = torch.arange(n)[None, :] - torch.arange(n)[:, None]
    ok = torch.ones(n, n, dtype=torch.bool)
    if wl >= 0:
        ok &= d >= -wl
    if wr >= 0:
        ok &= d <= wr
    s = (q @ k.transpose(-1, -2)) / math.sqrt(q.shape[-1])
    return torch.softmax(s.masked_fill(~ok, float("-inf")), -1) @ v


def _cpu_flash_attn_func(q, k, v, causal=False, window_size=(-1, -1), **_):
    """flash_attn_func on CPU: q, k, v [B, N, H, d] (fp16 as the reference passes them); fp32 math, output in
    q's dtype. Only the non-causal, equal-length form the DiT uses."""
    assert not causal
    out = torch.empty_like(q)
    for b in range(q.shape[0]):
        if q.shape[1] == k.shape[1]:
            y = _band_softmax(*(t[b].float().transpose(0, 1) for t in (q, k, v)), *window_size)
        else:
            assert tuple(window_size) in ((-1, -1), [-1, -1])
            qq, kk, vv = (t[b].float().transpose(0, 1) for t in (q, k, v))
            y = torch.softmax((qq @ kk.transpose(-1, -2)) / math.sqrt(q.shape[-1]), -1) @ vv
        out[b] = y.transpose(0, 1).to(q.dtype)
    return out


def _cpu_flash_attn_varlen_func(q, k, v, cu_seqlens_q, cu_seqlens_k, max_seqlen_q, max_seqlen_k, causal=False,
                                window_size=(-1, -1), **_):
    """flash_attn_varlen_func on CPU: packed [total, H, d]; sequence i is rows [cu[i], cu[i+1]) and attends
    within itself (window counted in packed positions)."""
    assert not causal and torch.equal(cu_seqlens_q, cu_seqlens_k)
    out = torch.empty_like(q)
    cu = cu_seqlens_q.tolist()
    for s0, s1 in zip(cu[:-1], cu[1:]):
        y = _band_softmax(*(t[s0:s1].float().transpose(0, 1) for t in (q, k, v)), *window_size)
        out[s0:s1] = y.transpose(0, 1).to(q.dtype)
    return out


def _cpu_index_first_axis(x, indices):
    return x[indices]


def _cpu_pad_input(x, indices, batch, seqlen):
    out = torch.zeros(batch * seqlen, *x.shape[1:], dtype=x.dtype)
    out[indices] = x
    return out.view(batch, seqlen, *x.shape[1:])


def _cpu_unpad_input(*_a, **_k):
    raise NotImplementedError("the DiT packs with precomputed indices; unpad_input is only tested for presence")


@contextlib.contextmanager
def flash_call_sites(T):
    """Route the reference's flash-attn call sites to the CPU functions above for the duration."""
    names = ("flash_attn_func", "flash_attn_varlen_func", "index_first_axis", "pad_input", "unpad_input")
    saved = {n: getattr(T, n, None) for n in names}
    T.flash_attn_func = _cpu_flash_attn_func
    T.flash_attn_varlen_func = _cpu_flash_attn_varlen_func
    T.index_first_axis = _cpu_index_first_axis
    T.pad_input = _cpu_pad_input
    T.unpad_input = _cpu_unpad_input
    try:
        yield
    finally:
        for n, v in saved.items():
            setattr(T, n, v)


def ref_block(T, cfg: DiTConfig):
    return T.TransformerBlock(cfg.embed_dim, dim_heads=cfg.head_dim, global_cond_dim=cfg.embed_dim,
                              norm_type="rms_norm", zero_init_branch_outputs=False,
                              attn_kwargs={"qk_norm": "rms", "qk_norm_eps": cfg.qk_norm_eps,
                                           "differential": cfg.differential},
                              ff_kwargs={"mult": cfg.ff_mult, "no_bias": False})


def ref_dit(Dm, cfg: DiTConfig):
    return Dm.DiffusionTransformer(
        io_channels=cfg.io_channels, embed_dim=cfg.embed_dim, depth=cfg.depth, num_heads=cfg.num_heads,
        cond_token_dim=cfg.cond_token_dim, global_cond_dim=cfg.global_cond_dim, project_cond_tokens=True,
        project_global_cond=True, global_cond_type="adaLN", timestep_features_type="expo",
        timestep_features_dim=cfg.timestep_features_dim, diffusion_objective="rf_denoiser",
        num_memory_tokens=cfg.num_memory_tokens, sliding_window=cfg.sliding_window,
        local_add_cond_dim=cfg.local_add_cond_dim, norm_type="rms_norm", zero_init_branch_outputs=False,
        attn_kwargs={"qk_norm": "rms", "qk_norm_eps": cfg.qk_norm_eps, "differential": cfg.differential},
        ff_kwargs={"mult": cfg.ff_mult, "no_bias": False})


def subsample(y: torch.Tensor, rows_every: int):
    return y[..., ::rows_every, :] if rows_every > 1 else y


def main(ref_root, only=()):
    T, Dm = load_reference(ref_root)
    torch.set_num_threads(max(1, os.cpu_count() or 1))
    for name, case in CASES.items():
        if only and name not in only:
            continue
        cfg = case.get("cfg")
        torch.manual_seed(0)
        extra = {}
        if case["kind"] == "block":
            mine = init_synthetic_(TransformerBlock(cfg, cross_attend=False), seed=case["seed"])
            ref = ref_block(T, cfg)
            ref.load_state_dict(mine.state_dict(), strict=True)
            x, g6 = block_inputs(case)
            freqs = T.RotaryEmbedding(max(cfg.head_dim // 2, 32)).forward_from_seq_len(x.shape[1])
            with torch.inference_mode():
                y = ref(x, global_cond=g6, rotary_pos_emb=freqs,
                        self_attention_flash_sliding_window=cfg.sliding_window)
            out = subsample(y, case.get("rows_every", 1))
        elif case["kind"] == "dit":
            mine = init_synthetic_(DiffusionTransformer(cfg), seed=case["seed"])
            ref = ref_dit(Dm, cfg)
            ref.load_state_dict(mine.state_dict(), strict=True)
            x, t, cond, gemb, loc = dit_inputs(case)
            with torch.inference_mode():
                y = ref(x, t, cross_attn_cond=cond, global_embed=gemb, local_add_cond=loc,
                        cfg_scale=case["cfg_scale"], apg_scale=case["apg_scale"])
                y16 = ref.to(torch.bfloat16)(x, t, cross_attn_cond=cond, global_embed=gemb, local_add_cond=loc,
                                             cfg_scale=case["cfg_scale"], apg_scale=case["apg_scale"])
            extra["ref_bf16_rel"] = np.float64(((y16.float() - y).norm() / y.norm()).item())
            out = y
        elif case["kind"] == "dit_mask":
            mine = init_synthetic_(DiffusionTransformer(cfg), seed=case["seed"])
            ref = ref_dit(Dm, cfg)
            ref.load_state_dict(mine.state_dict(), strict=True)
            x, t, cond, gemb, loc = dit_inputs(case)
            with torch.inference_mode(), flash_call_sites(T):
                y = ref(x, t, cross_attn_cond=cond, global_embed=gemb, local_add_cond=loc,
                        cfg_scale=case["cfg_scale"], apg_scale=case["apg_scale"],
                        padding_mask=dit_padding_mask(case))
                y16 = ref.to(torch.bfloat16)(x, t, cross_attn_cond=cond, global_embed=gemb, local_add_cond=loc,
                                             cfg_scale=case["cfg_scale"], apg_scale=case["apg_scale"],
                                             padding_mask=dit_padding_mask(case))
            extra["ref_bf16_rel"] = np.float64(((y16.float() - y).norm() / y.norm()).item())
            out = y
        elif case["kind"] == "attn":
            q, k, v = attn_inputs(case)
            wl, wr = case["window"]
            with torch.inference_mode():
                y = T._sliding_window_chunked_halo_sdpa(q, k, v, wl, wr)
            out = subsample(y, case.get("rows_every", 1))
        else:
            raise ValueError(case["kind"])
        path = os.path.join(HERE, f"{name}.npz")
        np.savez_compressed(path, out=out.float().numpy(), full_norm=np.float64(y.double().norm()),
                            full_sum=np.float64(y.double().sum()), **extra)
        print(f"{name}: {tuple(y.shape)} -> {path} ({os.path.getsize(path) // 1024} KB)")


if __name__ == "__main__":
    root = sys.argv[1] if len(sys.argv) > 1 else os.environ.get("SA3_REFERENCE")
    if not root:
        sys.exit("usage: make_golden.py /path/to/stable-audio-3   (or set SA3_REFERENCE)")
    only = sys.argv[2:]  # optional case names; default: every case
    main(root, only)
