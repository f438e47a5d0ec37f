"""Generate golden fixtures by running the REFERENCE modules (Stability-AI/stable-audio-3) on CPU in fp32.

Usage:  python tests/golden/make_golden.py [/path/to/stable-audio-3]

Weights come from sa3_b200.modules.init_synthetic_ applied to this project's
reference-shaped module tree and are loaded into the reference module with
load_state_dict(strict=True), so the fixtures also prove that the parameter
names and shapes match. flash-attn and flex-attention are disabled so the
reference takes its CPU chunked-halo SDPA path (transformer.py:686-699).
Inputs are regenerated from the seeds stored in each fixture; the fixture holds
the reference output (full for small cases, a fixed row subsample otherwise).
"""
import os
import sys

import numpy as np
import torch

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(os.path.dirname(HERE))
sys.path.insert(0, os.path.join(ROOT, "stable-audio-3_b200"))
sys.path.insert(0, ROOT)

from sa3_b200.modules import DiTConfig, DiffusionTransformer, TransformerBlock, init_synthetic_  # noqa: E402
from tests.golden.cases import CASES, block_inputs, dit_inputs, attn_inputs  # noqa: E402


def load_reference(ref_root):
    sys.path.insert(0, ref_root)
    import stable_audio_3.models.transformer as T
    T.flash_attn_func = None
    T.flash_attn_varlen_func = None
    T.flex_attention_available = False
    from stable_audio_3.models import dit as Dm
    return T, Dm


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


def main(ref_root):
    T, Dm = load_reference(ref_root)
    torch.set_num_threads(max(1, os.cpu_count() or 1))
    for name, case in CASES.items():
        cfg = case.get("cfg")
        torch.manual_seed(0)
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
                            full_sum=np.float64(y.double().sum()))
        print(f"{name}: {tuple(y.shape)} -> {path} ({os.path.getsize(path) // 1024} KB)")


if __name__ == "__main__":
    main(sys.argv[1] if len(sys.argv) > 1 else "/root/reference")
