"""Golden cases: shapes, seeds and input generators shared by make_golden.py and the tests.

Inputs are regenerated from seeds (activations ~N(0,1)); only reference
outputs are stored in the .npz fixtures.
"""
from dataclasses import replace

import torch

from sa3_b200.modules import DiTConfig

_small = DiTConfig(embed_dim=256, depth=2, num_heads=4, sliding_window=(64, 64), differential=True)

CASES = {
    # one block at the CPU block-benchmark shape: D=1024, 16 heads x 64, L=646, window (256, 256)
    "block_d1024_l646": dict(kind="block", seed=1, B=1, L=646,
                             cfg=DiTConfig(embed_dim=1024, num_heads=16, depth=1, differential=False,
                                           local_add_cond_dim=0, cond_token_dim=0), rows_every=8),
    # small blocks, standard and differential attention, narrow window (several key tiles masked)
    "block_d256_diff": dict(kind="block", seed=2, B=2, L=300, rows_every=3,
                            cfg=replace(_small, depth=1, local_add_cond_dim=0, cond_token_dim=0)),
    "block_d256_std": dict(kind="block", seed=3, B=1, L=257,
                           cfg=replace(_small, depth=1, differential=False, local_add_cond_dim=0,
                                       cond_token_dim=0, sliding_window=(17, 17))),
    # full denoiser (2 blocks), differential, memory tokens, cross-attention, local cond, CFG + APG
    "dit_small_cfg": dict(kind="dit", seed=4, B=1, L=200, Tc=16, cfg=_small, cfg_scale=5.0, apg_scale=1.0),
    # standard attention, no CFG
    "dit_small_nocfg": dict(kind="dit", seed=5, B=2, L=150, Tc=12, cfg=replace(_small, differential=False),
                            cfg_scale=1.0, apg_scale=1.0),
    # the reference's chunked-halo SDPA over several 1024-query chunks
    "attn_halo_n2500": dict(kind="attn", seed=6, B=1, H=2, N=2500, window=(256, 256), rows_every=5),
    # padding_mask as StableAudioModel.generate passes it (valid latent prefix per prompt), through the
    # reference's flash-varlen call sites: two prompts (one padded, one full), CFG + full APG
    "dit_small_cfg_mask": dict(kind="dit_mask", seed=7, B=2, L=200, Tc=16, cfg=_small, cfg_scale=5.0,
                               apg_scale=1.0, valid=[137, 200]),
    # standard attention, blended APG (the unmasked diff enters the combine), one prompt padded to 90 of 160
    "dit_small_std_mask": dict(kind="dit_mask", seed=8, B=1, L=160, Tc=12, cfg=replace(_small, differential=False),
                               cfg_scale=6.0, apg_scale=0.5, valid=[90]),
}


def _g(seed):
    return torch.Generator().manual_seed(1000 + seed)


def block_inputs(case):
    cfg = case["cfg"]
    g = _g(case["seed"])
    x = torch.randn(case["B"], case["L"], cfg.embed_dim, generator=g)
    g6 = torch.randn(case["B"], 6 * cfg.embed_dim, generator=g) * 0.5
    return x, g6


def dit_inputs(case):
    cfg = case["cfg"]
    g = _g(case["seed"])
    B, L, Tc = case["B"], case["L"], case["Tc"]
    x = torch.randn(B, cfg.io_channels, L, generator=g)
    t = torch.rand(B, generator=g) * 0.8 + 0.1
    cond = torch.randn(B, Tc, cfg.cond_token_dim, generator=g)
    gemb = torch.randn(B, cfg.global_cond_dim, generator=g)
    loc = torch.randn(B, cfg.local_add_cond_dim, L, generator=g) * 0.5
    return x, t, cond, gemb, loc


def dit_padding_mask(case):
    """[B, L] bool, True on each prompt's first `valid` latents (create_padding_mask_from_lengths,
    stable_audio_3/data/utils.py:195-212)."""
    return torch.arange(case["L"])[None, :] < torch.tensor(case["valid"])[:, None]


def attn_inputs(case):
    g = _g(case["seed"])
    shape = (case["B"], case["H"], case["N"], 64)
    return (torch.randn(shape, generator=g), torch.randn(shape, generator=g), torch.randn(shape, generator=g))
