"""CPU: the oracle's restatement reproduces the reference modules' outputs (fixtures from make_golden.py).

Both sides are fp32 on CPU, so only summation order separates them: the
tolerance is 1e-4 relative L2 (observed ~1e-6).
"""
import os

import numpy as np
import pytest
import torch

from oracle import dit as odit
from oracle import ref as orf
from sa3_b200.modules import DiffusionTransformer, TransformerBlock, init_synthetic_
from tests.golden.cases import CASES, attn_inputs, block_inputs, dit_inputs

HERE = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden")


def _cfg(c):
    return odit.Cfg(io_channels=c.io_channels, embed_dim=c.embed_dim, depth=c.depth, num_heads=c.num_heads,
                    cond_token_dim=c.cond_token_dim, global_cond_dim=c.global_cond_dim,
                    local_add_cond_dim=c.local_add_cond_dim, num_memory_tokens=c.num_memory_tokens,
                    sliding_window=c.sliding_window, differential=c.differential, ff_mult=c.ff_mult,
                    timestep_features_dim=c.timestep_features_dim, norm_eps=c.norm_eps, qk_norm_eps=c.qk_norm_eps)


def oracle_output(name):
    case = CASES[name]
    cfg = case.get("cfg")
    if case["kind"] == "block":
        sd = init_synthetic_(TransformerBlock(cfg, cross_attend=False), seed=case["seed"]).state_dict()
        sd = {"L." + k: v for k, v in sd.items()}
        x, g6 = block_inputs(case)
        y = odit.block_only(sd, "L", _cfg(cfg), x, g6)
    elif case["kind"] == "dit":
        sd = init_synthetic_(DiffusionTransformer(cfg), seed=case["seed"]).state_dict()
        x, t, cond, gemb, loc = dit_inputs(case)
        y = odit.dit_forward(sd, _cfg(cfg), x, t, cond, gemb, loc, case["cfg_scale"], case["apg_scale"])
    else:
        q, k, v = attn_inputs(case)
        y = orf.attention(q, k, v, *case["window"])
    return y


@pytest.mark.parametrize("name", sorted(CASES))
def test_oracle_matches_reference_golden(name):
    gold = np.load(os.path.join(HERE, f"{name}.npz"))
    torch.set_num_threads(max(1, os.cpu_count() or 1))
    with torch.inference_mode():
        y = oracle_output(name)
    every = CASES[name].get("rows_every", 1)
    ys = y[..., ::every, :] if every > 1 else y
    ref = torch.from_numpy(gold["out"])
    assert ys.shape == ref.shape
    err = ((ys.float() - ref).norm() / ref.norm()).item()
    assert err < 1e-4, err
    assert abs(float(y.double().norm()) - float(gold["full_norm"])) / float(gold["full_norm"]) < 1e-4


def test_chunked_halo_equals_masked_attention():
    """The reference's chunked-halo path (transformer.py:143-159) equals its masked SDPA (:118-127)."""
    g = torch.Generator().manual_seed(0)
    q, k, v = (torch.randn(1, 2, 1300, 64, generator=g) for _ in range(3))
    a = orf.chunked_halo_attention(q, k, v, 256, 256)
    b = orf.attention(q, k, v, 256, 256)
    assert ((a - b).norm() / b.norm()).item() < 1e-5
