"""padding_mask on a B200: the DiT called the way the reference sampler calls it under generate().

StableAudioModel.generate passes mask_padding_attention=True (stable_audio_3/model.py:327), so sample_diffusion
builds a valid-prefix mask per prompt (inference/sampling.py:444-452) and hands it, with cfg_scale / apg_scale,
to every model call (:468-475, :344). The reference then runs its flash-varlen path: memory tokens always valid
(transformer.py:1213-1232), attention among valid tokens only with zero output on padded rows (:620-651), the
feed-forward on valid rows only (:500-519), and an APG projection restricted to valid positions (dit.py:311-343).

Bounds: network velocity for both CFG halves <= 2e-2 relative L2 (bf16 vs the fp32 oracle; FP8 vs the FP8
definition at the bf16 deployment's activations); full CFG velocity <= 2e-2 for bf16; against the reference's own
output (golden fixture, weights rounded to bf16 on our side) <= 2e-2.
"""
import os
from dataclasses import replace

import numpy as np
import pytest
import torch

from oracle import dit as odit
from sa3_b200.modules import DiffusionTransformer, init_synthetic_
from tests.golden.cases import CASES, dit_inputs, dit_padding_mask
from tests.test_oracle_golden import _cfg

pytestmark = pytest.mark.gpu
HERE = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden")

# the model kwargs sample_diffusion builds under generate() (sampling.py:468-475 after DiTWrapper, diffusion.py:236-253)
SAMPLER_KW = dict(cross_attn_cond_mask=None, cfg_dropout_prob=0.0, scale_phi=0.0, cfg_interval=(0, 1))


def rel_l2(a, b):
    a, b = a.float().cpu(), b.float().cpu()
    return ((a - b).norm() / b.norm()).item()


def _model(case, mode):
    m = init_synthetic_(DiffusionTransformer(case["cfg"]), seed=case["seed"])
    if mode == "bf16":
        with torch.no_grad():
            for p in m.parameters():
                p.copy_(p.bfloat16().float())
    return m.quantize(mode)


@pytest.mark.parametrize("name", ["dit_small_cfg_mask", "dit_small_std_mask"])
@pytest.mark.parametrize("mode", ["bf16", "fp8"])
def test_masked_network_velocity_matches_oracle(cuda, name, mode):
    """Both CFG halves' network output with the mask (valid and padded rows) vs the oracle: <= 2e-2."""
    case = CASES[name]
    m = _model(case, mode)
    x, t, cond, gemb, loc = dit_inputs(case)
    pm = dit_padding_mask(case)
    bx, bt, bc, bg, bl = odit.cfg_batch(x, t, cond, gemb, loc)
    bm = torch.cat([pm, pm])
    with torch.inference_mode():
        sd = m.state_dict()
        ref = odit.dit_inner_forward(odit.Linears(sd, "fp8" if mode == "fp8" else "fp32"), sd,
                                     replace(_cfg(case["cfg"]), act_bf16=(mode == "fp8")), bx, bt, bc, bg, bl,
                                     padding_mask=bm)
        out = m.engine().inner(*(a.to(cuda) for a in (bx, bt, bc, bg, bl)), padding_mask=bm.to(cuda))
    torch.cuda.synchronize()
    err = rel_l2(out, ref)
    valid = bm[:, None, :].expand_as(ref)
    err_pad = rel_l2(out.cpu()[~valid], ref[~valid])
    print(f"{name} {mode}: network velocity rel L2 {err:.2e} (padded positions {err_pad:.2e})")
    assert err < 2e-2
    assert err_pad < 2e-2


@pytest.mark.parametrize("name", ["dit_small_cfg_mask", "dit_small_std_mask"])
def test_masked_cfg_velocity_bf16(cuda, name):
    """The full CFG/APG velocity through DiffusionTransformer.forward with the sampler's kwargs vs the oracle
    (fp32) and vs the reference's own output (golden): <= 2e-2 each."""
    case = CASES[name]
    m = _model(case, "bf16")
    x, t, cond, gemb, loc = dit_inputs(case)
    pm = dit_padding_mask(case)
    with torch.inference_mode():
        ref = odit.dit_forward(m.state_dict(), _cfg(case["cfg"]), x, t, cond, gemb, loc, case["cfg_scale"],
                               case["apg_scale"], padding_mask=pm)
        out = m(x.to(cuda), t.to(cuda), cross_attn_cond=cond.to(cuda), global_embed=gemb.to(cuda),
                local_add_cond=loc.to(cuda), cfg_scale=case["cfg_scale"], apg_scale=case["apg_scale"],
                padding_mask=pm.to(cuda), **SAMPLER_KW)
    err = rel_l2(out, ref)
    gold = torch.from_numpy(np.load(os.path.join(HERE, f"{name}.npz"))["out"])
    err_gold = rel_l2(out, gold)
    print(f"{name}: bf16 CFG velocity rel L2 {err:.2e} vs oracle, {err_gold:.2e} vs reference golden")
    assert err < 2e-2
    assert err_gold < 2e-2


def test_masked_equals_truncated_prompt(cuda):
    """A prompt whose mask is a valid prefix gets, on its valid latents, the network output of the same prompt
    truncated to that length (bf16 kernels on both sides; only row order and the FF batch differ)."""
    case = CASES["dit_small_cfg_mask"]
    m = _model(case, "bf16")
    x, t, cond, gemb, loc = (a.to(cuda) for a in dit_inputs(case))
    pm = dit_padding_mask(case).to(cuda)
    eng = m.engine()
    with torch.inference_mode():
        full = eng.inner(x, t, cond, gemb, loc, padding_mask=pm).clone()
        for b, n in enumerate(case["valid"]):
            one = eng.inner(x[b:b + 1, :, :n], t[b:b + 1], cond[b:b + 1], gemb[b:b + 1], loc[b:b + 1, :, :n])
            assert rel_l2(full[b:b + 1, :, :n], one) < 5e-3


def test_masked_graph_replay_matches_eager(cuda):
    """CUDA-graph replay with a padding mask (the mask fixes the row layout at capture) equals the eager call;
    a second mask gets its own graph and the first graph still replays correctly afterwards."""
    case = CASES["dit_small_cfg_mask"]
    m = _model(case, "fp8")
    x, t, cond, gemb, loc = (a.to(cuda) for a in dit_inputs(case))
    pm = dit_padding_mask(case).to(cuda)
    pm2 = dit_padding_mask(replace_valid(case, [60, 180])).to(cuda)
    kw = dict(cross_attn_cond=cond, global_embed=gemb, local_add_cond=loc, cfg_scale=case["cfg_scale"],
              apg_scale=case["apg_scale"])
    with torch.inference_mode():
        eager = m(x, t, padding_mask=pm, **kw).clone()
        eager2 = m(x, t, padding_mask=pm2, **kw).clone()
        m.enable_cuda_graph()
        g1 = m(x, t, padding_mask=pm, **kw).clone()
        g2 = m(x, t, padding_mask=pm2, **kw).clone()
        g1b = m(x, t, padding_mask=pm, **kw).clone()
    torch.cuda.synchronize()
    assert rel_l2(g1, eager) < 1e-3
    assert rel_l2(g2, eager2) < 1e-3
    assert torch.equal(g1, g1b)


def replace_valid(case, valid):
    c = dict(case)
    c["valid"] = valid
    return c


def test_cfg_interval_outside_skips_guidance(cuda):
    """cfg_interval (dit.py:479): outside the interval the call is a plain conditional forward."""
    case = CASES["dit_small_cfg_mask"]
    m = _model(case, "bf16")
    x, t, cond, gemb, loc = (a.to(cuda) for a in dit_inputs(case))
    with torch.inference_mode():
        plain = m(x, t, cross_attn_cond=cond, global_embed=gemb, local_add_cond=loc)
        out = m(x, t, cross_attn_cond=cond, global_embed=gemb, local_add_cond=loc, cfg_scale=5.0,
                cfg_interval=(0.95, 1.0))
    assert torch.equal(out, plain)

