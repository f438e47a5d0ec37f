"""Variable-length packed batches on a B200: prompts of different lengths packed back to back (no padding).

  * bf16: each packed prompt's network output equals running that prompt on its own (<= 1e-3; the kernels
    compute each row independently of the others, so only the packing tables differ).
  * FP8: the per-tensor activation scales span the packed batch, so a prompt's quantization grid depends on its
    batch-mates; the packed network output is checked against the oracle's packed restatement
    (dit_inner_forward_packed, FP8 definition at the bf16 deployment's activations, <= 2e-2), and each prompt's
    CFG/APG velocity against the oracle's combine of those outputs (tests.tolerance.fp8_network_bound).
"""
from dataclasses import replace

import pytest
import torch

from oracle import dit as odit
from tests.golden.cases import CASES
from tests.test_oracle_golden import _cfg
from tests.tolerance import fp8_network_bound

pytestmark = pytest.mark.gpu


def rel(a, b):
    a, b = a.float().cpu(), b.float().cpu()
    return ((a - b).norm() / b.norm()).item()


@pytest.mark.parametrize("mode", ["bf16", "fp8"])
def test_varlen_matches_per_prompt(cuda, mode):
    from sa3_b200.modules import DiffusionTransformer, init_synthetic_

    cfg = CASES["dit_small_cfg"]["cfg"]
    m = init_synthetic_(DiffusionTransformer(cfg), seed=9).quantize(mode)
    eng = m.engine()
    g = torch.Generator().manual_seed(3)
    lens = [100, 257, 40]
    P = len(lens)
    xs = [torch.randn(256, L, generator=g) for L in lens]
    locs = [torch.randn(257, L, generator=g) * 0.5 for L in lens]
    t = torch.rand(P, generator=g) * 0.8 + 0.1
    cond = torch.randn(P, 16, 768, generator=g)
    gemb = torch.randn(P, 768, generator=g)
    d = lambda a: a.to(cuda)  # noqa: E731
    with torch.inference_mode():
        packed = [o.clone() for o in eng.inner_varlen([d(x) for x in xs], d(t), d(cond), d(gemb),
                                                      [d(lc) for lc in locs])]
        v = eng.forward_varlen([d(x) for x in xs], d(t), d(cond), d(gemb), [d(lc) for lc in locs], cfg_scale=5.0,
                               apg_scale=1.0)
        if mode == "bf16":
            for i in range(P):
                single = eng.inner(d(xs[i])[None], d(t[i:i + 1]), d(cond[i:i + 1]), d(gemb[i:i + 1]),
                                   d(locs[i])[None])[0]
                assert rel(packed[i], single) < 1e-3, i
                vi = eng.forward(d(xs[i])[None], d(t[i:i + 1]), d(cond[i:i + 1]), d(gemb[i:i + 1]),
                                 d(locs[i])[None], 5.0, 1.0)[0]
                assert rel(v[i], vi) < 1e-3, i
            return
        sd = m.state_dict()
        lin = odit.Linears(sd, "fp8")
        ocfg = replace(_cfg(cfg), act_bf16=True)
        ref = odit.dit_inner_forward_packed(lin, sd, ocfg, xs, t, cond, gemb, locs)
        # both CFG halves of every prompt in one packed batch (cond halves first), as forward_varlen runs them
        zc = torch.zeros_like(cond)
        cfg_args = (xs + xs, torch.cat([t, t]), torch.cat([cond, zc]), torch.cat([gemb, gemb]), locs + locs)
        ref2 = odit.dit_inner_forward_packed(lin, sd, ocfg, *cfg_args)
        ref2_32 = odit.dit_inner_forward_packed(lin, sd, _cfg(cfg), *cfg_args)
    for i in range(P):
        e_net = rel(packed[i], ref[i])
        vref = odit.cfg_combine(xs[i][None], t[i:i + 1], torch.stack([ref2[i], ref2[P + i]]), 5.0, 1.0)[0]
        vref32 = odit.cfg_combine(xs[i][None], t[i:i + 1], torch.stack([ref2_32[i], ref2_32[P + i]]), 5.0, 1.0)[0]
        e_v = rel(v[i], vref)
        bound = fp8_network_bound(vref, vref32)
        print(f"prompt {i} (L={lens[i]}): FP8 packed network rel L2 {e_net:.3e}, CFG velocity {e_v:.3e} "
              f"(bound {bound:.3e})")
        assert e_net < 2e-2, i
        assert e_v < bound, i
