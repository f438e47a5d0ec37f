"""Variable-length packed batches on a B200: prompts of different lengths packed back to back (no padding)
give the same network output as running each prompt on its own (bf16: <= 1e-3; the kernels compute each
row independently of the others, so only the packing tables differ), and the FP8 path (whose per-tensor
activation scales span the packed batch) stays within 2e-2."""
import pytest
import torch

from tests.golden.cases import CASES

pytestmark = pytest.mark.gpu


def rel(a, b):
    return ((a.float() - b.float()).norm() / b.float().norm()).item()


@pytest.mark.parametrize("mode,tol", [("bf16", 1e-3), ("fp8", 2e-2)])
def test_varlen_matches_per_prompt(cuda, mode, tol):
    from sa3_b200.modules import DiffusionTransformer, init_synthetic_

    cfg = CASES["dit_small_cfg"]["cfg"]
    m = init_synthetic_(DiffusionTransformer(cfg), seed=9).quantize(mode)
    eng = m.engine()
    g = torch.Generator().manual_seed(3)
    lens = [100, 257, 40]
    P = len(lens)
    xs = [torch.randn(256, L, generator=g).to(cuda) for L in lens]
    locs = [torch.randn(257, L, generator=g).to(cuda) * 0.5 for L in lens]
    t = (torch.rand(P, generator=g) * 0.8 + 0.1).to(cuda)
    cond = torch.randn(P, 16, 768, generator=g).to(cuda)
    gemb = torch.randn(P, 768, generator=g).to(cuda)
    with torch.inference_mode():
        packed = [o.clone() for o in eng.inner_varlen(xs, t, cond, gemb, locs)]
        for i in range(P):
            single = eng.inner(xs[i][None], t[i:i + 1], cond[i:i + 1], gemb[i:i + 1], locs[i][None])[0].clone()
            assert rel(packed[i], single) < tol, i
        v = eng.forward_varlen(xs, t, cond, gemb, locs, cfg_scale=5.0, apg_scale=1.0)
        for i in range(P):
            vi = eng.forward(xs[i][None], t[i:i + 1], cond[i:i + 1], gemb[i:i + 1], locs[i][None], 5.0, 1.0)[0]
            assert torch.isfinite(v[i]).all()
            if mode == "bf16":
                assert rel(v[i], vi) < 1e-3, i
