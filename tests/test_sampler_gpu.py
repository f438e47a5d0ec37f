"""The ping-pong sampler (stable_audio_3/inference/sampling.py:308-351) on a B200.

* The whole 8-step loop captured as one CUDA graph (GraphedPingpong) replays to the eager loop through the
  public DiffusionTransformer call, draw for draw (same noise inputs): relative L2 <= 1e-3, for a global and a
  per-element schedule, with a padding mask, across two replays with different inputs.
* The eager loop against the reference loop restated here on the CPU oracle (fp32) with the same draws: the
  final sample within 2e-2 relative L2 (bf16 model).
"""
import pytest
import torch

from oracle import dit as odit
from sa3_b200.modules import DiffusionTransformer, init_synthetic_
from tests.golden.cases import CASES, dit_inputs, dit_padding_mask
from tests.test_oracle_golden import _cfg

pytestmark = pytest.mark.gpu
STEPS = 8


def rel(a, b):
    a, b = a.float().cpu(), b.float().cpu()
    return ((a - b).norm() / b.norm()).item()


def _model(case, mode):
    m = init_synthetic_(DiffusionTransformer(case["cfg"]), seed=case["seed"])
    with torch.no_grad():
        for p in m.parameters():
            p.copy_(p.bfloat16().float())
    return m.quantize(mode)


def _schedule(per_element: bool, batch: int):
    s = torch.linspace(1.0, 0.0, STEPS + 1)
    if per_element:
        s = torch.stack([s, s.pow(1.5)])[:batch]
    return s


@pytest.mark.parametrize("per_element,masked", [(False, False), (True, True)])
def test_graphed_pingpong_matches_eager(cuda, per_element, masked):
    from sa3_b200.sampler import GraphedPingpong, sample_flow_pingpong

    case = CASES["dit_small_cfg_mask"]
    m = _model(case, "fp8")
    x, _, cond, gemb, loc = (a.to(cuda) for a in dit_inputs(case))
    pm = dit_padding_mask(case).to(cuda) if masked else None
    sig = _schedule(per_element, x.shape[0]).to(cuda)
    g = torch.Generator(device=cuda).manual_seed(5)
    kw = dict(cross_attn_cond=cond, global_embed=gemb, local_add_cond=loc, cfg_scale=case["cfg_scale"],
              apg_scale=case["apg_scale"])
    with torch.inference_mode():
        graphed = GraphedPingpong(m.engine(), x, sig, torch.zeros(STEPS, *x.shape, device=cuda), cond, gemb, loc,
                                  case["cfg_scale"], case["apg_scale"], padding_mask=pm)
        for rep in range(2):
            x0 = torch.randn(x.shape, device=cuda, generator=g)
            noise = torch.randn(STEPS, *x.shape, device=cuda, generator=g)
            eager = sample_flow_pingpong(lambda xx, tt: m(xx, tt, padding_mask=pm, **kw), x0, sig, noise)
            out = graphed(x0, noise, cond, gemb, loc).clone()
            torch.cuda.synchronize()
            assert torch.isfinite(out).all()
            assert rel(out, eager) < 1e-3, rep


def test_pingpong_matches_oracle_loop(cuda):
    from sa3_b200.sampler import sample_flow_pingpong

    case = CASES["dit_small_cfg"]
    m = _model(case, "bf16")
    x, _, cond, gemb, loc = dit_inputs(case)
    sig = _schedule(False, x.shape[0])
    g = torch.Generator().manual_seed(8)
    noise = torch.randn(STEPS, *x.shape, generator=g)
    sd = m.state_dict()
    ocfg = _cfg(case["cfg"])
    # the reference loop (sampling.py:319-351), on the oracle's DiffusionTransformer.forward
    xr = x.clone()
    for i in range(STEPS):
        tc, tn = float(sig[i]), float(sig[i + 1])
        v = odit.dit_forward(sd, ocfg, xr, torch.full((x.shape[0],), tc), cond, gemb, loc, case["cfg_scale"],
                             case["apg_scale"])
        xr = (1 - tn) * (xr - tc * v) + tn * noise[i]
    kw = dict(cross_attn_cond=cond.to(cuda), global_embed=gemb.to(cuda), local_add_cond=loc.to(cuda),
              cfg_scale=case["cfg_scale"], apg_scale=case["apg_scale"])
    with torch.inference_mode():
        out = sample_flow_pingpong(lambda xx, tt: m(xx, tt, **kw), x.to(cuda), sig.to(cuda), noise.to(cuda))
    err = rel(out, xr)
    print(f"8-step ping-pong sample, bf16 vs oracle: rel L2 {err:.3e}")
    assert err < 2e-2
