"""GPTQ int4 path on a B200 vs the oracle's GPTQ definition.

* dequantisation (index math + arithmetic): bit-exact vs bf16(oracle W[:, perm]) (sorted channels) and vs
  bf16(oracle W) (original channel order, the large-batch path's dense weight).
* GEMM / QuantLinearGPTQ: relative Frobenius <= 2e-2 vs F.linear(x, dequant(W)) (asserted 5e-3;
  bf16 rounding of x and W is the only difference).
* DiT network output in GPTQ mode: <= 2e-2 relative L2 vs the oracle.
"""
import numpy as np
import pytest
import torch

from oracle import dit as odit
from oracle import quant as oq

pytestmark = pytest.mark.gpu


def rel_fro(a, b):
    a, b = a.float().cpu(), b.float().cpu()
    return ((a - b).norm() / b.norm()).item()


def test_gptq_dequant_bit_exact(cuda):
    from sa3_b200 import gptq, ops

    qw, qz, sc, gi = oq.random_gptq_layer(512, 1536, seed=11)
    p = gptq.to_device(gptq.repack(qw, qz, sc, gi), cuda)
    w = ops.gptq_dequant(p["qw"], p["sz"], 512, 1536)
    ref = torch.from_numpy(oq.gptq_dequant(qw, qz, sc, gi)[:, p["perm"].cpu().numpy()]).bfloat16()
    assert torch.equal(w.cpu().view(torch.int16), ref.view(torch.int16))


@pytest.mark.parametrize("N,K", [(512, 1536), (768, 6144), (256, 256)])
def test_gptq_dequant_orig_bit_exact(cuda, N, K):
    """Dense weight in the original input-channel order (act-order undone through inv_perm): every bf16 bit
    equals bf16 of the oracle's (q - z[g_idx]) * s[g_idx]."""
    from sa3_b200 import gptq, ops

    qw, qz, sc, gi = oq.random_gptq_layer(N, K, seed=N + K)
    p = gptq.to_device(gptq.repack(qw, qz, sc, gi), cuda)
    w = ops.gptq_dequant_orig(p["qw"], p["sz"], p["inv_perm"], N, K)
    ref = torch.from_numpy(oq.gptq_dequant(qw, qz, sc, gi)).bfloat16()
    assert torch.equal(w.cpu().view(torch.int16), ref.view(torch.int16))


@pytest.mark.parametrize("M,N,K", [(300, 512, 1536), (1000, 768, 6144), (2, 256, 256)])
def test_gptq_gemm(cuda, M, N, K):
    from sa3_b200 import gptq, ops

    qw, qz, sc, gi = oq.random_gptq_layer(N, K, seed=M + N)
    p = gptq.to_device(gptq.repack(qw, qz, sc, gi), cuda)
    g = torch.Generator().manual_seed(1)
    x = torch.randn(M, K, generator=g).bfloat16()
    xp = ops.permute_cols(x.to(cuda), p["perm"])
    assert torch.equal(xp.cpu(), x[:, p["perm"].cpu().long()])
    y = ops.gptq_gemm(xp, p["qw"], p["sz"], N)
    ref = oq.gptq_linear(x.float(), qw, qz, sc, gi)
    assert rel_fro(y, ref) < 5e-3


def test_quant_linear_gptq_module(cuda):
    from sa3_b200.gptq import QuantLinearGPTQ

    qw, qz, sc, gi = oq.random_gptq_layer(1536, 1536, seed=2)
    bias = torch.randn(1536) * 0.1
    m = QuantLinearGPTQ.from_gptq(qw, qz, sc, gi, bias=bias, device=cuda)
    x = torch.randn(2, 100, 1536).bfloat16()
    y = m(x.to(cuda))
    ref = oq.gptq_linear(x.float().reshape(-1, 1536), qw, qz, sc, gi, bias).reshape(2, 100, 1536)
    assert rel_fro(y, ref) < 5e-3


@pytest.mark.parametrize("L", [200, 600])
def test_dit_gptq_network_matches_oracle(cuda, L):
    """GPTQ DiT network output vs the oracle. L = 200 (528 token rows) runs every int4 linear on the
    shared-memory-dequantising kernel; L = 600 (1328 rows) runs the block linears on the large-batch path
    (dense weight dequantised once per call, bf16 GEMM on the unpermuted activations)."""
    from sa3_b200.modules import DiffusionTransformer, init_synthetic_
    from tests.golden.cases import CASES
    from tests.test_oracle_golden import _cfg
    from tests.test_model_gpu import _batched_inputs

    case = dict(CASES["dit_small_cfg"], L=L)
    m = init_synthetic_(DiffusionTransformer(case["cfg"]), seed=case["seed"])
    layers = {}
    for i, (name, mod) in enumerate(sorted(m.named_modules())):
        if isinstance(mod, torch.nn.Linear) and name.endswith(odit.QUANT_LINEARS):
            layers[name] = oq.random_gptq_layer(mod.out_features, mod.in_features, seed=100 + i)
    with torch.no_grad():
        for p_ in m.parameters():
            p_.copy_(p_.bfloat16().float())
    m.quantize("gptq", gptq_layers=layers)
    inputs = _batched_inputs(case)
    with torch.inference_mode():
        lin = odit.Linears(m.state_dict(), "gptq", layers)
        ref = odit.dit_inner_forward(lin, m.state_dict(), _cfg(case["cfg"]), *inputs)
        out = m.engine().inner(*(a.to(cuda) for a in inputs))
    assert torch.isfinite(out).all()
    err = rel_fro(out, ref)
    print(f"GPTQ DiT L={L}: network velocity rel L2 {err:.3e}")
    assert err < 2e-2, err
