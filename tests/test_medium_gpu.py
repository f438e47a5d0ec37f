"""Parity at the medium shape the benchmark times (B=2 CFG halves, N = 8183 + 64 tokens, M = 16494 token rows,
D = 1536, 24 heads x 64, window (256, 256), differential attention).

At this size every persistent kernel runs many work items per CTA (FF1: 65 x 48 = 3120 tiles of 256 x 256 over
74 CTA pairs; self-attention: 1584 items over 148 CTAs), so these tests cover the paths the small-shape tests
cannot reach: both TMEM accumulators of the GEMM, the accumulator hand-over between tiles, the epilogue's
prefetch of the next tile, and the attention kernel's item loop with shared V.

The oracle runs on a fixed subsample of rows (every 29th row plus the last 300, so every 256-row tile is
represented in every column tile) to keep the CPU side within seconds. Bounds (written per test):
  * FP8 / bf16 GEMM: relative Frobenius error <= 5e-3 against the quantized definition (contract: 2e-2);
  * attention: max|out - ref| / max|ref| <= 1e-2 against fp32;
  * the network's velocity prediction of a one-block medium DiT (FP8): tests.tolerance.fp8_network_bound.
"""
import math

import pytest
import torch

from oracle import quant as oq
from oracle import ref as orf
from tests.tolerance import fp8_network_bound

pytestmark = pytest.mark.gpu

B, L, NM, D, H = 2, 8183, 64, 1536, 24
N = L + NM
M = B * N
W = 256


def rel_fro(a, b):
    a, b = a.float().cpu(), b.float().cpu()
    return ((a - b).norm() / b.norm().clamp_min(1e-30)).item()


def max_rel(a, b):
    a, b = a.float().cpu(), b.float().cpu()
    return ((a - b).abs().max() / b.abs().max().clamp_min(1e-30)).item()


def _rows(m=M):
    return torch.cat([torch.arange(0, m, 29), torch.arange(m - 300, m)]).unique()


def _dgen(cuda, seed):
    return torch.Generator(device=cuda).manual_seed(seed)


def _quantized_activation(cuda, k, seed):
    """A bf16 activation [M, k] quantized on the device exactly as the DiT step does (max|x| pass, e4m3 pass)."""
    from sa3_b200 import ops

    x = torch.randn(M, k, device=cuda, generator=_dgen(cuda, seed)).bfloat16()
    amax = torch.zeros(1, device=cuda)
    s = torch.zeros(1, device=cuda)
    ops.absmax(x, amax)
    xq = ops.quantize_e4m3(x, amax, scale_out=s)
    return x, xq, s


def _fp8_ref(xq_rows, s, wq, sw, bias=None):
    """The FP8 linear's definition on device-quantized activation rows: (Xq s_x)(Wq s_w)^T + b in fp32."""
    y = (xq_rows.float() * s.cpu()) @ (wq.float() * sw[:, None]).T
    return y if bias is None else y + bias


def test_medium_activation_quantisation_bit_exact(cuda):
    """The FF hidden activation (M x 6144, 101 M elements): scale and every e4m3 byte equal the oracle's."""
    x, xq, s = _quantized_activation(cuda, 6144, 1)
    xc = x.float().cpu()
    assert torch.equal(s.cpu(), oq.act_scale(xc).reshape(1))
    ref = (xc * oq.act_inv_scale(xc)).clamp(-448, 448).to(torch.float8_e4m3fn)
    assert torch.equal(xq.cpu().view(torch.uint8), ref.view(torch.uint8))


@pytest.mark.parametrize("kind", ["ff1_swiglu", "qkv_qk_norm_rope", "ff2_gated_residual", "out_gated_residual",
                                  "cross_out_residual"])
def test_medium_fp8_gemm(cuda, kind):
    """Each FP8 GEMM of the block at M = 16494 with the epilogue the step uses, against the FP8 definition."""
    from sa3_b200 import ops, _lib
    from sa3_b200.quant import interleave_swiglu_rows

    n, k = {"ff1_swiglu": (12288, 1536), "qkv_qk_norm_rope": (7680, 1536), "ff2_gated_residual": (1536, 6144),
            "out_gated_residual": (1536, 1536), "cross_out_residual": (1536, 1536)}[kind]
    g = torch.Generator().manual_seed(n + k)
    w = torch.randn(n, k, generator=g) * 0.02
    bias = torch.randn(n, generator=g) * 0.1
    wq, sw = oq.quantize_weight_e4m3(w)
    x, xq, s = _quantized_activation(cuda, k, n)
    rows = _rows()
    h = _fp8_ref(xq[rows.to(cuda)].cpu(), s, wq, sw, bias)
    if kind == "ff1_swiglu":
        w8, sw8 = interleave_swiglu_rows(wq.view(torch.uint8), sw)
        _, b8 = interleave_swiglu_rows(w, bias)
        amax = torch.zeros(1, device=cuda)
        out = ops.gemm(xq, w8.view(torch.float8_e4m3fn).to(cuda), a_scale=s, b_scale=sw8.to(cuda), bias=b8.to(cuda),
                       kind=_lib.EPI_SWIGLU, amax_out=amax)
        torch.cuda.synchronize()
        err = rel_fro(out[rows.to(cuda)], orf.swiglu(h))
        assert amax.item() == out.float().abs().max().item()
    elif kind == "qkv_qk_norm_rope":
        gq = 1 + 0.1 * torch.randn(64, generator=g)
        gk = 1 + 0.1 * torch.randn(64, generator=g)
        pos = (torch.arange(M) % N).to(torch.int32)
        table = ops.rope_table(N, device=cuda)
        out = ops.gemm(xq, wq.to(cuda), a_scale=s, b_scale=sw.to(cuda), bias=bias.to(cuda), kind=_lib.EPI_QK_NORM,
                       qk=dict(gammas=[gq.to(cuda), gk.to(cuda), None, gq.to(cuda), gk.to(cuda)], group_width=D,
                               rope=[True, True, False, True, True], eps=1e-6, cos_sin=table,
                               row_pos=pos.to(cuda)))
        torch.cuda.synchronize()
        freqs = orf.rotary_freqs(N, 32)[pos[rows].long()]
        ref = h.view(len(rows), 5, H, 64).clone()
        for part, gm in ((0, gq), (1, gk), (3, gq), (4, gk)):
            t = ref[:, part].permute(1, 0, 2)  # [H, rows, 64]
            ref[:, part] = orf.apply_rotary(orf.rms_norm(t, gm, 1e-6), freqs).permute(1, 0, 2)
        err = rel_fro(out[rows.to(cuda)], ref.view(len(rows), n))
    else:
        res = torch.randn(M, n, device=cuda, generator=_dgen(cuda, 7))
        out = res.clone()
        if kind == "cross_out_residual":
            ops.gemm(xq, wq.to(cuda), out, a_scale=s, b_scale=sw.to(cuda), bias=bias.to(cuda), kind=_lib.EPI_RESIDUAL,
                     residual=out)
            branch = h
        else:
            gate = torch.randn(B, n, generator=g)
            row_batch = (torch.arange(M) // N).to(torch.int32)
            ops.gemm(xq, wq.to(cuda), out, a_scale=s, b_scale=sw.to(cuda), bias=bias.to(cuda),
                     kind=_lib.EPI_GATED_RESIDUAL, residual=out, gate=gate.to(cuda), row_batch=row_batch.to(cuda))
            branch = orf.gate_residual(h, gate[row_batch[rows].long()], torch.zeros_like(h))
        torch.cuda.synchronize()
        rd = rows.to(cuda)
        err = rel_fro(out[rd] - res[rd], branch)
    print(f"{kind}: rel Frobenius {err:.2e}")
    assert err < 5e-3
    assert _lib.device_error() == 0


def test_medium_local_cond_residual_row_map(cuda):
    """The local-conditioning output GEMM (bf16, K = 1536) adds into the latent rows of the fp32 stream through
    the output-row map; the 64 memory rows of each sequence stay untouched."""
    from sa3_b200 import ops, _lib

    R = B * L
    g = torch.Generator().manual_seed(5)
    w = (torch.randn(D, D, generator=g) * 0.02).bfloat16()
    bias = torch.randn(D, generator=g) * 0.1
    t1 = torch.randn(R, D, device=cuda, generator=_dgen(cuda, 11)).bfloat16()
    lat_rows = torch.cat([torch.arange(b * N + NM, (b + 1) * N) for b in range(B)]).to(torch.int32)
    h = torch.randn(M, D, device=cuda, generator=_dgen(cuda, 12))
    out = h.clone()
    ops.gemm(t1, w.to(cuda), out, bias=bias.to(cuda), kind=_lib.EPI_RESIDUAL, residual=out,
             out_row_map=lat_rows.to(cuda))
    torch.cuda.synchronize()
    rows = _rows(R)
    ref = t1[rows.to(cuda)].float().cpu() @ w.float().T + bias
    dst = lat_rows[rows].long().to(cuda)
    assert rel_fro(out[dst] - h[dst], ref) < 5e-3
    mem = torch.cat([torch.arange(b * N, b * N + NM) for b in range(B)]).to(cuda)
    assert torch.equal(out[mem], h[mem])
    assert _lib.device_error() == 0


def _band_attention_rows(q, k, v, q0, q1, wl, wr, n):
    """fp32 windowed attention of queries [q0, q1) of one sequence over its keys [q0 - wl, q1 + wr) (the band
    of transformer.py:598-700), for tensors [heads, n, 64]."""
    k0, k1 = max(0, q0 - wl), min(n, q1 + wr)
    d = torch.arange(k0, k1)[None, :] - torch.arange(q0, q1)[:, None]
    ok = (d >= -wl) & (d <= wr)
    s = (q[:, q0:q1] @ k[:, k0:k1].transpose(-1, -2)) / math.sqrt(64)
    s = s.masked_fill(~ok, float("-inf"))
    return torch.softmax(s, -1) @ v[:, k0:k1]


# query tiles checked per sequence: both sequence ends (the ragged last tile included) and tiles spread
# over the sequence
_QTILES = [(0, 128), (128, 384), (1000, 1128), (4096, 4224), (6000, 6300), (8064, 8192), (8192, N)]


def test_medium_differential_self_attention(cuda):
    """Differential +-256 self-attention with shared V, B=2, N=8247, 24 heads, called as the DiT step calls it
    (five column groups of the fused q|k|v|q'|k' rows, sequence table, max|out| for the next quantisation)."""
    from sa3_b200 import ops, _lib

    qkv = torch.randn(M, 5 * D, device=cuda, generator=_dgen(cuda, 21)).bfloat16()
    cu = torch.tensor([0, N, 2 * N], dtype=torch.int32, device=cuda)
    o = torch.empty(M, D, device=cuda, dtype=torch.bfloat16)
    amax = torch.zeros(1, device=cuda)
    ops.attention(qkv[:, 0:D], qkv[:, D:2 * D], qkv[:, 2 * D:3 * D], q2=qkv[:, 3 * D:4 * D], k2=qkv[:, 4 * D:5 * D],
                  heads=H, window=(W, W), out=o, amax_out=amax, cu_seqlens_q=cu, cu_seqlens_k=cu, max_seqlen_q=N,
                  max_seqlen_k=N)
    torch.cuda.synchronize()
    assert amax.item() == o.float().abs().max().item()
    worst = 0.0
    for b in range(B):
        parts = [qkv[b * N:(b + 1) * N, i * D:(i + 1) * D].float().cpu().view(N, H, 64).permute(1, 0, 2)
                 for i in range(5)]
        q, k, v, q2, k2 = parts
        ob = o[b * N:(b + 1) * N].float().cpu().view(N, H, 64).permute(1, 0, 2)
        for q0, q1 in _QTILES:
            ref = (_band_attention_rows(q, k, v, q0, q1, W, W, N) - _band_attention_rows(q2, k2, v, q0, q1, W, W, N))
            worst = max(worst, max_rel(ob[:, q0:q1], ref))
    print(f"medium differential attention: max rel {worst:.2e}")
    assert worst < 1e-2
    assert _lib.device_error() == 0


def test_medium_differential_cross_attention(cuda):
    """Differential cross-attention of the 16494 query rows over each sequence's 128 context tokens."""
    from sa3_b200 import ops, _lib

    Tc = 128
    qx = torch.randn(M, 2 * D, device=cuda, generator=_dgen(cuda, 31)).bfloat16()
    kv = torch.randn(B * Tc, 3 * D, device=cuda, generator=_dgen(cuda, 32)).bfloat16()
    cu = torch.tensor([0, N, 2 * N], dtype=torch.int32, device=cuda)
    cu_ctx = torch.tensor([0, Tc, 2 * Tc], dtype=torch.int32, device=cuda)
    o = torch.empty(M, D, device=cuda, dtype=torch.bfloat16)
    ops.attention(qx[:, 0:D], kv[:, 0:D], kv[:, 2 * D:3 * D], q2=qx[:, D:2 * D], k2=kv[:, D:2 * D], heads=H, out=o,
                  cu_seqlens_q=cu, cu_seqlens_k=cu_ctx, max_seqlen_q=N, max_seqlen_k=Tc)
    torch.cuda.synchronize()
    rows = _rows()
    worst = 0.0
    for b in range(B):
        r = rows[(rows >= b * N) & (rows < (b + 1) * N)]
        hd = lambda t: t.float().cpu().view(-1, H, 64).permute(1, 0, 2)  # noqa: E731
        q, q2 = hd(qx[r.to(cuda), 0:D]), hd(qx[r.to(cuda), D:2 * D])
        k, k2, v = (hd(kv[b * Tc:(b + 1) * Tc, i * D:(i + 1) * D]) for i in range(3))
        ref = orf.attention(q, k, v) - orf.attention(q2, k2, v)
        worst = max(worst, max_rel(hd(o[r.to(cuda)]), ref))
    print(f"medium differential cross-attention: max rel {worst:.2e}")
    assert worst < 1e-2
    assert _lib.device_error() == 0


def test_medium_one_block_dit_fp8(cuda):
    """A one-block medium DiT (D=1536, 24 heads, differential, +-256, FP8 linears) at the benchmarked length:
    the network's velocity prediction for both CFG halves (L = 8183, 128 context tokens, local conditioning)
    against the FP8 definition at the bf16 deployment's activations, held to tests.tolerance.fp8_network_bound
    (the FP8 definition itself moves by 2.7e-2 here when its activations are rounded to bf16)."""
    from oracle import dit as odit
    from sa3_b200 import _lib
    from sa3_b200.modules import MEDIUM, DiffusionTransformer, init_synthetic_, with_depth

    cfg = with_depth(MEDIUM, 1)
    m = init_synthetic_(DiffusionTransformer(cfg), seed=0).quantize("fp8")
    g = torch.Generator().manual_seed(0)
    x = torch.randn(1, 256, L, generator=g)
    t = torch.tensor([0.6])
    cond = torch.randn(1, 128, 768, generator=g)
    gemb = torch.randn(1, 768, generator=g)
    loc = torch.randn(1, 257, L, generator=g) * 0.5
    batched = odit.cfg_batch(x, t, cond, gemb, loc)
    with torch.inference_mode():
        out = m.engine().inner(*(a.to(cuda) for a in batched))
        torch.cuda.synchronize()
        sd = m.state_dict()
        lin = odit.Linears(sd, "fp8")
        ref = odit.dit_inner_forward(lin, sd, odit.Cfg(depth=1, act_bf16=True), *batched)
        ref32 = odit.dit_inner_forward(lin, sd, odit.Cfg(depth=1), *batched)
    err = ((out.float().cpu() - ref).norm() / ref.norm()).item()
    err32 = ((out.float().cpu() - ref32).norm() / ref32.norm()).item()
    bound = fp8_network_bound(ref, ref32)
    print(f"one-block medium FP8 DiT: network velocity rel L2 {err:.2e} vs the FP8 definition at bf16 activations "
          f"({err32:.2e} vs the fp32-activation definition), bound {bound:.2e}")
    assert err < bound
    assert _lib.device_error() == 0
