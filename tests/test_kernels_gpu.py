"""Kernel parity on a B200: each CUDA op through the C ABI vs the CPU oracle on seeded inputs.

Tolerances (from the path's parity contract):
  * bf16 attention: max|out - ref| / max|ref| <= 1e-2 vs the fp32 oracle.
  * FP8 / bf16 GEMM: relative Frobenius error <= 2e-2 vs the oracle's quantized definition
    (we assert the much tighter 5e-3 where only bf16 output rounding separates them).
  * FP8 activation quantisation: bit-exact bytes vs the oracle's e4m3 rounding.
  * glue (norm / modulation / RoPE): bf16 output rounding only, max-abs-rel <= 1e-2.
"""
import math

import pytest
import torch

from oracle import quant as oq
from oracle import ref as orf

pytestmark = pytest.mark.gpu


def _gen(seed):
    g = torch.Generator().manual_seed(seed)
    return g


def rel_fro(a, b):
    a, b = a.float().cpu(), b.float().cpu()
    return ((a - b).norm() / b.norm().clamp_min(1e-30)).item()


def max_rel(a, b):
    a, b = a.float().cpu(), b.float().cpu()
    return ((a - b).abs().max() / b.abs().max().clamp_min(1e-30)).item()


# ----------------------------------------------------------------------------- GEMM
@pytest.mark.parametrize("M,N,K", [(128, 256, 64), (300, 512, 320), (1000, 640, 1024), (2, 1536, 1536)])
def test_gemm_bf16(cuda, M, N, K):
    from sa3_b200 import ops

    g = _gen(M + N + K)
    a = torch.randn(M, K, generator=g)
    b = torch.randn(N, K, generator=g) * 0.05
    bias = torch.randn(N, generator=g)
    ref = a.bfloat16().float() @ b.bfloat16().float().T + bias
    out = ops.gemm(a.bfloat16().to(cuda), b.bfloat16().to(cuda), bias=bias.to(cuda))
    torch.cuda.synchronize()
    assert rel_fro(out, ref) < 5e-3


@pytest.mark.parametrize("M,N,K", [(256, 512, 256), (777, 768, 1536), (130, 256, 6144)])
def test_gemm_fp8_matches_quantized_definition(cuda, M, N, K):
    from sa3_b200 import ops

    g = _gen(7 * M + N)
    x = torch.randn(M, K, generator=g)
    w = torch.randn(N, K, generator=g) * 0.02
    wq, sw = oq.quantize_weight_e4m3(w)
    xb = x.bfloat16()
    ref = oq.fp8_linear(xb.float(), wq, sw)

    xd = xb.to(cuda)
    amax = torch.zeros(1, device=cuda)
    ops.absmax(xd, amax)
    s = torch.zeros(1, device=cuda)
    xq = ops.quantize_e4m3(xd, amax, scale_out=s)
    out = ops.gemm(xq, wq.to(cuda), a_scale=s, b_scale=sw.to(cuda))
    torch.cuda.synchronize()
    # activation quantisation is bit-exact with the oracle's definition
    s_ref = oq.act_scale(xb.float())
    assert torch.equal(s.cpu(), s_ref.reshape(1))
    xq_ref = (xb.float() * oq.act_inv_scale(xb.float())).clamp(-448, 448).to(torch.float8_e4m3fn)
    assert torch.equal(xq.cpu().view(torch.uint8), xq_ref.view(torch.uint8))
    assert rel_fro(out, ref) < 5e-3


@pytest.mark.parametrize("M", [600, 777, 1030])
@pytest.mark.parametrize("kind", ["store", "swiglu", "gated_residual_f32", "residual_f32", "gated_residual_f32_oop",
                                  "residual_f32_oop"])
def test_gemm_fp8_pair_epilogues(cuda, M, kind):
    """FP8 GEMMs with M >= 512 run on the 2-SM (CTA pair, 256 x 256 tile) kernel. Every epilogue kind
    against the FP8 definition, with M leaving the last pair tile partly or wholly empty for one CTA.
    In-place fp32 residuals (C is the residual) are added by TMA reduce-add; out-of-place ones (_oop)
    load the residual and store the result through TMA."""
    from sa3_b200 import ops, _lib

    g = _gen(M + len(kind))
    B, N, K = 2, 512, 384
    x = torch.randn(M, K, generator=g)
    w = torch.randn(N, K, generator=g) * 0.05
    bias = torch.randn(N, generator=g) * 0.1
    wq, sw = oq.quantize_weight_e4m3(w)
    xd = x.to(cuda)
    amax = torch.zeros(1, device=cuda)
    ops.absmax(xd.bfloat16(), amax)
    s = torch.zeros(1, device=cuda)
    # fp32 definition of the linear on the same bf16-rounded activation the device quantises
    h = oq.fp8_linear(x.bfloat16().float(), wq, sw, bias)
    xq = ops.quantize_e4m3(xd.bfloat16(), amax, scale_out=s)
    wd, swd, bd = wq.to(cuda), sw.to(cuda), bias.to(cuda)
    rows_per_batch = (M + 1) // 2
    if kind == "store":
        out = ops.gemm(xq, wd, a_scale=s, b_scale=swd, bias=bd)
        ref = h
    elif kind == "swiglu":
        out = ops.gemm(xq, wd, a_scale=s, b_scale=swd, bias=bd, kind=_lib.EPI_SWIGLU)
        # rows are [x | gate] per 256-row block (the interleave the model applies to GLU.proj)
        hb = h.view(M, N // 256, 2, 128)
        ref = (hb[:, :, 0] * torch.nn.functional.silu(hb[:, :, 1])).reshape(M, N // 2)
    else:
        res = torch.randn(M, N, generator=g)
        gate = torch.randn(B, N, generator=g)
        oop = kind.endswith("_oop")
        out = torch.full((M, N), float("nan"), device=cuda) if oop else res.clone().to(cuda)
        resd = res.to(cuda) if oop else out
        if kind.startswith("gated_residual_f32"):
            ops.gemm(xq, wd, out, a_scale=s, b_scale=swd, bias=bd, kind=_lib.EPI_GATED_RESIDUAL, residual=resd,
                     gate=gate.to(cuda), rows_per_batch=rows_per_batch)
            bidx = torch.arange(M) // rows_per_batch
            ref = res + h * torch.sigmoid(1 - gate[bidx])
        else:
            ops.gemm(xq, wd, out, a_scale=s, b_scale=swd, bias=bd, kind=_lib.EPI_RESIDUAL, residual=resd)
            ref = res + h
        if oop:
            assert torch.equal(resd.cpu(), res)
    torch.cuda.synchronize()
    assert rel_fro(out, ref) < 5e-3
    assert _lib.device_error() == 0


@pytest.mark.parametrize("variant", ["bf16_f32_rowmap", "bf16_store", "fp8_store"])
def test_gemm_pair_short_k_many_tiles(cuda, variant):
    """The 2-SM kernel with few K slices per tile and ~20 tiles per CTA pair (the project_in GEMM of a
    16-sequence batch: M = 65744, N = 1536, K = 256), 40 launches back to back. Every launch finishes without
    a device timeout (a lagging epilogue warp must never miss an accumulator phase), the 40 launches take
    well under a second, and the output matches the fp32 product (relative Frobenius <= 5e-3)."""
    import time

    from sa3_b200 import _lib, ops

    g = _gen(65)
    M, N, K, L = 65744, 1536, 256, 4109
    x = torch.randn(M, K, generator=g)
    w = torch.randn(N, K, generator=g) * 0.05
    xd = x.to(cuda)
    if variant == "fp8_store":
        wq, sw = oq.quantize_weight_e4m3(w)
        amax, s = torch.zeros(1, device=cuda), torch.zeros(1, device=cuda)
        ops.absmax(xd.bfloat16(), amax)
        xq = ops.quantize_e4m3(xd.bfloat16(), amax, scale_out=s)
        ref = oq.fp8_linear(x.bfloat16().float(), wq, sw, None)
        wd, swd = wq.to(cuda), sw.to(cuda)
        out = torch.empty(M, N, device=cuda, dtype=torch.bfloat16)
        call = lambda: ops.gemm(xq, wd, out, a_scale=s, b_scale=swd)  # noqa: E731
    else:
        xb, wb = x.bfloat16(), w.bfloat16()
        ref = xb.float() @ wb.float().T
        xbd, wbd = xb.to(cuda), wb.to(cuda)
        if variant == "bf16_store":
            out = torch.empty(M, N, device=cuda, dtype=torch.bfloat16)
            call = lambda: ops.gemm(xbd, wbd, out)  # noqa: E731
        else:
            # latent rows of 16 sequences scattered into a stream with 64 memory rows per sequence
            rmap = torch.cat([torch.arange(b * (L + 64) + 64, (b + 1) * (L + 64)) for b in range(16)]).int()
            stream = torch.zeros(16 * (L + 64), N, device=cuda)
            call = lambda: ops.gemm(xbd, wbd, stream, out_row_map=rmap.to(cuda))  # noqa: E731
    call()
    torch.cuda.synchronize()
    assert _lib.device_error() == 0
    t0 = time.perf_counter()
    for _ in range(40):
        call()
    torch.cuda.synchronize()
    elapsed = time.perf_counter() - t0
    assert _lib.device_error() == 0
    assert elapsed < 0.5, elapsed
    got = stream.cpu()[rmap.long()] if variant == "bf16_f32_rowmap" else out
    assert rel_fro(got, ref) < 5e-3


@pytest.mark.parametrize("fp8", [False, True])
@pytest.mark.parametrize("M", [300, 1030, 9000])
def test_gemm_fp16_stream(cuda, M, fp8):
    """Epilogues into an fp16 residual stream. In place (residual = C, no row map) the result is added by a TMA
    reduce-add in fp16: C = fp16(C + fp16(gate * acc)); with an output-row map (the local-conditioning add and
    project_in) the generic epilogue loads the fp16 residual and stores fp16(C + acc). M = 300 runs the single-SM
    kernel, 1030 and 9000 the 2-SM kernel (9000: 36 tiles per pair, both TMEM accumulators). Against the fp32
    product with the same fp16 roundings: at most one fp16 ulp apart, relative Frobenius <= 1e-3."""
    from sa3_b200 import _lib, ops

    g = _gen(M + 7 * fp8)
    N, K, B = 512, 384, 2
    x = torch.randn(M, K, generator=g)
    w = torch.randn(N, K, generator=g) * 0.05
    bias = torch.randn(N, generator=g) * 0.1
    res = (torch.randn(M, N, generator=g) * 2).half()
    gate = torch.randn(B, N, generator=g)
    rpb = (M + 1) // 2
    bidx = torch.arange(M) // rpb
    if fp8:
        wq, sw = oq.quantize_weight_e4m3(w)
        xd = x.to(cuda).bfloat16()
        amax, s = torch.zeros(1, device=cuda), torch.zeros(1, device=cuda)
        ops.absmax(xd, amax)
        a = ops.quantize_e4m3(xd, amax, scale_out=s)
        h = oq.fp8_linear(x.bfloat16().float(), wq, sw, bias)
        args = dict(a_scale=s, b_scale=sw.to(cuda), bias=bias.to(cuda))
        wd = wq.to(cuda)
    else:
        a, wd = x.bfloat16().to(cuda), w.bfloat16().to(cuda)
        h = a.float().cpu() @ w.bfloat16().float().T + bias
        args = dict(bias=bias.to(cuda))

    def close(out, ref):
        out = out.float().cpu()
        ulp = torch.finfo(torch.float16).eps * ref.abs().clamp_min(2.0 ** -14)
        assert ((out - ref).abs() <= 1.01 * ulp).float().mean().item() > 0.999
        assert rel_fro(out, ref) < 1e-3

    # in place, gated (to_out / FF2) and plain (cross to_out)
    out = res.clone().to(cuda)
    ops.gemm(a, wd, out, kind=_lib.EPI_GATED_RESIDUAL, residual=out, gate=gate.to(cuda), rows_per_batch=rpb, **args)
    close(out, (res.float() + (h * torch.sigmoid(1 - gate[bidx])).half().float()).half().float())
    out = res.clone().to(cuda)
    ops.gemm(a, wd, out, kind=_lib.EPI_RESIDUAL, residual=out, **args)
    close(out, (res.float() + h.half().float()).half().float())
    # row-mapped residual and store into a larger stream (rows interleaved with untouched memory-token rows)
    rmap = (torch.arange(M) * 2 + 1).to(torch.int32)
    big = (torch.randn(2 * M + 1, N, generator=g)).half()
    out = big.clone().to(cuda)
    ops.gemm(a, wd, out, kind=_lib.EPI_RESIDUAL, residual=out, out_row_map=rmap.to(cuda), **args)
    ref = big.clone().float()
    ref[rmap.long()] = (big[rmap.long()].float() + h).half().float()
    close(out, ref)
    out = big.clone().to(cuda)
    ops.gemm(a, wd, out, out_row_map=rmap.to(cuda), **args)
    ref = big.clone().float()
    ref[rmap.long()] = h.half().float()
    close(out, ref)
    torch.cuda.synchronize()
    assert _lib.device_error() == 0


@pytest.mark.parametrize("stream", [torch.float32, torch.float16])
@pytest.mark.parametrize("M", [300, 2000])
def test_gated_residual_row_mask(cuda, M, stream):
    """The local-conditioning add over all stream rows: a gated residual whose gate rows are -inf (factor
    sigmoid(+inf) = 1) and +inf (factor 0), chosen per row. Rows with factor 1 are bit-identical to the plain
    residual add; rows with factor 0 (the memory tokens) are left bit-identical."""
    from sa3_b200 import _lib, ops

    g = _gen(M + 3)
    N, K = 512, 256
    a = torch.randn(M, K, generator=g).bfloat16().to(cuda)
    w = (torch.randn(N, K, generator=g) * 0.05).bfloat16().to(cuda)
    bias = (torch.randn(N, generator=g) * 0.1).to(cuda)
    h0 = torch.randn(M, N, generator=g).to(stream).to(cuda)
    kind = (torch.rand(M, generator=g) < 0.2).to(torch.int32)
    gate = torch.tensor([-math.inf, math.inf]).repeat_interleave(N).view(2, N).to(cuda)
    plain = h0.clone()
    ops.gemm(a, w, plain, kind=_lib.EPI_RESIDUAL, residual=plain, bias=bias)
    gated = h0.clone()
    ops.gemm(a, w, gated, kind=_lib.EPI_GATED_RESIDUAL, residual=gated, gate=gate, row_batch=kind.to(cuda),
             bias=bias)
    torch.cuda.synchronize()
    lat, mem = kind == 0, kind == 1
    assert torch.equal(gated.cpu()[lat], plain.cpu()[lat])
    assert torch.equal(gated.cpu()[mem], h0.cpu()[mem])
    assert _lib.device_error() == 0


def test_gemm_epilogues(cuda):
    from sa3_b200 import ops, _lib

    g = _gen(11)
    B, T, D, K = 2, 200, 512, 256
    M = B * T
    a = torch.randn(M, K, generator=g).bfloat16()
    w = (torch.randn(D, K, generator=g) * 0.05).bfloat16()
    res = torch.randn(M, D, generator=g).bfloat16()
    gate = torch.randn(B, D, generator=g)
    h = a.float() @ w.float().T
    ad, wd = a.to(cuda), w.to(cuda)

    # gated residual: res + h * sigmoid(1 - gate[b])
    out = res.clone().to(cuda)
    ops.gemm(ad, wd, out, kind=_lib.EPI_GATED_RESIDUAL, residual=out, gate=gate.to(cuda), rows_per_batch=T)
    ref = orf.gate_residual(h.view(B, T, D), gate[:, None, :], res.float().view(B, T, D)).view(M, D)
    assert max_rel(out, ref) < 1e-2

    # plain residual and silu
    out = ops.gemm(ad, wd, res.clone().to(cuda), kind=_lib.EPI_RESIDUAL, residual=res.to(cuda))
    assert max_rel(out, h + res.float()) < 1e-2
    out = ops.gemm(ad, wd, kind=_lib.EPI_SILU)
    assert max_rel(out, orf.silu(h)) < 1e-2

    # swiglu with the interleaved [x | gate] blocks of 128 rows
    inner = 256
    w1 = (torch.randn(2 * inner, K, generator=g) * 0.05).bfloat16()
    b1 = torch.randn(2 * inner, generator=g)
    from sa3_b200.quant import interleave_swiglu_rows
    w1i, b1i = interleave_swiglu_rows(w1, b1)
    amax = torch.zeros(1, device=cuda)
    out = ops.gemm(ad, w1i.to(cuda), bias=b1i.to(cuda), kind=_lib.EPI_SWIGLU, amax_out=amax)
    ref = orf.swiglu(a.float() @ w1.float().T + b1)
    assert max_rel(out, ref) < 1e-2
    torch.cuda.synchronize()
    assert abs(amax.item() - out.float().abs().max().item()) == 0.0

    # left-pad row remap (local conditioning add): x[b, 64 + t] += y[b, t]
    Tin, Nout = 150, 214
    xin = torch.randn(B * Tin, K, generator=g).bfloat16()
    big = torch.randn(B * Nout, D, generator=g).bfloat16()
    outd = big.clone().to(cuda)
    ops.gemm(xin.to(cuda), wd, outd, kind=_lib.EPI_RESIDUAL, residual=outd, seg=(Tin, Nout, 64))
    ref = big.float().clone().view(B, Nout, D)
    ref[:, 64:, :] += (xin.float() @ w.float().T).view(B, Tin, D)
    assert max_rel(outd, ref.view(-1, D)) < 1e-2


def test_gemm_fp32_residual_stream(cuda):
    from sa3_b200 import ops, _lib

    g = _gen(21)
    B, T, D, K = 2, 190, 256, 192
    a = torch.randn(B * T, K, generator=g).bfloat16()
    w = (torch.randn(D, K, generator=g) * 0.05).bfloat16()
    res = torch.randn(B * T, D, generator=g)
    gate = torch.randn(B, D, generator=g)
    h = a.float() @ w.float().T
    out = res.clone().to(cuda)
    ops.gemm(a.to(cuda), w.to(cuda), out, kind=_lib.EPI_GATED_RESIDUAL, residual=out, gate=gate.to(cuda),
             rows_per_batch=T)
    ref = orf.gate_residual(h.view(B, T, D), gate[:, None, :], res.view(B, T, D)).view(-1, D)
    assert (out.cpu() - ref).abs().max().item() < 1e-4 * ref.abs().max().item() + 1e-5
    out32 = ops.gemm(a.to(cuda), w.to(cuda), torch.empty(B * T, D, device=cuda))
    assert (out32.cpu() - h).abs().max().item() < 1e-4 * h.abs().max().item()


def test_convert_and_fp32_norm_input(cuda):
    from sa3_b200 import ops

    g = _gen(23)
    x = torch.randn(301, 1536, generator=g)
    xb = ops.convert(x.to(cuda), torch.empty(301, 1536, device=cuda, dtype=torch.bfloat16))
    assert torch.equal(xb.cpu(), x.bfloat16())
    back = ops.convert(xb, torch.empty(301, 1536, device=cuda))
    assert torch.equal(back.cpu(), x.bfloat16().float())
    gamma = 1 + 0.1 * torch.randn(1536, generator=g)
    y = ops.rmsnorm_modulate(x.to(cuda), gamma.to(cuda), 1e-5)
    assert max_rel(y, orf.rms_norm(x, gamma, 1e-5)) < 1e-2
    # the fp16 stream: fp32 -> fp16 (round to nearest), fp16 -> bf16 with a row gather, fp16 -> fp32
    xh = ops.convert(x.to(cuda), torch.empty(301, 1536, device=cuda, dtype=torch.float16))
    assert torch.equal(xh.cpu(), x.half())
    rows = torch.randperm(301, generator=g)[:150].to(torch.int32)
    hb = ops.convert(xh, torch.empty(150, 1536, device=cuda, dtype=torch.bfloat16), src_rows=rows.to(cuda))
    assert torch.equal(hb.cpu(), x.half()[rows.long()].bfloat16())
    assert torch.equal(ops.convert(xh, torch.empty(301, 1536, device=cuda)).cpu(), x.half().float())


# ----------------------------------------------------------------------------- glue
def test_rmsnorm_modulate(cuda):
    from sa3_b200 import ops

    g = _gen(3)
    B, T, D = 2, 333, 1536
    x = torch.randn(B * T, D, generator=g).bfloat16()
    gamma = 1 + 0.1 * torch.randn(D, generator=g)
    mod = torch.randn(B, 6 * D, generator=g) * 0.3
    ref = orf.modulate(orf.rms_norm(x.float().view(B, T, D), gamma, 1e-5), mod[:, None, 0:D], mod[:, None, D:2 * D])
    ref = ref.reshape(B * T, D)
    out = ops.rmsnorm_modulate(x.to(cuda), gamma.to(cuda), 1e-5, mod=mod.to(cuda), scale_off=0, shift_off=D,
                               rows_per_batch=T)
    assert max_rel(out, ref) < 1e-2
    amax = torch.zeros(1, device=cuda)
    ops.rmsnorm_modulate(x.to(cuda), gamma.to(cuda), 1e-5, mod=mod.to(cuda), scale_off=0, shift_off=D,
                         rows_per_batch=T, amax_only=amax)
    torch.cuda.synchronize()
    assert abs(amax.item() - ref.abs().max().item()) / ref.abs().max().item() < 1e-5
    s = torch.zeros(1, device=cuda)
    q = ops.rmsnorm_modulate(x.to(cuda), gamma.to(cuda), 1e-5, mod=mod.to(cuda), scale_off=0, shift_off=D,
                             rows_per_batch=T, out_dtype=torch.float8_e4m3fn, quant_amax=amax, scale_out=s)
    deq = q.float().cpu() * s.cpu()
    assert rel_fro(deq, oq.fake_quant_act(ref)) < 2e-2
    # plain RMSNorm (no modulation)
    out = ops.rmsnorm_modulate(x.to(cuda), gamma.to(cuda), 1e-5)
    assert max_rel(out, orf.rms_norm(x.float(), gamma, 1e-5)) < 1e-2


@pytest.mark.parametrize("stream", [torch.float32, torch.float16])
@pytest.mark.parametrize("layout", ["two_batches", "three_batches", "row_batch", "no_mod"])
def test_rmsnorm_modulate_fp32_stream(cuda, layout, stream):
    """RMSNorm + modulate of the residual stream, fp32 or fp16 (the direct-load kernel): the per-block coefficient
    table (<= 2 CFG batches), the per-row global path (3 batches, or a row -> batch table as in packed
    variable-length batches) and plain RMSNorm; max|y| pass, e4m3 and bf16 outputs vs the oracle on the same
    (fp16-rounded) stream values."""
    from sa3_b200 import ops

    g = _gen(41)
    D = 1536
    lens = {"two_batches": [333, 333], "three_batches": [200, 200, 200], "row_batch": [120, 301, 77],
            "no_mod": [250]}[layout]
    B, M = len(lens), sum(lens)
    x = (torch.randn(M, D, generator=g) * 3).to(stream).float()
    gamma = 1 + 0.1 * torch.randn(D, generator=g)
    mod = torch.randn(B, 6 * D, generator=g) * 0.3
    bidx = torch.repeat_interleave(torch.arange(B), torch.tensor(lens))
    kw = {}
    if layout == "no_mod":
        ref = orf.rms_norm(x, gamma, 1e-5)
    else:
        ref = orf.modulate(orf.rms_norm(x, gamma, 1e-5), mod[bidx, 0:D], mod[bidx, D:2 * D])
        kw = dict(mod=mod.to(cuda), scale_off=0, shift_off=D)
        if layout == "row_batch":
            kw["row_batch"] = bidx.to(torch.int32).to(cuda)
        else:
            kw["rows_per_batch"] = lens[0]
    xd, gd = x.to(stream).to(cuda), gamma.to(cuda)
    out = ops.rmsnorm_modulate(xd, gd, 1e-5, **kw)
    assert max_rel(out, ref) < 1e-2
    amax = torch.zeros(1, device=cuda)
    ops.rmsnorm_modulate(xd, gd, 1e-5, amax_only=amax, **kw)
    torch.cuda.synchronize()
    assert abs(amax.item() - ref.abs().max().item()) / ref.abs().max().item() < 1e-5
    s = torch.zeros(1, device=cuda)
    q = ops.rmsnorm_modulate(xd, gd, 1e-5, out_dtype=torch.float8_e4m3fn, quant_amax=amax, scale_out=s, **kw)
    assert rel_fro(q.float().cpu() * s.cpu(), oq.fake_quant_act(ref)) < 2e-2
    # the two passes with a per-row 1/rms buffer (the block's FP8 norm): the max|y| pass stores it, the write
    # pass reads it (an elementwise kernel where the batches allow); outputs are the same bits as without it
    rr = torch.full((M,), float("nan"), device=cuda)
    amax2, s2 = torch.zeros(1, device=cuda), torch.zeros(1, device=cuda)
    ops.rmsnorm_modulate(xd, gd, 1e-5, amax_only=amax2, row_r=rr, **kw)
    q2 = ops.rmsnorm_modulate(xd, gd, 1e-5, out_dtype=torch.float8_e4m3fn, quant_amax=amax2, scale_out=s2, row_r=rr,
                              **kw)
    out2 = ops.rmsnorm_modulate(xd, gd, 1e-5, row_r=rr, **kw)
    torch.cuda.synchronize()
    assert amax2.item() == amax.item() and s2.item() == s.item()
    assert torch.equal(q2.view(torch.uint8), q.view(torch.uint8))
    assert torch.equal(out2, out)
    assert bool(torch.isfinite(rr).all())
    # both passes as one launch (grid barrier) where the kernel serves the shape, else the two passes: same
    # bytes, twice in a row on the same barrier words
    bar = torch.zeros(2, device=cuda, dtype=torch.int32)
    for _ in range(2):
        amax3, s3 = torch.zeros(1, device=cuda), torch.zeros(1, device=cuda)
        q3 = torch.empty_like(q)
        ops.rmsnorm_quant_fused(xd, gd, 1e-5, out=q3, amax=amax3, row_r=torch.empty(M, device=cuda), barrier=bar,
                                scale_out=s3, **kw)
        torch.cuda.synchronize()
        assert amax3.item() == amax.item() and s3.item() == s.item()
        assert torch.equal(q3.view(torch.uint8), q.view(torch.uint8))
    assert bar[0].item() == 0


def test_qk_norm_rope(cuda):
    from sa3_b200 import ops

    g = _gen(5)
    B, T, H = 2, 300, 4
    D = H * 64
    buf = torch.randn(B * T, 5 * D, generator=g).bfloat16()
    gq = 1 + 0.1 * torch.randn(64, generator=g)
    gk = 1 + 0.1 * torch.randn(64, generator=g)
    table = ops.rope_table(T, device=cuda)
    out = buf.clone().to(cuda)
    ops.qk_norm_rope(out, H, [0, D, 3 * D, 4 * D], [gq.to(cuda), gk.to(cuda), gq.to(cuda), gk.to(cuda)],
                     [True] * 4, 1e-6, table, rows_per_batch=T)
    freqs = orf.rotary_freqs(T, 32)
    x = buf.float().view(B, T, 5, H, 64)
    ref = x.clone()
    for part, gm in ((0, gq), (1, gk), (3, gq), (4, gk)):
        t = x[:, :, part].permute(0, 2, 1, 3)  # [B, H, T, 64]
        t = orf.apply_rotary(orf.rms_norm(t, gm, 1e-6), freqs)
        ref[:, :, part] = t.permute(0, 2, 1, 3)
    assert max_rel(out.view(B, T, 5, H, 64)[:, :, [0, 1, 3, 4]], ref[:, :, [0, 1, 3, 4]]) < 1e-2
    # v untouched
    assert torch.equal(out.view(B, T, 5, H, 64)[:, :, 2].cpu(), buf.view(B, T, 5, H, 64)[:, :, 2])


# ----------------------------------------------------------------------------- attention
def _heads(x, B, N, H):
    return x.float().cpu().view(B, N, H, 64).permute(0, 2, 1, 3)


@pytest.mark.parametrize("B,N,H,w", [(1, 646, 16, 256), (2, 300, 4, 17), (1, 130, 2, 0), (1, 1000, 2, -1)])
def test_attention_window(cuda, B, N, H, w):
    from sa3_b200 import ops

    g = _gen(N + H)
    D = H * 64
    qkv = torch.randn(B * N, 3 * D, generator=g).bfloat16().to(cuda)
    q, k, v = qkv[:, :D], qkv[:, D:2 * D], qkv[:, 2 * D:]
    out = ops.attention(q, k, v, heads=H, batch=B, max_seqlen_q=N, max_seqlen_k=N, window=(w, w))
    ref = orf.attention(_heads(q, B, N, H), _heads(k, B, N, H), _heads(v, B, N, H), w, w)
    assert max_rel(_heads(out, B, N, H), ref) < 1e-2


def test_attention_differential(cuda):
    from sa3_b200 import ops

    g = _gen(9)
    B, N, H, w = 2, 700, 3, 256
    D = H * 64
    qkv = torch.randn(B * N, 5 * D, generator=g).bfloat16().to(cuda)
    q, k, v, q2, k2 = (qkv[:, i * D:(i + 1) * D] for i in range(5))
    out = ops.attention(q, k, v, q2=q2, k2=k2, heads=H, batch=B, max_seqlen_q=N, max_seqlen_k=N, window=(w, w))
    hh = lambda t: _heads(t, B, N, H)  # noqa: E731
    ref = orf.differential_attention(hh(q), hh(k), hh(v), hh(q2), hh(k2), w, w)
    assert max_rel(hh(out), ref) < 1e-2


@pytest.mark.parametrize("diff", [False, True])
def test_attention_amax_out(cuda, diff):
    """amax_out (the max |out| that feeds the next FP8 quantisation) equals max |out| over the stored 16-bit
    output exactly, accumulated over earlier contents of the slot (never lowered)."""
    from sa3_b200 import ops

    g = _gen(31)
    B, N, H, w = 2, 700, 3, 256
    D = H * 64
    qkv = torch.randn(B * N, 5 * D, generator=g).bfloat16().to(cuda)
    q, k, v, q2, k2 = (qkv[:, i * D:(i + 1) * D] for i in range(5))
    kw = dict(q2=q2, k2=k2) if diff else {}
    am = torch.zeros(1, device=cuda)
    out = ops.attention(q, k, v, heads=H, batch=B, max_seqlen_q=N, max_seqlen_k=N, window=(w, w), amax_out=am, **kw)
    torch.cuda.synchronize()
    assert am.item() == out.float().abs().max().item()
    big = torch.full((1,), 1e3, device=cuda)
    ops.attention(q, k, v, heads=H, batch=B, max_seqlen_q=N, max_seqlen_k=N, window=(w, w), amax_out=big, **kw)
    torch.cuda.synchronize()
    assert big.item() == 1e3


@pytest.mark.parametrize("w,diff", [(-1, False), (256, False), (256, True)])
def test_attention_growing_scores(cuda, w, diff):
    """Key norms grow along the sequence, so a row's maximum score keeps rising across key tiles by far
    more than 2^8: the kernel has to move its reference maximum and rescale O (in TMEM) mid-row."""
    from sa3_b200 import ops

    g = _gen(21)
    B, N, H = 1, 1000, 2
    D = H * 64
    ramp = (0.5 + 6.0 * torch.arange(N) / N).view(N, 1)
    q = torch.randn(B * N, D, generator=g)
    k = torch.randn(B * N, D, generator=g) * ramp
    v = torch.randn(B * N, D, generator=g)
    q2 = torch.randn(B * N, D, generator=g)
    k2 = torch.randn(B * N, D, generator=g) * ramp
    q, k, v, q2, k2 = (t.bfloat16().to(cuda) for t in (q, k, v, q2, k2))
    hh = lambda t: _heads(t, B, N, H)  # noqa: E731
    if diff:
        out = ops.attention(q, k, v, q2=q2, k2=k2, heads=H, batch=B, max_seqlen_q=N, max_seqlen_k=N, window=(w, w))
        ref = orf.differential_attention(hh(q), hh(k), hh(v), hh(q2), hh(k2), w, w)
    else:
        out = ops.attention(q, k, v, heads=H, batch=B, max_seqlen_q=N, max_seqlen_k=N, window=(w, w))
        ref = orf.attention(hh(q), hh(k), hh(v), w, w)
    assert max_rel(hh(out), ref) < 1e-2


def test_attention_cross_full(cuda):
    from sa3_b200 import ops

    g = _gen(13)
    B, Nq, Nk, H = 2, 333, 128, 4
    D = H * 64
    q = torch.randn(B * Nq, D, generator=g).bfloat16().to(cuda)
    kv = torch.randn(B * Nk, 2 * D, generator=g).bfloat16().to(cuda)
    k, v = kv[:, :D], kv[:, D:]
    out = ops.attention(q, k, v, heads=H, batch=B, max_seqlen_q=Nq, max_seqlen_k=Nk)
    ref = orf.attention(_heads(q, B, Nq, H), _heads(k, B, Nk, H), _heads(v, B, Nk, H))
    assert max_rel(_heads(out, B, Nq, H), ref) < 1e-2


def test_attention_varlen(cuda):
    from sa3_b200 import ops

    g = _gen(17)
    lens = [100, 300, 77, 513]
    H, w = 2, 64
    D = H * 64
    tot = sum(lens)
    cu = torch.tensor([0] + list(torch.tensor(lens).cumsum(0)), dtype=torch.int32)
    qkv = torch.randn(tot, 3 * D, generator=g).bfloat16().to(cuda)
    q, k, v = qkv[:, :D], qkv[:, D:2 * D], qkv[:, 2 * D:]
    out = ops.attention(q, k, v, heads=H, cu_seqlens_q=cu.to(cuda), cu_seqlens_k=cu.to(cuda),
                        max_seqlen_q=max(lens), max_seqlen_k=max(lens), window=(w, w))
    for i, L in enumerate(lens):
        s, e = int(cu[i]), int(cu[i + 1])
        hh = lambda t: _heads(t[s:e], 1, L, H)  # noqa: E731
        ref = orf.attention(hh(q), hh(k), hh(v), w, w)
        assert max_rel(hh(out), ref) < 1e-2, f"sequence {i}"


def test_no_device_error_recorded(cuda):
    from sa3_b200 import _lib

    assert _lib.device_error() == 0


@pytest.mark.parametrize("fp8", [False, True])
def test_gemm_qk_norm_rope_epilogue(cuda, fp8):
    """to_qkv GEMM with qk RMSNorm + RoPE fused into the epilogue vs oracle linear -> rms_norm -> apply_rotary."""
    from sa3_b200 import ops, _lib

    g = _gen(31)
    B, T, H, K = 2, 300, 4, 512
    D = H * 64
    x = torch.randn(B * T, K, generator=g)
    w = torch.randn(5 * D, K, generator=g) * 0.05
    gq = 1 + 0.1 * torch.randn(64, generator=g)
    gk = 1 + 0.1 * torch.randn(64, generator=g)
    table = ops.rope_table(T, device=cuda)
    if fp8:
        wq, sw = oq.quantize_weight_e4m3(w)
        xd = x.bfloat16().to(cuda)
        amax, s = torch.zeros(1, device=cuda), torch.zeros(1, device=cuda)
        ops.absmax(xd, amax)
        a = ops.quantize_e4m3(xd, amax, scale_out=s)
        y = oq.fp8_linear(x.bfloat16().float(), wq, sw)
        kw = dict(a_scale=s, b_scale=sw.to(cuda))
        bmat = wq.to(cuda)
    else:
        a = x.bfloat16().to(cuda)
        bmat = w.bfloat16().to(cuda)
        y = x.bfloat16().float() @ w.bfloat16().float().T
        kw = {}
    out = ops.gemm(a, bmat, kind=_lib.EPI_QK_NORM, rows_per_batch=T,
                   qk=dict(gammas=[gq.to(cuda), gk.to(cuda), None, gq.to(cuda), gk.to(cuda)], group_width=D,
                           rope=[True, True, False, True, True], eps=1e-6, cos_sin=table), **kw)
    freqs = orf.rotary_freqs(T, 32)
    ref = y.view(B, T, 5, H, 64).clone()
    for part, gm in ((0, gq), (1, gk), (3, gq), (4, gk)):
        t = ref[:, :, part].permute(0, 2, 1, 3)
        ref[:, :, part] = orf.apply_rotary(orf.rms_norm(t, gm, 1e-6), freqs).permute(0, 2, 1, 3)
    assert max_rel(out.view(B, T, 5, H, 64), ref) < 1e-2


@pytest.mark.parametrize("M", [256, 700])
def test_gemm_qk_norm_gamma_table(cuda, M):
    """qk-norm epilogue with a gamma table (more than 8 column groups, as for every block's cross-attention
    K/V in one GEMM): groups below the table size are RMS-normalised per 64-column head with their row of
    the table, later groups are stored as computed."""
    from sa3_b200 import ops, _lib

    g = _gen(M + 5)
    K, gw, ngroups, ntab = 256, 128, 12, 9
    N = gw * ngroups
    a = torch.randn(M, K, generator=g).bfloat16()
    w = (torch.randn(N, K, generator=g) * 0.05).bfloat16()
    bias = torch.randn(N, generator=g) * 0.1
    tab = torch.rand(ntab, 64, generator=g) + 0.5
    y = a.float() @ w.float().T + bias
    ref = y.clone()
    for c in range(0, ntab * gw, 64):
        hd = y[:, c:c + 64]
        ref[:, c:c + 64] = hd * torch.rsqrt(hd.pow(2).mean(-1, keepdim=True) + 1e-6) * tab[c // gw]
    out = ops.gemm(a.to(cuda), w.to(cuda), bias=bias.to(cuda), kind=_lib.EPI_QK_NORM,
                   qk=dict(gamma_table=tab.to(cuda), group_width=gw, eps=1e-6))
    torch.cuda.synchronize()
    assert rel_fro(out[:, :ntab * gw], ref[:, :ntab * gw]) < 1e-2
    assert rel_fro(out[:, ntab * gw:], ref[:, ntab * gw:]) < 1e-2
