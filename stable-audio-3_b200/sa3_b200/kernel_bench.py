"""Per-kernel timing at the medium DiT shapes (CUDA events, after warm-up), also used as the
bounded workload for ncu captures of a single kernel.

  PYTHONPATH=stable-audio-3_b200 python -m sa3_b200.kernel_bench [--case NAME[,NAME]|all] [--iters N]

Cases (medium: B=2 CFG halves, N = 8183 + 64 tokens, M = 16494 rows, D = 1536):
  ff1_fp8    GLU.proj    FP8 GEMM  M x 12288 x 1536, SwiGLU epilogue
  qkv_fp8    to_qkv      FP8 GEMM  M x 7680 x 1536
  qkv_fp8_qk to_qkv as in the block: qk RMSNorm + RoPE epilogue
  ff2_fp8    linear_out  FP8 GEMM  M x 1536 x 6144, gate + fp32 residual epilogue
  out_fp8    to_out      FP8 GEMM  M x 1536 x 1536, gate + fp32 residual epilogue
  ff2_fp8_f16, out_fp8_f16, local2_bf16_f16  the residual epilogues into the fp16 stream
  attn_diff  differential SWA, 24 heads, window (256, 256)
  attn_cross differential cross-attention over 128 context tokens
  norm_fp8   RMSNorm + modulate of the fp32 stream: amax pass + e4m3 write pass
  norm_fp8_f16  the same on the fp16 stream
  qknorm     qk RMSNorm + RoPE on q, k, q_diff, k_diff in place
  ff1_gptq   GLU.proj GPTQ int4 GEMM (group 128, act-order gather included separately), M = 16 x 2648
  ff1_gptq_dense  the same layer on the large-batch path: dequantise once (original channel order) + bf16 GEMM
  samel_w17_N  SAME-L plugin operator (differential, window 17, 2 x 24 heads) at N tokens (200, 1836, 5000, 21964),
             CUDA-graph timed
The medium cases' operands exceed the 126 MB L2; the samel cases are the plugin's own small shapes (L2-resident).
"""
from __future__ import annotations

import argparse
import json

import torch

from . import _lib, ops
from .quant import interleave_swiglu_rows, quantize_weight_e4m3

B, L, NM, D, H = 2, 8183, 64, 1536, 24
N_GPTQ = 2584 + 64
N = L + NM
M = B * N


def _time(fn, iters: int, warm: int = 3) -> float:
    for _ in range(warm):
        fn()
    torch.cuda.synchronize()
    s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    s.record()
    for _ in range(iters):
        fn()
    e.record()
    torch.cuda.synchronize()
    return s.elapsed_time(e) / iters


def _time_graph(fn, reps: int, iters: int) -> float:
    """ms per call of `reps` calls captured in one CUDA graph (no host launch cost in the timed region)."""
    s = torch.cuda.Stream()
    with torch.cuda.stream(s):
        for _ in range(3):
            fn()
    torch.cuda.synchronize()
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g, stream=s):
        for _ in range(reps):
            fn()
    g.replay()
    torch.cuda.synchronize()
    a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    a.record()
    for _ in range(iters):
        g.replay()
    b.record()
    torch.cuda.synchronize()
    return a.elapsed_time(b) / (iters * reps)


def _fp8_weight(n, k, dev, g):
    wq, s = quantize_weight_e4m3(torch.randn(n, k, generator=g) * 0.02)
    return wq, s


def case(name: str, iters: int) -> dict:
    dev = torch.device("cuda")
    g = torch.Generator().manual_seed(0)
    one = torch.ones(1, device=dev)
    if name in ("ff1_fp8", "qkv_fp8", "qkv_fp8_qk", "ff2_fp8", "out_fp8", "ff2_fp8_f16", "out_fp8_f16"):
        # _f16: the gated residual goes into the fp16 stream (TMA reduce-add in fp16) instead of the fp32 one
        stream = torch.float16 if name.endswith("_f16") else torch.float32
        n, k = {"ff1_fp8": (12288, 1536), "qkv_fp8": (7680, 1536), "qkv_fp8_qk": (7680, 1536), "ff2_fp8": (1536, 6144),
                "out_fp8": (1536, 1536)}[name.replace("_f16", "")]
        a = torch.randn(M, k, device=dev).to(torch.float8_e4m3fn)
        wq, s = _fp8_weight(n, k, dev, g)
        if name == "ff1_fp8":
            w8, s = interleave_swiglu_rows(wq.view(torch.uint8), s)
            wq = w8.view(torch.float8_e4m3fn)
        wq, s = wq.to(dev), s.to(dev)
        if name == "ff1_fp8":
            out = torch.empty(M, n // 2, device=dev, dtype=torch.bfloat16)
            fn = lambda: ops.gemm(a, wq, out, a_scale=one, b_scale=s, kind=_lib.EPI_SWIGLU)  # noqa: E731
        elif name == "qkv_fp8":
            out = torch.empty(M, n, device=dev, dtype=torch.bfloat16)
            fn = lambda: ops.gemm(a, wq, out, a_scale=one, b_scale=s)  # noqa: E731
        elif name == "qkv_fp8_qk":
            # as in the DiT block: qk RMSNorm + RoPE of q | k | v | q_diff | k_diff in the epilogue
            out = torch.empty(M, n, device=dev, dtype=torch.bfloat16)
            gq, gk = torch.rand(64, device=dev) + 0.5, torch.rand(64, device=dev) + 0.5
            cs = ops.rope_table(N, device=dev)
            pos = (torch.arange(M, device=dev) % N).to(torch.int32)
            qk = dict(gammas=[gq, gk, None, gq, gk], group_width=D, rope=[True, True, False, True, True], eps=1e-6,
                      cos_sin=cs, row_pos=pos)
            fn = lambda: ops.gemm(a, wq, out, a_scale=one, b_scale=s, kind=_lib.EPI_QK_NORM, qk=qk)  # noqa: E731
        else:
            h = torch.randn(M, n, device=dev).to(stream)
            gate = torch.randn(B, n, device=dev)
            fn = lambda: ops.gemm(a, wq, h, a_scale=one, b_scale=s, kind=_lib.EPI_GATED_RESIDUAL,  # noqa: E731
                                  residual=h, gate=gate, rows_per_batch=N)
        ms = _time(fn, iters)
        return {"case": name, "ms": ms, "tflops": 2.0 * M * n * k / ms / 1e9}
    if name in ("out_fp8_store", "local2_bf16", "local2_bf16_f16", "local2_bf16_store", "local1_bf16"):
        # epilogue cost: the same M x 1536 x 1536 shapes with a plain bf16 store vs the fp32 residual
        k = 264 if name == "local1_bf16" else 1536
        n = 1536
        if name == "out_fp8_store":
            a = torch.randn(M, k, device=dev).to(torch.float8_e4m3fn)
            wq, s = _fp8_weight(n, k, dev, g)
            wq, s = wq.to(dev), s.to(dev)
            out = torch.empty(M, n, device=dev, dtype=torch.bfloat16)
            fn = lambda: ops.gemm(a, wq, out, a_scale=one, b_scale=s)  # noqa: E731
        else:
            a = torch.randn(M, k, device=dev).bfloat16()
            w = (torch.randn(n, k, generator=g) * 0.02).bfloat16().to(dev)
            if name in ("local2_bf16", "local2_bf16_f16"):
                h = torch.randn(M, n, device=dev).to(torch.float16 if name.endswith("_f16") else torch.float32)
                fn = lambda: ops.gemm(a, w, h, kind=_lib.EPI_RESIDUAL, residual=h)  # noqa: E731
            else:
                out = torch.empty(M, n, device=dev, dtype=torch.bfloat16)
                kind = _lib.EPI_SILU if name == "local1_bf16" else _lib.EPI_STORE
                fn = lambda: ops.gemm(a, w, out, kind=kind)  # noqa: E731
        ms = _time(fn, iters)
        return {"case": name, "ms": ms, "tflops": 2.0 * M * n * k / ms / 1e9}
    if name == "attn_diff":
        qkv = torch.randn(M, 5 * D, device=dev).bfloat16()
        q, k, v, q2, k2 = (qkv[:, i * D:(i + 1) * D] for i in range(5))
        am = torch.zeros(1, device=dev)  # max|out| for the FP8 quantisation that follows, as in the block
        fn = lambda: ops.attention(q, k, v, q2=q2, k2=k2, heads=H, batch=B, max_seqlen_q=N,  # noqa: E731
                                   max_seqlen_k=N, window=(256, 256), amax_out=am)
        pairs = N * 513 - 256 * 257
        ms = _time(fn, iters)
        return {"case": name, "ms": ms, "tflops": 4.0 * 64 * pairs * H * 2 * B / ms / 1e9}
    if name == "attn_cross":
        q = torch.randn(M, 2 * D, device=dev).bfloat16()
        kv = torch.randn(B * 128, 3 * D, device=dev).bfloat16()
        am = torch.zeros(1, device=dev)
        fn = lambda: ops.attention(q[:, :D], kv[:, :D], kv[:, 2 * D:], q2=q[:, D:], k2=kv[:, D:2 * D],  # noqa
                                   heads=H, batch=B, max_seqlen_q=N, max_seqlen_k=128, amax_out=am)
        ms = _time(fn, iters)
        return {"case": name, "ms": ms, "tflops": 4.0 * 64 * N * 128 * H * 2 * B / ms / 1e9}
    if name.startswith("samel_w17_"):
        # SAME-L plugin operator (window 17, 48 stacked heads = 2 x 24) at the reference kernel's self-test
        # lengths; each call is a few microseconds, so 20 calls are replayed from one CUDA graph
        n = int(name.rsplit("_", 1)[1])
        qb, kb, vb = (torch.randn(1, n, 48, 64, device=dev).bfloat16() for _ in range(3))
        out = torch.empty(1, n, 24, 64, device=dev, dtype=torch.bfloat16)
        fn = lambda: ops.diff_attn_swa(qb, kb, vb, 24, 17, out)  # noqa: E731
        ms = _time_graph(fn, 20, max(iters // 4, 3))
        pairs = n * 35 - 17 * 18
        return {"case": name, "ms": ms, "us": ms * 1e3, "tflops": 4.0 * 64 * pairs * 48 / ms / 1e9}
    if name == "ff1_gptq":
        from .gptq import random_layer
        Mg = 16 * N_GPTQ
        lay = random_layer(12288, 1536, 128, g, dev)
        a = torch.randn(Mg, 1536, device=dev).bfloat16()
        out = torch.empty(Mg, 6144, device=dev, dtype=torch.bfloat16)
        xp = torch.empty_like(a)
        ms_perm = _time(lambda: ops.permute_cols(a, lay["perm"], xp), iters)
        ms = _time(lambda: ops.gptq_gemm(xp, lay["qw"], lay["sz"], 12288, out, kind=_lib.EPI_SWIGLU), iters)
        return {"case": name, "ms": ms, "tflops": 2.0 * Mg * 12288 * 1536 / ms / 1e9, "gather_ms": ms_perm}
    if name == "ff1_gptq_dense":
        # the large-batch GPTQ path: dequantise the int4 weight once (original channel order, bf16), then the
        # 2-SM bf16 GEMM with the SwiGLU epilogue on the unpermuted activations
        from .gptq import random_layer
        Mg = 16 * N_GPTQ
        lay = random_layer(12288, 1536, 128, g, dev)
        a = torch.randn(Mg, 1536, device=dev).bfloat16()
        out = torch.empty(Mg, 6144, device=dev, dtype=torch.bfloat16)
        wd = torch.empty(12288, 1536, device=dev, dtype=torch.bfloat16)
        ms_dq = _time(lambda: ops.gptq_dequant_orig(lay["qw"], lay["sz"], lay["inv_perm"], 12288, 1536, 128, wd), iters)
        ms_mm = _time(lambda: ops.gemm(a, wd, out, kind=_lib.EPI_SWIGLU), iters)

        def fn():
            ops.gptq_dequant_orig(lay["qw"], lay["sz"], lay["inv_perm"], 12288, 1536, 128, wd)
            ops.gemm(a, wd, out, kind=_lib.EPI_SWIGLU)
        ms = _time(fn, iters)
        return {"case": name, "ms": ms, "tflops": 2.0 * Mg * 12288 * 1536 / ms / 1e9, "dequant_ms": ms_dq,
                "dequant_GBps": 12288 * 1536 * 2.5 / ms_dq / 1e6, "gemm_ms": ms_mm}
    if name in ("norm_fp8", "norm_fp8_f16"):
        # RMSNorm + modulate + FP8 quantisation of the residual stream (fp32, or the fp16 stream for _f16)
        x = torch.randn(M, D, device=dev).to(torch.float16 if name.endswith("f16") else torch.float32)
        gam = torch.ones(D, device=dev)
        mod = torch.randn(B, 6 * D, device=dev) * 0.1
        am = torch.zeros(1, device=dev)
        sc = torch.zeros(1, device=dev)
        out = torch.empty(M, D, device=dev, dtype=torch.float8_e4m3fn)
        rr = torch.empty(M, device=dev)  # per-row 1/rms from the max|y| pass, as in the block

        def fn():
            ops.rmsnorm_modulate(x, gam, 1e-5, mod=mod, scale_off=0, shift_off=D, rows_per_batch=N, amax_only=am,
                                 row_r=rr)
            ops.rmsnorm_modulate(x, gam, 1e-5, mod=mod, scale_off=0, shift_off=D, rows_per_batch=N, out=out,
                                 quant_amax=am, scale_out=sc, row_r=rr)
        ms = _time(fn, iters)
        ms_amax = _time(lambda: ops.rmsnorm_modulate(x, gam, 1e-5, mod=mod, scale_off=0, shift_off=D,  # noqa: E731
                                                     rows_per_batch=N, amax_only=am, row_r=rr), iters)
        ms_write = _time(lambda: ops.rmsnorm_modulate(x, gam, 1e-5, mod=mod, scale_off=0, shift_off=D,  # noqa: E731
                                                      rows_per_batch=N, out=out, quant_amax=am, scale_out=sc,
                                                      row_r=rr), iters)
        bar = torch.zeros(2, device=dev, dtype=torch.int32)
        ms_fused = _time(lambda: ops.rmsnorm_quant_fused(x, gam, 1e-5, out=out, amax=am, row_r=rr,  # noqa: E731
                                                         barrier=bar, scale_out=sc, mod=mod, scale_off=0,
                                                         shift_off=D, rows_per_batch=N), iters)
        return {"case": name, "ms": ms, "GBps": (2 * M * D * x.element_size() + M * D) / ms / 1e6,
                "ms_amax_pass": ms_amax, "ms_write_pass": ms_write, "ms_one_launch": ms_fused}
    if name in ("quant_attn", "quant_ff"):
        # activation quantisation with the scale from a producer's max|x|: M x 1536 (attention output) and
        # M x 6144 (FF hidden)
        c = D if name == "quant_attn" else 4 * D
        x = torch.randn(M, c, device=dev).bfloat16()
        am = x.float().abs().max().reshape(1)
        sc = torch.zeros(1, device=dev)
        out = torch.empty(M, c, device=dev, dtype=torch.float8_e4m3fn)
        fn = lambda: ops.quantize_e4m3(x, am, out=out, scale_out=sc)  # noqa: E731
        ms = _time(fn, iters)
        return {"case": name, "ms": ms, "GBps": 3 * M * c / ms / 1e6}
    if name == "qknorm":
        qkv = torch.randn(M, 5 * D, device=dev).bfloat16()
        gam = torch.ones(64, device=dev)
        tab = ops.rope_table(N, device=dev)
        fn = lambda: ops.qk_norm_rope(qkv, H, [0, D, 3 * D, 4 * D], [gam] * 4, [True] * 4, 1e-6, tab,  # noqa
                                      rows_per_batch=N)
        ms = _time(fn, iters)
        return {"case": name, "ms": ms, "GBps": 2 * M * 4 * D * 2 / ms / 1e6}
    raise ValueError(name)


CASES = ["ff1_fp8", "qkv_fp8", "qkv_fp8_qk", "ff2_fp8", "ff2_fp8_f16", "out_fp8", "out_fp8_f16", "out_fp8_store",
         "local2_bf16", "local2_bf16_f16", "local2_bf16_store", "local1_bf16", "attn_diff", "attn_cross", "norm_fp8",
         "norm_fp8_f16", "quant_attn", "quant_ff", "qknorm", "ff1_gptq", "ff1_gptq_dense", "samel_w17_200",
         "samel_w17_1836", "samel_w17_5000", "samel_w17_21964"]


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--case", default="all")
    ap.add_argument("--iters", type=int, default=20)
    args = ap.parse_args()
    names = CASES if args.case == "all" else args.case.split(",")
    for n in names:
        print(json.dumps(case(n, args.iters)), flush=True)
    print(json.dumps({"device_error": _lib.device_error()}))


if __name__ == "__main__":
    main()
