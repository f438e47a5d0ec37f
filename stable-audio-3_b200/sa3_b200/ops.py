"""Torch-facing wrappers over the C ABI (device memory and streams come from torch).

Each function validates its tensors, passes raw pointers, sizes and the
current CUDA stream to ``libsa3b200.so``, and raises RuntimeError on any
non-zero status. Nothing here computes on the CPU: a CPU tensor is an error.
"""
from __future__ import annotations

import ctypes
import math
from typing import Optional, Sequence

import torch

from . import _lib
from ._lib import Epilogue

E4M3_MAX = 448.0

# Number of kernel launches issued through the C ABI by this process (one per call).
LAUNCHES = 0


def _count():
    global LAUNCHES
    LAUNCHES += 1


def _stream() -> int:
    return torch.cuda.current_stream().cuda_stream


def _ptr(t: Optional[torch.Tensor]) -> Optional[int]:
    return None if t is None else t.data_ptr()


def _need_cuda(*ts: Optional[torch.Tensor]) -> None:
    for t in ts:
        if t is not None and not t.is_cuda:
            raise RuntimeError("sa3_b200 ops run on CUDA tensors only (no CPU path)")


def _row_stride(t: torch.Tensor) -> int:
    if t.dim() != 2 or t.stride(1) != 1:
        raise RuntimeError(f"expected a 2-D row-major view, got shape {tuple(t.shape)} strides {t.stride()}")
    return t.stride(0)


def _dt(t: torch.Tensor) -> int:
    if t.dtype == torch.bfloat16:
        return _lib.DT_BF16
    if t.dtype == torch.float8_e4m3fn:
        return _lib.DT_E4M3
    if t.dtype == torch.float16:
        return _lib.DT_F16
    if t.dtype == torch.float32:
        return _lib.DT_F32
    raise RuntimeError(f"unsupported dtype {t.dtype}")


# ---------------------------------------------------------------------- GEMM
def _epilogue(kind, bias, residual, gate, rows_per_batch, row_batch, amax_out, seg, qk, out,
              out_row_map=None) -> Epilogue:
    epi = Epilogue()
    epi.kind = kind
    epi.bias = _ptr(bias)
    epi.residual = _ptr(residual)
    epi.ld_residual = _row_stride(residual) if residual is not None else 0
    epi.gate = _ptr(gate)
    epi.ld_gate = _row_stride(gate) if gate is not None else 0
    epi.rows_per_batch = rows_per_batch
    epi.row_batch = _ptr(row_batch)
    epi.amax_out = _ptr(amax_out)
    if seg is not None:
        epi.seg_in, epi.seg_out, epi.seg_offset = seg
    epi.c_f32 = 1 if out.dtype == torch.float32 else 0
    epi.c_f16 = 1 if out.dtype == torch.float16 else 0
    epi.out_row_map = _ptr(out_row_map)
    if qk is not None:
        gams = list(qk.get("gammas", []))
        _need_cuda(*[g for g in gams if g is not None], qk.get("cos_sin"), qk.get("row_pos"), qk.get("gamma_table"))
        if len(gams) > 8:
            raise RuntimeError("more than 8 qk groups: pass gamma_table")
        for i, gm in enumerate(gams):
            epi.qk_gamma[i] = _ptr(gm)
        tab = qk.get("gamma_table")
        if tab is not None:
            if tab.dtype != torch.float32 or tab.dim() != 2 or tab.shape[1] != 64 or not tab.is_contiguous():
                raise RuntimeError("gamma_table must be contiguous float32 [groups, 64]")
            epi.qk_gamma_table = _ptr(tab)
            epi.qk_table_groups = int(tab.shape[0])
        epi.qk_group_width = int(qk["group_width"])
        epi.qk_rope_mask = sum(1 << i for i, r in enumerate(qk.get("rope", [])) if r)
        epi.qk_eps = float(qk.get("eps", 1e-6))
        cs = qk.get("cos_sin")
        epi.cos_sin = _ptr(cs)
        epi.max_pos = cs.shape[0] if cs is not None else 0
        epi.row_pos = _ptr(qk.get("row_pos"))
    return epi


def gemm(a: torch.Tensor, b: torch.Tensor, out: Optional[torch.Tensor] = None, *, a_scale=None, b_scale=None,
         bias=None, kind: int = _lib.EPI_STORE, residual=None, gate=None, rows_per_batch: int = 0,
         row_batch=None, amax_out=None, seg=None, qk=None, out_row_map=None) -> torch.Tensor:
    """out = epilogue(a @ b.T * a_scale * b_scale + bias); a [M,K], b [N,K] (K-major), bf16 or e4m3.

    qk (for kind EPI_QK_NORM): dict(gammas=[per column group: fp32 [64] or None], group_width=int,
    rope=[bool per group], eps=float, cos_sin=fp32 [max_pos, 32] or None, row_pos=int32 [M] or None),
    or for more than 8 groups dict(gamma_table=fp32 [G, 64], group_width=int, eps=float): groups < G are
    normalised with their table row, later groups are stored as computed (no rotary embedding).
    """
    _need_cuda(a, b, out, a_scale, b_scale, bias, residual, gate, row_batch, amax_out)
    if a.dtype != b.dtype:
        raise RuntimeError("a and b must have the same dtype")
    M, K = a.shape
    N, Kb = b.shape
    if K != Kb:
        raise RuntimeError(f"K mismatch {K} vs {Kb}")
    ncols = N // 2 if kind == _lib.EPI_SWIGLU else N
    if out is None:
        if seg is not None or out_row_map is not None:
            raise RuntimeError("row remap needs an explicit out")
        out = torch.empty(M, ncols, device=a.device, dtype=torch.bfloat16)
    if out.dtype not in (torch.bfloat16, torch.float32, torch.float16):
        raise RuntimeError("gemm output is bf16, fp32 or fp16")
    if kind == _lib.EPI_SWIGLU and out.dtype != torch.bfloat16:
        raise RuntimeError("SwiGLU epilogue writes bf16")
    if residual is not None and residual.dtype != out.dtype:
        raise RuntimeError("residual and output must share a dtype")
    for t, nm in ((a_scale, "a_scale"), (b_scale, "b_scale"), (bias, "bias"), (gate, "gate"), (amax_out, "amax")):
        if t is not None and t.dtype != torch.float32:
            raise RuntimeError(f"{nm} must be float32")
    epi = _epilogue(kind, bias, residual, gate, rows_per_batch, row_batch, amax_out, seg, qk, out, out_row_map)
    _count()
    rc = _lib.load().sa3_gemm(a.data_ptr(), b.data_ptr(), out.data_ptr(), M, N, K, _row_stride(a), _row_stride(b),
                              _row_stride(out), _dt(a), _ptr(a_scale), _ptr(b_scale), ctypes.byref(epi), _stream())
    _lib.check(rc, "sa3_gemm")
    return out


# ---------------------------------------------------------------------- glue
def rmsnorm_modulate(x: torch.Tensor, gamma: Optional[torch.Tensor], eps: float, *, mod=None, scale_off: int = 0,
                     shift_off: int = 0, rows_per_batch: int = 0, row_batch=None, out=None,
                     out_dtype=torch.bfloat16, quant_amax=None, scale_out=None, amax_only=None,
                     row_r=None) -> Optional[torch.Tensor]:
    """RMSNorm(x)*gamma*(1+scale)+shift per row; bf16 or e4m3 out, or only max|y| into `amax_only`.

    row_r (fp32 [rows], optional): the max|y| pass stores each row's 1/rms there, and a later write pass of
    the same x given the same buffer reads it instead of recomputing it (same output, one elementwise pass)."""
    _need_cuda(x, gamma, mod, row_batch, out, quant_amax, scale_out, amax_only, row_r)
    if row_r is not None and (row_r.dtype != torch.float32 or row_r.numel() < x.shape[0] or not row_r.is_contiguous()):
        raise RuntimeError("row_r must be a contiguous fp32 tensor of at least `rows` elements")
    rows, D = x.shape
    lib = _lib.load()
    if amax_only is not None:
        _count()
        rc = lib.sa3_rmsnorm_modulate(x.data_ptr(), _dt(x), None, rows, D, _row_stride(x), 0, _ptr(gamma), eps, _ptr(mod),
                                      _row_stride(mod) if mod is not None else 0, scale_off, shift_off,
                                      rows_per_batch, _ptr(row_batch), _lib.NORM_AMAX, _lib.DT_BF16, None, None,
                                      amax_only.data_ptr(), _ptr(row_r), _stream())
        _lib.check(rc, "sa3_rmsnorm_modulate(amax)")
        return None
    if out is None:
        out = torch.empty(rows, D, device=x.device, dtype=out_dtype)
    _count()
    rc = lib.sa3_rmsnorm_modulate(x.data_ptr(), _dt(x), out.data_ptr(), rows, D, _row_stride(x), _row_stride(out),
                                  _ptr(gamma), eps, _ptr(mod), _row_stride(mod) if mod is not None else 0, scale_off,
                                  shift_off, rows_per_batch, _ptr(row_batch), _lib.NORM_WRITE, _dt(out),
                                  _ptr(quant_amax), _ptr(scale_out), None, _ptr(row_r), _stream())
    _lib.check(rc, "sa3_rmsnorm_modulate")
    return out


def rmsnorm_quant_fused(x: torch.Tensor, gamma: Optional[torch.Tensor], eps: float, *, out: torch.Tensor,
                        amax: torch.Tensor, row_r: torch.Tensor, barrier: torch.Tensor, scale_out=None, mod=None,
                        scale_off: int = 0, shift_off: int = 0, rows_per_batch: int = 0, row_batch=None) -> torch.Tensor:
    """The two norm passes (max|y| into `amax`, then `out` quantised with it) as one launch where the kernel
    serves the shape (fp16 stream, D = 1536, <= 2 uniform batches), else as the two passes; same bytes either
    way. `barrier`: an int32 CUDA tensor of 2 zeros kept for the stream's later calls."""
    _need_cuda(x, gamma, mod, row_batch, out, amax, row_r, barrier, scale_out)
    rows, D = x.shape
    if row_r.dtype != torch.float32 or row_r.numel() < rows or not row_r.is_contiguous():
        raise RuntimeError("row_r must be a contiguous fp32 tensor of at least `rows` elements")
    if barrier.dtype != torch.int32 or barrier.numel() < 2 or not barrier.is_contiguous():
        raise RuntimeError("barrier must be a contiguous int32 tensor of 2 elements")
    _count()
    rc = _lib.load().sa3_rmsnorm_quant_fused(x.data_ptr(), _dt(x), out.data_ptr(), rows, D, _row_stride(x),
                                             _row_stride(out), _ptr(gamma), eps, _ptr(mod),
                                             _row_stride(mod) if mod is not None else 0, scale_off, shift_off,
                                             rows_per_batch, _ptr(row_batch), _dt(out), amax.data_ptr(),
                                             _ptr(scale_out), row_r.data_ptr(), barrier.data_ptr(), _stream())
    _lib.check(rc, "sa3_rmsnorm_quant_fused")
    return out


def quantize_e4m3(x: torch.Tensor, amax: torch.Tensor, out=None, scale_out=None) -> torch.Tensor:
    _need_cuda(x, amax, out, scale_out)
    rows, cols = x.shape
    if out is None:
        out = torch.empty(rows, cols, device=x.device, dtype=torch.float8_e4m3fn)
    _count()
    rc = _lib.load().sa3_quantize_e4m3(x.data_ptr(), out.data_ptr(), rows, cols, _row_stride(x), _row_stride(out),
                                       amax.data_ptr(), _ptr(scale_out), None, _stream())
    _lib.check(rc, "sa3_quantize_e4m3")
    return out


def absmax(x: torch.Tensor, amax_out: torch.Tensor) -> None:
    _need_cuda(x, amax_out)
    rows, cols = x.shape
    _count()
    rc = _lib.load().sa3_quantize_e4m3(x.data_ptr(), None, rows, cols, _row_stride(x), 0, None, None,
                                       amax_out.data_ptr(), _stream())
    _lib.check(rc, "sa3_quantize_e4m3(amax)")


def convert(x: torch.Tensor, out: torch.Tensor, src_rows: Optional[torch.Tensor] = None) -> torch.Tensor:
    """out = x cast between fp32, fp16 and bf16; with src_rows (int32), out[r] = x[src_rows[r]]."""
    _need_cuda(x, out, src_rows)
    rows, cols = out.shape
    _count()
    rc = _lib.load().sa3_convert(x.data_ptr(), _dt(x), out.data_ptr(), _dt(out), rows, cols, _row_stride(x),
                                 _row_stride(out), _ptr(src_rows), _stream())
    _lib.check(rc, "sa3_convert")
    return out


def qk_norm_rope(buf: torch.Tensor, heads: int, col_offsets: Sequence[int], gammas: Sequence[Optional[torch.Tensor]],
                 rope: Sequence[bool], eps: float, cos_sin: Optional[torch.Tensor] = None, rows_per_batch: int = 0,
                 row_pos: Optional[torch.Tensor] = None) -> torch.Tensor:
    """In-place per-head RMSNorm (+ partial RoPE) on column groups of a token-row buffer."""
    _need_cuda(buf, cos_sin, row_pos, *gammas)
    rows = buf.shape[0]
    n = len(col_offsets)
    offs = (ctypes.c_int * n)(*col_offsets)
    gps = (ctypes.c_void_p * n)(*[_ptr(g) for g in gammas])
    rps = (ctypes.c_int * n)(*[1 if r else 0 for r in rope])
    max_pos = cos_sin.shape[0] if cos_sin is not None else 0
    _count()
    rc = _lib.load().sa3_qk_norm_rope(buf.data_ptr(), rows, _row_stride(buf), heads, n, offs, gps, rps, eps,
                                      _ptr(cos_sin), max_pos, rows_per_batch, _ptr(row_pos), _stream())
    _lib.check(rc, "sa3_qk_norm_rope")
    return buf


def rope_table(max_pos: int, rot_dim: int = 32, base: float = 10000.0, device="cuda") -> torch.Tensor:
    """cos/sin table [max_pos, 32] as RotaryEmbedding computes it (transformer.py:239-294), in fp32."""
    inv_freq = 1.0 / (base ** (torch.arange(0, rot_dim, 2).float() / rot_dim))
    t = torch.arange(max_pos, dtype=torch.float32)
    f = torch.einsum("i,j->ij", t, inv_freq)
    return torch.cat([f.cos(), f.sin()], dim=-1).contiguous().to(device)


# ---------------------------------------------------------------------- attention
def attention(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor, *, heads: int, q2=None, k2=None, v2=None,
              cu_seqlens_q=None, cu_seqlens_k=None, batch: int = 1, max_seqlen_q: int = 0, max_seqlen_k: int = 0,
              window=(-1, -1), softmax_scale: Optional[float] = None, out=None, amax_out=None) -> torch.Tensor:
    """Windowed / full attention on token-row views (head h at columns h*64); differential if q2/k2 given.

    Without cu_seqlens the rows are `batch` sequences of max_seqlen_q (q) / max_seqlen_k (k) tokens.
    """
    _need_cuda(q, k, v, q2, k2, v2, cu_seqlens_q, cu_seqlens_k, out, amax_out)
    total_q, total_k = q.shape[0], k.shape[0]
    if out is None:
        out = torch.empty(total_q, heads * 64, device=q.device, dtype=q.dtype)
    if softmax_scale is None:
        softmax_scale = 1.0 / math.sqrt(64)
    if cu_seqlens_q is None:
        if total_q != batch * max_seqlen_q or total_k != batch * max_seqlen_k:
            raise RuntimeError("uniform attention needs rows = batch * seqlen")
        batch_n = batch
    else:
        batch_n = cu_seqlens_q.numel() - 1
        if cu_seqlens_q.dtype != torch.int32 or cu_seqlens_k.dtype != torch.int32:
            raise RuntimeError("cu_seqlens must be int32")
    wl, wr = (int(window[0]), int(window[1]))
    _count()
    rc = _lib.load().sa3_attention(q.data_ptr(), k.data_ptr(), v.data_ptr(), _ptr(q2), _ptr(k2), _ptr(v2),
                                   out.data_ptr(),
                                   _ptr(cu_seqlens_q), _ptr(cu_seqlens_k), batch_n, max_seqlen_q, max_seqlen_k,
                                   total_q, total_k, heads, 64, _row_stride(q), _row_stride(k), _row_stride(v),
                                   _row_stride(out), wl, wr, float(softmax_scale), _dt(q), _ptr(amax_out), _stream())
    _lib.check(rc, "sa3_attention")
    return out


def diff_attn_swa(q_bat: torch.Tensor, k_bat: torch.Tensor, v_bat: torch.Tensor, num_heads: int, window: int,
                  out: torch.Tensor) -> torch.Tensor:
    """SAME-L plugin operator: out[B,N,H,d] = attn(heads :H) - attn(heads H:) with window +-`window`."""
    _need_cuda(q_bat, k_bat, v_bat, out)
    B, N, H2, d = q_bat.shape
    for t in (q_bat, k_bat, v_bat, out):
        if not t.is_contiguous():
            raise RuntimeError("diff_attn_swa needs contiguous [B, N, heads, d] tensors")
    if H2 != 2 * num_heads or tuple(out.shape) != (B, N, num_heads, d):
        raise RuntimeError("q_bat must stack 2*num_heads heads and out must be [B, N, num_heads, d]")
    _count()
    rc = _lib.load().sa3_diff_attn_swa(q_bat.data_ptr(), k_bat.data_ptr(), v_bat.data_ptr(), out.data_ptr(),
                                       _dt(q_bat), B, N, num_heads, d, int(window), _stream())
    _lib.check(rc, "sa3_diff_attn_swa")
    return out


# ---------------------------------------------------------------------- GPTQ
def gptq_gemm(a: torch.Tensor, qw: torch.Tensor, sz: torch.Tensor, n: int, out: Optional[torch.Tensor] = None, *,
              group_size: int = 128, bias=None, kind: int = _lib.EPI_STORE, residual=None, gate=None,
              rows_per_batch: int = 0, row_batch=None, amax_out=None, seg=None, qk=None,
              out_row_map=None) -> torch.Tensor:
    """out = epilogue(a @ W^T) with W in the packed GPTQ layout of sa3_b200.gptq.repack; a must already hold the
    act-order-permuted input channels."""
    _need_cuda(a, qw, sz, out, bias, residual, gate, row_batch, amax_out)
    if a.dtype != torch.bfloat16:
        raise RuntimeError("GPTQ activations are bf16")
    M, K = a.shape
    ncols = n // 2 if kind == _lib.EPI_SWIGLU else n
    if out is None:
        out = torch.empty(M, ncols, device=a.device, dtype=torch.bfloat16)
    epi = _epilogue(kind, bias, residual, gate, rows_per_batch, row_batch, amax_out, seg, qk, out, out_row_map)
    _count()
    rc = _lib.load().sa3_gptq_gemm(a.data_ptr(), qw.data_ptr(), sz.data_ptr(), out.data_ptr(), M, n, K,
                                   _row_stride(a), _row_stride(out), group_size, ctypes.byref(epi), _stream())
    _lib.check(rc, "sa3_gptq_gemm")
    return out


def gptq_dequant(qw: torch.Tensor, sz: torch.Tensor, n: int, k: int, group_size: int = 128) -> torch.Tensor:
    _need_cuda(qw, sz)
    out = torch.empty(n, k, device=qw.device, dtype=torch.bfloat16)
    _count()
    rc = _lib.load().sa3_gptq_dequant(qw.data_ptr(), sz.data_ptr(), out.data_ptr(), n, k, group_size, _stream())
    _lib.check(rc, "sa3_gptq_dequant")
    return out


def gptq_dequant_orig(qw: torch.Tensor, sz: torch.Tensor, inv_perm: torch.Tensor, n: int, k: int,
                      group_size: int = 128, out: Optional[torch.Tensor] = None) -> torch.Tensor:
    """bf16 W [n, k] of a repacked GPTQ layer in the original input-channel order (the dense nn.Linear weight)."""
    _need_cuda(qw, sz, inv_perm, out)
    if inv_perm.dtype != torch.int32:
        raise RuntimeError("inv_perm must be int32")
    if out is None:
        out = torch.empty(n, k, device=qw.device, dtype=torch.bfloat16)
    if out.dtype != torch.bfloat16 or tuple(out.shape) != (n, k):
        raise RuntimeError(f"out must be bf16 [{n}, {k}]")
    _count()
    rc = _lib.load().sa3_gptq_dequant_orig(qw.data_ptr(), sz.data_ptr(), inv_perm.data_ptr(), out.data_ptr(), n, k,
                                           _row_stride(out), group_size, _stream())
    _lib.check(rc, "sa3_gptq_dequant_orig")
    return out


def permute_cols(x: torch.Tensor, perm: torch.Tensor, out: Optional[torch.Tensor] = None) -> torch.Tensor:
    _need_cuda(x, perm, out)
    rows, K = x.shape
    if out is None:
        out = torch.empty(rows, K, device=x.device, dtype=x.dtype)
    _count()
    rc = _lib.load().sa3_permute_cols(x.data_ptr(), perm.data_ptr(), out.data_ptr(), rows, K, _row_stride(x),
                                      _row_stride(out), _stream())
    _lib.check(rc, "sa3_permute_cols")
    return out
