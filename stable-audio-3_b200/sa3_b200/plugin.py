"""The SAME-L differential sliding-window attention plugin operator on the sm_100a kernel.

Mirrors the TensorRT Python plugin samel::diff_attn_swa of the reference
(optimized/tensorRT/scripts/diff_attn_nocast_plugin.py:14-41): the shape
function halves the head axis; the implementation receives q_bat, k_bat,
v_bat [B, N, 2H, d] (two differential streams stacked on the head axis), the
number of heads H, the output tensors and a CUDA stream handle, and writes
out[0] = attn(heads :H) - attn(heads H:) with window 17 on that stream
(triton_swa_attn_v2, optimized/tensorRT/scripts/triton_swa_v2.py:94-119).

register_trt_plugin() registers the same op with tensorrt.plugin when
TensorRT is importable; the functions below work with plain torch tensors.
"""
from __future__ import annotations

from typing import Sequence

import torch

from . import ops

SAMEL_WINDOW = 17
_streams = {}


def diff_attn_swa_shape(q_shape: Sequence[int]) -> tuple:
    """Output shape: q_bat's shape with the head axis (dim -2) halved (diff_attn_nocast_plugin.py:14-19)."""
    s = list(q_shape)
    s[-2] //= 2
    return tuple(s)


def diff_attn_swa_impl(q_bat: torch.Tensor, k_bat: torch.Tensor, v_bat: torch.Tensor, num_heads: int,
                       outputs: Sequence[torch.Tensor], stream: int, window: int = SAMEL_WINDOW) -> None:
    """Write outputs[0] = attn(q,k,v heads :H) - attn(heads H:) on CUDA stream `stream` (no return value)."""
    out = outputs[0]
    if stream not in _streams:
        _streams[stream] = torch.cuda.ExternalStream(stream)
    with torch.cuda.stream(_streams[stream]):
        if q_bat.dtype == torch.float32:
            # fp32 plugin I/O: run the bf16 kernel on converted copies, write back in fp32
            qb, kb, vb = (t.to(torch.bfloat16) for t in (q_bat, k_bat, v_bat))
            ob = torch.empty(diff_attn_swa_shape(q_bat.shape), device=q_bat.device, dtype=torch.bfloat16)
            ops.diff_attn_swa(qb, kb, vb, num_heads, window, ob)
            out.copy_(ob)
        else:
            ops.diff_attn_swa(q_bat.contiguous(), k_bat.contiguous(), v_bat.contiguous(), num_heads, window, out)


def diff_attn_swa(q_bat: torch.Tensor, k_bat: torch.Tensor, v_bat: torch.Tensor, num_heads: int,
                  window: int = SAMEL_WINDOW) -> torch.Tensor:
    """Functional form: returns the [B, N, H, d] difference on the current stream."""
    out = torch.empty(diff_attn_swa_shape(q_bat.shape), device=q_bat.device, dtype=q_bat.dtype)
    diff_attn_swa_impl(q_bat, k_bat, v_bat, num_heads, [out], torch.cuda.current_stream().cuda_stream, window)
    return out


def register_trt_plugin():
    """Register samel::diff_attn_swa with tensorrt.plugin, backed by this kernel (TensorRT must be installed)."""
    import tensorrt.plugin as trtp  # noqa: F401  (absent in this environment)

    @trtp.register("samel::diff_attn_swa")
    def _desc(q_bat: trtp.TensorDesc, k_bat: trtp.TensorDesc, v_bat: trtp.TensorDesc,
              num_heads: int) -> trtp.TensorDesc:
        out = q_bat.like()
        out.shape_expr[-2] = q_bat.shape_expr[-2] // 2
        return out

    @trtp.impl("samel::diff_attn_swa")
    def _impl(q_bat: trtp.Tensor, k_bat: trtp.Tensor, v_bat: trtp.Tensor, num_heads: int, outputs, stream: int):
        to = lambda t: torch.as_tensor(t, device="cuda")  # noqa: E731
        diff_attn_swa_impl(to(q_bat), to(k_bat), to(v_bat), num_heads, [to(outputs[0])], stream)

    return _impl
