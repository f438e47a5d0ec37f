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

import math
from typing import Optional, Sequence

import torch

from . import ops

SAMEL_WINDOW = 17
_streams = {}
_scratch = {}  # device index -> uint8 workspace of the fp32 path, grown only when a larger call arrives


def fp32_workspace_bytes(q_shape: Sequence[int]) -> int:
    """Scratch of the fp32 path: bf16 copies of q, k, v and the bf16 output (half of q's heads)."""
    n = math.prod(q_shape)
    return 2 * (3 * n + n // 2)


def _device_scratch(device: torch.device, nbytes: int) -> torch.Tensor:
    idx = device.index if device.index is not None else torch.cuda.current_device()
    buf = _scratch.get(idx)
    if buf is None or buf.numel() < nbytes:
        buf = _scratch[idx] = torch.empty(nbytes, device=device, dtype=torch.uint8)
    return buf


def _torch_stream(handle: int) -> torch.cuda.Stream:
    """The torch stream object that launches onto the CUDA stream `handle`.

    The caller's current stream (and the legacy default stream, handle 0) are used as they are:
    torch.cuda.ExternalStream(0) is not the default stream but maps to another stream, so work on it
    would not be ordered after what the caller queued on the default stream. Any other handle (a
    TensorRT enqueue's stream) is wrapped once per handle."""
    cur = torch.cuda.current_stream()
    if handle == cur.cuda_stream:
        return cur
    if handle == 0:
        return torch.cuda.default_stream()
    s = _streams.get(handle)
    if s is None:
        s = _streams[handle] = torch.cuda.ExternalStream(handle)
    return s


def diff_attn_swa_shape(q_shape: Sequence[int]) -> tuple:
    """Output shape: q_bat's shape with the head axis (dim -2) halved (diff_attn_nocast_plugin.py:14-19)."""
    s = list(q_shape)
    s[-2] //= 2
    return tuple(s)


def diff_attn_swa_impl(q_bat: torch.Tensor, k_bat: torch.Tensor, v_bat: torch.Tensor, num_heads: int,
                       outputs: Sequence[torch.Tensor], stream: int, window: int = SAMEL_WINDOW,
                       workspace: Optional[torch.Tensor] = None) -> None:
    """Write outputs[0] = attn(q,k,v heads :H) - attn(heads H:) on CUDA stream `stream` (no return value).

    fp32 I/O runs the bf16 kernel on bf16 copies and writes the result back in fp32. Those copies live in
    `workspace` (a uint8 CUDA tensor of at least fp32_workspace_bytes(q_bat.shape) bytes, e.g. the workspace
    a TensorRT plugin is given) or, without one, in a per-device buffer that is allocated only when a call
    larger than every earlier one arrives: a repeated call (every enqueue of a built engine) allocates nothing.
    Make the first call of the largest shape before any graph capture."""
    out = outputs[0]
    with torch.cuda.stream(_torch_stream(stream)):
        if q_bat.dtype == torch.float32:
            need = fp32_workspace_bytes(q_bat.shape)
            ws = workspace if workspace is not None else _device_scratch(q_bat.device, need)
            if ws.dtype != torch.uint8 or ws.numel() < need or not ws.is_cuda:
                raise RuntimeError(f"the fp32 path needs a CUDA uint8 workspace of {need} bytes")
            n = q_bat.numel()
            buf = ws[:need].view(torch.bfloat16)
            qb, kb, vb = (buf[i * n:(i + 1) * n].view(q_bat.shape) for i in range(3))
            ob = buf[3 * n:3 * n + n // 2].view(diff_attn_swa_shape(q_bat.shape))
            qb.copy_(q_bat)
            kb.copy_(k_bat)
            vb.copy_(v_bat)
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
