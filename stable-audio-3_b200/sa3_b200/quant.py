"""Quantized drop-in replacements for the DiT's nn.Linear layers.

The reference projections are plain nn.Linear modules
(stable_audio_3/models/transformer.py:547-560 Attention, :432 GLU.proj,
:485 FeedForward linear_out). The modules here are built from such a Linear
(mirroring LoRAParametrization.from_linear, stable_audio_3/models/lora/model.py:262-269)
and quantize at construction:

  QuantLinearFP8  : e4m3 weight with per-output-channel scale absmax/448,
                    per-tensor dynamic e4m3 activation scale, fp32 accumulate,
                    scale (and bias) applied in the GEMM epilogue.
  QuantLinearGPTQ : int4 weight-only (group 128, asymmetric, act-order g_idx),
                    bf16 activations.

Both keep the Linear's `in_features`, `out_features` and `bias` so a state
dict written for the reference maps onto them, and refuse a Linear that still
carries live LoRA parametrizations (merge them first).
"""
from __future__ import annotations

import torch
from torch import nn

E4M3_MAX = 448.0
SWIGLU_BLOCK = 128


def interleave_swiglu_rows(w: torch.Tensor, b=None, block: int = SWIGLU_BLOCK):
    """Reorder GLU.proj rows [x (I rows) ; gate (I rows)] into blocks [x_t (128) ; gate_t (128)] so each
    256-wide GEMM tile holds matching x and gate columns and the SwiGLU fuses into its epilogue."""
    two_i = w.shape[0]
    inner = two_i // 2
    if inner % block:
        raise ValueError(f"SwiGLU inner dim {inner} must be a multiple of {block}")
    idx = torch.arange(two_i).view(2, inner // block, block).permute(1, 0, 2).reshape(-1)
    w2 = w[idx].contiguous()
    b2 = None if b is None else b[idx].contiguous()
    return w2, b2


def _check_plain_linear(lin: nn.Module) -> None:
    if not isinstance(lin, nn.Linear):
        raise TypeError(f"expected nn.Linear, got {type(lin).__name__}")
    if getattr(lin, "parametrizations", None):
        raise RuntimeError("Linear has active parametrizations (e.g. LoRA); merge them before quantizing")


def quantize_weight_e4m3(w: torch.Tensor):
    """Per-output-channel e4m3: s[n] = max(absmax(W[n]), 1e-12)/448, Wq = e4m3(W / s[n])."""
    w = w.detach().float()
    s = torch.clamp(w.abs().amax(dim=1), min=1e-12) / E4M3_MAX
    wq = (w / s[:, None]).clamp(-E4M3_MAX, E4M3_MAX).to(torch.float8_e4m3fn)
    return wq, s
