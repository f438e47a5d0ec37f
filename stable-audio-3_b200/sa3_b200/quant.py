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


def swiglu_interleave_index(two_i: int, block: int = SWIGLU_BLOCK) -> torch.Tensor:
    """Row order that turns GLU.proj rows [x (I rows) ; gate (I rows)] into blocks [x_t (128) ; gate_t (128)]."""
    inner = two_i // 2
    if inner % block:
        raise ValueError(f"SwiGLU inner dim {inner} must be a multiple of {block}")
    return torch.arange(two_i).view(2, inner // block, block).permute(1, 0, 2).reshape(-1)


def interleave_swiglu_rows(w: torch.Tensor, b=None, block: int = SWIGLU_BLOCK):
    """Reorder GLU.proj rows [x (I rows) ; gate (I rows)] into blocks [x_t (128) ; gate_t (128)] so each
    256-wide GEMM tile holds matching x and gate columns and the SwiGLU fuses into its epilogue."""
    idx = swiglu_interleave_index(w.shape[0], block)
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


class QuantLinearFP8(nn.Module):
    """FP8 e4m3 drop-in for nn.Linear (per-output-channel weight scale, per-tensor dynamic activation scale).

    forward(x[..., in]) -> [..., out] in bf16 (x is bf16; other dtypes are cast). Each call runs three
    kernels: max|x| reduction, e4m3 quantisation of x, and the tcgen05 FP8 GEMM whose epilogue applies
    s_x * s_w[n] and the bias.
    """

    def __init__(self, in_features: int, out_features: int, bias: bool = True, device=None):
        super().__init__()
        self.in_features, self.out_features = in_features, out_features
        self.register_buffer("qweight", torch.zeros(out_features, in_features, dtype=torch.float8_e4m3fn,
                                                    device=device))
        self.register_buffer("weight_scale", torch.ones(out_features, dtype=torch.float32, device=device))
        if bias:
            self.register_buffer("bias", torch.zeros(out_features, dtype=torch.float32, device=device))
        else:
            self.bias = None

    @classmethod
    def from_linear(cls, lin: nn.Linear, device=None) -> "QuantLinearFP8":
        _check_plain_linear(lin)
        device = device or lin.weight.device
        m = cls(lin.in_features, lin.out_features, lin.bias is not None, device=device)
        wq, s = quantize_weight_e4m3(lin.weight)
        m.qweight.copy_(wq.to(device))
        m.weight_scale.copy_(s.to(device))
        if lin.bias is not None:
            m.bias.copy_(lin.bias.detach().float().to(device))
        return m

    def forward(self, x: torch.Tensor) -> torch.Tensor:
        from . import ops

        shape = x.shape
        x2 = x.reshape(-1, shape[-1])
        if x2.dtype != torch.bfloat16:
            x2 = x2.to(torch.bfloat16)
        x2 = x2.contiguous()
        amax = torch.zeros(1, device=x2.device, dtype=torch.float32)
        scale = torch.empty(1, device=x2.device, dtype=torch.float32)
        ops.absmax(x2, amax)
        xq = ops.quantize_e4m3(x2, amax, scale_out=scale)
        y = ops.gemm(xq, self.qweight, a_scale=scale, b_scale=self.weight_scale, bias=self.bias)
        return y.reshape(*shape[:-1], self.out_features)

    def extra_repr(self) -> str:
        return f"in_features={self.in_features}, out_features={self.out_features}, fp8=e4m3"


# names of the DiT linears the quantized paths replace (stable_audio_3/models/transformer.py:547-560, 432, 485)
QUANTIZABLE = ("to_qkv", "to_q", "to_kv", "to_out", "ff.0.proj", "ff.2")


def quantize_linears_fp8(model: nn.Module, names=QUANTIZABLE) -> nn.Module:
    """Replace the attention / FF nn.Linear modules of a reference DiT in place with QuantLinearFP8,
    walking the module tree the way add_lora does (stable_audio_3/models/lora/model.py:364-414)."""
    targets = []
    for full, mod in model.named_modules():
        for cname, child in mod.named_children():
            path = f"{full}.{cname}" if full else cname
            if isinstance(child, nn.Linear) and any(path.endswith(n) for n in names):
                targets.append((mod, cname, child))
    for parent, cname, child in targets:
        setattr(parent, cname, QuantLinearFP8.from_linear(child))
    return model
