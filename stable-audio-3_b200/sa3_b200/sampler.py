"""The ping-pong sampler loop over the B200 denoiser, and the same loop as one CUDA graph.

sample_flow_pingpong restates stable_audio_3/inference/sampling.py:308-351, the loop the distilled models use
under generate(): for each step i of the schedule, denoised = x - t_i * v(x, t_i), then
x = (1 - t_{i+1}) * denoised + t_{i+1} * noise_i (a fresh N(0, 1) draw, randn_like(x)). The schedule is either
global (sigmas [steps + 1]) or per element (sigmas [B, steps + 1]).

GraphedPingpong captures every step of that loop (the denoiser forward with its CFG/APG combine, and the
update) into one CUDA graph, the pattern of the reference TensorRT runner's graph-captured sampler
(optimized/tensorRT/scripts/sa3_trt_core.py:511-694): a replay runs all steps with no host work between them.
The noise draws are an input of the graph (noise [steps, *x.shape]), so a replay is reproducible and can be
compared with the eager loop draw for draw.
"""
from __future__ import annotations

from typing import Optional

import torch


def _step_times(sigmas: torch.Tensor, i: int, batch: int, dtype):
    """(t for the model [B], t_i and t_{i+1} broadcastable over [B, C, T]) of step i (sampling.py:322-340)."""
    if sigmas.dim() == 2:
        tc, tn = sigmas[:, i].to(dtype), sigmas[:, i + 1].to(dtype)
        return tc, tc.view(-1, 1, 1), tn.view(-1, 1, 1)
    tc, tn = sigmas[i].to(dtype), sigmas[i + 1].to(dtype)
    return tc * torch.ones(batch, dtype=dtype, device=sigmas.device), tc, tn


def sample_flow_pingpong(model, x: torch.Tensor, sigmas: torch.Tensor, noise: Optional[torch.Tensor] = None,
                         **extra_args) -> torch.Tensor:
    """The ping-pong loop (sampling.py:308-351). model(x, t, **extra_args) returns the velocity; noise, if
    given, holds the per-step draws [steps, *x.shape], otherwise each step draws randn_like(x)."""
    sigmas = sigmas.to(x.device)
    steps = sigmas.shape[-1] - 1
    for i in range(steps):
        t_model, tc, tn = _step_times(sigmas, i, x.shape[0], x.dtype)
        denoised = x - tc * model(x, t_model, **extra_args)
        z = noise[i] if noise is not None else torch.randn_like(x)
        x = (1 - tn) * denoised + tn * z
    return x


class GraphedPingpong:
    """All steps of sample_flow_pingpong on a DiTEngine as one CUDA graph.

    The shapes, the schedule, cfg_scale / apg_scale and the padding mask are fixed at capture; each call copies
    x, the noise draws and the conditioning into static buffers and replays the graph."""

    def __init__(self, engine, x, sigmas, noise, cross_attn_cond=None, global_embed=None, local_add_cond=None,
                 cfg_scale: float = 1.0, apg_scale: float = 1.0, padding_mask=None):
        dev = engine.dev
        self.engine = engine
        self.sigmas = sigmas.to(dev, torch.float32).clone()
        self.static = [None if a is None else a.to(dev).clone()
                       for a in (x, noise, cross_attn_cond, global_embed, local_add_cond)]
        self.padding_mask = None if padding_mask is None else padding_mask.to(dev).clone()
        self.kw = dict(cfg_scale=cfg_scale, apg_scale=apg_scale)

        def run():
            x0, nz, cc, ge, lc = self.static

            def model(xx, tt):
                return engine.forward(xx, tt, cc, ge, lc, padding_mask=self.padding_mask, **self.kw)

            return sample_flow_pingpong(model, x0, self.sigmas, nz)

        side = torch.cuda.Stream()
        side.wait_stream(torch.cuda.current_stream())
        with torch.cuda.stream(side):
            run()  # lays out the workspace for these shapes (and this mask) before capture
        torch.cuda.current_stream().wait_stream(side)
        self.graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(self.graph):
            self.out = run()
        # the graph replays into these buffers: keep them alive even after the engine switches to another shape
        self.workspace, self.rope = engine.ws, engine.rope

    def __call__(self, x, noise, cross_attn_cond=None, global_embed=None, local_add_cond=None) -> torch.Tensor:
        for dst, src in zip(self.static, (x, noise, cross_attn_cond, global_embed, local_add_cond)):
            if dst is not None:
                dst.copy_(src, non_blocking=True)
        self.graph.replay()
        return self.out
