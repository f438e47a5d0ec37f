"""Data-parallel denoising across GPUs: prompts shard naturally.

Each prompt's conditional / unconditional CFG pair stays on one GPU, because
the CFG/APG combine (stable_audio_3/models/dit.py:571-625) needs both halves.
Prompts are spread over the ranks by longest-processing-time-first
bin-packing on a per-prompt cost (linear layers ~ tokens, windowed attention ~
key pairs), each rank packs its prompts into variable-length batches of at
most `max_tokens` rows, and there is no collective inside a denoiser step.
Results are gathered to every rank in the original prompt order outside the
timed work.
"""
from __future__ import annotations

import heapq
from typing import Callable, List, Sequence

import numpy as np
import torch
import torch.distributed as dist

# per-token FLOPs of one medium block pass over both CFG halves (linears) and per key pair (attention);
# only the ratio matters for balancing
LINEAR_FLOP_PER_TOKEN = 2.510e9
ATTN_FLOP_PER_PAIR = 4 * 64 * 24 * 2 * 24


def band_pairs(n: int, wl: int = 256, wr: int = 256) -> int:
    """Visible (query, key) pairs of a length-n sequence under a (wl, wr) band."""
    i = np.arange(n)
    return int((np.minimum(n - 1, i + wr) - np.maximum(0, i - wl) + 1).sum())


def prompt_cost(n_tokens: int, memory_tokens: int = 64, window=(256, 256)) -> float:
    n = n_tokens + memory_tokens
    return 2.0 * (LINEAR_FLOP_PER_TOKEN * n + ATTN_FLOP_PER_PAIR * band_pairs(n, *window))


def lpt_shard(costs: Sequence[float], world: int) -> List[List[int]]:
    """Longest-processing-time-first assignment of items to `world` bins (deterministic tie-breaking)."""
    heap = [(0.0, r) for r in range(world)]
    heapq.heapify(heap)
    bins: List[List[int]] = [[] for _ in range(world)]
    for i in sorted(range(len(costs)), key=lambda k: (-costs[k], k)):
        load, r = heapq.heappop(heap)
        bins[r].append(i)
        heapq.heappush(heap, (load + costs[i], r))
    return [sorted(b) for b in bins]


def micro_batches(indices: Sequence[int], lengths: Sequence[int], max_tokens: int, memory_tokens: int = 64):
    """Split a rank's prompts into consecutive packed batches of at most max_tokens stream rows
    (both CFG halves counted)."""
    out, cur, rows = [], [], 0
    for i in indices:
        r = 2 * (lengths[i] + memory_tokens)
        if cur and rows + r > max_tokens:
            out.append(cur)
            cur, rows = [], 0
        cur.append(i)
        rows += r
    if cur:
        out.append(cur)
    return out


def run_data_parallel(step: Callable[[List[int]], List[torch.Tensor]], lengths: Sequence[int], world: int,
                      rank: int, max_tokens: int = 1 << 17, window=(256, 256)):
    """Run `step(prompt_indices) -> per-prompt results` over this rank's share; returns (my indices, my results)."""
    shard = lpt_shard([prompt_cost(n, window=window) for n in lengths], world)[rank]
    results = []
    for mb in micro_batches(shard, lengths, max_tokens):
        results.extend(step(mb))
    return shard, results


def gather_results(shard: List[int], results: List[torch.Tensor], n_items: int) -> List[torch.Tensor]:
    """All ranks receive every prompt's result, in prompt order (CPU tensors; outside the timed step)."""
    local = list(zip(shard, [r.detach().cpu() for r in results]))
    if dist.is_available() and dist.is_initialized() and dist.get_world_size() > 1:
        parts = [None] * dist.get_world_size()
        dist.all_gather_object(parts, local)
        local = [x for part in parts for x in part]
    ordered: List[torch.Tensor] = [None] * n_items  # type: ignore[list-item]
    for i, r in local:
        ordered[i] = r
    if any(r is None for r in ordered):
        raise RuntimeError("a prompt was not processed by any rank")
    return ordered
