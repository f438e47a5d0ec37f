"""One long sequence split across GPUs (sequence parallelism for the windowed DiT trunk).

The token stream of a sequence ([64 memory tokens | L latents], positions 0..N-1,
stable_audio_3/models/transformer.py:1215-1230) is cut into contiguous ranges, one
per rank; rank 0 holds the memory tokens. Everything in a block is row-local except
the windowed self-attention (transformer.py:598-700) with window (wl, wr): before it,
every rank sends the first wr rows of its post-RoPE q|k|v|q'|k' projection to its left
neighbour and the last wl rows to its right neighbour (NCCL send/recv through
torch.distributed), and attends over [left halo | own rows | right halo] with the window
re-centred on its own rows. RoPE uses global positions. The CFG/APG combine (dit.py:571-625) needs two
sums over the whole sequence per prompt; they are all-reduced. With FP8 linears, the max|x| behind each
per-tensor activation scale is max-reduced over the ranks as well, so the split step quantizes with the
unsplit step's scales. Cross-attention keys (the context) and the conditioning are replicated.
"""
from __future__ import annotations

import ctypes
from dataclasses import dataclass
from typing import List, Tuple

import torch
import torch.distributed as dist


@dataclass(frozen=True)
class SeqSplit:
    """This rank's share of one sequence: stream tokens [tok_start, tok_end) of N = memory + L, i.e. latents
    [lat_start, lat_end). Before every self-attention with window (wl, wr) the rank receives wl rows from its
    left neighbour and wr rows from its right neighbour."""

    rank: int
    world: int
    tok_start: int
    tok_end: int
    memory_tokens: int
    wl: int
    wr: int
    group: object = None

    @property
    def lat_start(self) -> int:
        return max(self.tok_start, self.memory_tokens) - self.memory_tokens

    @property
    def lat_end(self) -> int:
        return self.tok_end - self.memory_tokens

    @property
    def memory_here(self) -> int:
        """Memory tokens in this rank's rows (all of them on rank 0, none elsewhere)."""
        return max(0, min(self.tok_end, self.memory_tokens) - self.tok_start)

    @property
    def halo_left(self) -> int:
        return self.wl if self.rank > 0 else 0

    @property
    def halo_right(self) -> int:
        return self.wr if self.rank < self.world - 1 else 0


def split_ranges(latents: int, world: int, memory_tokens: int = 64, halo: int = 256) -> List[Tuple[int, int]]:
    """Contiguous, balanced token ranges of the N = memory + latents stream, one per rank. Every range
    must hold at least `halo` = max(wl, wr) tokens (a halo never reaches past the neighbouring rank)."""
    n = latents + memory_tokens
    bounds = [round(r * n / world) for r in range(world + 1)]
    ranges = [(bounds[r], bounds[r + 1]) for r in range(world)]
    if world > 1 and min(e - s for s, e in ranges) < halo:
        raise ValueError(f"{n} tokens over {world} ranks leave fewer than {halo} tokens on a rank")
    if ranges[0][1] < memory_tokens:
        raise ValueError("rank 0 must hold all memory tokens")
    return ranges


def make_split(latents: int, rank: int, world: int, memory_tokens: int = 64, window=(256, 256),
               group=None) -> SeqSplit:
    wl, wr = window
    if wl < 0 or wr < 0:
        raise ValueError("the sequence split needs a bounded window")
    s, e = split_ranges(latents, world, memory_tokens, max(wl, wr, 1))[rank]
    return SeqSplit(rank, world, s, e, memory_tokens, wl, wr, group)


def halo_window(wl: int, wr: int, halo_left: int, halo_right: int) -> Tuple[int, int]:
    """Window for queries = own rows, keys = [halo_left | own | halo_right] under the kernels' convention that
    the band is centred on key j = i + (lk - lq) (flash-attn's bottom-right alignment): own row i sits at key
    halo_left + i and lk - lq = halo_left + halo_right, so the band [i - wl, i + wr] becomes
    (wl + halo_right, wr - halo_right). The halos hold exactly wl (left) and wr (right) rows, or none at
    the ends of the sequence."""
    if wl < 0 or wr < 0:
        raise ValueError("the sequence split needs a bounded window")
    if halo_left not in (0, wl) or halo_right not in (0, wr):
        raise ValueError("halos must hold exactly the window's rows")
    return wl + halo_right, wr - halo_right


def view_window(wl: int, wr: int, q0: int, q1: int, k0: int, k1: int, hl: int) -> Tuple[int, int]:
    """Window for one attention call whose queries are own rows [q0, q1) and whose keys are rows [k0, k1) of
    [left halo (hl rows) | own rows | right halo], so that own row i still sees rows [i - wl, i + wr] of the
    sequence. Under the kernels' bottom-right convention key j' of the view is visible to query i' iff
    -wl2 <= j' - i' - dlt <= wr2 with dlt = (k1 - k0) - (q1 - q0); query i' is own row q0 + i', at view key
    c = q0 + hl - k0 + i'. Both bounds must come out non-negative (a negative bound would mean unbounded)."""
    c = q0 + hl - k0
    dlt = (k1 - k0) - (q1 - q0)
    wl2, wr2 = dlt - c + wl, c + wr - dlt
    if wl2 < 0 or wr2 < 0:
        raise ValueError(f"view [{q0},{q1}) x [{k0},{k1}) cannot express the window ({wl}, {wr})")
    return wl2, wr2


def attention_views(own: int, split: SeqSplit):
    """The self-attention of a split rank as calls that need no halo (issued while the halo exchange is in
    flight) and calls that do. Each entry is (q0, q1, k0, k1, (wl2, wr2)) with queries = own rows [q0, q1)
    and keys = rows [k0, k1) of [left halo | own | right halo]. Interior queries (window inside the own rows)
    attend over the own rows; the first wl and last wr own rows, next to a neighbour, over the halo too."""
    wl, wr, hl, hr = split.wl, split.wr, split.halo_left, split.halo_right
    q0, q1 = (wl if hl else 0), (own - wr if hr else own)
    if q1 - q0 <= 0:  # no interior: one call over everything after the exchange
        return [], [(0, own, 0, hl + own + hr, view_window(wl, wr, 0, own, 0, hl + own + hr, hl))]
    interior = [(q0, q1, hl, hl + own, view_window(wl, wr, q0, q1, hl, hl + own, hl))]
    edges = []
    if hl:
        k1 = min(hl + own + hr, hl + wl + wr)
        edges.append((0, wl, 0, k1, view_window(wl, wr, 0, wl, 0, k1, hl)))
    if hr:
        k0 = max(0, hl + own - wr - wl)
        edges.append((own - wr, own, k0, hl + own + hr, view_window(wl, wr, own - wr, own, k0, hl + own + hr, hl)))
    return interior, edges


def exchange_halos(ext: torch.Tensor, batch: int, own: int, split: SeqSplit, wait: bool = True):
    """ext: [batch * (hl + own + hr), C] rows laid out per sequence as [left halo | own rows | right halo].
    Fills the halo rows from the neighbours (their own rows next to the boundary) and sends this rank's
    boundary rows. All transfers of one call form one batched group of P2P operations. With wait=False the
    requests are returned: waiting on them later makes the current stream wait for the transfers, and work
    queued in between overlaps them."""
    hl, hr = split.halo_left, split.halo_right
    e = hl + own + hr
    ops = []
    for b in range(batch):
        base = b * e
        if hl:  # the left neighbour's right halo is wr rows; its last wl rows are this rank's left halo
            ops.append(dist.P2POp(dist.isend, ext[base + hl:base + hl + split.wr], split.rank - 1, split.group))
            ops.append(dist.P2POp(dist.irecv, ext[base:base + hl], split.rank - 1, split.group))
        if hr:
            ops.append(dist.P2POp(dist.isend, ext[base + hl + own - split.wl:base + hl + own], split.rank + 1,
                                  split.group))
            ops.append(dist.P2POp(dist.irecv, ext[base + hl + own:base + e], split.rank + 1, split.group))
    reqs = dist.batch_isend_irecv(ops) if ops else []
    if wait:
        for req in reqs:
            req.wait()
        return []
    return reqs


class PeerMax:
    """Max of one fp32 device value over the ranks of `group` through NVLink peer memory (sa3_peer_max): each
    rank owns a mailbox in its GPU memory, opened by the other ranks through CUDA IPC handles. One kernel per
    call, no NCCL. Construct it on every rank of the group at the same point (it gathers the handles)."""

    def __init__(self, group=None):
        from . import _lib

        lib = _lib.load()
        self.rank, self.world = dist.get_rank(group), dist.get_world_size(group)
        self._lib, self._opened = lib, []
        box = ctypes.c_void_p()
        _lib.check(lib.sa3_peer_box_alloc(ctypes.byref(box)), "sa3_peer_box_alloc")
        self._box = box
        h = (ctypes.c_char * lib.sa3_ipc_handle_bytes())()
        _lib.check(lib.sa3_ipc_get_handle(box, h), "sa3_ipc_get_handle")
        handles = [None] * self.world
        dist.all_gather_object(handles, bytes(h), group=group)
        ptrs, ok = [], True
        for r, hb in enumerate(handles):
            if r == self.rank:
                ptrs.append(box.value)
                continue
            p = ctypes.c_void_p()
            if lib.sa3_ipc_open_handle(hb, ctypes.byref(p)) != 0:
                ok = False
                break
            self._opened.append(p)
            ptrs.append(p.value)
        oks = [None] * self.world
        dist.all_gather_object(oks, ok, group=group)
        self.ok = all(oks)
        self._boxes = (ctypes.c_void_p * self.world)(*ptrs) if self.ok else None

    def __call__(self, t: torch.Tensor) -> None:
        from . import _lib

        rc = self._lib.sa3_peer_max(t.data_ptr(), self._boxes, self.rank, self.world,
                                    torch.cuda.current_stream().cuda_stream)
        _lib.check(rc, "sa3_peer_max")


# id(process group) -> (the group object, PeerMax or None where the group keeps the NCCL all-reduce). The entry
# holds the group object and is used only while that very object is the group asked for, so a group destroyed
# and created again (with other peers) never reaches mailboxes opened for the old one.
_peer_max = {}


def _resolve_group(group):
    return group if group is not None else dist.distributed_c10d._get_default_group()


def _peer_entry(group):
    g = _resolve_group(group)
    ent = _peer_max.get(id(g))
    return ent if ent is not None and ent[0] is g else None


def peer_max_active(group=None) -> bool:
    """True when all_reduce_max of `group` goes through peer memory."""
    ent = _peer_entry(group) if dist.is_initialized() else None
    return ent is not None and ent[1] is not None


def prepare_peer_max(group=None) -> None:
    """Collective (every rank of `group`, same point): set up the peer-memory max exchange when every rank runs on
    its own GPU of one host (distinct device UUIDs) and has opened every other rank's mailbox; otherwise the
    group keeps the NCCL all-reduce. SA3_PEER_MAX=0 in the environment keeps NCCL everywhere."""
    if not dist.is_initialized() or _peer_entry(group) is not None:
        return
    import os
    import socket

    world = dist.get_world_size(group)
    use = os.environ.get("SA3_PEER_MAX", "1") != "0" and torch.cuda.is_available() and 2 <= world <= 8
    me = (socket.gethostname(), str(torch.cuda.get_device_properties(torch.cuda.current_device()).uuid)
          if torch.cuda.is_available() else "", use)
    who = [None] * world
    dist.all_gather_object(who, me, group=group)
    eligible = all(w[2] for w in who) and len({w[0] for w in who}) == 1 and len({w[1] for w in who}) == world
    pm = PeerMax(group) if eligible else None
    g = _resolve_group(group)
    _peer_max[id(g)] = (g, pm if pm is not None and pm.ok else None)


def all_reduce_max(t: torch.Tensor, group=None) -> None:
    """In-place max over the split's ranks (a per-tensor FP8 activation amax: the tensor is the whole
    sequence, so every rank quantizes with the scale the unsplit step would use): through peer memory where
    prepare_peer_max set that up for the group, else one NCCL all-reduce."""
    if dist.is_initialized():
        ent = _peer_entry(group)
        pm = ent[1] if ent is not None else None
        if pm is not None and t.is_cuda:
            pm(t)
        else:
            dist.all_reduce(t, op=dist.ReduceOp.MAX, group=group)


def cfg_combine_split(x: torch.Tensor, t: torch.Tensor, out: torch.Tensor, cfg_scale: float, apg_scale: float,
                      group=None) -> torch.Tensor:
    """CFG + APG (dit.py:571-625, apg_project dit.py:311-343) on this rank's latent columns x [B, C, Lr],
    out [2B, C, Lr] (cond | uncond). The projection's two sums over (C, T) of each prompt, |cond_den|^2 and
    <diff, cond_den>, are summed over the ranks; the rest is elementwise. fp32."""
    x = x.float()
    cond_out, uncond_out = out.float().chunk(2)
    sigma = t.float()[:, None, None]
    cond_den = x - cond_out * sigma
    diff = (uncond_out - cond_out) * sigma
    if apg_scale == 0.0:
        cfg_diff = diff
    else:
        sums = torch.stack([cond_den.pow(2).sum(dim=(1, 2)), (diff * cond_den).sum(dim=(1, 2))])
        if dist.is_initialized():
            dist.all_reduce(sums, group=group)
        nrm = sums[0].sqrt().clamp_min(1e-12)
        # apg_project: v1 = cond_den / |cond_den|; parallel = <diff, v1> v1
        par = (sums[1] / (nrm * nrm))[:, None, None] * cond_den
        orth = diff - par
        cfg_diff = orth if apg_scale == 1.0 else apg_scale * orth + (1 - apg_scale) * diff
    cfg_den = cond_den + (cfg_scale - 1) * cfg_diff
    return (x - cfg_den) / sigma
