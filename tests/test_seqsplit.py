"""CPU: one sequence split across ranks (sa3_b200.seqsplit), with 2-4 gloo ranks as separate processes.

The split must reproduce the unsplit computation: windowed attention of each rank's own rows over
[left halo | own | right halo] with the re-centred window equals the rows of the full-sequence oracle
attention (oracle/ref.py attention, the masked-SDPA definition of transformer.py:696-699), and the
CFG/APG combine with its two sums all-reduced equals the combine over the whole sequence."""
import os
import socket

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from oracle import ref as orf
from sa3_b200 import seqsplit as ss


def test_split_ranges_cover_the_stream():
    for latents, world in ((8183, 2), (16384, 8), (1000, 4), (300, 2)):
        r = ss.split_ranges(latents, world, 64, 64)
        assert r[0][0] == 0 and r[-1][1] == latents + 64
        assert all(a[1] == b[0] for a, b in zip(r, r[1:]))
        assert max(e - s for s, e in r) - min(e - s for s, e in r) <= 1
        sp = [ss.make_split(latents, k, world, 64, (64, 64)) for k in range(world)]
        assert sp[0].memory_here == 64 and all(x.memory_here == 0 for x in sp[1:])
        assert sum(x.lat_end - x.lat_start for x in sp) == latents
    with pytest.raises(ValueError):
        ss.split_ranges(200, 4, 64, 256)


def test_halo_window_recentres_the_band():
    for wl, wr, hl, hr in ((256, 256, 0, 256), (256, 256, 256, 256), (256, 256, 256, 0), (64, 32, 64, 32),
                           (64, 32, 0, 32), (17, 40, 17, 0)):
        wl2, wr2 = ss.halo_window(wl, wr, hl, hr)
        n = 700
        m = orf.band_mask(n, hl + n + hr, wl2, wr2)
        i = torch.arange(n)[:, None]
        j = torch.arange(hl + n + hr)[None, :] - hl  # key position relative to the own rows
        assert torch.equal(m, (j - i >= -wl) & (j - i <= wr))


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    port = s.getsockname()[1]
    s.close()
    return port


def _worker(rank, world, port, n_tok, window, outq):
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        g = torch.Generator().manual_seed(0)
        B, d = 2, 64
        q = torch.randn(B, n_tok, d, generator=g)
        k = torch.randn(B, n_tok, d, generator=g)
        v = torch.randn(B, n_tok, d, generator=g)
        sp = ss.make_split(n_tok - 64, rank, world, 64, window)
        s0, s1 = sp.tok_start, sp.tok_end
        own = s1 - s0
        hl, hr = sp.halo_left, sp.halo_right
        e = hl + own + hr
        ext = torch.zeros(B * e, 2 * d)  # columns k | v
        for b in range(B):
            ext[b * e + hl:b * e + hl + own] = torch.cat([k[b, s0:s1], v[b, s0:s1]], dim=1)
        ss.exchange_halos(ext, B, own, sp)
        wl2, wr2 = ss.halo_window(*window, hl, hr)
        outs = []
        for b in range(B):
            blk = ext[b * e:(b + 1) * e]
            outs.append(orf.attention(q[b, s0:s1], blk[:, :d], blk[:, d:], wl2, wr2))
        # CFG/APG combine on this rank's latent columns
        C = 8
        x = torch.randn(1, C, n_tok - 64, generator=g)
        out2 = torch.randn(2, C, n_tok - 64, generator=g)
        t = torch.tensor([0.6])
        comb = ss.cfg_combine_split(x[..., sp.lat_start:sp.lat_end], t, out2[..., sp.lat_start:sp.lat_end], 5.0, 0.7)
        # the FP8 amax max-reduction: without GPUs every rank agrees to keep the collective (no peer memory)
        ss.prepare_peer_max(None)
        amax = torch.tensor([float(3 * rank + 1)])
        ss.all_reduce_max(amax)
        # numpy payloads travel by value (a shared-memory tensor could outlive its sender)
        outq.put((rank, s0, s1, torch.stack(outs).numpy(), sp.lat_start, sp.lat_end, comb.numpy(), amax.item(),
                  not ss.peer_max_active()))
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("world,n_tok,window", [(2, 1100, (256, 256)), (3, 900, (64, 48)), (4, 700, (17, 40))])
def test_split_attention_and_cfg_match_unsplit(world, n_tok, window):
    ctx = mp.get_context("spawn")
    outq = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, world, port, n_tok, window, outq)) for r in range(world)]
    for p in procs:
        p.start()
    res = sorted([outq.get(timeout=300) for _ in range(world)], key=lambda r: r[0])
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    g = torch.Generator().manual_seed(0)
    B, d = 2, 64
    q = torch.randn(B, n_tok, d, generator=g)
    k = torch.randn(B, n_tok, d, generator=g)
    v = torch.randn(B, n_tok, d, generator=g)
    full = torch.stack([orf.attention(q[b], k[b], v[b], *window) for b in range(B)])
    got = torch.cat([torch.from_numpy(r[3]) for r in res], dim=1)
    assert [r[1] for r in res] == sorted(r[1] for r in res) and res[-1][2] == n_tok
    assert torch.allclose(got, full, atol=1e-5, rtol=1e-5)
    x = torch.randn(1, 8, n_tok - 64, generator=g)
    out2 = torch.randn(2, 8, n_tok - 64, generator=g)
    ref = ss.cfg_combine_split(x, torch.tensor([0.6]), out2, 5.0, 0.7)
    comb = torch.cat([torch.from_numpy(r[6]) for r in res], dim=-1)
    assert torch.allclose(comb, ref, atol=1e-5, rtol=1e-4)
    assert all(r[7] == 3 * (world - 1) + 1 and r[8] for r in res)


def test_split_workspace_tables():
    """The per-row tables of a split rank: global RoPE positions, memory rows only on rank 0, latent rows after
    them, and the halo-extended projection buffer (built on the CPU: only shapes and tables are checked)."""
    from sa3_b200.engine import _Workspace
    from sa3_b200.modules import DiTConfig

    cfg = DiTConfig(embed_dim=256, depth=2, num_heads=4, sliding_window=(64, 48), differential=True)
    lat = 1000
    for world in (2, 3):
        for rank in range(world):
            sp = ss.make_split(lat, rank, world, cfg.num_memory_tokens, cfg.sliding_window)
            own_lat = sp.lat_end - sp.lat_start
            ws = _Workspace(cfg, [own_lat, own_lat], 0, torch.device("cpu"), False, split=sp)
            n = sp.tok_end - sp.tok_start
            assert ws.uniform_n == n and ws.nm == sp.memory_here
            assert torch.equal(ws.row_pos[:n], torch.arange(sp.tok_start, sp.tok_end, dtype=torch.int32))
            assert torch.equal(ws.row_pos[n:], ws.row_pos[:n])
            assert ws.lat_rows.tolist() == list(range(sp.memory_here, n)) + list(range(n + sp.memory_here, 2 * n))
            assert (ws.mem_rows is not None) == (rank == 0)
            assert ws.halo_e == sp.halo_left + n + sp.halo_right
            assert ws.qkv_ext.shape == (2 * ws.halo_e, 5 * cfg.embed_dim)
            assert ws.max_pos == sp.tok_end


@pytest.mark.parametrize("apg_scale", [0.0, 0.5, 1.0])
def test_split_combine_matches_oracle_on_one_rank(apg_scale):
    """Without a process group the split combine is the oracle's CFG/APG combine (dit.py:571-625)."""
    from oracle import dit as odit

    g = torch.Generator().manual_seed(7)
    x = torch.randn(2, 8, 300, generator=g)
    out = torch.randn(4, 8, 300, generator=g)
    t = torch.tensor([0.3, 0.8])
    ref = odit.cfg_combine(x, t, out, 5.0, apg_scale)
    got = ss.cfg_combine_split(x, t, out, 5.0, apg_scale)
    assert torch.allclose(got, ref, atol=1e-5, rtol=1e-5)


@pytest.mark.parametrize("world", [2, 3, 4])
@pytest.mark.parametrize("window", [(64, 64), (256, 256), (17, 17), (32, 64)])
def test_attention_views_cover_each_window_exactly(world, window):
    """The split self-attention runs as calls without halo (interior queries, issued while the halo exchange is
    in flight) and calls with it (queries next to a neighbour). Under the kernel's band convention every own
    row must see exactly the rows [i - wl, i + wr] of the sequence, and be computed by exactly one call."""
    for L in (700, 1500, 3000):
        try:
            splits = [ss.make_split(L, r, world, 64, window) for r in range(world)]
        except ValueError:
            continue
        for sp in splits:
            n = sp.tok_end - sp.tok_start
            hl, hr = sp.halo_left, sp.halo_right
            interior, edges = ss.attention_views(n, sp)
            seen, owner = {}, {}
            for q0, q1, k0, k1, (wl2, wr2) in interior + edges:
                dlt = (k1 - k0) - (q1 - q0)
                for i in range(q1 - q0):
                    assert q0 + i not in owner
                    owner[q0 + i] = (q0, q1)
                    seen[q0 + i] = {k0 + j for j in range(k1 - k0) if -wl2 <= j - i - dlt <= wr2}
            assert sorted(owner) == list(range(n))
            for i in range(n):
                want = {hl + i + d for d in range(-sp.wl, sp.wr + 1) if 0 <= hl + i + d < hl + n + hr}
                assert seen[i] == want, (sp.rank, i)
