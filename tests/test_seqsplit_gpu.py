"""One long sequence split over 2 GPUs (sa3_b200.seqsplit): the denoiser velocity of the split forward, with the
per-layer NCCL halo exchange and the all-reduced CFG/APG sums, against the unsplit forward on one GPU; and the
peer-memory max exchange of the FP8 scales on its own.
Skipped with fewer than 2 GPUs.

Asserted on the network output for both CFG halves (before the combine) and on the full CFG/APG velocity.
bf16: the split changes the row grouping and the key-tile grouping of the attention, so it agrees with the
unsplit forward to rounding; the CFG/APG combine (cfg 5) amplifies that rounding, as it does for the
reference's own bf16 module, so the velocity gets the full-step bound. FP8: the max|x| behind every per-tensor
activation scale is max-reduced over the ranks, so the split step quantizes with the unsplit step's scales;
the attention's different key-tile grouping still moves activations at rounding level, which e4m3 rounding
can turn into whole-step differences, so the velocity gets tests.tolerance.fp8_network_bound (measured with
the oracle on the same inputs)."""
import datetime
import os
import queue
import socket
import time

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from sa3_b200.modules import DiffusionTransformer, init_synthetic_
from tests.golden.cases import _small

pytestmark = pytest.mark.gpu

L, TC, SEED = 900, 16, 11


def _inputs():
    g = torch.Generator().manual_seed(SEED)
    x = torch.randn(1, _small.io_channels, L, generator=g)
    t = torch.tensor([0.55])
    cond = torch.randn(1, TC, _small.cond_token_dim, generator=g)
    gemb = torch.randn(1, _small.global_cond_dim, generator=g)
    loc = torch.randn(1, _small.local_add_cond_dim, L, generator=g) * 0.5
    return x, t, cond, gemb, loc


def _model(mode):
    return init_synthetic_(DiffusionTransformer(_small), seed=SEED).quantize(mode)


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    port = s.getsockname()[1]
    s.close()
    return port


def _worker(rank, world, port, mode, outq):
    from sa3_b200 import seqsplit as ss
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    torch.cuda.set_device(rank)
    # a short timeout: a rank whose peer died errors out instead of waiting in the halo exchange
    dist.init_process_group("nccl", rank=rank, world_size=world, device_id=torch.device("cuda", rank),
                            timeout=datetime.timedelta(seconds=120))
    try:
        eng = _model(mode).engine()
        sp = ss.make_split(L, rank, world, _small.num_memory_tokens, _small.sliding_window)
        x, t, cond, gemb, loc = (v.cuda() for v in _inputs())
        a, b = sp.lat_start, sp.lat_end
        with torch.inference_mode():
            for _ in range(2):  # the second call reuses the workspace
                v = eng.forward_split(x[..., a:b], t, sp, cond, gemb, loc[..., a:b], cfg_scale=5.0, apg_scale=1.0)
            xb, lb = x[..., a:b], loc[..., a:b]
            net = eng.inner_split(torch.cat([xb, xb]), torch.cat([t, t]), sp, torch.cat([cond, torch.zeros_like(cond)]),
                                  torch.cat([gemb, gemb]), torch.cat([lb, lb]))
        torch.cuda.synchronize()
        peer = ss.peer_max_active()
        # by value: the sender exits right after
        outq.put((rank, a, b, v.cpu().numpy(), net.cpu().numpy(), peer))
    finally:
        dist.destroy_process_group()


def _peer_worker(rank, world, port, outq):
    """200 peer-memory max exchanges of known values, then 10 captured in one CUDA graph and replayed 3 times,
    each result checked; the exchange timed against the NCCL all-reduce it replaces."""
    from sa3_b200 import _lib
    from sa3_b200 import seqsplit as ss
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    torch.cuda.set_device(rank)
    dist.init_process_group("nccl", rank=rank, world_size=world, device_id=torch.device("cuda", rank),
                            timeout=datetime.timedelta(seconds=120))
    try:
        ss.prepare_peer_max(None)
        used = ss.peer_max_active()
        vals = torch.rand(200, world, generator=torch.Generator().manual_seed(3)) * 100
        t = torch.zeros(1, device="cuda")
        bad = 0
        for i in range(200):
            t.fill_(float(vals[i, rank]))
            ss.all_reduce_max(t)
            bad += int(t.item() != float(vals[i].max()))
        # a CUDA graph of 10 exchanges (the epoch counter lives on the device, so replays stay in step)
        buf = torch.zeros(10, device="cuda")
        src = torch.tensor([float(vals[i, rank]) for i in range(10)], device="cuda")
        s = torch.cuda.Stream()
        s.wait_stream(torch.cuda.current_stream())
        g = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g, stream=s):
            buf.copy_(src)
            for i in range(10):
                ss.all_reduce_max(buf[i:i + 1])
        for _ in range(3):
            buf.zero_()
            g.replay()
            torch.cuda.synchronize()
            bad += int(not torch.equal(buf.cpu(), vals[:10].max(dim=1).values))
        del g
        # timing: 100 exchanges, peer memory vs NCCL
        times = {}
        for name, fn in (("peer", lambda: ss.all_reduce_max(t)),
                         ("nccl", lambda: dist.all_reduce(t, op=dist.ReduceOp.MAX))):
            for _ in range(10):
                fn()
            torch.cuda.synchronize()
            dist.barrier()
            e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            e0.record()
            for _ in range(100):
                fn()
            e1.record()
            torch.cuda.synchronize()
            times[name] = e0.elapsed_time(e1) * 10.0  # us per exchange
        outq.put((rank, used, bad, _lib.device_error(), times))
    finally:
        dist.destroy_process_group()


def _spawn(target, extra, timeout_s=600):
    ctx = mp.get_context("spawn")
    outq = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=target, args=(r, 2, port, *extra, outq)) for r in range(2)]
    for p in procs:
        p.start()
    res, deadline = [], time.monotonic() + timeout_s
    try:
        while len(res) < 2:
            try:
                res.append(outq.get(timeout=5))
            except queue.Empty:
                dead = [p.exitcode for p in procs if p.exitcode not in (None, 0)]
                if dead or time.monotonic() > deadline:
                    pytest.fail(f"split workers failed (exit codes {[p.exitcode for p in procs]})")
        for p in procs:
            p.join(timeout=120)
            assert p.exitcode == 0
    finally:
        for p in procs:
            if p.is_alive():
                p.kill()
    return sorted(res, key=lambda r: r[0])


def test_peer_max_exchange(cuda):
    """The FP8 amax max-reduction of the sequence split through NVLink peer memory (sa3_peer_max) on 2 GPUs:
    the peer path is chosen, every eager and graph-replayed exchange returns the exact max of the ranks' values,
    no wait runs out, and it is timed against the NCCL all-reduce."""
    if torch.cuda.device_count() < 2:
        pytest.skip("needs 2 GPUs")
    res = _spawn(_peer_worker, ())
    for rank, used, bad, err, times in res:
        print(f"rank {rank}: peer path {used}, wrong results {bad}, device error {err}, "
              f"us per exchange: peer {times['peer']:.2f}, NCCL all-reduce {times['nccl']:.2f}")
        assert used and bad == 0 and err == 0


def _fp8_velocity_bound():
    from dataclasses import replace

    from oracle import dit as odit
    from tests.test_oracle_golden import _cfg
    from tests.tolerance import fp8_network_bound

    sd = _model("fp8").state_dict()
    x, t, cond, gemb, loc = _inputs()
    with torch.inference_mode():
        a = odit.dit_forward(sd, replace(_cfg(_small), act_bf16=True), x, t, cond, gemb, loc, 5.0, 1.0, mode="fp8")
        b = odit.dit_forward(sd, _cfg(_small), x, t, cond, gemb, loc, 5.0, 1.0, mode="fp8")
    return fp8_network_bound(a, b)


@pytest.mark.parametrize("mode,tol_net,tol_vel", [("bf16", 5e-3, 2e-2), ("fp8", 2e-2, None)])
def test_sequence_split_matches_unsplit(cuda, mode, tol_net, tol_vel):
    if torch.cuda.device_count() < 2:
        pytest.skip("needs 2 GPUs")
    res = _spawn(_worker, (mode,))
    assert res[0][1] == 0 and res[0][2] == res[1][1] and res[1][2] == L
    if mode == "fp8":
        assert all(r[5] for r in res), "FP8 split: the amax exchange did not take the peer-memory path"
    split = torch.cat([torch.from_numpy(r[3]) for r in res], dim=-1)
    net = torch.cat([torch.from_numpy(r[4]) for r in res], dim=-1)
    x, t, cond, gemb, loc = _inputs()
    eng = _model(mode).engine()
    with torch.inference_mode():
        ref = eng.forward(x.to(cuda), t.to(cuda), cond.to(cuda), gemb.to(cuda), loc.to(cuda), cfg_scale=5.0,
                          apg_scale=1.0).cpu()
        ref_net = eng.inner(torch.cat([x, x]).to(cuda), torch.cat([t, t]).to(cuda),
                            torch.cat([cond, torch.zeros_like(cond)]).to(cuda), torch.cat([gemb, gemb]).to(cuda),
                            torch.cat([loc, loc]).to(cuda)).cpu()
    assert torch.isfinite(split).all() and torch.isfinite(net).all()
    err_net = ((net - ref_net).norm() / ref_net.norm()).item()
    err_vel = ((split - ref).norm() / ref.norm()).item()
    if tol_vel is None:
        tol_vel = _fp8_velocity_bound()
    print(f"split over 2 GPUs, {mode}: network rel L2 {err_net:.3e} (bound {tol_net:.1e}), CFG velocity "
          f"{err_vel:.3e} (bound {tol_vel:.3e})")
    assert err_net < tol_net, err_net
    assert err_vel < tol_vel, err_vel
