"""Channel-sharded scan (config 5's decomposition) on CPU with 2 and 3 gloo ranks: each
rank scans its channel shard (the oracle stands in for the GPU scan) and the
all-gather + reassembly must reproduce the unsharded oracle bit for bit."""

import os
import socket

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from mambaqc_b200.kernels.sharded import channel_shard, ssm_scan_cayley_channel_sharded
from oracle import ref


def _inputs():
    g = torch.Generator().manual_seed(5)
    bsz, seqlen, dm, ds = 1, 24, 6, 4
    delta = torch.nn.functional.softplus(torch.randn(bsz, seqlen, dm, generator=g) - 3)
    lam = torch.randn(dm, ds, 4, generator=g) * 0.3
    lam[..., 0] = -lam[..., 0].abs()
    Bm = torch.randn(bsz, seqlen, ds, 4, generator=g)
    Cm = torch.randn(bsz, seqlen, ds, 4, generator=g)
    x = torch.randn(bsz, seqlen, dm, generator=g)
    Dk = torch.ones(dm)
    return [t.double() for t in (delta, lam, Bm, Cm, x, Dk)]


def _oracle_scan(d, L, Bm, Cm, s, Dk, h0=None):
    return ref.ssm_scan_cayley(d, L, Bm, Cm, s, Dk, h0=h0)


def _worker(rank, world, port, q):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        delta, lam, Bm, Cm, x, Dk = _inputs()
        shard = (channel_shard(delta, rank, world, 2), channel_shard(lam, rank, world, 0), Bm, Cm,
                 channel_shard(x, rank, world, 2), channel_shard(Dk, rank, world, 0))
        y1 = ssm_scan_cayley_channel_sharded(*shard, scan_fn=_oracle_scan)
        # three time segments, each scanned from the previous one's final state
        y3 = ssm_scan_cayley_channel_sharded(*shard, scan_fn=_oracle_scan, segments=3)
        q.put((rank, (y1, y3)))
    finally:
        dist.destroy_process_group()


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


@pytest.mark.parametrize("world", [2, 3])
def test_channel_sharded_scan_matches_unsharded(world):
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, world, port, q)) for r in range(world)]
    for p in procs:
        p.start()
    results = dict(q.get(timeout=120) for _ in range(world))
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    full = _oracle_scan(*_inputs())[0]
    for r in range(world):
        y1, y3 = results[r]
        assert torch.equal(y1, full)
        assert torch.allclose(y3, full, rtol=1e-12, atol=1e-12)


def test_channel_shard_rejects_uneven_split():
    with pytest.raises(ValueError):
        channel_shard(torch.zeros(1, 2, 5), 0, 2, 2)


# ------------------------------------------------------------ time-sharded scan

def _oracle_summary(d, L, Bm, Cm, s, Dk):
    """(P, E) of a time range from the oracle: P the left-ordered product of the
    Cayley steps, E the final state from zero."""
    bsz, seqlen, dm = d.shape
    q = ref.cayley(d[..., None, None] * L[None, None])          # [B,T,D,N,4]
    P = torch.zeros(bsz, dm, L.shape[1], 4, dtype=d.dtype)
    P[..., 0] = 1
    for t in range(seqlen):
        P = ref.qmul(q[:, t], P)
    E = ref.ssm_scan_cayley(d, L, Bm, Cm, s, Dk)[1]
    return P, E


def _oracle_carry(P_all, E_all, h0):
    H = torch.zeros_like(P_all[0]) if h0 is None else h0
    hin = []
    for s in range(P_all.shape[0]):
        hin.append(H)
        H = ref.qmul(P_all[s], H) + E_all[s]
    return torch.stack(hin), H


def _time_worker(rank, world, port, q):
    from mambaqc_b200.kernels.sharded import ssm_scan_cayley_time_sharded, time_shard

    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        delta, lam, Bm, Cm, x, Dk = _inputs()
        h0 = torch.randn(1, 6, 4, 4, generator=torch.Generator().manual_seed(8)).double()
        shard = (time_shard(delta, rank, world), lam, time_shard(Bm, rank, world),
                 time_shard(Cm, rank, world), time_shard(x, rank, world), Dk)
        y, hT = ssm_scan_cayley_time_sharded(*shard, h0=h0, summary_fn=_oracle_summary,
                                             carry_fn=_oracle_carry, scan_fn=_oracle_scan)
        q.put((rank, (y, hT)))
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("world", [2, 3])
def test_time_sharded_scan_matches_unsharded(world):
    """Each rank summarises its time range, the summaries are all-gathered and
    folded into each rank's start state; the ranks' outputs, concatenated in
    time, and the final state equal the unsharded scan."""
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_time_worker, args=(r, world, port, q)) for r in range(world)]
    for p in procs:
        p.start()
    results = dict(q.get(timeout=120) for _ in range(world))
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    inp = _inputs()
    h0 = torch.randn(1, 6, 4, 4, generator=torch.Generator().manual_seed(8)).double()
    y_full, h_full = ref.ssm_scan_cayley(*inp, h0=h0)
    y = torch.cat([results[r][0] for r in range(world)], dim=1)
    assert torch.allclose(y, y_full, rtol=1e-10, atol=1e-12)
    for r in range(world):
        assert torch.allclose(results[r][1], h_full, rtol=1e-10, atol=1e-12)
