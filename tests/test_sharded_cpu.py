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
