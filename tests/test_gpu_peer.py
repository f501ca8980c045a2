"""The peer-memory exchange of the channel-sharded scan.

* ``mqc_channel_push`` on one GPU, with several local buffers standing in for
  the ranks' outputs: every destination must hold every rank's channel shard in
  the final [B, T, D, 4] layout (bit-exact copy), for fp32 and bf16, and for a
  shard width whose rows are not whole 16-byte pieces (8-byte path).
* ``mqc_ssm_scan_fwd_chunked_peer`` on one GPU, the scan kernel storing y into
  several local buffers standing in for the ranks' outputs.
* On two GPUs (skipped with fewer): two NCCL ranks run the channel-sharded scan
  with ``gather="peer"`` (IPC buffers; y stored by the scan kernel, or pushed
  per segment) and ``gather="nccl"``; the results must be equal bit for bit
  and match the unsharded scan.
"""

import os
import socket

import pytest
import torch

from tests.gpu_util import DEV, gen, make_scan_inputs, rel_l2, to_dev

pytestmark = pytest.mark.gpu

from mambaqc_b200.kernels.sharded import channel_push  # noqa: E402


@pytest.mark.parametrize("dtype,dl", [(torch.float32, 6), (torch.bfloat16, 6),
                                      (torch.bfloat16, 3)])
def test_channel_push_emulated_ranks(dtype, dl):
    world, bsz, seqlen, segs = 3, 2, 48, 4
    seg = seqlen // segs
    g = gen(1)
    full = torch.randn(bsz, seqlen, world * dl, 4, generator=g).to(DEV, dtype)
    outs = [torch.full_like(full, float("nan")) for _ in range(world)]
    ptrs = [o.data_ptr() for o in outs]
    for r in range(world):
        shard = full[:, :, r * dl:(r + 1) * dl]
        for k in range(segs):
            src = shard[:, k * seg:(k + 1) * seg].contiguous()
            channel_push(src, ptrs, seqlen, world * dl, r * dl, k * seg)
    torch.cuda.synchronize()
    for o in outs:
        assert torch.equal(o, full)


@pytest.mark.parametrize("dtype,nc", [(torch.float32, 4), (torch.bfloat16, 4),
                                      (torch.bfloat16, 1)])
def test_scan_with_peer_outputs_emulated_ranks(dtype, nc):
    """mqc_ssm_scan_fwd_chunked_peer on one GPU: three channel shards, each
    scanned with its y stored into three local buffers standing in for the
    ranks' outputs. Every buffer must equal the shards' ordinary chunked scans
    laid side by side, bit for bit (same kernel, same chunks)."""
    from mambaqc_b200.kernels.ssm_fused import _run_scan_chunked
    world, dl = 3, 5
    inp = to_dev(make_scan_inputs(1, 256, world * dl, 32, shared=True, s_real=True, seed=11),
                 dtype)
    outs = [torch.full((1, 256, world * dl, 4), float("nan"), device=DEV, dtype=dtype)
            for _ in range(world)]
    ptrs = [o.data_ptr() for o in outs]
    want = []
    for r in range(world):
        cs = slice(r * dl, (r + 1) * dl)
        args = (inp["delta"][..., cs], inp["Lambda"][cs], inp["B"], inp["C"], inp["S"][..., cs],
                inp["D"][cs])
        y, _ = _run_scan_chunked(*args, None, 1e-6, nc, False)
        want.append(y)
        _run_scan_chunked(*args, None, 1e-6, nc, False, peer=(ptrs, world * dl, r * dl))
    torch.cuda.synchronize()
    full = torch.cat(want, dim=2)
    for o in outs:
        assert torch.equal(o, full)


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _two_rank_worker(rank, world, port, q):
    import torch.distributed as dist

    from mambaqc_b200.kernels import ssm_scan_cayley
    from mambaqc_b200.kernels.sharded import (release_peer_outputs,
                                              ssm_scan_cayley_channel_sharded)
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    torch.cuda.set_device(rank)
    dev = torch.device(f"cuda:{rank}")
    dist.init_process_group("nccl", rank=rank, world_size=world, device_id=dev)
    try:
        inp = make_scan_inputs(1, 1024, 16, 32, shared=True, s_real=True, seed=7)
        d = {k: v.to(dev, torch.bfloat16 if k not in ("Lambda", "D") else torch.float32)
             for k, v in inp.items()}
        dl = 16 // world
        sh = {k: (v[..., rank * dl:(rank + 1) * dl] if k in ("delta", "S") else v)
              for k, v in d.items()}
        sh["Lambda"] = d["Lambda"][rank * dl:(rank + 1) * dl]
        sh["D"] = d["D"][rank * dl:(rank + 1) * dl]
        args = (sh["delta"], sh["Lambda"], sh["B"], sh["C"], sh["S"], sh["D"])
        # y stored into both ranks' buffers by the scan kernel itself
        y_nccl1 = ssm_scan_cayley_channel_sharded(*args, time_chunks=4).clone()
        for _ in range(2):  # the second call reuses the cached peer buffers
            y_fused = ssm_scan_cayley_channel_sharded(*args, time_chunks=4,
                                                      gather="peer").clone()
        # NVLink SHARP multicast stores, where the platform has them: the same bits
        used_mc = True
        try:
            for _ in range(2):
                y_mc = ssm_scan_cayley_channel_sharded(*args, time_chunks=4,
                                                       gather="multicast").clone()
        except RuntimeError:  # no multicast on this platform
            used_mc = False
            y_mc = y_fused

        # segments pushed by mqc_channel_push (an explicit scan function)
        def scan_fn(dd, L, Bm, Cm, s, Dk, h0=None):
            return ssm_scan_cayley(dd, L, Bm, Cm, s, Dk, h0=h0, return_final_state=True,
                                   time_chunks=4)
        y_nccl4 = ssm_scan_cayley_channel_sharded(*args, scan_fn=scan_fn, segments=4).clone()
        y_push = ssm_scan_cayley_channel_sharded(*args, scan_fn=scan_fn, segments=4,
                                                 gather="peer").clone()
        y_full = ssm_scan_cayley(d["delta"], d["Lambda"], d["B"], d["C"], d["S"], d["D"])
        torch.cuda.synchronize()
        q.put((rank, torch.equal(y_fused, y_nccl1) and torch.equal(y_push, y_nccl4) and
               torch.equal(y_mc, y_nccl1),
               max(rel_l2(y_fused.float(), y_full.float()), rel_l2(y_push.float(), y_full.float())),
               used_mc))
        release_peer_outputs()
    finally:
        dist.destroy_process_group()


@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs 2 GPUs")
def test_peer_gather_matches_nccl_gather_on_two_ranks():
    import torch.multiprocessing as mp
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_two_rank_worker, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout=300)
    assert all(p.exitcode == 0 for p in procs)
    res = sorted(q.get(timeout=10) for _ in range(2))
    print("multicast stores used:", [r[3] for r in res])
    for rank, equal, err, _ in res:
        assert equal, f"rank {rank}: peer gather differs from the NCCL gather"
        assert err < 5e-3, f"rank {rank}: rel-L2 vs unsharded scan {err}"
