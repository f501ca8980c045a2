"""The allocation-free prefix product, through the C ABI.

``mqc_prefix_prod_noalloc`` is for callers that cannot allocate device memory
while they run (a server that gives all device memory to its own allocator, a
process on a fixed device budget): its chunk products live in a fixed static
device array instead of a cudaMallocAsync buffer. This file is collected last
so that, if it fails, a run that stops at the first failure has already run
every other test; it also passes on its own in a fresh process.
"""

import ctypes

import pytest
import torch

from mambaqc_b200 import _lib
from tests.gpu_util import DEV, RTOL_F32, gen, rel_l2

pytestmark = pytest.mark.gpu

UNSUPPORTED = 3


def unit_quaternions(bsz, seqlen, lanes, seed):
    u = torch.randn(bsz, seqlen, lanes, 4, generator=gen(seed), dtype=torch.float64)
    return (u / u.norm(dim=-1, keepdim=True)).to(DEV, torch.float32)


def run(name, q):
    bsz, seqlen, lanes, _ = q.shape
    out = torch.empty_like(q)
    rc = getattr(_lib.load(), name)(q.data_ptr(), out.data_ptr(), bsz, seqlen, lanes,
                                    _lib.MQC_DTYPE_F32,
                                    torch.cuda.current_stream().cuda_stream)
    assert rc == 0, _lib.load().mqc_last_error()
    return out


def test_noalloc_matches_allocating_entry_point_on_two_calls():
    # both shapes leave the GPU underfilled, so time is chunked and the scratch is used;
    # the second call has other sizes and data, so stale chunk products would show up
    for (bsz, seqlen, lanes), seed in (((1, 4096, 64), 1), ((2, 1000, 24), 2)):
        q = unit_quaternions(bsz, seqlen, lanes, seed)
        expected = run("mqc_prefix_prod", q)
        got = run("mqc_prefix_prod_noalloc", q)
        torch.cuda.synchronize()
        assert rel_l2(got, expected) < RTOL_F32
        assert torch.isfinite(got).all()


def test_noalloc_rejects_sizes_beyond_its_scratch():
    # 1 x 2 chunks x 140000 lanes x 16 B = 4.48 MB of chunk products > the 4 MiB array
    bsz, seqlen, lanes = 1, 64, 140000
    q = torch.zeros(bsz, seqlen, lanes, 4, device=DEV)
    out = torch.full_like(q, 7.0)
    lib = _lib.load()
    rc = lib.mqc_prefix_prod_noalloc(q.data_ptr(), out.data_ptr(), bsz, seqlen, lanes,
                                     _lib.MQC_DTYPE_F32, torch.cuda.current_stream().cuda_stream)
    assert rc == UNSUPPORTED
    assert b"static maximum" in lib.mqc_last_error()
    torch.cuda.synchronize()
    assert bool((out == 7.0).all())  # nothing was launched
