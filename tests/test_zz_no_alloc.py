"""The allocation-free prefix product, through the C ABI.

``mqc_prefix_prod_noalloc`` is for callers that cannot allocate device memory
while they run (a server that gives all device memory to its own allocator, a
process on a fixed device budget): its chunk products live in a fixed static
device array instead of a cudaMallocAsync buffer, with the chunk count capped
to what the array holds. This file is collected last so that, if it fails, a
run that stops at the first failure has already run every other test; it also
passes on its own in a fresh process.
"""

import pytest
import torch

from oracle import ref
from mambaqc_b200 import _lib
from tests.gpu_util import DEV, RTOL_BF16, RTOL_F32, gen, rel_l2

pytestmark = pytest.mark.gpu

# the static array's size, as documented in include/mambaqc_b200.h
NOALLOC_SCRATCH_BYTES = 4 << 20


def unit_quaternions(bsz, seqlen, lanes, seed):
    u = torch.randn(bsz, seqlen, lanes, 4, generator=gen(seed), dtype=torch.float64)
    return u / u.norm(dim=-1, keepdim=True)


def run(name, q):
    bsz, seqlen, lanes, _ = q.shape
    out = torch.empty_like(q)
    dtype = _lib.MQC_DTYPE_F32 if q.dtype == torch.float32 else _lib.MQC_DTYPE_BF16
    rc = getattr(_lib.load(), name)(q.data_ptr(), out.data_ptr(), bsz, seqlen, lanes, dtype,
                                    torch.cuda.current_stream().cuda_stream)
    assert rc == 0, _lib.load().mqc_last_error()
    return out


def time_chunks(bsz, seqlen, lanes):
    """Chunk count the entry point picks (mqc_prefix_prod's rule, capped by the array)."""
    sms = torch.cuda.get_device_properties(DEV).multi_processor_count
    have, want = bsz * lanes, sms * 256
    if have >= want or seqlen < 64:
        return 1
    n = min(-(-want // have), seqlen // 32, 1024, NOALLOC_SCRATCH_BYTES // (have * 16))
    if n <= 1:
        return 1
    chunk = -(-seqlen // n)
    return -(-seqlen // chunk)


def oracle(q64):
    bsz, seqlen, lanes, _ = q64.shape
    return ref.prefix_product(q64.view(bsz, seqlen, lanes, 1, 4)).view(bsz, seqlen, lanes, 4)


@pytest.mark.parametrize("dtype", [torch.float32, torch.bfloat16])
def test_noalloc_matches_allocating_entry_point_and_oracle_on_two_calls(dtype):
    # the first two shapes leave the GPU underfilled, so time is chunked and the
    # static array is used; the second call has other sizes and data, so stale
    # chunk products left by the first would show up
    shapes = [((1, 4096, 64), 1), ((2, 1000, 24), 2)]
    for (bsz, seqlen, lanes), seed in shapes:
        assert time_chunks(bsz, seqlen, lanes) > 1
        q64 = unit_quaternions(bsz, seqlen, lanes, seed)
        q = q64.to(DEV, dtype)
        expected = run("mqc_prefix_prod", q)
        got = run("mqc_prefix_prod_noalloc", q)
        torch.cuda.synchronize()
        # same chunking as the allocating entry point here: bit for bit
        assert torch.equal(got, expected)
        want = oracle(q.double().cpu())
        assert rel_l2(got, want) < (RTOL_F32 if dtype == torch.float32 else RTOL_BF16)
        assert torch.isfinite(got.float()).all()


def test_noalloc_serves_sizes_too_wide_for_chunking():
    """A wide, short problem runs as one pass over time (no scratch) and equals
    the allocating entry point and the oracle."""
    bsz, seqlen, lanes = 1, 64, 140000
    q64 = unit_quaternions(bsz, seqlen, lanes, 3)
    q = q64.to(DEV, torch.float32)
    got = run("mqc_prefix_prod_noalloc", q)
    expected = run("mqc_prefix_prod", q)
    torch.cuda.synchronize()
    assert rel_l2(got, expected) < 1e-6
    assert rel_l2(got, oracle(q64)) < RTOL_F32
