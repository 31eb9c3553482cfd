"""Allocation-free CRC-32 entry point, called through its exported C symbol.

mpcomm_crc32_blocks_noalloc serves callers that cannot allocate GPU memory
when they need a checksum (an engine that reserved all HBM for its own pool,
a latency-critical path that must not risk cudaMalloc's device sync, a plain
C caller without a CUDA allocator). Its scratch is a fixed __device__ array,
so the results must equal those of the allocating entry point
(mpcomm.ops.crc32_blocks) call after call. This file is named to be
collected last, and passes alone or after the rest of the suite.
"""
import ctypes

import pytest
import torch

import mpcomm
from mpcomm import ops

pytestmark = pytest.mark.gpu

MAX_WORDS = 65536  # MPCOMM_CRC32_NOALLOC_MAX_WORDS


def _entry():
    lib = ctypes.CDLL(mpcomm.native_library_path())
    fn = lib.mpcomm_crc32_blocks_noalloc
    fn.argtypes = [ctypes.c_void_p, ctypes.c_int64, ctypes.c_int64, ctypes.c_void_p, ctypes.c_void_p]
    fn.restype = ctypes.c_int
    return fn


def _call(fn, data, n, bs, out):
    stream = torch.cuda.current_stream().cuda_stream
    return fn(ctypes.c_void_p(data.data_ptr()), n, bs, ctypes.c_void_p(out.data_ptr()), ctypes.c_void_p(stream))


def test_noalloc_matches_allocating_entry_point_twice():
    fn = _entry()
    cases = [(6, (3 << 20) + 5, 11), (64, 4096, 12)]  # second call reuses the scratch
    for n, bs, seed in cases:
        g = torch.Generator(device="cuda").manual_seed(seed)
        data = torch.randint(0, 256, (n * bs,), dtype=torch.uint8, device="cuda", generator=g)
        out = torch.zeros(n, dtype=torch.int32, device="cuda")
        assert _call(fn, data, n, bs, out) == 0
        ref = ops.crc32_blocks(data, n)
        torch.cuda.synchronize()
        assert torch.equal(out, ref), (n, bs)


def test_noalloc_at_the_scratch_and_block_count_limits():
    """65,536 blocks of one piece each fill every scratch word (and pass the
    65,535 a grid's y extent allows); 65,535 blocks of an odd size sit just
    below. Both equal the allocating entry point."""
    fn = _entry()
    for n, bs, seed in [(MAX_WORDS, 4096, 21), (MAX_WORDS - 1, 4097, 22)]:
        g = torch.Generator(device="cuda").manual_seed(seed)
        data = torch.randint(0, 256, (n * bs,), dtype=torch.uint8, device="cuda", generator=g)
        out = torch.zeros(n, dtype=torch.int32, device="cuda")
        assert _call(fn, data, n, bs, out) == 0
        ref = ops.crc32_blocks(data, n)
        torch.cuda.synchronize()
        assert torch.equal(out, ref), (n, bs)
        del data


def test_noalloc_rejects_requests_beyond_scratch():
    fn = _entry()
    data = torch.zeros(16, dtype=torch.uint8, device="cuda")
    out = torch.zeros(1, dtype=torch.int32, device="cuda")
    stream = torch.cuda.current_stream().cuda_stream
    # 2 blocks x (MAX_WORDS/2 + 1) pieces of 512 KiB would need MAX_WORDS + 2
    # words; rejected before anything touches memory.
    bs = (MAX_WORDS // 2 + 1) * (512 << 10)
    rc = fn(ctypes.c_void_p(data.data_ptr()), 2, bs, ctypes.c_void_p(out.data_ptr()), ctypes.c_void_p(stream))
    assert rc == -1
    # One block more than the scratch has words (16-byte blocks): rejected.
    rc = fn(ctypes.c_void_p(data.data_ptr()), MAX_WORDS + 1, 16, ctypes.c_void_p(out.data_ptr()),
            ctypes.c_void_p(stream))
    assert rc == -1
    torch.cuda.synchronize()
