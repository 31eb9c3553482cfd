"""Tensor-level wrappers of mpcomm's sm_100a kernels.

Every function launches this package's own CUDA kernels (no torch or
library copy on the data path) on the caller's current CUDA stream unless a
stream is given, and raises on a launch error. There is no CPU fallback: on
a host without the native module or a GPU these functions raise.

  paged_gather(pool, indices, out=None)   out[i] = pool[indices[i]]
  paged_scatter(src, indices, pool)       pool[indices[i]] = src[i]
  crc32_blocks(tensor, num_blocks)        zlib CRC-32 of each block
  copy_spans(srcs, dsts, lengths)         raw device copy of up to 64 spans
  pxn_gather_forward(...)                 fused gather + forward (peer dst)
  gather_bcast(...)                       fused host-page gather + broadcast
                                          (NVLS multimem or P2P bulk stores)
  nvls_broadcast(src, mc_ptr)             multimem.st broadcast
  p2p_fanout(src, dst_ptrs)               store the same bytes to peers

``pool`` may be pinned host memory (page-locked CPU tensor: the GPU reads it
over PCIe through UVA) or device memory.
"""
from __future__ import annotations

from typing import Optional, Sequence

import torch

from .. import _native

MODE_AUTO, MODE_SM, MODE_TMA = 0, 1, 2

__all__ = [
    "MODE_AUTO", "MODE_SM", "MODE_TMA", "paged_gather", "paged_scatter", "crc32_blocks",
    "copy_spans", "pxn_gather_forward", "gather_bcast", "nvls_broadcast", "p2p_fanout", "wait_flag",
    "crc32_host",
]


def _stream_ptr(stream: Optional[torch.cuda.Stream]) -> int:
    s = stream if stream is not None else torch.cuda.current_stream()
    return int(s.cuda_stream)


def _check(err: int, what: str) -> None:
    if err != 0:
        raise RuntimeError(f"mpcomm {what} failed with CUDA error {err}")


def _block_view(t: torch.Tensor) -> tuple[int, int]:
    if t.dim() < 2:
        raise ValueError("expected a [num_blocks, ...] tensor")
    if not t.is_contiguous():
        raise ValueError("tensor must be contiguous")
    n = t.shape[0]
    return n, t.numel() * t.element_size() // n


def paged_gather(pool: torch.Tensor, indices: torch.Tensor, out: Optional[torch.Tensor] = None,
                 mode: int = MODE_AUTO, max_ctas: int = 0,
                 stream: Optional[torch.cuda.Stream] = None) -> torch.Tensor:
    """Gathers whole blocks (first dimension) of ``pool`` into ``out``."""
    pool_blocks, bs = _block_view(pool)
    if indices.dtype != torch.int64 or not indices.is_cuda:
        raise ValueError("indices must be an int64 CUDA tensor")
    n = indices.numel()
    if out is None:
        out = torch.empty((n,) + tuple(pool.shape[1:]), dtype=pool.dtype, device=indices.device)
    if out.numel() * out.element_size() != n * bs:
        raise ValueError("out has the wrong size")
    err, _, _ = _native.paged_gather(pool.data_ptr(), pool_blocks, indices.data_ptr(), out.data_ptr(),
                                     n, bs, mode, max_ctas, _stream_ptr(stream))
    _check(err, "paged_gather")
    return out


def paged_scatter(src: torch.Tensor, indices: torch.Tensor, pool: torch.Tensor,
                  mode: int = MODE_AUTO, max_ctas: int = 0,
                  stream: Optional[torch.cuda.Stream] = None) -> torch.Tensor:
    """Scatters the blocks of ``src`` into ``pool`` at ``indices``."""
    pool_blocks, bs = _block_view(pool)
    n = indices.numel()
    if src.numel() * src.element_size() != n * bs:
        raise ValueError("src has the wrong size")
    err, _, _ = _native.paged_scatter(src.data_ptr(), indices.data_ptr(), pool.data_ptr(), pool_blocks,
                                      n, bs, mode, max_ctas, _stream_ptr(stream))
    _check(err, "paged_scatter")
    return pool


def crc32_blocks(t: torch.Tensor, num_blocks: int, out: Optional[torch.Tensor] = None,
                 stream: Optional[torch.cuda.Stream] = None) -> torch.Tensor:
    """CRC-32 (zlib polynomial) of ``num_blocks`` equal blocks of ``t``'s bytes."""
    nbytes = t.numel() * t.element_size()
    if nbytes % num_blocks:
        raise ValueError("tensor bytes not divisible by num_blocks")
    if out is None:
        out = torch.empty(num_blocks, dtype=torch.int32, device=t.device)
    _check(_native.crc32_blocks(t.data_ptr(), num_blocks, nbytes // num_blocks, out.data_ptr(),
                                _stream_ptr(stream)), "crc32_blocks")
    return out


def crc32_host(data: bytes, crc: int = 0) -> int:
    """Host CRC-32 (same polynomial/conventions as zlib.crc32)."""
    return _native.crc32_host(data, crc)


def copy_spans(srcs: Sequence[int], dsts: Sequence[int], lengths: Sequence[int], max_ctas: int = 0,
               stream: Optional[torch.cuda.Stream] = None, mode: int = MODE_AUTO, gate: int = 0,
               gate_budget_ns: int = 0) -> None:
    """Copies up to 64 spans in one launch (bulk pipeline, or the vector SM
    kernel with ``mode=MODE_SM``); any device-reachable addresses. ``gate``
    (a device uint32 address) makes every pipeline pause before its next
    tile while the word is non-zero, for at most ``gate_budget_ns`` in total
    per pipeline (the QoS yield of background copies)."""
    _check(_native.copy_spans(list(srcs), list(dsts), list(lengths), max_ctas, _stream_ptr(stream), mode,
                              gate, gate_budget_ns), "copy_spans")


def pxn_gather_forward(pool_ptr: int, pool_blocks: int, indices: torch.Tensor, dst_ptr: int,
                       block_size: int, done_flag: int = 0, flag_value: int = 1, counter: int = 0,
                       max_ctas: int = 0, stream: Optional[torch.cuda.Stream] = None) -> None:
    _check(_native.pxn_gather_forward(pool_ptr, pool_blocks, indices.data_ptr(), dst_ptr,
                                      indices.numel(), block_size, max_ctas, _stream_ptr(stream),
                                      done_flag, flag_value, counter), "pxn_gather_forward")


def gather_bcast(pool_ptr: int, pool_blocks: int, indices: torch.Tensor, block_size: int, mc_ptr: int = 0,
                 dst_ptrs: Sequence[int] = (), mc_flag: int = 0, flags: Sequence[int] = (), flag_value: int = 1,
                 counter: int = 0, max_ctas: int = 0, stream: Optional[torch.cuda.Stream] = None,
                 status_ptr: int = 0) -> None:
    """One launch that gathers ``indices`` pages of ``block_size`` bytes from
    a host pool (device-visible pointer) and delivers page i to byte offset
    ``i * block_size`` of every consumer GPU, without staging the batch in
    local HBM: ``multimem.st`` to ``mc_ptr`` (NVLS multicast address; every
    bound GPU receives it) or, with ``mc_ptr == 0``, bulk stores to each of
    ``dst_ptrs`` (<= 8 local or IPC-mapped peer buffers).

    Completion: with ``mc_ptr`` and ``mc_flag`` (multicast address of a
    64-bit word), every bound GPU's copy of that word is incremented once the
    whole batch has been stored; without multicast, ``flag_value`` is stored
    to each address in ``flags``. ``counter`` is a zeroed int32 device word
    (required with a flag). Consumers wait with :func:`wait_flag`.
    """
    if indices.dtype != torch.int64 or not indices.is_cuda:
        raise ValueError("indices must be an int64 CUDA tensor")
    _check(_native.gather_bcast(pool_ptr, pool_blocks, indices.data_ptr(), indices.numel(), block_size, mc_ptr,
                                list(dst_ptrs), mc_flag, list(flags), flag_value, counter, max_ctas,
                                _stream_ptr(stream), status_ptr), "gather_bcast")


def nvls_broadcast(src: torch.Tensor, mc_ptr: int, nbytes: Optional[int] = None, max_ctas: int = 0,
                   stream: Optional[torch.cuda.Stream] = None) -> None:
    n = src.numel() * src.element_size() if nbytes is None else nbytes
    _check(_native.nvls_broadcast(src.data_ptr(), mc_ptr, n, max_ctas, _stream_ptr(stream)), "nvls_broadcast")


def p2p_fanout(src: torch.Tensor, dst_ptrs: Sequence[int], nbytes: Optional[int] = None, max_ctas: int = 0,
               stream: Optional[torch.cuda.Stream] = None) -> None:
    n = src.numel() * src.element_size() if nbytes is None else nbytes
    _check(_native.p2p_fanout(src.data_ptr(), list(dst_ptrs), n, max_ctas, _stream_ptr(stream)), "p2p_fanout")


def wait_flag(flag_ptr: int, value: int, budget_ns: int, status_ptr: int = 0,
              stream: Optional[torch.cuda.Stream] = None) -> None:
    _check(_native.wait_flag(flag_ptr, value, budget_ns, _stream_ptr(stream), status_ptr), "wait_flag")
