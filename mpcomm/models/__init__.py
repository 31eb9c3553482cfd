"""Workload shapes used by the benchmarks (data layouts, not neural models).

* ``KVPoolSpec``   — paged KV-cache pool of a decoder (default Llama-3-8B:
                     32 layers x 8 KV heads x head_dim 128, 16-token pages,
                     bf16, K+V): one page of one layer = 2*8*128*16*2 bytes
                     = 64 KiB, the block the H2D movers copy.
* ``RolloutBatch`` — RL rollout / R3 batch: int32 expert IDs [tokens, top_k]
                     plus variable-length int32 token sequences (lognormal
                     lengths), packed into one contiguous byte buffer.
"""
from __future__ import annotations

from dataclasses import dataclass

import torch

__all__ = ["KVPoolSpec", "LLAMA3_8B_KV", "RolloutBatch"]


@dataclass(frozen=True)
class KVPoolSpec:
    layers: int = 32
    kv_heads: int = 8
    head_dim: int = 128
    page_tokens: int = 16
    dtype_bytes: int = 2  # bf16

    @property
    def page_bytes(self) -> int:
        """Bytes of one page of one layer, K and V."""
        return 2 * self.kv_heads * self.head_dim * self.page_tokens * self.dtype_bytes

    def make_pool(self, pages: int, seed: int = 0, pinned: bool = True) -> torch.Tensor:
        """[pages, page_bytes] uint8 view of bf16 values ~ N(0, 1)."""
        g = torch.Generator().manual_seed(seed)
        elems = self.page_bytes // self.dtype_bytes
        pool = torch.empty((pages, elems), dtype=torch.bfloat16, pin_memory=pinned)
        chunk = max(1, (256 << 20) // self.page_bytes)
        for s in range(0, pages, chunk):
            e = min(pages, s + chunk)
            pool[s:e].copy_(torch.randn((e - s, elems), generator=g, dtype=torch.float32))
        return pool.view(torch.uint8).view(pages, self.page_bytes)

    def sample_pages(self, pages: int, n: int, seed: int) -> torch.Tensor:
        """n page indices drawn uniformly without replacement."""
        g = torch.Generator().manual_seed(seed)
        return torch.randperm(pages, generator=g)[:n].to(torch.int64)


LLAMA3_8B_KV = KVPoolSpec()


@dataclass
class RolloutBatch:
    """Expert-ID + token batch of an RL rollout step (packed, 16-byte padded)."""

    tokens: int = 1 << 20
    top_k: int = 8
    num_experts: int = 256
    sequences: int = 4096
    len_mu: float = 7.0
    len_sigma: float = 0.8
    min_len: int = 16
    max_len: int = 32768

    def make(self, seed: int = 4) -> tuple[torch.Tensor, torch.Tensor, torch.Tensor]:
        """Returns (packed uint8 buffer, expert_ids int32 [tokens, top_k], seq lengths int64)."""
        g = torch.Generator().manual_seed(seed)
        ids = torch.randint(0, self.num_experts, (self.tokens, self.top_k), dtype=torch.int32, generator=g)
        normal = torch.randn(self.sequences, generator=g, dtype=torch.float64)
        lens = torch.exp(self.len_mu + self.len_sigma * normal).round().clamp(self.min_len, self.max_len)
        lens = lens.to(torch.int64)
        toks = torch.randint(0, 1 << 31, (int(lens.sum()),), dtype=torch.int32, generator=g)
        raw = torch.cat([ids.view(-1).view(torch.uint8), lens.to(torch.int32).view(torch.uint8),
                         toks.view(torch.uint8)])
        pad = (-raw.numel()) % 16
        if pad:
            raw = torch.cat([raw, torch.zeros(pad, dtype=torch.uint8)])
        return raw, ids, lens
