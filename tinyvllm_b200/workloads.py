"""Seeded synthetic inputs for the benchmark configurations of the hot path.

There is no public dataset behind any of these: every input is drawn from
fixed seeds (``1234 + config index``) with the shapes and value distributions
the benchmark configurations name.  Lengths and block draws use numpy's
``default_rng``; tensor values use a torch generator on the target device.

* config 1 -- paged decode, fp32, TinyLlama heads (32/4, D=64), 4 sequences of
  context {17, 64, 130, 255}, pool of 128 blocks, tables drawn from a seeded
  permutation of the pool without replacement, padded with block 0.
* config 2 -- causal prefill, fp16, 8 prompts L in {1,15,16,17,128,500,1024,2048},
  32/4 heads, D=64, paged write into a fresh 1024-block pool.
* config 3 -- paged decode at scale, fp16, 32/8 heads, D=128, 256 sequences with
  context ~ U{128..4096}, pool 1.2x the blocks needed, random non-contiguous tables.
"""

from __future__ import annotations

import math
from dataclasses import dataclass
from typing import List, Optional

import numpy as np
import torch

SEED_BASE = 1234


@dataclass
class DecodeCase:
    q: torch.Tensor             # [B,1,Hq,D]
    k_cache: torch.Tensor       # [N,bs,Hkv,D]
    v_cache: torch.Tensor
    block_tables: torch.Tensor  # int32 [B,max_blocks]
    context_lens: torch.Tensor  # int32 [B]
    n_heads: int
    n_kv_heads: int
    head_dim: int
    block_size: int

    @property
    def batch(self) -> int:
        return self.q.shape[0]

    def kv_bytes(self) -> int:
        """Algorithmic K+V bytes one call must read: live tokens only."""
        es = self.k_cache.element_size()
        ctx = self.context_lens.to("cpu", torch.int64)
        width = self.block_tables.shape[1] * self.block_size
        return int(ctx.clamp(max=width).sum()) * self.n_kv_heads * self.head_dim * es * 2

    def algorithmic_bytes(self) -> int:
        """K/V of live tokens + q in + out + the table rows and lengths."""
        es = self.k_cache.element_size()
        qo = 2 * self.q.numel() * es
        ctx = self.context_lens.to("cpu", torch.int64)
        tbl = int(((ctx + self.block_size - 1) // self.block_size).clamp(
            max=self.block_tables.shape[1]).sum()) * 4 + self.batch * 4
        return self.kv_bytes() + qo + tbl


def _tables_from_pool(rng: np.random.Generator, num_blocks: int, ctx: np.ndarray, block_size: int,
                      width: Optional[int] = None) -> np.ndarray:
    need = (ctx + block_size - 1) // block_size
    width = int(need.max()) if width is None else width
    perm = rng.permutation(num_blocks)
    bt = np.zeros((len(ctx), width), dtype=np.int32)
    off = 0
    for i, n in enumerate(need):
        bt[i, :n] = perm[off:off + n]
        off += n
    return bt


def _randn(shape, dtype, device, gen) -> torch.Tensor:
    return torch.randn(shape, generator=gen, device=device, dtype=torch.float32).to(dtype)


def decode_config1(device="cuda") -> DecodeCase:
    rng = np.random.default_rng(SEED_BASE + 1)
    gen = torch.Generator(device=device).manual_seed(SEED_BASE + 1)
    B, Hq, Hkv, D, bs, N = 4, 32, 4, 64, 16, 128
    ctx = np.array([17, 64, 130, 255], dtype=np.int32)
    bt = _tables_from_pool(rng, N, ctx, bs, width=16)
    return DecodeCase(
        q=_randn((B, 1, Hq, D), torch.float32, device, gen),
        k_cache=_randn((N, bs, Hkv, D), torch.float32, device, gen),
        v_cache=_randn((N, bs, Hkv, D), torch.float32, device, gen),
        block_tables=torch.from_numpy(bt).to(device),
        context_lens=torch.from_numpy(ctx).to(device),
        n_heads=Hq, n_kv_heads=Hkv, head_dim=D, block_size=bs)


def decode_config3(device="cuda", batch: int = 256, dtype=torch.float16, ctx_lo: int = 128,
                   ctx_hi: int = 4096, seed_offset: int = 0, shared_contexts: bool = False) -> DecodeCase:
    """Config 3's decode batch.  ``seed_offset`` reseeds the values and the tables;
    with ``shared_contexts`` the context lengths stay those of offset 0, so that
    every rank of a weak-scaling run holds the same amount of K/V."""
    rng = np.random.default_rng(SEED_BASE + 3 + seed_offset)
    gen = torch.Generator(device=device).manual_seed(SEED_BASE + 3 + seed_offset)
    Hq, Hkv, D, bs = 32, 8, 128, 16
    ctx_rng = np.random.default_rng(SEED_BASE + 3) if (shared_contexts and seed_offset) else rng
    ctx = ctx_rng.integers(ctx_lo, ctx_hi + 1, size=batch).astype(np.int32)
    need = (ctx + bs - 1) // bs
    N = int(math.ceil(1.2 * int(need.sum())))
    bt = _tables_from_pool(rng, N, ctx, bs)
    return DecodeCase(
        q=_randn((batch, 1, Hq, D), dtype, device, gen),
        k_cache=_randn((N, bs, Hkv, D), dtype, device, gen),
        v_cache=_randn((N, bs, Hkv, D), dtype, device, gen),
        block_tables=torch.from_numpy(bt).to(device),
        context_lens=torch.from_numpy(ctx).to(device),
        n_heads=Hq, n_kv_heads=Hkv, head_dim=D, block_size=bs)


def decode_case(batch: int, n_heads: int, n_kv_heads: int, head_dim: int, block_size: int,
                ctx: List[int], dtype=torch.float16, device="cuda", seed: int = 0,
                extra_blocks: int = 5, width: Optional[int] = None,
                contiguous: bool = False) -> DecodeCase:
    """A general seeded decode case: shuffled (or contiguous) tables, ragged contexts."""
    rng = np.random.default_rng(seed)
    gen = torch.Generator(device=device).manual_seed(seed)
    ctx_a = np.asarray(ctx, dtype=np.int32)
    need = np.maximum((ctx_a + block_size - 1) // block_size, 0)
    N = int(need.sum()) + extra_blocks
    if contiguous:
        w = int(need.max()) if width is None else width
        bt = np.zeros((batch, w), dtype=np.int32)
        off = 0
        for i, n in enumerate(need):
            bt[i, :n] = np.arange(off, off + n)
            off += n
    else:
        bt = _tables_from_pool(rng, N, ctx_a, block_size, width)
    return DecodeCase(
        q=_randn((batch, 1, n_heads, head_dim), dtype, device, gen),
        k_cache=_randn((N, block_size, n_kv_heads, head_dim), dtype, device, gen),
        v_cache=_randn((N, block_size, n_kv_heads, head_dim), dtype, device, gen),
        block_tables=torch.from_numpy(bt).to(device),
        context_lens=torch.from_numpy(ctx_a).to(device),
        n_heads=n_heads, n_kv_heads=n_kv_heads, head_dim=head_dim, block_size=block_size)
