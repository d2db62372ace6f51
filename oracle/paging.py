"""CPU oracle: restatement of tinyvllm's block bookkeeping and paged K/V writes.

TEST INFRASTRUCTURE ONLY (see ``oracle/attention.py``).  Integer work here is
the bit-exact reference for the product's slot mapping and table building.

* ``OracleBlockManager`` restates ``tinyvllm/core/block_manager.py:6-92``:
  per-GPU free lists created as ``list(range(N))`` and consumed with ``pop()``
  (so the first block handed out is ``N-1``), blocks returned with ``append``
  in block-table order, reference counts, fork by sharing.
* ``OracleKVCache`` restates ``tinyvllm/core/kv_cache.py:13-61`` on numpy
  arrays: one zero-initialised ``[N, bs, Hkv, D]`` pool per layer.
* ``write_prompt_kv`` restates ``Attention._write_kv_to_blocks``
  (``tinyvllm/model/llama.py:188-209``): chunked per block; layer 0 allocates
  through ``ensure_block_for_position``, later layers read the table.
* ``prepare_batch_tables`` restates ``LLMEngine._prepare_batch_tensors``
  (``tinyvllm/core/engine.py:235-255``): pad each table with block 0 to a
  fixed width (64 in the engine), truncate beyond it, ``ctx = pos + 1``.
"""

from __future__ import annotations

from typing import Dict, List, Optional, Tuple

import numpy as np


class OracleBlockManager:
    """block_manager.py:6-92, statement for statement."""

    def __init__(self, num_gpus: int, blocks_per_gpu: int, block_size: int):
        self.num_gpus = num_gpus
        self.blocks_per_gpu = blocks_per_gpu
        self.block_size = block_size
        self.free_blocks: Dict[int, List[int]] = {g: list(range(blocks_per_gpu)) for g in range(num_gpus)}
        self.ref_counts: Dict[int, Dict[int, int]] = {
            g: {b: 0 for b in range(blocks_per_gpu)} for g in range(num_gpus)}
        self.seq_to_gpu: Dict[int, int] = {}
        self.block_tables: Dict[int, List[int]] = {}
        self.seq_positions: Dict[int, int] = {}

    def register_sequence(self, seq_id: int, gpu_id: int = 0) -> None:
        self.seq_to_gpu[seq_id] = gpu_id
        self.block_tables[seq_id] = []
        self.seq_positions[seq_id] = 0

    def ensure_block_for_position(self, seq_id: int, pos: int) -> int:
        block_idx = pos // self.block_size
        while len(self.block_tables[seq_id]) <= block_idx:
            gpu_id = self.seq_to_gpu[seq_id]
            if len(self.free_blocks[gpu_id]) == 0:
                raise RuntimeError("Out of KV cache memory!")
            new_block = self.free_blocks[gpu_id].pop()
            self.ref_counts[gpu_id][new_block] = 1
            self.block_tables[seq_id].append(new_block)
        return self.block_tables[seq_id][block_idx]

    def get_slot(self, seq_id: int) -> Tuple[int, int, int]:
        pos = self.seq_positions[seq_id]
        block_id = self.ensure_block_for_position(seq_id, pos)
        return (self.seq_to_gpu[seq_id], block_id, pos % self.block_size)

    def advance_position(self, seq_id: int) -> None:
        self.seq_positions[seq_id] += 1

    def get_block_table(self, seq_id: int) -> List[int]:
        return self.block_tables[seq_id]

    def get_context_length(self, seq_id: int) -> int:
        return self.seq_positions[seq_id]

    def get_gpu_for_seq(self, seq_id: int) -> int:
        return self.seq_to_gpu[seq_id]

    def free_sequence(self, seq_id: int) -> None:
        gpu_id = self.seq_to_gpu[seq_id]
        for block in self.block_tables[seq_id]:
            self.ref_counts[gpu_id][block] -= 1
            if self.ref_counts[gpu_id][block] == 0:
                self.free_blocks[gpu_id].append(block)
        del self.seq_to_gpu[seq_id]
        del self.block_tables[seq_id]
        del self.seq_positions[seq_id]

    def get_num_free_blocks(self, gpu_id: Optional[int] = None) -> int:
        if gpu_id is None:
            return sum(len(b) for b in self.free_blocks.values())
        return len(self.free_blocks[gpu_id])

    def fork_sequence(self, src_seq_id: int, dst_seq_id: int) -> None:
        gpu_id = self.seq_to_gpu[src_seq_id]
        self.block_tables[dst_seq_id] = self.block_tables[src_seq_id].copy()
        self.seq_to_gpu[dst_seq_id] = gpu_id
        self.seq_positions[dst_seq_id] = self.seq_positions[src_seq_id]
        for block_id in self.block_tables[src_seq_id]:
            self.ref_counts[gpu_id][block_id] += 1


class OracleKVCache:
    """kv_cache.py:13-61 on numpy: zero-initialised per-layer pools."""

    def __init__(self, num_layers: int, num_blocks: int, block_size: int,
                 n_kv_heads: int, head_dim: int, dtype=np.float32):
        self.num_layers = num_layers
        self.num_blocks = num_blocks
        self.block_size = block_size
        self.n_kv_heads = n_kv_heads
        self.head_dim = head_dim
        self.dtype = np.dtype(dtype)
        shape = (num_blocks, block_size, n_kv_heads, head_dim)
        self.k_cache = [np.zeros(shape, dtype=self.dtype) for _ in range(num_layers)]
        self.v_cache = [np.zeros(shape, dtype=self.dtype) for _ in range(num_layers)]

    def write_kv(self, layer_idx: int, block_id: int, start_offset: int, k, v) -> None:
        end = start_offset + k.shape[0]
        self.k_cache[layer_idx][block_id, start_offset:end] = k
        self.v_cache[layer_idx][block_id, start_offset:end] = v

    def read_kv_blocks(self, layer_idx: int, block_ids: List[int], context_len: int):
        if not block_ids:
            z = np.zeros((0, self.n_kv_heads, self.head_dim), dtype=self.dtype)
            return z, z.copy()
        k = np.stack([self.k_cache[layer_idx][b] for b in block_ids]).reshape(-1, self.n_kv_heads, self.head_dim)
        v = np.stack([self.v_cache[layer_idx][b] for b in block_ids]).reshape(-1, self.n_kv_heads, self.head_dim)
        return k[:context_len], v[:context_len]

    def get_memory_bytes(self) -> int:
        return (self.num_layers * self.num_blocks * self.block_size * self.n_kv_heads
                * self.head_dim * 2) * self.dtype.itemsize


def write_prompt_kv(kv_cache: OracleKVCache, bm: OracleBlockManager, layer_idx: int,
                    seq_id: int, k, v, start_pos: int) -> None:
    """llama.py:188-209: write one sequence's K/V block chunk by block chunk."""
    seq_len = k.shape[0]
    bs = bm.block_size
    token_idx, pos = 0, start_pos
    while token_idx < seq_len:
        offset = pos % bs
        n = min(bs - offset, seq_len - token_idx)
        if layer_idx == 0:
            block_id = bm.ensure_block_for_position(seq_id, pos)
        else:
            block_id = bm.get_block_table(seq_id)[pos // bs]
        kv_cache.write_kv(layer_idx, block_id, offset, k[token_idx:token_idx + n], v[token_idx:token_idx + n])
        token_idx += n
        pos += n


def slot_mapping_for_prompt(bm: OracleBlockManager, seq_id: int, start_pos: int, n_tokens: int) -> np.ndarray:
    """Flat slot ``block * bs + pos % bs`` of each prompt token (llama.py:203-209), allocating
    blocks exactly as layer 0 of ``_write_kv_to_blocks`` does."""
    bs = bm.block_size
    out = np.empty(n_tokens, dtype=np.int64)
    for i in range(n_tokens):
        pos = start_pos + i
        blk = bm.ensure_block_for_position(seq_id, pos)
        out[i] = blk * bs + pos % bs
    return out


def prepare_batch_tables(bm: OracleBlockManager, seq_ids: List[int], start_positions: List[int],
                         max_blocks: int = 64) -> Tuple[np.ndarray, np.ndarray]:
    """engine.py:235-255: 0-padded/truncated int32 tables of width ``max_blocks``; ctx = pos + 1."""
    b = len(seq_ids)
    bt = np.zeros((b, max_blocks), dtype=np.int32)
    ctx = np.zeros(b, dtype=np.int32)
    for i, (sid, sp) in enumerate(zip(seq_ids, start_positions)):
        t = bm.get_block_table(sid)
        for j in range(max_blocks):
            bt[i, j] = t[j] if j < len(t) else 0
        ctx[i] = sp + 1
    return bt, ctx
