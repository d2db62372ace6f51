"""KV-cache block bookkeeping on the host (integer work, bit-exact with the reference).

``BlockManager`` keeps the API and the allocation order of
``tinyvllm/core/block_manager.py:6-92``: per-GPU LIFO free lists created as
``range(N)`` (so the first block handed out is ``N-1``), blocks returned in
block-table order when a sequence is freed, reference counts shared by
``fork_sequence``, and ``RuntimeError("Out of KV cache memory!")`` when a
list runs dry.  On top of that it produces the device-side inputs of the
kernels in one vectorised step instead of per-token Python loops:

* ``slot_mapping(seq_id, start_pos, n)`` -- flat slots (``block*bs + pos%bs``)
  of ``n`` consecutive positions, allocating blocks in exactly the order the
  reference's per-chunk ``ensure_block_for_position`` calls do
  (``tinyvllm/model/llama.py:188-209``);
* ``block_table_array(seq_ids, width)`` -- the padded ``int32 [B, width]``
  table of ``LLMEngine._prepare_batch_tensors`` (``core/engine.py:235-255``):
  block 0 as padding, truncated at ``width``.
"""

from __future__ import annotations

from typing import Dict, List, Optional, Sequence, Tuple

import numpy as np


class BlockManager:
    def __init__(self, num_gpus: int, blocks_per_gpu: int, block_size: int):
        self.num_gpus = num_gpus
        self.blocks_per_gpu = blocks_per_gpu
        self.block_size = block_size
        self.free_blocks: Dict[int, List[int]] = {g: list(range(blocks_per_gpu)) for g in range(num_gpus)}
        self.ref_counts: Dict[int, Dict[int, int]] = {
            g: dict.fromkeys(range(blocks_per_gpu), 0) for g in range(num_gpus)}
        self.seq_to_gpu: Dict[int, int] = {}
        self.block_tables: Dict[int, List[int]] = {}
        self.seq_positions: Dict[int, int] = {}

    # -- reference API ---------------------------------------------------------
    def register_sequence(self, seq_id: int, gpu_id: int = 0) -> None:
        self.seq_to_gpu[seq_id] = gpu_id
        self.block_tables[seq_id] = []
        self.seq_positions[seq_id] = 0

    def ensure_block_for_position(self, seq_id: int, pos: int) -> int:
        table = self.block_tables[seq_id]
        need = pos // self.block_size + 1
        if len(table) < need:
            self._grow(seq_id, need)
        return table[pos // self.block_size]

    def get_slot(self, seq_id: int) -> Tuple[int, int, int]:
        pos = self.seq_positions[seq_id]
        block_id = self.ensure_block_for_position(seq_id, pos)
        return (self.seq_to_gpu[seq_id], block_id, pos % self.block_size)

    def advance_position(self, seq_id: int, n: int = 1) -> None:
        self.seq_positions[seq_id] += n

    def get_block_table(self, seq_id: int) -> List[int]:
        return self.block_tables[seq_id]

    def get_context_length(self, seq_id: int) -> int:
        return self.seq_positions[seq_id]

    def get_gpu_for_seq(self, seq_id: int) -> int:
        return self.seq_to_gpu[seq_id]

    def free_sequence(self, seq_id: int) -> None:
        gpu_id = self.seq_to_gpu[seq_id]
        refs = self.ref_counts[gpu_id]
        free = self.free_blocks[gpu_id]
        for block in self.block_tables[seq_id]:
            refs[block] -= 1
            if refs[block] == 0:
                free.append(block)
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
        refs = self.ref_counts[gpu_id]
        for block_id in self.block_tables[src_seq_id]:
            refs[block_id] += 1

    # -- vectorised helpers for the kernels -------------------------------------
    def _grow(self, seq_id: int, n_blocks: int) -> None:
        """Append blocks to the table until it has ``n_blocks``, popping the free
        list one block at a time as the reference does (the error is raised at
        the first block that cannot be had, leaving earlier pops in place)."""
        table = self.block_tables[seq_id]
        gpu_id = self.seq_to_gpu[seq_id]
        free = self.free_blocks[gpu_id]
        refs = self.ref_counts[gpu_id]
        while len(table) < n_blocks:
            if not free:
                raise RuntimeError("Out of KV cache memory!")
            b = free.pop()
            refs[b] = 1
            table.append(b)

    def slot_mapping(self, seq_id: int, start_pos: int, n: int) -> np.ndarray:
        """int64 flat slots of positions ``start_pos .. start_pos+n-1``, allocating
        any blocks they need."""
        if n <= 0:
            return np.zeros(0, dtype=np.int64)
        bs = self.block_size
        last = start_pos + n - 1
        self.ensure_block_for_position(seq_id, last)
        table = np.asarray(self.block_tables[seq_id], dtype=np.int64)
        pos = np.arange(start_pos, start_pos + n, dtype=np.int64)
        return table[pos // bs] * bs + pos % bs

    def block_table_array(self, seq_ids: Sequence[int], width: Optional[int] = None,
                          out: Optional[np.ndarray] = None) -> np.ndarray:
        """int32 [len(seq_ids), width] tables padded with block 0 and truncated at
        ``width`` (default: the longest table)."""
        tables = [self.block_tables[s] for s in seq_ids]
        if width is None:
            width = max((len(t) for t in tables), default=1) or 1
        if out is None:
            out = np.zeros((len(tables), width), dtype=np.int32)
        else:
            out[:len(tables), :width] = 0
        for i, t in enumerate(tables):
            n = min(len(t), width)
            out[i, :n] = t[:n]
        return out
