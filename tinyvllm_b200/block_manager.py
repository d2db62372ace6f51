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
  block 0 as padding, truncated at ``width``.  Every registered sequence also
  owns a row of a dense int32 array that mirrors its block list (zeros past
  its end), so a batch's table is one gather instead of a per-sequence copy.
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
        # dense mirror of the block lists: one int32 row per registered sequence
        self._rows = np.zeros((64, 64), dtype=np.int32)
        self._row_of: Dict[int, int] = {}
        self._free_rows: List[int] = list(range(63, -1, -1))

    def _take_row(self, seq_id: int) -> int:
        if not self._free_rows:
            n = self._rows.shape[0]
            self._rows = np.concatenate([self._rows, np.zeros_like(self._rows)], axis=0)
            self._free_rows = list(range(2 * n - 1, n - 1, -1))
        r = self._free_rows.pop()
        self._row_of[seq_id] = r
        return r

    def _mirror(self, seq_id: int, start: int) -> None:
        """Copy block-list entries from ``start`` on into the sequence's row."""
        table = self.block_tables[seq_id]
        if len(table) > self._rows.shape[1]:
            w = self._rows.shape[1]
            while w < len(table):
                w *= 2
            self._rows = np.pad(self._rows, ((0, 0), (0, w - self._rows.shape[1])))
        self._rows[self._row_of[seq_id], start:len(table)] = table[start:]

    # -- reference API ---------------------------------------------------------
    def register_sequence(self, seq_id: int, gpu_id: int = 0) -> None:
        if seq_id in self._row_of:           # re-registered: start from an empty row
            self._release_row(seq_id)
        self.seq_to_gpu[seq_id] = gpu_id
        self.block_tables[seq_id] = []
        self.seq_positions[seq_id] = 0
        self._take_row(seq_id)

    def _release_row(self, seq_id: int) -> None:
        r = self._row_of.pop(seq_id)
        self._rows[r, :] = 0
        self._free_rows.append(r)

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
        self._release_row(seq_id)

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
        if dst_seq_id in self._row_of:
            self._release_row(dst_seq_id)
        self._take_row(dst_seq_id)
        self._mirror(dst_seq_id, 0)

    # -- vectorised helpers for the kernels -------------------------------------
    def _grow(self, seq_id: int, n_blocks: int) -> None:
        """Append blocks to the table until it has ``n_blocks``, popping the free
        list one block at a time as the reference does (the error is raised at
        the first block that cannot be had, leaving earlier pops in place)."""
        table = self.block_tables[seq_id]
        gpu_id = self.seq_to_gpu[seq_id]
        free = self.free_blocks[gpu_id]
        refs = self.ref_counts[gpu_id]
        start = len(table)
        try:
            while len(table) < n_blocks:
                if not free:
                    raise RuntimeError("Out of KV cache memory!")
                b = free.pop()
                refs[b] = 1
                table.append(b)
        finally:
            if seq_id in self._row_of and len(table) > start:
                self._mirror(seq_id, start)

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
        if width is None:
            width = max((len(self.block_tables[s]) for s in seq_ids), default=1) or 1
        rows = np.fromiter((self._row_of[s] for s in seq_ids), dtype=np.int64, count=len(seq_ids))
        w = min(width, self._rows.shape[1])
        if out is None:
            out = np.zeros((len(rows), width), dtype=np.int32)
        else:
            out[:len(rows), :width] = 0
        out[:len(rows), :w] = self._rows[rows, :w]
        return out
