"""The host BlockManager against the oracle restatement of the reference (CPU).

Integer work is compared bit-exactly: block ids, tables, free-list order,
reference counts, slot mappings and the padded batch tables.
"""

import numpy as np
import pytest

from oracle import paging as op
from tinyvllm_b200.block_manager import BlockManager


def _state(bm):
    return (bm.free_blocks, bm.ref_counts, bm.seq_to_gpu, bm.block_tables, bm.seq_positions)


def test_reference_unit_cases():
    """tests/test_block_manager.py: counts, LIFO, OOM message, fork refcounts, lifecycle."""
    bm = BlockManager(num_gpus=2, blocks_per_gpu=4, block_size=16)
    assert bm.get_num_free_blocks() == 8 and bm.get_num_free_blocks(1) == 4
    bm.register_sequence(0, gpu_id=1)
    assert bm.get_block_table(0) == [] and bm.get_context_length(0) == 0
    assert bm.ensure_block_for_position(0, 40) == 1   # blocks 3, 2, 1 popped in order
    assert bm.get_block_table(0) == [3, 2, 1]
    assert bm.get_slot(0) == (1, 3, 0)
    bm.advance_position(0)
    assert bm.get_slot(0) == (1, 3, 1)
    with pytest.raises(RuntimeError, match="Out of KV cache memory!"):
        bm.ensure_block_for_position(0, 80)
    assert bm.get_block_table(0) == [3, 2, 1, 0]        # the last block was still taken
    bm.fork_sequence(0, 9)
    assert bm.ref_counts[1][2] == 2 and bm.get_gpu_for_seq(9) == 1
    bm.free_sequence(0)
    assert bm.get_num_free_blocks(1) == 0
    bm.free_sequence(9)
    assert bm.free_blocks[1] == [3, 2, 1, 0]


@pytest.mark.parametrize("seed", range(6))
def test_random_operation_sequences_match_oracle(seed):
    rng = np.random.default_rng(seed)
    a = BlockManager(2, 40, 16)
    b = op.OracleBlockManager(2, 40, 16)
    live, next_id = [], 0
    for _ in range(400):
        r = rng.random()
        try:
            if r < 0.15 or not live:
                g = int(rng.integers(0, 2))
                a.register_sequence(next_id, g)
                b.register_sequence(next_id, g)
                live.append(next_id)
                next_id += 1
            elif r < 0.45:
                s = live[int(rng.integers(0, len(live)))]
                pos = int(rng.integers(0, 120))
                ra = rb = None
                try:
                    ra = a.ensure_block_for_position(s, pos)
                except RuntimeError as e:
                    ra = str(e)
                try:
                    rb = b.ensure_block_for_position(s, pos)
                except RuntimeError as e:
                    rb = str(e)
                assert ra == rb
            elif r < 0.65:
                s = live[int(rng.integers(0, len(live)))]
                try:
                    sa = a.get_slot(s)
                except RuntimeError as e:
                    sa = str(e)
                try:
                    sb = b.get_slot(s)
                except RuntimeError as e:
                    sb = str(e)
                assert sa == sb
                a.advance_position(s)
                b.advance_position(s)
            elif r < 0.75 and live:
                s = live[int(rng.integers(0, len(live)))]
                a.fork_sequence(s, next_id)
                b.fork_sequence(s, next_id)
                live.append(next_id)
                next_id += 1
            else:
                s = live.pop(int(rng.integers(0, len(live))))
                a.free_sequence(s)
                b.free_sequence(s)
        finally:
            assert _state(a) == _state(b)
            if live:  # the dense table mirror agrees with the oracle's lists at any width
                w = int(rng.integers(1, 12))
                exp = np.zeros((len(live), w), dtype=np.int32)
                for i, sid in enumerate(live):
                    t = b.block_tables[sid][:w]
                    exp[i, :len(t)] = t
                assert np.array_equal(a.block_table_array(live, w), exp)


def test_slot_mapping_matches_chunked_prompt_writes():
    lens = [1, 15, 16, 17, 128, 500, 1024, 2048]
    a = BlockManager(1, 1024, 16)
    b = op.OracleBlockManager(1, 1024, 16)
    for sid, L in enumerate(lens):
        a.register_sequence(sid)
        b.register_sequence(sid)
        assert np.array_equal(a.slot_mapping(sid, 0, L), op.slot_mapping_for_prompt(b, sid, 0, L))
    assert _state(a) == _state(b)


def test_slot_mapping_from_offset_and_decode_slots():
    a = BlockManager(1, 64, 16)
    b = op.OracleBlockManager(1, 64, 16)
    for m in (a, b):
        m.register_sequence(0)
    assert np.array_equal(a.slot_mapping(0, 7, 40), op.slot_mapping_for_prompt(b, 0, 7, 40))
    a.advance_position(0, 47)
    for _ in range(47):
        b.advance_position(0)
    for _ in range(20):
        ga, blk, off = a.get_slot(0)
        assert (ga, blk, off) == b.get_slot(0)
        assert a.slot_mapping(0, a.get_context_length(0), 1)[0] == blk * 16 + off
        a.advance_position(0)
        b.advance_position(0)


def test_block_table_array_matches_engine_padding():
    a = BlockManager(1, 300, 16)
    b = op.OracleBlockManager(1, 300, 16)
    lens = [3, 40, 1100, 16, 17]
    for sid, L in enumerate(lens):
        for m in (a, b):
            m.register_sequence(sid)
            m.ensure_block_for_position(sid, L - 1)
    bt_ref, _ = op.prepare_batch_tables(b, list(range(5)), [L - 1 for L in lens], max_blocks=64)
    assert np.array_equal(a.block_table_array(range(5), 64), bt_ref)     # 1100 tokens -> truncated at 64
    assert a.block_table_array(range(5)).shape == (5, 69)


def test_oom_on_slot_mapping_keeps_reference_state():
    a = BlockManager(1, 3, 16)
    b = op.OracleBlockManager(1, 3, 16)
    a.register_sequence(0)
    b.register_sequence(0)
    with pytest.raises(RuntimeError, match="Out of KV cache memory!"):
        a.slot_mapping(0, 0, 60)
    with pytest.raises(RuntimeError, match="Out of KV cache memory!"):
        op.slot_mapping_for_prompt(b, 0, 0, 60)
    assert _state(a) == _state(b)
