"""The synthetic workloads the bench and the parity tests draw (CPU)."""

import torch

from tinyvllm_b200 import workloads


def test_config3_ranks_share_contexts_but_not_values():
    """bench.py --gpus N gives every rank config 3's context lengths (the same K/V
    bytes per GPU) with its own queries, K/V values and tables."""
    a = workloads.decode_config3("cpu", batch=32)
    b = workloads.decode_config3("cpu", batch=32, seed_offset=3, shared_contexts=True)
    c = workloads.decode_config3("cpu", batch=32, seed_offset=3)
    assert torch.equal(a.context_lens, b.context_lens)
    assert not torch.equal(a.q, b.q)
    assert not torch.equal(a.block_tables, b.block_tables)
    assert not torch.equal(a.context_lens, c.context_lens)
    # offset 0 is config 3 itself whichever way it is asked for
    d = workloads.decode_config3("cpu", batch=32, shared_contexts=True)
    assert torch.equal(a.q, d.q) and torch.equal(a.block_tables, d.block_tables)
    for case in (a, b):
        ctx = case.context_lens
        assert int(ctx.min()) >= 128 and int(ctx.max()) <= 4096
        # every table row covers its own context with distinct blocks
        need = (ctx + 15) // 16
        for r in range(case.batch):
            row = case.block_tables[r, :int(need[r])]
            assert len(set(row.tolist())) == int(need[r])
