"""Generate the golden fixtures in this folder from the CPU oracle.

    python tests/golden/make_golden.py

The reference (tinygrad) cannot run in this image, so the expected outputs
come from the numpy restatement in ``oracle/``; the oracle itself is pinned
against the reference tests' known answers in ``tests/test_oracle.py``.
Inputs are drawn from numpy generators with fixed seeds; float values are
rounded to float16 before use so the fixtures stay small and exact.
"""

from __future__ import annotations

import sys
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent
sys.path.insert(0, str(HERE.parent.parent))

from oracle import attention as oa  # noqa: E402
from oracle import paging as op  # noqa: E402


def decode_config1():
    """Config 1: B=4, Hq=32, Hkv=4, D=64, bs=16, ctx {17,64,130,255}, pool 128, fp32."""
    rng = np.random.default_rng(1235)
    B, Hq, Hkv, D, bs, N = 4, 32, 4, 64, 16, 128
    ctx = np.array([17, 64, 130, 255], dtype=np.int32)
    need = (ctx + bs - 1) // bs
    perm = rng.permutation(N)
    bt = np.zeros((B, 16), dtype=np.int32)
    off = 0
    for i, n in enumerate(need):
        bt[i, :n] = perm[off:off + n]
        off += n
    q = rng.standard_normal((B, 1, Hq, D)).astype(np.float16)
    k = np.zeros((N, bs, Hkv, D), dtype=np.float16)
    v = np.zeros((N, bs, Hkv, D), dtype=np.float16)
    used = np.unique(bt[bt >= 0])
    k[used] = rng.standard_normal((len(used), bs, Hkv, D)).astype(np.float16)
    v[used] = rng.standard_normal((len(used), bs, Hkv, D)).astype(np.float16)
    out = oa.paged_decode_attention(q.astype(np.float32), k.astype(np.float32), v.astype(np.float32),
                                    bt, ctx, Hq, Hkv, D, bs)
    np.savez_compressed(HERE / "decode_config1.npz", q=q, k_cache=k, v_cache=v, block_tables=bt,
                        context_lens=ctx, out=out.astype(np.float32),
                        meta=np.array([Hq, Hkv, D, bs], dtype=np.int32))


def prefill_slots_config2():
    """Config 2 slot mapping: 8 prompts admitted in order into a fresh 1024-block pool."""
    lens = [1, 15, 16, 17, 128, 500, 1024, 2048]
    bm = op.OracleBlockManager(num_gpus=1, blocks_per_gpu=1024, block_size=16)
    slots = []
    tables = np.zeros((len(lens), 128), dtype=np.int32)
    for sid, L in enumerate(lens):
        bm.register_sequence(sid)
        slots.append(op.slot_mapping_for_prompt(bm, sid, 0, L))
        t = bm.get_block_table(sid)
        tables[sid, :len(t)] = t
    np.savez_compressed(HERE / "prefill_slots_config2.npz", lens=np.array(lens, dtype=np.int32),
                        slot_mapping=np.concatenate(slots).astype(np.int64), block_tables=tables,
                        free_after=np.array(bm.free_blocks[0], dtype=np.int32))


def main():
    decode_config1()
    prefill_slots_config2()
    for p in sorted(HERE.glob("*.npz")):
        print(p.name, p.stat().st_size)


if __name__ == "__main__":
    main()
