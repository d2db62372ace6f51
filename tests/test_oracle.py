"""Pin the CPU oracle to the reference's own tests (CPU only).

The reference suite holds no stored arrays, so the oracle is pinned to what
its tests assert: paged == dense attention on contiguous tables
(tests/test_paged_attention.py:126-251), masked dense == flash prefill and the
two causal known answers (tests/test_flash_attention.py:97-232), RMSNorm /
RoPE properties (tests/test_llama.py:59-185), BlockManager counts, LIFO order
and the OOM message (tests/test_block_manager.py), KVCache slot sums
(tests/test_kv_cache.py).  It is also checked against the committed golden
fixtures it generated.
"""

import math
from pathlib import Path

import numpy as np
import pytest

from oracle import attention as oa
from oracle import paging as op

GOLDEN = Path(__file__).resolve().parent / "golden"


def _assert_allclose(actual, expected, rtol, atol):
    a = np.asarray(actual, dtype=np.float64).ravel()
    e = np.asarray(expected, dtype=np.float64).ravel()
    bad = np.abs(a - e) > atol + rtol * np.abs(e)
    assert not bad.any(), f"max diff {np.abs(a - e)[bad].max()} (rtol={rtol}, atol={atol})"


def _standard_decode(q, k, v, n_heads, n_kv_heads):
    """tests/test_paged_attention.py:14-49 (dense reference, no mask)."""
    b, ctx, _, d = k.shape
    if n_kv_heads != n_heads:
        r = n_heads // n_kv_heads
        k = np.broadcast_to(k[:, :, :, None], (b, ctx, n_kv_heads, r, d)).reshape(b, ctx, n_heads, d)
        v = np.broadcast_to(v[:, :, :, None], (b, ctx, n_kv_heads, r, d)).reshape(b, ctx, n_heads, d)
    s = np.matmul(q.transpose(0, 2, 1, 3), k.transpose(0, 2, 3, 1)) / math.sqrt(d)
    w = oa.softmax_lastdim(s)
    return np.matmul(w, v.transpose(0, 2, 1, 3)).transpose(0, 2, 1, 3)


def _setup_paged(rng, batch, ctx, n_kv, d, bs):
    """tests/test_paged_attention.py:65-103: consecutive blocks per sequence, +5 spare."""
    nps = (ctx + bs - 1) // bs
    total = nps * batch + 5
    kc = rng.standard_normal((total, bs, n_kv, d)).astype(np.float32)
    vc = rng.standard_normal((total, bs, n_kv, d)).astype(np.float32)
    bt = np.array([list(range(i * nps, (i + 1) * nps)) for i in range(batch)], dtype=np.int32)
    cl = np.full(batch, ctx, dtype=np.int32)
    kref = np.stack([np.concatenate([kc[j] for j in bt[i]])[:ctx] for i in range(batch)])
    vref = np.stack([np.concatenate([vc[j] for j in bt[i]])[:ctx] for i in range(batch)])
    return kc, vc, bt, cl, kref, vref


@pytest.mark.parametrize("batch,nh,nkv,d,ctx", [
    (1, 4, 4, 32, 32),      # test_matches_standard_attention
    (1, 32, 8, 64, 32),     # test_gqa_4x
    (1, 32, 4, 64, 64),     # test_gqa_8x
    (4, 8, 8, 32, 32),      # test_batch_size_4
    (1, 4, 4, 32, 16), (1, 4, 4, 32, 64), (1, 4, 4, 32, 128),  # test_various_context_lengths
])
def test_oracle_paged_matches_dense(batch, nh, nkv, d, ctx):
    rng = np.random.default_rng(7)
    kc, vc, bt, cl, kref, vref = _setup_paged(rng, batch, ctx, nkv, d, 16)
    q = rng.standard_normal((batch, 1, nh, d)).astype(np.float32)
    got = oa.paged_decode_attention(q, kc, vc, bt, cl, nh, nkv, d, 16)
    assert got.shape == (batch, 1, nh, d)
    _assert_allclose(got, _standard_decode(q, kref, vref, nh, nkv), 1e-3, 1e-3)


def test_oracle_paged_ctx_not_multiple_of_block():
    rng = np.random.default_rng(8)
    kc, vc, bt, cl, kref, vref = _setup_paged(rng, 1, 25, 4, 32, 16)
    q = rng.standard_normal((1, 1, 4, 32)).astype(np.float32)
    got = oa.paged_decode_attention(q, kc, vc, bt, cl, 4, 4, 32, 16)
    assert np.isfinite(got).all()
    _assert_allclose(got, _standard_decode(q, kref, vref, 4, 4), 1e-3, 1e-3)


def _standard_prefill(q, k, v, causal):
    """tests/test_flash_attention.py:33-87: repeat_kv + -inf causal mask."""
    L, nh, d = q.shape
    nkv = k.shape[1]
    if nkv != nh:
        r = nh // nkv
        k = np.repeat(k, r, axis=1)
        v = np.repeat(v, r, axis=1)
    s = np.matmul(q.transpose(1, 0, 2), k.transpose(1, 2, 0)) / math.sqrt(d)
    if causal:
        s = s + np.where(np.tril(np.ones((L, L))) == 1, 0.0, -np.inf)[None]
    w = oa.softmax_lastdim(s.astype(np.float32))
    return np.matmul(w, v.transpose(1, 0, 2)).transpose(1, 0, 2)


def _flash(q, k, v, causal=True):
    return oa.flash_prefill_attention(q[None], k[None], v[None], causal)[0]


@pytest.mark.parametrize("L,nh,nkv,d", [
    (32, 4, 4, 32), (32, 32, 8, 64), (16, 8, 4, 32), (16, 32, 8, 64), (16, 32, 4, 64),
    (1, 4, 4, 32), (2, 4, 4, 32), (7, 4, 4, 32), (8, 4, 4, 32), (15, 4, 4, 32), (16, 4, 4, 32),
    (31, 4, 4, 32), (63, 4, 4, 32), (128, 4, 4, 32), (1, 8, 8, 64), (16, 4, 4, 128), (64, 32, 8, 64),
])
def test_oracle_prefill_matches_masked_dense(L, nh, nkv, d):
    rng = np.random.default_rng(L * 131 + nh)
    q = rng.standard_normal((L, nh, d)).astype(np.float32)
    k = rng.standard_normal((L, nkv, d)).astype(np.float32)
    v = rng.standard_normal((L, nkv, d)).astype(np.float32)
    _assert_allclose(_flash(q, k, v), _standard_prefill(q, k, v, True), 1e-4, 1e-4)


def test_oracle_prefill_non_causal():
    rng = np.random.default_rng(3)
    q, k, v = (rng.standard_normal((16, 4, 32)).astype(np.float32) for _ in range(3))
    _assert_allclose(_flash(q, k, v, causal=False), _standard_prefill(q, k, v, False), 1e-4, 1e-4)


def test_oracle_prefill_first_token_attends_to_itself():
    """tests/test_flash_attention.py:123-130."""
    rng = np.random.default_rng(4)
    q = np.array([[[1.0] * 16] * 2] + [[[0.0] * 16] * 2] * 7, dtype=np.float32)
    k = rng.standard_normal((8, 2, 16)).astype(np.float32)
    v = np.broadcast_to(np.eye(8, dtype=np.float32)[:, None, :], (8, 2, 8)).copy()
    out = _flash(q, k, v)
    assert out[0, 0, 0] > 0.5


def test_oracle_prefill_last_token_mean():
    """tests/test_flash_attention.py:132-139: last row averages v = arange(8) -> 3.5."""
    q = np.ones((8, 2, 16), np.float32)
    k = np.zeros((8, 2, 16), np.float32)
    v = np.broadcast_to(np.arange(8, dtype=np.float32).reshape(8, 1, 1), (8, 2, 16)).copy()
    assert abs(_flash(q, k, v)[-1, 0, 0] - 3.5) < 1e-2


def test_oracle_rmsnorm_properties():
    """tests/test_llama.py:67-100: unit RMS, zero input, scale invariance."""
    rng = np.random.default_rng(5)
    x = rng.standard_normal((2, 4, 64)).astype(np.float32)
    y = oa.rms_norm(x, np.ones(64, np.float32))
    assert np.allclose(np.sqrt((y ** 2).mean(-1)), 1.0, atol=1e-3)
    assert np.allclose(oa.rms_norm(np.zeros((1, 64), np.float32), np.ones(64, np.float32)), 0.0)
    assert np.allclose(oa.rms_norm(x * 7.0, np.ones(64, np.float32)), y, atol=1e-4)


def test_oracle_rope_properties():
    """tests/test_llama.py:113-185: cos/sin in range, identity at 0, norm preserved."""
    cos, sin = oa.precompute_freqs_cis(64, 128)
    assert cos.shape == (128, 32) and np.abs(cos).max() <= 1.0 and np.abs(sin).max() <= 1.0
    assert np.allclose(cos[0], 1.0) and np.allclose(sin[0], 0.0)
    rng = np.random.default_rng(6)
    x = rng.standard_normal((1, 16, 4, 64)).astype(np.float32)
    y = oa.apply_rope(x, cos, sin)
    assert np.allclose(y[:, 0], x[:, 0], atol=1e-6)
    assert np.allclose(np.linalg.norm(y, axis=-1), np.linalg.norm(x, axis=-1), rtol=1e-5)


def test_oracle_block_manager_lifo_and_oom():
    """tests/test_block_manager.py:51-133: LIFO pop, counts, the OOM message."""
    bm = op.OracleBlockManager(num_gpus=1, blocks_per_gpu=4, block_size=16)
    bm.register_sequence(0)
    assert bm.ensure_block_for_position(0, 0) == 3
    assert bm.ensure_block_for_position(0, 16) == 2
    assert bm.get_num_free_blocks() == 2
    assert bm.get_slot(0) == (0, 3, 0)
    for _ in range(17):
        bm.advance_position(0)
    assert bm.get_slot(0) == (0, 2, 1)
    bm.register_sequence(1)
    bm.ensure_block_for_position(1, 16)
    with pytest.raises(RuntimeError, match="Out of KV cache memory!"):
        bm.ensure_block_for_position(1, 32)
    bm.free_sequence(0)
    assert bm.free_blocks[0] == [3, 2]
    bm.fork_sequence(1, 5)
    assert bm.ref_counts[0][1] == 2
    bm.free_sequence(1)
    assert bm.get_num_free_blocks() == 2
    bm.free_sequence(5)
    assert bm.free_blocks[0] == [3, 2, 1, 0]


def test_oracle_kv_cache_sums():
    """tests/test_kv_cache.py: exact sums after writes, layer isolation, memory formula."""
    c = op.OracleKVCache(num_layers=2, num_blocks=4, block_size=8, n_kv_heads=2, head_dim=4)
    c.write_kv(0, 1, 3, np.ones((2, 2, 4), np.float32), 2 * np.ones((2, 2, 4), np.float32))
    assert c.k_cache[0][1, 3].sum() == 8 and c.v_cache[0][1, 4].sum() == 16
    assert c.k_cache[1].sum() == 0
    assert c.get_memory_bytes() == 2 * 4 * 8 * 2 * 4 * 2 * 4


def test_oracle_prompt_write_matches_slot_mapping():
    """llama.py:188-209 chunked writes == per-token slot scatter."""
    rng = np.random.default_rng(9)
    lens = [1, 15, 16, 17, 40]
    bm_a = op.OracleBlockManager(1, 32, 16)
    bm_b = op.OracleBlockManager(1, 32, 16)
    cache = op.OracleKVCache(1, 32, 16, 2, 8)
    flat_k = np.zeros((32 * 16, 2, 8), np.float32)
    for sid, L in enumerate(lens):
        k = rng.standard_normal((L, 2, 8)).astype(np.float32)
        bm_a.register_sequence(sid)
        bm_b.register_sequence(sid)
        op.write_prompt_kv(cache, bm_a, 0, sid, k, k, 0)
        slots = op.slot_mapping_for_prompt(bm_b, sid, 0, L)
        flat_k[slots] = k
    assert np.array_equal(cache.k_cache[0].reshape(-1, 2, 8), flat_k)


def test_oracle_reproduces_golden_decode():
    g = np.load(GOLDEN / "decode_config1.npz")
    hq, hkv, d, bs = (int(x) for x in g["meta"])
    out = oa.paged_decode_attention(g["q"].astype(np.float32), g["k_cache"].astype(np.float32),
                                    g["v_cache"].astype(np.float32), g["block_tables"], g["context_lens"],
                                    hq, hkv, d, bs)
    assert np.array_equal(out, g["out"])


def test_oracle_reproduces_golden_slots():
    g = np.load(GOLDEN / "prefill_slots_config2.npz")
    bm = op.OracleBlockManager(1, 1024, 16)
    slots = []
    for sid, L in enumerate(g["lens"]):
        bm.register_sequence(sid)
        slots.append(op.slot_mapping_for_prompt(bm, sid, 0, int(L)))
    assert np.array_equal(np.concatenate(slots), g["slot_mapping"])
    # prompt 0 takes the last block of the pool first (LIFO pop)
    assert g["slot_mapping"][0] == 1023 * 16
