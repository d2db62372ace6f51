"""Host staging of a prefill graph's inputs (CPU): the live prompts at the front of
the packed buffer, one padding prompt of token 0 / position 0 / slot -1 up to the
graph's token count, and cu_seqlens that end at that count."""

import numpy as np

from tinyvllm_b200.model import prefill_staging_layout, stage_prefill_inputs


def test_live_prompts_then_one_padding_prompt():
    n, T = 3, 256
    off_cu, off_slots, words = prefill_staging_layout(n, T)
    assert off_slots % 2 == 0 and words == off_slots + 2 * T
    h = np.full(words, 7, dtype=np.int32)
    lens = [37, 1, 130]
    rng = np.random.default_rng(0)
    toks = rng.integers(0, 32000, sum(lens)).astype(np.int32)
    pos = np.concatenate([np.arange(L, dtype=np.int32) for L in lens])
    slots = rng.integers(0, 1 << 40, sum(lens)).astype(np.int64)
    stage_prefill_inputs(h, n, T, toks, pos, lens, slots)
    t = sum(lens)
    assert np.array_equal(h[:t], toks) and not h[t:T].any()
    assert np.array_equal(h[T:T + t], pos) and not h[T + t:2 * T].any()
    assert h[off_cu:off_cu + n + 2].tolist() == [0, 37, 38, 168, T]
    hs = h[off_slots:].view(np.int64)
    assert np.array_equal(hs[:t], slots) and (hs[t:] == -1).all()


def test_capture_contents_store_nothing():
    n, T = 4, 128
    off_cu, off_slots, words = prefill_staging_layout(n, T)
    h = np.full(words, 9, dtype=np.int32)
    stage_prefill_inputs(h, n, T, np.zeros(0, np.int32), np.zeros(0, np.int32), None, np.zeros(0, np.int64))
    assert not h[:2 * T].any()
    assert h[off_cu:off_cu + n + 2].tolist() == [0, 1, 2, 3, 4, T]
    assert (h[off_slots:].view(np.int64) == -1).all()
