"""Parity of the flash-prefill kernels (tcgen05 and SIMT) with the CPU oracle, and
the fused paged K/V write against the reference slot mapping (GPU).

Tolerances: fp32 1e-3 max-abs (the reference tests use 1e-4..1e-3 between two
fp32 paths); fp16/bf16 2e-2 max-abs and 1e-2 mean-relative.  The paged write
is checked bit-exactly.
"""

from pathlib import Path

import numpy as np
import pytest
import torch

from oracle import attention as oa
from oracle import paging as op

pytestmark = pytest.mark.gpu

GOLDEN = Path(__file__).resolve().parent / "golden"
TOL = {torch.float32: (1e-3, None), torch.float16: (2e-2, 1e-2), torch.bfloat16: (2e-2, 1e-2)}


def _np(t):
    return t.detach().float().cpu().numpy()


def _check(got, expect, dtype):
    max_abs, mean_rel = TOL[dtype]
    g = _np(got).astype(np.float64)
    e = np.asarray(expect, dtype=np.float64)
    assert np.isfinite(g).all()
    err = np.abs(g - e)
    assert err.max() <= max_abs, f"max-abs {err.max()} > {max_abs}"
    if mean_rel is not None:
        rel = err.mean() / max(np.abs(e).mean(), 1e-12)
        assert rel <= mean_rel, f"mean-rel {rel} > {mean_rel}"


def _rand(shape, dtype, g, dev):
    return torch.randn(shape, generator=g, device=dev).to(dtype)


def _flash(q, k, v, causal=True):
    from tinyvllm_b200.attention import flash_prefill_attention
    out = flash_prefill_attention(q[None], k[None], v[None], causal)[0]
    torch.cuda.synchronize()
    return out


def _oracle(q, k, v, causal=True):
    return oa.flash_prefill_attention(_np(q)[None], _np(k)[None], _np(v)[None], causal)[0]


DTYPES = [torch.float32, torch.float16, torch.bfloat16]


@pytest.fixture(params=[0, 1], ids=["auto", "one_head"])
def kernel(request, cuda):
    """Runs the test with the automatic kernel choice (the paired-head kernel where
    the query heads per KV head are even) and again with the one-head kernel."""
    from tinyvllm_b200 import _lib
    lib = _lib.lib()
    assert lib.tvk_prefill_select_kernel(request.param) == 0
    yield request.param
    assert lib.tvk_prefill_select_kernel(0) == 0


# tests/test_flash_attention.py shapes
@pytest.mark.parametrize("dtype", DTYPES)
@pytest.mark.parametrize("L", [1, 2, 7, 8, 15, 16, 31, 32, 63, 64, 128])
@pytest.mark.parametrize("D", [32, 64, 128])
def test_lengths_and_head_dims(cuda, dtype, L, D):
    g = torch.Generator(device=cuda).manual_seed(L * 10 + D)
    q, k, v = (_rand((L, 4, D), dtype, g, cuda) for _ in range(3))
    _check(_flash(q, k, v), _oracle(q, k, v), dtype)


@pytest.mark.parametrize("dtype", DTYPES)
@pytest.mark.parametrize("L,nh,nkv,D", [(16, 8, 4, 32), (16, 32, 8, 64), (16, 32, 4, 64), (32, 32, 8, 64),
                                        (64, 32, 8, 64), (256, 32, 8, 64), (200, 32, 4, 128), (1, 8, 8, 64)])
def test_gqa(cuda, kernel, dtype, L, nh, nkv, D):
    g = torch.Generator(device=cuda).manual_seed(L + nh + nkv + D)
    q = _rand((L, nh, D), dtype, g, cuda)
    k = _rand((L, nkv, D), dtype, g, cuda)
    v = _rand((L, nkv, D), dtype, g, cuda)
    _check(_flash(q, k, v), _oracle(q, k, v), dtype)


@pytest.mark.parametrize("dtype", DTYPES)
@pytest.mark.parametrize("L,D", [(16, 32), (16, 64), (300, 64), (129, 128)])
def test_non_causal(cuda, dtype, L, D):
    g = torch.Generator(device=cuda).manual_seed(L + D)
    q, k, v = (_rand((L, 4, D), dtype, g, cuda) for _ in range(3))
    _check(_flash(q, k, v, causal=False), _oracle(q, k, v, causal=False), dtype)


@pytest.mark.parametrize("dtype", DTYPES)
def test_first_token_attends_to_itself(cuda, dtype):
    """tests/test_flash_attention.py:123-130 (head_dim 16 there; 32 here, the smallest kernel size)."""
    q = torch.zeros(8, 2, 32, device=cuda)
    q[0] = 1.0
    k = torch.randn(8, 2, 32, generator=torch.Generator(device=cuda).manual_seed(1), device=cuda)
    v = torch.zeros(8, 2, 32, device=cuda)
    v[:, :, :8] = torch.eye(8, device=cuda)[:, None, :]
    out = _flash(q.to(dtype), k.to(dtype), v.to(dtype))
    assert out[0, 0, 0].item() > 0.5


@pytest.mark.parametrize("dtype", DTYPES)
@pytest.mark.parametrize("D", [32, 64, 128])
def test_last_token_mean(cuda, dtype, D):
    """tests/test_flash_attention.py:132-139: last row of v = arange(8) averages to 3.5."""
    q = torch.ones(8, 2, D, device=cuda, dtype=dtype)
    k = torch.zeros(8, 2, D, device=cuda, dtype=dtype)
    v = torch.arange(8, device=cuda, dtype=torch.float32).reshape(8, 1, 1).expand(8, 2, D).contiguous().to(dtype)
    assert abs(_flash(q, k, v)[-1, 0, 0].item() - 3.5) < 1e-2


def _config2_inputs(dev, dtype=torch.float16, lens=(1, 15, 16, 17, 128, 500, 1024, 2048), D=64, nkv=4):
    g = torch.Generator(device=dev).manual_seed(1236)
    T = sum(lens)
    q = _rand((T, 32, D), dtype, g, dev)
    k = _rand((T, nkv, D), dtype, g, dev)
    v = _rand((T, nkv, D), dtype, g, dev)
    cu = torch.tensor(np.concatenate([[0], np.cumsum(lens)]), dtype=torch.int32, device=dev)
    return q, k, v, cu, list(lens)


@pytest.mark.parametrize("dtype,D,nkv", [(torch.float16, 64, 4), (torch.bfloat16, 128, 8), (torch.float32, 64, 4)])
def test_config2_ragged_batch_with_paged_write(cuda, kernel, dtype, D, nkv):
    """Config 2: 8 ragged prompts in one call; attention vs oracle per prompt and the
    paged pool bit-exact against the reference slot mapping (LIFO allocation)."""
    from tinyvllm_b200.attention import flash_prefill_attention_varlen
    q, k, v, cu, lens = _config2_inputs(cuda, dtype, D=D, nkv=nkv)
    gold = np.load(GOLDEN / "prefill_slots_config2.npz")
    assert list(gold["lens"]) == lens
    slots = torch.from_numpy(gold["slot_mapping"]).to(cuda)
    kc = torch.zeros(1024, 16, nkv, D, dtype=dtype, device=cuda)
    vc = torch.zeros_like(kc)
    out = flash_prefill_attention_varlen(q, k, v, cu, max(lens), True, slot_mapping=slots, k_cache=kc, v_cache=vc)
    torch.cuda.synchronize()
    # paged write: every token's row at its slot, everything else untouched (zero)
    exp_k = torch.zeros(1024 * 16, nkv, D, dtype=dtype, device=cuda)
    exp_v = torch.zeros_like(exp_k)
    exp_k[slots] = k
    exp_v[slots] = v
    assert torch.equal(kc.view(-1, nkv, D), exp_k)
    assert torch.equal(vc.view(-1, nkv, D), exp_v)
    # attention, prompt by prompt
    for i, L in enumerate(lens):
        a, b = int(cu[i]), int(cu[i + 1])
        _check(out[a:b], _oracle(q[a:b], k[a:b], v[a:b]), dtype)


def test_paged_write_matches_chunked_reference_write(cuda, kernel):
    """The fused write equals the reference's block-chunked write_kv sequence
    (llama.py:188-209) replayed by the oracle on the same BlockManager state."""
    from tinyvllm_b200.attention import flash_prefill_attention_varlen
    lens = [5, 40, 16, 33]
    q, k, v, cu, _ = _config2_inputs(cuda, torch.float16, lens=lens)
    bm = op.OracleBlockManager(1, 32, 16)
    cache = op.OracleKVCache(1, 32, 16, 4, 64, dtype=np.float16)
    slots = []
    kn, vn = k.cpu().numpy(), v.cpu().numpy()
    for sid, L in enumerate(lens):
        bm.register_sequence(sid)
        a, b = int(cu[sid]), int(cu[sid + 1])
        op.write_prompt_kv(cache, bm, 0, sid, kn[a:b], vn[a:b], 0)
        t = bm.get_block_table(sid)
        slots += [t[p // 16] * 16 + p % 16 for p in range(L)]
    kc = torch.zeros(32, 16, 4, 64, dtype=torch.float16, device=cuda)
    vc = torch.zeros_like(kc)
    flash_prefill_attention_varlen(q, k, v, cu, max(lens), True,
                                   slot_mapping=torch.tensor(slots, dtype=torch.int64, device=cuda),
                                   k_cache=kc, v_cache=vc)
    torch.cuda.synchronize()
    assert np.array_equal(kc.cpu().numpy(), cache.k_cache[0])
    assert np.array_equal(vc.cpu().numpy(), cache.v_cache[0])


def test_negative_slots_are_skipped(cuda, kernel):
    from tinyvllm_b200.attention import flash_prefill_attention_varlen
    q, k, v, cu, lens = _config2_inputs(cuda, torch.float16, lens=[20])
    slots = torch.arange(20, dtype=torch.int64, device=cuda)
    slots[3] = -1
    slots[7] = 10 ** 9  # beyond the pool
    kc = torch.zeros(4, 16, 4, 64, dtype=torch.float16, device=cuda)
    vc = torch.zeros_like(kc)
    flash_prefill_attention_varlen(q, k, v, cu, 20, True, slot_mapping=slots, k_cache=kc, v_cache=vc)
    torch.cuda.synchronize()
    flat = kc.view(-1, 4, 64)
    keep = [i for i in range(20) if i not in (3, 7)]
    assert torch.equal(flat[keep], k[keep])
    assert torch.count_nonzero(flat[3]) == 0 and torch.count_nonzero(flat[7]) == 0


def test_repeat_calls_are_deterministic(cuda, kernel):
    from tinyvllm_b200.attention import flash_prefill_attention_varlen
    q, k, v, cu, lens = _config2_inputs(cuda, torch.float16)
    a = flash_prefill_attention_varlen(q, k, v, cu, max(lens)).clone()
    b = flash_prefill_attention_varlen(q, k, v, cu, max(lens))
    torch.cuda.synchronize()
    assert torch.equal(a, b)


@pytest.mark.parametrize("n", [33, 70])
def test_many_prompts_take_the_device_schedule(cuda, kernel, n):
    """More than 32 prompts: the work list is built by the schedule kernel rather
    than by the producer warps; alternating with a small batch on the same
    workspace checks that every call returns the item counters to zero."""
    from tinyvllm_b200.attention import flash_prefill_attention_varlen
    rng = np.random.default_rng(40 + n)
    lens = [int(x) for x in rng.integers(1, 300, size=n)]
    q, k, v, cu, _ = _config2_inputs(cuda, torch.float16, lens=lens)
    small = _config2_inputs(cuda, torch.float16, lens=[130, 7, 260])
    for _ in range(2):
        out = flash_prefill_attention_varlen(q, k, v, cu, max(lens)).clone()
        out_s = flash_prefill_attention_varlen(*small[:4], max(small[4])).clone()
        torch.cuda.synchronize()
        for i in (0, 1, n // 2, n - 1):
            a, b = int(cu[i]), int(cu[i + 1])
            _check(out[a:b], _oracle(q[a:b], k[a:b], v[a:b]), torch.float16)
        sq, sk, sv, scu, slens = small
        for i in range(3):
            a, b = int(scu[i]), int(scu[i + 1])
            _check(out_s[a:b], _oracle(sq[a:b], sk[a:b], sv[a:b]), torch.float16)
    from tinyvllm_b200.attention import workspace_status
    assert workspace_status(kind="prefill") == 0


@pytest.mark.parametrize("n,hi,max_extra", [(32, 700, 0), (9, 260, 3000), (1, 5, 0)])
def test_small_batches_with_shared_tile_counts(cuda, kernel, n, hi, max_extra):
    """Up to 32 prompts, many with the same number of query tiles, and a
    ``max_seqlen`` that may exceed the longest prompt (empty top bands of the
    schedule): every prompt's rows and its paged K/V write come out exactly once,
    on two calls in a row (CTA b's first item is item b, the rest come from the
    ticket counter)."""
    from tinyvllm_b200.attention import flash_prefill_attention_varlen, workspace_status
    rng = np.random.default_rng(700 + n)
    lens = [int(x) for x in rng.integers(1, hi, size=n)]
    q, k, v, cu, _ = _config2_inputs(cuda, torch.float16, lens=lens)
    T = sum(lens)
    n_blocks = sum((L + 15) // 16 for L in lens) + 3
    slots = torch.from_numpy(rng.permutation(n_blocks * 16)[:T].astype(np.int64)).to(cuda)
    kc = torch.zeros(n_blocks, 16, 4, 64, dtype=torch.float16, device=cuda)
    vc = torch.zeros_like(kc)
    for _ in range(2):
        out = flash_prefill_attention_varlen(q, k, v, cu, max(lens) + max_extra, True, slot_mapping=slots,
                                             k_cache=kc, v_cache=vc, check=True)
        torch.cuda.synchronize()
        for i in range(n):
            a, b = int(cu[i]), int(cu[i + 1])
            _check(out[a:b], _oracle(q[a:b], k[a:b], v[a:b]), torch.float16)
        exp_k = torch.zeros(n_blocks * 16, 4, 64, dtype=torch.float16, device=cuda)
        exp_v = torch.zeros_like(exp_k)
        exp_k[slots] = k
        exp_v[slots] = v
        assert torch.equal(kc.view(-1, 4, 64), exp_k)
        assert torch.equal(vc.view(-1, 4, 64), exp_v)
    assert workspace_status(kind="prefill") == 0


@pytest.mark.parametrize("dtype", [torch.float16, torch.bfloat16])
@pytest.mark.parametrize("L,nh,nkv,D", [(300, 32, 4, 64), (129, 8, 2, 64), (260, 32, 8, 128), (1, 16, 4, 64)])
def test_non_causal_gqa(cuda, kernel, dtype, L, nh, nkv, D):
    g = torch.Generator(device=cuda).manual_seed(L * 3 + nh + D)
    q = _rand((L, nh, D), dtype, g, cuda)
    k = _rand((L, nkv, D), dtype, g, cuda)
    v = _rand((L, nkv, D), dtype, g, cuda)
    _check(_flash(q, k, v, causal=False), _oracle(q, k, v, causal=False), dtype)


@pytest.mark.parametrize("dtype,D,nkv", [(torch.float16, 64, 4), (torch.bfloat16, 128, 8)])
def test_running_max_jumps(cuda, kernel, dtype, D, nkv):
    """Keys grow along the prompt, so the running row max rises by more than 2^8
    several times: the lazy O rescale (skipped while the max grows less) runs."""
    g = torch.Generator(device=cuda).manual_seed(77 + D)
    L = 700
    ramp = (0.25 + torch.arange(L, device=cuda, dtype=torch.float32) / 48.0)[:, None, None]
    q = _rand((L, 32, D), dtype, g, cuda)
    k = (torch.randn(L, nkv, D, generator=g, device=cuda) * ramp).to(dtype)
    v = _rand((L, nkv, D), dtype, g, cuda)
    _check(_flash(q, k, v), _oracle(q, k, v), dtype)


@pytest.mark.parametrize("dtype,D,nkv", [(torch.float16, 64, 4), (torch.bfloat16, 128, 8)])
def test_long_prompts(cuda, kernel, dtype, D, nkv):
    """Two 2,500-token prompts: items of up to 20 key tiles, the K/V ring and both Q
    buffers wrap many times inside one CTA."""
    from tinyvllm_b200.attention import flash_prefill_attention_varlen
    q, k, v, cu, lens = _config2_inputs(cuda, dtype, lens=(2500, 1900), D=D, nkv=nkv)
    out = flash_prefill_attention_varlen(q, k, v, cu, max(lens))
    torch.cuda.synchronize()
    for i in range(2):
        a, b = int(cu[i]), int(cu[i + 1])
        _check(out[a:b], _oracle(q[a:b], k[a:b], v[a:b]), dtype)


def test_both_kernels_agree_on_config2(cuda):
    """The paired-head and one-head kernels compute the same function: on config 2
    they agree to within one output rounding."""
    from tinyvllm_b200 import _lib
    from tinyvllm_b200.attention import flash_prefill_attention_varlen
    lib = _lib.lib()
    q, k, v, cu, lens = _config2_inputs(cuda, torch.float16)
    outs = []
    for choice in (0, 1):
        assert lib.tvk_prefill_select_kernel(choice) == 0
        outs.append(flash_prefill_attention_varlen(q, k, v, cu, max(lens)).clone())
    assert lib.tvk_prefill_select_kernel(0) == 0
    torch.cuda.synchronize()
    diff = (outs[0].float() - outs[1].float()).abs().max().item()
    assert diff <= 4e-3, diff


@pytest.fixture(params=[2, 3, 4], ids=["paired_mufu", "paired_fma_2of8", "paired_fma_3of8"])
def pair_variant(request, cuda):
    """The paired kernel with 0, 2/8 and 3/8 of the softmax exponentials computed by
    a polynomial on the FMA pipe instead of the exponential unit."""
    from tinyvllm_b200 import _lib
    lib = _lib.lib()
    assert lib.tvk_prefill_select_kernel(request.param) == 0
    yield request.param
    assert lib.tvk_prefill_select_kernel(0) == 0


@pytest.mark.parametrize("dtype,D,nkv", [(torch.float16, 64, 4), (torch.bfloat16, 64, 8), (torch.bfloat16, 128, 8)])
def test_paired_variants_vs_oracle(cuda, pair_variant, dtype, D, nkv):
    """Config 2's prompts plus a running-max ramp through every exponential variant."""
    from tinyvllm_b200.attention import flash_prefill_attention_varlen
    q, k, v, cu, lens = _config2_inputs(cuda, dtype, D=D, nkv=nkv)
    out = flash_prefill_attention_varlen(q, k, v, cu, max(lens))
    torch.cuda.synchronize()
    for i in range(len(lens)):
        a, b = int(cu[i]), int(cu[i + 1])
        _check(out[a:b], _oracle(q[a:b], k[a:b], v[a:b]), dtype)
    g = torch.Generator(device=cuda).manual_seed(91)
    L = 600
    ramp = (0.25 + torch.arange(L, device=cuda, dtype=torch.float32) / 48.0)[:, None, None]
    q2 = _rand((L, 32, D), dtype, g, cuda)
    k2 = (torch.randn(L, nkv, D, generator=g, device=cuda) * ramp).to(dtype)
    v2 = _rand((L, nkv, D), dtype, g, cuda)
    _check(_flash(q2, k2, v2), _oracle(q2, k2, v2), dtype)
    _check(_flash(q2, k2, v2, causal=False), _oracle(q2, k2, v2, causal=False), dtype)
