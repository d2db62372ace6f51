"""Parity of the sm_100a paged-decode kernels with the CPU oracle (GPU).

Tolerances (from the hot-path contract): fp32 1e-3 max-abs; fp16/bf16 2e-2
max-abs and 1e-2 mean-relative, against the fp32 oracle run on the same
rounded inputs.
"""

import math
from pathlib import Path

import numpy as np
import pytest
import torch

from oracle import attention as oa

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


def _oracle(case, max_context_len=None):
    return oa.paged_decode_attention(_np(case.q), _np(case.k_cache), _np(case.v_cache),
                                     case.block_tables.cpu().numpy(), case.context_lens.cpu().numpy(),
                                     case.n_heads, case.n_kv_heads, case.head_dim, case.block_size,
                                     max_context_len)


def _run(case, **kw):
    from tinyvllm_b200.attention import paged_decode_attention
    out = paged_decode_attention(case.q, case.k_cache, case.v_cache, case.block_tables, case.context_lens,
                                 case.n_heads, case.n_kv_heads, case.head_dim, case.block_size, **kw)
    torch.cuda.synchronize()
    return out


def test_config1_fp32_vs_oracle(cuda):
    from tinyvllm_b200 import workloads
    case = workloads.decode_config1(cuda)
    _check(_run(case), _oracle(case), torch.float32)


def test_golden_decode_config1(cuda):
    g = np.load(GOLDEN / "decode_config1.npz")
    hq, hkv, d, bs = (int(x) for x in g["meta"])
    from tinyvllm_b200.attention import paged_decode_attention
    for dtype in (torch.float32, torch.float16):
        t = lambda a: torch.from_numpy(np.ascontiguousarray(a)).to(cuda)
        out = paged_decode_attention(t(g["q"]).to(dtype), t(g["k_cache"]).to(dtype), t(g["v_cache"]).to(dtype),
                                     t(g["block_tables"]), t(g["context_lens"]), hq, hkv, d, bs)
        torch.cuda.synchronize()
        _check(out, g["out"], dtype)


# The reference tests' shapes (tests/test_paged_attention.py:126-251), contiguous tables.
@pytest.mark.parametrize("dtype", [torch.float32, torch.float16, torch.bfloat16])
@pytest.mark.parametrize("batch,nh,nkv,d,ctx", [
    (2, 8, 8, 64, 32), (1, 4, 4, 32, 32), (1, 32, 8, 64, 32), (1, 32, 4, 64, 64), (4, 8, 8, 32, 32),
    (1, 4, 4, 32, 16), (1, 4, 4, 32, 64), (1, 4, 4, 32, 128), (1, 4, 4, 32, 25),
])
def test_reference_shapes(cuda, dtype, batch, nh, nkv, d, ctx):
    from tinyvllm_b200 import workloads
    case = workloads.decode_case(batch, nh, nkv, d, 16, [ctx] * batch, dtype=dtype, device=cuda,
                                 seed=ctx * 7 + nh, contiguous=True)
    _check(_run(case), _oracle(case), dtype)


# Shuffled tables, ragged contexts, every supported head_dim / GQA group / block size.
@pytest.mark.parametrize("dtype", [torch.float32, torch.float16, torch.bfloat16])
@pytest.mark.parametrize("d", [32, 64, 128])
@pytest.mark.parametrize("nh,nkv", [(8, 8), (16, 8), (32, 8), (32, 4), (32, 2)])
def test_shuffled_ragged(cuda, dtype, d, nh, nkv):
    from tinyvllm_b200 import workloads
    ctx = [1, 15, 16, 17, 63, 64, 65, 300, 1000]
    case = workloads.decode_case(len(ctx), nh, nkv, d, 16, ctx, dtype=dtype, device=cuda, seed=nh + d)
    _check(_run(case), _oracle(case), dtype)


@pytest.mark.parametrize("dtype", [torch.float32, torch.float16, torch.bfloat16])
@pytest.mark.parametrize("bs", [1, 5, 8, 16, 32, 64])
def test_block_sizes(cuda, dtype, bs):
    from tinyvllm_b200 import workloads
    ctx = [1, bs, bs + 1, 3 * bs + 2, 200]
    case = workloads.decode_case(len(ctx), 32, 4, 64, bs, ctx, dtype=dtype, device=cuda, seed=bs)
    _check(_run(case), _oracle(case), dtype)


@pytest.mark.parametrize("dtype", [torch.float32, torch.float16])
def test_engine_padding_width_64(cuda, dtype):
    """The engine pads every table to 64 blocks with block 0 (engine.py:81,235-255)."""
    from tinyvllm_b200 import workloads
    ctx = [5, 100, 700, 1024]
    case = workloads.decode_case(len(ctx), 32, 4, 64, 16, ctx, dtype=dtype, device=cuda, seed=11, width=64)
    _check(_run(case), _oracle(case), dtype)


@pytest.mark.parametrize("dtype", [torch.float32, torch.float16])
def test_context_beyond_table_is_truncated(cuda, dtype):
    """ctx larger than table width: the reference attends only over the table (llama.py:117-118)."""
    from tinyvllm_b200 import workloads
    case = workloads.decode_case(3, 32, 8, 128, 16, [40, 64, 64], dtype=dtype, device=cuda, seed=12)
    case.context_lens = torch.tensor([40, 5000, 64], dtype=torch.int32, device=cuda)
    _check(_run(case), _oracle(case), dtype)


@pytest.mark.parametrize("dtype", [torch.float32, torch.float16])
@pytest.mark.parametrize("mcl", [1, 16, 100, 1000])
def test_max_context_len(cuda, dtype, mcl):
    from tinyvllm_b200 import workloads
    ctx = [10, 90, 400, 700]
    case = workloads.decode_case(len(ctx), 32, 4, 64, 16, ctx, dtype=dtype, device=cuda, seed=mcl)
    _check(_run(case, max_context_len=mcl), _oracle(case, mcl), dtype)


def test_zero_context_gives_zeros(cuda):
    """Documented deviation: ctx <= 0 -> zeros (the reference would average padding)."""
    from tinyvllm_b200 import workloads
    case = workloads.decode_case(3, 32, 4, 64, 16, [0, 20, 0], dtype=torch.float16, device=cuda, seed=13)
    out = _run(case)
    assert torch.count_nonzero(out[0]) == 0 and torch.count_nonzero(out[2]) == 0
    ref = _oracle(case)
    _check(out[1:2], ref[1:2], torch.float16)


def test_out_of_range_block_ids_read_zero(cuda):
    from tinyvllm_b200 import workloads
    for dtype in (torch.float16, torch.float32):
        case = workloads.decode_case(1, 32, 4, 64, 16, [48], dtype=dtype, device=cuda, seed=14)
        n = case.k_cache.shape[0]
        case.block_tables[0, 1] = n + 100   # second block points outside the pool
        out = _run(case)
        kc, vc = case.k_cache.clone(), case.v_cache.clone()
        kc = torch.cat([kc, torch.zeros_like(kc[:1])])
        vc = torch.cat([vc, torch.zeros_like(vc[:1])])
        bt = case.block_tables.clone()
        bt[0, 1] = n   # the appended zero block
        ref = oa.paged_decode_attention(_np(case.q), _np(kc), _np(vc), bt.cpu().numpy(),
                                        case.context_lens.cpu().numpy(), 32, 4, 64, 16)
        _check(out, ref, dtype)


def test_nan_outside_context_does_not_leak(cuda):
    """Stale non-finite values past the context (same block) must not reach the output."""
    from tinyvllm_b200 import workloads
    for dtype in (torch.float16, torch.bfloat16, torch.float32):
        case = workloads.decode_case(2, 32, 8, 128, 16, [20, 33], dtype=dtype, device=cuda, seed=15)
        ref = _oracle(case)
        for b, c in enumerate([20, 33]):
            blk = int(case.block_tables[b, c // 16])
            case.k_cache[blk, c % 16:] = float("nan")
            case.v_cache[blk, c % 16:] = float("inf")
        _check(_run(case), ref, dtype)


def _per_sequence_oracle_check(case, out, dtype):
    """Every sequence of ``case`` against the oracle, one sequence per oracle call.
    Each call gets only that sequence's own blocks (gathered into a compact pool)
    and a table cut to its own context: the cut positions are masked by
    ``context_lens`` in the reference (their -1e9 scores give exact zeros after
    the softmax), so the oracle's result for the row is unchanged, and the CPU
    cost grows with the live tokens instead of batch x table width."""
    ref = np.empty(tuple(out.shape), dtype=np.float32)
    ctx = case.context_lens.cpu().numpy()
    for b in range(case.batch):
        width = max(1, int((ctx[b] + case.block_size - 1) // case.block_size))
        blocks = case.block_tables[b, :width].long()
        ref[b] = oa.paged_decode_attention(_np(case.q[b:b + 1]), _np(case.k_cache[blocks]), _np(case.v_cache[blocks]),
                                           np.arange(width, dtype=np.int32)[None], ctx[b:b + 1], case.n_heads,
                                           case.n_kv_heads, case.head_dim, case.block_size)[0]
    _check(out, ref, dtype)


def test_config3_all_sequences_vs_oracle(cuda):
    """Config 3 exactly as benchmarked (256 sequences, 32q/8kv, D=128, fp16, contexts
    U{128..4096}, shuffled tables in a 1.2x pool): every sequence against the oracle."""
    from tinyvllm_b200 import workloads
    case = workloads.decode_config3(cuda)
    out = _run(case)
    assert torch.isfinite(out.float()).all()
    _per_sequence_oracle_check(case, out, torch.float16)


def test_config5_shape_bf16_long_contexts_vs_oracle(cuda):
    """Config 5's attention shape (Llama-3-8B: 32q/8kv, D=128, block 16, bf16) with
    contexts U{512..8192}: 64 sequences take the persistent plan with several units
    per sequence, so the split-K partials and the combine kernel are on the path."""
    import ctypes
    from tinyvllm_b200 import _lib, workloads
    rng = np.random.default_rng(1234 + 5)
    ctx = rng.integers(512, 8193, size=64)
    ctx[:4] = [8192, 8191, 4097, 512]
    case = workloads.decode_case(64, 32, 8, 128, 16, ctx.tolist(), dtype=torch.bfloat16, device=cuda, seed=1239,
                                 extra_blocks=int(0.2 * ((ctx + 15) // 16).sum()))
    plan = (ctypes.c_int * 4)()
    assert _lib.lib().tvk_paged_decode_plan(64, 32, 8, 128, 16, case.block_tables.shape[1], -1, 2, plan) == 0
    assert plan[3] == 1 and plan[2] == 2          # persistent CTAs, split-K combine launched
    out = _run(case)
    _per_sequence_oracle_check(case, out, torch.bfloat16)


def test_config3_relabel_invariance(cuda):
    """Size-independent property at full size: permuting physical block ids (and the
    tables with them) leaves the output bit-identical."""
    from tinyvllm_b200 import workloads
    case = workloads.decode_config3(cuda)
    out = _run(case).clone()
    n = case.k_cache.shape[0]
    g = torch.Generator(device=cuda).manual_seed(99)
    perm = torch.randperm(n, device=cuda, generator=g)          # new id of old block i
    kc = torch.empty_like(case.k_cache)
    vc = torch.empty_like(case.v_cache)
    kc[perm] = case.k_cache
    vc[perm] = case.v_cache
    case.k_cache, case.v_cache = kc, vc
    case.block_tables = perm[case.block_tables.long()].int()
    out2 = _run(case)
    assert torch.equal(out, out2)


def test_repeat_calls_are_deterministic(cuda):
    from tinyvllm_b200 import workloads
    case = workloads.decode_config3(cuda, batch=64)
    a = _run(case).clone()
    b = _run(case)
    assert torch.equal(a, b)


def _call_abi(case, ws, nbytes):
    from tinyvllm_b200 import _lib
    out = torch.empty_like(case.q)
    rc = _lib.lib().tvk_paged_decode_attention(
        case.q.data_ptr(), case.k_cache.data_ptr(), case.v_cache.data_ptr(), case.block_tables.data_ptr(),
        case.context_lens.data_ptr(), out.data_ptr(), case.batch, case.n_heads, case.n_kv_heads, case.head_dim,
        case.block_size, case.k_cache.shape[0], case.block_tables.shape[1], -1, _lib.dtype_code(case.q),
        None if ws is None else ws.data_ptr(), nbytes, torch.cuda.current_stream().cuda_stream)
    assert rc == 0, _lib.lib().tvk_last_error()
    torch.cuda.synchronize()
    return out


def test_work_list_counters_return_to_zero(cuda):
    """The tensor-core kernel hands out its (sequence, KV head, split) units from
    counters in the workspace header (status word at byte 0, counters at 64 and
    128); every call leaves them zeroed, so back-to-back calls on one workspace
    give identical results.  Bytes 192.. hold the unit size of the last call."""
    from tinyvllm_b200 import _lib, workloads
    case = workloads.decode_config3(cuda, batch=96)
    n = _lib.lib().tvk_paged_decode_workspace_size(case.batch, 32, 8, 128, 16, case.block_tables.shape[1], -1)
    ws = torch.zeros(n, dtype=torch.uint8, device=cuda)
    outs = [_call_abi(case, ws, n).clone() for _ in range(3)]
    assert torch.count_nonzero(ws[:192]) == 0
    assert torch.equal(outs[0], outs[1]) and torch.equal(outs[1], outs[2])
    _check(outs[0][:8], _oracle_rows(case, range(8)), torch.float16)


def _oracle_rows(case, idx):
    idx = list(idx)
    return oa.paged_decode_attention(_np(case.q[idx]), _np(case.k_cache), _np(case.v_cache),
                                     case.block_tables[idx].cpu().numpy(), case.context_lens[idx].cpu().numpy(),
                                     case.n_heads, case.n_kv_heads, case.head_dim, case.block_size)


@pytest.mark.parametrize("dtype", [torch.float16, torch.bfloat16])
def test_without_workspace_matches_with(cuda, dtype):
    """Single-split batches may pass no workspace: the units then go to CTAs in a
    fixed order instead of from the header counters; results are the same."""
    from tinyvllm_b200 import workloads
    ctx = [1, 17, 64, 5, 2, 33, 48, 63] * 40
    case = workloads.decode_case(len(ctx), 32, 8, 128, 16, ctx, dtype=dtype, device=cuda, seed=21, width=4,
                                 contiguous=True)
    a = _call_abi(case, None, 0)
    ws = torch.zeros(1 << 16, dtype=torch.uint8, device=cuda)
    b = _call_abi(case, ws, ws.numel())
    assert torch.equal(a, b)
    _check(a, _oracle(case), dtype)


def _subset_check(case, out, idx, dtype):
    bt = case.block_tables[idx]
    used = torch.unique(bt)
    remap = torch.full((case.k_cache.shape[0],), -1, dtype=torch.int64, device=bt.device)
    remap[used.long()] = torch.arange(len(used), device=bt.device)
    sub_bt = remap[bt.long()].int()
    ref = oa.paged_decode_attention(_np(case.q[idx]), _np(case.k_cache[used.long()]),
                                    _np(case.v_cache[used.long()]), sub_bt.cpu().numpy(),
                                    case.context_lens[idx].cpu().numpy(), case.n_heads, case.n_kv_heads,
                                    case.head_dim, case.block_size)
    _check(out[idx], ref, dtype)


@pytest.mark.parametrize("dtype", [torch.float16, torch.bfloat16])
def test_persistent_plan_with_wide_tables_and_empty_sequences(cuda, dtype):
    """A large batch (persistent CTAs, ticket counter) whose tables are far wider
    than its contexts, with some empty sequences: the kernel sizes units from the
    live contexts and empty sequences give zeros."""
    from tinyvllm_b200 import _lib, workloads
    rng = np.random.default_rng(31)
    ctx = rng.integers(1, 300, size=256)
    ctx[::17] = 0
    case = workloads.decode_case(256, 32, 8, 128, 16, ctx.tolist(), dtype=dtype, device=cuda, seed=31, width=256)
    plan = (__import__("ctypes").c_int * 4)()
    assert _lib.lib().tvk_paged_decode_plan(256, 32, 8, 128, 16, 256, -1, _lib.dtype_code(case.q), plan) == 0
    assert plan[3] == 1                               # persistent plan
    out = _run(case)
    zero = [i for i in range(256) if ctx[i] == 0]
    assert torch.count_nonzero(out[zero]) == 0
    _subset_check(case, out, [1, 2, 3, 50, 99, 128, 200, 254], dtype)   # 255 is empty


def test_persistent_plan_with_a_sparse_long_tail(cuda):
    """Most sequences short and a few long: the later splits are mostly dead
    tickets, which the scan skips."""
    ctx = [64] * 120 + [4000, 3000, 2500, 4096, 64, 1, 17, 4095]
    from tinyvllm_b200 import workloads
    case = workloads.decode_case(len(ctx), 32, 8, 128, 16, ctx, dtype=torch.float16, device=cuda, seed=32)
    a = _run(case).clone()
    b = _run(case)
    assert torch.equal(a, b)
    _subset_check(case, a, [0, 119, 120, 121, 122, 123, 124, 125, 126, 127], torch.float16)
