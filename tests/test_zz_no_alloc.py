"""tvk_paged_decode_attention_noalloc: the decode entry point that allocates nothing.

Some callers cannot allocate device memory for scratch -- an engine that has
handed (nearly) all free HBM to its KV pool, or a host binding with no device
allocator of its own -- so this entry point keeps its split-K scratch in a
fixed array inside the library.  These tests call it through the C ABI and
compare it with the workspace-taking entry point, within the decode parity
tolerances, on two calls in a row (the array keeps the previous call's
contents, so the second call must not depend on it).  The file is named to be
collected last.
"""

import ctypes

import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu

TOL = {torch.float32: 1e-3, torch.float16: 2e-2, torch.bfloat16: 2e-2}
CODE = {torch.float32: 0, torch.float16: 1, torch.bfloat16: 2}


def _noalloc(lib, case, out):
    stream = torch.cuda.current_stream().cuda_stream
    return lib.tvk_paged_decode_attention_noalloc(
        case.q.data_ptr(), case.k_cache.data_ptr(), case.v_cache.data_ptr(), case.block_tables.data_ptr(),
        case.context_lens.data_ptr(), out.data_ptr(), case.batch, case.n_heads, case.n_kv_heads, case.head_dim,
        case.block_size, case.k_cache.shape[0], case.block_tables.shape[1], -1, CODE[case.q.dtype], stream)


def _with_workspace(case):
    from tinyvllm_b200.attention import paged_decode_attention
    return paged_decode_attention(case.q, case.k_cache, case.v_cache, case.block_tables, case.context_lens,
                                  case.n_heads, case.n_kv_heads, case.head_dim, case.block_size)


def _close(a, b, dtype):
    err = (a.float() - b.float()).abs().max().item()
    assert np.isfinite(err) and err <= TOL[dtype], f"max-abs {err} > {TOL[dtype]}"


def test_noalloc_matches_workspace_entry_two_calls(cuda):
    from tinyvllm_b200 import _lib, workloads
    lib = _lib.lib()
    # call 1: 64 config-3 sequences (several splits each, so the scratch is used)
    a = workloads.decode_config3(cuda, batch=64, seed_offset=7)
    # call 2: a different shape and dtype path (fp32, SIMT kernel, GQA 8)
    b = workloads.decode_case(5, 32, 4, 64, 16, [3, 70, 300, 900, 1500], dtype=torch.float32, device=cuda, seed=21)
    out_a = torch.full_like(a.q, float("nan"))
    out_b = torch.full_like(b.q, float("nan"))
    status = ctypes.c_int(-1)
    stream = torch.cuda.current_stream().cuda_stream
    assert _noalloc(lib, a, out_a) == 0, lib.tvk_last_error()
    assert lib.tvk_paged_decode_noalloc_status(ctypes.byref(status), stream) == 0 and status.value == 0
    assert _noalloc(lib, b, out_b) == 0, lib.tvk_last_error()
    assert lib.tvk_paged_decode_noalloc_status(ctypes.byref(status), stream) == 0 and status.value == 0
    torch.cuda.synchronize()
    _close(out_a, _with_workspace(a), a.q.dtype)
    _close(out_b, _with_workspace(b), b.q.dtype)
    # and once more on the first case, after the scratch held the second call's partials
    out_a2 = torch.full_like(a.q, float("nan"))
    assert _noalloc(lib, a, out_a2) == 0, lib.tvk_last_error()
    assert lib.tvk_paged_decode_noalloc_status(ctypes.byref(status), stream) == 0 and status.value == 0
    torch.cuda.synchronize()
    _close(out_a2, out_a, a.q.dtype)


def test_noalloc_refuses_calls_beyond_its_scratch(cuda):
    from tinyvllm_b200 import _lib
    lib = _lib.lib()
    need = lib.tvk_paged_decode_workspace_size(4096, 32, 8, 128, 16, 4096, -1)
    assert need > (64 << 20)
    stream = torch.cuda.current_stream().cuda_stream
    # a batch of 4096 with 4096-block tables is refused by the size guard before any
    # launch; the buffers are null, so a regressed guard would still be stopped by the
    # null-pointer check instead of launching over undersized buffers
    rc = lib.tvk_paged_decode_attention_noalloc(None, None, None, None, None, None, 4096, 32, 8, 128, 16, 1000,
                                                4096, -1, 1, stream)
    assert rc == -4
    assert b"fixed" in lib.tvk_last_error()
