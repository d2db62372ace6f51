"""Bounded kernel waits: a wait that runs out sets the status word, the kernel
returns, the caller is told, and the next call is correct (GPU).

``tvk_debug_arm_wait_timeout`` arms the next tensor-core decode or prefill launch
on this thread with a short wait limit and tells its producer warp to issue no
loads.  Nothing ever arrives on the consumers' barriers, so their first bounded
wait runs out: the kernel writes 1 into the workspace status word and returns.
No GPU fault, trap or hang is involved -- every wait in both kernels carries a
wall-time limit.  The reference's counterpart is an exception on the host
(tinyvllm raises on out-of-memory, core/block_manager.py:35-36).
"""

import ctypes
import time

import numpy as np
import pytest
import torch

from oracle import attention as oa

pytestmark = pytest.mark.gpu

LIMIT_NS = 5_000_000   # 5 ms


def _np(t):
    return t.detach().float().cpu().numpy()


def _decode_case(cuda, seed=41):
    from tinyvllm_b200 import workloads
    return workloads.decode_case(6, 32, 8, 128, 16, [5, 70, 300, 900, 1500, 2100], dtype=torch.float16,
                                 device=cuda, seed=seed)


def _decode_ref(case):
    return oa.paged_decode_attention(_np(case.q), _np(case.k_cache), _np(case.v_cache),
                                     case.block_tables.cpu().numpy(), case.context_lens.cpu().numpy(),
                                     case.n_heads, case.n_kv_heads, case.head_dim, case.block_size)


def _arm():
    from tinyvllm_b200 import _lib
    assert _lib.lib().tvk_debug_arm_wait_timeout(LIMIT_NS) == 0


def test_decode_wait_runs_out_then_next_call_is_correct(cuda):
    from tinyvllm_b200 import _lib
    from tinyvllm_b200.attention import check_workspace, paged_decode_attention, workspace_status
    case = _decode_case(cuda)
    args = (case.q, case.k_cache, case.v_cache, case.block_tables, case.context_lens, 32, 8, 128, 16)
    paged_decode_attention(*args)              # creates this stream's workspace
    torch.cuda.synchronize()
    assert workspace_status(cuda) == 0
    _arm()
    t0 = time.perf_counter()
    paged_decode_attention(*args)
    torch.cuda.synchronize()
    assert time.perf_counter() - t0 < 1.5      # returned after its own short limit
    assert workspace_status(cuda) == 1
    with pytest.raises(_lib.TvkError, match="timed out"):
        check_workspace(cuda, "decode")        # raises and re-zeroes the header
    assert workspace_status(cuda) == 0
    out = paged_decode_attention(*args, check=True)
    err = np.abs(_np(out) - _decode_ref(case)).max()
    assert err <= 2e-2


def test_decode_check_flag_raises(cuda):
    from tinyvllm_b200 import _lib
    from tinyvllm_b200.attention import paged_decode_attention, workspace_status
    case = _decode_case(cuda, seed=42)
    args = (case.q, case.k_cache, case.v_cache, case.block_tables, case.context_lens, 32, 8, 128, 16)
    _arm()
    with pytest.raises(_lib.TvkError, match="timed out"):
        paged_decode_attention(*args, check=True)
    assert workspace_status(cuda) == 0
    out = paged_decode_attention(*args, check=True)
    assert np.abs(_np(out) - _decode_ref(case)).max() <= 2e-2


def test_prefill_wait_runs_out_then_next_call_is_correct(cuda):
    from tinyvllm_b200 import _lib
    from tinyvllm_b200.attention import flash_prefill_attention_varlen, workspace_status
    g = torch.Generator(device=cuda).manual_seed(43)
    lens = [40, 300]
    T = sum(lens)
    q = torch.randn(T, 32, 64, generator=g, device=cuda).half()
    k = torch.randn(T, 4, 64, generator=g, device=cuda).half()
    v = torch.randn(T, 4, 64, generator=g, device=cuda).half()
    cu = torch.tensor([0, lens[0], T], dtype=torch.int32, device=cuda)
    flash_prefill_attention_varlen(q, k, v, cu, max(lens), True, check=True)
    _arm()
    t0 = time.perf_counter()
    with pytest.raises(_lib.TvkError, match="timed out"):
        flash_prefill_attention_varlen(q, k, v, cu, max(lens), True, check=True)
    assert time.perf_counter() - t0 < 1.5
    assert workspace_status(cuda, "prefill") == 0
    out = flash_prefill_attention_varlen(q, k, v, cu, max(lens), True, check=True)
    for i in range(2):
        a, b = int(cu[i]), int(cu[i + 1])
        ref = oa.flash_prefill_attention(_np(q[a:b])[None], _np(k[a:b])[None], _np(v[a:b])[None], True)[0]
        assert np.abs(_np(out[a:b]) - ref).max() <= 2e-2


def test_noalloc_status_reports_a_timed_out_call(cuda):
    """The no-allocation entry point keeps its status word inside the library's
    fixed scratch; tvk_paged_decode_noalloc_status reads it back."""
    from tinyvllm_b200 import _lib
    lib = _lib.lib()
    case = _decode_case(cuda, seed=44)
    stream = torch.cuda.current_stream().cuda_stream

    def call(out):
        return lib.tvk_paged_decode_attention_noalloc(
            case.q.data_ptr(), case.k_cache.data_ptr(), case.v_cache.data_ptr(), case.block_tables.data_ptr(),
            case.context_lens.data_ptr(), out.data_ptr(), case.batch, 32, 8, 128, 16, case.k_cache.shape[0],
            case.block_tables.shape[1], -1, 1, stream)

    status = ctypes.c_int(-1)
    out = torch.zeros_like(case.q)
    _arm()
    assert call(out) == 0, lib.tvk_last_error()
    assert lib.tvk_paged_decode_noalloc_status(ctypes.byref(status), stream) == 0
    assert status.value == 1
    assert call(out) == 0, lib.tvk_last_error()        # clears the word, runs normally
    assert lib.tvk_paged_decode_noalloc_status(ctypes.byref(status), stream) == 0
    assert status.value == 0
    assert np.abs(_np(out) - _decode_ref(case)).max() <= 2e-2


def test_engine_step_raises_on_a_timed_out_kernel(cuda):
    """The engine reads the status word every step: a timed-out kernel inside a step
    raises instead of yielding tokens computed from incomplete attention."""
    from tinyvllm_b200 import _lib
    from tinyvllm_b200.engine import LLMEngine, SamplingParams
    from tinyvllm_b200.model import Llama, LlamaConfig
    cfg = LlamaConfig(dim=256, n_layers=2, n_heads=4, n_kv_heads=2, vocab_size=97, hidden_dim=512,
                      max_seq_len=256, dtype="float16")
    model = Llama(cfg, device="cuda", seed=45, init_std=0.1)
    eng = LLMEngine(model, max_batch_size=2, num_blocks=32, use_cuda_graphs=True)
    eng.add_request(list(range(1, 40)), SamplingParams(max_tokens=4))
    _arm()                                  # consumed by the prefill's first attention launch
    with pytest.raises(_lib.TvkError, match="timed out"):
        eng.step()
    # the workspace header was re-zeroed: a fresh engine on the same model runs normally
    eng2 = LLMEngine(model, max_batch_size=2, num_blocks=32, use_cuda_graphs=True)
    eng2.add_request(list(range(1, 40)), SamplingParams(max_tokens=4))
    outs = list(eng2.run())
    assert len(outs) == 1 and len(outs[0].tokens) == 4
