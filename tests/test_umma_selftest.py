"""tcgen05 operand-layout self-test (GPU): one 128 x n x k UMMA tile through the
same descriptors and TMA swizzles the prefill kernel uses (A from shared memory
or from TMEM), against torch fp32."""

import pytest
import torch

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("dtype", [torch.float16, torch.bfloat16])
@pytest.mark.parametrize("n", [64, 128])
@pytest.mark.parametrize("k", [64, 128])
@pytest.mark.parametrize("b_mn_major", [0, 1])
@pytest.mark.parametrize("a_in_tmem", [0, 1])
def test_umma_tile(cuda, dtype, n, k, b_mn_major, a_in_tmem):
    from tinyvllm_b200 import _lib
    lib = _lib.lib()
    g = torch.Generator(device=cuda).manual_seed(n * 1000 + k + b_mn_major)
    a = torch.randn(128, k, generator=g, device=cuda).to(dtype)
    b = torch.randn((k, n) if b_mn_major else (n, k), generator=g, device=cuda).to(dtype)
    c = torch.full((128, n), float("nan"), device=cuda)
    status = torch.zeros(1, dtype=torch.int32, device=cuda)
    rc = lib.tvk_selftest_umma_gemm(a.data_ptr(), b.data_ptr(), c.data_ptr(), n, k, b_mn_major, a_in_tmem,
                                    1 if dtype == torch.float16 else 2, status.data_ptr(),
                                    torch.cuda.current_stream().cuda_stream)
    assert rc == 0, lib.tvk_last_error()
    torch.cuda.synchronize()
    assert int(status.item()) == 0
    ref = a.float() @ (b.float() if b_mn_major else b.float().t())
    err = (c - ref).abs().max().item()
    assert err < 1e-2 * max(1.0, ref.abs().max().item() / 10), f"max-abs {err}"
