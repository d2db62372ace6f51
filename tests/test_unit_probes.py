"""Measurement probes (GPU): the tcgen05 issue probe and the exponential-unit
probe run to completion, and their rates stay within what the hardware can do
(an MMA cannot finish faster than the tensor pipe's nominal rate, nor the
exponential unit return more than 16 results per clock per SM)."""

import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu


def _sms(cuda):
    return torch.cuda.get_device_properties(cuda).multi_processor_count


@pytest.mark.parametrize("n", [64, 128, 256])
def test_mma_issue_probe(cuda, n):
    from tinyvllm_b200 import _lib
    lib = _lib.lib()
    n_sm = _sms(cuda)
    out = torch.zeros(2 * n_sm, dtype=torch.int64, device=cuda)
    n_mma = 1024
    for _ in range(2):
        rc = lib.tvk_probe_mma_issue(n, n_mma, out.data_ptr(), n_sm, torch.cuda.current_stream().cuda_stream)
        assert rc == 0, lib.tvk_last_error()
    torch.cuda.synchronize()
    c = out.view(n_sm, 2).cpu().numpy()
    assert (c[:, 1] > 0).all(), "a CTA's completion wait gave up"
    assert (c[:, 1] >= c[:, 0]).all()
    per_mma = np.median(c[:, 1]) / n_mma
    ideal = 128 * n * 16 * 2 / 8192.0
    assert 0.9 * ideal <= per_mma <= 8 * ideal, per_mma


@pytest.mark.parametrize("form", [0, 1, 2, 3])
def test_exp_unit_probe(cuda, form):
    from tinyvllm_b200 import _lib
    lib = _lib.lib()
    n_sm = _sms(cuda)
    out = torch.zeros(n_sm, dtype=torch.int64, device=cuda)
    sink = torch.zeros(1, dtype=torch.int32, device=cuda)
    n_iter = 256
    for _ in range(2):
        rc = lib.tvk_probe_exp_unit(form, n_iter, out.data_ptr(), n_sm, sink.data_ptr(),
                                    torch.cuda.current_stream().cuda_stream)
        assert rc == 0, lib.tvk_last_error()
    torch.cuda.synchronize()
    cyc = float(np.median(out.cpu().numpy()))
    per_op = 1 if form == 0 else 2
    rate = n_iter * 8 * 512 * per_op / cyc
    assert 2.0 <= rate <= 17.0, rate
