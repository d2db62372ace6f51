"""Per-layer kernels against the CPU oracle (GPU).

Tolerances: fp32 1e-4 max-abs for elementwise ops (RMSNorm/RoPE/SiLU); fp16/bf16
within one or two ulps of the oracle computed on the same rounded inputs
(2e-2 max-abs, 1e-2 mean-relative).  Gathers, slot writes and argmax indices
are compared exactly.
"""

import numpy as np
import pytest
import torch

from oracle import attention as oa

pytestmark = pytest.mark.gpu

DTYPES = [torch.float32, torch.float16, torch.bfloat16]
TOL = {torch.float32: (1e-4, None), torch.float16: (2e-2, 1e-2), torch.bfloat16: (2e-2, 1e-2)}


def _np(t):
    return t.detach().float().cpu().numpy()


# per-element relative allowance: about two units in the last place of the dtype
RTOL = {torch.float32: 1e-5, torch.float16: 2.0 ** -9, torch.bfloat16: 2.0 ** -6}


def _check(got, expect, dtype, scale=1.0):
    """|got - expect| <= max_abs*scale + rtol*|expect| per element, plus the mean-relative bound."""
    max_abs, mean_rel = TOL[dtype]
    g = _np(got).astype(np.float64)
    e = np.asarray(expect, dtype=np.float64)
    err = np.abs(g - e)
    assert np.isfinite(g).all()
    bound = max_abs * scale + RTOL[dtype] * np.abs(e)
    assert (err <= bound).all(), f"max excess {(err - bound).max()} (max-abs {err.max()})"
    if mean_rel is not None:
        assert err.mean() / max(np.abs(e).mean(), 1e-12) <= mean_rel


def _gen(cuda, seed):
    return torch.Generator(device=cuda).manual_seed(seed)


@pytest.mark.parametrize("dtype", DTYPES)
@pytest.mark.parametrize("rows,dim", [(1, 64), (7, 2048), (64, 4096), (3, 32)])
def test_rms_norm(cuda, dtype, rows, dim):
    from tinyvllm_b200.layers import rms_norm
    g = _gen(cuda, rows + dim)
    x = torch.randn(rows, dim, generator=g, device=cuda).to(dtype)
    w = (1 + 0.1 * torch.randn(dim, generator=g, device=cuda)).to(dtype)
    out = rms_norm(x, w, 1e-5)
    _check(out, oa.rms_norm(_np(x), _np(w), 1e-5), dtype, scale=4)


@pytest.mark.parametrize("dtype", DTYPES)
def test_rms_norm_with_residual(cuda, dtype):
    from tinyvllm_b200.layers import rms_norm
    g = _gen(cuda, 5)
    x = torch.randn(16, 2048, generator=g, device=cuda).to(dtype)
    r = torch.randn(16, 2048, generator=g, device=cuda).to(dtype)
    w = torch.ones(2048, device=cuda, dtype=dtype)
    s_ref = (x.float() + r.float()).to(dtype)          # what TransformerBlock stores (llama.py:248)
    out = rms_norm(x, w, 1e-5, residual=r)
    assert torch.equal(r, s_ref)
    _check(out, oa.rms_norm(_np(s_ref), _np(w), 1e-5), dtype, scale=4)


def test_rms_norm_reference_properties(cuda):
    """tests/test_llama.py:67-100: unit RMS, zero input, scale invariance."""
    from tinyvllm_b200.layers import rms_norm
    x = torch.randn(2, 4, 64, device=cuda)
    w = torch.ones(64, device=cuda)
    y = rms_norm(x, w)
    assert torch.allclose(y.pow(2).mean(-1).sqrt(), torch.ones(2, 4, device=cuda), atol=1e-3)
    assert torch.count_nonzero(rms_norm(torch.zeros(1, 64, device=cuda), w)) == 0
    assert torch.allclose(rms_norm(x * 7, w), y, atol=1e-4)


@pytest.mark.parametrize("dtype", DTYPES)
@pytest.mark.parametrize("hq,hkv,d,theta", [(32, 4, 64, 1e4), (32, 8, 128, 5e5), (4, 4, 32, 1e4)])
def test_rope(cuda, dtype, hq, hkv, d, theta):
    from tinyvllm_b200.layers import apply_rope_, precompute_freqs_cis
    T = 37
    g = _gen(cuda, hq + d)
    q = torch.randn(T, hq, d, generator=g, device=cuda).to(dtype)
    k = torch.randn(T, hkv, d, generator=g, device=cuda).to(dtype)
    pos = torch.randint(0, 4096, (T,), generator=g, device=cuda, dtype=torch.int32)
    cos, sin = precompute_freqs_cis(d, 4096, theta, cuda)
    c_ref, s_ref = oa.precompute_freqs_cis(d, 4096, theta)
    assert np.array_equal(cos.cpu().numpy(), c_ref) and np.array_equal(sin.cpu().numpy(), s_ref)
    qn, kn, pn = _np(q), _np(k), pos.cpu().numpy()
    apply_rope_(q, k, cos, sin, pos)
    # decode form of the reference: per-token cos/sin rows [B, 1, D/2]
    exp_q = oa.apply_rope(qn[:, None], c_ref[pn][:, None], s_ref[pn][:, None])[:, 0]
    exp_k = oa.apply_rope(kn[:, None], c_ref[pn][:, None], s_ref[pn][:, None])[:, 0]
    _check(q, exp_q, dtype, scale=2)
    _check(k, exp_k, dtype, scale=2)


def test_rope_reference_properties(cuda):
    """tests/test_llama.py:155-185: identity at position 0, norm preserved."""
    from tinyvllm_b200.layers import apply_rope_, precompute_freqs_cis
    cos, sin = precompute_freqs_cis(64, 128, device=cuda)
    q = torch.randn(16, 4, 64, device=cuda)
    k = torch.randn(16, 4, 64, device=cuda)
    q0, k0 = q.clone(), k.clone()
    apply_rope_(q, k, cos, sin, torch.arange(16, dtype=torch.int32, device=cuda))
    assert torch.allclose(q[0], q0[0], atol=1e-6)
    assert torch.allclose(q.norm(dim=-1), q0.norm(dim=-1), rtol=1e-5)


@pytest.mark.parametrize("dtype", DTYPES)
def test_write_kv_slots_and_fused_rope(cuda, dtype):
    from tinyvllm_b200.layers import apply_rope_, apply_rope_write_kv_, precompute_freqs_cis, write_kv_slots
    g = _gen(cuda, 9)
    T, hq, hkv, d = 10, 32, 4, 64
    q = torch.randn(T, hq, d, generator=g, device=cuda).to(dtype)
    k = torch.randn(T, hkv, d, generator=g, device=cuda).to(dtype)
    v = torch.randn(T, hkv, d, generator=g, device=cuda).to(dtype)
    slots = torch.tensor([5, 17, 0, -1, 63, 40, 41, 42, 1000, 7], dtype=torch.int64, device=cuda)
    pos = torch.arange(100, 100 + T, dtype=torch.int32, device=cuda)
    cos, sin = precompute_freqs_cis(d, 256, device=cuda)
    # separate path: rope then write
    q1, k1 = q.clone(), k.clone()
    apply_rope_(q1, k1, cos, sin, pos)
    kc1 = torch.zeros(4, 16, hkv, d, dtype=dtype, device=cuda)
    vc1 = torch.zeros_like(kc1)
    write_kv_slots(k1, v, slots, kc1, vc1)
    # fused path
    q2, k2 = q.clone(), k.clone()
    kc2 = torch.zeros_like(kc1)
    vc2 = torch.zeros_like(kc1)
    apply_rope_write_kv_(q2, k2, v, cos, sin, pos, slots, kc2, vc2)
    torch.cuda.synchronize()
    assert torch.equal(q1, q2) and torch.equal(k1, k2)
    assert torch.equal(kc1, kc2) and torch.equal(vc1, vc2)
    flat_k, flat_v = kc1.view(-1, hkv, d), vc1.view(-1, hkv, d)
    for t, s in enumerate(slots.tolist()):
        if 0 <= s < 64:
            assert torch.equal(flat_k[s], k1[t]) and torch.equal(flat_v[s], v[t])
    written = {s for s in slots.tolist() if 0 <= s < 64}
    untouched = [i for i in range(64) if i not in written]
    assert torch.count_nonzero(flat_k[untouched]) == 0


@pytest.mark.parametrize("dtype", DTYPES)
@pytest.mark.parametrize("hkv,d", [(4, 64), (8, 128)])
def test_rms_norm_write_kv_matches_separate_ops(cuda, dtype, hkv, d):
    """rms_norm(write_kv=...) == rms_norm(residual=...) then tvk_write_kv_slots, bit for bit."""
    from tinyvllm_b200.layers import rms_norm, write_kv_slots
    g = _gen(cuda, 33 + d)
    B, dim = 10, 2048
    x = torch.randn(B, dim, generator=g, device=cuda).to(dtype)
    r = torch.randn(B, dim, generator=g, device=cuda).to(dtype)
    w = (1 + 0.1 * torch.randn(dim, generator=g, device=cuda)).to(dtype)
    k = torch.randn(B, hkv, d, generator=g, device=cuda).to(dtype)
    v = torch.randn(B, hkv, d, generator=g, device=cuda).to(dtype)
    slots = torch.tensor([5, 17, 0, -1, 63, 40, 41, 42, 1000, 7], dtype=torch.int64, device=cuda)
    kc1 = torch.randn(4, 16, hkv, d, generator=g, device=cuda).to(dtype)
    vc1 = torch.randn(4, 16, hkv, d, generator=g, device=cuda).to(dtype)
    kc2, vc2 = kc1.clone(), vc1.clone()
    r1, r2 = r.clone(), r.clone()
    out1 = rms_norm(x, w, 1e-5, residual=r1)
    write_kv_slots(k, v, slots, kc1, vc1)
    out2 = rms_norm(x, w, 1e-5, residual=r2, write_kv=(k, v, slots, kc2, vc2))
    torch.cuda.synchronize()
    # against the oracle directly: the stored residual sum is the dtype-rounded
    # x + r (llama.py:248), the output rms_norm of it (llama.py:14-23)
    s_ref = (x.float() + r.float()).to(dtype)
    assert torch.equal(r2, s_ref)
    _check(out2, oa.rms_norm(_np(s_ref), _np(w), 1e-5), dtype, scale=4)
    assert torch.equal(out1, out2) and torch.equal(r1, r2)
    assert torch.equal(kc1, kc2) and torch.equal(vc1, vc2)
    flat_k, flat_v = kc2.view(-1, hkv, d), vc2.view(-1, hkv, d)
    for t, s in enumerate(slots.tolist()):
        if 0 <= s < 64:
            assert torch.equal(flat_k[s], k[t]) and torch.equal(flat_v[s], v[t])
    with pytest.raises(ValueError):
        rms_norm(x, w, residual=r2, write_kv=(k, v, slots[:3], kc2, vc2))


@pytest.mark.parametrize("dtype", DTYPES)
@pytest.mark.parametrize("with_slots", [False, True])
def test_qkv_rope_matches_separate_ops(cuda, dtype, with_slots):
    """One packed projection row split + RoPE == slicing then tvk_rope (and tvk_write_kv_slots)."""
    from tinyvllm_b200.layers import apply_rope_, precompute_freqs_cis, qkv_rope, write_kv_slots
    g = _gen(cuda, 21)
    T, hq, hkv, d = 13, 32, 8, 128
    cols = (hq + 2 * hkv) * d
    qkv = torch.randn(T, cols + 64, generator=g, device=cuda).to(dtype)[:, :cols]   # strided rows
    pos = torch.randint(0, 512, (T,), generator=g, device=cuda, dtype=torch.int32)
    cos, sin = precompute_freqs_cis(d, 1024, 5e5, cuda)
    slots = torch.arange(3, 3 + T, dtype=torch.int64, device=cuda) if with_slots else None
    kc = torch.zeros(4, 16, hkv, d, dtype=dtype, device=cuda)
    vc = torch.zeros_like(kc)
    q, k, v = qkv_rope(qkv, hq, hkv, d, cos, sin, pos, slots=slots, k_cache=kc, v_cache=vc)
    torch.cuda.synchronize()
    # against the oracle directly: split of the packed projection row, RoPE of q
    # and k with the per-token table rows (llama.py:26-55, :316-326)
    c_ref, s_ref = oa.precompute_freqs_cis(d, 1024, 5e5)
    pn = pos.cpu().numpy()
    qkv_n = _np(qkv)
    q_n = qkv_n[:, :hq * d].reshape(T, hq, d)
    k_n = qkv_n[:, hq * d:(hq + hkv) * d].reshape(T, hkv, d)
    v_n = qkv_n[:, (hq + hkv) * d:].reshape(T, hkv, d)
    _check(q, oa.apply_rope(q_n[:, None], c_ref[pn][:, None], s_ref[pn][:, None])[:, 0], dtype, scale=2)
    _check(k, oa.apply_rope(k_n[:, None], c_ref[pn][:, None], s_ref[pn][:, None])[:, 0], dtype, scale=2)
    assert np.array_equal(_np(v), v_n)
    q2 = qkv[:, :hq * d].reshape(T, hq, d).contiguous()
    k2 = qkv[:, hq * d:(hq + hkv) * d].reshape(T, hkv, d).contiguous()
    v2 = qkv[:, (hq + hkv) * d:].reshape(T, hkv, d).contiguous()
    apply_rope_(q2, k2, cos, sin, pos)
    torch.cuda.synchronize()
    assert torch.equal(q, q2) and torch.equal(k, k2) and torch.equal(v, v2)
    if with_slots:
        kc2 = torch.zeros_like(kc)
        vc2 = torch.zeros_like(kc)
        write_kv_slots(k2, v2, slots, kc2, vc2)
        torch.cuda.synchronize()
        assert torch.equal(kc, kc2) and torch.equal(vc, vc2)
    else:
        assert torch.count_nonzero(kc) == 0


@pytest.mark.parametrize("dtype", DTYPES)
def test_silu_mul_packed_and_separate(cuda, dtype):
    from tinyvllm_b200.layers import silu_mul
    g = _gen(cuda, 11)
    H = 5632
    gu = (3 * torch.randn(9, 2 * H, generator=g, device=cuda)).to(dtype)
    a, b = gu[:, :H], gu[:, H:]
    out = silu_mul(a, b)
    an, bn = _np(a), _np(b)
    silu_rounded = torch.from_numpy(oa.silu(an)).to(dtype).float().numpy()  # silu stored in the dtype first
    _check(out, silu_rounded * bn, dtype, scale=4)
    out2 = silu_mul(a.contiguous(), b.contiguous())
    assert torch.equal(out, out2)


@pytest.mark.parametrize("dtype", DTYPES)
def test_embedding(cuda, dtype):
    from tinyvllm_b200.layers import embedding
    g = _gen(cuda, 12)
    table = torch.randn(1000, 2048, generator=g, device=cuda).to(dtype)
    tok = torch.randint(0, 1000, (3, 17), generator=g, device=cuda, dtype=torch.int32)
    out = embedding(table, tok)
    assert out.shape == (3, 17, 2048)
    assert torch.equal(out, table[tok.long()])


@pytest.mark.parametrize("dtype", DTYPES)
@pytest.mark.parametrize("vocab", [32000, 128256, 50, 33])
def test_argmax(cuda, dtype, vocab):
    from tinyvllm_b200.layers import greedy_argmax
    g = _gen(cuda, vocab)
    logits = torch.randn(64, vocab, generator=g, device=cuda).to(dtype)
    # force ties at the max to check the first-index rule
    logits[0, 5] = logits[0, 9] = 100
    logits[1, -1] = 100
    out = greedy_argmax(logits)
    exp = oa.greedy_argmax(_np(logits))
    assert np.array_equal(out.cpu().numpy(), exp)
    assert out[0].item() == 5


@pytest.mark.parametrize("dtype", DTYPES)
def test_argmax_ties_nans_and_infs(cuda, dtype):
    """First index on ties wherever the equal values sit (one 16-byte vector, two
    vectors of one thread, two threads); the first NaN wins a row that has one;
    a row of -inf gives index 0 -- all as numpy's argmax (sampling.py:133-134)."""
    from tinyvllm_b200.layers import greedy_argmax
    vocab = 128256
    g = _gen(cuda, 7)
    logits = torch.randn(6, vocab, generator=g, device=cuda).to(dtype)
    logits[0, 3] = logits[0, 1] = 50           # same 16-byte vector
    logits[1, 8 * 512 + 2] = logits[1, 2] = 50  # same thread, two of its in-flight vectors
    logits[2, 4000] = logits[2, 77] = 50        # different threads
    logits[3, 20] = float("nan")
    logits[3, 7] = float("nan")
    logits[4] = float("-inf")
    logits[5, -1] = float("nan")
    out = greedy_argmax(logits).cpu().numpy()
    assert out.tolist()[:5] == [1, 2, 77, 7, 0]
    assert out[5] == vocab - 1
    assert np.array_equal(out, oa.greedy_argmax(_np(logits)))


def test_argmax_strided_rows(cuda):
    from tinyvllm_b200.layers import greedy_argmax
    x = torch.randn(8, 3, 4096, device=cuda, dtype=torch.float16)
    last = x[:, -1, :]           # logits[:, -1, :] of a prefill (engine.py:134)
    out = greedy_argmax(last)
    assert np.array_equal(out.cpu().numpy(), oa.greedy_argmax(_np(last)))
