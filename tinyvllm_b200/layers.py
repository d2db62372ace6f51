"""The per-layer ops around the attention, on the sm_100a kernels.

Each function mirrors one piece of ``tinyvllm/model/llama.py`` (cited per
function) on torch CUDA tensors and calls ``libtvk.so`` directly; arithmetic is
fp32 with one rounding to the storage dtype.
"""

from __future__ import annotations

from typing import Optional, Tuple

import numpy as np
import torch

from . import _lib


def _stream(dev):
    return _lib.stream_ptr(dev)


def _contig(*ts):
    for t in ts:
        if t is not None and not t.is_contiguous():
            raise ValueError("tensors must be contiguous")


def precompute_freqs_cis(dim: int, seq_len: int, theta: float = 10000.0,
                         device="cuda") -> Tuple[torch.Tensor, torch.Tensor]:
    """fp32 cos/sin tables [seq_len, dim/2] (llama.py:26-31), built on the host in
    float32 the way the reference builds them, then copied to the device once."""
    freqs = np.float32(1.0) / (np.float32(theta) ** (np.arange(0, dim, 2, dtype=np.float32) / np.float32(dim)))
    f = np.arange(seq_len, dtype=np.float32)[:, None] * freqs[None, :]
    return (torch.from_numpy(np.cos(f).astype(np.float32)).to(device),
            torch.from_numpy(np.sin(f).astype(np.float32)).to(device))


def rms_norm(x: torch.Tensor, weight: torch.Tensor, eps: float = 1e-5, *,
             residual: Optional[torch.Tensor] = None, out: Optional[torch.Tensor] = None,
             write_kv: Optional[Tuple[torch.Tensor, torch.Tensor, torch.Tensor, torch.Tensor, torch.Tensor]] = None
             ) -> torch.Tensor:
    """RMSNorm (llama.py:21-23) over the last dim.  With ``residual`` the kernel first
    forms ``residual += x`` (in place, rounded to the dtype) and normalises that sum.
    With ``write_kv = (k, v, slots, k_cache, v_cache)`` the same launch also stores
    row r's k/v rows [rows, Hkv, D] at pool slot slots[r] (the decode K/V append of
    llama.py:381-386, after the attention that read the slot's old contents)."""
    extra = write_kv if write_kv is not None else ()
    dev = _lib.require_cuda(x, weight, *(t for t in (residual, out) if t is not None), *extra)
    _contig(x, weight, residual, out, *extra)
    dim = x.shape[-1]
    rows = x.numel() // dim
    if out is None:
        out = torch.empty_like(x)
    if write_kv is None:
        rc = _lib.lib().tvk_rms_norm(_lib.ptr(x), _lib.ptr(residual), _lib.ptr(residual), _lib.ptr(weight),
                                     _lib.ptr(out), rows, dim, float(eps), _lib.dtype_code(x), _stream(dev))
        _lib.check(rc, "tvk_rms_norm")
        return out
    k, v, slots, kc, vc = write_kv
    if slots.dtype != torch.int64 or slots.numel() != rows or k.shape[0] != rows:
        raise ValueError("write_kv needs one int64 slot and one k/v row per norm row")
    rc = _lib.lib().tvk_rms_norm_write_kv(
        _lib.ptr(x), _lib.ptr(residual), _lib.ptr(residual), _lib.ptr(weight), _lib.ptr(out), rows, dim, float(eps),
        _lib.ptr(k), _lib.ptr(v), _lib.ptr(slots), _lib.ptr(kc), _lib.ptr(vc), kc.shape[2], kc.shape[3], kc.shape[0],
        kc.shape[1], _lib.dtype_code(x), _stream(dev))
    _lib.check(rc, "tvk_rms_norm_write_kv")
    return out


def apply_rope_(q: torch.Tensor, k: torch.Tensor, cos: torch.Tensor, sin: torch.Tensor,
                positions: torch.Tensor) -> None:
    """In-place interleaved RoPE (llama.py:34-55) on q [T,Hq,D] and k [T,Hkv,D];
    ``positions`` int32 [T] indexes the fp32 tables."""
    dev = _lib.require_cuda(q, k, cos, sin, positions)
    _contig(q, k, cos, sin, positions)
    T, hq, d = q.shape
    rc = _lib.lib().tvk_rope(_lib.ptr(q), _lib.ptr(k), _lib.ptr(cos), _lib.ptr(sin), _lib.ptr(positions), T, hq,
                             k.shape[1], d, cos.shape[0], _lib.dtype_code(q), _stream(dev))
    _lib.check(rc, "tvk_rope")


def apply_rope_write_kv_(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor, cos: torch.Tensor, sin: torch.Tensor,
                         positions: torch.Tensor, slots: torch.Tensor, k_cache: torch.Tensor,
                         v_cache: torch.Tensor) -> None:
    """RoPE on q/k in place, then the roped k and v rows stored at their paged slots."""
    dev = _lib.require_cuda(q, k, v, cos, sin, positions, slots, k_cache, v_cache)
    _contig(q, k, v, cos, sin, positions, slots, k_cache, v_cache)
    T, hq, d = q.shape
    rc = _lib.lib().tvk_rope_write_kv(
        _lib.ptr(q), _lib.ptr(k), _lib.ptr(v), _lib.ptr(cos), _lib.ptr(sin), _lib.ptr(positions), _lib.ptr(slots),
        _lib.ptr(k_cache), _lib.ptr(v_cache), T, hq, k.shape[1], d, cos.shape[0], k_cache.shape[0],
        k_cache.shape[1], _lib.dtype_code(q), _stream(dev))
    _lib.check(rc, "tvk_rope_write_kv")


def qkv_rope(qkv: torch.Tensor, n_heads: int, n_kv_heads: int, head_dim: int, cos: torch.Tensor,
             sin: torch.Tensor, positions: torch.Tensor, *, slots: Optional[torch.Tensor] = None,
             k_cache: Optional[torch.Tensor] = None, v_cache: Optional[torch.Tensor] = None,
             out: Optional[Tuple[torch.Tensor, torch.Tensor, torch.Tensor]] = None):
    """Split packed projection rows ``qkv`` [T, >= (Hq+2Hkv)*D] (one GEMM against
    wq|wk|wv, llama.py:174-176) into contiguous q [T,Hq,D], k, v [T,Hkv,D] with RoPE
    on q and k (llama.py:178-179); with ``slots`` the roped k and v also go to the pool."""
    dev = _lib.require_cuda(qkv, cos, sin, positions, *(t for t in (slots, k_cache, v_cache) if t is not None))
    if qkv.stride(-1) != 1 or qkv.dim() != 2:
        raise ValueError("qkv must be [T, C] with contiguous rows")
    T = qkv.shape[0]
    if out is None:
        q = torch.empty(T, n_heads, head_dim, dtype=qkv.dtype, device=qkv.device)
        k = torch.empty(T, n_kv_heads, head_dim, dtype=qkv.dtype, device=qkv.device)
        v = torch.empty(T, n_kv_heads, head_dim, dtype=qkv.dtype, device=qkv.device)
    else:
        q, k, v = out
    nb = k_cache.shape[0] if k_cache is not None else 0
    bs = k_cache.shape[1] if k_cache is not None else 0
    rc = _lib.lib().tvk_qkv_rope(_lib.ptr(qkv), qkv.stride(0), _lib.ptr(q), _lib.ptr(k), _lib.ptr(v), _lib.ptr(cos),
                                 _lib.ptr(sin), _lib.ptr(positions), _lib.ptr(slots), _lib.ptr(k_cache),
                                 _lib.ptr(v_cache), T, n_heads, n_kv_heads, head_dim, cos.shape[0], nb, bs,
                                 _lib.dtype_code(qkv), _stream(dev))
    _lib.check(rc, "tvk_qkv_rope")
    return q, k, v


def write_kv_slots(k: torch.Tensor, v: torch.Tensor, slots: torch.Tensor, k_cache: torch.Tensor,
                   v_cache: torch.Tensor) -> None:
    """KVCache.write_kv for a batch of rows (core/kv_cache.py:34-38): k/v [T,Hkv,D] ->
    pool slots (int64 [T], flat ``block*block_size + offset``; negative skips)."""
    dev = _lib.require_cuda(k, v, slots, k_cache, v_cache)
    _contig(k, v, slots, k_cache, v_cache)
    if slots.dtype != torch.int64:
        raise TypeError("slots must be int64")
    T, hkv, d = k.shape
    rc = _lib.lib().tvk_write_kv_slots(_lib.ptr(k), _lib.ptr(v), _lib.ptr(slots), _lib.ptr(k_cache),
                                       _lib.ptr(v_cache), T, hkv, d, k_cache.shape[0], k_cache.shape[1],
                                       _lib.dtype_code(k), _stream(dev))
    _lib.check(rc, "tvk_write_kv_slots")


def silu_mul(a: torch.Tensor, b: torch.Tensor, out: Optional[torch.Tensor] = None) -> torch.Tensor:
    """silu(a) * b over the last dim (llama.py:221); a/b may be column slices of one
    packed [rows, 2H] gate|up tensor."""
    dev = _lib.require_cuda(a, b)
    cols = a.shape[-1]
    rows = a.numel() // cols
    if a.stride(-1) != 1 or b.stride(-1) != 1:
        raise ValueError("last dim must be contiguous")
    if out is None:
        out = torch.empty(a.shape, dtype=a.dtype, device=a.device)
    a2 = a.reshape(rows, cols) if a.is_contiguous() else a
    b2 = b.reshape(rows, cols) if b.is_contiguous() else b
    rc = _lib.lib().tvk_silu_mul(_lib.ptr(a), _lib.ptr(b), _lib.ptr(out), rows, cols, a2.stride(0), b2.stride(0),
                                 cols, _lib.dtype_code(a), _stream(dev))
    _lib.check(rc, "tvk_silu_mul")
    return out


def embedding(table: torch.Tensor, tokens: torch.Tensor, out: Optional[torch.Tensor] = None) -> torch.Tensor:
    """Row gather (llama.py:276,310): tokens int32 [...] -> [..., dim]."""
    dev = _lib.require_cuda(table, tokens)
    _contig(table, tokens)
    vocab, dim = table.shape
    n = tokens.numel()
    if out is None:
        out = torch.empty(*tokens.shape, dim, dtype=table.dtype, device=table.device)
    rc = _lib.lib().tvk_embedding(_lib.ptr(table), _lib.ptr(tokens), _lib.ptr(out), n, dim, vocab,
                                  _lib.dtype_code(table), None, _stream(dev))
    _lib.check(rc, "tvk_embedding")
    return out


def greedy_argmax(logits: torch.Tensor, out: Optional[torch.Tensor] = None) -> torch.Tensor:
    """Greedy pick (core/sampling.py:133-134): int32 argmax per row, first index on ties."""
    dev = _lib.require_cuda(logits)
    vocab = logits.shape[-1]
    rows = logits.numel() // vocab
    if logits.stride(-1) != 1:
        raise ValueError("last dim must be contiguous")
    stride = logits.stride(-2) if logits.dim() > 1 else vocab
    if out is None:
        out = torch.empty(rows, dtype=torch.int32, device=logits.device)
    rc = _lib.lib().tvk_argmax(_lib.ptr(logits), _lib.ptr(out), rows, vocab, stride, _lib.dtype_code(logits),
                               _stream(dev))
    _lib.check(rc, "tvk_argmax")
    return out
