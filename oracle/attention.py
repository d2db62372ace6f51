"""CPU oracle: numpy restatement of tinyvllm's attention hot path.

TEST INFRASTRUCTURE ONLY. Nothing in the product package imports this module;
only ``tests/``, ``__graft_entry__.smoke()`` and ``bench.py``'s CPU-baseline /
reference arm may call it, and only as the checker or the timed CPU baseline.

Every function restates the reference algorithm step for step (gather order,
GQA expand on a new axis, additive ``-1e9`` masks, softmax over the full
padded length) in float32, following the cited lines of
``tinyvllm/model/llama.py``.  The reference runs on tinygrad, which is not
installable here, so numeric parity with tinygrad itself is pinned only
through the reference tests' own known answers and self-consistency checks
(paged == dense attention, first-token / last-token causal answers); those
checks live in ``tests/test_oracle.py``.

Inputs may be any float dtype; they are promoted to float32 first, which is
how the oracle defines fp16/bf16 precision ("fp32 arithmetic on the rounded
inputs").
"""

from __future__ import annotations

import math
from typing import Optional, Tuple

import numpy as np

NEG_MASK = np.float32(-1e9)


def _f32(x) -> np.ndarray:
    return np.asarray(x, dtype=np.float32)


def softmax_lastdim(x: np.ndarray) -> np.ndarray:
    """tinygrad ``Tensor.softmax``: ``e = exp(x - max); e / sum(e)``."""
    m = x.max(axis=-1, keepdims=True)
    e = np.exp(x - m)
    return e / e.sum(axis=-1, keepdims=True)


def paged_decode_attention(queries, k_cache, v_cache, block_tables, context_lens,
                           n_heads: int, n_kv_heads: int, head_dim: int,
                           block_size: int, max_context_len: Optional[int] = None) -> np.ndarray:
    """Restates ``paged_decode_attention`` (tinyvllm/model/llama.py:97-144).

    queries [B,1,Hq,D]; k_cache/v_cache [N,bs,Hkv,D]; block_tables int [B,maxblk];
    context_lens int [B].  Returns float32 [B,1,Hq,D].
    """
    q_in = _f32(queries)
    kc = _f32(k_cache)
    vc = _f32(v_cache)
    bt = np.asarray(block_tables, dtype=np.int64)
    ctx = np.asarray(context_lens, dtype=np.int64)
    batch_size = q_in.shape[0]
    total_max_blocks = bt.shape[1]

    # llama.py:113-118 -- optional truncation of the table to max_context_len
    if max_context_len is not None:
        blocks_needed = min((max_context_len + block_size - 1) // block_size, total_max_blocks)
        max_context = blocks_needed * block_size
        bt = bt[:, :blocks_needed]
    else:
        max_context = total_max_blocks * block_size

    # llama.py:120-122 -- gather every table entry (padding included)
    block_indices = bt.reshape(-1)
    k_g = kc[block_indices].reshape(batch_size, max_context, n_kv_heads, head_dim)
    v_g = vc[block_indices].reshape(batch_size, max_context, n_kv_heads, head_dim)

    # llama.py:125-128 -- GQA expand along a new axis 3, then merge
    if n_kv_heads != n_heads:
        n_rep = n_heads // n_kv_heads
        k_g = np.broadcast_to(k_g[:, :, :, None, :], (batch_size, max_context, n_kv_heads, n_rep, head_dim)
                              ).reshape(batch_size, max_context, n_heads, head_dim)
        v_g = np.broadcast_to(v_g[:, :, :, None, :], (batch_size, max_context, n_kv_heads, n_rep, head_dim)
                              ).reshape(batch_size, max_context, n_heads, head_dim)

    q = q_in.transpose(0, 2, 1, 3)            # [B,Hq,1,D]
    k = k_g.transpose(0, 2, 1, 3)             # [B,Hq,T,D]
    v = v_g.transpose(0, 2, 1, 3)

    scale = np.float32(1.0 / math.sqrt(head_dim))
    scores = np.matmul(q, k.transpose(0, 1, 3, 2)) * scale          # llama.py:134-135

    # llama.py:137-140 -- additive -1e9 mask where position >= ctx
    positions = np.arange(max_context).reshape(1, max_context)
    valid = (positions < ctx.reshape(batch_size, 1)).astype(np.float32)
    attn_mask = (np.float32(1.0) - valid) * NEG_MASK
    scores = scores + attn_mask.reshape(batch_size, 1, 1, max_context)

    w = softmax_lastdim(scores)                                       # llama.py:142
    out = np.matmul(w, v)                                             # llama.py:143
    return out.transpose(0, 2, 1, 3).astype(np.float32)               # llama.py:144


def flash_prefill_attention(queries, keys, values, causal: bool = True) -> np.ndarray:
    """Restates ``flash_prefill_attention`` (tinyvllm/model/llama.py:58-94).

    Inputs [1,L,H,D] (keys/values may have fewer heads).  Returns float32 [1,L,Hq,D].
    """
    q_in = _f32(queries)[0]
    k_in = _f32(keys)[0]
    v_in = _f32(values)[0]
    q_len, n_heads, head_dim = q_in.shape
    kv_len, n_kv_heads, _ = k_in.shape
    scale = np.float32(1.0 / math.sqrt(head_dim))

    # llama.py:73-77 -- GQA expand on a new axis 2
    if n_kv_heads != n_heads:
        n_rep = n_heads // n_kv_heads
        k_in = np.broadcast_to(k_in[:, :, None, :], (kv_len, n_kv_heads, n_rep, head_dim)).reshape(kv_len, n_heads, head_dim)
        v_in = np.broadcast_to(v_in[:, :, None, :], (kv_len, n_kv_heads, n_rep, head_dim)).reshape(kv_len, n_heads, head_dim)

    q = q_in.transpose(1, 0, 2)
    k = k_in.transpose(1, 0, 2)
    v = v_in.transpose(1, 0, 2)

    scores = np.matmul(q, k.transpose(0, 2, 1)) * scale              # llama.py:84
    if causal:                                                        # llama.py:86-90
        q_pos = np.arange(q_len).reshape(q_len, 1)
        kv_pos = np.arange(kv_len).reshape(1, kv_len)
        mask = (kv_pos > q_pos).astype(np.float32) * NEG_MASK
        scores = scores + mask[None]
    w = softmax_lastdim(scores)                                       # llama.py:92
    out = np.matmul(w, v)                                             # llama.py:93
    return out.transpose(1, 0, 2)[None].astype(np.float32)           # llama.py:94


def rms_norm(x, weight, eps: float = 1e-5) -> np.ndarray:
    """Restates ``RMSNorm.__call__`` (llama.py:21-23): x * rsqrt(mean(x^2)+eps) * w."""
    x = _f32(x)
    rms = np.float32(1.0) / np.sqrt((x * x).mean(axis=-1, keepdims=True) + np.float32(eps))
    return x * rms * _f32(weight)


def precompute_freqs_cis(dim: int, seq_len: int, theta: float = 10000.0) -> Tuple[np.ndarray, np.ndarray]:
    """Restates ``precompute_freqs_cis`` (llama.py:26-31) in float32."""
    freqs = np.float32(1.0) / (np.float32(theta) ** (np.arange(0, dim, 2, dtype=np.float32) / np.float32(dim)))
    t = np.arange(seq_len, dtype=np.float32)
    f = t[:, None] * freqs[None, :]
    return np.cos(f).astype(np.float32), np.sin(f).astype(np.float32)


def apply_rope(x, cos, sin) -> np.ndarray:
    """Restates ``apply_rope`` (llama.py:34-55): interleaved pairs (x[2i], x[2i+1]).

    x [B,S,H,D]; cos/sin [S,D/2] (prefill) or [B,S,D/2] (decode).
    """
    x = _f32(x)
    b, s, h, d = x.shape
    xr = x.reshape(b, s, h, d // 2, 2)
    x0, x1 = xr[..., 0], xr[..., 1]
    cos = _f32(cos)
    sin = _f32(sin)
    if cos.ndim == 2:
        c = cos[:s][None, :, None, :]
        sn = sin[:s][None, :, None, :]
    else:
        c = cos[:, :, None, :]
        sn = sin[:, :, None, :]
    out0 = x0 * c - x1 * sn
    out1 = x0 * sn + x1 * c
    return np.stack([out0, out1], axis=-1).reshape(b, s, h, d)


def silu(x) -> np.ndarray:
    x = _f32(x)
    return x / (np.float32(1.0) + np.exp(-x))


def silu_mul(a, b) -> np.ndarray:
    """The SwiGLU gate of ``FeedForward.__call__`` (llama.py:220-221): silu(w1 x) * (w3 x)."""
    return silu(a) * _f32(b)


def embedding(table, tokens) -> np.ndarray:
    """``tinygrad.nn.Embedding`` row gather (llama.py:258,276,310)."""
    return np.asarray(table)[np.asarray(tokens, dtype=np.int64)]


def greedy_argmax(logits) -> np.ndarray:
    """Greedy pick (core/sampling.py:133-134): argmax over the vocab, first index on ties."""
    return np.argmax(_f32(logits), axis=-1).astype(np.int64)
