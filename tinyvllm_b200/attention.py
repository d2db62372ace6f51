"""Drop-in replacements for tinyvllm's attention functions, on the sm_100a kernels.

``paged_decode_attention`` and ``flash_prefill_attention`` keep the signatures
and argument meaning of ``tinyvllm/model/llama.py:97-108`` and ``:58-63``;
the arguments are torch CUDA tensors instead of tinygrad Tensors.  Each call
goes straight to ``libtvk.so`` through ctypes with raw device pointers on the
current torch stream.
"""

from __future__ import annotations

import threading
from typing import Dict, Optional, Tuple

import torch

from . import _lib

_ws_lock = threading.Lock()
_workspaces: Dict[Tuple[int, int, str], torch.Tensor] = {}


def _workspace(device: torch.device, nbytes: int, kind: str = "decode") -> torch.Tensor:
    """Per-(device, stream, kernel family) scratch buffer, grown on demand and zeroed
    when created (its first word is the kernels' time-out status)."""
    key = (device.index if device.index is not None else torch.cuda.current_device(),
           torch.cuda.current_stream(device).cuda_stream, kind)
    with _ws_lock:
        ws = _workspaces.get(key)
        if ws is None or ws.numel() < nbytes:
            ws = torch.zeros(max(nbytes, 1 << 20), dtype=torch.uint8, device=device)
            _workspaces[key] = ws
        return ws


def workspace_status(device: Optional[torch.device] = None, kind: str = "decode") -> int:
    """Status word of the current stream's workspace (non-zero: a kernel wait timed out)."""
    device = device or torch.device("cuda", torch.cuda.current_device())
    ws = _workspace(device, 0, kind)
    return int(ws[:4].view(torch.int32).item())


def status_word(device: Optional[torch.device] = None, kind: str = "decode") -> torch.Tensor:
    """The current stream's workspace status word as a one-element int32 device tensor
    (a view: a CUDA graph can copy it out alongside its results)."""
    device = device or torch.device("cuda", torch.cuda.current_device())
    return _workspace(device, 0, kind)[:4].view(torch.int32)


def check_workspace(device: Optional[torch.device] = None, kind: str = "decode", what: str = "kernel") -> None:
    """Raise ``TvkError`` if a bounded wait inside a kernel that used the current
    stream's ``kind`` workspace gave up (its output is then incomplete).  Reads the
    status word (a device-to-host copy, so the stream is synchronised); on a
    time-out the workspace header is zeroed first, so the next call starts clean."""
    device = device or torch.device("cuda", torch.cuda.current_device())
    ws = _workspace(device, 0, kind)
    if int(ws[:4].view(torch.int32).item()) != 0:
        ws[:256].zero_()
        raise _lib.TvkError(f"{what}: a bounded wait inside the kernel timed out; the output is incomplete")


def paged_decode_attention(queries: torch.Tensor, k_cache: torch.Tensor, v_cache: torch.Tensor,
                           block_tables: torch.Tensor, context_lens: torch.Tensor,
                           n_heads: int, n_kv_heads: int, head_dim: int, block_size: int,
                           max_context_len: Optional[int] = None, *,
                           out: Optional[torch.Tensor] = None, check: bool = False) -> torch.Tensor:
    """Paged attention for decode (tinyvllm/model/llama.py:97-144).

    queries [B,1,Hq,D]; k_cache/v_cache [N,block_size,Hkv,D] (one layer's pool);
    block_tables int32 [B,max_blocks]; context_lens int32 [B].  Returns [B,1,Hq,D]
    in the pool dtype.  ``max_context_len=None`` attends over the whole table
    width masked by ``context_lens`` like the reference; an int truncates the
    table to ``ceil(max_context_len / block_size)`` blocks first.  ``check=True``
    synchronises the stream and raises ``TvkError`` if a bounded wait inside the
    kernel timed out (the call is otherwise asynchronous; the engine checks once
    per step instead).
    """
    dev = _lib.require_cuda(queries, k_cache, v_cache, block_tables, context_lens)
    B = queries.shape[0]
    if queries.shape[1:] != (1, n_heads, head_dim):
        raise ValueError(f"queries must be [B,1,{n_heads},{head_dim}], got {tuple(queries.shape)}")
    if k_cache.dim() != 4 or k_cache.shape[1:] != (block_size, n_kv_heads, head_dim) or v_cache.shape != k_cache.shape:
        raise ValueError(f"k_cache/v_cache must be [N,{block_size},{n_kv_heads},{head_dim}], got "
                         f"{tuple(k_cache.shape)} / {tuple(v_cache.shape)}")
    if queries.dtype != k_cache.dtype or v_cache.dtype != k_cache.dtype:
        raise TypeError("queries, k_cache and v_cache must share one dtype")
    if block_tables.dtype != torch.int32 or context_lens.dtype != torch.int32:
        raise TypeError("block_tables and context_lens must be int32")
    if block_tables.dim() != 2 or block_tables.shape[0] != B or context_lens.shape != (B,):
        raise ValueError("block_tables must be [B,max_blocks] and context_lens [B]")
    for name, t in (("queries", queries), ("k_cache", k_cache), ("v_cache", v_cache),
                    ("block_tables", block_tables), ("context_lens", context_lens)):
        if not t.is_contiguous():
            raise ValueError(f"{name} must be contiguous")
    if out is None:
        out = torch.empty_like(queries)
    max_blocks = block_tables.shape[1]
    mcl = -1 if max_context_len is None else int(max_context_len)
    L = _lib.lib()
    nbytes = L.tvk_paged_decode_workspace_size(B, n_heads, n_kv_heads, head_dim, block_size, max_blocks, mcl)
    ws = _workspace(dev, nbytes)
    rc = L.tvk_paged_decode_attention(
        _lib.ptr(queries), _lib.ptr(k_cache), _lib.ptr(v_cache), _lib.ptr(block_tables),
        _lib.ptr(context_lens), _lib.ptr(out),
        B, n_heads, n_kv_heads, head_dim, block_size, k_cache.shape[0], max_blocks, mcl,
        _lib.dtype_code(k_cache), ws.data_ptr(), ws.numel(), _lib.stream_ptr(dev))
    _lib.check(rc, "tvk_paged_decode_attention")
    if check:
        check_workspace(dev, "decode", "tvk_paged_decode_attention")
    return out


def flash_prefill_attention_varlen(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor,
                                   cu_seqlens: torch.Tensor, max_seqlen: int, causal: bool = True, *,
                                   slot_mapping: Optional[torch.Tensor] = None,
                                   k_cache: Optional[torch.Tensor] = None,
                                   v_cache: Optional[torch.Tensor] = None,
                                   out: Optional[torch.Tensor] = None, check: bool = False) -> torch.Tensor:
    """Causal (or full) attention over a ragged batch of prompts packed along tokens.

    q [T,Hq,D], k/v [T,Hkv,D]; ``cu_seqlens`` int32 [n+1] prefix sums of the prompt
    lengths (device); ``max_seqlen`` >= the longest prompt.  With ``slot_mapping``
    (int64 [T], device; -1 skips a token) the kernel also writes each token's k/v
    row into ``k_cache/v_cache`` [N,block_size,Hkv,D] at flat slot
    ``block*block_size + offset`` -- the paged write of llama.py:188-209 fused
    into the attention kernel.  Returns [T,Hq,D].  ``check=True`` synchronises and
    raises ``TvkError`` if a bounded wait inside the kernel timed out.
    """
    tensors = [q, k, v, cu_seqlens] + [t for t in (slot_mapping, k_cache, v_cache) if t is not None]
    dev = _lib.require_cuda(*tensors)
    if q.dim() != 3 or k.dim() != 3 or v.shape != k.shape or q.shape[0] != k.shape[0] or q.shape[2] != k.shape[2]:
        raise ValueError(f"q must be [T,Hq,D] and k/v [T,Hkv,D]; got {tuple(q.shape)}, {tuple(k.shape)}, "
                         f"{tuple(v.shape)}")
    if q.dtype != k.dtype or v.dtype != k.dtype:
        raise TypeError("q, k and v must share one dtype")
    if cu_seqlens.dtype != torch.int32 or cu_seqlens.dim() != 1:
        raise TypeError("cu_seqlens must be a 1-D int32 tensor")
    for name, t in (("q", q), ("k", k), ("v", v), ("cu_seqlens", cu_seqlens)):
        if not t.is_contiguous():
            raise ValueError(f"{name} must be contiguous")
    T, Hq, D = q.shape
    Hkv = k.shape[1]
    n_seqs = cu_seqlens.shape[0] - 1
    num_blocks = block_size = 0
    if slot_mapping is not None:
        if k_cache is None or v_cache is None:
            raise ValueError("slot_mapping needs k_cache and v_cache")
        if slot_mapping.dtype != torch.int64 or slot_mapping.shape != (T,):
            raise TypeError("slot_mapping must be int64 [T]")
        if (k_cache.dim() != 4 or k_cache.shape[2:] != (Hkv, D) or v_cache.shape != k_cache.shape
                or k_cache.dtype != q.dtype or v_cache.dtype != q.dtype
                or not k_cache.is_contiguous() or not v_cache.is_contiguous()):
            raise ValueError("k_cache/v_cache must be contiguous [N,block_size,Hkv,D] in the dtype of q")
        num_blocks, block_size = k_cache.shape[0], k_cache.shape[1]
    if out is None:
        out = torch.empty_like(q)
    L = _lib.lib()
    ws = _workspace(dev, L.tvk_flash_prefill_workspace_size(n_seqs, T), "prefill")
    rc = L.tvk_flash_prefill_attention(
        _lib.ptr(q), _lib.ptr(k), _lib.ptr(v), _lib.ptr(out), _lib.ptr(cu_seqlens), n_seqs, int(max_seqlen), T,
        Hq, Hkv, D, 1 if causal else 0, _lib.dtype_code(q), _lib.ptr(slot_mapping), _lib.ptr(k_cache),
        _lib.ptr(v_cache), num_blocks, block_size, ws.data_ptr(), ws.numel(), _lib.stream_ptr(dev))
    _lib.check(rc, "tvk_flash_prefill_attention")
    if check:
        check_workspace(dev, "prefill", "tvk_flash_prefill_attention")
    return out


def flash_prefill_attention(queries: torch.Tensor, keys: torch.Tensor, values: torch.Tensor,
                            causal: bool = True) -> torch.Tensor:
    """Flash attention for prefill (tinyvllm/model/llama.py:58-94).

    Inputs [1,L,H,D] (keys/values may have fewer heads, GQA); returns [1,L,Hq,D].
    """
    dev = _lib.require_cuda(queries, keys, values)
    if queries.dim() != 4 or queries.shape[0] != 1:
        raise ValueError("queries must be [1,L,H,D]")
    q = queries[0].contiguous()
    k = keys[0].contiguous()
    v = values[0].contiguous()
    L = q.shape[0]
    cu = torch.tensor([0, L], dtype=torch.int32, device=dev)
    return flash_prefill_attention_varlen(q, k, v, cu, L, causal)[None]
