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
_workspaces: Dict[Tuple[int, int], torch.Tensor] = {}


def _workspace(device: torch.device, nbytes: int) -> torch.Tensor:
    """Per-(device, stream) scratch buffer, grown on demand, zeroed when created
    (its first word is the kernels' time-out status)."""
    key = (device.index if device.index is not None else torch.cuda.current_device(),
           torch.cuda.current_stream(device).cuda_stream)
    with _ws_lock:
        ws = _workspaces.get(key)
        if ws is None or ws.numel() < nbytes:
            ws = torch.zeros(max(nbytes, 1 << 20), dtype=torch.uint8, device=device)
            _workspaces[key] = ws
        return ws


def workspace_status(device: Optional[torch.device] = None) -> int:
    """Status word of the current stream's workspace (non-zero: a kernel wait timed out)."""
    device = device or torch.device("cuda", torch.cuda.current_device())
    ws = _workspace(device, 0)
    return int(ws[:4].view(torch.int32).item())


def paged_decode_attention(queries: torch.Tensor, k_cache: torch.Tensor, v_cache: torch.Tensor,
                           block_tables: torch.Tensor, context_lens: torch.Tensor,
                           n_heads: int, n_kv_heads: int, head_dim: int, block_size: int,
                           max_context_len: Optional[int] = None, *,
                           out: Optional[torch.Tensor] = None) -> torch.Tensor:
    """Paged attention for decode (tinyvllm/model/llama.py:97-144).

    queries [B,1,Hq,D]; k_cache/v_cache [N,block_size,Hkv,D] (one layer's pool);
    block_tables int32 [B,max_blocks]; context_lens int32 [B].  Returns [B,1,Hq,D]
    in the pool dtype.  ``max_context_len=None`` attends over the whole table
    width masked by ``context_lens`` like the reference; an int truncates the
    table to ``ceil(max_context_len / block_size)`` blocks first.
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
    return out
