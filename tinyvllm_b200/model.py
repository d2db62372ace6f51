"""Llama forward passes built on the sm_100a kernels.

``Llama`` restates ``tinyvllm/model/llama.py:224-388`` for the hot path: the
decode step (``Llama.create_jit_decode`` / ``Llama.decode``, llama.py:290-388)
and a ragged prefill of several prompts at once (the reference prefills one
prompt per call, ``Llama.prefill`` llama.py:266-288; prompts are independent, so
batching them changes no result).  Every per-token op is one of this
package's kernels; the projections are plain library GEMMs (``torch.matmul`` on
cuBLAS) into preallocated buffers.

Weights are random N(0, std) from a seeded device generator (the benchmark
configurations load no checkpoints) with RMSNorm weights of one (llama.py:19).
Layout: every projection weight is stored [in, out] so a projection is x @ W.

K/V write order: ``kv_order="reference"`` reproduces the reference decode,
which attends over the cache *before* the step's own K/V is written
(llama.py:328-332 then 381-386) with block tables built before the new slot is
allocated (engine.py:247, llama.py:383); ``"append_first"`` writes the step's
K/V first, so the query also sees its own key.
"""

from __future__ import annotations

import math
from dataclasses import dataclass, field
from typing import Dict, List, Optional, Sequence

import numpy as np
import torch

from . import _lib, layers
from .attention import flash_prefill_attention_varlen, paged_decode_attention, status_word

_DTYPES = {"float32": torch.float32, "float16": torch.float16, "bfloat16": torch.bfloat16}


@dataclass
class LlamaConfig:
    """Fields of ``LlamaConfig`` (tinyvllm/model/weights.py:18-44); ``dtype`` also accepts "bfloat16"."""
    dim: int = 4096
    n_layers: int = 32
    n_heads: int = 32
    n_kv_heads: Optional[int] = None
    vocab_size: int = 32000
    hidden_dim: Optional[int] = None
    norm_eps: float = 1e-5
    max_seq_len: int = 2048
    rope_theta: float = 10000.0
    dtype: str = "float32"

    def __post_init__(self):
        self.n_kv_heads = self.n_kv_heads or self.n_heads
        self.hidden_dim = self.hidden_dim or 4 * self.dim
        if self.dtype not in _DTYPES:
            raise ValueError(f"dtype must be one of {sorted(_DTYPES)}")

    @property
    def head_dim(self) -> int:
        return self.dim // self.n_heads

    @property
    def torch_dtype(self) -> torch.dtype:
        return _DTYPES[self.dtype]


def tinyllama_config(dtype: str = "float16") -> LlamaConfig:
    """TinyLlama-1.1B shapes (benchmark config 4)."""
    return LlamaConfig(dim=2048, n_layers=22, n_heads=32, n_kv_heads=4, vocab_size=32000, hidden_dim=5632,
                       norm_eps=1e-5, max_seq_len=2048, rope_theta=10000.0, dtype=dtype)


def llama3_8b_config(dtype: str = "bfloat16") -> LlamaConfig:
    """Llama-3-8B shapes (benchmark config 5)."""
    return LlamaConfig(dim=4096, n_layers=32, n_heads=32, n_kv_heads=8, vocab_size=128256, hidden_dim=14336,
                       norm_eps=1e-5, max_seq_len=8192, rope_theta=500000.0, dtype=dtype)


@dataclass
class LayerWeights:
    attention_norm: torch.Tensor
    wqkv: torch.Tensor    # [dim, (n_heads + 2 n_kv_heads) * head_dim]: wq | wk | wv columns
    wo: torch.Tensor
    ffn_norm: torch.Tensor
    w13: torch.Tensor     # [dim, 2*hidden]: gate (w1) columns then up (w3) columns
    w2: torch.Tensor


class KVCache:
    """Per-layer K and V pools ``[num_blocks, block_size, n_kv_heads, head_dim]``,
    zero-initialised (core/kv_cache.py:13-32), as device tensors."""

    def __init__(self, num_layers: int, num_blocks: int, block_size: int, n_kv_heads: int, head_dim: int,
                 dtype: torch.dtype, device="cuda"):
        self.num_layers = num_layers
        self.num_blocks = num_blocks
        self.block_size = block_size
        self.n_kv_heads = n_kv_heads
        self.head_dim = head_dim
        self.dtype = dtype
        shape = (num_blocks, block_size, n_kv_heads, head_dim)
        self.k_cache = [torch.zeros(shape, dtype=dtype, device=device) for _ in range(num_layers)]
        self.v_cache = [torch.zeros(shape, dtype=dtype, device=device) for _ in range(num_layers)]

    def write_kv(self, layer_idx: int, block_id: int, start_offset: int, k: torch.Tensor, v: torch.Tensor) -> None:
        """KVCache.write_kv (kv_cache.py:34-38): rows [n, Hkv, D] at ``block_id`` from ``start_offset``."""
        n = k.shape[0]
        slots = torch.arange(block_id * self.block_size + start_offset,
                             block_id * self.block_size + start_offset + n, dtype=torch.int64, device=k.device)
        layers.write_kv_slots(k.contiguous(), v.contiguous(), slots, self.k_cache[layer_idx], self.v_cache[layer_idx])

    def read_kv_blocks(self, layer_idx: int, block_ids: List[int], context_len: int):
        """kv_cache.py:40-55 (test helper): [context_len, Hkv, D] gathered from ``block_ids``."""
        if not block_ids:
            z = torch.zeros(0, self.n_kv_heads, self.head_dim, dtype=self.dtype, device=self.k_cache[0].device)
            return z, z.clone()
        idx = torch.tensor(block_ids, dtype=torch.int64, device=self.k_cache[0].device)
        k = self.k_cache[layer_idx][idx].reshape(-1, self.n_kv_heads, self.head_dim)
        v = self.v_cache[layer_idx][idx].reshape(-1, self.n_kv_heads, self.head_dim)
        return k[:context_len], v[:context_len]

    def get_memory_bytes(self) -> int:
        return (self.num_layers * self.num_blocks * self.block_size * self.n_kv_heads * self.head_dim * 2
                * torch.tensor([], dtype=self.dtype).element_size())


class Llama:
    def __init__(self, config: LlamaConfig, device="cuda", seed: int = 0, init_std: float = 0.02):
        self.config = config
        self.device = torch.device(device)
        c = config
        dt = c.torch_dtype
        g = torch.Generator(device=self.device).manual_seed(seed)

        def rnd(*shape):
            return (torch.randn(*shape, generator=g, device=self.device, dtype=torch.float32) * init_std).to(dt)

        D = c.head_dim
        self.tok_embeddings = rnd(c.vocab_size, c.dim)
        self.layers: List[LayerWeights] = []
        for _ in range(c.n_layers):
            self.layers.append(LayerWeights(
                attention_norm=torch.ones(c.dim, dtype=dt, device=self.device),
                wqkv=rnd(c.dim, (c.n_heads + 2 * c.n_kv_heads) * D),
                wo=rnd(c.n_heads * D, c.dim),
                ffn_norm=torch.ones(c.dim, dtype=dt, device=self.device),
                w13=rnd(c.dim, 2 * c.hidden_dim), w2=rnd(c.hidden_dim, c.dim)))
        self.norm = torch.ones(c.dim, dtype=dt, device=self.device)
        self.output = rnd(c.dim, c.vocab_size)
        # precompute_freqs_cis(head_dim, 2 * max_seq_len) as the reference does (llama.py:263-264)
        self.cos, self.sin = layers.precompute_freqs_cis(D, 2 * c.max_seq_len, c.rope_theta, self.device)

    def numpy_weights(self) -> Dict[str, np.ndarray]:
        """All weights as float32 numpy arrays (for the CPU oracle)."""
        f = lambda t: t.float().cpu().numpy()
        w = {"tok_embeddings": f(self.tok_embeddings), "norm": f(self.norm), "output": f(self.output)}
        c = self.config
        H = c.hidden_dim
        nq, nk = c.n_heads * c.head_dim, c.n_kv_heads * c.head_dim
        for i, L in enumerate(self.layers):
            w13 = f(L.w13)
            wqkv = f(L.wqkv)
            w.update({f"l{i}.attention_norm": f(L.attention_norm), f"l{i}.wq": wqkv[:, :nq],
                      f"l{i}.wk": wqkv[:, nq:nq + nk], f"l{i}.wv": wqkv[:, nq + nk:], f"l{i}.wo": f(L.wo),
                      f"l{i}.ffn_norm": f(L.ffn_norm), f"l{i}.w1": w13[:, :H], f"l{i}.w3": w13[:, H:],
                      f"l{i}.w2": f(L.w2)})
        return w

    # ------------------------------------------------------------------ blocks
    def _layer_ffn(self, L: LayerWeights, h: torch.Tensor, attn: torch.Tensor, next_norm: torch.Tensor,
                   T: int, write_kv=None) -> torch.Tensor:
        """O-projection, residual + ffn_norm, SwiGLU FFN, residual + next norm.  ``write_kv``
        (k, v, slots, k_cache, v_cache) rides on the first norm's launch."""
        c = self.config
        o = torch.matmul(attn.view(T, c.n_heads * c.head_dim), L.wo)
        x = layers.rms_norm(o, L.ffn_norm, c.norm_eps, residual=h, write_kv=write_kv)  # h += o; x = ffn_norm(h)
        gu = torch.matmul(x, L.w13)
        a = layers.silu_mul(gu[:, :c.hidden_dim], gu[:, c.hidden_dim:])
        f = torch.matmul(a, L.w2)
        return layers.rms_norm(f, next_norm, c.norm_eps, residual=h)     # h += f; x = next_norm(h)

    def _qkv(self, L: LayerWeights, x: torch.Tensor, positions: torch.Tensor, slots=None, kv_cache=None, i=0):
        """One GEMM against wq|wk|wv, then RoPE'd q, k and v split out by one kernel
        (with ``slots`` the roped k and v are also stored to layer ``i``'s pool)."""
        c = self.config
        qkv = torch.matmul(x, L.wqkv)
        kc = kv_cache.k_cache[i] if slots is not None else None
        vc = kv_cache.v_cache[i] if slots is not None else None
        return layers.qkv_rope(qkv, c.n_heads, c.n_kv_heads, c.head_dim, self.cos, self.sin, positions,
                               slots=slots, k_cache=kc, v_cache=vc)

    # ---------------------------------------------------------------- prefill
    def prefill(self, tokens: torch.Tensor, positions: torch.Tensor, cu_seqlens: torch.Tensor, max_seqlen: int,
                slot_mapping: torch.Tensor, kv_cache: KVCache, n_out: Optional[int] = None) -> torch.Tensor:
        """Ragged prefill of several prompts packed along tokens.

        tokens/positions int32 [T]; cu_seqlens int32 [n+1]; slot_mapping int64 [T].
        Writes every layer's post-RoPE K and raw V into ``kv_cache`` at the slots
        (fused into the attention kernel) and returns the last-position logits
        [n, vocab] (of the first ``n_out`` prompts only, when given).
        """
        c = self.config
        T = tokens.shape[0]
        h = layers.embedding(self.tok_embeddings, tokens)
        x = layers.rms_norm(h, self.layers[0].attention_norm, c.norm_eps)
        for i, L in enumerate(self.layers):
            q, k, v = self._qkv(L, x, positions)
            attn = flash_prefill_attention_varlen(q, k, v, cu_seqlens, max_seqlen, True, slot_mapping=slot_mapping,
                                                  k_cache=kv_cache.k_cache[i], v_cache=kv_cache.v_cache[i])
            nxt = self.layers[i + 1].attention_norm if i + 1 < c.n_layers else self.norm
            x = self._layer_ffn(L, h, attn, nxt, T)
        last = (cu_seqlens[1:] if n_out is None else cu_seqlens[1:n_out + 1]) - 1
        return torch.matmul(x[last.long()], self.output)

    def capture_prefill(self, n_prompts: int, padded_tokens: int, kv_cache: "KVCache",
                        pool=None, stream: Optional[torch.cuda.Stream] = None) -> "PrefillGraph":
        """A CUDA graph of one ragged prefill of ``n_prompts`` prompts totalling fewer
        than ``padded_tokens`` tokens, plus the greedy pick of each prompt's first token."""
        return PrefillGraph(self, n_prompts, padded_tokens, kv_cache, pool, stream)

    def capture_decode(self, batch: int, table_width: int, kv_cache: "KVCache",
                       kv_order: str = "reference") -> "DecodeGraph":
        """A CUDA graph of one decode step (plus the greedy pick) for ``batch`` rows --
        the counterpart of the reference's per-batch-size TinyJit (engine.py:157-159)."""
        return DecodeGraph(self, batch, table_width, kv_cache, kv_order)

    # ----------------------------------------------------------------- decode
    def decode(self, tokens: torch.Tensor, positions: torch.Tensor, block_tables: torch.Tensor,
               context_lens: torch.Tensor, slots: torch.Tensor, kv_cache: KVCache,
               kv_order: str = "reference") -> torch.Tensor:
        """One decode step for B sequences (llama.py:298-388).

        tokens/positions int32 [B]; block_tables int32 [B, W]; context_lens int32 [B]
        (= position + 1); slots int64 [B] (the slot of each new token).  Returns
        logits [B, vocab].
        """
        c = self.config
        B = tokens.shape[0]
        h = layers.embedding(self.tok_embeddings, tokens)
        x = layers.rms_norm(h, self.layers[0].attention_norm, c.norm_eps)
        for i, L in enumerate(self.layers):
            kc, vc = kv_cache.k_cache[i], kv_cache.v_cache[i]
            if kv_order == "append_first":
                q, k, v = self._qkv(L, x, positions, slots, kv_cache, i)
            else:
                q, k, v = self._qkv(L, x, positions)
            attn = paged_decode_attention(q.view(B, 1, c.n_heads, c.head_dim), kc, vc, block_tables, context_lens,
                                          c.n_heads, c.n_kv_heads, c.head_dim, kv_cache.block_size)
            # reference order: the new token's K/V reaches the pool after the attention
            # (llama.py:381-386), stored by the launch of the norm that follows wo
            late_kv = (k, v, slots, kc, vc) if kv_order != "append_first" else None
            nxt = self.layers[i + 1].attention_norm if i + 1 < c.n_layers else self.norm
            x = self._layer_ffn(L, h, attn, nxt, B, write_kv=late_kv)
        return torch.matmul(x, self.output)


class DecodeGraph:
    """One decode step of ``Llama.decode`` followed by the greedy argmax, captured as a
    CUDA graph over static input buffers.  ``run`` copies a step's inputs from host
    arrays into the buffers, replays the graph and returns the sampled tokens.

    Rows beyond the live batch are padding: token 0, context 1 over block 0,
    slot -1 (no K/V write), and their outputs are ignored.

    The graph also copies the decode workspace's status word out with the
    tokens; ``run`` raises ``TvkError`` if a bounded wait inside an attention
    kernel of the step timed out.
    """

    def __init__(self, model: Llama, batch: int, table_width: int, kv_cache: KVCache, kv_order: str):
        dev = model.device
        self.model, self.batch, self.width, self.kv_cache, self.kv_order = model, batch, table_width, kv_cache, kv_order
        self.tok = torch.zeros(batch, dtype=torch.int32, device=dev)
        self.pos = torch.zeros(batch, dtype=torch.int32, device=dev)
        self.bt = torch.zeros(batch, table_width, dtype=torch.int32, device=dev)
        self.ctx = torch.ones(batch, dtype=torch.int32, device=dev)
        self.slots = torch.full((batch,), -1, dtype=torch.int64, device=dev)
        self.out = torch.zeros(batch + 1, dtype=torch.int32, device=dev)   # tokens, then the status word
        # pinned staging for the per-step host -> device copies
        self.h_tok = torch.zeros(batch, dtype=torch.int32).pin_memory()
        self.h_pos = torch.zeros(batch, dtype=torch.int32).pin_memory()
        self.h_bt = torch.zeros(batch, table_width, dtype=torch.int32).pin_memory()
        self.h_ctx = torch.ones(batch, dtype=torch.int32).pin_memory()
        self.h_slots = torch.full((batch,), -1, dtype=torch.int64).pin_memory()
        self.h_out = torch.zeros(batch + 1, dtype=torch.int32).pin_memory()
        self.stream = torch.cuda.Stream(dev)
        self.stream.wait_stream(torch.cuda.current_stream(dev))
        with torch.cuda.stream(self.stream):
            for _ in range(2):   # warm-up: workspaces, kernel attributes, cuBLAS handles
                self._forward()
        self.stream.synchronize()
        self.graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(self.graph, stream=self.stream):
            self._forward()
        self.stream.synchronize()

    def _forward(self):
        logits = self.model.decode(self.tok, self.pos, self.bt, self.ctx, self.slots, self.kv_cache, self.kv_order)
        layers.greedy_argmax(logits, out=self.out[:self.batch])
        # the attention calls of this step used this stream's workspace; the view
        # also keeps that workspace alive for as long as the graph exists
        self._status = status_word(self.model.device, "decode")
        self.out[self.batch:].copy_(self._status)

    def run(self, tokens: np.ndarray, positions: np.ndarray, tables: np.ndarray, ctx: np.ndarray,
            slots: np.ndarray) -> np.ndarray:
        n = tokens.shape[0]
        if n > self.batch or tables.shape[1] > self.width:
            raise ValueError("step larger than the captured graph")
        ht, hp, hb, hc, hs = (x.numpy() for x in (self.h_tok, self.h_pos, self.h_bt, self.h_ctx, self.h_slots))
        ht[:n], hp[:n], hc[:n], hs[:n] = tokens, positions, ctx, slots
        ht[n:], hp[n:], hc[n:], hs[n:] = 0, 0, 1, -1
        hb[:] = 0
        hb[:n, :tables.shape[1]] = tables
        cur = torch.cuda.current_stream(self.model.device)
        self.stream.wait_stream(cur)
        with torch.cuda.stream(self.stream):
            self.tok.copy_(self.h_tok, non_blocking=True)
            self.pos.copy_(self.h_pos, non_blocking=True)
            self.bt.copy_(self.h_bt, non_blocking=True)
            self.ctx.copy_(self.h_ctx, non_blocking=True)
            self.slots.copy_(self.h_slots, non_blocking=True)
            self.graph.replay()
            self.h_out.copy_(self.out, non_blocking=True)
        self.stream.synchronize()
        cur.wait_stream(self.stream)
        if int(self.h_out[self.batch]) != 0:
            with torch.cuda.stream(self.stream):
                self._status.zero_()
            self.stream.synchronize()
            raise _lib.TvkError("decode step: a bounded wait inside an attention kernel timed out; "
                                "the step's tokens are not valid")
        return self.h_out.numpy()[:n].copy()


def prefill_staging_layout(n: int, T: int):
    """Word offsets of a prefill graph's packed int32 input buffer: tokens [T] at 0,
    positions [T] at T, cu_seqlens [n + 2] at the first returned offset (padded to
    an even count), the slots as int64 [T] at the second; the third value is the
    buffer's length in int32 words."""
    off_cu = 2 * T
    off_slots = off_cu + ((n + 2 + 1) // 2) * 2
    return off_cu, off_slots, off_slots + 2 * T


def stage_prefill_inputs(h: np.ndarray, n: int, T: int, tokens, positions, lens, slots) -> None:
    """Fill the packed buffer ``h`` (int32, ``prefill_staging_layout(n, T)``): the
    prompts of ``lens`` (tokens, positions and slots concatenated) at the front,
    then one padding prompt of token 0, position 0 and slot -1 up to T tokens, so
    cu_seqlens = [0, prefix sums of lens..., T].  ``lens=None`` stages the
    capture-time contents: n one-token prompts of token 0 that store nothing."""
    off_cu, off_slots, _ = prefill_staging_layout(n, T)
    t_real = 0 if lens is None else int(sum(lens))
    h[:t_real], h[t_real:T] = tokens, 0
    h[T:T + t_real], h[T + t_real:2 * T] = positions, 0
    cu = h[off_cu:off_cu + n + 2]
    cu[0] = 0
    cu[1:n + 1] = np.arange(1, n + 1) if lens is None else np.cumsum(lens)
    cu[n + 1] = T
    hs = h[off_slots:off_slots + 2 * T].view(np.int64)
    hs[:t_real], hs[t_real:] = slots, -1


class PrefillGraph:
    """``Llama.prefill`` of ``n`` prompts followed by the greedy argmax, captured as a
    CUDA graph over static buffers of ``T`` tokens.  The prompts fill the first
    tokens; the rest of the buffer is one more (padding) prompt with token 0,
    position 0 and slot -1, whose K/V is never stored and whose rows are
    dropped, so every row the graph computes is finite and the real prompts see
    the same kernels as an eager call (the projections run as GEMMs over ``T``
    rows instead of the live count).  ``run`` copies a step's inputs from pinned
    host memory into the buffers in one copy, replays the graph and returns the
    sampled tokens; like ``DecodeGraph`` it raises ``TvkError`` if a bounded wait
    inside an attention kernel of the step timed out.

    An eager prefill step issues about ten launches per layer from Python, so
    its length follows the host's speed; the graph issues one.
    """

    def __init__(self, model: Llama, n: int, T: int, kv_cache: KVCache, pool=None,
                 stream: Optional[torch.cuda.Stream] = None):
        if n < 1 or T < n + 1:
            raise ValueError("a prefill graph needs n >= 1 prompts and T > n tokens")
        dev = model.device
        self.model, self.n, self.T, self.kv_cache = model, n, T, kv_cache
        self._off_cu, self._off_slots, words = prefill_staging_layout(n, T)
        self.h_in = torch.zeros(words, dtype=torch.int32).pin_memory()
        self.d_in = torch.zeros(words, dtype=torch.int32, device=dev)
        self.tok = self.d_in[:T]
        self.pos = self.d_in[T:2 * T]
        self.cu = self.d_in[self._off_cu:self._off_cu + n + 2]
        self.slots = self.d_in[self._off_slots:].view(torch.int64)
        self.out = torch.zeros(n + 1, dtype=torch.int32, device=dev)   # tokens, then the status word
        self.h_out = torch.zeros(n + 1, dtype=torch.int32).pin_memory()
        self._stage(np.zeros(0, np.int32), np.zeros(0, np.int32), None, np.zeros(0, np.int64))
        self.d_in.copy_(self.h_in)
        self.stream = stream or torch.cuda.Stream(dev)
        self.stream.wait_stream(torch.cuda.current_stream(dev))
        with torch.cuda.stream(self.stream):
            for _ in range(2):   # warm-up: workspaces, kernel attributes, cuBLAS handles
                self._forward()
        self.stream.synchronize()
        self.graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(self.graph, pool=pool, stream=self.stream):
            self._forward()
        self.stream.synchronize()

    def _forward(self):
        m = self.model
        logits = m.prefill(self.tok, self.pos, self.cu, self.T, self.slots, self.kv_cache, n_out=self.n)
        layers.greedy_argmax(logits, out=self.out[:self.n])
        # the attention calls used this stream's prefill workspace; the view keeps it
        # alive for as long as the graph exists
        self._status = status_word(m.device, "prefill")
        self.out[self.n:].copy_(self._status)

    def _stage(self, tokens, positions, lens, slots):
        stage_prefill_inputs(self.h_in.numpy(), self.n, self.T, tokens, positions, lens, slots)

    def run(self, tokens: np.ndarray, positions: np.ndarray, lens: List[int], slots: np.ndarray) -> np.ndarray:
        if len(lens) != self.n or int(sum(lens)) >= self.T or min(lens) < 1:
            raise ValueError("prompts do not fit the captured prefill graph")
        self._stage(tokens, positions, lens, slots)
        cur = torch.cuda.current_stream(self.model.device)
        self.stream.wait_stream(cur)
        with torch.cuda.stream(self.stream):
            self.d_in.copy_(self.h_in, non_blocking=True)
            self.graph.replay()
            self.h_out.copy_(self.out, non_blocking=True)
        self.stream.synchronize()
        cur.wait_stream(self.stream)
        if int(self.h_out[self.n]) != 0:
            with torch.cuda.stream(self.stream):
                self._status.zero_()
            self.stream.synchronize()
            raise _lib.TvkError("prefill step: a bounded wait inside an attention kernel timed out; "
                                "the step's tokens are not valid")
        return self.h_out.numpy()[:self.n].copy()
