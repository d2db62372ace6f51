"""CPU oracle: numpy restatement of the reference model and engine step order.

TEST INFRASTRUCTURE ONLY (see ``oracle/attention.py``).  Used to check greedy
token streams of the product engine bit-for-bit on small models.

Follows, statement by statement where it matters for the token stream:
* ``Llama.prefill`` (tinyvllm/model/llama.py:266-288) -- one prompt per call,
  K/V written chunk by chunk with layer 0 allocating blocks (llama.py:188-209),
  ``flash_prefill_attention`` over the prompt itself;
* ``Llama.decode`` (llama.py:346-388) -- block tables padded / truncated to
  ``max_blocks`` with block 0, ``context_lens = start_pos + 1`` (engine.py:251),
  attention over the cache *before* the step's K/V is written, then per
  sequence ``get_slot`` -> ``write_kv`` for every layer -> ``advance_position``;
* ``LLMEngine.step`` (core/engine.py:114-196) and ``Scheduler``
  (core/scheduler.py:32-64) -- FCFS admission, prefill then decode, blocks
  freed after the step;
* greedy pick = argmax, first index (core/sampling.py:133-134).

Weights come from the product model in float32 numpy form (``x @ W`` with W
stored [in, out]); all arithmetic is float32.
"""

from __future__ import annotations

from typing import Dict, List

import numpy as np

from . import attention as oa
from . import paging as op


def _top2_gap(logits: np.ndarray) -> float:
    top = np.sort(np.asarray(logits, dtype=np.float64))[-2:]
    return float(top[1] - top[0])


class OracleLlama:
    def __init__(self, weights: Dict[str, np.ndarray], n_layers: int, n_heads: int, n_kv_heads: int,
                 head_dim: int, norm_eps: float, rope_theta: float, max_seq_len: int):
        self.w = weights
        self.n_layers, self.n_heads, self.n_kv_heads, self.head_dim = n_layers, n_heads, n_kv_heads, head_dim
        self.eps = norm_eps
        self.cos, self.sin = oa.precompute_freqs_cis(head_dim, 2 * max_seq_len, rope_theta)

    def _ffn(self, i, h):
        x = oa.rms_norm(h, self.w[f"l{i}.ffn_norm"], self.eps)
        return oa.silu_mul(x @ self.w[f"l{i}.w1"], x @ self.w[f"l{i}.w3"]) @ self.w[f"l{i}.w2"]

    def prefill(self, tokens: List[int], cache: op.OracleKVCache, bm: op.OracleBlockManager, seq_id: int):
        """llama.py:266-288 with batch 1 and start_pos 0; returns last-position logits."""
        L = len(tokens)
        H, Hk, D = self.n_heads, self.n_kv_heads, self.head_dim
        h = self.w["tok_embeddings"][np.asarray(tokens)]               # [L, dim]
        cos, sin = self.cos[:L], self.sin[:L]
        for i in range(self.n_layers):
            x = oa.rms_norm(h, self.w[f"l{i}.attention_norm"], self.eps)
            q = (x @ self.w[f"l{i}.wq"]).reshape(1, L, H, D)
            k = (x @ self.w[f"l{i}.wk"]).reshape(1, L, Hk, D)
            v = (x @ self.w[f"l{i}.wv"]).reshape(1, L, Hk, D)
            q = oa.apply_rope(q, cos, sin)
            k = oa.apply_rope(k, cos, sin)
            op.write_prompt_kv(cache, bm, i, seq_id, k[0], v[0], 0)
            attn = oa.flash_prefill_attention(q, k, v, True)[0]         # [L, H, D]
            h = h + attn.reshape(L, H * D) @ self.w[f"l{i}.wo"]
            h = h + self._ffn(i, h)
        for _ in range(L):
            bm.advance_position(seq_id)
        x = oa.rms_norm(h[-1:], self.w["norm"], self.eps)
        return (x @ self.w["output"])[0]

    def decode(self, tokens: List[int], start_positions: List[int], seq_ids: List[int], cache: op.OracleKVCache,
               bm: op.OracleBlockManager, max_blocks: int = 64):
        """llama.py:346-388 (and the JIT body :298-342); returns logits [B, vocab]."""
        B = len(tokens)
        H, Hk, D = self.n_heads, self.n_kv_heads, self.head_dim
        bt, ctx = op.prepare_batch_tables(bm, seq_ids, start_positions, max_blocks)
        cos = self.cos[np.asarray(start_positions)][:, None]           # [B, 1, D/2]
        sin = self.sin[np.asarray(start_positions)][:, None]
        h = self.w["tok_embeddings"][np.asarray(tokens)]               # [B, dim]
        k_all, v_all = [], []
        for i in range(self.n_layers):
            x = oa.rms_norm(h, self.w[f"l{i}.attention_norm"], self.eps)
            q = (x @ self.w[f"l{i}.wq"]).reshape(B, 1, H, D)
            k = (x @ self.w[f"l{i}.wk"]).reshape(B, 1, Hk, D)
            v = (x @ self.w[f"l{i}.wv"]).reshape(B, 1, Hk, D)
            q = oa.apply_rope(q, cos, sin)
            k = oa.apply_rope(k, cos, sin)
            k_all.append(k[:, 0])
            v_all.append(v[:, 0])
            attn = oa.paged_decode_attention(q, cache.k_cache[i], cache.v_cache[i], bt, ctx, H, Hk, D,
                                             bm.block_size)
            h = h + attn.reshape(B, H * D) @ self.w[f"l{i}.wo"]
            h = h + self._ffn(i, h)
        logits = oa.rms_norm(h, self.w["norm"], self.eps) @ self.w["output"]
        for b, sid in enumerate(seq_ids):                              # llama.py:381-386
            _, block_id, offset = bm.get_slot(sid)
            for i in range(self.n_layers):
                cache.write_kv(i, block_id, offset, k_all[i][b:b + 1], v_all[i][b:b + 1])
            bm.advance_position(sid)
        return logits


class OracleEngine:
    """LLMEngine.step / Scheduler (engine.py:114-196, scheduler.py:32-64), greedy only."""

    def __init__(self, model: OracleLlama, max_batch_size: int, num_blocks: int, block_size: int = 16,
                 num_scheduler_steps: int = 1, eos_id: int = -1, max_blocks: int = 64):
        self.model = model
        self.max_batch_size = max_batch_size
        self.bm = op.OracleBlockManager(1, num_blocks, block_size)
        self.cache = op.OracleKVCache(model.n_layers, num_blocks, block_size, model.n_kv_heads, model.head_dim)
        self.num_scheduler_steps = num_scheduler_steps
        self.eos_id = eos_id
        self.max_blocks = max_blocks
        self.waiting = []       # (request_id, prompt, max_tokens)
        self.running = {}       # seq_id -> dict
        self.next_seq_id = 0
        self.next_request_id = 0
        self.outputs = {}
        self.gaps = {}      # request -> top-1 minus top-2 logit of every picked token
        self.logits = {}    # request -> the logits each token was picked from

    def add_request(self, prompt: List[int], max_tokens: int) -> int:
        rid = self.next_request_id
        self.next_request_id += 1
        self.waiting.append((rid, list(prompt), max_tokens))
        return rid

    def has_unfinished(self) -> bool:
        return bool(self.waiting) or bool(self.running)

    def _finished(self, s) -> bool:
        return s["out"][-1] == self.eos_id or len(s["out"]) >= s["max_tokens"]

    def step(self) -> List[int]:
        batch = list(self.running.values())
        while len(batch) < self.max_batch_size and self.waiting:
            rid, prompt, mt = self.waiting.pop(0)
            self.bm.register_sequence(self.next_seq_id)
            s = {"seq_id": self.next_seq_id, "rid": rid, "prompt": prompt, "out": [], "max_tokens": mt, "gaps": [], "logits": []}
            self.running[self.next_seq_id] = s
            self.next_seq_id += 1
            batch.append(s)
        finished = []
        prefill = [s for s in batch if not s["out"]]
        decode = [s for s in batch if s["out"]]
        for s in prefill:
            logits = self.model.prefill(s["prompt"], self.cache, self.bm, s["seq_id"])
            s["out"].append(int(oa.greedy_argmax(logits[None])[0]))
            s["gaps"].append(_top2_gap(logits))
            s["logits"].append(np.asarray(logits, dtype=np.float32))
            if self._finished(s):
                finished.append(s["seq_id"])
        for _ in range(self.num_scheduler_steps):
            if not decode:
                break
            toks = [s["out"][-1] for s in decode]
            pos = [len(s["prompt"]) + len(s["out"]) - 1 for s in decode]
            logits = self.model.decode(toks, pos, [s["seq_id"] for s in decode], self.cache, self.bm,
                                       self.max_blocks)
            nxt = oa.greedy_argmax(logits)
            still = []
            for s, t, lg in zip(decode, nxt, logits):
                s["out"].append(int(t))
                s["gaps"].append(_top2_gap(lg))
                s["logits"].append(np.asarray(lg, dtype=np.float32))
                if self._finished(s):
                    finished.append(s["seq_id"])
                else:
                    still.append(s)
            decode = still
        for sid in finished:
            s = self.running.pop(sid)
            self.bm.free_sequence(sid)
            self.outputs[s["rid"]] = list(s["out"])
            self.gaps[s["rid"]] = list(s["gaps"])
            self.logits[s["rid"]] = list(s["logits"])
        return finished
