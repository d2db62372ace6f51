"""Continuous-batching engine over the sm_100a kernels.

Mirrors ``tinyvllm/core/engine.py``, ``core/scheduler.py`` and ``core/sequence.py``
for the hot path: FCFS admission up to ``max_batch_size`` (scheduler.py:32-54),
prefill of newly admitted sequences then ``num_scheduler_steps`` batched decode
iterations (engine.py:114-196), blocks freed when a sequence finishes
(scheduler.py:56-64).  Differences, all on the device side:

* newly admitted prompts are prefilled in one ragged kernel call per layer
  (the reference runs one prompt at a time, engine.py:125-132); block
  allocation still happens prompt by prompt in admission order, so the slots
  are the reference's;
* each decode step builds its block tables and context lengths in one numpy
  pass (engine.py:235-255) and writes all sequences' new K/V with one launch
  per layer (the reference issues batch x layers writes, llama.py:381-386);
* sampling is greedy only (temperature < 1e-5): an on-device argmax; the
  reference's random sampling paths (sampling.py) are not part of this build;
* with ``use_cuda_graphs`` a decode step replays a CUDA graph per padded batch
  size and a prefill step one per (prompt count, token count rounded up to
  128), the latter over a token buffer whose tail is a padding prompt that
  stores nothing; up to 64 prefill graphs are kept, further shapes run eagerly.

``kv_order="reference"`` (default) reproduces the reference decode exactly:
tables padded / truncated to 64 blocks (engine.py:81, llama.py:368-374),
attention over ``position + 1`` slots before the step's own K/V is written.
``kv_order="append_first"`` writes first and uses full-width tables.
"""

from __future__ import annotations

import time
from dataclasses import dataclass, field
from enum import Enum, auto
from typing import Any, Callable, Dict, Iterator, List, Optional

import numpy as np
import torch

from . import layers
from .attention import check_workspace
from .block_manager import BlockManager
from .model import KVCache, Llama

_SAMPLING_EPS = 1e-5
_GRAPH_BATCHES = (1, 2, 4, 8, 16, 24, 32, 48, 64, 96, 128, 192, 256, 384, 512)
# prefill graphs hold a whole number of these tokens (the live prompts plus at least one padding token)
_PREFILL_TOKEN_QUANTUM = 128
# prefill graphs an engine keeps; a step of another (prompt count, token count) shape runs eagerly
_MAX_PREFILL_GRAPHS = 64


@dataclass
class SamplingParams:
    """core/sampling.py:12-18.  Only greedy decoding (temperature < 1e-5) is run here."""
    temperature: float = 0.0
    top_k: int = 40
    top_p: float = 0.95
    repetition_penalty: float = 1.0
    max_tokens: int = 1024


class SequenceStatus(Enum):
    WAITING = auto()
    RUNNING = auto()
    FINISHED = auto()


@dataclass
class Sequence:
    seq_id: int
    request_id: int
    prompt_tokens: List[int]
    output_tokens: List[int] = field(default_factory=list)
    status: SequenceStatus = SequenceStatus.WAITING

    def get_all_tokens(self) -> List[int]:
        return self.prompt_tokens + self.output_tokens

    def get_len(self) -> int:
        return len(self.prompt_tokens) + len(self.output_tokens)

    def get_prompt_len(self) -> int:
        return len(self.prompt_tokens)

    def get_output_len(self) -> int:
        return len(self.output_tokens)

    def append_token(self, token_id: int) -> None:
        self.output_tokens.append(token_id)

    def is_finished(self) -> bool:
        return self.status == SequenceStatus.FINISHED


@dataclass
class Request:
    request_id: int
    prompt: Any
    prompt_tokens: List[int]
    sampling_params: SamplingParams
    arrival_time: float = field(default_factory=time.time)
    sequence: Optional[Sequence] = None
    prefilled_first_token: Optional[int] = None


@dataclass
class SchedulerOutput:
    scheduled_seqs: List[Sequence] = field(default_factory=list)


@dataclass
class GenerationOutput:
    request_id: int
    text: str
    tokens: List[int]
    finish_reason: str  # 'eos', 'length' or 'abort'


class Scheduler:
    """FCFS continuous batching (core/scheduler.py:10-88)."""

    def __init__(self, max_batch_size: int, block_manager: BlockManager, gpu_id: int = 0):
        self.max_batch_size = max_batch_size
        self.block_manager = block_manager
        self.gpu_id = gpu_id
        self.waiting: List[Request] = []
        self.running: Dict[int, Sequence] = {}
        self.next_seq_id = 0

    def add_request(self, request: Request) -> None:
        self.waiting.append(request)

    def has_unfinished(self) -> bool:
        return bool(self.waiting) or bool(self.running)

    def schedule(self) -> SchedulerOutput:
        batch = SchedulerOutput(scheduled_seqs=list(self.running.values()))
        while len(batch.scheduled_seqs) < self.max_batch_size and self.waiting:
            request = self.waiting.pop(0)
            self.block_manager.register_sequence(self.next_seq_id, self.gpu_id)
            seq = Sequence(self.next_seq_id, request.request_id, request.prompt_tokens,
                           status=SequenceStatus.RUNNING)
            request.sequence = seq
            self.next_seq_id += 1
            self.running[seq.seq_id] = seq
            batch.scheduled_seqs.append(seq)
        return batch

    def update(self, finished_seqs: List[int]) -> None:
        for seq_id in finished_seqs:
            seq = self.running.pop(seq_id, None)
            if seq is not None:
                seq.status = SequenceStatus.FINISHED
                self.block_manager.free_sequence(seq_id)

    def get_num_waiting(self) -> int:
        return len(self.waiting)

    def get_num_running(self) -> int:
        return len(self.running)

    def abort_request(self, request_id: int) -> bool:
        for i, req in enumerate(self.waiting):
            if req.request_id == request_id:
                self.waiting.pop(i)
                return True
        for seq_id, seq in list(self.running.items()):
            if seq.request_id == request_id:
                del self.running[seq_id]
                self.block_manager.free_sequence(seq_id)
                return True
        return False


class TokenIdTokenizer:
    """Pass-through tokenizer: prompts are lists of token ids; ``eos_id`` defaults to
    an id outside any vocabulary so generation runs to ``max_tokens``."""

    def __init__(self, eos_id: int = -1):
        self.eos_id = eos_id

    def encode(self, prompt) -> List[int]:
        return list(prompt)

    def decode(self, tokens: List[int]) -> str:
        return " ".join(map(str, tokens))


class LLMEngine:
    def __init__(self, model: Llama, tokenizer: Any = None, max_batch_size: int = 8, num_blocks: int = 1024,
                 block_size: int = 16, num_scheduler_steps: int = 1, kv_order: str = "reference",
                 max_table_blocks: Optional[int] = None, gpu_id: int = 0,
                 output_callback: Optional[Callable[[GenerationOutput], None]] = None,
                 use_cuda_graphs: bool = False):
        if kv_order not in ("reference", "append_first"):
            raise ValueError("kv_order must be 'reference' or 'append_first'")
        self.model = model
        self.tokenizer = tokenizer or TokenIdTokenizer()
        self.max_batch_size = max_batch_size
        self.block_size = block_size
        self.num_scheduler_steps = num_scheduler_steps
        self.kv_order = kv_order
        # the reference pads / truncates decode tables to 64 blocks (engine.py:81)
        self.table_width = max_table_blocks or (64 if kv_order == "reference" else None)
        cfg = model.config
        self.device = model.device
        self.block_manager = BlockManager(num_gpus=gpu_id + 1, blocks_per_gpu=num_blocks, block_size=block_size)
        self.gpu_id = gpu_id
        self.kv_cache = KVCache(cfg.n_layers, num_blocks, block_size, cfg.n_kv_heads, cfg.head_dim,
                                cfg.torch_dtype, self.device)
        self.scheduler = Scheduler(max_batch_size, self.block_manager, gpu_id)
        self.next_request_id = 0
        self.requests: Dict[int, Request] = {}
        self.output_callback = output_callback
        self._outputs: List[GenerationOutput] = []
        self.stats = {"prefill_tokens": 0, "decode_tokens": 0, "decode_steps": 0}
        # decode graphs, one per padded batch size (the reference keeps one TinyJit per batch size)
        self.use_cuda_graphs = use_cuda_graphs
        self._graphs = {}
        # prefill graphs, one per (prompt count, padded token count); they replay one at
        # a time on one stream, so they share one memory pool
        self._prefill_graphs = {}
        self._prefill_pool = None
        self._prefill_stream = None
        self._graph_width = self.table_width or -(-2 * cfg.max_seq_len // block_size)

    # ------------------------------------------------------------------ API
    def add_request(self, prompt, sampling_params: Optional[SamplingParams] = None,
                    request_id: Optional[int] = None) -> int:
        sp = sampling_params or SamplingParams()
        if sp.temperature >= _SAMPLING_EPS:
            raise ValueError("only greedy decoding (temperature < 1e-5) is supported by this engine")
        tokens = self.tokenizer.encode(prompt)
        if not tokens:
            raise ValueError("empty prompt")
        if request_id is None:
            request_id = self.next_request_id
            self.next_request_id += 1
        elif request_id in self.requests:
            raise ValueError(f"Request ID {request_id} already exists")
        elif request_id >= self.next_request_id:
            self.next_request_id = request_id + 1
        req = Request(request_id, prompt, tokens, sp)
        self.requests[request_id] = req
        self.scheduler.add_request(req)
        return request_id

    def add_prefilled_request(self, context_tokens, sampling_params: Optional[SamplingParams] = None,
                              first_token: int = 0, request_id: Optional[int] = None) -> int:
        """Admit a sequence whose K/V for ``context_tokens`` is already resident in the
        pool contents (e.g. synthetic K/V for a decode benchmark): on admission its
        blocks are allocated and its position advanced as a prefill would, no
        prefill is run, and ``first_token`` is taken as the prompt's sampled token."""
        rid = self.add_request(context_tokens, sampling_params, request_id)
        self.requests[rid].prefilled_first_token = int(first_token)
        return rid

    def has_unfinished(self) -> bool:
        return self.scheduler.has_unfinished()

    def abort_request(self, request_id: int) -> bool:
        return self.scheduler.abort_request(request_id)

    def run(self) -> Iterator[GenerationOutput]:
        while self.scheduler.has_unfinished():
            yield from self.step()

    # ----------------------------------------------------------------- step
    def step(self) -> List[GenerationOutput]:
        batch = self.scheduler.schedule()
        if not batch.scheduled_seqs:
            return []
        finished: List[int] = []
        prefill = [s for s in batch.scheduled_seqs if s.get_output_len() == 0]
        decode = [s for s in batch.scheduled_seqs if s.get_output_len() > 0]
        if prefill:
            first = self._prefill(prefill)
            for seq, tok in zip(prefill, first):
                seq.append_token(tok)
                if self._check_finished(seq):
                    finished.append(seq.seq_id)
        for _ in range(self.num_scheduler_steps):
            if not decode:
                break
            next_tokens = self._decode(decode)
            still = []
            for seq, tok in zip(decode, next_tokens):
                seq.append_token(tok)
                if self._check_finished(seq):
                    finished.append(seq.seq_id)
                else:
                    still.append(seq)
            decode = still
        self.scheduler.update(finished)
        outs = []
        for sid in finished:
            for rid, req in list(self.requests.items()):
                if req.sequence is not None and req.sequence.seq_id == sid:
                    out = GenerationOutput(rid, self.tokenizer.decode(req.sequence.output_tokens),
                                           list(req.sequence.output_tokens), self._reason(req.sequence))
                    outs.append(out)
                    if self.output_callback:
                        self.output_callback(out)
                    del self.requests[rid]
                    break
        return outs

    def _reason(self, seq: Sequence) -> str:
        return "eos" if seq.output_tokens[-1] == self.tokenizer.eos_id else "length"

    def _check_finished(self, seq: Sequence) -> bool:
        req = self.requests[seq.request_id]
        return seq.output_tokens[-1] == self.tokenizer.eos_id or seq.get_output_len() >= req.sampling_params.max_tokens

    # --------------------------------------------------------------- device
    def _prefill(self, seqs: List[Sequence]) -> List[int]:
        bm = self.block_manager
        first = {}
        live = []
        for s in seqs:
            tok = self.requests[s.request_id].prefilled_first_token
            if tok is None:
                live.append(s)
            else:                      # K/V already resident: allocate and advance only
                bm.slot_mapping(s.seq_id, 0, s.get_prompt_len())
                bm.advance_position(s.seq_id, s.get_prompt_len())
                first[s.seq_id] = tok
        if live:
            for s, t in zip(live, self._prefill_live(live)):
                first[s.seq_id] = t
        return [first[s.seq_id] for s in seqs]

    def _prefill_live(self, seqs: List[Sequence]) -> List[int]:
        bm = self.block_manager
        lens = [s.get_prompt_len() for s in seqs]
        slots = np.concatenate([bm.slot_mapping(s.seq_id, 0, L) for s, L in zip(seqs, lens)])
        toks = np.concatenate([np.asarray(s.prompt_tokens, dtype=np.int32) for s in seqs])
        pos = np.concatenate([np.arange(L, dtype=np.int32) for L in lens])
        cu = np.concatenate([[0], np.cumsum(lens)]).astype(np.int32)
        dev = self.device
        n, t_pad = len(seqs), -(-(int(cu[-1]) + 1) // _PREFILL_TOKEN_QUANTUM) * _PREFILL_TOKEN_QUANTUM
        graph = self._prefill_graphs.get((n, t_pad)) if self.use_cuda_graphs else None
        if self.use_cuda_graphs and (graph is not None or len(self._prefill_graphs) < _MAX_PREFILL_GRAPHS):
            if graph is None:
                if self._prefill_pool is None:
                    self._prefill_pool = torch.cuda.graph_pool_handle()
                    self._prefill_stream = torch.cuda.Stream(dev)
                graph = self.model.capture_prefill(n, t_pad, self.kv_cache, self._prefill_pool, self._prefill_stream)
                self._prefill_graphs[(n, t_pad)] = graph
            sampled = graph.run(toks, pos, lens, slots).tolist()   # raises if a kernel wait timed out
        else:
            logits = self.model.prefill(torch.from_numpy(toks).to(dev), torch.from_numpy(pos).to(dev),
                                        torch.from_numpy(cu).to(dev), max(lens), torch.from_numpy(slots).to(dev),
                                        self.kv_cache)
            sampled = self._sample(logits, seqs)
            check_workspace(dev, "prefill", "prefill step")     # a kernel wait that timed out raises here
        for s, L in zip(seqs, lens):
            bm.advance_position(s.seq_id, L)
        self.stats["prefill_tokens"] += int(sum(lens))
        return sampled

    def _decode(self, seqs: List[Sequence]) -> List[int]:
        bm = self.block_manager
        ids = [s.seq_id for s in seqs]
        pos = np.asarray([s.get_len() - 1 for s in seqs], dtype=np.int32)
        ctx = pos + 1

        def new_slots():
            out = np.empty(len(ids), dtype=np.int64)
            for j, i in enumerate(ids):
                _, blk, off = bm.get_slot(i)           # allocates a block when the position needs one
                out[j] = blk * self.block_size + off
            return out

        if self.kv_order == "reference":
            # tables are built before the new slot is allocated (engine.py:247, llama.py:383)
            bt = bm.block_table_array(ids, self.table_width)
            slots = new_slots()
        else:
            slots = new_slots()
            bt = bm.block_table_array(ids, self.table_width)
        if self.use_cuda_graphs:
            B = len(seqs)
            cap = next((b for b in _GRAPH_BATCHES if b >= B), -(-B // 64) * 64)
            graph = self._graphs.get(cap)
            if graph is None:
                graph = self.model.capture_decode(cap, self._graph_width, self.kv_cache, self.kv_order)
                self._graphs[cap] = graph
            toks = np.asarray([s.output_tokens[-1] for s in seqs], dtype=np.int32)
            sampled = graph.run(toks, pos, bt, ctx, slots).tolist()
        else:
            dev = self.device
            tok = torch.tensor([s.output_tokens[-1] for s in seqs], dtype=torch.int32, device=dev)
            logits = self.model.decode(tok, torch.from_numpy(pos).to(dev), torch.from_numpy(bt).to(dev),
                                       torch.from_numpy(ctx).to(dev), torch.from_numpy(slots).to(dev),
                                       self.kv_cache, self.kv_order)
            sampled = None
        if sampled is None:
            sampled = self._sample(logits, seqs)
            check_workspace(self.device, "decode", "decode step")
        for i in ids:
            bm.advance_position(i)
        self.stats["decode_tokens"] += len(seqs)
        self.stats["decode_steps"] += 1
        return sampled

    def _sample(self, logits: torch.Tensor, seqs: List[Sequence]) -> List[int]:
        """Greedy pick for each row of ``logits`` [len(seqs), vocab] (sampling.py:133-134)."""
        return layers.greedy_argmax(logits).cpu().tolist()


def generate_batch(engine: LLMEngine, prompts: List, sampling_params: Optional[SamplingParams] = None) -> List[str]:
    """core/engine.py:258-266: completions in input order."""
    ids = [engine.add_request(p, sampling_params) for p in prompts]
    results = {o.request_id: o.text for o in engine.run()}
    return [results[i] for i in ids]
