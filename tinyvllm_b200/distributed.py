"""Sequence-sharded decoding across the GPUs of one node.

One process per GPU.  Every rank holds the full weights and its own KV pool;
requests are assigned to ranks as they arrive and never move.  The only data
exchanged is, once per engine step, an all-gather of the int32 tokens each rank
sampled (over NCCL on GPUs, or gloo for CPU tests), so that every rank ends the
step knowing every stream.  The reference models this partitioning in
``BlockManager(num_gpus, blocks_per_gpu)`` / ``seq_to_gpu``
(tinyvllm/core/block_manager.py:9-26) but runs one GPU.

Assignment is deterministic and identical on every rank (all ranks see the same
``add_request`` calls): a new request goes to the rank with the least
outstanding work, measured as prompt tokens + tokens still to generate, ties to
the lowest rank -- greedy longest-processing-time balancing of the decode load.

Failure handling: a rank whose local step raises still joins the step's
collective with an error flag, so every rank raises ``ShardError`` at the same
step instead of hanging; a rank that dies outright is detected by the process
group timeout of the next collective.
"""

from __future__ import annotations

import time
from dataclasses import dataclass, field
from typing import Any, Dict, List, Optional

import numpy as np
import torch
import torch.distributed as dist

# per-step record layout (int32): [status, has_unfinished, n, (request_id, token, finished) * capacity]
_HDR = 3
_OK, _ERROR = 0, 1


class ShardError(RuntimeError):
    """A rank failed during a step; raised on every rank at the same step."""


@dataclass
class _Req:
    request_id: int
    rank: int
    prompt_len: int
    max_tokens: int
    tokens: List[int] = field(default_factory=list)
    finished: bool = False


class ShardedEngine:
    """Drives one local engine per rank and merges the token streams.

    ``engine`` needs ``add_request(prompt, params, request_id=...)``, ``step()``
    returning finished outputs, ``has_unfinished()``, ``max_batch_size`` and
    ``num_scheduler_steps``; the new tokens of a step are read from the
    engine's request table (``engine.requests[rid].sequence.output_tokens``)
    and its finished outputs.
    """

    def __init__(self, engine: Any, rank: int, world_size: int, device: torch.device,
                 group: Optional[dist.ProcessGroup] = None):
        self.engine = engine
        self.rank = rank
        self.world = world_size
        self.device = device
        self.group = group
        self.requests: Dict[int, _Req] = {}
        self.next_request_id = 0
        self.load = [0] * world_size
        # tokens one rank can emit in one step: a prefill token per admitted sequence
        # plus one per decode iteration per running sequence.  The all-gather needs
        # one record size on every rank, and ranks may run engines of different
        # batch sizes (each sizes its batch to its own memory), so take the largest.
        cap = engine.max_batch_size * (engine.num_scheduler_steps + 1)
        if world_size > 1 and dist.is_available() and dist.is_initialized():
            t = torch.tensor([cap], dtype=torch.int64, device=device)
            dist.all_reduce(t, op=dist.ReduceOp.MAX, group=group)
            cap = int(t.item())
        self.capacity = cap
        self.steps = 0
        self.exchange_seconds = 0.0   # host wall time spent in the per-step token exchange

    # ------------------------------------------------------------------ API
    def add_request(self, prompt, sampling_params, prefilled_first_token: Optional[int] = None) -> int:
        """Assign a request to a rank (least outstanding work) and hand it to that rank's
        engine; with ``prefilled_first_token`` the owner admits it as already prefilled."""
        rid = self.next_request_id
        self.next_request_id += 1
        n_prompt = len(prompt)
        work = n_prompt + sampling_params.max_tokens
        rank = min(range(self.world), key=lambda r: (self.load[r], r))
        self.load[rank] += work
        self.requests[rid] = _Req(rid, rank, n_prompt, sampling_params.max_tokens)
        if rank == self.rank:
            if prefilled_first_token is None:
                self.engine.add_request(prompt, sampling_params, request_id=rid)
            else:
                self.engine.add_prefilled_request(prompt, sampling_params, prefilled_first_token, request_id=rid)
        return rid

    def owner(self, request_id: int) -> int:
        return self.requests[request_id].rank

    def has_unfinished(self) -> bool:
        return any(not r.finished for r in self.requests.values())

    def step(self) -> List[int]:
        """One engine step on every rank plus the token all-gather.  Returns the ids
        of requests that finished (on any rank) during this step."""
        rec = np.full(_HDR + 3 * self.capacity, -1, dtype=np.int32)
        rec[0] = _OK
        err: Optional[BaseException] = None
        try:
            new = self._local_step()
            if len(new) > self.capacity:
                raise RuntimeError(f"{len(new)} tokens in one step exceed the record capacity {self.capacity}")
            rec[1] = 1 if self.engine.has_unfinished() else 0
            rec[2] = len(new)
            if new:
                rec[_HDR:_HDR + 3 * len(new)] = np.asarray(new, dtype=np.int32).reshape(-1)
        except Exception as e:  # joins the collective anyway, flagged
            err = e
            rec[0] = _ERROR
            rec[1] = 0
            rec[2] = 0
        t0 = time.perf_counter()
        gathered = self._all_gather(torch.from_numpy(rec))
        self.exchange_seconds += time.perf_counter() - t0
        self.steps += 1
        if err is not None:
            raise ShardError(f"rank {self.rank} failed at step {self.steps}: {err}") from err
        bad = [r for r in range(self.world) if int(gathered[r, 0]) != _OK]
        if bad:
            raise ShardError(f"rank(s) {bad} failed at step {self.steps}")
        finished = []
        for r in range(self.world):
            n = int(gathered[r, 2])
            rows = gathered[r, _HDR:_HDR + 3 * n].reshape(n, 3)
            for rid, tok, fin in rows.tolist():
                req = self.requests[rid]
                req.tokens.append(tok)
                if fin:
                    req.finished = True
                    finished.append(rid)
        return finished

    def run(self) -> Dict[int, List[int]]:
        while self.has_unfinished():
            self.step()
        return {rid: r.tokens for rid, r in self.requests.items()}

    # -------------------------------------------------------------- helpers
    def _all_gather(self, rec: torch.Tensor) -> np.ndarray:
        src = rec.to(self.device)
        out = torch.empty(self.world * src.numel(), dtype=torch.int32, device=self.device)
        dist.all_gather_into_tensor(out, src, group=self.group)
        return out.view(self.world, -1).cpu().numpy()

    def _local_step(self):
        """Run the local engine step; return [(request_id, token, finished)] of the tokens it made."""
        reqs = getattr(self.engine, "requests", {})
        before = {rid: len(r.sequence.output_tokens) for rid, r in reqs.items()
                  if getattr(r, "sequence", None) is not None}
        finished_outs = self.engine.step()
        new = []
        for rid, r in reqs.items():                 # still running after the step
            seq = getattr(r, "sequence", None)
            if seq is not None:
                new.extend((rid, int(t), 0) for t in seq.output_tokens[before.get(rid, 0):])
        for o in finished_outs:
            tail = list(o.tokens)[before.get(o.request_id, 0):]
            new.extend((o.request_id, int(t), int(j == len(tail) - 1)) for j, t in enumerate(tail))
        return new
