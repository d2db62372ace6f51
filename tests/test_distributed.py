"""Sequence sharding across ranks: host logic over the gloo backend on CPU.

The local engine is a deterministic fake with the LLMEngine interface, so the
tests need no GPU: they check assignment, the per-step token all-gather, the
merged streams against a single-rank run, and failure propagation (a rank that
raises, a rank that dies).
"""

import multiprocessing as mp
import os
import socket
import traceback
from dataclasses import dataclass, field
from typing import List

import pytest


@dataclass
class _Seq:
    output_tokens: List[int] = field(default_factory=list)


@dataclass
class _Req:
    prompt: list
    max_tokens: int
    sequence: _Seq = None


@dataclass
class _Out:
    request_id: int
    tokens: List[int]


class FakeEngine:
    """FCFS admission up to max_batch_size; token k of request r is (31*r + 7*k + len(prompt)) % 97."""

    def __init__(self, max_batch_size=3, num_scheduler_steps=2, fail_at_step=None):
        self.max_batch_size = max_batch_size
        self.num_scheduler_steps = num_scheduler_steps
        self.requests = {}
        self.waiting = []
        self.running = []
        self.fail_at_step = fail_at_step
        self.steps = 0

    def add_request(self, prompt, params, request_id):
        self.requests[request_id] = _Req(list(prompt), params.max_tokens)
        self.waiting.append(request_id)

    def has_unfinished(self):
        return bool(self.waiting or self.running)

    def _tok(self, rid):
        r = self.requests[rid]
        return (31 * rid + 7 * len(r.sequence.output_tokens) + len(r.prompt)) % 97

    def step(self):
        self.steps += 1
        if self.fail_at_step == self.steps:
            raise RuntimeError("Out of KV cache memory!")
        fresh = []
        while len(self.running) < self.max_batch_size and self.waiting:
            rid = self.waiting.pop(0)
            self.requests[rid].sequence = _Seq()
            self.running.append(rid)
            fresh.append(rid)
        done = []
        for rid in fresh:
            self.requests[rid].sequence.output_tokens.append(self._tok(rid))
        decode = [r for r in self.running if r not in fresh]
        for _ in range(self.num_scheduler_steps):
            for rid in list(decode):
                seq = self.requests[rid].sequence
                if len(seq.output_tokens) < self.requests[rid].max_tokens:
                    seq.output_tokens.append(self._tok(rid))
        outs = []
        for rid in list(self.running):
            r = self.requests[rid]
            if len(r.sequence.output_tokens) >= r.max_tokens:
                self.running.remove(rid)
                outs.append(_Out(rid, list(r.sequence.output_tokens)))
                del self.requests[rid]
        return outs


@dataclass
class _Params:
    max_tokens: int


PROMPTS = [[1] * n for n in (5, 40, 3, 17, 9, 60, 2, 11, 30)]
MAX_TOKENS = [4, 9, 2, 7, 5, 3, 8, 6, 1]


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def _worker(rank, world, port, mode, q):
    import datetime
    import torch
    import torch.distributed as dist
    from tinyvllm_b200.distributed import ShardedEngine, ShardError
    try:
        os.environ["MASTER_ADDR"] = "127.0.0.1"
        os.environ["MASTER_PORT"] = str(port)
        dist.init_process_group("gloo", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=10))
        fail = 2 if (mode == "raise" and rank == 1) else None
        mbs = 3 + 2 * rank if mode == "uneven" else 3
        eng = ShardedEngine(FakeEngine(max_batch_size=mbs, fail_at_step=fail), rank, world, torch.device("cpu"))
        for p, m in zip(PROMPTS, MAX_TOKENS):
            eng.add_request(p, _Params(m))
        if mode == "die" and rank == 1:
            eng.step()
            os._exit(0)           # leaves between steps, without joining the next collective
        try:
            streams = eng.run()
            q.put((rank, "ok", streams, [eng.owner(i) for i in range(len(PROMPTS))], eng.steps))
        except ShardError as e:
            q.put((rank, "shard_error", str(e), None, eng.steps))
        except Exception as e:  # collective failure after a peer died
            q.put((rank, "error", type(e).__name__, None, eng.steps))
        dist.destroy_process_group()
    except Exception:
        q.put((rank, "crash", traceback.format_exc(), None, -1))


def _launch(world, mode, timeout=60):
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, world, port, mode, q)) for r in range(world)]
    for p in procs:
        p.start()
    results = {}
    expected = world if mode != "die" else world - 1
    for _ in range(expected):
        r = q.get(timeout=timeout)
        results[r[0]] = r
    for p in procs:
        p.join(timeout=timeout)
        if p.is_alive():
            p.kill()
    return results


def _single_rank_streams():
    eng = FakeEngine()
    outs = {}
    for i, (p, m) in enumerate(zip(PROMPTS, MAX_TOKENS)):
        eng.add_request(p, _Params(m), request_id=i)
    while eng.has_unfinished():
        for o in eng.step():
            outs[o.request_id] = o.tokens
    return outs


@pytest.mark.slow
def test_two_ranks_merge_to_the_single_rank_streams():
    res = _launch(2, "ok")
    assert all(r[1] == "ok" for r in res.values()), res
    s0, s1 = res[0][2], res[1][2]
    assert s0 == s1                                   # every rank ends with every stream
    assert s0 == _single_rank_streams()               # sharding changes no token
    owners = res[0][3]
    assert set(owners) == {0, 1} and owners == res[1][3]
    assert res[0][4] == res[1][4]                     # same number of collective steps


@pytest.mark.slow
def test_ranks_with_different_batch_sizes_agree_on_the_record_size():
    """Each rank may size its engine to its own memory; the per-step all-gather
    still needs one record size, so the ranks agree on the largest."""
    res = _launch(2, "uneven")
    assert all(r[1] == "ok" for r in res.values()), res
    assert res[0][2] == res[1][2] == _single_rank_streams()


@pytest.mark.slow
def test_a_rank_that_raises_fails_every_rank_at_the_same_step():
    res = _launch(2, "raise")
    assert res[0][1] == "shard_error" and res[1][1] == "shard_error", res
    assert res[0][4] == res[1][4] == 2


@pytest.mark.slow
def test_a_rank_that_dies_is_detected_by_the_next_collective():
    res = _launch(2, "die")
    assert res[0][1] in ("error", "shard_error"), res


def test_assignment_balances_outstanding_work():
    import torch
    from tinyvllm_b200.distributed import ShardedEngine
    eng = ShardedEngine(FakeEngine(), 0, 4, torch.device("cpu"))
    for n in (100, 10, 10, 10, 10, 50):
        eng.add_request([0] * n, _Params(0))
    assert [eng.owner(i) for i in range(6)] == [0, 1, 2, 3, 1, 2]
