"""Benchmark of the tinyvllm attention hot path on B200.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]

Headline workload (config 3 of the hot-path contract), per GPU: one decode
step of the attention layer over 256 sequences, 32 query / 8 KV heads,
head_dim 128, block 16, fp16 K/V, contexts ~ U{128..4096}, random
non-contiguous tables in a pool 1.2x the blocks needed; then, as the
sequence-sharded engine does every step, the greedy pick over a per-rank
[256, vocab 128256] logits buffer and the NCCL all-gather of the int32 tokens
over all ranks.  A *step* is that attention call + argmax + token all-gather.
``value`` = decode tokens (sequences) per second, summed over all GPUs.  Each
rank holds its own seeded batch (queries, K/V values, tables) with config 3's
context lengths (weak scaling: the same K/V bytes per GPU); the all-gather is
the only exchange, and it runs on its own stream, so step i's exchange
overlaps step i+1's attention (a rank's next step needs only its own tokens).
Every step reads ~2.2 GB of K/V per GPU, far larger than the 126 MB L2, so no
flush is needed between steps.

``roofline`` covers the attention call alone (its own CUDA events).  ``e2e``
times the same step through the public Python API with the per-step inputs
(queries, block tables, context lengths) copied from pinned host memory and
the gathered tokens copied back inside the timed region; the KV pool is
device-resident state, as it is in the reference engine.

The same JSON line nests the other configurations' results (``--no-nested``
skips them): ``prefill`` (config 2, one ragged causal prefill call with the
paged K/V write), ``engine_config4`` (TinyLlama-1.1B fp16 under continuous
batching, N=1 only) and ``engine_config5`` (Llama-3-8B-shape bf16 decode,
512 sequences sharded by sequence over the N ranks with the per-step token
all-gather).

``--impl reference`` times the reference algorithm on the host cores: the
numpy restatement of tinyvllm/model/llama.py:97-144 plus the greedy pick
(tinygrad itself is not installable in this image), on a bounded sample of
the same workload.
"""

from __future__ import annotations

import argparse
import ctypes
import json
import os
import statistics
import subprocess
import sys
import threading
import time
from pathlib import Path

ROOT = Path(__file__).resolve().parent
sys.path.insert(0, str(ROOT))

METRIC = ("decode tok/s: one paged-decode attention layer over the batch + greedy pick + int32 token "
          "all-gather across ranks per step")
UNIT = "tok/s"
CPU_SAMPLE_SEQS = 16
VOCAB = 128256     # Llama-3-8B vocabulary (config 3 has its attention layout)


def _peaks():
    p = ROOT / "MEASURED_PEAKS.json"
    if p.exists():
        d = json.loads(p.read_text())
        return float(d["hbm_gbs"]), "measured"
    return 6650.0, "fallback"


class ClockSampler:
    """Samples nvidia-smi SM clocks and throttle reasons while the timed region runs."""

    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, n_gpus: int):
        self.n = n_gpus
        self.rows = []
        self.proc = None
        self.thread = None

    def start(self):
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", f"--query-gpu={self.FIELDS}", "--format=csv,noheader,nounits", "-lms", "200"],
                stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
        except (FileNotFoundError, OSError):
            self.proc = None
            return
        self.thread = threading.Thread(target=self._read, daemon=True)
        self.thread.start()

    def _read(self):
        for line in self.proc.stdout:
            parts = [x.strip() for x in line.split(",")]
            if len(parts) >= 9:
                self.rows.append(parts)

    def stop(self):
        if self.proc is None:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["nvidia-smi unavailable"]}
        self.proc.terminate()
        try:
            self.proc.wait(timeout=5)
        except subprocess.TimeoutExpired:
            self.proc.kill()
        if self.thread:
            self.thread.join(timeout=5)
        rows = [r for r in self.rows if r[0].isdigit() and int(r[0]) < self.n]
        if not rows:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["no samples"], "samples": 0}

        def num(x):
            try:
                return float(x)
            except ValueError:
                return None
        sm = [num(r[1]) for r in rows if num(r[1]) is not None]
        mx = [num(r[2]) for r in rows if num(r[2]) is not None]
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        reasons = sorted({names[i] for r in rows for i in range(4) if r[5 + i].lower().startswith("active")})
        return {"sm_mhz": statistics.median(sm) if sm else None, "sm_max_mhz": max(mx) if mx else None,
                "reasons": reasons, "samples": len(rows),
                "power_w_max": max((num(r[3]) or 0.0) for r in rows)}


_BLAS_LIMITS = None


def _all_host_threads() -> int:
    """Let the BLAS behind numpy use every host core and return the threads it now
    uses.  torchrun exports OMP_NUM_THREADS=1 to each rank, which would otherwise
    leave the CPU restatement single-threaded under --gpus N > 1."""
    global _BLAS_LIMITS
    try:
        from threadpoolctl import threadpool_info, threadpool_limits
        _BLAS_LIMITS = threadpool_limits(limits=os.cpu_count() or 1, user_api="blas")
        n = max((int(i.get("num_threads", 1)) for i in threadpool_info() if i.get("user_api") == "blas"), default=1)
        return max(n, 1)
    except Exception:   # no threadpoolctl: report what the environment allows
        return int(os.environ.get("OMP_NUM_THREADS", os.cpu_count() or 1))


def _fastest_blas_threads(call) -> int:
    """Time one call with every host core and one with a single BLAS thread (the
    restatement's matmuls are small, and on some hosts threading only costs), keep
    the faster setting for the timed calls and return its thread count."""
    global _BLAS_LIMITS
    n_all = _all_host_threads()
    t0 = time.perf_counter()
    call()
    t_all = time.perf_counter() - t0
    if n_all <= 1:
        return 1
    try:
        from threadpoolctl import threadpool_limits
    except Exception:
        return n_all
    one = threadpool_limits(limits=1, user_api="blas")
    t0 = time.perf_counter()
    call()
    t_one = time.perf_counter() - t0
    if t_one < t_all:
        _BLAS_LIMITS = one
        return 1
    one.restore_original_limits()
    return _all_host_threads()


def cpu_baseline_sample(n_seqs: int = CPU_SAMPLE_SEQS, reps: int = 5):
    """Time the oracle restatement of the reference step on a bounded sample of
    config 3: the first ``n_seqs`` sequences with their own blocks (attention,
    llama.py:97-144) plus the greedy pick over their [n_seqs, vocab] logits
    (sampling.py:133-134), on the host."""
    import numpy as np
    from oracle import attention as oa
    from tinyvllm_b200 import workloads
    case = workloads.decode_config3("cpu", batch=n_seqs)
    q = case.q.float().numpy()
    kc = case.k_cache.float().numpy()
    vc = case.v_cache.float().numpy()
    bt = case.block_tables.numpy()
    ctx = case.context_lens.numpy()
    logits = np.random.default_rng(4321).standard_normal((n_seqs, VOCAB), dtype=np.float32)

    def one():
        oa.paged_decode_attention(q, kc, vc, bt, ctx, 32, 8, 128, 16)
        oa.greedy_argmax(logits)

    threads = _fastest_blas_threads(one)
    times = []
    for _ in range(reps):
        t0 = time.perf_counter()
        one()
        times.append(time.perf_counter() - t0)
    med = statistics.median(times)
    sample = (f"first {n_seqs} sequences of config 3 (ctx sum {int(ctx.sum())}, table width "
              f"{bt.shape[1]} blocks) + argmax over [{n_seqs}, {VOCAB}] logits, numpy restatement of "
              f"llama.py:97-144 and sampling.py:133-134, median of {reps}, {threads} BLAS thread(s), the "
              "faster of one and all host cores")
    return {"value": n_seqs / med, "unit": UNIT, "cores": threads, "kind": "port", "sample": sample,
            "seconds_per_call": med}


def run_reference(args, rank: int, world: int) -> int:
    if rank != 0:
        return 0
    import numpy as np
    from oracle import attention as oa
    from tinyvllm_b200 import workloads
    n = CPU_SAMPLE_SEQS
    case = workloads.decode_config3("cpu", batch=n)
    q = case.q.float().numpy()
    kc = case.k_cache.float().numpy()
    vc = case.v_cache.float().numpy()
    bt = case.block_tables.numpy()
    ctx = case.context_lens.numpy()
    logits = np.random.default_rng(4321).standard_normal((n, VOCAB), dtype=np.float32)

    def one():
        oa.paged_decode_attention(q, kc, vc, bt, ctx, 32, 8, 128, 16)
        oa.greedy_argmax(logits)

    threads = _fastest_blas_threads(one)
    for _ in range(args.warmup):
        one()
    t0 = time.perf_counter()
    for _ in range(args.steps):
        one()
    dt = (time.perf_counter() - t0) / args.steps
    value = n / dt
    line = {
        "impl": "reference", "metric": METRIC, "value": value, "unit": UNIT, "n_gpus": args.gpus,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": dt * 1e3, "higher_is_better": True,
        "scaling": "weak", "vs_baseline": None, "dtype": "f32", "data": "synthetic",
        "config": {"workload": "config3 paged decode + greedy pick, bounded sample", "batch": n, "n_heads": 32,
                   "n_kv_heads": 8, "head_dim": 128, "block_size": 16, "ctx": "U{128..4096}", "vocab": VOCAB},
        "cpu_baseline": {"value": value, "unit": UNIT, "cores": threads, "kind": "port",
                         "sample": f"first {n} sequences of config 3 per step; tinygrad absent, so the numpy "
                                   f"restatement of llama.py:97-144 and sampling.py:133-134 on {threads} BLAS "
                                   "thread(s), the faster of one and all host cores"},
        "e2e": {"value": value, "unit": UNIT, "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)
    return 0


def _free_port() -> int:
    import socket
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _init_group(rank: int, world: int, dev) -> None:
    """One NCCL process group for the whole run (a one-rank group at N=1, so the
    step's token all-gather runs at every N).  Short timeout: ranks that wait for
    one another end with an error instead of hanging."""
    import datetime
    import torch.distributed as dist
    if dist.is_initialized():
        return
    os.environ.setdefault("MASTER_ADDR", "127.0.0.1")
    if "MASTER_PORT" not in os.environ:
        os.environ["MASTER_PORT"] = str(_free_port())
    dist.init_process_group("nccl", device_id=dev, rank=rank, world_size=world,
                            timeout=datetime.timedelta(seconds=120))


def decode_headline(args, rank: int, world: int, local_rank: int):
    """Config 3 per rank: attention + greedy pick + token all-gather per step."""
    import torch
    import torch.distributed as dist
    from tinyvllm_b200 import layers, workloads
    from tinyvllm_b200.attention import paged_decode_attention

    dev = torch.device("cuda", local_rank)
    # Every rank holds config 3's batch: its own queries, K/V values and tables,
    # the same context lengths (weak scaling: fixed work per GPU).
    case = workloads.decode_config3(dev, batch=args.batch, seed_offset=rank, shared_contexts=True)
    B = case.batch
    g = torch.Generator(device=dev).manual_seed(4321 + rank)
    logits = torch.randn(B, VOCAB, generator=g, device=dev, dtype=torch.float32).half()
    stream = torch.cuda.current_stream(dev)
    # The token all-gather runs on its own stream: a rank's next step needs only
    # its own tokens, so step i's exchange overlaps step i+1's attention (the
    # next argmax waits for it, since both use the token buffer).
    comm = torch.cuda.Stream(dev)
    ag_done = [None]

    def step(q, bt, ctx, o, tokens, gathered, ev=None):
        if ev is not None:
            ev[0].record(stream)
        paged_decode_attention(q, case.k_cache, case.v_cache, bt, ctx, 32, 8, 128, 16, out=o)
        if ev is not None:
            ev[1].record(stream)
        if ag_done[0] is not None:
            stream.wait_event(ag_done[0])
        layers.greedy_argmax(logits, out=tokens)
        if ev is not None:
            ev[2].record(stream)
        picked = torch.cuda.Event()
        picked.record(stream)
        done = torch.cuda.Event()
        with torch.cuda.stream(comm):
            comm.wait_event(picked)
            dist.all_gather_into_tensor(gathered, tokens)
            done.record(comm)
        ag_done[0] = done

    out = torch.empty_like(case.q)
    tokens = torch.empty(B, dtype=torch.int32, device=dev)
    gathered = torch.empty(world * B, dtype=torch.int32, device=dev)

    def barrier():
        dist.barrier(device_ids=[local_rank])
        torch.cuda.synchronize(dev)

    for _ in range(args.warmup):
        step(case.q, case.block_tables, case.context_lens, out, tokens, gathered)
    barrier()

    clocks = ClockSampler(world) if rank == 0 else None
    if clocks:
        clocks.start()
        time.sleep(0.3)
    # ---- device-resident timed region ----
    ev = [tuple(torch.cuda.Event(enable_timing=True) for _ in range(3)) for _ in range(args.steps)]
    barrier()
    t_start = torch.cuda.Event(enable_timing=True)
    t_end = torch.cuda.Event(enable_timing=True)
    t_start.record(stream)
    for i in range(args.steps):
        step(case.q, case.block_tables, case.context_lens, out, tokens, gathered, ev[i])
    stream.wait_stream(comm)
    t_end.record(stream)
    barrier()
    total_ms = t_start.elapsed_time(t_end)
    per_attn = [e[0].elapsed_time(e[1]) for e in ev]
    per_argmax = [e[1].elapsed_time(e[2]) for e in ev]

    # ---- end-to-end through the public API with host buffers ----
    # Every step copies its inputs from pinned host memory and the gathered tokens
    # back.  The copies run on their own streams into two alternating sets of
    # device buffers, so the transfers of neighbouring steps overlap this step's
    # kernels (as a serving loop overlaps them); events order each slot's reuse.
    q_h = case.q.cpu().pin_memory()
    bt_h = case.block_tables.cpu().pin_memory()
    ctx_h = case.context_lens.cpu().pin_memory()
    tok_h = torch.empty(world * B, dtype=torch.int32).pin_memory()
    bufs = [(torch.empty_like(case.q), torch.empty_like(case.block_tables), torch.empty_like(case.context_lens),
             torch.empty_like(case.q), torch.empty_like(tokens), torch.empty_like(gathered)) for _ in range(2)]
    h2d, d2h = torch.cuda.Stream(dev), torch.cuda.Stream(dev)
    ev_in = [torch.cuda.Event() for _ in range(2)]
    ev_done = [torch.cuda.Event() for _ in range(2)]
    ev_out = [torch.cuda.Event() for _ in range(2)]
    n_issued = [0]

    def e2e_step():
        i = n_issued[0]
        n_issued[0] += 1
        sl = i % 2
        q_d, bt_d, ctx_d, o_d, t_d, g_d = bufs[sl]
        with torch.cuda.stream(h2d):
            if i >= 2:
                h2d.wait_event(ev_done[sl])          # step i-2's kernels have read this slot
            q_d.copy_(q_h, non_blocking=True)
            bt_d.copy_(bt_h, non_blocking=True)
            ctx_d.copy_(ctx_h, non_blocking=True)
            ev_in[sl].record(h2d)
        stream.wait_event(ev_in[sl])
        if i >= 2:
            stream.wait_event(ev_out[sl])            # step i-2's tokens have left this slot
        step(q_d, bt_d, ctx_d, o_d, t_d, g_d)
        ev_done[sl].record(stream)
        with torch.cuda.stream(d2h):
            d2h.wait_event(ag_done[0])              # this step's tokens are gathered
            tok_h.copy_(g_d, non_blocking=True)
            ev_out[sl].record(d2h)

    for _ in range(3):
        e2e_step()
    torch.cuda.synchronize(dev)
    barrier()
    e0 = torch.cuda.Event(enable_timing=True)
    e1 = torch.cuda.Event(enable_timing=True)
    e0.record(h2d)
    stream.wait_event(e0)
    for _ in range(args.steps):
        e2e_step()
    e1.record(d2h)
    torch.cuda.synchronize(dev)
    barrier()
    e2e_ms = e0.elapsed_time(e1)
    # the same steps with every copy and kernel in one stream, for reference
    q_d, bt_d, ctx_d, o_d, t_d, g_d = bufs[0]
    s0 = torch.cuda.Event(enable_timing=True)
    s1 = torch.cuda.Event(enable_timing=True)
    s0.record(stream)
    for _ in range(args.steps):
        q_d.copy_(q_h, non_blocking=True)
        bt_d.copy_(bt_h, non_blocking=True)
        ctx_d.copy_(ctx_h, non_blocking=True)
        step(q_d, bt_d, ctx_d, o_d, t_d, g_d)
        stream.wait_stream(comm)
        tok_h.copy_(g_d, non_blocking=True)
    s1.record(stream)
    torch.cuda.synchronize(dev)
    serial_ms = s0.elapsed_time(s1)
    barrier()
    clk = clocks.stop() if clocks else None

    # max over ranks
    t = torch.tensor([total_ms, e2e_ms, serial_ms], dtype=torch.float64, device=dev)
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    total_ms, e2e_ms, serial_ms = float(t[0]), float(t[1]), float(t[2])
    if rank != 0:
        return None
    from tinyvllm_b200 import _lib
    ms = total_ms / args.steps
    value = B * world * args.steps / (total_ms / 1e3)
    e2e_value = B * world * args.steps / (e2e_ms / 1e3)
    peak, peak_kind = _peaks()
    alg = case.algorithmic_bytes()
    avg_attn_ms = statistics.mean(per_attn)
    achieved = alg / (avg_attn_ms / 1e3) / 1e9
    L = _lib.lib()
    plan = (ctypes.c_int * 4)()
    _lib.check(L.tvk_paged_decode_plan(B, 32, 8, 128, 16, case.block_tables.shape[1], -1, 1, plan),
               "tvk_paged_decode_plan")
    traffic_path = ROOT / "profiles" / "paged_decode_tc_config3.traffic.json"
    traffic = None
    if traffic_path.exists():
        traffic = json.loads(traffic_path.read_text()).get("bytes_per_launch")
    cpu = cpu_baseline_sample() if world == 1 and not args.no_cpu_baseline else None
    h2d_bytes = q_h.numel() * q_h.element_size() + bt_h.numel() * 4 + ctx_h.numel() * 4
    d2h_bytes = tok_h.numel() * 4
    return {
        "metric": METRIC, "value": value, "unit": UNIT, "n_gpus": world, "steps": args.steps,
        "warmup": args.warmup, "ms_per_step": ms, "higher_is_better": True, "scaling": "weak",
        "vs_baseline": None, "dtype": "f16", "data": "synthetic",
        "config": {"workload": "config3 paged-decode attention (256 seqs/GPU, 32q/8kv heads, D=128, "
                               "block 16, fp16, ctx U{128..4096}, shuffled tables, pool 1.2x) + greedy pick over "
                               f"[256, {VOCAB}] fp16 logits + NCCL all-gather of the int32 tokens",
                   "batch_per_gpu": B, "global_batch": B * world, "ctx_sum_rank0": int(case.context_lens.sum()),
                   "l2": "no flush: each step reads ~2.2 GB of K/V per GPU (> 126 MB L2)",
                   "parallelism": f"sequence-sharded x{world}; per step one all-gather of {B} int32 tokens per rank, "
                                  "on its own stream, overlapping the next step's attention",
                   "contexts": "config 3's draw on every rank (same K/V bytes per GPU); values and tables "
                               "seeded per rank"},
        "roofline": {"bound": "hbm", "achieved": achieved, "peak": peak, "unit": "GB/s",
                     "frac": achieved / peak, "traffic": traffic, "peak_kind": peak_kind,
                     "algorithmic_bytes_per_launch": alg,
                     "avg_attention_ms": avg_attn_ms,
                     "note": "the attention call's own CUDA events (main kernel, plus the split-K combine when "
                             "the plan has one); the step adds the argmax and the all-gather",
                     "unit_tokens": plan[0], "max_splits": plan[1], "persistent": bool(plan[3])},
        "step_breakdown_ms": {"attention": avg_attn_ms, "argmax": statistics.mean(per_argmax),
                              "rest": ms - avg_attn_ms - statistics.mean(per_argmax)},
        "cpu_baseline": cpu,
        "e2e": {"value": e2e_value, "unit": UNIT, "h2d_bytes_per_step": h2d_bytes, "d2h_bytes_per_step": d2h_bytes,
                "ms_per_step": e2e_ms / args.steps,
                "overlap": "copies on two extra streams, double-buffered: step i+1's inputs and step i-1's "
                           "tokens move while step i's kernels run",
                "serial": {"value": B * world * args.steps / (serial_ms / 1e3),
                           "ms_per_step": serial_ms / args.steps,
                           "note": "copies and kernels in one stream, nothing overlapped"}},
        "clocks": clk,
        "gpu_launches": (plan[2] + 1) * args.steps,
        "gpu_launches_note": "per step: the attention kernel(s) and the argmax kernel; NCCL's own kernel "
                             "for the all-gather is not counted",
    }


def decode_engine_shape_line(args, rank: int, world: int, local_rank: int):
    """The decode attention call the config-4 engine makes at full batch: 64
    sequences x 32 query / 4 KV heads, head_dim 64, fp16, 64-block tables (the
    reference's 1024-token cap), every context 1024 tokens.  One call per step
    with L2 flushed before it (each engine layer reads its own pool); CUDA events
    around each call.  For profiling and the engine-shape figures; not a headline."""
    import torch
    from tinyvllm_b200 import workloads
    from tinyvllm_b200.attention import paged_decode_attention
    dev = torch.device("cuda", local_rank)
    case = workloads.decode_case(64, 32, 4, 64, 16, [1024] * 64, dtype=torch.float16, device=dev, seed=3, width=64)
    out = torch.empty_like(case.q)
    flush = torch.empty(256 << 20, dtype=torch.uint8, device=dev)
    args_call = (case.q, case.k_cache, case.v_cache, case.block_tables, case.context_lens, 32, 4, 64, 16)
    for _ in range(args.warmup):
        paged_decode_attention(*args_call, out=out)
    torch.cuda.synchronize(dev)
    ts = []
    for i in range(args.steps):
        flush.fill_(i & 0xFF)
        a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        a.record()
        paged_decode_attention(*args_call, out=out)
        b.record()
        torch.cuda.synchronize(dev)
        ts.append(a.elapsed_time(b))
    if rank != 0:
        return None
    ms = statistics.median(ts)
    alg = case.algorithmic_bytes()
    peak, kind = _peaks()
    return {"metric": "paged-decode attention, engine shape (64 seqs x 4 KV heads, D=64, ctx 1024)",
            "value": 64 / (ms / 1e3), "unit": "tok/s", "ms_per_step": ms, "steps": args.steps,
            "warmup": args.warmup, "n_gpus": 1, "higher_is_better": True, "dtype": "f16", "data": "synthetic",
            "roofline": {"bound": "hbm", "achieved": alg / (ms / 1e3) / 1e9, "peak": peak, "unit": "GB/s",
                         "frac": alg / (ms / 1e3) / 1e9 / peak, "peak_kind": kind},
            "config": {"workload": "decode attention at the config-4 engine shape", "l2": "flushed before each call"}}


PREFILL_LENS = (1, 15, 16, 17, 128, 500, 1024, 2048)


def _tensor_peak():
    p = ROOT / "MEASURED_PEAKS.json"
    if p.exists():
        d = json.loads(p.read_text())
        return float(d["bf16_tflops"]), "measured (bf16 burst; fp16 dense rate is the same)"
    return 1590.0, "fallback"


def prefill_line(args, rank: int, world: int, local_rank: int):
    """Config 2: 8 fp16 prompts (32q/4kv heads, D=64) through one ragged causal
    prefill call with the paged K/V write into a fresh 1024-block pool."""
    import numpy as np
    import torch
    from tinyvllm_b200.attention import flash_prefill_attention_varlen
    from tinyvllm_b200.block_manager import BlockManager

    dev = torch.device("cuda", local_rank)
    from tinyvllm_b200 import _lib
    choice = {"auto": 0, "one-head": 1, "paired": 2}[args.prefill_kernel]
    _lib.check(_lib.lib().tvk_prefill_select_kernel(choice), "tvk_prefill_select_kernel")
    lens = tuple(int(x) for x in args.prefill_lens.split(",")) if args.prefill_lens else PREFILL_LENS
    hq, hkv, hd = 32, args.prefill_kv_heads, args.prefill_head_dim
    dt = torch.bfloat16 if args.prefill_dtype == "bf16" else torch.float16
    is_cfg2 = lens == PREFILL_LENS and (hkv, hd, dt) == (4, 64, torch.float16)
    T = sum(lens)
    g = torch.Generator(device=dev).manual_seed(1236 + rank)
    q = torch.randn(T, hq, hd, generator=g, device=dev).to(dt)
    k = torch.randn(T, hkv, hd, generator=g, device=dev).to(dt)
    v = torch.randn(T, hkv, hd, generator=g, device=dev).to(dt)
    cu = torch.tensor(np.concatenate([[0], np.cumsum(lens)]), dtype=torch.int32, device=dev)
    n_blocks = max(1024, sum((L + 15) // 16 for L in lens))
    bm = BlockManager(1, n_blocks, 16)
    slots = []
    for sid, L in enumerate(lens):
        bm.register_sequence(sid)
        slots.append(bm.slot_mapping(sid, 0, L))
    slots = torch.from_numpy(np.concatenate(slots)).to(dev)
    kc = torch.zeros(n_blocks, 16, hkv, hd, dtype=dt, device=dev)
    vc = torch.zeros_like(kc)
    out = torch.empty_like(q)
    flush = torch.empty(256 << 20, dtype=torch.uint8, device=dev)   # > 126 MB L2
    stream = torch.cuda.current_stream(dev)
    steps = args.prefill_steps

    def call():
        flash_prefill_attention_varlen(q, k, v, cu, max(lens), True, slot_mapping=slots, k_cache=kc, v_cache=vc,
                                       out=out)

    for _ in range(args.warmup):
        call()
    torch.cuda.synchronize(dev)
    # The device-resident number replays the call from a CUDA graph, so the host's
    # launch work (argument checks, tensor-map encoding) does not leave the GPU
    # idle inside the events; the e2e number below keeps it.
    # Device timing: two CUDA graphs, [L2 flush + call] and [L2 flush] alone, each
    # replayed `steps` times back to back between CUDA events; the call's time is
    # the difference per replay.  Every call starts with q/k/v evicted from L2 (a
    # 256 MB write, then its read-back so that the dirty lines leave L2 inside the
    # flush), and the launch gap of a lone replay after an idle stream is not counted.
    def flush_l2():
        flush.fill_(7)
        flush.view(torch.int64).sum()

    side = torch.cuda.Stream(dev)
    graphs = {}
    with torch.cuda.stream(side):
        for name, fn in (("flush", flush_l2), ("both", lambda: (flush_l2(), call()))):
            fn()
            torch.cuda.synchronize(dev)
            gr = torch.cuda.CUDAGraph()
            with torch.cuda.graph(gr, stream=side):
                fn()
            graphs[name] = gr
    torch.cuda.synchronize(dev)
    for _ in range(args.warmup):
        graphs["both"].replay()
        graphs["flush"].replay()
    torch.cuda.synchronize(dev)
    clocks = ClockSampler(1) if rank == 0 else None
    if clocks:
        clocks.start()
        time.sleep(0.3)
    loop_ms = {}
    for rep in range(3):                         # three rounds, alternating; the median of the differences
        for name in ("both", "flush"):
            a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            a.record(stream)
            for _ in range(steps):
                graphs[name].replay()
            b.record(stream)
            torch.cuda.synchronize(dev)
            loop_ms.setdefault(name, []).append(a.elapsed_time(b) / steps)
    per_step = [x - y for x, y in zip(loop_ms["both"], loop_ms["flush"])]

    # ---- end-to-end through the public API with host buffers ----
    q_h, k_h, v_h = q.cpu().pin_memory(), k.cpu().pin_memory(), v.cpu().pin_memory()
    cu_h, slots_h = cu.cpu().pin_memory(), slots.cpu().pin_memory()
    out_h = torch.empty(out.shape, dtype=out.dtype).pin_memory()
    q_d, k_d, v_d = torch.empty_like(q), torch.empty_like(k), torch.empty_like(v)
    cu_d, slots_d = torch.empty_like(cu), torch.empty_like(slots)

    def e2e_step():
        for d_, h_ in ((q_d, q_h), (k_d, k_h), (v_d, v_h), (cu_d, cu_h), (slots_d, slots_h)):
            d_.copy_(h_, non_blocking=True)
        o = flash_prefill_attention_varlen(q_d, k_d, v_d, cu_d, max(lens), True, slot_mapping=slots_d,
                                           k_cache=kc, v_cache=vc)
        out_h.copy_(o, non_blocking=True)

    for _ in range(3):
        e2e_step()
    torch.cuda.synchronize(dev)
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(stream)
    for _ in range(steps):
        e2e_step()
    e1.record(stream)
    torch.cuda.synchronize(dev)
    e2e_ms = e0.elapsed_time(e1) / steps
    h2d = sum(t.numel() * t.element_size() for t in (q_h, k_h, v_h, cu_h, slots_h))
    d2h = out_h.numel() * out_h.element_size()
    clk = clocks.stop() if clocks else None
    del graphs
    if rank != 0:
        return None
    ms = statistics.median(per_step)
    flops = 4.0 * hq * hd * sum(L * (L + 1) / 2 for L in lens)
    achieved = flops / (ms / 1e3) / 1e12
    peak, kind = _tensor_peak()
    cpu = None
    if not args.no_cpu_baseline and is_cfg2 and world == 1:
        from oracle import attention as oa
        threads = _all_host_threads()
        qn, kn, vn = q.float().cpu().numpy(), k.float().cpu().numpy(), v.float().cpu().numpy()
        t0 = time.perf_counter()
        for i, L in enumerate(lens):
            a, b = int(cu[i]), int(cu[i + 1])
            oa.flash_prefill_attention(qn[None, a:b], kn[None, a:b], vn[None, a:b], True)
        dt_cpu = time.perf_counter() - t0
        cpu = {"value": T / dt_cpu, "unit": "prompt tok/s", "cores": threads, "kind": "port",
               "sample": "all 8 config-2 prompts once, numpy restatement of llama.py:58-94"}
    traffic = None
    tp = ROOT / "profiles" / "flash_prefill_pair_config2.traffic.json"
    if is_cfg2 and tp.exists():
        traffic = json.loads(tp.read_text()).get("bytes_per_launch")
    exp_bound = 2.0 * 2 * 128 * 64 * hd / 512 * 148 * 1.965e9 / 1e12
    return {
        "metric": "flash-prefill attention: prompt tok/s (" + ("config 2" if is_cfg2 else "custom prompts") +
                  ", one ragged call per step)",
        "value": T / (ms / 1e3), "unit": "prompt tok/s", "n_gpus": 1, "steps": steps, "warmup": args.warmup,
        "ms_per_step": ms, "higher_is_better": True, "scaling": "weak", "vs_baseline": None,
        "dtype": "bf16" if dt == torch.bfloat16 else "f16",
        "data": "synthetic",
        "config": {"workload": ("config2" if is_cfg2 else "custom") + f" causal prefill, {len(lens)} prompts L=" +
                               ",".join(map(str, lens)) + f", {hq}q/{hkv}kv heads, D={hd}, " +
                               ("bf16" if dt == torch.bfloat16 else "fp16") + f", paged write into {n_blocks} blocks",
                   "l2": "flushed before every call (256 MB write, then read back)",
                   "timing": "graphs [flush + call] and [flush] each replayed back to back between CUDA events; "
                             "the call's time is the difference per replay (median of three rounds)",
                   "flush_ms": statistics.median(loop_ms["flush"])},
        "roofline": {"bound": "tensor", "achieved": achieved, "peak": peak, "unit": "TFLOP/s",
                     "frac": achieved / peak, "traffic": traffic, "peak_kind": kind,
                     "algorithmic_flops_per_launch": flops,
                     # a 128x64 tile needs 8192 exponentials (512 cycles of the 16/cycle
                     # MUFU unit) for 2 * 2 * 128 * 64 * head_dim FLOP of MMA work
                     "exp_unit_bound_tflops": exp_bound,
                     "frac_of_exp_unit_bound": achieved / exp_bound},
        "cpu_baseline": cpu, "clocks": clk,
        "e2e": {"value": T / (e2e_ms / 1e3), "unit": "prompt tok/s", "h2d_bytes_per_step": h2d,
                "d2h_bytes_per_step": d2h, "ms_per_step": e2e_ms},
        "gpu_launches": 2 * steps,
        "kernel_choice": ("paired-head kernel" if (32 // hkv) % 2 == 0 and args.prefill_kernel != "one-head"
                          else "one-head kernel"),
    }


def e2e_cpu_baseline(model, n_req: int = 8, prompt_len: int = 32, gen: int = 16):
    """Small-horizon CPU run of the same engine semantics: the oracle restatement
    of the reference engine (engine.py:114-196 over llama.py:266-388, numpy fp32)
    with this model's weights, ``n_req`` requests of ``prompt_len`` random ids
    and ``gen`` greedy tokens each."""
    import numpy as np
    from oracle.engine import OracleEngine, OracleLlama
    c = model.config
    om = OracleLlama(model.numpy_weights(), c.n_layers, c.n_heads, c.n_kv_heads, c.head_dim, c.norm_eps,
                     c.rope_theta, prompt_len + gen + 16)
    eng = OracleEngine(om, max_batch_size=n_req, num_blocks=n_req * 8, block_size=16)
    threads = _all_host_threads()
    rng = np.random.default_rng(4321)
    for _ in range(n_req):
        eng.add_request(rng.integers(3, c.vocab_size, size=prompt_len).tolist(), gen)
    t0 = time.perf_counter()
    while eng.has_unfinished():
        eng.step()
    dt = time.perf_counter() - t0
    return {"value": n_req * gen / dt, "unit": "tok/s", "cores": threads, "kind": "port",
            "sample": f"{n_req} requests x {prompt_len}-token prompts x {gen} greedy tokens (prefill included), "
                      "numpy restatement of the reference engine and model with the same weights"}


def engine4_line(args, rank: int, world: int, local_rank: int):
    """Config 4: random-init TinyLlama-1.1B fp16 under continuous batching.  64 requests,
    prompt ids uniform in [3, 32000) with lengths U{32..512}, 128 greedy tokens each,
    four new requests before every engine step, max_batch_size 64, 4096 blocks of 16,
    reference K/V ordering, decode steps replayed as CUDA graphs.  A step of this
    workload is one complete run of all 64 requests; value = generated tokens / s."""
    import numpy as np
    import torch
    from tinyvllm_b200.engine import LLMEngine, SamplingParams
    from tinyvllm_b200.model import Llama, tinyllama_config

    dev = torch.device("cuda", local_rank)
    cfg = tinyllama_config("float16")
    model = Llama(cfg, device=dev, seed=1234 + 4 + rank)
    rng = np.random.default_rng(1238 + rank)
    n_req, max_tokens = args.e2e_requests, args.e2e_max_tokens
    prompts = [rng.integers(3, 32000, size=int(rng.integers(32, 513))).tolist() for _ in range(n_req)]
    eng = LLMEngine(model, max_batch_size=64, num_blocks=4096, num_scheduler_steps=1, use_cuda_graphs=True)
    steps = args.engine_steps
    ctx_trace = []

    step_wall = {"prefill": [], "decode": []}   # host wall time of each engine step, by kind

    def one_run(trace=False):
        i, made = 0, 0
        while i < len(prompts) or eng.has_unfinished():
            for _ in range(4):
                if i < len(prompts):
                    eng.add_request(prompts[i], SamplingParams(max_tokens=max_tokens))
                    i += 1
            if trace:
                ctx_trace.append([s.get_len() for s in eng.scheduler.running.values()])
            p0 = eng.stats["prefill_tokens"]
            t = time.perf_counter()
            made += sum(len(o.tokens) for o in eng.step())
            if not trace:
                step_wall["prefill" if eng.stats["prefill_tokens"] != p0 else "decode"].append(time.perf_counter() - t)
        return made

    one_run(trace=True)        # warm-up (graph captures) and the per-step context trace
    torch.cuda.synchronize(dev)
    clocks = ClockSampler(1) if rank == 0 else None
    if clocks:
        clocks.start()
        time.sleep(0.3)
    s0 = dict(eng.stats)
    ev0, ev1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    t0 = time.perf_counter()
    ev0.record()
    made = sum(one_run() for _ in range(steps))
    ev1.record()
    torch.cuda.synchronize(dev)
    dt = time.perf_counter() - t0
    dev_s = ev0.elapsed_time(ev1) / 1e3
    clk = clocks.stop() if clocks else None
    if rank != 0:
        return None
    dec_steps = (eng.stats["decode_steps"] - s0["decode_steps"]) // steps
    # bytes one decode step must read: every weight once + the live K/V of the running batch
    w_bytes = sum(p.numel() * p.element_size() for L in model.layers for p in (L.wqkv, L.wo, L.w13, L.w2)) \
        + model.output.numel() * model.output.element_size()
    tok_bytes = cfg.n_layers * cfg.n_kv_heads * cfg.head_dim * 2 * 2
    kv_read = sum(min(c, 64 * 16) for step_ctx in ctx_trace for c in step_ctx) * tok_bytes
    alg_bytes_run = w_bytes * len(ctx_trace) + kv_read
    hbm, kind = _peaks()
    achieved = alg_bytes_run / (dev_s / steps) / 1e9
    cpu = None if args.no_cpu_baseline else e2e_cpu_baseline(model)
    del eng._graphs
    return {
        "metric": f"e2e decode tok/s (config 4: TinyLlama-1.1B fp16, {n_req} requests x {max_tokens} greedy tokens)",
        "value": made / dev_s, "unit": "tok/s", "n_gpus": 1, "steps": steps, "warmup": 1,
        "ms_per_step": dev_s * 1e3 / steps, "higher_is_better": True, "scaling": "weak", "vs_baseline": None,
        "dtype": "f16", "data": "synthetic (random-init weights N(0,0.02), random prompt ids)",
        "config": {"workload": "config4 e2e engine, staggered arrivals (4 per step), max_batch 64, 4096 blocks",
                   "step": "one full run of the 64 requests (prefills included)",
                   "generated_tokens_per_step": made // steps, "engine_steps_per_run": len(ctx_trace),
                   "decode_steps_per_run": dec_steps, "cuda_graphs": True},
        "roofline": {"bound": "hbm", "achieved": achieved, "peak": hbm, "unit": "GB/s", "frac": achieved / hbm,
                     "peak_kind": kind,
                     "note": "(weights once per engine step + live K/V each decode step reads) / run time; "
                             "prefill FLOPs are not counted, so this is a lower bound on the HBM share"},
        "wall_ms_per_step": dt * 1e3 / steps,
        "engine_step_wall_ms": {k: {"count": len(v) // steps, "mean": 1e3 * statistics.mean(v) if v else None,
                                    "total_per_run": 1e3 * sum(v) / steps}
                                for k, v in step_wall.items()},
        "clocks": clk, "cpu_baseline": cpu,
        "gpu_launches": None,
        "note": "device events around whole engine runs, host scheduling included (every engine step "
                "synchronises); the engine mixes our kernels with cuBLAS GEMMs inside CUDA graphs",
    }


def engine5_line(args, rank: int, world: int, local_rank: int):
    """Config 5: random-init Llama-3-8B-shaped model in bf16; 512 sequences with
    contexts ~ U{512..8192} whose K/V is synthetic N(0,1) already in the pool,
    256 greedy tokens each, sharded by sequence over the ranks (least outstanding
    work first) with one int32 token all-gather per step over NCCL.  Each rank
    keeps resident as many of its sequences as its HBM holds (weights are
    replicated).  A step is one engine step (one decode iteration for every
    resident sequence on every rank); value = tokens produced by all ranks / s."""
    import numpy as np
    import torch
    import torch.distributed as dist
    from tinyvllm_b200.distributed import ShardedEngine
    from tinyvllm_b200.engine import LLMEngine, SamplingParams
    from tinyvllm_b200.model import Llama, llama3_8b_config

    dev = torch.device("cuda", local_rank)
    cfg = llama3_8b_config("bfloat16")
    model = Llama(cfg, device=dev, seed=1234 + 5)
    n_total, gen = 512, 256
    steps, warmup = args.engine_steps_c5, 3
    rng = np.random.default_rng(1239)
    ctx = rng.integers(512, 8193, size=n_total)
    first = rng.integers(0, cfg.vocab_size, size=n_total)
    prompts = [rng.integers(0, cfg.vocab_size, size=int(c)).tolist() for c in ctx]
    # replay the sharding (same rule as ShardedEngine) to size this rank's pool
    loads = [0] * world
    mine = []
    for i, c in enumerate(ctx):
        r = min(range(world), key=lambda x: (loads[x], x))
        loads[r] += int(c) + gen
        if r == rank:
            mine.append(i)
    steps_total = warmup + steps + 2
    tok_bytes = cfg.n_layers * cfg.n_kv_heads * cfg.head_dim * 2 * 2
    free, _ = torch.cuda.mem_get_info(dev)
    budget = free - (8 << 30)                     # activations, graphs, workspaces
    resident, blocks = 0, 0
    for i in mine:
        b = -(-(int(ctx[i]) + steps_total) // 16)
        if (blocks + b) * 16 * tok_bytes > budget:
            break
        resident += 1
        blocks += b
    width = -(-(int(ctx.max()) + steps_total) // 16)
    eng = LLMEngine(model, max_batch_size=resident, num_blocks=blocks + 8, num_scheduler_steps=1,
                    kv_order="reference", max_table_blocks=width, use_cuda_graphs=True)
    for t in eng.kv_cache.k_cache + eng.kv_cache.v_cache:
        t.normal_()                                # synthetic pre-filled K/V
    sharded = ShardedEngine(eng, rank, world, dev)
    for i in range(n_total):
        sharded.add_request(prompts[i], SamplingParams(max_tokens=gen), prefilled_first_token=int(first[i]))
    for _ in range(warmup):
        sharded.step()
    torch.cuda.synchronize(dev)
    dist.barrier(device_ids=[local_rank])
    clocks = ClockSampler(world) if rank == 0 else None
    if clocks:
        clocks.start()
        time.sleep(0.3)
    dist.barrier(device_ids=[local_rank])
    n0 = sum(len(r.tokens) for r in sharded.requests.values())
    x0 = sharded.exchange_seconds
    ev0, ev1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    t0 = time.perf_counter()
    ev0.record()
    for _ in range(steps):
        sharded.step()
    ev1.record()
    torch.cuda.synchronize(dev)
    wall = time.perf_counter() - t0
    dist.barrier(device_ids=[local_rank])
    clk = clocks.stop() if clocks else None
    made = sum(len(r.tokens) for r in sharded.requests.values()) - n0
    running = [s for s in eng.scheduler.running.values()]
    ctx_sum = sum(s.get_len() for s in running)
    xchg = sharded.exchange_seconds - x0
    stats = torch.tensor([ev0.elapsed_time(ev1) / 1e3, wall, resident, ctx_sum, xchg], dtype=torch.float64,
                         device=dev)
    allst = torch.empty(world * 5, dtype=torch.float64, device=dev)
    dist.all_gather_into_tensor(allst, stats)
    allst = allst.view(world, 5).cpu().numpy()
    del eng._graphs
    if rank != 0:
        return None
    secs = float(allst[:, 0].max())
    step_s = secs / steps
    w_bytes = sum(p.numel() * p.element_size() for L in model.layers for p in
                  (L.wqkv, L.wo, L.w13, L.w2)) + model.output.numel() * 2
    kv_bytes = float(allst[0, 3]) * tok_bytes
    hbm, kind = _peaks()
    achieved = (w_bytes + kv_bytes) / step_s / 1e9
    return {
        "metric": "e2e decode tok/s (config 5: Llama-3-8B shape bf16, 512 seqs ctx U[512,8192], "
                  "sequence-sharded)",
        "value": made / secs, "unit": "tok/s", "n_gpus": world, "steps": steps, "warmup": warmup,
        "ms_per_step": step_s * 1e3, "higher_is_better": True, "scaling": "strong", "vs_baseline": None,
        "dtype": "bf16", "data": "synthetic (random-init weights, synthetic N(0,1) pre-filled K/V)",
        "config": {"workload": "config5 sharded decode", "sequences": n_total,
                   "resident_per_rank": [int(x) for x in allst[:, 2]],
                   "ctx_sum_per_rank": [int(x) for x in allst[:, 3]],
                   "parallelism": f"sequence-sharded x{world}, int32 token all-gather per step (NCCL)"},
        "roofline": {"bound": "hbm", "achieved": achieved, "peak": hbm, "unit": "GB/s",
                     "frac": achieved / hbm, "peak_kind": kind,
                     "note": "rank 0: (weights + live K/V bytes per step) / step time"},
        "timing": "device events around the timed engine steps, max over ranks (every step synchronises "
                  "the host); wall clock max over ranks beside it",
        "wall_ms_per_step": float(allst[:, 1].max()) / steps * 1e3,
        "token_exchange_ms_per_step": float(allst[:, 4].max()) / steps * 1e3,
        "token_exchange_note": "host wall time per step in ShardedEngine's exchange: the record's copy to the "
                               "device, the NCCL all-gather and the copy back (max over ranks)",
        "clocks": clk,
    }


def _free_cuda():
    import gc
    import torch
    gc.collect()
    torch.cuda.empty_cache()


def run_ours(args, rank: int, world: int, local_rank: int) -> int:
    import torch
    import torch.distributed as dist
    torch.cuda.set_device(local_rank)
    dev = torch.device("cuda", local_rank)
    _init_group(rank, world, dev)
    line = decode_headline(args, rank, world, local_rank)
    _free_cuda()
    if not args.no_nested:
        nested = {}
        for key, fn in (("prefill", prefill_line), ("engine_config4", engine4_line),
                        ("engine_config5", engine5_line)):
            if key == "engine_config4" and world > 1:
                continue                           # config 4 is a one-GPU workload
            t0 = time.perf_counter()
            res = fn(args, rank, world, local_rank)
            _free_cuda()
            dist.barrier(device_ids=[local_rank])
            if rank == 0:
                res["wall_s"] = time.perf_counter() - t0
                nested[key] = res
        if rank == 0:
            line.update(nested)
    if rank == 0:
        print(json.dumps(line), flush=True)
    dist.barrier(device_ids=[local_rank])
    dist.destroy_process_group()
    return 0


def unit_probes_line(args, rank: int, world: int, local_rank: int):
    """The two on-chip rates that bound the prefill kernels, measured by the
    library's probes (tinyvllm_b200/csrc/probe_units.cu), one CTA per SM:
    cycles per tcgen05.mma issued back to back by one thread (M = 128, K = 16,
    N = 64 / 128 / 256) against the N-proportional ideal of 8,192 dense
    FLOP per clock per SM, and exponentials per clock per SM for each ex2 form and
    for the softmax's step per score pair.  Medians over CTAs; not a headline."""
    import numpy as np
    import torch
    from tinyvllm_b200 import _lib
    dev = torch.device("cuda", local_rank)
    lib = _lib.lib()
    n_sm = torch.cuda.get_device_properties(dev).multi_processor_count
    out = torch.zeros(2 * n_sm, dtype=torch.int64, device=dev)
    sink = torch.zeros(1, dtype=torch.int32, device=dev)
    stream = torch.cuda.current_stream(dev).cuda_stream
    mma = {}
    n_mma = 4096
    for n in (64, 128, 256):
        for _ in range(2):  # the first round warms up
            _lib.check(lib.tvk_probe_mma_issue(n, n_mma, out.data_ptr(), n_sm, stream), "tvk_probe_mma_issue")
        torch.cuda.synchronize(dev)
        c = out.view(n_sm, 2).cpu().numpy()
        if (c[:, 1] < 0).any():
            raise RuntimeError("an MMA probe CTA gave up waiting for completion")
        ideal = 128 * n * 16 * 2 / 8192.0  # cycles per MMA at 8,192 FLOP per clock per SM
        mma[f"n{n}"] = {"issue_cycles_per_mma": round(float(np.median(c[:, 0])) / n_mma, 1),
                        "complete_cycles_per_mma": round(float(np.median(c[:, 1])) / n_mma, 1),
                        "ideal_cycles_per_mma": ideal}
    forms = {0: ("ex2.approx.ftz.f32", 1), 1: ("ex2.approx.f16x2", 2), 2: ("ex2.approx.ftz.bf16x2", 2),
             3: ("softmax step per score pair (f32x2 fma, 2 ex2.f32, f32x2 add, f16x2 pack)", 2)}
    exp = {}
    n_iter = 2048
    for form, (name, per_op) in forms.items():
        for _ in range(2):
            _lib.check(lib.tvk_probe_exp_unit(form, n_iter, out.data_ptr(), n_sm, sink.data_ptr(), stream),
                       "tvk_probe_exp_unit")
        torch.cuda.synchronize(dev)
        cyc = float(np.median(out[:n_sm].cpu().numpy()))
        ops = n_iter * 8 * 512  # per SM
        exp[name] = {"exponentials_per_clock_per_sm": round(ops * per_op / cyc, 2)}
    return {"metric": "on-chip unit rates (probes)", "n_gpus": 1, "data": "synthetic (zero operands)",
            "config": {"workload": "unit-probes", "sms": n_sm, "mma_per_cta": n_mma, "exp_rounds": n_iter},
            "tcgen05_mma_one_issuer": mma, "exp_unit": exp}


def run_single(args, rank: int, world: int, local_rank: int, fn) -> int:
    import torch
    import torch.distributed as dist
    torch.cuda.set_device(local_rank)
    dev = torch.device("cuda", local_rank)
    _init_group(rank, world, dev)
    res = fn(args, rank, world, local_rank)
    if rank == 0:
        print(json.dumps(res), flush=True)
    dist.barrier(device_ids=[local_rank])
    dist.destroy_process_group()
    return 0


def main() -> int:
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=50)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--no-nested", action="store_true",
                    help="headline only: skip the nested prefill / engine configurations")
    ap.add_argument("--batch", type=int, default=256,
                    help="sequences per GPU (default 256 = config 3; smaller only for profiling captures)")
    ap.add_argument("--workload", choices=["decode", "prefill", "e2e", "e2e8b", "decode-engine-shape", "unit-probes"],
                    default="decode",
                    help="decode = config 3 headline (+ nested configurations); prefill = config 2 flash prefill; "
                         "e2e = config 4 TinyLlama engine; e2e8b = config 5 sharded Llama-3-8B-shape decode")
    ap.add_argument("--prefill-steps", type=int, default=20)
    ap.add_argument("--e2e-requests", type=int, default=64, help="config-4 requests (64 = the configuration)")
    ap.add_argument("--e2e-max-tokens", type=int, default=128, help="config-4 tokens per request (128 = the configuration)")
    ap.add_argument("--engine-steps", type=int, default=2, help="config-4 runs timed")
    ap.add_argument("--engine-steps-c5", type=int, default=20, help="config-5 engine steps timed")
    ap.add_argument("--prefill-lens", default=None,
                    help="prefill workload: comma-separated prompt lengths (default: config 2's eight prompts)")
    ap.add_argument("--prefill-head-dim", type=int, choices=[64, 128], default=64)
    ap.add_argument("--prefill-kv-heads", type=int, default=4, help="prefill workload: KV heads (32 query heads)")
    ap.add_argument("--prefill-dtype", choices=["fp16", "bf16"], default="fp16")
    ap.add_argument("--prefill-kernel", choices=["auto", "one-head", "paired"], default="auto",
                    help="prefill workload: which tcgen05 kernel (auto = paired where the heads per KV head are even)")
    args = ap.parse_args()
    rank = int(os.environ.get("RANK", "0"))
    world = int(os.environ.get("WORLD_SIZE", "1"))
    local_rank = int(os.environ.get("LOCAL_RANK", "0"))
    if args.warmup < 3:
        print("warning: fewer than 3 warm-up steps", file=sys.stderr)
    if args.impl == "reference":
        return run_reference(args, rank, world)
    if args.workload == "prefill":
        return run_single(args, rank, world, local_rank, prefill_line)
    if args.workload == "e2e":
        return run_single(args, rank, world, local_rank, engine4_line)
    if args.workload == "e2e8b":
        return run_single(args, rank, world, local_rank, engine5_line)
    if args.workload == "decode-engine-shape":
        return run_single(args, rank, world, local_rank, decode_engine_shape_line)
    if args.workload == "unit-probes":
        return run_single(args, rank, world, local_rank, unit_probes_line)
    return run_ours(args, rank, world, local_rank)


if __name__ == "__main__":
    sys.exit(main())
