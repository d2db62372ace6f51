"""End-to-end engine on the kernels vs the CPU oracle engine: identical greedy
token streams (GPU).

The oracle (``oracle/engine.py``) replays the reference's step order exactly:
one prompt per prefill with chunked K/V writes, decode attention over the cache
before the step's own K/V is written, tables padded to 64 blocks with block 0,
LIFO block reuse after sequences finish.  A tight pool forces reuse, so stale
K/V in reused blocks is read exactly as the reference reads it.
"""

import numpy as np
import pytest
import torch

from oracle.engine import OracleEngine, OracleLlama

pytestmark = pytest.mark.gpu


def _requests(seed, n, vocab, len_lo, len_hi, tok_lo, tok_hi):
    rng = np.random.default_rng(seed)
    prompts = [rng.integers(0, vocab, size=int(rng.integers(len_lo, len_hi + 1))).tolist() for _ in range(n)]
    max_toks = rng.integers(tok_lo, tok_hi + 1, size=n).tolist()
    return prompts, max_toks


def _run_product(model, prompts, max_toks, **kw):
    from tinyvllm_b200.engine import LLMEngine, SamplingParams
    eng = LLMEngine(model, **kw)
    outs, i = {}, 0
    while i < len(prompts) or eng.has_unfinished():
        for _ in range(2):                 # staggered arrivals: two new requests per step
            if i < len(prompts):
                eng.add_request(prompts[i], SamplingParams(temperature=0.0, max_tokens=max_toks[i]))
                i += 1
        for o in eng.step():
            outs[o.request_id] = o.tokens
    return outs, eng


def _run_oracle(model, prompts, max_toks, max_batch_size, num_blocks, num_scheduler_steps=1, with_gaps=False):
    c = model.config
    om = OracleLlama(model.numpy_weights(), c.n_layers, c.n_heads, c.n_kv_heads, c.head_dim, c.norm_eps,
                     c.rope_theta, c.max_seq_len)
    eng = OracleEngine(om, max_batch_size, num_blocks, 16, num_scheduler_steps)
    i = 0
    while i < len(prompts) or eng.has_unfinished():
        for _ in range(2):
            if i < len(prompts):
                eng.add_request(prompts[i], max_toks[i])
                i += 1
        eng.step()
    return (eng.outputs, eng.gaps) if with_gaps else eng.outputs


def _tiny(dtype, dim, heads, kv_heads, seed=0, max_seq_len=256, init_std=0.25):
    from tinyvllm_b200.model import Llama, LlamaConfig
    cfg = LlamaConfig(dim=dim, n_layers=2, n_heads=heads, n_kv_heads=kv_heads, vocab_size=97, hidden_dim=2 * dim,
                      max_seq_len=max_seq_len, dtype=dtype)
    # std 0.25 keeps the logits spread wide enough that fp32 rounding cannot flip the argmax
    return Llama(cfg, device="cuda", seed=seed, init_std=init_std)


@pytest.mark.parametrize("graphs", [False, True])
@pytest.mark.parametrize("steps", [1, 3])
def test_greedy_streams_match_oracle_fp32(cuda, steps, graphs):
    model = _tiny("float32", 128, 4, 2)
    prompts, max_toks = _requests(1, 7, 97, 3, 40, 5, 25)
    got, eng = _run_product(model, prompts, max_toks, max_batch_size=4, num_blocks=24, num_scheduler_steps=steps,
                            use_cuda_graphs=graphs)
    exp = _run_oracle(model, prompts, max_toks, 4, 24, steps)
    assert got == exp
    assert eng.block_manager.get_num_free_blocks() == 24


def _teacher_forced(model, prompts, max_toks, max_batch_size, num_blocks, frac):
    """Run the oracle engine free, then the product engine fed the oracle's tokens.
    Every logit row the product produces must lie within ``frac`` times the row's
    standard deviation of the oracle's row, and its own argmax must equal the
    oracle's token wherever the oracle's top-1/top-2 margin exceeds twice that
    bound.  Returns (rows whose argmax was checked, largest error / std seen)."""
    from tinyvllm_b200.engine import LLMEngine, SamplingParams
    c = model.config
    om = OracleLlama(model.numpy_weights(), c.n_layers, c.n_heads, c.n_kv_heads, c.head_dim, c.norm_eps,
                     c.rope_theta, c.max_seq_len)
    oe = OracleEngine(om, max_batch_size, num_blocks)
    i = 0
    while i < len(prompts) or oe.has_unfinished():
        for _ in range(2):
            if i < len(prompts):
                oe.add_request(prompts[i], max_toks[i])
                i += 1
        oe.step()
    exp, gaps, oracle_logits = oe.outputs, oe.gaps, oe.logits
    del om, oe

    recorded = {}

    class Forced(LLMEngine):
        def _sample(self, logits, seqs):
            rows = logits.float().cpu().numpy()
            out = []
            for s, row in zip(seqs, rows):
                k = len(s.output_tokens)
                recorded.setdefault(s.request_id, []).append(row)
                out.append(exp[s.request_id][k])
            return out

    eng = Forced(model, max_batch_size=max_batch_size, num_blocks=num_blocks)
    i = 0
    while i < len(prompts) or eng.has_unfinished():
        for _ in range(2):
            if i < len(prompts):
                eng.add_request(prompts[i], SamplingParams(max_tokens=max_toks[i]))
                i += 1
        eng.step()
    n_checked, worst = 0, 0.0
    for rid in exp:
        got_rows, exp_rows = recorded[rid], oracle_logits[rid]
        assert len(got_rows) == len(exp_rows)
        for k, (g, e) in enumerate(zip(got_rows, exp_rows)):
            std = float(np.std(e))
            tol = frac * std
            err = float(np.abs(g - e).max())
            worst = max(worst, err / std)
            assert err <= tol, f"request {rid} token {k}: logits off by {err} > {tol}"
            if gaps[rid][k] > 2 * tol:
                assert int(np.argmax(g)) == exp[rid][k]
                n_checked += 1
    return n_checked, worst


@pytest.mark.parametrize("dtype,frac", [("float16", 0.05), ("bfloat16", 0.2)])
def test_half_precision_engine_tracks_oracle(cuda, dtype, frac):
    """head_dim 64 in fp16 / bf16 runs the TMA/mma decode kernel and the tcgen05 prefill
    kernel.  Half-precision activations move the logits against the fp32 oracle by a
    few percent of their spread (more for bf16's 8-bit mantissa), enough to flip
    near-ties, so the streams are teacher-forced (``_teacher_forced``).  Block reuse
    is on (a tight pool), as in the fp32 stream test.
    """
    model = _tiny(dtype, 256, 4, 2, seed=3, init_std=0.1)
    prompts, max_toks = _requests(2, 6, 97, 3, 150, 4, 16)
    n_checked, _ = _teacher_forced(model, prompts, max_toks, 3, 40, frac)
    assert n_checked > 0


# Config 4's model (TinyLlama-1.1B shape: 22 layers, dim 2048, hidden 5632, 32/4
# heads, head_dim 64, vocab 32000, RoPE theta 1e4, weights N(0, 0.02), RMSNorm
# weights 1) at a short horizon the CPU oracle finishes in seconds: 8 requests
# with 24-180 random prompt ids, 16 greedy tokens each, two arrivals per step,
# max_batch_size 4 and a pool so tight that later requests reuse freed blocks.
def _config4_model(dtype):
    from tinyvllm_b200.model import Llama, tinyllama_config
    return Llama(tinyllama_config(dtype), device="cuda", seed=1234 + 4)


def test_config4_shape_fp32_greedy_streams_identical(cuda):
    """fp32: greedy token streams identical to the oracle engine (a restatement of
    engine.py:114-196 over llama.py:266-388), decode steps replayed as CUDA graphs."""
    model = _config4_model("float32")
    prompts, max_toks = _requests(1238, 8, 32000, 24, 180, 16, 16)
    got, eng = _run_product(model, prompts, max_toks, max_batch_size=4, num_blocks=56, use_cuda_graphs=True)
    exp = _run_oracle(model, prompts, max_toks, 4, 56)
    assert got == exp
    assert eng.block_manager.get_num_free_blocks() == 56


def test_config4_shape_fp16_tracks_oracle(cuda):
    """fp16 (the config's dtype), which runs the tcgen05 prefill and the TMA decode
    kernels: teacher-forced against the fp32 oracle, every logit within 10 % of the
    row's standard deviation, argmax equal wherever the oracle's margin is wider
    than twice that."""
    model = _config4_model("float16")
    prompts, max_toks = _requests(1239, 8, 32000, 24, 180, 16, 16)
    n_checked, worst = _teacher_forced(model, prompts, max_toks, 4, 56, 0.10)
    print(f"config-4 fp16: worst logit error {worst:.4f} of the row std, {n_checked} argmaxes checked")
    assert n_checked >= 32


def test_context_beyond_64_blocks_is_truncated_like_the_reference(cuda):
    """Decode tables are cut at 64 blocks (1024 tokens) in the reference engine."""
    model = _tiny("float32", 128, 4, 2, seed=4, max_seq_len=1024)
    prompts = [np.random.default_rng(5).integers(0, 97, size=1030).tolist()]
    got, _ = _run_product(model, prompts, [6], max_batch_size=1, num_blocks=80)
    exp = _run_oracle(model, prompts, [6], 1, 80)
    assert got == exp


def test_append_first_mode_sees_its_own_key(cuda):
    """append_first differs from the reference ordering only in what the new query sees."""
    from tinyvllm_b200.engine import LLMEngine, SamplingParams
    model = _tiny("float32", 128, 4, 2, seed=6)
    prompts, max_toks = _requests(7, 3, 97, 5, 30, 8, 8)
    a, _ = _run_product(model, prompts, max_toks, max_batch_size=3, num_blocks=20, kv_order="append_first")
    r, _ = _run_product(model, prompts, max_toks, max_batch_size=3, num_blocks=20)
    assert set(a) == set(r) and all(len(a[k]) == len(r[k]) for k in a)
    assert all(a[k][0] == r[k][0] for k in a)   # the prefill token does not depend on the decode order


def test_engine_api(cuda):
    from tinyvllm_b200.engine import LLMEngine, SamplingParams, TokenIdTokenizer, generate_batch
    model = _tiny("float32", 128, 4, 2, seed=8)
    eng = LLMEngine(model, max_batch_size=2, num_blocks=16)
    with pytest.raises(ValueError, match="greedy"):
        eng.add_request([1, 2, 3], SamplingParams(temperature=1.0))
    rid = eng.add_request([1, 2, 3], SamplingParams(max_tokens=4))
    with pytest.raises(ValueError, match="already exists"):
        eng.add_request([4], request_id=rid)
    eng.add_request([5, 6], SamplingParams(max_tokens=4))
    eng.add_request([7, 8, 9], SamplingParams(max_tokens=4))
    assert eng.abort_request(2) is True and eng.abort_request(99) is False
    outs = list(eng.run())
    assert sorted(o.request_id for o in outs) == [0, 1]
    assert all(len(o.tokens) == 4 and o.finish_reason == "length" for o in outs)
    assert eng.block_manager.get_num_free_blocks() == 16
    texts = generate_batch(LLMEngine(model, max_batch_size=4, num_blocks=16), [[1, 2], [3, 4, 5]],
                           SamplingParams(max_tokens=3))
    assert len(texts) == 2 and all(len(t.split()) == 3 for t in texts)
    # eos stops a stream early
    first = LLMEngine(model, max_batch_size=1, num_blocks=16)
    first.add_request([1, 2, 3], SamplingParams(max_tokens=5))
    tok0 = list(first.run())[0].tokens[0]
    e2 = LLMEngine(model, TokenIdTokenizer(eos_id=tok0), max_batch_size=1, num_blocks=16)
    e2.add_request([1, 2, 3], SamplingParams(max_tokens=5))
    out = list(e2.run())[0]
    assert out.tokens == [tok0] and out.finish_reason == "eos"


def test_out_of_blocks_raises_the_reference_error(cuda):
    from tinyvllm_b200.engine import LLMEngine, SamplingParams
    model = _tiny("float32", 128, 4, 2, seed=9)
    eng = LLMEngine(model, max_batch_size=2, num_blocks=2)
    eng.add_request(list(range(40)), SamplingParams(max_tokens=2))
    with pytest.raises(RuntimeError, match="Out of KV cache memory!"):
        eng.step()


@pytest.mark.parametrize("dtype", ["float32", "float16"])
def test_prefill_graph_matches_eager_prefill(cuda, dtype):
    """A prefill replayed as a CUDA graph over a padded token buffer samples the same
    first tokens as the eager ragged prefill and writes the same K/V into the same
    slots; the padding prompt and the capture-time runs write nothing."""
    from tinyvllm_b200 import layers
    from tinyvllm_b200.model import KVCache
    model = _tiny(dtype, 256, 4, 2, seed=5)
    c = model.config
    rng = np.random.default_rng(9)
    lens = [37, 1, 130]
    toks = rng.integers(0, c.vocab_size, size=sum(lens)).astype(np.int32)
    pos = np.concatenate([np.arange(L, dtype=np.int32) for L in lens])
    nb = 64
    perm = rng.permutation(nb)[:sum(-(-L // 16) for L in lens)]
    slots, b = [], 0
    for L in lens:
        blocks = perm[b:b + -(-L // 16)]
        b += len(blocks)
        slots.extend(int(blocks[t // 16]) * 16 + t % 16 for t in range(L))
    slots = np.asarray(slots, dtype=np.int64)
    cu = np.concatenate([[0], np.cumsum(lens)]).astype(np.int32)
    kv_e = KVCache(c.n_layers, nb, 16, c.n_kv_heads, c.head_dim, c.torch_dtype, cuda)
    logits = model.prefill(torch.from_numpy(toks).to(cuda), torch.from_numpy(pos).to(cuda),
                           torch.from_numpy(cu).to(cuda), max(lens), torch.from_numpy(slots).to(cuda), kv_e)
    eager = layers.greedy_argmax(logits).cpu().numpy()
    kv_g = KVCache(c.n_layers, nb, 16, c.n_kv_heads, c.head_dim, c.torch_dtype, cuda)
    graph = model.capture_prefill(len(lens), 256, kv_g)
    for t in kv_g.k_cache + kv_g.v_cache:
        assert not t.any()
    got = graph.run(toks, pos, lens, slots)
    got2 = graph.run(toks, pos, lens, slots)
    torch.cuda.synchronize()
    assert np.array_equal(got, eager) and np.array_equal(got2, eager)
    tol = 1e-4 if dtype == "float32" else 2e-2
    used = torch.zeros(nb * 16, dtype=torch.bool, device=cuda)
    used[torch.from_numpy(slots).to(cuda)] = True
    for a, e in zip(kv_g.k_cache + kv_g.v_cache, kv_e.k_cache + kv_e.v_cache):
        assert ((a.float() - e.float()).abs() <= tol * (1 + e.float().abs())).all()
        assert not a.view(nb * 16, -1)[~used].any()
    with pytest.raises(ValueError):
        graph.run(toks, pos, lens[:2], slots)


def test_prefill_graph_cap_runs_further_shapes_eagerly(cuda, monkeypatch):
    """Past its cap of prefill graphs an engine runs prefill steps of new shapes
    eagerly; the streams stay those of an engine without the cap."""
    from tinyvllm_b200 import engine as E
    model = _tiny("float32", 128, 4, 2, seed=3)
    prompts, max_toks = _requests(17, 6, 97, 5, 60, 3, 6)
    ref, _ = _run_product(model, prompts, max_toks, max_batch_size=4, num_blocks=64, use_cuda_graphs=True)
    monkeypatch.setattr(E, "_MAX_PREFILL_GRAPHS", 1)
    got, eng = _run_product(model, prompts, max_toks, max_batch_size=4, num_blocks=64, use_cuda_graphs=True)
    assert len(eng._prefill_graphs) == 1
    assert got == ref
