/*
 * tvk.h -- C ABI of the B200 (sm_100a) attention hot path for tinyvllm.
 *
 * Every entry point takes raw device pointers that the caller owns, plain
 * integer sizes, a dtype code and a CUDA stream (as void*, 0 = legacy default
 * stream).  Nothing here allocates device memory except where stated; scratch
 * space is passed in by the caller.  All launches are stream-ordered and
 * asynchronous.  Return value: TVK_OK (0) or a negative TVK_ERR_* code; the
 * message for the last failure on the calling thread is tvk_last_error().
 *
 * Reference interfaces replaced (paths inside jonirajala/tinyvllm):
 *   tvk_paged_decode_attention  <- paged_decode_attention   tinyvllm/model/llama.py:97-144
 *   tvk_flash_prefill_attention <- flash_prefill_attention  tinyvllm/model/llama.py:58-94
 *                                  + Attention._write_kv_to_blocks llama.py:188-209 (fused)
 *   tvk_write_kv_slots          <- KVCache.write_kv          tinyvllm/core/kv_cache.py:34-38
 *                                  (decode append loop       tinyvllm/model/llama.py:381-386)
 */
#ifndef TVK_H_
#define TVK_H_

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* dtype codes (the reference supports float32 and float16: model/weights.py:44) */
#define TVK_DTYPE_F32 0
#define TVK_DTYPE_F16 1
#define TVK_DTYPE_BF16 2

/* status codes */
#define TVK_OK 0
#define TVK_ERR_INVALID (-1)     /* bad pointer, shape or size                     */
#define TVK_ERR_UNSUPPORTED (-2) /* valid call, but no kernel for this shape/dtype */
#define TVK_ERR_CUDA (-3)        /* a CUDA runtime call or launch failed           */
#define TVK_ERR_WORKSPACE (-4)   /* workspace missing or too small                 */

/* ABI version of this header (bumped on any signature change). */
int tvk_abi_version(void);

/* Message of the last failed call on this thread ("" if none). */
const char* tvk_last_error(void);

/*
 * Bytes of scratch that tvk_paged_decode_attention needs for a batch whose
 * block tables are `max_blocks` wide: a 256-byte header (a device status word
 * at byte 0, work-list counters at bytes 64 and 128, the unit size of the last
 * call at byte 192) followed by the split-K partials (fp32 output rows plus
 * max / sum pairs).  Zero the header once after allocating the workspace;
 * every call returns the status word and the counters to zero unless a
 * kernel wait timed out.  One workspace serves one stream at a time.
 * Replaces nothing in the reference (tinygrad allocates its temporaries).
 */
size_t tvk_paged_decode_workspace_size(int batch, int n_heads, int n_kv_heads, int head_dim,
                                       int block_size, int max_blocks, int max_context_len);

/*
 * How tvk_paged_decode_attention cuts and launches a call with these sizes
 * (nothing is launched here).  plan_out[0] = the smallest unit of context
 * tokens (one unit = one split of one (sequence, KV head)); plan_out[1] = the
 * most splits a sequence may take; plan_out[2] = kernel launches per call
 * (2 when a split-K combine follows); plan_out[3] = 1 when persistent CTAs
 * take units from the workspace's ticket counter and size them from the live
 * contexts (units then hold at least plan_out[0] tokens), 0 when every unit
 * gets its own CTA.  No counterpart in the reference.
 */
int tvk_paged_decode_plan(int batch, int n_heads, int n_kv_heads, int head_dim, int block_size,
                          int max_blocks, int max_context_len, int dtype, int* plan_out);

/*
 * Paged-decode attention, one query token per sequence.
 * Replaces paged_decode_attention (tinyvllm/model/llama.py:97-144).
 *
 *   q            [batch, 1, n_heads, head_dim]               dtype
 *   k_cache      [num_blocks, block_size, n_kv_heads, head_dim] dtype (one layer)
 *   v_cache      same shape as k_cache
 *   block_tables int32 [batch, max_blocks], padded with any valid id (the
 *                reference pads with block 0)
 *   context_lens int32 [batch]
 *   out          [batch, 1, n_heads, head_dim]               dtype
 *   max_context_len  < 0 means "None" (attend over max_blocks*block_size
 *                positions masked by context_lens, llama.py:113-118)
 *
 * out[b,0,h,:] = softmax_t(q[b,h].K[b,t,h/g] / sqrt(head_dim)) . V[b,t,h/g]
 * over t < min(context_lens[b], table width), with g = n_heads / n_kv_heads and
 * K[b,t] = k_cache[block_tables[b, t / block_size], t % block_size].
 * A sequence with context_lens[b] <= 0 gets zeros (the reference's output is
 * then a uniform average over the padded positions; the engine never does this).
 * Block ids outside [0, num_blocks) read as zeros.
 * Softmax and accumulation are float32 for every storage dtype.
 */
int tvk_paged_decode_attention(const void* q, const void* k_cache, const void* v_cache,
                               const int32_t* block_tables, const int32_t* context_lens,
                               void* out,
                               int batch, int n_heads, int n_kv_heads, int head_dim,
                               int block_size, int num_blocks, int max_blocks,
                               int max_context_len, int dtype,
                               void* workspace, size_t workspace_bytes, void* stream);

/*
 * Causal (or full) prefill attention over a ragged batch of prompts, with the
 * prompt K/V written into the paged pool by the same kernel.
 * Replaces flash_prefill_attention (tinyvllm/model/llama.py:58-94) and the
 * block-chunked writes of Attention._write_kv_to_blocks (llama.py:188-209,
 * core/kv_cache.py:34-38).  The reference handles one prompt per call
 * (inputs [1, L, H, D]); n_seqs == 1 is that case.
 *
 *   q    [total_tokens, n_heads, head_dim]      prompts packed along tokens
 *   k, v [total_tokens, n_kv_heads, head_dim]   (post-RoPE k, as the reference writes)
 *   out  [total_tokens, n_heads, head_dim]
 *   cu_seqlens int32 [n_seqs + 1] on the device: prompt s is tokens
 *              [cu_seqlens[s], cu_seqlens[s+1]); max_seqlen >= every length
 *   causal     key j is visible to query i iff j <= i (else all keys of the prompt)
 *   slot_mapping int64 [total_tokens] or NULL: when given, token t's k/v rows are
 *              also stored at k_cache/v_cache [num_blocks, block_size, n_kv_heads,
 *              head_dim] flat slot slot_mapping[t] (= block * block_size + offset);
 *              negative or out-of-pool slots are skipped.
 *   workspace  >= tvk_flash_prefill_workspace_size(n_seqs, total_tokens) bytes for the
 *              tcgen05 path (its work schedule lives there; optional otherwise); its
 *              first int is set non-zero if a bounded wait expired.
 * fp16/bf16 with head_dim 64 or 128 run on tcgen05 (TMEM accumulators, TMA
 * loads, persistent CTAs over a heaviest-first tile schedule built on the
 * device; see tvk_prefill_select_kernel); fp32 and head_dim 32 use a CUDA-core
 * kernel.  Softmax is fp32.
 */
size_t tvk_flash_prefill_workspace_size(int n_seqs, int total_tokens);

/*
 * Selects the tensor-core prefill kernel for later tvk_flash_prefill_attention
 * calls on the calling thread: 0 (default) = automatic -- the paired-head kernel
 * (two query heads that share a KV head per CTA item, one CTA per SM) whenever
 * n_heads / n_kv_heads is even, else the one-head kernel; 1 = always the
 * one-head kernel; 2, 3, 4 = the paired kernel (where it applies) computing
 * 0, 2/8 or 3/8 of the softmax exponentials with a polynomial on the FMA pipe
 * instead of the exponential unit.  All compute the same function to within
 * one 16-bit rounding of P; this exists so tests and timings can run each.
 * No counterpart in the reference.
 */
int tvk_prefill_select_kernel(int choice);
int tvk_flash_prefill_attention(const void* q, const void* k, const void* v, void* out,
                                const int32_t* cu_seqlens, int n_seqs, int max_seqlen, int total_tokens,
                                int n_heads, int n_kv_heads, int head_dim, int causal, int dtype,
                                const int64_t* slot_mapping, void* k_cache, void* v_cache,
                                int num_blocks, int block_size,
                                void* workspace, size_t workspace_bytes, void* stream);

/* ------------------------------------------------------------------------
 * Per-layer ops around the attention (fp32 arithmetic, one rounding to dtype;
 * pointers 16-byte aligned, contiguous rows unless a stride is given).
 * ------------------------------------------------------------------------ */

/*
 * RMSNorm, RMSNorm.__call__ (tinyvllm/model/llama.py:21-23):
 *   out = s * rsqrt(mean(s^2) + eps) * weight,  s = x            (residual == NULL)
 *                                               s = x + residual (rounded to dtype; also
 *                                               stored to residual_out -- the residual add of
 *                                               TransformerBlock.__call__, llama.py:247-250)
 * x, residual, residual_out, out [rows, dim]; weight [dim].  dim <= 2048 * (16 / sizeof(dtype)).
 */
int tvk_rms_norm(const void* x, const void* residual, void* residual_out, const void* weight, void* out,
                 int rows, int dim, float eps, int dtype, void* stream);

/*
 * tvk_rms_norm plus the decode K/V append of one token per row, in one launch:
 * row r's k and v rows ([rows, n_kv_heads, head_dim]) are stored at flat slot
 * slots[r] of k_cache / v_cache [num_blocks, block_size, n_kv_heads, head_dim]
 * (negative or out-of-pool slots skipped).  Replaces the post-attention write
 * of Llama.decode (tinyvllm/model/llama.py:381-386) when the norm after the
 * attention output projection is the next kernel, so the attention still reads
 * the slot's previous contents as the reference does.
 */
int tvk_rms_norm_write_kv(const void* x, const void* residual, void* residual_out, const void* weight, void* out,
                          int rows, int dim, float eps, const void* k, const void* v, const int64_t* slots,
                          void* k_cache, void* v_cache, int n_kv_heads, int head_dim, int num_blocks,
                          int block_size, int dtype, void* stream);

/*
 * In-place interleaved-pair RoPE on q [n_tokens, n_heads, head_dim] and
 * k [n_tokens, n_kv_heads, head_dim], apply_rope (llama.py:34-55):
 *   (x[2i], x[2i+1]) -> (x0 c - x1 s, x0 s + x1 c),  c/s = table[positions[t], i]
 * cos_table / sin_table fp32 [max_pos, head_dim / 2] (precompute_freqs_cis, llama.py:26-31).
 */
int tvk_rope(void* q, void* k, const float* cos_table, const float* sin_table, const int32_t* positions,
             int n_tokens, int n_heads, int n_kv_heads, int head_dim, int max_pos, int dtype, void* stream);

/*
 * tvk_rope, then the roped k rows and the v rows [n_tokens, n_kv_heads, head_dim]
 * stored into k_cache / v_cache [num_blocks, block_size, n_kv_heads, head_dim] at
 * flat slot slots[t] (negative or out-of-pool slots skipped): RoPE fused with the
 * K/V write of llama.py:322-323 + 381-386 / 188-209.
 */
int tvk_rope_write_kv(void* q, void* k, const void* v, const float* cos_table, const float* sin_table,
                      const int32_t* positions, const int64_t* slots, void* k_cache, void* v_cache,
                      int n_tokens, int n_heads, int n_kv_heads, int head_dim, int max_pos,
                      int num_blocks, int block_size, int dtype, void* stream);

/*
 * Split one packed projection row per token, qkv[t] = [q (n_heads*head_dim) |
 * k (n_kv_heads*head_dim) | v (n_kv_heads*head_dim)] with row stride `row_stride`
 * elements (the output of one GEMM against the concatenated wq|wk|wv,
 * llama.py:174-176), into contiguous q [n_tokens, n_heads, head_dim] and k, v
 * [n_tokens, n_kv_heads, head_dim], applying RoPE to q and k as tvk_rope does
 * (llama.py:178-179).  With slots != NULL the roped k and the v rows are also
 * stored at their paged slots like tvk_rope_write_kv (k_cache/v_cache and the
 * pool sizes are ignored otherwise).
 */
int tvk_qkv_rope(const void* qkv, long long row_stride, void* q, void* k, void* v, const float* cos_table,
                 const float* sin_table, const int32_t* positions, const int64_t* slots, void* k_cache,
                 void* v_cache, int n_tokens, int n_heads, int n_kv_heads, int head_dim, int max_pos,
                 int num_blocks, int block_size, int dtype, void* stream);

/*
 * k/v rows [n_tokens, n_kv_heads, head_dim] -> paged slots, KVCache.write_kv
 * (core/kv_cache.py:34-38); one launch for a whole decode batch replaces the
 * reference's per-sequence, per-layer writes (llama.py:381-386).
 */
int tvk_write_kv_slots(const void* k, const void* v, const int64_t* slots, void* k_cache, void* v_cache,
                       int n_tokens, int n_kv_heads, int head_dim, int num_blocks, int block_size,
                       int dtype, void* stream);

/*
 * SwiGLU gate of FeedForward.__call__ (llama.py:220-221):
 *   out[r, c] = silu(a[r, c]) * b[r, c]   (silu rounded to dtype before the product)
 * Row strides in elements (a packed gate|up GEMM output: a = base, b = base + cols,
 * a_stride = b_stride = 2 * cols).
 */
int tvk_silu_mul(const void* a, const void* b, void* out, int rows, int cols, long long a_stride,
                 long long b_stride, long long out_stride, int dtype, void* stream);

/*
 * Embedding row gather (llama.py:276,310): out[t] = table[tokens[t]].  Ids outside
 * [0, vocab) give zero rows and set *status = 3 (status may be NULL).
 */
int tvk_embedding(const void* table, const int32_t* tokens, void* out, int n_tokens, int dim, int vocab,
                  int dtype, int* status, void* stream);

/*
 * Greedy pick (core/sampling.py:133-134): out[r] = argmax over logits[r, :vocab],
 * first index on ties, compared in fp32 after conversion from dtype.
 */
int tvk_argmax(const void* logits, int32_t* out, int rows, int vocab, long long row_stride, int dtype,
               void* stream);

/*
 * Paged-decode attention that allocates nothing (no counterpart in the
 * reference, which lets tinygrad allocate its temporaries).
 *
 * Same arguments and result as tvk_paged_decode_attention, minus the
 * workspace: the split-K scratch is a fixed 64 MiB array compiled into this
 * library (TVK_NOALLOC_SCRATCH_BYTES), held by every GPU that loads the
 * library until the process exits.  It is for callers that cannot allocate
 * device memory: an engine that gives (nearly) all free HBM to its KV pool at
 * start-up, a host binding without a device allocator of its own, or a decode
 * loop that cannot take cudaMalloc's device-wide synchronisation.
 *
 * A call whose scratch need (tvk_paged_decode_workspace_size) exceeds the
 * array returns TVK_ERR_WORKSPACE without launching anything.  No cudaMalloc,
 * cudaFree or other allocating routine is called.  The first call on each
 * device looks the array's device address up (cudaGetSymbolAddress, with that
 * device current); make that first call before any stream capture.  Every
 * call shares the one array and the array keeps the last call's contents:
 * calls whose kernels overlap on the GPU (different streams, or different
 * threads) race on it and must be serialised by the caller.
 */
#define TVK_NOALLOC_SCRATCH_BYTES (64ull << 20)
int tvk_paged_decode_attention_noalloc(const void* q, const void* k_cache, const void* v_cache,
                                       const int32_t* block_tables, const int32_t* context_lens,
                                       void* out,
                                       int batch, int n_heads, int n_kv_heads, int head_dim,
                                       int block_size, int num_blocks, int max_blocks,
                                       int max_context_len, int dtype, void* stream);

/*
 * Status word of the no-allocation entry point on the current device: waits
 * for `stream`, then stores the word at *status (host memory).  0 = the last
 * tvk_paged_decode_attention_noalloc call on this device completed; non-zero =
 * a bounded wait inside its kernel gave up (after 2 s) and its output is
 * incomplete.  The next no-allocation call on the device clears the word.
 * Allocates nothing.  No counterpart in the reference (tinygrad raises on the host).
 */
int tvk_paged_decode_noalloc_status(int* status, void* stream);

/*
 * Test hook for the kernels' bounded waits (no counterpart in the reference).
 * Arms the next tvk_paged_decode_attention / tvk_flash_prefill_attention call
 * made on the calling thread that reaches a tensor-core kernel (fp16/bf16):
 * that launch gets `limit_ns` (1e5 .. 2e9) as the wall-time limit of its
 * mbarrier waits, and its producer warp issues no loads, so the consumers'
 * first wait runs out.  The kernel then sets the workspace status word to 1
 * and returns; nothing faults, traps or hangs.  The caller must zero the
 * workspace header (256 bytes) before the next call.  One-shot: the arming is
 * consumed by the next decode or prefill call on the thread that passes its
 * argument checks (an fp32 call consumes it without effect).
 */
int tvk_debug_arm_wait_timeout(long long limit_ns);

/*
 * Tensor-core layout self-test (no reference counterpart): one 128 x n x k
 * tcgen05 GEMM through the operand paths the prefill kernel uses (A written
 * swizzled into shared memory by threads, or into TMEM with tcgen05.st when
 * a_in_tmem != 0; TMA-loaded B; TMEM accumulator).
 *   b_mn_major == 0: c[128,n] = a[128,k] . b[n,k]^T
 *   b_mn_major == 1: c[128,n] = a[128,k] . b[k,n]
 * n, k in {64, 128}; dtype TVK_DTYPE_F16 or TVK_DTYPE_BF16; c is fp32.
 * `status` (device int, may be NULL) is set to 1 if a bounded wait expired.
 */
int tvk_selftest_umma_gemm(const void* a, const void* b, float* c, int n, int k, int b_mn_major,
                           int a_in_tmem, int dtype, int* status, void* stream);

/*
 * Measurement probes (no reference counterpart; nothing on the attention path
 * uses them).  One CTA per SM for n_ctas CTAs (use the SM count), cycles from
 * clock64, written to device memory `out`:
 *   tvk_probe_mma_issue: one thread issues n_mma tcgen05.mma.cta_group::1
 *     kind::f16 (M = 128, N = n in {64, 128, 256}, K = 16, zero bf16 operands
 *     in shared memory) back to back; out[2c] = cycles of CTA c's issue loop,
 *     out[2c + 1] = cycles until the last MMA completed (-1: wait gave up).
 *   tvk_probe_exp_unit: 16 warps per SM run 8 dependent chains each per thread
 *     for n_iter rounds of one form -- 0 ex2.approx.ftz.f32, 1 ex2.approx.f16x2,
 *     2 ex2.approx.ftz.bf16x2, 3 the prefill softmax step per score pair (f32x2
 *     FMA, two f32 ex2, f32x2 add, f16x2 pack); out[c] = cycles.  `sink` is a
 *     4-byte device scratch word.
 */
int tvk_probe_mma_issue(int n, int n_mma, long long* out, int n_ctas, void* stream);
int tvk_probe_exp_unit(int form, int n_iter, long long* out, int n_ctas, void* sink, void* stream);

#ifdef __cplusplus
}
#endif

#endif /* TVK_H_ */
