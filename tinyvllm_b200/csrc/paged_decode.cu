// paged_decode.cu -- paged-decode attention for sm_100a.
//
// Replaces paged_decode_attention (tinyvllm/model/llama.py:97-144).  The
// reference gathers every table entry into a dense [B, maxctx, Hkv, D] copy,
// materialises the GQA expand and runs two batched matmuls over the padded
// length.  Here the work is cut into units of one (sequence, KV head, context
// split); a unit reads only the blocks that hold live tokens, once, for all
// n_heads/n_kv_heads query heads that share that KV head.
//
// Two kernels:
//  * tc  (fp16 / bf16, block_size in {8,16,32,64}, head_dim in {32,64,128}):
//    persistent CTAs, about two per SM, take units from an atomic counter.
//    One producer warp issues 4-D TMA loads of whole K/V blocks (one KV head,
//    all block_size rows, swizzled) into a multi-stage shared-memory ring
//    guarded by mbarriers that runs on across unit boundaries; four consumer
//    warps each take 16 tokens of a stage and run Q.K^T and P.V on the tensor
//    cores (m16n8k16, fp32 accumulate) with the GQA group as the M dimension,
//    and an fp32 online softmax in registers.
//  * simt (any dtype incl. fp32, any block size): one CTA per unit,
//    cooperative vector loads of 32-token tiles into shared memory and fp32
//    CUDA-core math.
// Sequences longer than one split are reduced by a small combine kernel from
// fp32 partials (max, sum, unnormalised output) kept in the caller workspace.
#include <math.h>

#include <mutex>

#include "tvk_common.cuh"

namespace {

constexpr int kStageTok = 64;  // tokens per pipeline stage / split granularity
constexpr int kSimtTile = 32;  // tokens per tile in the simt kernel
constexpr int kMaxGroup = 16;  // query heads per KV head (MMA M dimension)

struct DecodeParams {
  const void* q;
  void* out;
  const int32_t* block_tables;
  const int32_t* context_lens;
  const void* k_cache;  // simt path only
  const void* v_cache;  // simt path only
  float* part_o;        // [B, Hq, max_splits, D]
  float* part_ml;       // [B, Hq, max_splits, 2]
  int* status;          // may be null
  uint8_t* sched;       // workspace header (work-list counters); null: static unit order
  int batch, n_heads, n_kv_heads, group, head_dim, block_size, num_blocks, max_blocks;
  int max_ctx_tokens;  // (possibly truncated) table width * block_size
  int split_tokens;    // tokens per unit (the smallest the call may use), multiple of kStageTok
  int device_split;    // 1: the tc kernel picks the unit size from the live contexts
  int dynamic;         // 1: tc CTAs past their first unit take tickets from the workspace counter
  int max_splits;
  float scale_log2;  // log2(e) / sqrt(head_dim)
  unsigned long long wait_ns;  // wall-time limit of every mbarrier wait
  int drop_loads;              // wait-limit test: the producer issues nothing, so waits run out
};

__device__ __forceinline__ void report_timeout(int* status) {
  if (status) atomicExch(status, tvk::kStatusWaitTimeout);
}

// Effective context of sequence b (the reference never looks past the table).
__device__ __forceinline__ int effective_ctx(const DecodeParams& p, int b) {
  int c = p.context_lens[b];
  return c < p.max_ctx_tokens ? c : p.max_ctx_tokens;
}

// Byte offset of 16-byte chunk k16 of row t inside a TMA-swizzled tile whose
// rows are RB bytes (128 -> SWIZZLE_128B, 64 -> SWIZZLE_64B).
template <int RB>
__device__ __forceinline__ uint32_t swz(int t, int k16) {
  if constexpr (RB == 128) {
    return t * 128 + ((k16 ^ (t & 7)) << 4);
  } else {
    return t * 64 + ((k16 ^ ((t >> 1) & 3)) << 4);
  }
}

template <typename T>
__device__ __forceinline__ void write_zero_rows(const DecodeParams& p, int b, int kvh) {
  T* out = reinterpret_cast<T*>(p.out);
  const int n = p.group * p.head_dim;
  for (int i = threadIdx.x; i < n; i += blockDim.x)
    out[((size_t)b * p.n_heads + kvh * p.group) * p.head_dim + i] = DT<T>::from_f(0.f);
}

// -----------------------------------------------------------------------------
// Tensor-core kernel (fp16 / bf16)
// -----------------------------------------------------------------------------
template <int D, int RB>
struct TcCfg {
  static constexpr int kChunks = D * 2 / RB;               // row chunks per token
  static constexpr int kChunkBytes = kStageTok * RB;       // one chunk of one stage
  static constexpr int kKVBytes = kChunks * kChunkBytes;   // K (or V) part of a stage
  static constexpr int kStageBytes = 2 * kKVBytes;
  static constexpr int kStages = D == 128 ? 3 : (D == 64 ? 5 : 8);
  static constexpr int kRingBytes = kStages * kStageBytes;
  static constexpr int kBarOffset = kRingBytes;             // full / empty barriers
  static constexpr int kMetaOffset = kRingBytes + 128;      // one int4 of unit data per stage
  static constexpr int kMergeBarOffset = kRingBytes + 256;  // two barriers of the per-unit merge
  static constexpr int kQOffset = kRingBytes + 384;         // one query slot [group][D] per stage
  static_assert(2 * kStages * 8 <= 128 && kStages * 16 <= 128, "barrier / meta area");
  // merge scratch of the four consumer warps: m, l [4][16] then O [4][group][D]
  static __host__ __device__ constexpr int merge_offset(int group) { return kQOffset + kStages * group * D * 2; }
  static __host__ __device__ constexpr int smem_bytes(int group) {
    return merge_offset(group) + 2 * 4 * 16 * 4 + 4 * group * D * 4 + 1024;  // +1024 alignment slack
  }
};

// Work-list counters in the caller workspace header (the status word is at 0),
// and the unit size the last tc launch chose (read by the combine kernel).
constexpr int kTicketOffset = 64;
constexpr int kDoneOffset = 128;
constexpr int kSplitOffset = 192;

// Resident tc CTAs on a B200 (two per SM), and the unit counts the split
// policies aim for: close to one wave when every unit gets its own CTA (a
// small call gains more from skipping the split-K combine than from shorter
// units: 64 sequences x 4 KV heads with contexts up to 640 take 11.8 us as one
// 1024-token unit each, 15.6 us as 512-token units plus the combine); about
// four units per resident CTA for persistent grids, enough for the ticket
// counter to even out ragged contexts while keeping units long.
constexpr long kSlots = 148L * 2;
constexpr long kStaticTarget = 256;
constexpr int kStaticMaxSplit = 1024;
constexpr long kTargetUnits = kSlots * 4;
constexpr int kMaxSplitTokens = 4096;
// Block ids the producer keeps in registers per unit (a multiple of 32, at least
// the largest stage's 64 / 8 = 8 blocks).
constexpr int kBidWindow = 128;

// One unit of decode work: one context split of one (sequence, KV head).
// Tickets run over splits slowest, so every CTA sees a mix of sequences and
// the short tail splits of the longest sequences come last.
struct Unit {
  int b, kvh, split, n_tok, nsplit;
};

// Unit of ticket t; false if that split holds no live token.  A sequence with
// no context is one unit (split 0) with n_tok 0 whose output rows are zeros.
__device__ __forceinline__ bool decode_unit(const DecodeParams& p, int split_tokens, int t, Unit& un) {
  const int bk_count = p.batch * p.n_kv_heads;
  un.split = t / bk_count;
  const int bk = t - un.split * bk_count;
  un.kvh = bk % p.n_kv_heads;
  un.b = bk / p.n_kv_heads;
  const int ctx = effective_ctx(p, un.b);
  if (ctx <= 0) {
    un.n_tok = un.nsplit = 0;
    return un.split == 0;
  }
  const int tok_begin = un.split * split_tokens;
  if (tok_begin >= ctx) return false;
  un.n_tok = min(split_tokens, ctx - tok_begin);
  un.nsplit = (ctx + split_tokens - 1) / split_tokens;
  return true;
}

__device__ __forceinline__ void unit_of_ticket(const DecodeParams& p, int t, Unit& un) {
  const int bk_count = p.batch * p.n_kv_heads;
  un.split = t / bk_count;
  const int bk = t - un.split * bk_count;
  un.kvh = bk % p.n_kv_heads;
  un.b = bk / p.n_kv_heads;
}

// Persistent CTAs (about two per SM).  The producer warp takes units from an
// atomic ticket counter (a fixed stride over tickets when no workspace is
// given) and streams their K/V blocks through one TMA ring that runs across
// unit boundaries, so the next unit's blocks are in flight while the consumers
// merge and store the previous one.  Each stage carries the unit's ticket,
// its stage index and token count, and on a unit's first stage its query rows,
// so the consumer warps read nothing from global memory but the K/V stages.
template <typename T, int D, int RB>
__global__ void __launch_bounds__(160, 2)
    paged_decode_tc_kernel(const DecodeParams p, const __grid_constant__ CUtensorMap tm_k,
                           const __grid_constant__ CUtensorMap tm_v) {
  using C = TcCfg<D, RB>;
  constexpr int RC = RB / 2;  // elements per row chunk
  constexpr int K16_PER_ROW = RB / 16;
  const int bs = p.block_size;
  const int G = p.group;
  const int total = p.batch * p.n_kv_heads * p.max_splits;

  extern __shared__ uint8_t smem_raw[];
  const uint32_t raw_u32 = ptx::smem_u32(smem_raw);
  const uint32_t base_u32 = (raw_u32 + 1023u) & ~1023u;
  uint8_t* base = smem_raw + (base_u32 - raw_u32);
  uint64_t* full_bar = reinterpret_cast<uint64_t*>(base + C::kBarOffset);
  uint64_t* empty_bar = full_bar + C::kStages;
  int4* meta = reinterpret_cast<int4*>(base + C::kMetaOffset);
  uint64_t* merge_bar = reinterpret_cast<uint64_t*>(base + C::kMergeBarOffset);
  uint8_t* qslot = base + C::kQOffset;
  const int q_bytes = G * D * 2;

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  if (threadIdx.x == 0) {
    for (int s = 0; s < C::kStages; ++s) {
      ptx::mbar_init(&full_bar[s], 1);
      ptx::mbar_init(&empty_bar[s], 4);
    }
    ptx::mbar_init(&merge_bar[0], 4);  // one arrival per consumer warp
    ptx::mbar_init(&merge_bar[1], 4);
    ptx::fence_mbar_init();
  }
  __syncthreads();
  // Launched as a programmatic dependent: wait for the kernel before it (which
  // may have written q, the tables or this step's K/V) before any global read.
  asm volatile("griddepcontrol.wait;" ::: "memory");

  if (warp == 4) {
    // ---------------- producer warp ----------------------------------------
    if (lane == 0) {
      ptx::prefetch_tmap(&tm_k);
      ptx::prefetch_tmap(&tm_v);
    }
    // CTA i starts with ticket i; later tickets come from the counter (offset
    // by the grid size) or, without it, in steps of the grid size.
    unsigned* ticket = (p.sched && p.dynamic) ? reinterpret_cast<unsigned*>(p.sched + kTicketOffset) : nullptr;

    // Unit size of this call: the largest power of two (<= 4096, >= the host's
    // split) that still gives about kTargetUnits live units.  Every CTA reads
    // the same contexts and reaches the same answer.
    int split_tokens = p.split_tokens;
    int live_total = total;
    if (p.device_split) {
      constexpr int NS = 7;  // 4096 .. 64
      int cnt[NS];
#pragma unroll
      for (int k = 0; k < NS; ++k) cnt[k] = 0;
      int max_ctx = 0;
      for (int b = lane; b < p.batch; b += 32) {
        const int c = effective_ctx(p, b);
        if (c > 0) {
          max_ctx = max(max_ctx, c);
#pragma unroll
          for (int k = 0; k < NS; ++k) cnt[k] = min(cnt[k] + ((c + (kMaxSplitTokens >> k) - 1) >> (12 - k)), 1 << 24);
        }
      }
#pragma unroll
      for (int off = 16; off > 0; off >>= 1) {
        max_ctx = max(max_ctx, __shfl_xor_sync(0xffffffffu, max_ctx, off));
#pragma unroll
        for (int k = 0; k < NS; ++k) cnt[k] += __shfl_xor_sync(0xffffffffu, cnt[k], off);
      }
#pragma unroll
      for (int k = 0; k < NS; ++k) {
        const int sk = kMaxSplitTokens >> k;
        if (sk < p.split_tokens) break;
        split_tokens = sk;
        if ((long)cnt[k] * p.n_kv_heads >= kTargetUnits) break;
      }
      const int splits = max_ctx > 0 ? (max_ctx + split_tokens - 1) / split_tokens : 1;
      live_total = p.batch * p.n_kv_heads * splits;
      if (blockIdx.x == 0 && lane == 0 && p.sched) *reinterpret_cast<int*>(p.sched + kSplitOffset) = split_tokens;
    }

    // One atomic per claimed ticket.  A dead ticket (a split past its
    // sequence's context) starts a scan: the lanes test the following
    // (split, sequence) pairs 32 at a time and the counter is raised past the
    // dead run in one atomicMax, so runs of dead tickets cost a few round trips
    // instead of one atomic each.
    int next_static = blockIdx.x;
    uint32_t it_g = 0;
    bool running = true;
    const int bk_count = p.batch * p.n_kv_heads;
    while (running) {
      // next live unit (or the end of the list)
      int t = total;
      Unit un;
      while (true) {
        if (!ticket || next_static == (int)blockIdx.x) {
          t = next_static;
          next_static += gridDim.x;
        } else {
          int v = 0;
          if (lane == 0) v = (int)atomicAdd(ticket, 1u);
          t = __shfl_sync(0xffffffffu, v, 0) + (int)gridDim.x;
        }
        if (t >= live_total) {
          t = total;
          break;
        }
        if (decode_unit(p, split_tokens, t, un)) break;
        if (!ticket) continue;
        // Dead: every ticket of this (split, sequence) is dead; scan onwards.
        // Split 0 is always live, so the scan runs over splits >= 1 only.
        const int c_end = (live_total / bk_count) * p.batch;
        int c = (t / bk_count) * p.batch + (t % bk_count) / p.n_kv_heads + 1;
        int found = -1;
        while (c < c_end) {
          const int ci = c + lane;
          bool ok = false;
          if (ci < c_end) {
            const int lvl = ci / p.batch;
            ok = effective_ctx(p, ci - lvl * p.batch) > lvl * split_tokens;
          }
          const uint32_t m = __ballot_sync(0xffffffffu, ok);
          if (m) {
            found = c + __ffs(m) - 1;
            break;
          }
          c += 32;
        }
        if (found < 0) {  // nothing live after t: the list is done
          t = total;
          break;
        }
        const int t_live = (found / p.batch) * bk_count + (found % p.batch) * p.n_kv_heads;
        if (lane == 0 && t_live > (int)gridDim.x) atomicMax(ticket, (unsigned)(t_live - (int)gridDim.x));
      }
      const bool live = t < total;
      running = live;
      const int n_stage = live ? max((un.n_tok + kStageTok - 1) / kStageTok, 1) : 1;
      const int tok_begin = live ? un.split * split_tokens : 0;
      const int ctx_end = live ? tok_begin + un.n_tok : 0;
      const int32_t* bt = live ? p.block_tables + (size_t)un.b * p.max_blocks : p.block_tables;
      // The unit's block ids, kBidWindow at a time, one per lane and register, loaded
      // once per window so that no stage waits on a table read before its copies.
      const int blk_end = live ? (ctx_end + bs - 1) / bs : 0;  // one past the unit's last block
      int win_base = -kBidWindow;                              // first block of the loaded window
      int bid[kBidWindow / 32];
      for (int it = 0; it < n_stage; ++it, ++it_g) {
        const int s = it_g % C::kStages;
        const uint32_t ph = (it_g / C::kStages) & 1;
        if (!ptx::mbar_wait(&empty_bar[s], ph ^ 1, p.wait_ns)) {
          report_timeout(p.status);
          running = false;
          break;
        }
        if (p.drop_loads) continue;  // test hook: nothing reaches the consumers
        if (!live || un.n_tok == 0) {
          // end of the list, or a sequence without context: no data
          if (lane == 0) {
            meta[s] = make_int4(live ? t : -1, 0, 0, 0);
            ptx::mbar_arrive(&full_bar[s]);
          }
          continue;
        }
        const int tok0 = tok_begin + it * kStageTok;  // absolute token of stage row 0
        const int live_tok = min(kStageTok, ctx_end - tok0);
        const int nblk = (live_tok + bs - 1) / bs;
        const uint32_t q_tx = it == 0 ? (uint32_t)q_bytes : 0u;
        if (lane == 0) {
          meta[s] = make_int4(t, it, un.n_tok, un.nsplit);
          ptx::mbar_arrive_expect_tx(&full_bar[s], (uint32_t)(nblk * bs * D * 2 * 2) + q_tx);
          if (it == 0) {
            const uint8_t* qsrc = reinterpret_cast<const uint8_t*>(p.q) +
                                  ((size_t)un.b * p.n_heads + (size_t)un.kvh * G) * D * 2;
            ptx::bulk_load(qslot + s * q_bytes, qsrc, (uint32_t)q_bytes, &full_bar[s]);
          }
        }
        const int first_blk = tok0 / bs;
        if (first_blk + nblk > win_base + kBidWindow) {  // stage runs past the window: load the next one
          win_base = first_blk;
#pragma unroll
          for (int r = 0; r < kBidWindow / 32; ++r) {
            const int bi = win_base + r * 32 + lane;
            bid[r] = bi < blk_end ? __ldg(bt + bi) : 0;
          }
        }
        __syncwarp();
        const uint32_t stage_off = s * C::kStageBytes;
        const int n_loads = nblk * C::kChunks * 2;
        for (int i0 = 0; i0 < n_loads; i0 += 32) {  // warp-uniform trip count: every lane shuffles
          const int i = i0 + lane;
          const int j = min(i / (C::kChunks * 2), nblk - 1);
          const int rel = first_blk + j - win_base;  // in [0, kBidWindow)
          int blk = 0;
#pragma unroll
          for (int r = 0; r < kBidWindow / 32; ++r) {
            const int v = __shfl_sync(0xffffffffu, bid[r], rel & 31);
            blk = (rel >> 5) == r ? v : blk;
          }
          if (i >= n_loads) continue;
          const int rest = i % (C::kChunks * 2);
          const int kv = rest / C::kChunks;
          const int c = rest % C::kChunks;
          uint8_t* dst = base + stage_off + kv * C::kKVBytes + c * C::kChunkBytes + j * bs * RB;
          ptx::tma_load_4d(dst, kv ? &tm_v : &tm_k, &full_bar[s], c * RC, un.kvh, 0, blk);
        }
      }
    }
    // Last CTA out returns the counters to zero for the next call.
    if (ticket && lane == 0) {
      unsigned* done = reinterpret_cast<unsigned*>(p.sched + kDoneOffset);
      __threadfence();
      if (atomicAdd(done, 1u) == gridDim.x - 1) {
        atomicExch(ticket, 0u);
        atomicExch(done, 0u);
      }
    }
    return;
  }

  // ---------------- consumer warps ----------------------------------------
  const int g = lane >> 2, tig = lane & 3;
  float* cm = reinterpret_cast<float*>(base + C::merge_offset(G));
  uint32_t n_merge = 0;
  float* cl = cm + 4 * 16;
  float* co = cl + 4 * 16;

  uint32_t qa[D / 16][4];
  float o[D / 8][4];
  float m0 = -INFINITY, m1 = -INFINITY, l0 = 0.f, l1 = 0.f;
  Unit un{};
  int n_tok = 0, nsplit = 0;

  for (uint32_t it_g = 0;; ++it_g) {
    const int s = it_g % C::kStages;
    const uint32_t ph = (it_g / C::kStages) & 1;
    if (!ptx::mbar_wait(&full_bar[s], ph, p.wait_ns)) {
      report_timeout(p.status);
      return;
    }
    const int4 md = meta[s];
    if (md.x < 0) return;  // end of the work list
    const int it = md.y;
    if (it == 0) {
      unit_of_ticket(p, md.x, un);
      n_tok = md.z;
      nsplit = md.w;
      if (n_tok == 0) {
        __syncwarp();
        if (lane == 0) ptx::mbar_arrive(&empty_bar[s]);
        T* out = reinterpret_cast<T*>(p.out) + ((size_t)un.b * p.n_heads + un.kvh * G) * D;
        for (int i = threadIdx.x; i < G * D; i += 128) out[i] = DT<T>::from_f(0.f);
        continue;
      }
      // Q fragments (A operand, rows = query heads of this KV group, zero padded).
      const uint32_t* q32 = reinterpret_cast<const uint32_t*>(qslot + s * q_bytes);
#pragma unroll
      for (int kk = 0; kk < D / 16; ++kk) {
        const int c0 = kk * 16 + tig * 2;
        qa[kk][0] = g < G ? q32[(g * D + c0) >> 1] : 0u;
        qa[kk][1] = g + 8 < G ? q32[((g + 8) * D + c0) >> 1] : 0u;
        qa[kk][2] = g < G ? q32[(g * D + c0 + 8) >> 1] : 0u;
        qa[kk][3] = g + 8 < G ? q32[((g + 8) * D + c0 + 8) >> 1] : 0u;
      }
#pragma unroll
      for (int i = 0; i < D / 8; ++i) o[i][0] = o[i][1] = o[i][2] = o[i][3] = 0.f;
      m0 = m1 = -INFINITY;
      l0 = l1 = 0.f;
    }

    const int t_base = it * kStageTok + warp * 16;  // token of this warp's row 0, relative to the split
    if (t_base < n_tok) {
      const uint32_t kbase = base_u32 + s * C::kStageBytes;
      const uint32_t vbase = kbase + C::kKVBytes;
      const int row0 = warp * 16;

      // S = Q K^T  (16 heads x 16 tokens)
      float sc[2][4] = {{0.f, 0.f, 0.f, 0.f}, {0.f, 0.f, 0.f, 0.f}};
#pragma unroll
      for (int kk = 0; kk < D / 16; ++kk) {
        const int chunk16 = kk * 2 + ((lane >> 3) & 1);
        const int c = chunk16 / K16_PER_ROW, k16 = chunk16 % K16_PER_ROW;
        const int t = row0 + (lane & 7) + ((lane >> 4) << 3);
        uint32_t r0, r1, r2, r3;
        ptx::ldmatrix_x4(kbase + c * C::kChunkBytes + swz<RB>(t, k16), r0, r1, r2, r3);
        ptx::Mma<T>::run(sc[0], qa[kk], r0, r1);
        ptx::Mma<T>::run(sc[1], qa[kk], r2, r3);
      }

      // scale, mask, online softmax (fp32, log2 domain)
      const bool partial = t_base + 16 > n_tok;
#pragma unroll
      for (int n = 0; n < 2; ++n)
#pragma unroll
        for (int j = 0; j < 4; ++j) {
          const int tok = t_base + n * 8 + tig * 2 + (j & 1);
          sc[n][j] = (!partial || tok < n_tok) ? sc[n][j] * p.scale_log2 : -INFINITY;
        }
      float mx0 = fmaxf(fmaxf(sc[0][0], sc[0][1]), fmaxf(sc[1][0], sc[1][1]));
      float mx1 = fmaxf(fmaxf(sc[0][2], sc[0][3]), fmaxf(sc[1][2], sc[1][3]));
      mx0 = fmaxf(mx0, __shfl_xor_sync(0xffffffffu, mx0, 1));
      mx0 = fmaxf(mx0, __shfl_xor_sync(0xffffffffu, mx0, 2));
      mx1 = fmaxf(mx1, __shfl_xor_sync(0xffffffffu, mx1, 1));
      mx1 = fmaxf(mx1, __shfl_xor_sync(0xffffffffu, mx1, 2));
      // Lazy rescale: the running max (and with it l and O) moves only when a row's
      // new max exceeds it by more than 2^8, so P stays below 2^8 and most stages
      // skip the O rescale.  The first processed stage always takes it (m = -inf).
      const float mn0 = fmaxf(m0, mx0), mn1 = fmaxf(m1, mx1);
      if (__any_sync(0xffffffffu, mn0 > m0 + 8.f || mn1 > m1 + 8.f)) {
        const float corr0 = ptx::ex2(m0 - mn0), corr1 = ptx::ex2(m1 - mn1);
        m0 = mn0;
        m1 = mn1;
        l0 *= corr0;
        l1 *= corr1;
#pragma unroll
        for (int i = 0; i < D / 8; ++i) {
          o[i][0] *= corr0;
          o[i][1] *= corr0;
          o[i][2] *= corr1;
          o[i][3] *= corr1;
        }
      }
      float pr[2][4];
#pragma unroll
      for (int n = 0; n < 2; ++n) {
        pr[n][0] = ptx::ex2(sc[n][0] - m0);
        pr[n][1] = ptx::ex2(sc[n][1] - m0);
        pr[n][2] = ptx::ex2(sc[n][2] - m1);
        pr[n][3] = ptx::ex2(sc[n][3] - m1);
      }
      l0 += (pr[0][0] + pr[0][1]) + (pr[1][0] + pr[1][1]);
      l1 += (pr[0][2] + pr[0][3]) + (pr[1][2] + pr[1][3]);
      uint32_t pa[4];
      pa[0] = DT<T>::pack2(pr[0][0], pr[0][1]);
      pa[1] = DT<T>::pack2(pr[0][2], pr[0][3]);
      pa[2] = DT<T>::pack2(pr[1][0], pr[1][1]);
      pa[3] = DT<T>::pack2(pr[1][2], pr[1][3]);

      // Rows past the context may hold stale shared memory: zero their V.
      uint32_t vm_lo = 0xffffffffu, vm_hi = 0xffffffffu;
      if (partial) {
        const int tl = t_base + tig * 2, th = t_base + 8 + tig * 2;
        vm_lo = (tl < n_tok ? 0x0000ffffu : 0u) | (tl + 1 < n_tok ? 0xffff0000u : 0u);
        vm_hi = (th < n_tok ? 0x0000ffffu : 0u) | (th + 1 < n_tok ? 0xffff0000u : 0u);
      }

      // O += P V
#pragma unroll
      for (int np = 0; np < D / 16; ++np) {
        const int chunk16 = np * 2 + (lane >> 4);
        const int c = chunk16 / K16_PER_ROW, k16 = chunk16 % K16_PER_ROW;
        const int t = row0 + (lane & 7) + (((lane >> 3) & 1) << 3);
        uint32_t r0, r1, r2, r3;
        ptx::ldmatrix_x4_trans(vbase + c * C::kChunkBytes + swz<RB>(t, k16), r0, r1, r2, r3);
        r0 &= vm_lo;
        r1 &= vm_hi;
        r2 &= vm_lo;
        r3 &= vm_hi;
        ptx::Mma<T>::run(o[2 * np], pa, r0, r1);
        ptx::Mma<T>::run(o[2 * np + 1], pa, r2, r3);
      }
    }
    __syncwarp();
    if (lane == 0) ptx::mbar_arrive(&empty_bar[s]);
    if ((it + 1) * kStageTok < n_tok) continue;

    // ---------------- last stage of the unit: merge the four warps ----------
    float L0 = l0 + __shfl_xor_sync(0xffffffffu, l0, 1);
    L0 += __shfl_xor_sync(0xffffffffu, L0, 2);
    float L1 = l1 + __shfl_xor_sync(0xffffffffu, l1, 1);
    L1 += __shfl_xor_sync(0xffffffffu, L1, 2);
    // The four warps meet twice (bounded waits, so a warp that gave up cannot
    // strand the others): first when all have read the previous unit's merge,
    // then when all have written this one.
    __syncwarp();
    if (lane == 0) ptx::mbar_arrive(&merge_bar[0]);
    if (!ptx::mbar_wait(&merge_bar[0], n_merge & 1, p.wait_ns)) {
      report_timeout(p.status);
      return;
    }
    if (tig == 0) {
      cm[warp * 16 + g] = m0;
      cm[warp * 16 + g + 8] = m1;
      cl[warp * 16 + g] = L0;
      cl[warp * 16 + g + 8] = L1;
    }
#pragma unroll
    for (int i = 0; i < D / 8; ++i) {
      const int col = i * 8 + tig * 2;
      if (g < G) {
        co[(warp * G + g) * D + col] = o[i][0];
        co[(warp * G + g) * D + col + 1] = o[i][1];
      }
      if (g + 8 < G) {
        co[(warp * G + g + 8) * D + col] = o[i][2];
        co[(warp * G + g + 8) * D + col + 1] = o[i][3];
      }
    }
    __syncwarp();
    if (lane == 0) ptx::mbar_arrive(&merge_bar[1]);
    if (!ptx::mbar_wait(&merge_bar[1], n_merge & 1, p.wait_ns)) {
      report_timeout(p.status);
      return;
    }
    ++n_merge;

    for (int idx = threadIdx.x; idx < G * D; idx += 128) {
      const int r = idx / D, col = idx % D;
      float M = -INFINITY;
#pragma unroll
      for (int w = 0; w < 4; ++w) M = fmaxf(M, cm[w * 16 + r]);
      float L = 0.f, A = 0.f;
#pragma unroll
      for (int w = 0; w < 4; ++w) {
        const float e = exp2f(cm[w * 16 + r] - M);
        L += cl[w * 16 + r] * e;
        A += co[(w * G + r) * D + col] * e;
      }
      const int h = un.kvh * G + r;
      if (nsplit == 1) {
        reinterpret_cast<T*>(p.out)[((size_t)un.b * p.n_heads + h) * D + col] = DT<T>::from_f(A / L);
      } else {
        const size_t row = ((size_t)un.b * p.n_heads + h) * p.max_splits + un.split;
        p.part_o[row * D + col] = A;
        if (col == 0) {
          p.part_ml[row * 2] = M;
          p.part_ml[row * 2 + 1] = L;
        }
      }
    }
  }
}

// -----------------------------------------------------------------------------
// SIMT kernel (any dtype, any block size)
// -----------------------------------------------------------------------------
template <typename T>
__device__ __forceinline__ void load4(const T* src, float* dst) {
  if constexpr (sizeof(T) == 4) {
    const float4 v = *reinterpret_cast<const float4*>(src);
    dst[0] = v.x;
    dst[1] = v.y;
    dst[2] = v.z;
    dst[3] = v.w;
  } else {
    const uint2 v = *reinterpret_cast<const uint2*>(src);
    const T* h = reinterpret_cast<const T*>(&v);
#pragma unroll
    for (int i = 0; i < 4; ++i) dst[i] = DT<T>::to_f(h[i]);
  }
}

template <typename T, int D>
__global__ void __launch_bounds__(128) paged_decode_simt_kernel(const DecodeParams p) {
  asm volatile("griddepcontrol.wait;" ::: "memory");  // programmatic dependent launch
  constexpr int DP = D + 4;               // padded row (floats)
  constexpr int MAXK = kMaxGroup * D / 128;  // (head, dim) outputs per thread
  __shared__ __align__(16) float qs[kMaxGroup][D];
  __shared__ __align__(16) float ks[kSimtTile][DP];
  __shared__ __align__(16) float vs[kSimtTile][DP];
  __shared__ float ps[kMaxGroup][kSimtTile];
  __shared__ float corr_s[kMaxGroup];
  __shared__ float mfin[kMaxGroup], lfin[kMaxGroup];

  const int split = blockIdx.x, kvh = blockIdx.y, b = blockIdx.z;
  const int ctx = effective_ctx(p, b);
  if (ctx <= 0) {
    if (split == 0) write_zero_rows<T>(p, b, kvh);
    return;
  }
  const int tok_begin = split * p.split_tokens;
  if (tok_begin >= ctx) return;
  const int n_tok = min(p.split_tokens, ctx - tok_begin);
  const int nsplit = (ctx + p.split_tokens - 1) / p.split_tokens;
  const int G = p.group, Hkv = p.n_kv_heads, bs = p.block_size;
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;

  const T* q = reinterpret_cast<const T*>(p.q) + ((size_t)b * p.n_heads + kvh * G) * D;
  for (int i = tid; i < G * D; i += 128) qs[i / D][i % D] = DT<T>::to_f(q[i]);

  const T* kc = reinterpret_cast<const T*>(p.k_cache);
  const T* vc = reinterpret_cast<const T*>(p.v_cache);
  const int32_t* bt = p.block_tables + (size_t)b * p.max_blocks;

  float acc[MAXK];
#pragma unroll
  for (int k = 0; k < MAXK; ++k) acc[k] = 0.f;
  // online-softmax state of heads owned by this warp (g = warp + 4*i)
  float m_own[kMaxGroup / 4], l_own[kMaxGroup / 4];
#pragma unroll
  for (int i = 0; i < kMaxGroup / 4; ++i) {
    m_own[i] = -INFINITY;
    l_own[i] = 0.f;
  }

  for (int t0 = 0; t0 < n_tok; t0 += kSimtTile) {
    __syncthreads();
    for (int i = tid; i < kSimtTile * (D / 4); i += 128) {
      const int t = i / (D / 4), d4 = (i % (D / 4)) * 4;
      float kv4[4] = {0.f, 0.f, 0.f, 0.f}, vv4[4] = {0.f, 0.f, 0.f, 0.f};
      const int tok = t0 + t;
      if (tok < n_tok) {
        const int abs_tok = tok_begin + tok;
        const int blk = __ldg(bt + abs_tok / bs);
        if (blk >= 0 && blk < p.num_blocks) {
          const size_t off = (((size_t)blk * bs + abs_tok % bs) * Hkv + kvh) * D + d4;
          load4<T>(kc + off, kv4);
          load4<T>(vc + off, vv4);
        }
      }
      *reinterpret_cast<float4*>(&ks[t][d4]) = make_float4(kv4[0], kv4[1], kv4[2], kv4[3]);
      *reinterpret_cast<float4*>(&vs[t][d4]) = make_float4(vv4[0], vv4[1], vv4[2], vv4[3]);
    }
    __syncthreads();

    // scores: warp owns heads warp, warp+4, ...; lane = token
#pragma unroll
    for (int i = 0; i < kMaxGroup / 4; ++i) {
      const int gh = warp + 4 * i;
      if (gh < G) {
        float s = 0.f;
#pragma unroll 8
        for (int d = 0; d < D; d += 4) {
          const float4 kk = *reinterpret_cast<const float4*>(&ks[lane][d]);
          const float4 qq = *reinterpret_cast<const float4*>(&qs[gh][d]);
          s = fmaf(qq.x, kk.x, s);
          s = fmaf(qq.y, kk.y, s);
          s = fmaf(qq.z, kk.z, s);
          s = fmaf(qq.w, kk.w, s);
        }
        s = (t0 + lane < n_tok) ? s * p.scale_log2 : -INFINITY;
        float mx = s;
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, o));
        const float mn = fmaxf(m_own[i], mx);
        const float corr = exp2f(m_own[i] - mn);
        const float pv = exp2f(s - mn);
        float sum = pv;
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) sum += __shfl_xor_sync(0xffffffffu, sum, o);
        l_own[i] = l_own[i] * corr + sum;
        m_own[i] = mn;
        ps[gh][lane] = pv;
        if (lane == 0) corr_s[gh] = corr;
      }
    }
    __syncthreads();

#pragma unroll
    for (int k = 0; k < MAXK; ++k) {
      const int idx = tid + 128 * k;
      if (idx < G * D) {
        const int gh = idx / D, d = idx % D;
        float a = acc[k] * corr_s[gh];
#pragma unroll 8
        for (int t = 0; t < kSimtTile; ++t) a = fmaf(ps[gh][t], vs[t][d], a);
        acc[k] = a;
      }
    }
  }

#pragma unroll
  for (int i = 0; i < kMaxGroup / 4; ++i) {
    const int gh = warp + 4 * i;
    if (gh < G && lane == 0) {
      mfin[gh] = m_own[i];
      lfin[gh] = l_own[i];
    }
  }
  __syncthreads();
#pragma unroll
  for (int k = 0; k < MAXK; ++k) {
    const int idx = tid + 128 * k;
    if (idx < G * D) {
      const int gh = idx / D, d = idx % D;
      const int h = kvh * G + gh;
      if (nsplit == 1) {
        reinterpret_cast<T*>(p.out)[((size_t)b * p.n_heads + h) * D + d] = DT<T>::from_f(acc[k] / lfin[gh]);
      } else {
        const size_t row = ((size_t)b * p.n_heads + h) * p.max_splits + split;
        p.part_o[row * D + d] = acc[k];
        if (d == 0) {
          p.part_ml[row * 2] = mfin[gh];
          p.part_ml[row * 2 + 1] = lfin[gh];
        }
      }
    }
  }
}

// -----------------------------------------------------------------------------
// split-K combine
// -----------------------------------------------------------------------------
// One CTA per (sequence, KV head); warp w merges query-head rows w, w+4, ...
// The lanes first take 32 splits at a time for the max and the weights
// exp2(m_i - M); then each lane owns D/32 output columns and adds the split
// rows with the weights broadcast by shuffle, eight independent loads in
// flight per lane.
template <typename T, int D>
__global__ void __launch_bounds__(128) paged_decode_combine_kernel(const DecodeParams p) {
  asm volatile("griddepcontrol.wait;" ::: "memory");  // programmatic dependent launch
  const int kvh = blockIdx.x, b = blockIdx.y;
  const int ctx = effective_ctx(p, b);
  if (ctx <= 0) return;
  const int split_tokens = p.device_split ? *reinterpret_cast<const int*>(p.sched + kSplitOffset) : p.split_tokens;
  const int nsplit = (ctx + split_tokens - 1) / split_tokens;
  if (nsplit <= 1) return;
  const int G = p.group;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  constexpr int per_lane = D / 32;  // 1, 2 or 4 columns
  for (int r = warp; r < G; r += 4) {
    const int h = kvh * G + r;
    const size_t row0 = ((size_t)b * p.n_heads + h) * p.max_splits;
    const float* ml = p.part_ml + row0 * 2;
    const float* po = p.part_o + row0 * D;
    float M = -INFINITY;
    for (int i = lane; i < nsplit; i += 32) M = fmaxf(M, ml[i * 2]);
#pragma unroll
    for (int off = 16; off > 0; off >>= 1) M = fmaxf(M, __shfl_xor_sync(0xffffffffu, M, off));
    float L = 0.f;
    float acc[4] = {0.f, 0.f, 0.f, 0.f};
    for (int c0 = 0; c0 < nsplit; c0 += 32) {
      const int i = c0 + lane;
      const float w = i < nsplit ? exp2f(ml[i * 2] - M) : 0.f;
      L += i < nsplit ? ml[i * 2 + 1] * w : 0.f;
      const int n = min(32, nsplit - c0);
#pragma unroll 8
      for (int j = 0; j < n; ++j) {
        const float wj = __shfl_sync(0xffffffffu, w, j);
        const float* src = po + (size_t)(c0 + j) * D + lane * per_lane;
        if constexpr (per_lane == 4) {
          const float4 v = *reinterpret_cast<const float4*>(src);
          acc[0] += wj * v.x;
          acc[1] += wj * v.y;
          acc[2] += wj * v.z;
          acc[3] += wj * v.w;
        } else if constexpr (per_lane == 2) {
          const float2 v = *reinterpret_cast<const float2*>(src);
          acc[0] += wj * v.x;
          acc[1] += wj * v.y;
        } else {
          acc[0] += wj * src[0];
        }
      }
    }
#pragma unroll
    for (int off = 16; off > 0; off >>= 1) L += __shfl_xor_sync(0xffffffffu, L, off);
    T* out = reinterpret_cast<T*>(p.out) + ((size_t)b * p.n_heads + h) * D + lane * per_lane;
#pragma unroll
    for (int k = 0; k < per_lane; ++k) out[k] = DT<T>::from_f(acc[k] / L);
  }
}

// -----------------------------------------------------------------------------
// host side
// -----------------------------------------------------------------------------
int table_tokens(int block_size, int max_blocks, int max_context_len) {
  int blocks = max_blocks;
  if (max_context_len >= 0) {
    const int need = (max_context_len + block_size - 1) / block_size;
    blocks = need < max_blocks ? need : max_blocks;
  }
  return blocks * block_size;
}

// Largest power of two in [64, max_split] that gives at least `target` units
// when every sequence uses its whole table.
int split_for(long bk, int table_tok, int max_split, long target) {
  for (int s = max_split; s > kStageTok; s >>= 1)
    if (bk * ((table_tok + s - 1) / s) >= target) return s;
  return kStageTok;
}

// How one call is cut into units and launched.
//  * One CTA per unit (the simt kernel always; the tc kernel when that grid
//    is at most two waves): units of up to 1024 tokens, about one wave.
//  * Otherwise persistent tc CTAs with the ticket counter: `split` is the
//    smallest unit the kernel may use (it sizes the partials); the kernel
//    picks the actual size from the live contexts.
struct Plan {
  int split, max_splits, dynamic;
};

Plan make_plan(int batch, int n_kv_heads, int table_tok, bool persistent_ok) {
  const long bk = (long)batch * n_kv_heads;
  Plan pl{};
  pl.split = split_for(bk, table_tok, kStaticMaxSplit, kStaticTarget);
  pl.max_splits = table_tok > 0 ? (table_tok + pl.split - 1) / pl.split : 1;
  pl.dynamic = 0;
  if (!persistent_ok || bk * pl.max_splits <= 2 * kSlots) return pl;
  pl.split = split_for(bk, table_tok, kMaxSplitTokens, kTargetUnits);
  pl.max_splits = table_tok > 0 ? (table_tok + pl.split - 1) / pl.split : 1;
  pl.dynamic = 1;
  return pl;
}

size_t workspace_bytes_for(int batch, int n_heads, int head_dim, int max_splits) {
  size_t bytes = tvk::kWorkspaceHeader;
  if (max_splits > 1) bytes += (size_t)batch * n_heads * max_splits * (head_dim + 2) * sizeof(float);
  return bytes;
}

template <typename T, int D, int RB>
int launch_tc(const DecodeParams& p, const void* k_cache, const void* v_cache, CUtensorMapDataType tdt,
              cudaStream_t stream) {
  using C = TcCfg<D, RB>;
  tvk::EncodeTiledFn encode = tvk::encode_tiled_fn();
  if (!encode) {
    tvk::set_error("cuTensorMapEncodeTiled is not available from the driver");
    return TVK_ERR_CUDA;
  }
  const size_t es = sizeof(T);
  CUtensorMap tmk, tmv;
  cuuint64_t dims[4] = {(cuuint64_t)D, (cuuint64_t)p.n_kv_heads, (cuuint64_t)p.block_size,
                        (cuuint64_t)p.num_blocks};
  cuuint64_t strides[3] = {(cuuint64_t)(D * es), (cuuint64_t)(p.n_kv_heads * D * es),
                           (cuuint64_t)((size_t)p.block_size * p.n_kv_heads * D * es)};
  cuuint32_t box[4] = {(cuuint32_t)(RB / es), 1u, (cuuint32_t)p.block_size, 1u};
  cuuint32_t estr[4] = {1u, 1u, 1u, 1u};
  const CUtensorMapSwizzle sw = RB == 128 ? CU_TENSOR_MAP_SWIZZLE_128B : CU_TENSOR_MAP_SWIZZLE_64B;
  CUresult r1 = encode(&tmk, tdt, 4, const_cast<void*>(k_cache), dims, strides, box, estr,
                       CU_TENSOR_MAP_INTERLEAVE_NONE, sw, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                       CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  CUresult r2 = encode(&tmv, tdt, 4, const_cast<void*>(v_cache), dims, strides, box, estr,
                       CU_TENSOR_MAP_INTERLEAVE_NONE, sw, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                       CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r1 != CUDA_SUCCESS || r2 != CUDA_SUCCESS) {
    tvk::set_error("cuTensorMapEncodeTiled failed (%d, %d)", (int)r1, (int)r2);
    return TVK_ERR_CUDA;
  }
  auto kern = paged_decode_tc_kernel<T, D, RB>;
  const int smem = C::smem_bytes(p.group);
  static unsigned long long attr_set_mask = 0;  // per instantiation, one bit per device
  static int ctas_per_sm[64][kMaxGroup + 1] = {};
  static int num_sms[64] = {};
  int dev = 0;
  TVK_CHECK_CUDA(cudaGetDevice(&dev));
  if (dev >= 64) {
    tvk::set_error("device index %d beyond 63", dev);
    return TVK_ERR_UNSUPPORTED;
  }
  if (!(attr_set_mask & (1ull << dev))) {
    TVK_CHECK_CUDA(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, C::smem_bytes(kMaxGroup)));
    TVK_CHECK_CUDA(cudaDeviceGetAttribute(&num_sms[dev], cudaDevAttrMultiProcessorCount, dev));
    attr_set_mask |= (1ull << dev);
  }
  if (ctas_per_sm[dev][p.group] == 0) {
    int n = 0;
    TVK_CHECK_CUDA(cudaOccupancyMaxActiveBlocksPerMultiprocessor(&n, kern, 160, smem));
    ctas_per_sm[dev][p.group] = n > 0 ? n : 1;
  }
  const long long units = (long long)p.batch * p.n_kv_heads * p.max_splits;
  const long long slots = (long long)num_sms[dev] * ctas_per_sm[dev][p.group];
  // Persistent grids fill the resident slots; otherwise one CTA per unit.
  const int grid = (int)(p.dynamic && units > slots ? slots : units);
  TVK_CHECK_CUDA(tvk::launch_pdl(kern, grid, 160, smem, stream, p, tmk, tmv));
  TVK_CHECK_LAUNCH("paged_decode_tc");
  return TVK_OK;
}

template <typename T>
int launch_typed(DecodeParams& p, bool use_tc, CUtensorMapDataType tdt, cudaStream_t stream) {
  int rc = TVK_OK;
  if (use_tc) {
    if constexpr (sizeof(T) == 2) {
      switch (p.head_dim) {
        case 32: rc = launch_tc<T, 32, 64>(p, p.k_cache, p.v_cache, tdt, stream); break;
        case 64: rc = launch_tc<T, 64, 128>(p, p.k_cache, p.v_cache, tdt, stream); break;
        default: rc = launch_tc<T, 128, 128>(p, p.k_cache, p.v_cache, tdt, stream); break;
      }
    }
  } else {
    dim3 grid(p.max_splits, p.n_kv_heads, p.batch);
    switch (p.head_dim) {
      case 32: tvk::launch_pdl(paged_decode_simt_kernel<T, 32>, grid, 128, 0, stream, p); break;
      case 64: tvk::launch_pdl(paged_decode_simt_kernel<T, 64>, grid, 128, 0, stream, p); break;
      default: tvk::launch_pdl(paged_decode_simt_kernel<T, 128>, grid, 128, 0, stream, p); break;
    }
    TVK_CHECK_LAUNCH("paged_decode_simt");
  }
  if (rc != TVK_OK) return rc;
  if (p.max_splits > 1) {
    const dim3 cgrid(p.n_kv_heads, p.batch);
    switch (p.head_dim) {
      case 32: tvk::launch_pdl(paged_decode_combine_kernel<T, 32>, cgrid, 128, 0, stream, p); break;
      case 64: tvk::launch_pdl(paged_decode_combine_kernel<T, 64>, cgrid, 128, 0, stream, p); break;
      default: tvk::launch_pdl(paged_decode_combine_kernel<T, 128>, cgrid, 128, 0, stream, p); break;
    }
    TVK_CHECK_LAUNCH("paged_decode_combine");
  }
  return TVK_OK;
}

}  // namespace

extern "C" size_t tvk_paged_decode_workspace_size(int batch, int n_heads, int n_kv_heads, int head_dim,
                                                  int block_size, int max_blocks, int max_context_len) {
  if (batch <= 0 || n_heads <= 0 || n_kv_heads <= 0 || head_dim <= 0 || block_size <= 0 || max_blocks <= 0)
    return tvk::kWorkspaceHeader;
  // The dtype is not known here: size for whichever plan needs more.
  const int tt = table_tokens(block_size, max_blocks, max_context_len);
  const Plan a = make_plan(batch, n_kv_heads, tt, false);
  const Plan b = make_plan(batch, n_kv_heads, tt, true);
  return workspace_bytes_for(batch, n_heads, head_dim, a.max_splits > b.max_splits ? a.max_splits : b.max_splits);
}

extern "C" int tvk_paged_decode_plan(int batch, int n_heads, int n_kv_heads, int head_dim, int block_size,
                                     int max_blocks, int max_context_len, int dtype, int* plan_out) {
  TVK_CHECK_ARG(plan_out, "null plan_out");
  TVK_CHECK_ARG(batch > 0 && n_heads > 0 && n_kv_heads > 0 && head_dim > 0 && block_size > 0 && max_blocks > 0,
                "sizes must be positive");
  const int tt = table_tokens(block_size, max_blocks, max_context_len);
  const bool tc_shape = (dtype != TVK_DTYPE_F32) &&
                        (block_size == 8 || block_size == 16 || block_size == 32 || block_size == 64);
  const Plan pl = make_plan(batch, n_kv_heads, tt, tc_shape);
  plan_out[0] = pl.split;
  plan_out[1] = pl.max_splits;
  plan_out[2] = pl.max_splits > 1 ? 2 : 1;
  plan_out[3] = pl.dynamic;
  return TVK_OK;
}

extern "C" int tvk_paged_decode_attention(const void* q, const void* k_cache, const void* v_cache,
                                          const int32_t* block_tables, const int32_t* context_lens, void* out,
                                          int batch, int n_heads, int n_kv_heads, int head_dim, int block_size,
                                          int num_blocks, int max_blocks, int max_context_len, int dtype,
                                          void* workspace, size_t workspace_bytes, void* stream) {
  TVK_CHECK_ARG(batch >= 0, "batch must be >= 0 (got %d)", batch);
  if (batch == 0) return TVK_OK;
  TVK_CHECK_ARG(q && k_cache && v_cache && block_tables && context_lens && out, "null pointer argument");
  TVK_CHECK_ARG(n_heads > 0 && n_kv_heads > 0 && n_heads % n_kv_heads == 0,
                "n_heads (%d) must be a positive multiple of n_kv_heads (%d)", n_heads, n_kv_heads);
  TVK_CHECK_ARG(n_heads / n_kv_heads <= kMaxGroup, "n_heads / n_kv_heads = %d exceeds %d", n_heads / n_kv_heads,
                kMaxGroup);
  TVK_CHECK_ARG(batch <= 65535 && n_kv_heads <= 65535, "batch and n_kv_heads must be <= 65535");
  TVK_CHECK_ARG((long long)batch * n_kv_heads * ((long long)max_blocks * block_size / 64 + 1) < 0x7fffffffLL,
                "batch x KV heads x table splits exceeds the 32-bit work index");
  TVK_CHECK_ARG(block_size > 0 && num_blocks > 0 && max_blocks > 0,
                "block_size, num_blocks and max_blocks must be positive");
  TVK_CHECK_ARG(dtype == TVK_DTYPE_F32 || dtype == TVK_DTYPE_F16 || dtype == TVK_DTYPE_BF16, "unknown dtype %d",
                dtype);
  if (head_dim != 32 && head_dim != 64 && head_dim != 128) {
    tvk::set_error("head_dim %d unsupported (32, 64 or 128)", head_dim);
    return TVK_ERR_UNSUPPORTED;
  }
  const size_t es = tvk::dtype_size(dtype);
  TVK_CHECK_ARG(((uintptr_t)q % 16 == 0) && ((uintptr_t)k_cache % 16 == 0) && ((uintptr_t)v_cache % 16 == 0) &&
                    ((uintptr_t)out % 4 == 0),
                "q, k_cache and v_cache must be 16-byte aligned");

  DecodeParams p{};
  p.q = q;
  p.out = out;
  p.block_tables = block_tables;
  p.context_lens = context_lens;
  p.k_cache = k_cache;
  p.v_cache = v_cache;
  p.batch = batch;
  p.n_heads = n_heads;
  p.n_kv_heads = n_kv_heads;
  p.group = n_heads / n_kv_heads;
  p.head_dim = head_dim;
  p.block_size = block_size;
  p.num_blocks = num_blocks;
  p.max_blocks = max_blocks;
  p.max_ctx_tokens = table_tokens(block_size, max_blocks, max_context_len);
  const bool tc_shape = (dtype != TVK_DTYPE_F32) &&
                        (block_size == 8 || block_size == 16 || block_size == 32 || block_size == 64);
  const Plan plan = make_plan(batch, n_kv_heads, p.max_ctx_tokens, tc_shape);
  p.split_tokens = plan.split;
  p.max_splits = plan.max_splits;
  p.scale_log2 = (float)(1.4426950408889634 / sqrt((double)head_dim));
  const tvk::WaitTest wt = tvk::take_wait_test();
  p.wait_ns = wt.armed ? wt.limit_ns : tvk::kDefaultWaitNs;
  p.drop_loads = wt.armed && tc_shape ? 1 : 0;

  const size_t need = workspace_bytes_for(batch, n_heads, head_dim, p.max_splits);
  if (p.max_splits > 1) {
    if (!workspace || workspace_bytes < need) {
      tvk::set_error("workspace of %zu bytes needed, %zu given", need, workspace ? workspace_bytes : (size_t)0);
      return TVK_ERR_WORKSPACE;
    }
  }
  if (workspace) {
    TVK_CHECK_ARG((uintptr_t)workspace % 16 == 0, "workspace must be 16-byte aligned");
    p.status = reinterpret_cast<int*>(workspace);
    p.sched = reinterpret_cast<uint8_t*>(workspace);
    float* f = reinterpret_cast<float*>(reinterpret_cast<uint8_t*>(workspace) + tvk::kWorkspaceHeader);
    p.part_o = f;
    p.part_ml = f + (size_t)batch * n_heads * p.max_splits * head_dim;
  }

  // The ticket counter and the device-side unit size need the header.
  p.dynamic = (plan.dynamic && p.sched) ? 1 : 0;
  p.device_split = p.dynamic;
  cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
  (void)es;
  switch (dtype) {
    case TVK_DTYPE_F16: return launch_typed<__half>(p, tc_shape, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, s);
    case TVK_DTYPE_BF16: return launch_typed<__nv_bfloat16>(p, tc_shape, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, s);
    default: return launch_typed<float>(p, false, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, s);
  }
}

// -----------------------------------------------------------------------------
// Paged decode without any device allocation.
//
// For callers that cannot allocate device memory for the split-K scratch: an
// engine that hands (nearly) all free HBM to its KV pool at start-up, as
// tinyvllm sizes its pool from free GPU memory, leaving no room for per-call
// buffers; a host binding (ctypes, cgo, JNI) that has no device allocator of
// its own; or a decode loop that cannot afford cudaMalloc's implicit device
// synchronisation.  This entry point uses a fixed scratch array compiled into
// the library instead of a caller workspace.
// -----------------------------------------------------------------------------
namespace {

// Every GPU that loads this library holds this array until the process exits.
// 64 MiB covers the split-K partials of 256 sequences x 32 heads x 4096-token
// tables at head_dim 128 (34 MB); larger calls are refused.
constexpr size_t kNoAllocScratchBytes = 64ull << 20;
__device__ __align__(256) uint8_t g_noalloc_scratch[kNoAllocScratchBytes];

constexpr int kNoAllocMaxDevices = 64;
std::mutex g_noalloc_mu;
void* g_noalloc_dev_ptr[kNoAllocMaxDevices] = {};

// Device address of the scratch array on the current device.  The host-side
// symbol `g_noalloc_scratch` is only a stand-in: passing it to a kernel would
// fault (or silently touch host memory), so the real address is looked up once
// per device with that device current.
int noalloc_scratch_ptr(void** out) {
  int dev = 0;
  TVK_CHECK_CUDA(cudaGetDevice(&dev));
  TVK_CHECK_ARG(dev >= 0 && dev < kNoAllocMaxDevices, "device %d beyond the %d supported", dev, kNoAllocMaxDevices);
  std::lock_guard<std::mutex> lock(g_noalloc_mu);
  if (!g_noalloc_dev_ptr[dev]) {
    void* p = nullptr;
    const cudaError_t e = cudaGetSymbolAddress(&p, g_noalloc_scratch);
    if (e != cudaSuccess || p == nullptr) {
      tvk::set_error("cudaGetSymbolAddress(g_noalloc_scratch) failed on device %d: %s", dev, cudaGetErrorString(e));
      return TVK_ERR_CUDA;
    }
    g_noalloc_dev_ptr[dev] = p;
  }
  *out = g_noalloc_dev_ptr[dev];
  return TVK_OK;
}

}  // namespace

extern "C" int tvk_paged_decode_attention_noalloc(const void* q, const void* k_cache, const void* v_cache,
                                                  const int32_t* block_tables, const int32_t* context_lens,
                                                  void* out, int batch, int n_heads, int n_kv_heads, int head_dim,
                                                  int block_size, int num_blocks, int max_blocks,
                                                  int max_context_len, int dtype, void* stream) {
  TVK_CHECK_ARG(batch >= 0, "batch must be >= 0 (got %d)", batch);
  if (batch == 0) return TVK_OK;
  const size_t need = tvk_paged_decode_workspace_size(batch, n_heads, n_kv_heads, head_dim, block_size, max_blocks,
                                                      max_context_len);
  if (need > kNoAllocScratchBytes) {
    tvk::set_error(
        "this call needs %zu bytes of split-K scratch; the no-allocation entry point has a fixed %zu bytes "
        "(use tvk_paged_decode_attention with a caller workspace)",
        need, kNoAllocScratchBytes);
    return TVK_ERR_WORKSPACE;
  }
  void* scratch = nullptr;
  const int rc = noalloc_scratch_ptr(&scratch);
  if (rc != TVK_OK) return rc;
  // The scratch keeps the previous call's contents; only the header (status
  // word and work-list counters) has to start at zero (the split-K partials
  // are written before they are read).
  TVK_CHECK_CUDA(cudaMemsetAsync(scratch, 0, tvk::kWorkspaceHeader, reinterpret_cast<cudaStream_t>(stream)));
  return tvk_paged_decode_attention(q, k_cache, v_cache, block_tables, context_lens, out, batch, n_heads, n_kv_heads,
                                    head_dim, block_size, num_blocks, max_blocks, max_context_len, dtype, scratch,
                                    kNoAllocScratchBytes, stream);
}

// Status word of the no-allocation entry point's scratch on the current device
// (byte 0 of the fixed array): waits for `stream`, then copies the word to the
// host.  Non-zero means a bounded wait inside the last call's kernel gave up and
// its output is incomplete.  The next no-allocation call clears the word.
extern "C" int tvk_paged_decode_noalloc_status(int* status, void* stream) {
  TVK_CHECK_ARG(status, "null status pointer");
  void* scratch = nullptr;
  const int rc = noalloc_scratch_ptr(&scratch);
  if (rc != TVK_OK) return rc;
  cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
  int word = 0;
  TVK_CHECK_CUDA(cudaMemcpyAsync(&word, scratch, sizeof(int), cudaMemcpyDeviceToHost, s));
  TVK_CHECK_CUDA(cudaStreamSynchronize(s));
  *status = word;
  return TVK_OK;
}
