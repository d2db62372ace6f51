// prefill_sm100.cu -- causal flash prefill with the fused paged K/V write.
//
// Replaces flash_prefill_attention (tinyvllm/model/llama.py:58-94) and the
// per-block K/V writes of Attention._write_kv_to_blocks (llama.py:188-209,
// core/kv_cache.py:34-38).  The reference materialises the whole [H, L, L]
// score matrix, expands GQA heads and masks after the full Q.K^T; here each CTA
// owns one 128-row query tile of one head of one prompt, walks only the key
// tiles at or below the diagonal, and never leaves the chip with scores.
//
// tcgen05 kernel (fp16/bf16, head_dim 64 or 128), 6 warps, persistent CTAs
// walking a heaviest-first list of (prompt, 128-row query tile, head) items:
//   warp 0  TMA producer: Q once per item, then 64-key K/V tiles into a ring;
//           for the two diagonal tiles (this query tile's own tokens) of the
//           first query head of a KV group it also copies the landed K/V rows
//           into their paged slots.
//   warp 1  owns TMEM and issues the MMAs from one thread: S(g) = Q.K(g)^T
//           (M=128, N=64, fp32, two TMEM buffers), then O += P(g-1).V(g-1)
//           (M=128, N=head_dim, A = P from TMEM, O in TMEM for the whole item),
//           so the next tile's scores are computed while the softmax works.
//   warps 2-5  softmax: one query row per thread, S read once with
//           tcgen05.ld, online softmax in the log2 domain with a lazy O
//           rescale, P packed to 16-bit pairs and stored to TMEM (two buffers).
// SIMT kernel (any dtype incl. fp32, head_dim 32/64/128): one warp per four
// query rows, fp32 CUDA-core math; also does the paged write.
#include <math.h>

#include <type_traits>

#include "tvk_common.cuh"
#include "sm100_umma.cuh"

namespace {

struct PrefillParams {
  const void* q;
  const void* k;
  const void* v;
  void* out;
  const int32_t* cu_seqlens;
  const int64_t* slot_mapping;  // may be null: no paged write
  void* k_cache;
  void* v_cache;
  int* status;                  // may be null
  const int4* sched;            // tc path: {seq, query tile, first token, length} items, heaviest first
  const int32_t* sched_count;   // tc path: number of entries in sched
  int* ticket;                  // tc path: next item to hand out (zeroed by the schedule kernel)
  int n_seqs, n_heads, n_kv_heads, group, head_dim, causal, num_blocks, block_size, n_mtiles;
  int total_tokens;
  int sched_cap;                // tc path: entries the schedule can hold
  float scale_log2;
  unsigned long long wait_ns;   // wall-time limit of every mbarrier wait
  int drop_loads;               // wait-limit test: the producer loads nothing, so waits run out
};

__device__ __forceinline__ void report(int* status) {
  if (status) atomicExch(status, tvk::kStatusWaitTimeout);
}

// Bounded mbarrier wait shared by all roles of a CTA: gives up after 2 s, or at
// once when another thread of the CTA already gave up (abort flag in smem).
__device__ __forceinline__ bool wait_or_abort(uint64_t* bar, uint32_t parity, volatile int* abort_flag,
                                              uint64_t limit_ns = 2000000000ull) {
  if (ptx::mbar_try_wait(bar, parity)) return true;
  const uint64_t t0 = ptx::globaltimer();
  while (true) {
    if (ptx::mbar_try_wait(bar, parity)) return true;
    if (*abort_flag) return false;
    if (ptx::globaltimer() - t0 > limit_ns) {
      *abort_flag = 1;
      return false;
    }
  }
}

__device__ __forceinline__ void tma_load_3d(void* dst, const CUtensorMap* m, uint64_t* bar, int c0, int c1, int c2) {
  asm volatile(
      "cp.async.bulk.tensor.3d.shared::cluster.global.tile.mbarrier::complete_tx::bytes"
      " [%0], [%1, {%2, %3, %4}], [%5];" ::"r"(ptx::smem_u32(dst)),
      "l"(reinterpret_cast<uint64_t>(m)), "r"(c0), "r"(c1), "r"(c2), "r"(ptx::smem_u32(bar))
      : "memory");
}

// Hardware 2^x (ex2.approx, flush-to-zero): the softmax's exponentials.
__device__ __forceinline__ float ex2(float x) {
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}

// max(a, b, c) in one instruction (sm_100).
__device__ __forceinline__ float max3f(float a, float b, float c) {
  float d;
  asm("max.f32 %0, %1, %2, %3;" : "=f"(d) : "f"(a), "f"(b), "f"(c));
  return d;
}

// (a0, a1) * b + c on the paired fp32 pipe: two results per instruction.
__device__ __forceinline__ void fma2(float& d0, float& d1, float a0, float a1, float b, float c) {
  uint64_t A, B, Cc, Dd;
  asm("mov.b64 %0, {%1, %2};" : "=l"(A) : "f"(a0), "f"(a1));
  asm("mov.b64 %0, {%1, %1};" : "=l"(B) : "f"(b));
  asm("mov.b64 %0, {%1, %1};" : "=l"(Cc) : "f"(c));
  asm("fma.rn.f32x2 %0, %1, %2, %3;" : "=l"(Dd) : "l"(A), "l"(B), "l"(Cc));
  asm("mov.b64 {%0, %1}, %2;" : "=f"(d0), "=f"(d1) : "l"(Dd));
}

template <int D>
struct PfCfg {
  static constexpr int kKB = D / 64;                  // 64-element (128 B) column blocks per row
  static constexpr int kQBlockBytes = 128 * 128;      // one column block of the 128-row Q tile
  static constexpr int kQBytes = 128 * D * 2;
  static constexpr int kKvRows = 64;                  // keys per K/V tile
  static constexpr int kKvBlockBytes = kKvRows * 128; // one column block of a 64-row K or V tile
  static constexpr int kKvBytes = kKvRows * D * 2;
  // P.V runs with N = head_dim + 16: the extra B columns are a block of ones,
  // so O's column head_dim accumulates the row sum of P on the tensor cores.
  // In the MN-major V operand the ones are one more 64-column block at the
  // descriptor's block stride: after each stage's V tile at head_dim 128, one
  // shared block after all stages at head_dim 64 (stride = its distance).
  static constexpr int kVStageBytes = D == 128 ? kKvBytes + kKvBlockBytes : kKvBytes;
  static constexpr int kStages = 4;                   // K/V ring depth (64-key tiles)
  // two Q tiles: the next item's Q loads while this item's last scores compute
  static constexpr int kQSlots = 2;
  static constexpr int kQOff = 0;
  static constexpr int kKOff = kQOff + kQSlots * kQBytes;
  static constexpr int kVOff = kKOff + kStages * kKvBytes;
  static constexpr int kOnesOff = kVOff + kStages * kVStageBytes;  // head_dim 64 only
  static constexpr int kBarOff = kOnesOff + (D == 64 ? kKvBlockBytes : 0);
  // q_full[2], q_empty[2], k_full[S], v_full[S], kv_empty[S], s_full[2], p_full[2], pv_done[2], o_empty, final,
  // item_full[4], item_empty[4]
  static constexpr int kItemSlots = 4;
  static constexpr int kNumBars = 2 * kQSlots + 3 * kStages + 6 + 2 + 2 * kItemSlots;
  static constexpr int kMiscOff = kBarOff + kNumBars * 8;  // tmem slot, abort flag, item ring
  static constexpr int kUsed = kMiscOff + 16 + 32 * kItemSlots;  // 8 ints per ring slot
  // head_dim 64: at most 113 KB so that two CTAs share an SM
  // (2 x (113 + 1 reserved) KB = 228 KB); the slack above kUsed absorbs the
  // 1024-byte alignment of the base.
  static constexpr int kCtasPerSm = D == 64 ? 2 : 1;
  static constexpr int kSmemBytes = kUsed + 1024;
  static_assert(D != 64 || kSmemBytes <= 115712, "two CTAs per SM at head_dim 64");
  static_assert(kSmemBytes <= 232448, "shared memory per CTA");
  // TMEM columns: two S buffers of 64 fp32 columns (64 keys); once a tile's
  // scores are in registers its P (64 keys as 32 columns of packed 16-bit
  // pairs, the A operand of P.V) is written over the first half of the same
  // buffer.  Then O: head_dim columns plus the row-sum column (and 15 unused).
  static constexpr uint32_t kSCol = 0;
  static constexpr uint32_t kOCol = 128;
  static constexpr int kOCols = D + 16;
  static constexpr uint32_t kTmemCols = kOCol + kOCols <= 256 ? 256 : 512;
};

// One unit of work: a 128-row query tile of one head of one prompt.
struct Item {
  int seq, mtile, h, s0, L;
};

// Item w of the schedule: query tiles sorted heaviest first, each expanded
// over the query heads.  CTAs take items from the ticket counter as they free
// up, so the heavy items start first and the light ones fill the gaps.  The
// schedule and the prompt offsets are read through L2 (the schedule kernel,
// and possibly other work before it, wrote them while this grid was already
// running its prologue); an entry that does not describe a query tile of a
// prompt inside the token range comes back with seq = -1.
__device__ __forceinline__ Item item_of(const PrefillParams& p, int w) {
  const int4 e = __ldcg(p.sched + w / p.n_heads);
  const int seq = e.x, m = e.y, s0 = e.z, L = e.w;
  if (seq < 0 || seq >= p.n_seqs || m < 0 || m >= p.n_mtiles) return Item{-1, 0, 0, 0, 0};
  if (s0 < 0 || L <= m * 128 || s0 + L > p.total_tokens) return Item{-1, 0, 0, 0, 0};
  return Item{seq, m, w % p.n_heads, s0, L};
}

// 64-key tiles an item visits: up to and including the diagonal when causal.
__device__ __forceinline__ int kv_tiles(const PrefillParams& p, const Item& it) {
  const int all = (it.L + 63) / 64;
  return p.causal ? min(2 * it.mtile + 2, all) : all;
}

template <typename T, int D>
__global__ void __launch_bounds__(192, PfCfg<D>::kCtasPerSm)
    flash_prefill_tc_kernel(const PrefillParams p, const __grid_constant__ CUtensorMap tm_q,
                            const __grid_constant__ CUtensorMap tm_k, const __grid_constant__ CUtensorMap tm_v) {
  using C = PfCfg<D>;
  constexpr int S = C::kStages;
  constexpr bool kBf16 = std::is_same<T, __nv_bfloat16>::value;

  extern __shared__ uint8_t smem_raw[];
  const uint32_t raw_u32 = ptx::smem_u32(smem_raw);
  const uint32_t base_u32 = (raw_u32 + 1023u) & ~1023u;
  if (base_u32 + C::kUsed > raw_u32 + C::kSmemBytes) {  // cannot happen with a >=16 B aligned base
    if (threadIdx.x == 0) report(p.status);
    return;
  }
  uint8_t* base = smem_raw + (base_u32 - raw_u32);
  uint64_t* q_full = reinterpret_cast<uint64_t*>(base + C::kBarOff);
  uint64_t* q_empty = q_full + C::kQSlots;
  uint64_t* k_full = q_empty + C::kQSlots;
  uint64_t* v_full = k_full + S;
  uint64_t* kv_empty = v_full + S;
  uint64_t* s_full = kv_empty + S;
  uint64_t* p_full = s_full + 2;
  uint64_t* pv_done = p_full + 2;
  uint64_t* o_empty = pv_done + 2;
  uint64_t* final_bar = o_empty + 1;
  uint64_t* item_full = final_bar + 1;
  uint64_t* item_empty = item_full + C::kItemSlots;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(base + C::kMiscOff);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(base + C::kMiscOff + 4);
  volatile int* item_ring = reinterpret_cast<volatile int*>(base + C::kMiscOff + 16);  // [slot][8]

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  if (warp == 1) {
    umma::tmem_alloc(tmem_slot, C::kTmemCols);
    umma::tmem_relinquish();
  }
  if (threadIdx.x == 0) {
    for (int i = 0; i < C::kQSlots; ++i) {
      ptx::mbar_init(&q_full[i], 1);
      ptx::mbar_init(&q_empty[i], 1);
    }
    for (int s = 0; s < S; ++s) {
      ptx::mbar_init(&k_full[s], 1);
      ptx::mbar_init(&v_full[s], 1);
      ptx::mbar_init(&kv_empty[s], 1);
    }
    for (int b = 0; b < 2; ++b) {
      ptx::mbar_init(&s_full[b], 1);
      ptx::mbar_init(&p_full[b], 4);
      ptx::mbar_init(&pv_done[b], 1);
    }
    ptx::mbar_init(o_empty, 4);
    ptx::mbar_init(final_bar, 1);
    for (int i = 0; i < C::kItemSlots; ++i) {
      ptx::mbar_init(&item_full[i], 1);
      ptx::mbar_init(&item_empty[i], 5);  // the MMA thread and the four softmax warps
    }
    *abort_flag = 0;
    ptx::fence_mbar_init();
  }
  {
    // the ones block(s) of the row-sum columns, read by the tensor cores
    const uint32_t one2 = std::is_same<T, __half>::value ? 0x3C003C00u : 0x3F803F80u;
    constexpr int kOnesBlocks = D == 64 ? 1 : S;
    for (int i = threadIdx.x; i < kOnesBlocks * C::kKvBlockBytes / 16; i += blockDim.x) {
      const int blk = i / (C::kKvBlockBytes / 16), w = i % (C::kKvBlockBytes / 16);
      const int off = D == 64 ? C::kOnesOff : C::kVOff + blk * C::kVStageBytes + C::kKvBytes;
      reinterpret_cast<uint4*>(base + off)[w] = make_uint4(one2, one2, one2, one2);
    }
    umma::fence_proxy_async_smem();
  }
  umma::fence_before_sync();
  __syncthreads();
  umma::fence_after_sync();
  const uint32_t tmem = *tmem_slot;
  // The schedule kernel runs just before this one (programmatic dependent
  // launch): everything above overlapped it; its list and counter are read below.
  asm volatile("griddepcontrol.wait;" ::: "memory");
  const int n_items = min(__ldcg(p.sched_count), p.sched_cap) * p.n_heads;
  // Items reach the MMA and softmax warps, decoded, through a small ring that
  // the producer fills from the ticket counter; seq -1 ends the list.
  uint32_t n_seen = 0;
  auto take_item = [&](Item& it, bool arrive) -> int {  // 1: item, 0: end of list, -1: gave up
    const int slot = n_seen % C::kItemSlots;
    if (!wait_or_abort(&item_full[slot], (n_seen / C::kItemSlots) & 1, abort_flag, p.wait_ns)) return -1;
    volatile int* e = item_ring + slot * 8;
    it = Item{e[0], e[1], e[2], e[3], e[4]};
    if (arrive) ptx::mbar_arrive(&item_empty[slot]);
    ++n_seen;
    return it.seq < 0 ? 0 : 1;
  };

  if (warp == 0) {
    // =========================== TMA producer ===============================
    uint32_t kv_it = 0, q_it = 0;
    bool ok = true;
    if (lane == 0) {
      ptx::prefetch_tmap(&tm_q);
      ptx::prefetch_tmap(&tm_k);
      ptx::prefetch_tmap(&tm_v);
    }
    const long long n_slots = (long long)p.num_blocks * p.block_size;
    uint32_t n_claim = 0;
    Item it{};
    while (ok) {
      const int slot = n_claim % C::kItemSlots;
      int w = 0;
      if (lane == 0) w = (int)atomicAdd(p.ticket, 1);
      w = __shfl_sync(0xffffffffu, w, 0);
      if (w >= n_items) w = -1;
      if (w >= 0) {
        it = item_of(p, w);
        if (it.seq < 0) {  // a corrupt schedule entry: stop here and say so
          report(p.status);
          w = -1;
        }
      }
      ok = __all_sync(0xffffffffu, wait_or_abort(&item_empty[slot], ((n_claim / C::kItemSlots) & 1) ^ 1, abort_flag, p.wait_ns));
      if (!ok) break;
      if (lane == 0) {
        volatile int* e = item_ring + slot * 8;
        e[0] = w < 0 ? -1 : it.seq;
        e[1] = it.mtile;
        e[2] = it.h;
        e[3] = it.s0;
        e[4] = it.L;
        ptx::mbar_arrive(&item_full[slot]);
      }
      ++n_claim;
      if (w < 0) break;
      if (p.drop_loads) break;  // test hook: the item's Q and K/V never arrive
      const int n_kv = kv_tiles(p, it);
      const int kvh = it.h / p.group;
      const int qs = q_it % C::kQSlots;
      ok = __all_sync(0xffffffffu, wait_or_abort(&q_empty[qs], ((q_it / C::kQSlots) & 1) ^ 1, abort_flag, p.wait_ns));
      if (!ok) break;
      if (lane == 0) {
        ptx::mbar_arrive_expect_tx(&q_full[qs], C::kQBytes);
        for (int kb = 0; kb < C::kKB; ++kb)
          tma_load_3d(base + C::kQOff + qs * C::kQBytes + kb * C::kQBlockBytes, &tm_q, &q_full[qs], kb * 64, it.h,
                      it.s0 + it.mtile * 128);
      }
      ++q_it;
      const bool write_kv = p.slot_mapping != nullptr && (it.h % p.group) == 0;
      for (int j = 0; j < n_kv; ++j, ++kv_it) {
        const int st = kv_it % S;
        const uint32_t ph = (kv_it / S) & 1;
        ok = __all_sync(0xffffffffu, wait_or_abort(&kv_empty[st], ph ^ 1, abort_flag, p.wait_ns));
        if (!ok) break;
        uint8_t* ks = base + C::kKOff + st * C::kKvBytes;
        uint8_t* vs = base + C::kVOff + st * C::kVStageBytes;
        if (lane == 0) {
          ptx::mbar_arrive_expect_tx(&k_full[st], C::kKvBytes);
          for (int kb = 0; kb < C::kKB; ++kb)
            tma_load_3d(ks + kb * C::kKvBlockBytes, &tm_k, &k_full[st], kb * 64, kvh, it.s0 + j * 64);
          ptx::mbar_arrive_expect_tx(&v_full[st], C::kKvBytes);
          for (int kb = 0; kb < C::kKB; ++kb)
            tma_load_3d(vs + kb * C::kKvBlockBytes, &tm_v, &v_full[st], kb * 64, kvh, it.s0 + j * 64);
        }
        if (write_kv && (j >> 1) == it.mtile) {
          // The two diagonal tiles hold exactly this query tile's own tokens: copy
          // the landed rows into their paged slots (slot = block * block_size + offset).
          ok = __all_sync(0xffffffffu, wait_or_abort(&k_full[st], ph, abort_flag, p.wait_ns) &&
                                           wait_or_abort(&v_full[st], ph, abort_flag, p.wait_ns));
          if (!ok) break;
          const int tok0 = it.s0 + j * 64, rows = min(64, it.L - j * 64);
          T* kc = reinterpret_cast<T*>(p.k_cache);
          T* vc = reinterpret_cast<T*>(p.v_cache);
          // one slot per lane for rows lane and lane + 32, shared by shuffles
          const long long slot_lo = lane < rows ? __ldcg(p.slot_mapping + tok0 + lane) : -1;
          const long long slot_hi = lane + 32 < rows ? __ldcg(p.slot_mapping + tok0 + lane + 32) : -1;
          for (int i0 = 0; i0 < rows * (D / 8); i0 += 32) {
            const int i = i0 + lane;
            const int r = i / (D / 8), c8 = i % (D / 8);
            const long long a = __shfl_sync(0xffffffffu, slot_lo, r & 31);
            const long long b = __shfl_sync(0xffffffffu, slot_hi, r & 31);
            const long long slot = r < 32 ? a : b;
            if (i >= rows * (D / 8) || slot < 0 || slot >= n_slots) continue;
            const uint32_t off = (c8 / 8) * C::kKvBlockBytes + r * 128 + ((((c8 & 7) ^ (r & 7))) << 4);
            const size_t dst = ((size_t)slot * p.n_kv_heads + kvh) * D + c8 * 8;
            *reinterpret_cast<uint4*>(kc + dst) = *reinterpret_cast<const uint4*>(ks + off);
            *reinterpret_cast<uint4*>(vc + dst) = *reinterpret_cast<const uint4*>(vs + off);
          }
        }
      }
    }
    if (!ok) report(p.status);
    // Do not leave with copies in flight: the last issued loads must have landed.
    if (lane == 0) {
      for (uint32_t j = kv_it >= (uint32_t)S ? kv_it - S : 0; j < kv_it; ++j) {
        ptx::mbar_wait(&k_full[j % S], (j / S) & 1, 100000000ull);
        ptx::mbar_wait(&v_full[j % S], (j / S) & 1, 100000000ull);
      }
      for (uint32_t j = q_it >= (uint32_t)C::kQSlots ? q_it - C::kQSlots : 0; j < q_it; ++j)
        ptx::mbar_wait(&q_full[j % C::kQSlots], (j / C::kQSlots) & 1, 100000000ull);
    }
  } else if (warp == 1) {
    // =========================== MMA issuer =================================
    // Order per tile g: S(g) = Q.K(g)^T into TMEM buffer g%2, then O += P(g-1).V(g-1),
    // so the next tile's scores are computed while the softmax works on this one.
    // Buffer g%2 holds P(g-2) until that P.V completes, so S(g) waits for it.
    if (lane == 0) {
      const uint32_t idesc_s = umma::idesc_f16(128, 64, kBf16, false);
      const uint32_t idesc_o = umma::idesc_f16(128, C::kOCols, kBf16, true);
      uint32_t g = 0, q_it = 0, item_it = 0;
      bool ok = true;
      Item it;
      auto issue_pv = [&](uint32_t gg, bool first) -> bool {
        const int st = gg % S;
        const int pb = gg & 1;
        if (!wait_or_abort(&p_full[pb], (gg >> 1) & 1, abort_flag, p.wait_ns)) return false;
        if (first && !wait_or_abort(o_empty, (item_it & 1) ^ 1, abort_flag, p.wait_ns)) return false;
        if (!wait_or_abort(&v_full[st], (gg / S) & 1, abort_flag, p.wait_ns)) return false;
        umma::fence_after_sync();
        const uint32_t v_addr = base_u32 + C::kVOff + st * C::kVStageBytes;
        const uint32_t lbo = D == 64 ? (uint32_t)(C::kOnesOff - (C::kVOff + st * C::kVStageBytes)) : C::kKvBlockBytes;
#pragma unroll
        for (int ks = 0; ks < 4; ++ks) {  // 16 keys per MMA: 8 TMEM columns of P
          const uint64_t bd = umma::smem_desc_sw128(v_addr + ks * 2048, lbo, 1024);
          umma::mma_f16_ts(tmem + C::kOCol, tmem + C::kSCol + pb * 64 + ks * 8, bd, idesc_o,
                           (first && ks == 0) ? 0u : 1u);
        }
        umma::commit(&pv_done[pb]);
        umma::commit(&kv_empty[st]);
        return true;
      };
      while (ok) {
        const int got = take_item(it, true);
        if (got <= 0) {
          ok = got == 0;
          break;
        }
        const int n_kv = kv_tiles(p, it);
        const int qs = q_it % C::kQSlots;
        const uint32_t q_addr = base_u32 + C::kQOff + qs * C::kQBytes;
        ok = wait_or_abort(&q_full[qs], (q_it / C::kQSlots) & 1, abort_flag, p.wait_ns);
        for (int j = 0; ok && j < n_kv; ++j, ++g) {
          const int st = g % S;
          const int sb = g & 1;
          ok = wait_or_abort(&k_full[st], (g / S) & 1, abort_flag, p.wait_ns) &&
               wait_or_abort(&pv_done[sb], ((g >> 1) & 1) ^ 1, abort_flag, p.wait_ns);
          if (!ok) break;
          umma::fence_after_sync();
          const uint32_t k_addr = base_u32 + C::kKOff + st * C::kKvBytes;
#pragma unroll
          for (int ks = 0; ks < D / 16; ++ks) {
            const uint64_t ad =
                umma::smem_desc_sw128(q_addr + (ks >> 2) * C::kQBlockBytes + (ks & 3) * 32, 16, 1024);
            const uint64_t bd =
                umma::smem_desc_sw128(k_addr + (ks >> 2) * C::kKvBlockBytes + (ks & 3) * 32, 16, 1024);
            umma::mma_f16_ss(tmem + C::kSCol + sb * 64, ad, bd, idesc_s, ks > 0 ? 1u : 0u);
          }
          umma::commit(&s_full[sb]);
          if (j == n_kv - 1) umma::commit(&q_empty[qs]);  // Q is free once this item's S MMAs are done
          if (j >= 1) ok = issue_pv(g - 1, j == 1);
        }
        if (ok) ok = issue_pv(g - 1, n_kv == 1);
        ++q_it;
        ++item_it;
      }
      if (!ok) report(p.status);
      // Drain: every MMA issued so far completes before TMEM is released.
      umma::commit(final_bar);
      ptx::mbar_wait(final_bar, 0, 100000000ull);
    }
    __syncwarp();
  } else {
    // =========================== softmax warps ==============================
    const int quarter = warp & 3;  // TMEM lane quarter this warp may access
    const int r = quarter * 32 + lane;
    const uint32_t t_lane = tmem + ((uint32_t)(quarter * 32) << 16);
    const float sl2 = p.scale_log2;
    uint32_t g = 0;  // K/V tiles seen by this CTA (S, P and P.V buffers follow it)
    bool ok = true;
    Item it;
    // wait until O += P(gg).V(gg) has completed
    auto wait_pv = [&](uint32_t gg) -> bool {
      return __all_sync(0xffffffffu, wait_or_abort(&pv_done[gg & 1], (gg >> 1) & 1, abort_flag, p.wait_ns));
    };
    while (ok) {
      int got = take_item(it, false);
      ok = __all_sync(0xffffffffu, got >= 0);
      if (!ok) break;
      __syncwarp();
      if (lane == 0) ptx::mbar_arrive(&item_empty[(n_seen - 1) % C::kItemSlots]);
      if (got == 0) break;
      const int n_kv = kv_tiles(p, it);
      const int q_pos = it.mtile * 128 + r;
      const int lim = p.causal ? min(q_pos + 1, it.L) : it.L;  // keys [0, lim) are visible
      float m = -INFINITY;  // running max (log2 domain) that P and O are scaled by
      for (int j = 0; j < n_kv; ++j, ++g) {
        const int sb = g & 1;
        ok = __all_sync(0xffffffffu, wait_or_abort(&s_full[sb], (g >> 1) & 1, abort_flag, p.wait_ns));
        if (!ok) break;
        umma::fence_after_sync();
        float s[64];
        umma::ld_32x32b_x32(t_lane + C::kSCol + sb * 64, *reinterpret_cast<float(*)[32]>(&s[0]));
        umma::ld_32x32b_x32(t_lane + C::kSCol + sb * 64 + 32, *reinterpret_cast<float(*)[32]>(&s[32]));
        umma::ld_wait();

        const int lim_rel = lim - j * 64;  // keys [0, lim_rel) of this tile are visible
        if (__any_sync(0xffffffffu, lim_rel < 64)) {
#pragma unroll
          for (int x = 0; x < 64; ++x) s[x] = x < lim_rel ? s[x] : -INFINITY;
        }
        // row max: eight independent partial maxima, three inputs per instruction
        float mp[8];
#pragma unroll
        for (int i = 0; i < 8; ++i) {
          mp[i] = max3f(s[i], s[8 + i], s[16 + i]);
          mp[i] = max3f(mp[i], s[24 + i], s[32 + i]);
          mp[i] = max3f(mp[i], s[40 + i], s[48 + i]);
          mp[i] = fmaxf(mp[i], s[56 + i]);
        }
        const float mx = max3f(max3f(mp[0], mp[1], mp[2]), max3f(mp[3], mp[4], mp[5]), fmaxf(mp[6], mp[7]));
        float m_cand = fmaxf(m, mx * sl2);
        if (m_cand == -INFINITY) m_cand = 0.f;  // no visible key (cannot happen for a live tile)
        if (j == 0) {
          m = m_cand;
        } else if (__any_sync(0xffffffffu, m_cand > m + 8.f)) {
          // Lazy rescale: the stale max is kept unless the new one is 2^8 larger.
          // O is stable once the previous tile's P.V is done (this tile's needs P).
          ok = wait_pv(g - 1);
          if (!ok) break;
          umma::fence_after_sync();
          const float corr = ex2(m - m_cand);
#pragma unroll
          for (int c = 0; c < (C::kOCols + 31) / 32; ++c) {  // O and its row-sum column
            float o[32];
            umma::ld_32x32b_x32(t_lane + C::kOCol + c * 32, o);
            umma::ld_wait();
#pragma unroll
            for (int x = 0; x < 32; ++x) o[x] *= corr;
            umma::st_32x32b_x32(t_lane + C::kOCol + c * 32, o);
          }
          umma::st_wait();
          m = m_cand;
        }
        // P = 2^(s*scale - m), packed to 16-bit pairs (row r = lane, 32 columns
        // for 64 keys): the A operand of P.V
        // (the row sum comes from the ones column of P.V)
        uint32_t pk[32];
#pragma unroll
        for (int x = 0; x < 32; ++x) {
          float x0, x1;
          fma2(x0, x1, s[2 * x], s[2 * x + 1], sl2, -m);
          pk[x] = DT<T>::pack2(ex2(x0), ex2(x1));
        }
        // P(g) overwrites the scores of tile g; S(g) has been read and the P.V of
        // tile g-2, the buffer's previous P, completed before S(g) was issued.
        umma::st_32x32b_x32_u(t_lane + C::kSCol + sb * 64, pk);
        umma::st_wait();
        umma::fence_before_sync();
        __syncwarp();
        if (lane == 0) ptx::mbar_arrive(&p_full[sb]);
      }
      if (!ok) break;
      // ---- item done: O (TMEM) / l -> out
      ok = wait_pv(g - 1);
      if (!ok) break;
      umma::fence_after_sync();
      float l;
      {
        float o[32];
        umma::ld_32x32b_x32(t_lane + C::kOCol + D, o);
        umma::ld_wait();
        l = o[0];
      }
      const float inv = l > 0.f ? 1.f / l : 0.f;
      T* orow = reinterpret_cast<T*>(p.out) + ((size_t)(it.s0 + q_pos) * p.n_heads + it.h) * D;
#pragma unroll
      for (int c = 0; c < D / 32; ++c) {
        float o[32];
        umma::ld_32x32b_x32(t_lane + C::kOCol + c * 32, o);
        umma::ld_wait();
        if (q_pos < it.L) {
#pragma unroll
          for (int c8 = 0; c8 < 4; ++c8) {
            uint4 w;
            w.x = DT<T>::pack2(o[c8 * 8 + 0] * inv, o[c8 * 8 + 1] * inv);
            w.y = DT<T>::pack2(o[c8 * 8 + 2] * inv, o[c8 * 8 + 3] * inv);
            w.z = DT<T>::pack2(o[c8 * 8 + 4] * inv, o[c8 * 8 + 5] * inv);
            w.w = DT<T>::pack2(o[c8 * 8 + 6] * inv, o[c8 * 8 + 7] * inv);
            *reinterpret_cast<uint4*>(orow + c * 32 + c8 * 8) = w;
          }
        }
      }
      umma::fence_before_sync();
      __syncwarp();
      if (lane == 0) ptx::mbar_arrive(o_empty);
    }
    if (!ok) report(p.status);
  }

  umma::fence_before_sync();
  __syncthreads();
  if (warp == 1) {
    umma::fence_after_sync();
    umma::tmem_dealloc(tmem, C::kTmemCols);
  }
}

// -----------------------------------------------------------------------------
// Paired-head tcgen05 kernel (fp16/bf16, head_dim 64 or 128, an even number of
// query heads per KV head).  One CTA per SM walks the heaviest-first item list;
// an item is one 128-row query tile of a PAIR of query heads (h, h+1) that read
// the same KV head, so every K/V tile is loaded once for both.  Keys come in
// tiles of 128.  16 warps in four warpgroups:
//   warp 0      TMA producer: both heads' Q tiles once per item, then the K/V
//               ring; copies the diagonal tile's landed K/V rows into their
//               paged slots when the pair holds the KV group's first head.
//   warp 1      TMEM owner; issues S_t = Q_t.K^T for both heads t = 0, 1
//               (M=128, N=128) from one thread.
//   warps 2, 3  issue O_t += P_t.V for head 0 and head 1 (A = P_t from TMEM,
//               N = head_dim).  One thread issues an MMA about every 130
//               cycles whatever its size, so the three issuers keep the tensor
//               pipe fed where one could not (a key tile is 24 MMAs).
//   warps 4-7   softmax of head h, warps 8-11 softmax of head h+1: one query
//               row per thread, 128 scores per key tile in registers, online
//               softmax in the log2 domain with a lazy O rescale, P packed to
//               16-bit pairs into TMEM, row sums in fp32 registers handed to
//               the epilogue warps at the end of an item.
//               Warps 4+q and 8+q share scheduler q and its exponential unit
//               (16 results per cycle per SM, the floor at head_dim 64); they
//               take turns on it tile by tile (exp_turn barriers), so one head
//               stores P and waits for its next scores while the other
//               exponentiates, instead of both leaving the unit idle at once.
//   warps 12-15 epilogue: once a head's last P.V of an item completes, O / l
//               is read from TMEM and stored, while the softmax warps already
//               work on the next item.
// TMEM columns, head_dim 64:  S0 0-127, S1 128-255, P0 256-319, P1 320-383,
//                              O0 384-447, O1 448-511 (P apart from S, so the
//                              next S never waits for the previous P.V).
//              head_dim 128: S0 0-127 (P0 over its first 64), S1 128-255 (P1),
//                              O0 256-383, O1 384-511.
// -----------------------------------------------------------------------------
template <int D>
struct PairCfg {
  static constexpr int kKB = D / 64;                    // 64-element (128 B) column blocks
  static constexpr int kRows = 128;                     // query rows per tile = keys per K/V tile
  static constexpr int kBlockBytes = kRows * 128;       // one column block of a 128-row tile
  static constexpr int kTileBytes = kRows * D * 2;      // one 128-row tile (Q of one head, K or V)
  static constexpr int kQBufs = D == 64 ? 2 : 1;        // Q buffers (items in flight), two heads each
  static constexpr int kStages = D == 64 ? 4 : 2;       // K/V ring depth
  static constexpr int kQOff = 0;
  static constexpr int kKOff = kQOff + kQBufs * 2 * kTileBytes;
  static constexpr int kVOff = kKOff + kStages * kTileBytes;
  static constexpr int kBarOff = kVOff + kStages * kTileBytes;
  static constexpr int kItemSlots = 4;
  // q_full[QB], q_empty[QB], k_full[S], v_full[S], k_empty[S], v_empty[S], s_full[2], s_free[2], p_full[2],
  // pv_done[2], o_empty[2], final[3], item_full[4], item_empty[4], exp_turn[4][2], epi_ready[2][2],
  // item_started
  static constexpr int kNumBars = 2 * kQBufs + 4 * kStages + 10 + 3 + 2 * kItemSlots + 8 + 4 + 1;
  static constexpr int kMiscOff = kBarOff + kNumBars * 8;
  static constexpr int kLOff = kMiscOff + 16 + 32 * kItemSlots;  // row sums for the epilogue [2][2][128]
  static constexpr int kUsed = kLOff + 2 * 2 * 128 * 4;
  static constexpr int kSmemBytes = kUsed + 1024;
  static_assert(kSmemBytes <= 232448, "shared memory per CTA");
  static constexpr bool kPAlias = D == 128;             // P written over the first half of its S
  static constexpr uint32_t kTmemCols = 512;
  static constexpr int kThreads = 512;
  // register split (setmaxnreg): warpgroup 0 drops to kRegsLow, the epilogue
  // warpgroup to kRegsEpi, the two softmax warpgroups rise to kRegsHigh; the
  // launch must provide 512 x kRegsLaunchMin.
  static constexpr int kRegsLow = 56, kRegsEpi = 56, kRegsHigh = 192;
  static constexpr int kRegsLaunchMin = (128 * kRegsLow + 128 * kRegsEpi + 256 * kRegsHigh + kThreads - 1) / kThreads;
};

__device__ __forceinline__ uint32_t pcol(int D, int t) {
  return D == 128 ? (t ? 128u : 0u) : (t ? 320u : 256u);
}
__device__ __forceinline__ uint32_t ocol(int D, int t) {
  return D == 128 ? (t ? 384u : 256u) : (t ? 448u : 384u);
}

// One unit of work of the paired kernel: a 128-row query tile of heads (h0, h0+1).
struct PairItem {
  int seq, mtile, h0, s0, L;
};

__device__ __forceinline__ PairItem pair_item_of(const PrefillParams& p, int w) {
  const int n_pairs = p.n_heads >> 1;
  if (w < 0 || w / n_pairs >= p.sched_cap) return PairItem{-1, 0, 0, 0, 0};
  const int4 e = __ldcg(p.sched + w / n_pairs);
  const int seq = e.x, m = e.y, s0 = e.z, L = e.w;
  if (seq < 0 || seq >= p.n_seqs || m < 0 || m >= p.n_mtiles) return PairItem{-1, 0, 0, 0, 0};
  if (s0 < 0 || L <= m * 128 || s0 + L > p.total_tokens) return PairItem{-1, 0, 0, 0, 0};
  return PairItem{seq, m, 2 * (w % n_pairs), s0, L};
}

// 128-key tiles an item visits: up to and including the diagonal when causal.
__device__ __forceinline__ int pair_kv_tiles(const PrefillParams& p, const PairItem& it) {
  const int all = (it.L + 127) / 128;
  return p.causal ? min(it.mtile + 1, all) : all;
}

__device__ __forceinline__ void add2(float& a0, float& a1, float b0, float b1) {
  uint64_t A, B, Dd;
  asm("mov.b64 %0, {%1, %2};" : "=l"(A) : "f"(a0), "f"(a1));
  asm("mov.b64 %0, {%1, %2};" : "=l"(B) : "f"(b0), "f"(b1));
  asm("add.rn.f32x2 %0, %1, %2;" : "=l"(Dd) : "l"(A), "l"(B));
  asm("mov.b64 {%0, %1}, %2;" : "=f"(a0), "=f"(a1) : "l"(Dd));
}

// (a0, a1) + (b, b) on the paired fp32 pipe.
__device__ __forceinline__ void add2s(float& d0, float& d1, float a0, float a1, float b) {
  uint64_t A, B, Dd;
  asm("mov.b64 %0, {%1, %2};" : "=l"(A) : "f"(a0), "f"(a1));
  asm("mov.b64 %0, {%1, %1};" : "=l"(B) : "f"(b));
  asm("add.rn.f32x2 %0, %1, %2;" : "=l"(Dd) : "l"(A), "l"(B));
  asm("mov.b64 {%0, %1}, %2;" : "=f"(d0), "=f"(d1) : "l"(Dd));
}
// (a0, a1) * (b0, b1) + (c, c) on the paired fp32 pipe.
__device__ __forceinline__ void fma2v(float& d0, float& d1, float a0, float a1, float b0, float b1, float c) {
  uint64_t A, B, Cc, Dd;
  asm("mov.b64 %0, {%1, %2};" : "=l"(A) : "f"(a0), "f"(a1));
  asm("mov.b64 %0, {%1, %2};" : "=l"(B) : "f"(b0), "f"(b1));
  asm("mov.b64 %0, {%1, %1};" : "=l"(Cc) : "f"(c));
  asm("fma.rn.f32x2 %0, %1, %2, %3;" : "=l"(Dd) : "l"(A), "l"(B), "l"(Cc));
  asm("mov.b64 {%0, %1}, %2;" : "=f"(d0), "=f"(d1) : "l"(Dd));
}

// 2^x for two values on the FMA and integer pipes instead of the exponential unit
// (which computes only 16 results per cycle per SM and bounds the softmax at
// head_dim 64).  Range reduction: x = j + f with j = round(x), taken by adding and
// subtracting 1.5 * 2^23, and f in [-1/2, 1/2]; 2^f from a cubic whose
// coefficients were fitted here to 2^f on [-1/2, 1/2] by reweighted least squares
// on the relative error (largest relative error 7.5e-5 in fp32, below half a
// 16-bit ulp of P); 2^j enters through the exponent bits.  x is clamped to
// [-125, 127] so that the exponent stays normal (2^-125 rounds to zero in P).
__device__ __forceinline__ void exp2_fma(float& y0, float& y1, float x0, float x1) {
  constexpr float kRound = 12582912.0f;  // 1.5 * 2^23
  x0 = fminf(fmaxf(x0, -125.f), 127.f);
  x1 = fminf(fmaxf(x1, -125.f), 127.f);
  float t0, t1, r0, r1, f0, f1, p0, p1;
  add2s(t0, t1, x0, x1, kRound);  // 1.5 * 2^23 + round(x)
  add2s(r0, r1, t0, t1, -kRound);  // round(x)
  f0 = x0 - r0;
  f1 = x1 - r1;
  fma2v(p0, p1, f0, f1, 0.0551716573536396f, 0.0551716573536396f, 0.2426111400127411f);
  fma2v(p0, p1, p0, p1, f0, f1, 0.6932609677314758f);
  fma2v(p0, p1, p0, p1, f0, f1, 0.9999280571937561f);
  const int j0 = __float_as_int(t0) - 0x4B400000, j1 = __float_as_int(t1) - 0x4B400000;
  y0 = __int_as_float(__float_as_int(p0) + (j0 << 23));
  y1 = __int_as_float(__float_as_int(p1) + (j1 << 23));
}

// EMU: of every 8 pairs of exponentials of a score row, those with index % 8 < EMU
// are computed with exp2_fma, the rest on the exponential unit.
template <typename T, int D, int EMU>
__global__ void __launch_bounds__(512, 1)
    flash_prefill_pair_kernel(const PrefillParams p, const __grid_constant__ CUtensorMap tm_q,
                              const __grid_constant__ CUtensorMap tm_k, const __grid_constant__ CUtensorMap tm_v) {
  using C = PairCfg<D>;
  constexpr int S = C::kStages;
  constexpr int QB = C::kQBufs;
  constexpr bool kBf16 = std::is_same<T, __nv_bfloat16>::value;

  extern __shared__ uint8_t smem_raw[];
  const uint32_t raw_u32 = ptx::smem_u32(smem_raw);
  const uint32_t base_u32 = (raw_u32 + 1023u) & ~1023u;
  if (base_u32 + C::kUsed > raw_u32 + C::kSmemBytes) {  // cannot happen with a >=16 B aligned base
    if (threadIdx.x == 0) report(p.status);
    return;
  }
  uint8_t* base = smem_raw + (base_u32 - raw_u32);
  uint64_t* q_full = reinterpret_cast<uint64_t*>(base + C::kBarOff);
  uint64_t* q_empty = q_full + QB;
  uint64_t* k_full = q_empty + QB;
  uint64_t* v_full = k_full + S;
  // K(g) is released once both heads' S(g) are done, V(g) once both P.V are: the
  // producer's K loads then run well ahead of the S MMAs instead of waiting for
  // the later P.V of the same tile.
  uint64_t* k_empty = v_full + S;
  uint64_t* v_empty = k_empty + S;
  uint64_t* s_full = v_empty + S;  // [2] per head
  uint64_t* s_free = s_full + 2;
  uint64_t* p_full = s_free + 2;
  uint64_t* pv_done = p_full + 2;
  uint64_t* o_empty = pv_done + 2;
  uint64_t* final_bar = o_empty + 2;  // [3] one per MMA-issuing warp
  uint64_t* item_full = final_bar + 3;
  uint64_t* item_empty = item_full + C::kItemSlots;
  // exp_turn[q][t]: head t's softmax warp on scheduler q may start its exponentials
  uint64_t* exp_turn = item_empty + C::kItemSlots;
  // epi_ready[item parity][t]: head t's item is complete, its rows' sums are in
  // l_buf.  One barrier per item parity: the softmax warps can finish the next
  // (one-tile) item before the epilogue has waited for this one, and a single
  // barrier would then have moved two phases on, which a parity wait cannot tell
  // from none (they cannot get further ahead: the item after that needs a P.V
  // that waits for the epilogue to release O).
  uint64_t* epi_ready = exp_turn + 8;
  // The S issuer has taken item n.  The producer claims item n + 1 only then: a CTA
  // holds at most the running item and the next, so the last, small items of the
  // list go to CTAs that are about to run out of work instead of queueing behind
  // two items on one CTA.
  uint64_t* item_started = epi_ready + 4;
  // l_buf[item parity][head][row]: two items in flight, so a one-tile item's sums
  // cannot overwrite those the epilogue has yet to read
  float* l_buf = reinterpret_cast<float*>(base + C::kLOff);
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(base + C::kMiscOff);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(base + C::kMiscOff + 4);
  volatile int* item_ring = reinterpret_cast<volatile int*>(base + C::kMiscOff + 16);  // [slot][8]

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  if (warp == 1) {
    umma::tmem_alloc(tmem_slot, C::kTmemCols);
    umma::tmem_relinquish();
  }
  if (threadIdx.x == 0) {
    for (int i = 0; i < QB; ++i) {
      ptx::mbar_init(&q_full[i], 1);
      ptx::mbar_init(&q_empty[i], 1);
    }
    for (int s = 0; s < S; ++s) {
      ptx::mbar_init(&k_full[s], 1);
      ptx::mbar_init(&v_full[s], 1);
      ptx::mbar_init(&k_empty[s], 1);  // the S issuer
      ptx::mbar_init(&v_empty[s], 2);  // both P.V issuers
    }
    for (int t = 0; t < 2; ++t) {
      ptx::mbar_init(&s_full[t], 1);
      ptx::mbar_init(&s_free[t], 4);
      ptx::mbar_init(&p_full[t], 4);
      ptx::mbar_init(&pv_done[t], 1);
      ptx::mbar_init(&o_empty[t], 4);
    }
    for (int i = 0; i < 3; ++i) ptx::mbar_init(&final_bar[i], 1);
    for (int i = 0; i < C::kItemSlots; ++i) {
      ptx::mbar_init(&item_full[i], 1);
      ptx::mbar_init(&item_empty[i], 15);  // the three MMA issuers, eight softmax and four epilogue warps
    }
    for (int i = 0; i < 8; ++i) ptx::mbar_init(&exp_turn[i], 1);
    for (int t = 0; t < 4; ++t) ptx::mbar_init(&epi_ready[t], 4);
    ptx::mbar_init(item_started, 1);
    *abort_flag = 0;
    ptx::fence_mbar_init();
  }
  umma::fence_before_sync();
  __syncthreads();
  umma::fence_after_sync();
  const uint32_t tmem = *tmem_slot;
  asm volatile("griddepcontrol.wait;" ::: "memory");
  const int n_items = min(__ldcg(p.sched_count), p.sched_cap) * (p.n_heads >> 1);
  uint32_t n_seen = 0;
  auto take_item = [&](PairItem& it, bool arrive) -> int {  // 1: item, 0: end of list, -1: gave up
    const int slot = n_seen % C::kItemSlots;
    if (!wait_or_abort(&item_full[slot], (n_seen / C::kItemSlots) & 1, abort_flag, p.wait_ns)) return -1;
    volatile int* e = item_ring + slot * 8;
    it = PairItem{e[0], e[1], e[2], e[3], e[4]};
    if (arrive) ptx::mbar_arrive(&item_empty[slot]);
    ++n_seen;
    return it.seq < 0 ? 0 : 1;
  };

  // Each warpgroup sets its register share at the top of its own branch (code
  // after a join is held to the smaller share).
  if (warp < 4) {
   asm volatile("setmaxnreg.dec.sync.aligned.u32 %0;" ::"n"(C::kRegsLow));
   if (warp == 0) {
    // =========================== TMA producer ===============================
    uint32_t kv_it = 0, q_it = 0, n_claim = 0;
    bool ok = true;
    if (lane == 0) {
      ptx::prefetch_tmap(&tm_q);
      ptx::prefetch_tmap(&tm_k);
      ptx::prefetch_tmap(&tm_v);
    }
    PairItem it{};
    while (ok) {
      const int slot = n_claim % C::kItemSlots;
      // The first item of CTA b is item b (the heaviest ones, with no atomic on
      // the way to the first loads); later ones come from the ticket counter.
      int w = (int)blockIdx.x;
      if (n_claim > 0) {
        // Item n_claim - 1 has been taken by the S issuer (it has taken every item
        // before it, so the barrier's phase cannot be two behind this wait).
        ok = __all_sync(0xffffffffu, wait_or_abort(item_started, (n_claim - 1) & 1, abort_flag, p.wait_ns));
        if (!ok) break;
        if (lane == 0) w = (int)atomicAdd(p.ticket, 1) + (int)gridDim.x;
        w = __shfl_sync(0xffffffffu, w, 0);
      }
      // The entry is read before it is checked against the list length, so that the
      // two reads overlap; an entry at or past the length is discarded.
      const PairItem cand = pair_item_of(p, w);
      if (w >= n_items) w = -1;
      if (w >= 0) {
        it = cand;
        if (it.seq < 0) {  // a corrupt schedule entry: stop here and say so
          report(p.status);
          w = -1;
        }
      }
      ok = __all_sync(0xffffffffu,
                      wait_or_abort(&item_empty[slot], ((n_claim / C::kItemSlots) & 1) ^ 1, abort_flag, p.wait_ns));
      if (!ok) break;
      if (lane == 0) {
        volatile int* e = item_ring + slot * 8;
        e[0] = w < 0 ? -1 : it.seq;
        e[1] = it.mtile;
        e[2] = it.h0;
        e[3] = it.s0;
        e[4] = it.L;
        ptx::mbar_arrive(&item_full[slot]);
      }
      ++n_claim;
      if (w < 0) break;
      if (p.drop_loads) break;  // test hook: the item's Q and K/V never arrive
      const int n_kv = pair_kv_tiles(p, it);
      const int kvh = it.h0 / p.group;
      const int qb = q_it % QB;
      ok = __all_sync(0xffffffffu, wait_or_abort(&q_empty[qb], ((q_it / QB) & 1) ^ 1, abort_flag, p.wait_ns));
      if (!ok) break;
      if (lane == 0) {
        ptx::mbar_arrive_expect_tx(&q_full[qb], 2 * C::kTileBytes);
        for (int t = 0; t < 2; ++t)
          for (int kb = 0; kb < C::kKB; ++kb)
            tma_load_3d(base + C::kQOff + (qb * 2 + t) * C::kTileBytes + kb * C::kBlockBytes, &tm_q, &q_full[qb],
                        kb * 64, it.h0 + t, it.s0 + it.mtile * 128);
      }
      ++q_it;
      for (int j = 0; j < n_kv; ++j, ++kv_it) {
        const int st = kv_it % S;
        const uint32_t ph = (kv_it / S) & 1;
        uint8_t* ks = base + C::kKOff + st * C::kTileBytes;
        uint8_t* vs = base + C::kVOff + st * C::kTileBytes;
        ok = __all_sync(0xffffffffu, wait_or_abort(&k_empty[st], ph ^ 1, abort_flag, p.wait_ns));
        if (!ok) break;
        if (lane == 0) {
          ptx::mbar_arrive_expect_tx(&k_full[st], C::kTileBytes);
          for (int kb = 0; kb < C::kKB; ++kb)
            tma_load_3d(ks + kb * C::kBlockBytes, &tm_k, &k_full[st], kb * 64, kvh, it.s0 + j * 128);
        }
        ok = __all_sync(0xffffffffu, wait_or_abort(&v_empty[st], ph ^ 1, abort_flag, p.wait_ns));
        if (!ok) break;
        if (lane == 0) {
          ptx::mbar_arrive_expect_tx(&v_full[st], C::kTileBytes);
          for (int kb = 0; kb < C::kKB; ++kb)
            tma_load_3d(vs + kb * C::kBlockBytes, &tm_v, &v_full[st], kb * 64, kvh, it.s0 + j * 128);
        }
      }
    }
    if (!ok) report(p.status);
    // Do not leave with copies in flight: the last issued loads must have landed.
    if (lane == 0) {
      for (uint32_t j = kv_it >= (uint32_t)S ? kv_it - S : 0; j < kv_it; ++j) {
        ptx::mbar_wait(&k_full[j % S], (j / S) & 1, 100000000ull);
        ptx::mbar_wait(&v_full[j % S], (j / S) & 1, 100000000ull);
      }
      for (uint32_t j = q_it >= (uint32_t)QB ? q_it - QB : 0; j < q_it; ++j)
        ptx::mbar_wait(&q_full[j % QB], (j / QB) & 1, 100000000ull);
    }
  } else if (warp == 1) {
    // ======================= S issuer (both heads) ==========================
    if (lane == 0) {
      const uint32_t idesc_s = umma::idesc_f16(128, 128, kBf16, false);
      uint32_t g = 0, q_it = 0;  // g: K/V tiles of this CTA
      bool ok = true;
      PairItem it;
      while (ok) {
        const int got = take_item(it, true);
        if (got <= 0) {
          ok = got == 0;
          break;
        }
        ptx::mbar_arrive(item_started);  // the producer may claim the next item
        const int n_kv = pair_kv_tiles(p, it);
        const int qb = q_it % QB;
        ok = wait_or_abort(&q_full[qb], (q_it / QB) & 1, abort_flag, p.wait_ns);
        for (int j = 0; ok && j < n_kv; ++j, ++g) {
          ok = wait_or_abort(&k_full[g % S], (g / S) & 1, abort_flag, p.wait_ns);
          const uint32_t k_addr = base_u32 + C::kKOff + (g % S) * C::kTileBytes;
          for (int t = 0; t < 2 && ok; ++t) {
            if (C::kPAlias) {
              // P_t lives over S_t: S_t(g) waits for P_t(g-1).V to complete (which
              // also means softmax t has read S_t(g-1)).
              if (g > 0) ok = wait_or_abort(&pv_done[t], (g - 1) & 1, abort_flag, p.wait_ns);
            } else {
              ok = wait_or_abort(&s_free[t], (g & 1) ^ 1, abort_flag, p.wait_ns);  // S_t(g-1) was read
            }
            if (!ok) break;
            umma::fence_after_sync();
            const uint32_t q_addr = base_u32 + C::kQOff + (qb * 2 + t) * C::kTileBytes;
#pragma unroll
            for (int ks = 0; ks < D / 16; ++ks) {
              const uint64_t ad = umma::smem_desc_sw128(q_addr + (ks >> 2) * C::kBlockBytes + (ks & 3) * 32, 16, 1024);
              const uint64_t bd = umma::smem_desc_sw128(k_addr + (ks >> 2) * C::kBlockBytes + (ks & 3) * 32, 16, 1024);
              umma::mma_f16_ss(tmem + (t ? 128u : 0u), ad, bd, idesc_s, ks > 0 ? 1u : 0u);
            }
            umma::commit(&s_full[t]);
          }
          if (!ok) break;
          umma::commit(&k_empty[g % S]);                  // K(g) consumed
          if (j == n_kv - 1) umma::commit(&q_empty[qb]);  // Q is free once the item's S MMAs are done
        }
        ++q_it;
      }
      if (!ok) report(p.status);
      // Drain: every MMA issued by this thread completes before TMEM is released.
      umma::commit(&final_bar[0]);
      ptx::mbar_wait(&final_bar[0], 0, 100000000ull);
    }
    __syncwarp();
  } else if (warp == 2 || warp == 3) {
    // ===================== P.V issuer of head t = warp - 2 ===================
    if (lane == 0) {
      const int t = warp - 2;
      const uint32_t idesc_o = umma::idesc_f16(128, D, kBf16, true);
      uint32_t g = 0, item_it = 0;
      bool ok = true;
      PairItem it;
      while (ok) {
        const int got = take_item(it, true);
        if (got <= 0) {
          ok = got == 0;
          break;
        }
        const int n_kv = pair_kv_tiles(p, it);
        for (int j = 0; ok && j < n_kv; ++j, ++g) {
          ok = wait_or_abort(&v_full[g % S], (g / S) & 1, abort_flag, p.wait_ns) &&
               wait_or_abort(&p_full[t], g & 1, abort_flag, p.wait_ns);
          // the item's first P.V overwrites O_t: the previous item's O_t must have been read
          if (ok && j == 0) ok = wait_or_abort(&o_empty[t], (item_it & 1) ^ 1, abort_flag, p.wait_ns);
          if (!ok) break;
          umma::fence_after_sync();
          const uint32_t v_addr = base_u32 + C::kVOff + (g % S) * C::kTileBytes;
#pragma unroll
          for (int ks = 0; ks < 8; ++ks) {  // 16 keys per MMA: 8 TMEM columns of P
            const uint64_t bd = umma::smem_desc_sw128(v_addr + ks * 2048, C::kBlockBytes, 1024);
            umma::mma_f16_ts(tmem + ocol(D, t), tmem + pcol(D, t) + ks * 8, bd, idesc_o, (j == 0 && ks == 0) ? 0u : 1u);
          }
          umma::commit(&pv_done[t]);
          umma::commit(&v_empty[g % S]);  // V(g) consumed by this head
        }
        ++item_it;
      }
      if (!ok) report(p.status);
      umma::commit(&final_bar[warp - 1]);
      ptx::mbar_wait(&final_bar[warp - 1], 0, 100000000ull);
    }
    __syncwarp();
   }
  } else if (warp >= 12) {
    asm volatile("setmaxnreg.dec.sync.aligned.u32 %0;" ::"n"(C::kRegsEpi));
    // ====================== epilogue warps (O -> out) =======================
    // Warp 12+q reads TMEM lane quarter q: for each item and head, once the
    // head's last P.V has completed, O / l for its 32 rows go to global memory
    // and O_t is released to the next item's first P.V.
    const int quarter = warp & 3;
    const int r = quarter * 32 + lane;
    const uint32_t t_lane = tmem + ((uint32_t)(quarter * 32) << 16);
    uint32_t g = 0, item_it = 0;
    bool ok = true;
    PairItem it;
    while (ok) {
      const int got = take_item(it, false);
      ok = __all_sync(0xffffffffu, got >= 0);
      if (!ok) break;
      __syncwarp();
      if (lane == 0) ptx::mbar_arrive(&item_empty[(n_seen - 1) % C::kItemSlots]);
      if (got == 0) break;
      g += pair_kv_tiles(p, it);  // g - 1: the item's last key tile
      const int q_pos = it.mtile * 128 + r;
      if (p.slot_mapping != nullptr && it.h0 % p.group == 0 && q_pos < it.L) {
        // Paged K/V write (the first pair of every KV head's group): row q_pos of
        // this prompt's k and v goes to its slot (block * block_size + offset).  The
        // producer loads the same rows for this item, so they are usually in L2; the
        // copy overlaps the item's softmax instead of holding up the producer's loads.
        const long long slot = __ldcg(p.slot_mapping + it.s0 + q_pos);
        const long long n_slots = (long long)p.num_blocks * p.block_size;
        if (slot >= 0 && slot < n_slots) {
          const int kvh = it.h0 / p.group;
          const size_t src = ((size_t)(it.s0 + q_pos) * p.n_kv_heads + kvh) * D;
          const size_t dst = ((size_t)slot * p.n_kv_heads + kvh) * D;
#pragma unroll
          for (int kv = 0; kv < 2; ++kv) {
            const uint4* sp = reinterpret_cast<const uint4*>(reinterpret_cast<const T*>(kv ? p.v : p.k) + src);
            uint4* dp = reinterpret_cast<uint4*>(reinterpret_cast<T*>(kv ? p.v_cache : p.k_cache) + dst);
#pragma unroll
            for (int c0 = 0; c0 < D / 8; c0 += 4) {
              uint4 x[4];
#pragma unroll
              for (int c = 0; c < 4; ++c) x[c] = __ldcg(sp + c0 + c);
#pragma unroll
              for (int c = 0; c < 4; ++c) dp[c0 + c] = x[c];
            }
          }
        }
      }
      for (int t = 0; t < 2 && ok; ++t) {
        ok = __all_sync(0xffffffffu, wait_or_abort(&epi_ready[(item_it & 1) * 2 + t], (item_it >> 1) & 1, abort_flag,
                                                   p.wait_ns) &&
                                         wait_or_abort(&pv_done[t], (g - 1) & 1, abort_flag, p.wait_ns));
        if (!ok) break;
        umma::fence_after_sync();
        const float l = l_buf[((item_it & 1) * 2 + t) * 128 + r];
        const float inv = l > 0.f ? 1.f / l : 0.f;
        T* orow = reinterpret_cast<T*>(p.out) + ((size_t)(it.s0 + q_pos) * p.n_heads + it.h0 + t) * D;
#pragma unroll
        for (int c = 0; c < D / 32; ++c) {
          float o[32];
          umma::ld_32x32b_x32(t_lane + ocol(D, t) + c * 32, o);
          umma::ld_wait();
          if (q_pos < it.L) {
#pragma unroll
            for (int c8 = 0; c8 < 4; ++c8) {
              uint4 w;
              w.x = DT<T>::pack2(o[c8 * 8 + 0] * inv, o[c8 * 8 + 1] * inv);
              w.y = DT<T>::pack2(o[c8 * 8 + 2] * inv, o[c8 * 8 + 3] * inv);
              w.z = DT<T>::pack2(o[c8 * 8 + 4] * inv, o[c8 * 8 + 5] * inv);
              w.w = DT<T>::pack2(o[c8 * 8 + 6] * inv, o[c8 * 8 + 7] * inv);
              *reinterpret_cast<uint4*>(orow + c * 32 + c8 * 8) = w;
            }
          }
        }
        umma::fence_before_sync();
        __syncwarp();
        if (lane == 0) ptx::mbar_arrive(&o_empty[t]);
      }
      ++item_it;
    }
    if (!ok) report(p.status);
  } else {
    asm volatile("setmaxnreg.inc.sync.aligned.u32 %0;" ::"n"(C::kRegsHigh));
    // =========================== softmax warps ==============================
    const int t = (warp - 4) >> 2;     // head of the pair
    const int quarter = warp & 3;      // TMEM lane quarter this warp may access
    const int r = quarter * 32 + lane; // query row of the tile
    const uint32_t t_lane = tmem + ((uint32_t)(quarter * 32) << 16);
    const uint32_t s_col = t ? 128u : 0u, p_col = pcol(D, t), o_col = ocol(D, t);
    const float sl2 = p.scale_log2;
    uint32_t item_it = 0;  // items finished (l_buf slot parity)
    uint32_t g = 0;  // K/V tiles seen (S, P and P.V phases follow it)
    bool ok = true;
    PairItem it;
    while (ok) {
      int got = take_item(it, false);
      ok = __all_sync(0xffffffffu, got >= 0);
      if (!ok) break;
      __syncwarp();
      if (lane == 0) ptx::mbar_arrive(&item_empty[(n_seen - 1) % C::kItemSlots]);
      if (got == 0) break;
      const int n_kv = pair_kv_tiles(p, it);
      const int q_pos = it.mtile * 128 + r;
      const int lim = p.causal ? min(q_pos + 1, it.L) : it.L;  // keys [0, lim) are visible
      float m = -INFINITY;  // running max (log2 domain) that P and O are scaled by
      float l0 = 0.f, l1 = 0.f;
      for (int j = 0; j < n_kv; ++j, ++g) {
        ok = __all_sync(0xffffffffu, wait_or_abort(&s_full[t], g & 1, abort_flag, p.wait_ns));
        if (!ok) break;
        umma::fence_after_sync();
        float s[128];
#pragma unroll
        for (int c = 0; c < 4; ++c)
          umma::ld_32x32b_x32(t_lane + s_col + c * 32, *reinterpret_cast<float(*)[32]>(&s[c * 32]));
        umma::ld_wait();
        if (!C::kPAlias) {  // S_t is free for the next tile's scores
          umma::fence_before_sync();
          __syncwarp();
          if (lane == 0) ptx::mbar_arrive(&s_free[t]);
        }
        const int lim_rel = lim - j * 128;  // keys [0, lim_rel) of this tile are visible
        if (__any_sync(0xffffffffu, lim_rel < 128)) {
#pragma unroll
          for (int x = 0; x < 128; ++x) s[x] = x < lim_rel ? s[x] : -INFINITY;
        }
        float mp[8];
#pragma unroll
        for (int i = 0; i < 8; ++i) {
          mp[i] = max3f(s[i], s[8 + i], s[16 + i]);
#pragma unroll
          for (int k = 24; k < 128; k += 16) mp[i] = max3f(mp[i], s[k + i], s[k + 8 + i]);
        }
        const float mx = max3f(max3f(mp[0], mp[1], mp[2]), max3f(mp[3], mp[4], mp[5]), fmaxf(mp[6], mp[7]));
        float m_cand = fmaxf(m, mx * sl2);
        if (m_cand == -INFINITY) m_cand = 0.f;  // no visible key (a row past the prompt's end)
        // Lazy rescale: the stale max is kept unless the new one is 2^8 larger; O_t
        // itself is rescaled after P is stored (the scores are dead by then), still
        // before P_t.V is released to add to it.
        float corr = 1.f;
        const bool rescale = j > 0 && __any_sync(0xffffffffu, m_cand > m + 8.f);
        if (j == 0 || rescale) {
          corr = j == 0 ? 1.f : ex2(m - m_cand);
          l0 *= corr;
          l1 *= corr;
          m = m_cand;
        }
        // Wait for this head's turn on the exponential unit (head 0 goes first on
        // every tile; the turn order only schedules the unit, results do not depend on it).
        ok = __all_sync(0xffffffffu, wait_or_abort(&exp_turn[quarter * 2 + t], (g & 1) ^ (t ? 0u : 1u), abort_flag,
                                                   p.wait_ns));
        if (!ok) break;
        // P = 2^(s*scale - m), packed to 16-bit pairs in registers (the A operand of
        // P.V); these exponentials overlap the previous tile's P_t.V.
        uint32_t pk[64];
#pragma unroll
        for (int x = 0; x < 64; ++x) {
          float x0, x1;
          fma2(x0, x1, s[2 * x], s[2 * x + 1], sl2, -m);
          float e0, e1;
          if ((x & 7) < EMU) {
            exp2_fma(e0, e1, x0, x1);
          } else {
            e0 = ex2(x0);
            e1 = ex2(x1);
          }
          add2(l0, l1, e0, e1);
          pk[x] = DT<T>::pack2(e0, e1);
        }
        __syncwarp();
        if (lane == 0) ptx::mbar_arrive(&exp_turn[quarter * 2 + (t ^ 1)]);  // the other head's turn
        // P_t's columns are rewritten now: the previous tile's P_t.V must have completed.
        if (g > 0) {
          ok = __all_sync(0xffffffffu, wait_or_abort(&pv_done[t], (g - 1) & 1, abort_flag, p.wait_ns));
          if (!ok) break;
          umma::fence_after_sync();
        }
        umma::st_32x32b_x32_u(t_lane + p_col, pk);
        umma::st_32x32b_x32_u(t_lane + p_col + 32, pk + 32);
        if (rescale) {  // O_t is stable: P_t(g-1).V completed, P_t(g).V not released yet
#pragma unroll
          for (int c = 0; c < D / 32; ++c) {
            float o[32];
            umma::ld_32x32b_x32(t_lane + o_col + c * 32, o);
            umma::ld_wait();
#pragma unroll
            for (int x = 0; x < 32; ++x) o[x] *= corr;
            umma::st_32x32b_x32(t_lane + o_col + c * 32, o);
          }
        }
        umma::st_wait();
        umma::fence_before_sync();
        __syncwarp();
        if (lane == 0) ptx::mbar_arrive(&p_full[t]);
      }
      if (!ok) break;
      // ---- item done: the row sums go to the epilogue warps, which write O / l
      // once the last P.V completes; this warp moves on to the next item.  The
      // slot written here was last read by the epilogue two items back, which had
      // finished before that item's first P.V (and so our previous P store) ran.
      l_buf[((item_it & 1) * 2 + t) * 128 + r] = l0 + l1;
      __syncwarp();
      if (lane == 0) ptx::mbar_arrive(&epi_ready[(item_it & 1) * 2 + t]);
      ++item_it;
    }
    if (!ok) report(p.status);
  }

  umma::fence_before_sync();
  __syncthreads();
  if (warp == 1) {
    umma::fence_after_sync();
    umma::tmem_dealloc(tmem, C::kTmemCols);
  }
}

// -----------------------------------------------------------------------------
// SIMT prefill (any dtype, head_dim 32/64/128): one warp handles four query
// rows, lanes split head_dim, fp32 online softmax.  Also does the paged write.
// -----------------------------------------------------------------------------
constexpr int kSimtRows = 16;  // query rows per CTA (4 warps x 4 rows)

template <typename T, int D>
__global__ void __launch_bounds__(128) flash_prefill_simt_kernel(const PrefillParams p) {
  constexpr int E = D / 32;  // elements per lane
  const int seq = blockIdx.z, h = blockIdx.y;
  const int s0 = p.cu_seqlens[seq];
  const int L = p.cu_seqlens[seq + 1] - s0;
  const int row0 = blockIdx.x * kSimtRows;
  if (row0 >= L) return;
  const int kvh = h / p.group;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const T* q = reinterpret_cast<const T*>(p.q);
  const T* k = reinterpret_cast<const T*>(p.k);
  const T* v = reinterpret_cast<const T*>(p.v);

  if (p.slot_mapping != nullptr && (h % p.group) == 0) {
    const long long n_slots = (long long)p.num_blocks * p.block_size;
    T* kc = reinterpret_cast<T*>(p.k_cache);
    T* vc = reinterpret_cast<T*>(p.v_cache);
    const int rows = min(kSimtRows, L - row0);
    for (int i = threadIdx.x; i < rows * D; i += blockDim.x) {
      const int rr = i / D, d = i % D;
      const int tok = s0 + row0 + rr;
      const long long slot = p.slot_mapping[tok];
      if (slot < 0 || slot >= n_slots) continue;
      const size_t src = ((size_t)tok * p.n_kv_heads + kvh) * D + d;
      const size_t dst = ((size_t)slot * p.n_kv_heads + kvh) * D + d;
      kc[dst] = k[src];
      vc[dst] = v[src];
    }
  }

  float qr[4][E], acc[4][E], m[4], l[4];
  int qp[4];
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    qp[i] = row0 + warp * 4 + i;
    m[i] = -INFINITY;
    l[i] = 0.f;
#pragma unroll
    for (int e = 0; e < E; ++e) {
      acc[i][e] = 0.f;
      qr[i][e] = qp[i] < L ? DT<T>::to_f(q[((size_t)(s0 + qp[i]) * p.n_heads + h) * D + lane + 32 * e]) : 0.f;
    }
  }
  const int last = qp[3] < L ? qp[3] : L - 1;
  const int kv_end = p.causal ? last + 1 : L;
  for (int t = 0; t < kv_end; ++t) {
    float kr[E], vr[E];
    const size_t off = ((size_t)(s0 + t) * p.n_kv_heads + kvh) * D;
#pragma unroll
    for (int e = 0; e < E; ++e) {
      kr[e] = DT<T>::to_f(k[off + lane + 32 * e]);
      vr[e] = DT<T>::to_f(v[off + lane + 32 * e]);
    }
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      float s = 0.f;
#pragma unroll
      for (int e = 0; e < E; ++e) s = fmaf(qr[i][e], kr[e], s);
#pragma unroll
      for (int o = 16; o > 0; o >>= 1) s += __shfl_xor_sync(0xffffffffu, s, o);
      const bool vis = qp[i] < L && (!p.causal || t <= qp[i]);
      if (vis) {
        const float s2 = s * p.scale_log2;
        const float mn = fmaxf(m[i], s2);
        const float corr = exp2f(m[i] - mn);
        const float pr = exp2f(s2 - mn);
        l[i] = l[i] * corr + pr;
#pragma unroll
        for (int e = 0; e < E; ++e) acc[i][e] = fmaf(acc[i][e], corr, pr * vr[e]);
        m[i] = mn;
      }
    }
  }
  T* out = reinterpret_cast<T*>(p.out);
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    if (qp[i] >= L) continue;
    const float inv = l[i] > 0.f ? 1.f / l[i] : 0.f;
#pragma unroll
    for (int e = 0; e < E; ++e)
      out[((size_t)(s0 + qp[i]) * p.n_heads + h) * D + lane + 32 * e] = DT<T>::from_f(acc[i][e] * inv);
  }
}

// -----------------------------------------------------------------------------
// Work schedule for the tcgen05 kernel: every (prompt, query tile) pair, the
// heaviest first (query tile m of a causal prompt costs m + 1 key tiles), in a
// dense list so that persistent CTAs never visit empty tiles.  One CTA.
// -----------------------------------------------------------------------------
constexpr int kMaxBands = 4096;  // query tiles per prompt: max_seqlen <= 524288

__global__ void __launch_bounds__(1024) prefill_schedule_kernel(const int32_t* __restrict__ cu, int n_seqs,
                                                                int n_bands, int capacity, int4* sched,
                                                                int32_t* count, int* ticket, int* status) {
  __shared__ int band[kMaxBands];
  // let the attention kernel start its prologue now; it waits for this grid
  // to finish before it reads the schedule
  asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
  if (threadIdx.x == 0) *ticket = 0;
  for (int m = threadIdx.x; m < n_bands; m += blockDim.x) band[m] = 0;
  __syncthreads();
  for (int s = threadIdx.x; s < n_seqs; s += blockDim.x) {
    const int nt = min((cu[s + 1] - cu[s] + 127) / 128, n_bands);
    for (int m = 0; m < nt; ++m) atomicAdd(&band[m], 1);
  }
  __syncthreads();
  if (threadIdx.x == 0) {
    int run = 0;
    for (int m = n_bands - 1; m >= 0; --m) {
      const int c = band[m];
      band[m] = run;  // first slot of band m
      run += c;
    }
    *count = min(run, capacity);
    if (run > capacity && status) atomicExch(status, 2);
  }
  __syncthreads();
  for (int s = threadIdx.x; s < n_seqs; s += blockDim.x) {
    const int s0 = cu[s], L = cu[s + 1] - s0;
    const int nt = min((L + 127) / 128, n_bands);
    for (int m = nt - 1; m >= 0; --m) {
      const int pos = atomicAdd(&band[m], 1);
      if (pos < capacity) sched[pos] = make_int4(s, m, s0, L);
    }
  }
}

// -----------------------------------------------------------------------------
// host side
// -----------------------------------------------------------------------------
int encode_rows_map(CUtensorMap* m, const void* ptr, CUtensorMapDataType tdt, int D, int heads, int total,
                    int box_rows) {
  tvk::EncodeTiledFn encode = tvk::encode_tiled_fn();
  if (!encode) {
    tvk::set_error("cuTensorMapEncodeTiled is not available from the driver");
    return TVK_ERR_CUDA;
  }
  cuuint64_t dims[3] = {(cuuint64_t)D, (cuuint64_t)heads, (cuuint64_t)total};
  cuuint64_t strides[2] = {(cuuint64_t)D * 2, (cuuint64_t)heads * D * 2};
  cuuint32_t box[3] = {64u, 1u, (cuuint32_t)box_rows};
  cuuint32_t estr[3] = {1u, 1u, 1u};
  CUresult r = encode(m, tdt, 3, const_cast<void*>(ptr), dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
                      CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) {
    tvk::set_error("cuTensorMapEncodeTiled failed (%d)", (int)r);
    return TVK_ERR_CUDA;
  }
  return TVK_OK;
}

template <typename T, int D>
int launch_tc(const PrefillParams& p, int total, int sched_capacity, CUtensorMapDataType tdt, cudaStream_t stream) {
  using C = PfCfg<D>;
  CUtensorMap tq, tk, tv;
  int rc = encode_rows_map(&tq, p.q, tdt, D, p.n_heads, total, 128);
  if (rc == TVK_OK) rc = encode_rows_map(&tk, p.k, tdt, D, p.n_kv_heads, total, C::kKvRows);
  if (rc == TVK_OK) rc = encode_rows_map(&tv, p.v, tdt, D, p.n_kv_heads, total, C::kKvRows);
  if (rc != TVK_OK) return rc;
  auto kern = flash_prefill_tc_kernel<T, D>;
  prefill_schedule_kernel<<<1, 1024, 0, stream>>>(p.cu_seqlens, p.n_seqs, p.n_mtiles, sched_capacity,
                                                  const_cast<int4*>(p.sched), const_cast<int32_t*>(p.sched_count),
                                                  p.ticket, p.status);
  TVK_CHECK_LAUNCH("prefill_schedule");
  static unsigned long long attr_mask = 0;
  int dev = 0;
  TVK_CHECK_CUDA(cudaGetDevice(&dev));
  if (dev >= 64 || !(attr_mask & (1ull << dev))) {
    TVK_CHECK_CUDA(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, C::kSmemBytes));
    if (dev < 64) attr_mask |= 1ull << dev;
  }
  // Persistent CTAs (as many as fit at once), each walking its share of the
  // (query tile, head, prompt) items.
  static int num_sms[64] = {0};
  if (dev < 64 && num_sms[dev] == 0)
    TVK_CHECK_CUDA(cudaDeviceGetAttribute(&num_sms[dev], cudaDevAttrMultiProcessorCount, dev));
  const long long items = (long long)p.n_mtiles * p.n_seqs * p.n_heads;
  const long long slots = (long long)(dev < 64 ? num_sms[dev] : 148) * C::kCtasPerSm;
  const int grid = (int)(items < slots ? items : slots);
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(grid);
  cfg.blockDim = dim3(192);
  cfg.dynamicSmemBytes = C::kSmemBytes;
  cfg.stream = stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  TVK_CHECK_CUDA(cudaLaunchKernelEx(&cfg, kern, p, tq, tk, tv));
  TVK_CHECK_LAUNCH("flash_prefill_tc");
  return TVK_OK;
}

template <typename T, int D, int EMU>
int launch_pair(const PrefillParams& p, int total, int sched_capacity, CUtensorMapDataType tdt, cudaStream_t stream) {
  using C = PairCfg<D>;
  CUtensorMap tq, tk, tv;
  int rc = encode_rows_map(&tq, p.q, tdt, D, p.n_heads, total, 128);
  if (rc == TVK_OK) rc = encode_rows_map(&tk, p.k, tdt, D, p.n_kv_heads, total, 128);
  if (rc == TVK_OK) rc = encode_rows_map(&tv, p.v, tdt, D, p.n_kv_heads, total, 128);
  if (rc != TVK_OK) return rc;
  auto kern = flash_prefill_pair_kernel<T, D, EMU>;
  static unsigned long long attr_mask = 0;
  static int num_sms[64] = {0};
  int dev = 0;
  TVK_CHECK_CUDA(cudaGetDevice(&dev));
  if (dev >= 64) {
    tvk::set_error("device index %d beyond 63", dev);
    return TVK_ERR_UNSUPPORTED;
  }
  if (!(attr_mask & (1ull << dev))) {
    TVK_CHECK_CUDA(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, C::kSmemBytes));
    // The warpgroups' register shares (setmaxnreg) must fit in what the launch provides.
    cudaFuncAttributes fa;
    TVK_CHECK_CUDA(cudaFuncGetAttributes(&fa, kern));
    if (fa.numRegs < C::kRegsLaunchMin) {
      tvk::set_error("prefill kernel built with %d registers per thread; its register split needs %d", fa.numRegs,
                     C::kRegsLaunchMin);
      return TVK_ERR_UNSUPPORTED;
    }
    TVK_CHECK_CUDA(cudaDeviceGetAttribute(&num_sms[dev], cudaDevAttrMultiProcessorCount, dev));
    attr_mask |= 1ull << dev;
  }
  prefill_schedule_kernel<<<1, 1024, 0, stream>>>(p.cu_seqlens, p.n_seqs, p.n_mtiles, sched_capacity,
                                                  const_cast<int4*>(p.sched), const_cast<int32_t*>(p.sched_count),
                                                  p.ticket, p.status);
  TVK_CHECK_LAUNCH("prefill_schedule");
  const long long items = (long long)p.n_mtiles * p.n_seqs * (p.n_heads / 2);
  const int grid = (int)(items < num_sms[dev] ? items : num_sms[dev]);  // one CTA per SM
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(grid);
  cfg.blockDim = dim3(C::kThreads);
  cfg.dynamicSmemBytes = C::kSmemBytes;
  cfg.stream = stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  TVK_CHECK_CUDA(cudaLaunchKernelEx(&cfg, kern, p, tq, tk, tv));
  TVK_CHECK_LAUNCH("flash_prefill_pair");
  return TVK_OK;
}

template <typename T>
int launch_simt(const PrefillParams& p, int max_seqlen, cudaStream_t stream) {
  dim3 grid((max_seqlen + kSimtRows - 1) / kSimtRows, p.n_heads, p.n_seqs);
  switch (p.head_dim) {
    case 32: flash_prefill_simt_kernel<T, 32><<<grid, 128, 0, stream>>>(p); break;
    case 64: flash_prefill_simt_kernel<T, 64><<<grid, 128, 0, stream>>>(p); break;
    default: flash_prefill_simt_kernel<T, 128><<<grid, 128, 0, stream>>>(p); break;
  }
  TVK_CHECK_LAUNCH("flash_prefill_simt");
  return TVK_OK;
}

// Which tcgen05 kernel this thread's prefill calls use (tvk_prefill_select_kernel).
thread_local int g_prefill_choice = 0;
// Share of the softmax exponentials the automatic choice moves to the FMA pipe
// (eighths of the pairs), per head_dim.
constexpr int kAutoEmu64 = 0;
constexpr int kAutoEmu128 = 0;
int tvk_prefill_kernel_choice() { return g_prefill_choice; }

}  // namespace

extern "C" int tvk_prefill_select_kernel(int choice) {
  TVK_CHECK_ARG(choice >= 0 && choice <= 4,
                "kernel choice %d (0 automatic, 1 one-head, 2-4 paired with 0, 2 or 3 eighths of the exponentials "
                "on the FMA pipe)", choice);
  g_prefill_choice = choice;
  return TVK_OK;
}

extern "C" size_t tvk_flash_prefill_workspace_size(int n_seqs, int total_tokens) {
  if (n_seqs < 0 || total_tokens < 0) return tvk::kWorkspaceHeader;
  const size_t items = (size_t)total_tokens / 128 + (size_t)n_seqs + 1;
  return tvk::kWorkspaceHeader + ((items * sizeof(int4) + 255) / 256) * 256;
}

extern "C" int tvk_flash_prefill_attention(const void* q, const void* k, const void* v, void* out,
                                           const int32_t* cu_seqlens, int n_seqs, int max_seqlen, int total_tokens,
                                           int n_heads, int n_kv_heads, int head_dim, int causal, int dtype,
                                           const int64_t* slot_mapping, void* k_cache, void* v_cache, int num_blocks,
                                           int block_size, void* workspace, size_t workspace_bytes, void* stream) {
  TVK_CHECK_ARG(n_seqs >= 0 && total_tokens >= 0 && max_seqlen >= 0, "negative size");
  if (n_seqs == 0 || total_tokens == 0 || max_seqlen == 0) return TVK_OK;
  TVK_CHECK_ARG(q && k && v && out && cu_seqlens, "null pointer argument");
  TVK_CHECK_ARG(n_seqs <= 65535 && n_heads <= 65535, "n_seqs and n_heads must be <= 65535");
  TVK_CHECK_ARG(n_heads > 0 && n_kv_heads > 0 && n_heads % n_kv_heads == 0,
                "n_heads (%d) must be a positive multiple of n_kv_heads (%d)", n_heads, n_kv_heads);
  TVK_CHECK_ARG(dtype == TVK_DTYPE_F32 || dtype == TVK_DTYPE_F16 || dtype == TVK_DTYPE_BF16, "unknown dtype %d",
                dtype);
  if (head_dim != 32 && head_dim != 64 && head_dim != 128) {
    tvk::set_error("head_dim %d unsupported (32, 64 or 128)", head_dim);
    return TVK_ERR_UNSUPPORTED;
  }
  TVK_CHECK_ARG((uintptr_t)q % 16 == 0 && (uintptr_t)k % 16 == 0 && (uintptr_t)v % 16 == 0 &&
                    (uintptr_t)out % 16 == 0,
                "q, k, v and out must be 16-byte aligned");
  if (slot_mapping) {
    TVK_CHECK_ARG(k_cache && v_cache && num_blocks > 0 && block_size > 0,
                  "a slot mapping needs k_cache, v_cache, num_blocks and block_size");
    TVK_CHECK_ARG((uintptr_t)k_cache % 16 == 0 && (uintptr_t)v_cache % 16 == 0, "caches must be 16-byte aligned");
  }
  PrefillParams p{};
  p.q = q;
  p.k = k;
  p.v = v;
  p.out = out;
  p.cu_seqlens = cu_seqlens;
  p.slot_mapping = slot_mapping;
  p.k_cache = k_cache;
  p.v_cache = v_cache;
  p.status = workspace && workspace_bytes >= sizeof(int) ? reinterpret_cast<int*>(workspace) : nullptr;
  p.n_seqs = n_seqs;
  p.n_heads = n_heads;
  p.n_kv_heads = n_kv_heads;
  p.group = n_heads / n_kv_heads;
  p.head_dim = head_dim;
  p.causal = causal ? 1 : 0;
  p.num_blocks = num_blocks;
  p.block_size = block_size;
  p.n_mtiles = (max_seqlen + 127) / 128;
  p.total_tokens = total_tokens;
  p.scale_log2 = (float)(1.4426950408889634 / sqrt((double)head_dim));
  cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
  const bool tc = dtype != TVK_DTYPE_F32 && (head_dim == 64 || head_dim == 128);
  const tvk::WaitTest wt = tvk::take_wait_test();
  p.wait_ns = wt.armed ? wt.limit_ns : tvk::kDefaultWaitNs;
  p.drop_loads = wt.armed && tc ? 1 : 0;
  if (tc) {
    if (p.n_mtiles > kMaxBands) {
      tvk::set_error("max_seqlen %d exceeds the %d-token limit of the tcgen05 path", max_seqlen, kMaxBands * 128);
      return TVK_ERR_UNSUPPORTED;
    }
    const size_t need = tvk_flash_prefill_workspace_size(n_seqs, total_tokens);
    if (!workspace || workspace_bytes < need) {
      tvk::set_error("workspace of %zu bytes needed, %zu given", need, workspace ? workspace_bytes : (size_t)0);
      return TVK_ERR_WORKSPACE;
    }
    TVK_CHECK_ARG((uintptr_t)workspace % 16 == 0, "workspace must be 16-byte aligned");
    int32_t* w32 = reinterpret_cast<int32_t*>(workspace);
    p.sched_count = w32 + 1;
    p.ticket = w32 + 2;
    p.sched = reinterpret_cast<const int4*>(reinterpret_cast<uint8_t*>(workspace) + tvk::kWorkspaceHeader);
    const int cap = (int)((need - tvk::kWorkspaceHeader) / sizeof(int4));
    p.sched_cap = cap;
    // Heads in pairs sharing a KV head: the paired kernel (one CTA per SM, both heads'
    // softmax in flight); otherwise (one query head per KV head, or an odd group) the
    // one-head kernel.
    const int choice = tvk_prefill_kernel_choice();
    if (p.group % 2 == 0 && choice != 1) {
      // share of the exponentials computed on the FMA pipe (eighths of the pairs)
      const int emu = choice == 2 ? 0 : choice == 3 ? 2 : choice == 4 ? 3 : (head_dim == 64 ? kAutoEmu64 : kAutoEmu128);
      const CUtensorMapDataType tdt = dtype == TVK_DTYPE_F16 ? CU_TENSOR_MAP_DATA_TYPE_FLOAT16 : CU_TENSOR_MAP_DATA_TYPE_BFLOAT16;
#define TVK_PAIR(TT, DD)                                                   \
  switch (emu) {                                                           \
    case 2: return launch_pair<TT, DD, 2>(p, total_tokens, cap, tdt, s);   \
    case 3: return launch_pair<TT, DD, 3>(p, total_tokens, cap, tdt, s);   \
    default: return launch_pair<TT, DD, 0>(p, total_tokens, cap, tdt, s);  \
  }
      if (dtype == TVK_DTYPE_F16) {
        if (head_dim == 64) { TVK_PAIR(__half, 64) } else { TVK_PAIR(__half, 128) }
      } else {
        if (head_dim == 64) { TVK_PAIR(__nv_bfloat16, 64) } else { TVK_PAIR(__nv_bfloat16, 128) }
      }
#undef TVK_PAIR
    }
    if (dtype == TVK_DTYPE_F16)
      return head_dim == 64 ? launch_tc<__half, 64>(p, total_tokens, cap, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, s)
                            : launch_tc<__half, 128>(p, total_tokens, cap, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, s);
    return head_dim == 64 ? launch_tc<__nv_bfloat16, 64>(p, total_tokens, cap, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, s)
                          : launch_tc<__nv_bfloat16, 128>(p, total_tokens, cap, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, s);
  }
  switch (dtype) {
    case TVK_DTYPE_F16: return launch_simt<__half>(p, max_seqlen, s);
    case TVK_DTYPE_BF16: return launch_simt<__nv_bfloat16>(p, max_seqlen, s);
    default: return launch_simt<float>(p, max_seqlen, s);
  }
}
