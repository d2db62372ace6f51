// prefill_sm100.cu -- causal flash prefill with the fused paged K/V write.
//
// Replaces flash_prefill_attention (tinyvllm/model/llama.py:58-94) and the
// per-block K/V writes of Attention._write_kv_to_blocks (llama.py:188-209,
// core/kv_cache.py:34-38).  The reference materialises the whole [H, L, L]
// score matrix, expands GQA heads and masks after the full Q.K^T; here each CTA
// owns one 128-row query tile of one head of one prompt, walks only the key
// tiles at or below the diagonal, and never leaves the chip with scores.
//
// tcgen05 kernel (fp16/bf16, head_dim 64 or 128), 6 warps:
//   warp 0  TMA producer: Q once, then K/V 128-token tiles into a ring; for the
//           diagonal tile (this CTA's own tokens) of the first query head of a
//           KV group it also copies the landed K/V rows into their paged slots.
//   warp 1  owns TMEM (512 columns) and issues the MMAs from one thread:
//           S_j = Q.K_j^T (M=128, N=128, fp32 in TMEM, double buffered) and
//           O_j = P_j.V_j (M=128, N=head_dim, fp32 in TMEM, double buffered).
//   warps 2-5  softmax: one query row per thread, S read with tcgen05.ld,
//           online softmax in the log2 domain, P written to shared memory in
//           the 128-byte swizzled K-major layout, O_j folded into a register
//           accumulator with the running rescale.
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
  const int32_t* sched;         // tc path: (seq << 16 | query tile) items, heaviest first
  const int32_t* sched_count;   // tc path: number of entries in sched
  int n_seqs, n_heads, n_kv_heads, group, head_dim, causal, num_blocks, block_size, n_mtiles;
  float scale_log2;
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

template <int D>
struct PfCfg {
  static constexpr int kKB = D / 64;               // 64-element (128 B) column blocks per row
  static constexpr int kBlockBytes = 128 * 128;    // one column block of a 128-row tile
  static constexpr int kTileBytes = 128 * D * 2;   // one 128-row tile of Q, K or V
  static constexpr int kStages = 3;                // K/V ring depth
  static constexpr int kSBufs = D == 64 ? 1 : 2;   // S buffers in TMEM
  static constexpr int kQOff = 0;
  static constexpr int kKOff = kQOff + kTileBytes;
  static constexpr int kVOff = kKOff + kStages * kTileBytes;
  static constexpr int kBarOff = kVOff + kStages * kTileBytes;
  // q_full, q_empty, k_full[S], v_full[S], kv_empty[S], s_full[SB], s_empty[SB], p_full, pv_done, o_empty, final
  static constexpr int kNumBars = 2 + 3 * kStages + 2 * kSBufs + 4;
  static constexpr int kMiscOff = kBarOff + kNumBars * 8;  // tmem slot, abort flag
  static constexpr int kUsed = kMiscOff + 16;
  // head_dim 64: 113 KB so that two CTAs share an SM (2 x (113 + 1 reserved) KB = 228 KB);
  // the slack above kUsed absorbs the 1024-byte alignment of the base.
  static constexpr int kCtasPerSm = D == 64 ? 2 : 1;
  static constexpr int kSmemBytes = D == 64 ? 115712 : kUsed + 1024;
  // TMEM columns: S buffers, then the O accumulator, then P (128 keys as 64
  // columns of packed 16-bit pairs, the A operand of P.V)
  static constexpr uint32_t kOCol = kSBufs * 128;
  static constexpr uint32_t kPCol = kOCol + D;
  static constexpr uint32_t kTmemCols = kPCol + 64 <= 256 ? 256 : 512;
  static_assert(kUsed <= kSmemBytes, "shared memory layout overflows");
};

// One unit of work: a 128-row query tile of one head of one prompt.
struct Item {
  int seq, mtile, h, s0, L;
};

// Round k of this CTA's work: item w = k*G + i (k even) or k*G + G-1-i (k odd)
// of the schedule (query tiles sorted heaviest first, each expanded over the
// query heads).  The snake order balances the heavy early items with light
// late ones across CTAs.
__device__ __forceinline__ bool next_item(const PrefillParams& p, int n_items, int& k, Item& it) {
  const int G = gridDim.x, i = blockIdx.x;
  const int w = k * G + ((k & 1) ? (G - 1 - i) : i);
  if (w >= n_items) return false;
  const int e = __ldg(p.sched + w / p.n_heads);
  const int seq = e >> 16, m = e & 0xFFFF;
  const int s0 = __ldg(p.cu_seqlens + seq);
  it = Item{seq, m, w % p.n_heads, s0, __ldg(p.cu_seqlens + seq + 1) - s0};
  ++k;
  return true;
}

template <typename T, int D>
__global__ void __launch_bounds__(192, PfCfg<D>::kCtasPerSm)
    flash_prefill_tc_kernel(const PrefillParams p, const __grid_constant__ CUtensorMap tm_q,
                            const __grid_constant__ CUtensorMap tm_k, const __grid_constant__ CUtensorMap tm_v) {
  using C = PfCfg<D>;
  constexpr int S = C::kStages, SB = C::kSBufs;
  constexpr bool kBf16 = std::is_same<T, __nv_bfloat16>::value;

  extern __shared__ uint8_t smem_raw[];
  const uint32_t raw_u32 = ptx::smem_u32(smem_raw);
  const uint32_t base_u32 = (raw_u32 + 1023u) & ~1023u;
  if (base_u32 + C::kUsed > raw_u32 + C::kSmemBytes) {  // cannot happen with a >=128 B aligned base
    if (threadIdx.x == 0) report(p.status);
    return;
  }
  uint8_t* base = smem_raw + (base_u32 - raw_u32);
  uint64_t* q_full = reinterpret_cast<uint64_t*>(base + C::kBarOff);
  uint64_t* q_empty = q_full + 1;
  uint64_t* k_full = q_empty + 1;
  uint64_t* v_full = k_full + S;
  uint64_t* kv_empty = v_full + S;
  uint64_t* s_full = kv_empty + S;
  uint64_t* s_empty = s_full + SB;
  uint64_t* p_full = s_empty + SB;
  uint64_t* pv_done = p_full + 1;
  uint64_t* o_empty = pv_done + 1;
  uint64_t* final_bar = o_empty + 1;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(base + C::kMiscOff);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(base + C::kMiscOff + 4);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  if (warp == 1) {
    umma::tmem_alloc(tmem_slot, C::kTmemCols);
    umma::tmem_relinquish();
  }
  if (threadIdx.x == 0) {
    ptx::mbar_init(q_full, 1);
    ptx::mbar_init(q_empty, 1);
    for (int s = 0; s < S; ++s) {
      ptx::mbar_init(&k_full[s], 1);
      ptx::mbar_init(&v_full[s], 1);
      ptx::mbar_init(&kv_empty[s], 1);
    }
    for (int b = 0; b < SB; ++b) {
      ptx::mbar_init(&s_full[b], 1);
      ptx::mbar_init(&s_empty[b], 4);
    }
    ptx::mbar_init(p_full, 4);
    ptx::mbar_init(pv_done, 1);
    ptx::mbar_init(o_empty, 4);
    ptx::mbar_init(final_bar, 1);
    *abort_flag = 0;
    ptx::fence_mbar_init();
  }
  umma::fence_before_sync();
  __syncthreads();
  umma::fence_after_sync();
  const uint32_t tmem = *tmem_slot;
  const int n_items = __ldg(p.sched_count) * p.n_heads;

  if (warp == 0) {
    // =========================== TMA producer ===============================
    uint32_t kv_it = 0, q_it = 0;
    bool ok = true;
    if (lane == 0) {
      ptx::prefetch_tmap(&tm_q);
      ptx::prefetch_tmap(&tm_k);
      ptx::prefetch_tmap(&tm_v);
    }
    int k = 0;
    Item it;
    while (ok && next_item(p, n_items, k, it)) {
      const int n_kv = p.causal ? it.mtile + 1 : (it.L + 127) / 128;
      const int kvh = it.h / p.group;
      ok = __all_sync(0xffffffffu, wait_or_abort(q_empty, (q_it & 1) ^ 1, abort_flag));
      if (!ok) break;
      if (lane == 0) {
        ptx::mbar_arrive_expect_tx(q_full, C::kTileBytes);
        for (int kb = 0; kb < C::kKB; ++kb)
          tma_load_3d(base + C::kQOff + kb * C::kBlockBytes, &tm_q, q_full, kb * 64, it.h, it.s0 + it.mtile * 128);
      }
      ++q_it;
      const bool write_kv = p.slot_mapping != nullptr && (it.h % p.group) == 0;
      for (int j = 0; j < n_kv; ++j, ++kv_it) {
        const int st = kv_it % S;
        const uint32_t ph = (kv_it / S) & 1;
        ok = __all_sync(0xffffffffu, wait_or_abort(&kv_empty[st], ph ^ 1, abort_flag));
        if (!ok) break;
        uint8_t* ks = base + C::kKOff + st * C::kTileBytes;
        uint8_t* vs = base + C::kVOff + st * C::kTileBytes;
        if (lane == 0) {
          ptx::mbar_arrive_expect_tx(&k_full[st], C::kTileBytes);
          for (int kb = 0; kb < C::kKB; ++kb)
            tma_load_3d(ks + kb * C::kBlockBytes, &tm_k, &k_full[st], kb * 64, kvh, it.s0 + j * 128);
          ptx::mbar_arrive_expect_tx(&v_full[st], C::kTileBytes);
          for (int kb = 0; kb < C::kKB; ++kb)
            tma_load_3d(vs + kb * C::kBlockBytes, &tm_v, &v_full[st], kb * 64, kvh, it.s0 + j * 128);
        }
        if (write_kv && j == it.mtile) {
          // The diagonal tile holds exactly this query tile's own tokens: copy the
          // landed rows into their paged slots (slot = block * block_size + offset).
          ok = __all_sync(0xffffffffu, wait_or_abort(&k_full[st], ph, abort_flag) &&
                                           wait_or_abort(&v_full[st], ph, abort_flag));
          if (!ok) break;
          const int rows = min(128, it.L - it.mtile * 128);
          const long long n_slots = (long long)p.num_blocks * p.block_size;
          T* kc = reinterpret_cast<T*>(p.k_cache);
          T* vc = reinterpret_cast<T*>(p.v_cache);
          for (int i = lane; i < rows * (D / 8); i += 32) {
            const int r = i / (D / 8), c8 = i % (D / 8);
            const long long slot = p.slot_mapping[it.s0 + it.mtile * 128 + r];
            if (slot < 0 || slot >= n_slots) continue;
            const uint32_t off = (c8 / 8) * C::kBlockBytes + r * 128 + ((((c8 & 7) ^ (r & 7))) << 4);
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
      if (q_it > 0) ptx::mbar_wait(q_full, (q_it - 1) & 1, 100000000ull);
    }
  } else if (warp == 1) {
    // =========================== MMA issuer =================================
    if (lane == 0) {
      const uint32_t idesc_s = umma::idesc_f16(128, 128, kBf16, false);
      const uint32_t idesc_o = umma::idesc_f16(128, D, kBf16, true);
      const uint32_t q_addr = base_u32 + C::kQOff;
      uint32_t kv_it = 0, q_it = 0, s_it = 0, pv_it = 0, item_it = 0;
      bool ok = true;
      int k = 0;
      Item it;
      while (ok && next_item(p, n_items, k, it)) {
        const int n_kv = p.causal ? it.mtile + 1 : (it.L + 127) / 128;
        const uint32_t kv_base = kv_it;
        auto issue_pv = [&](int i) -> bool {
          const uint32_t g = kv_base + i;
          const int st = g % S;
          if (!wait_or_abort(p_full, pv_it & 1, abort_flag)) return false;
          if (i == 0 && !wait_or_abort(o_empty, (item_it & 1) ^ 1, abort_flag)) return false;
          if (!wait_or_abort(&v_full[st], (g / S) & 1, abort_flag)) return false;
          umma::fence_after_sync();
          const uint32_t v_addr = base_u32 + C::kVOff + st * C::kTileBytes;
#pragma unroll
          for (int ks = 0; ks < 8; ++ks) {  // 16 keys per MMA: 8 TMEM columns of P
            const uint64_t bd = umma::smem_desc_sw128(v_addr + ks * 2048, C::kBlockBytes, 1024);
            umma::mma_f16_ts(tmem + C::kOCol, tmem + C::kPCol + ks * 8, bd, idesc_o, (i > 0 || ks > 0) ? 1u : 0u);
          }
          umma::commit(pv_done);
          umma::commit(&kv_empty[st]);
          ++pv_it;
          return true;
        };
        ok = wait_or_abort(q_full, q_it & 1, abort_flag);
        for (int j = 0; ok && j < n_kv; ++j) {
          const uint32_t g = kv_base + j;
          const int st = g % S;
          const int sb = s_it % SB;
          ok = wait_or_abort(&k_full[st], (g / S) & 1, abort_flag) &&
               wait_or_abort(&s_empty[sb], ((s_it / SB) & 1) ^ 1, abort_flag);
          if (!ok) break;
          umma::fence_after_sync();
          const uint32_t k_addr = base_u32 + C::kKOff + st * C::kTileBytes;
#pragma unroll
          for (int ks = 0; ks < D / 16; ++ks) {
            const uint64_t ad = umma::smem_desc_sw128(q_addr + (ks >> 2) * C::kBlockBytes + (ks & 3) * 32, 16, 1024);
            const uint64_t bd = umma::smem_desc_sw128(k_addr + (ks >> 2) * C::kBlockBytes + (ks & 3) * 32, 16, 1024);
            umma::mma_f16_ss(tmem + sb * 128, ad, bd, idesc_s, ks > 0 ? 1u : 0u);
          }
          umma::commit(&s_full[sb]);
          ++s_it;
          if (j == n_kv - 1) umma::commit(q_empty);  // Q is free once this item's S MMAs are done
          if (j >= 1) ok = issue_pv(j - 1);
        }
        if (ok) ok = issue_pv(n_kv - 1);
        kv_it += n_kv;
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
    uint32_t s_it = 0, pv_it = 0;
    bool ok = true;
    int k = 0;
    Item it;
    while (ok && next_item(p, n_items, k, it)) {
      const int n_kv = p.causal ? it.mtile + 1 : (it.L + 127) / 128;
      const int q_pos = it.mtile * 128 + r;
      const int lim = p.causal ? min(q_pos + 1, it.L) : it.L;  // keys [0, lim) are visible
      float m = -INFINITY;  // running max (log2 domain) that P and O are scaled by
      float l = 0.f;
      for (int j = 0; j < n_kv; ++j) {
        const int sb = s_it % SB;
        ok = __all_sync(0xffffffffu, wait_or_abort(&s_full[sb], (s_it / SB) & 1, abort_flag));
        if (!ok) break;
        umma::fence_after_sync();
        const int lim_rel = lim - j * 128;  // keys [0, lim_rel) of this tile are visible
        const uint32_t s_addr = t_lane + sb * 128;
        // pass 1: row max of the visible raw scores (two 64-column loads per wait)
        float mx = -INFINITY;
#pragma unroll
        for (int c = 0; c < 4; c += 2) {
          float s[64];
          umma::ld_32x32b_x32(s_addr + c * 32, *reinterpret_cast<float(*)[32]>(&s[0]));
          umma::ld_32x32b_x32(s_addr + c * 32 + 32, *reinterpret_cast<float(*)[32]>(&s[32]));
          umma::ld_wait();
          if (lim_rel >= 128) {
#pragma unroll
            for (int x = 0; x < 64; ++x) mx = fmaxf(mx, s[x]);
          } else {
#pragma unroll
            for (int x = 0; x < 64; ++x) mx = fmaxf(mx, c * 32 + x < lim_rel ? s[x] : -INFINITY);
          }
        }
        float m_cand = fmaxf(m, mx * sl2);
        if (m_cand == -INFINITY) m_cand = 0.f;  // no visible key (cannot happen for a live tile)
        // P is single-buffered and O is rescaled in place, so the previous P.V must be
        // complete before either is touched; wait for it as late as possible.
        bool pv_waited = (j == 0);
        if (j == 0) {
          m = m_cand;
        } else if (__any_sync(0xffffffffu, m_cand > m + 8.f)) {
          // Lazy rescale: the stale max is kept unless the new one is 2^8 larger.
          ok = __all_sync(0xffffffffu, wait_or_abort(pv_done, pv_it & 1, abort_flag));
          if (!ok) break;
          ++pv_it;
          pv_waited = true;
          umma::fence_after_sync();
          const float corr = ex2(m - m_cand);
#pragma unroll
          for (int c = 0; c < D / 32; ++c) {
            float o[32];
            umma::ld_32x32b_x32(t_lane + C::kOCol + c * 32, o);
            umma::ld_wait();
#pragma unroll
            for (int x = 0; x < 32; ++x) o[x] *= corr;
            umma::st_32x32b_x32(t_lane + C::kOCol + c * 32, o);
          }
          umma::st_wait();
          l *= corr;
          m = m_cand;
        }
        // P (TMEM, single-buffered) is still the A operand of the previous P.V until it completes
        if (!pv_waited) {
          ok = __all_sync(0xffffffffu, wait_or_abort(pv_done, pv_it & 1, abort_flag));
          if (!ok) break;
          ++pv_it;
        }
        // pass 2: P = 2^(s*scale - m), packed to fp16/bf16 pairs and stored to TMEM
        // (row r = lane, 64 columns for 128 keys): the A operand of P.V
        float sum = 0.f;
#pragma unroll
        for (int hf = 0; hf < 2; ++hf) {
          float s[64];
          umma::ld_32x32b_x32(s_addr + hf * 64, *reinterpret_cast<float(*)[32]>(&s[0]));
          umma::ld_32x32b_x32(s_addr + hf * 64 + 32, *reinterpret_cast<float(*)[32]>(&s[32]));
          umma::ld_wait();
          if (lim_rel < 128) {
#pragma unroll
            for (int x = 0; x < 64; ++x) s[x] = hf * 64 + x < lim_rel ? s[x] : -INFINITY;
          }
          uint32_t pk[32];
#pragma unroll
          for (int x = 0; x < 32; ++x) {
            const float p0 = ex2(fmaf(s[2 * x], sl2, -m));
            const float p1 = ex2(fmaf(s[2 * x + 1], sl2, -m));
            sum += p0 + p1;
            pk[x] = DT<T>::pack2(p0, p1);
          }
          umma::st_32x32b_x32_u(t_lane + C::kPCol + hf * 32, pk);
        }
        umma::st_wait();
        // S has been read: hand the TMEM buffer back to the MMA warp.
        umma::fence_before_sync();
        __syncwarp();
        if (lane == 0) ptx::mbar_arrive(&s_empty[sb]);
        ++s_it;
        l += sum;
        umma::fence_before_sync();
        __syncwarp();
        if (lane == 0) ptx::mbar_arrive(p_full);
      }
      if (!ok) break;
      // ---- item done: O (TMEM) / l -> out
      ok = __all_sync(0xffffffffu, wait_or_abort(pv_done, pv_it & 1, abort_flag));
      if (!ok) break;
      ++pv_it;
      umma::fence_after_sync();
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
                                                                int n_bands, int capacity, int32_t* sched,
                                                                int32_t* count, int* status) {
  __shared__ int band[kMaxBands];
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
    const int nt = min((cu[s + 1] - cu[s] + 127) / 128, n_bands);
    for (int m = nt - 1; m >= 0; --m) {
      const int pos = atomicAdd(&band[m], 1);
      if (pos < capacity) sched[pos] = (s << 16) | m;
    }
  }
}

// -----------------------------------------------------------------------------
// host side
// -----------------------------------------------------------------------------
int encode_rows_map(CUtensorMap* m, const void* ptr, CUtensorMapDataType tdt, int D, int heads, int total) {
  tvk::EncodeTiledFn encode = tvk::encode_tiled_fn();
  if (!encode) {
    tvk::set_error("cuTensorMapEncodeTiled is not available from the driver");
    return TVK_ERR_CUDA;
  }
  cuuint64_t dims[3] = {(cuuint64_t)D, (cuuint64_t)heads, (cuuint64_t)total};
  cuuint64_t strides[2] = {(cuuint64_t)D * 2, (cuuint64_t)heads * D * 2};
  cuuint32_t box[3] = {64u, 1u, 128u};
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
  int rc = encode_rows_map(&tq, p.q, tdt, D, p.n_heads, total);
  if (rc == TVK_OK) rc = encode_rows_map(&tk, p.k, tdt, D, p.n_kv_heads, total);
  if (rc == TVK_OK) rc = encode_rows_map(&tv, p.v, tdt, D, p.n_kv_heads, total);
  if (rc != TVK_OK) return rc;
  auto kern = flash_prefill_tc_kernel<T, D>;
  prefill_schedule_kernel<<<1, 1024, 0, stream>>>(p.cu_seqlens, p.n_seqs, p.n_mtiles, sched_capacity,
                                                  const_cast<int32_t*>(p.sched), const_cast<int32_t*>(p.sched_count),
                                                  p.status);
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
  kern<<<grid, 192, C::kSmemBytes, stream>>>(p, tq, tk, tv);
  TVK_CHECK_LAUNCH("flash_prefill_tc");
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

}  // namespace

extern "C" size_t tvk_flash_prefill_workspace_size(int n_seqs, int total_tokens) {
  if (n_seqs < 0 || total_tokens < 0) return tvk::kWorkspaceHeader;
  const size_t items = (size_t)total_tokens / 128 + (size_t)n_seqs + 1;
  return tvk::kWorkspaceHeader + ((items * 4 + 255) / 256) * 256;
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
  p.scale_log2 = (float)(1.4426950408889634 / sqrt((double)head_dim));
  cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
  const bool tc = dtype != TVK_DTYPE_F32 && (head_dim == 64 || head_dim == 128);
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
    p.sched = w32 + tvk::kWorkspaceHeader / 4;
    const int cap = (int)((need - tvk::kWorkspaceHeader) / 4);
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
