// layer_ops.cu -- the per-layer elementwise / reduction kernels around the
// attention hot path, each one vectorised pass over HBM (16-byte accesses).
//
//   tvk_rms_norm          RMSNorm.__call__             tinyvllm/model/llama.py:21-23 (+ the residual add
//                                                      of TransformerBlock.__call__ llama.py:247-250 fused)
//   tvk_rope              apply_rope                   llama.py:34-55 (interleaved pairs, fp32 tables)
//   tvk_write_kv_slots    KVCache.write_kv             core/kv_cache.py:34-38, decode append llama.py:381-386
//   tvk_rope_write_kv     apply_rope on q and k, then the roped k and v stored into their paged slots
//   tvk_qkv_rope          the same from one packed [q | k | v] projection row (one GEMM for q, k, v)
//   tvk_silu_mul          FeedForward gate             llama.py:220-221
//   tvk_embedding         Embedding row gather         llama.py:276,310
//   tvk_argmax            greedy pick                  core/sampling.py:133-134 (first index on ties)
//
// Arithmetic is fp32; results are rounded once to the storage dtype.
#include <math.h>

#include "tvk_common.cuh"

namespace {

// Every kernel here is launched as a programmatic dependent (tvk::launch_pdl):
// it waits for the kernel before it, and its memory, before its first read, then
// lets the next launch on the stream start.
#define TVK_PDL_ENTER() asm volatile("griddepcontrol.wait;\n\tgriddepcontrol.launch_dependents;" ::: "memory")


// ---- vector helpers: 8 elements of a 16-bit type or 4 floats per 16 bytes ----
template <typename T> struct Vec { static constexpr int N = 16 / sizeof(T); };

template <typename T>
__device__ __forceinline__ void load_vec(const T* p, float* f) {
  const uint4 u = *reinterpret_cast<const uint4*>(p);
  const T* h = reinterpret_cast<const T*>(&u);
#pragma unroll
  for (int i = 0; i < Vec<T>::N; ++i) f[i] = DT<T>::to_f(h[i]);
}
template <typename T>
__device__ __forceinline__ void store_vec(T* p, const float* f) {
  uint4 u;
  T* h = reinterpret_cast<T*>(&u);
#pragma unroll
  for (int i = 0; i < Vec<T>::N; ++i) h[i] = DT<T>::from_f(f[i]);
  *reinterpret_cast<uint4*>(p) = u;
}
// round-trip through the storage dtype (what a separate kernel would have stored)
template <typename T>
__device__ __forceinline__ float round_to(float x) { return DT<T>::to_f(DT<T>::from_f(x)); }

__device__ __forceinline__ float block_sum(float v, float* red) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  if (lane == 0) red[warp] = v;
  __syncthreads();
  const int nw = (blockDim.x + 31) >> 5;
  float t = lane < nw ? red[lane] : 0.f;
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) t += __shfl_xor_sync(0xffffffffu, t, o);
  __syncthreads();
  return t;
}

// ---------------------------------------------------------------------------
// RMSNorm (optionally residual-fused): s = x (+ r); r_out = s; out = s * rsqrt(mean(s^2) + eps) * w
// ---------------------------------------------------------------------------
constexpr int kNormThreads = 256;
constexpr int kNormMaxVec = 8;  // per thread: dim <= 256 * 8 * N

// Optional K/V append carried by the norm kernel (slots null: none).
template <typename T>
struct KvAppend {
  const T* k;
  const T* v;
  const int64_t* slots;
  T* k_cache;
  T* v_cache;
  int row_elems;       // n_kv_heads * head_dim
  long long n_slots;   // num_blocks * block_size
};

// VPT: vectors per thread the row needs (ceil(dim / N / kNormThreads), 1/2/4/8).
template <typename T, int VPT>
__global__ void __launch_bounds__(kNormThreads) rms_norm_kernel(const T* __restrict__ x, const T* residual,
                                                                T* residual_out, const T* __restrict__ w,
                                                                T* __restrict__ out, int dim, float eps,
                                                                KvAppend<T> kv) {
  TVK_PDL_ENTER();
  constexpr int N = Vec<T>::N;
  __shared__ float red[32];
  const size_t row = blockIdx.x;
  // Every load this row needs is issued up front (the slot of the K/V append,
  // the row, the residual and the weight), so their latencies overlap instead of
  // following the reduction.
  const long long slot = kv.slots ? kv.slots[row] : -1;
  const T* xr = x + row * dim;
  const int nvec = dim / N;
  float v[VPT][N], wv[VPT][N];
  float ss = 0.f;
#pragma unroll
  for (int k = 0; k < VPT; ++k) {
    const int i = threadIdx.x + k * kNormThreads;
    if (i < nvec) {
      load_vec<T>(xr + i * N, v[k]);
      load_vec<T>(w + i * N, wv[k]);
      if (residual) {
        float rv[N];
        load_vec<T>(residual + row * dim + i * N, rv);
#pragma unroll
        for (int e = 0; e < N; ++e) v[k][e] = round_to<T>(v[k][e] + rv[e]);
        store_vec<T>(residual_out + row * dim + i * N, v[k]);
      }
#pragma unroll
      for (int e = 0; e < N; ++e) ss = fmaf(v[k][e], v[k][e], ss);
    }
  }
  if (kv.slots && slot >= 0 && slot < kv.n_slots) {
    // This row's new k and v rows go to its paged slot (decode append done
    // after the attention that read the slot's old contents).
    for (int i = threadIdx.x; i < kv.row_elems / N; i += kNormThreads) {
      const size_t src = row * kv.row_elems + (size_t)i * N, dst = (size_t)slot * kv.row_elems + (size_t)i * N;
      *reinterpret_cast<uint4*>(kv.k_cache + dst) = *reinterpret_cast<const uint4*>(kv.k + src);
      *reinterpret_cast<uint4*>(kv.v_cache + dst) = *reinterpret_cast<const uint4*>(kv.v + src);
    }
  }
  const float tot = block_sum(ss, red);
  const float inv = rsqrtf(tot / (float)dim + eps);
#pragma unroll
  for (int k = 0; k < VPT; ++k) {
    const int i = threadIdx.x + k * kNormThreads;
    if (i < nvec) {
      float o[N];
#pragma unroll
      for (int e = 0; e < N; ++e) o[e] = v[k][e] * inv * wv[k][e];
      store_vec<T>(out + row * dim + i * N, o);
    }
  }
}

// ---------------------------------------------------------------------------
// RoPE on interleaved pairs (x[2i], x[2i+1]) with fp32 cos/sin tables [max_pos, D/2]
// ---------------------------------------------------------------------------
// (x0, x1) -> (x0 c - x1 s, x0 s + x1 c), rounded product by product (no fused
// multiply-add), the same in every kernel and as the reference's elementwise ops.
__device__ __forceinline__ void rotate_pair(float& x0, float& x1, float c, float s) {
  const float a = __fsub_rn(__fmul_rn(x0, c), __fmul_rn(x1, s));
  const float b = __fadd_rn(__fmul_rn(x0, s), __fmul_rn(x1, c));
  x0 = a;
  x1 = b;
}

template <typename T>
__device__ __forceinline__ void rope_vec(T* p, const float* c, const float* s) {
  constexpr int N = Vec<T>::N;
  float f[N];
  load_vec<T>(p, f);
#pragma unroll
  for (int e = 0; e < N; e += 2) rotate_pair(f[e], f[e + 1], c[e / 2], s[e / 2]);
  store_vec<T>(p, f);
}

// One thread per 16-byte vector of one head of one token; q heads first, then k heads.
// With slots != null, the roped k vector and the matching v vector are also
// written to the paged pool at flat slot slots[t].
template <typename T>
__global__ void rope_kernel(T* q, T* k, const T* v, const float* __restrict__ cos_t, const float* __restrict__ sin_t,
                            const int32_t* __restrict__ pos, int n_tokens, int hq, int hkv, int D, int max_pos,
                            const int64_t* __restrict__ slots, T* k_cache, T* v_cache, long long n_slots) {
  TVK_PDL_ENTER();
  constexpr int N = Vec<T>::N;
  const int vpr = D / N;  // vectors per head row
  const long long total = (long long)n_tokens * (hq + hkv) * vpr;
  for (long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x; i < total;
       i += (long long)gridDim.x * blockDim.x) {
    const int vi = (int)(i % vpr);
    const long long th = i / vpr;
    const int head = (int)(th % (hq + hkv));
    const int t = (int)(th / (hq + hkv));
    int p = pos[t];
    p = p < 0 ? 0 : (p >= max_pos ? max_pos - 1 : p);
    float c[N / 2], s[N / 2];
#pragma unroll
    for (int e = 0; e < N / 2; ++e) {
      c[e] = cos_t[(size_t)p * (D / 2) + vi * (N / 2) + e];
      s[e] = sin_t[(size_t)p * (D / 2) + vi * (N / 2) + e];
    }
    if (head < hq) {
      rope_vec<T>(q + ((size_t)t * hq + head) * D + vi * N, c, s);
    } else {
      const int kh = head - hq;
      T* kp = k + ((size_t)t * hkv + kh) * D + vi * N;
      rope_vec<T>(kp, c, s);
      if (slots) {
        const long long slot = slots[t];
        if (slot >= 0 && slot < n_slots) {
          const size_t dst = ((size_t)slot * hkv + kh) * D + vi * N;
          *reinterpret_cast<uint4*>(k_cache + dst) = *reinterpret_cast<const uint4*>(kp);
          *reinterpret_cast<uint4*>(v_cache + dst) =
              *reinterpret_cast<const uint4*>(v + ((size_t)t * hkv + kh) * D + vi * N);
        }
      }
    }
  }
}

// ---------------------------------------------------------------------------
// Packed projection rows [q | k | v] -> RoPE'd q and k and v as separate
// contiguous tensors (optionally also the roped k and v into paged slots).
// ---------------------------------------------------------------------------
template <typename T>
__global__ void qkv_rope_kernel(const T* __restrict__ qkv, long long row_stride, T* __restrict__ q,
                                T* __restrict__ k, T* __restrict__ v, const float* __restrict__ cos_t,
                                const float* __restrict__ sin_t, const int32_t* __restrict__ pos, int n_tokens, int hq,
                                int hkv, int D, int max_pos, const int64_t* __restrict__ slots, T* k_cache,
                                T* v_cache, long long n_slots) {
  TVK_PDL_ENTER();
  constexpr int N = Vec<T>::N;
  const int vpr = D / N;
  const int heads = hq + 2 * hkv;
  const long long total = (long long)n_tokens * heads * vpr;
  for (long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x; i < total;
       i += (long long)gridDim.x * blockDim.x) {
    const int vi = (int)(i % vpr);
    const long long th = i / vpr;
    const int head = (int)(th % heads);
    const int t = (int)(th / heads);
    float f[N];
    load_vec<T>(qkv + t * row_stride + (size_t)head * D + vi * N, f);
    if (head < hq + hkv) {
      int p = pos[t];
      p = p < 0 ? 0 : (p >= max_pos ? max_pos - 1 : p);
#pragma unroll
      for (int e = 0; e < N; e += 2)
        rotate_pair(f[e], f[e + 1], cos_t[(size_t)p * (D / 2) + vi * (N / 2) + e / 2],
                    sin_t[(size_t)p * (D / 2) + vi * (N / 2) + e / 2]);
    }
    T* dst;
    T* cache = nullptr;
    int kvh = 0;
    if (head < hq) {
      dst = q + ((size_t)t * hq + head) * D;
    } else if (head < hq + hkv) {
      kvh = head - hq;
      dst = k + ((size_t)t * hkv + kvh) * D;
      cache = k_cache;
    } else {
      kvh = head - hq - hkv;
      dst = v + ((size_t)t * hkv + kvh) * D;
      cache = v_cache;
    }
    store_vec<T>(dst + vi * N, f);
    if (slots && cache) {
      const long long slot = slots[t];
      if (slot >= 0 && slot < n_slots) store_vec<T>(cache + ((size_t)slot * hkv + kvh) * D + vi * N, f);
    }
  }
}

// ---------------------------------------------------------------------------
// K/V rows -> paged slots
// ---------------------------------------------------------------------------
template <typename T>
__global__ void write_kv_kernel(const T* __restrict__ k, const T* __restrict__ v, const int64_t* __restrict__ slots,
                                T* k_cache, T* v_cache, int n_tokens, int row_elems, long long n_slots) {
  TVK_PDL_ENTER();
  constexpr int N = Vec<T>::N;
  const int vpr = row_elems / N;
  const long long total = (long long)n_tokens * vpr;
  for (long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x; i < total;
       i += (long long)gridDim.x * blockDim.x) {
    const int t = (int)(i / vpr), vi = (int)(i % vpr);
    const long long slot = slots[t];
    if (slot < 0 || slot >= n_slots) continue;
    const size_t src = (size_t)t * row_elems + vi * N, dst = (size_t)slot * row_elems + vi * N;
    *reinterpret_cast<uint4*>(k_cache + dst) = *reinterpret_cast<const uint4*>(k + src);
    *reinterpret_cast<uint4*>(v_cache + dst) = *reinterpret_cast<const uint4*>(v + src);
  }
}

// ---------------------------------------------------------------------------
// SiLU gate: out = silu(a) * b, rows with independent strides
// ---------------------------------------------------------------------------
template <typename T>
__global__ void silu_mul_kernel(const T* __restrict__ a, const T* __restrict__ b, T* __restrict__ out, int rows,
                                int cols, long long a_stride, long long b_stride, long long o_stride) {
  TVK_PDL_ENTER();
  constexpr int N = Vec<T>::N;
  const int vpr = cols / N;
  const long long total = (long long)rows * vpr;
  for (long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x; i < total;
       i += (long long)gridDim.x * blockDim.x) {
    const long long r = i / vpr;
    const int c = (int)(i % vpr) * N;
    float fa[N], fb[N];
    load_vec<T>(a + r * a_stride + c, fa);
    load_vec<T>(b + r * b_stride + c, fb);
#pragma unroll
    for (int e = 0; e < N; ++e) {
      const float g = fa[e];
      // silu as the reference composes it: x * sigmoid(x), rounded to the dtype before the product
      fa[e] = round_to<T>(g / (1.f + expf(-g))) * fb[e];
    }
    store_vec<T>(out + r * o_stride + c, fa);
  }
}

// ---------------------------------------------------------------------------
// Embedding gather: out[t] = table[tokens[t]] (out-of-range ids give zeros)
// ---------------------------------------------------------------------------
template <typename T>
__global__ void embedding_kernel(const T* __restrict__ table, const int32_t* __restrict__ tokens, T* __restrict__ out,
                                 int n_tokens, int dim, int vocab, int* status) {
  TVK_PDL_ENTER();
  constexpr int N = Vec<T>::N;
  const int vpr = dim / N;
  const long long total = (long long)n_tokens * vpr;
  for (long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x; i < total;
       i += (long long)gridDim.x * blockDim.x) {
    const int t = (int)(i / vpr), vi = (int)(i % vpr);
    const int id = tokens[t];
    uint4 u = make_uint4(0, 0, 0, 0);
    if (id >= 0 && id < vocab)
      u = *reinterpret_cast<const uint4*>(table + (size_t)id * dim + vi * N);
    else if (vi == 0 && status)
      atomicExch(status, 3);
    *reinterpret_cast<uint4*>(out + (size_t)t * dim + vi * N) = u;
  }
}

// ---------------------------------------------------------------------------
// Greedy argmax per row, first index on ties (NaN rows report the first NaN).
// ---------------------------------------------------------------------------
constexpr int kArgmaxThreads = 512;

__device__ __forceinline__ bool better(float v, int i, float bv, int bi) {
  // larger value wins; equal values: lower index wins; NaN beats everything (first NaN)
  if (isnan(v)) return !isnan(bv) || i < bi;
  if (isnan(bv)) return false;
  return v > bv || (v == bv && i < bi);
}

template <typename T>
__global__ void __launch_bounds__(kArgmaxThreads) argmax_kernel(const T* __restrict__ logits, int32_t* __restrict__ out,
                                                                int vocab, long long row_stride, int vec) {
  TVK_PDL_ENTER();
  constexpr int N = Vec<T>::N;
  __shared__ float sv[32];
  __shared__ int si[32];
  const T* row = logits + blockIdx.x * row_stride;
  float bv = -INFINITY;
  int bi = 0x7fffffff;
  const int nvec = vec ? vocab / N : 0;  // 16-byte loads only when every row is 16-byte aligned
  // Eight independent 16-byte loads in flight per thread, each feeding its own
  // running (max, index) pair so that the compares form eight short chains
  // instead of one long one; the pairs merge at the end (ties go to the lower
  // index whatever the visiting order).
  constexpr int U = 8;
  float cv[U];
  int ci[U];
  int nan_i = 0x7fffffff;  // first NaN seen by this thread's chains
#pragma unroll
  for (int k = 0; k < U; ++k) {
    cv[k] = -INFINITY;
    ci[k] = 0x7fffffff;
  }
  int i = threadIdx.x;
  for (; i + (U - 1) * (int)blockDim.x < nvec; i += U * blockDim.x) {
    uint4 u[U];
#pragma unroll
    for (int k = 0; k < U; ++k) u[k] = __ldg(reinterpret_cast<const uint4*>(row + (size_t)(i + k * blockDim.x) * N));
#pragma unroll
    for (int k = 0; k < U; ++k) {
      const T* h = reinterpret_cast<const T*>(&u[k]);
      const int i0 = (i + k * blockDim.x) * N;
      // Inside one chain the indices only grow, so a strict '>' keeps the first of
      // equal values; NaNs never win a '>' and are tracked apart (first index).
#pragma unroll
      for (int e = 0; e < N; ++e) {
        const float f = DT<T>::to_f(h[e]);
        // a chain's first non-NaN value is always taken (so rows of -inf keep their first index)
        const bool gt = (f > cv[k] || ci[k] == 0x7fffffff) && f == f;
        cv[k] = gt ? f : cv[k];
        ci[k] = gt ? i0 + e : ci[k];
        if (f != f) nan_i = min(nan_i, i0 + e);
      }
    }
  }
#pragma unroll
  for (int k = 0; k < U; ++k)
    if (better(cv[k], ci[k], bv, bi)) {
      bv = cv[k];
      bi = ci[k];
    }
  if (nan_i != 0x7fffffff && better(__int_as_float(0x7fc00000), nan_i, bv, bi)) {
    bv = __int_as_float(0x7fc00000);
    bi = nan_i;
  }
  for (; i < nvec; i += blockDim.x) {
    float f[N];
    load_vec<T>(row + (size_t)i * N, f);
#pragma unroll
    for (int e = 0; e < N; ++e)
      if (better(f[e], i * N + e, bv, bi)) {
        bv = f[e];
        bi = i * N + e;
      }
  }
  for (int i = nvec * N + threadIdx.x; i < vocab; i += blockDim.x) {
    const float f = DT<T>::to_f(row[i]);
    if (better(f, i, bv, bi)) {
      bv = f;
      bi = i;
    }
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    const float ov = __shfl_xor_sync(0xffffffffu, bv, o);
    const int oi = __shfl_xor_sync(0xffffffffu, bi, o);
    if (better(ov, oi, bv, bi)) {
      bv = ov;
      bi = oi;
    }
  }
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  if (lane == 0) {
    sv[warp] = bv;
    si[warp] = bi;
  }
  __syncthreads();
  if (warp == 0) {
    const int nw = blockDim.x >> 5;
    bv = lane < nw ? sv[lane] : -INFINITY;
    bi = lane < nw ? si[lane] : 0x7fffffff;
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
      const float ov = __shfl_xor_sync(0xffffffffu, bv, o);
      const int oi = __shfl_xor_sync(0xffffffffu, bi, o);
      if (better(ov, oi, bv, bi)) {
        bv = ov;
        bi = oi;
      }
    }
    if (lane == 0) out[blockIdx.x] = bi == 0x7fffffff ? 0 : bi;
  }
}

// 16-bit logits: per 16-byte vector a packed max tree (NaN-propagating), one
// compare with the thread's running max, and only when a vector holds a new
// maximum (a few times per thread) a scan for its first index.  A vector whose
// max is NaN records the thread's first NaN instead (NaN beats every value).
// Comparing in the 16-bit type orders values exactly as comparing their fp32
// conversions does.
template <typename T> struct Pack2;
template <> struct Pack2<__half> {
  using type = __half2;
};
template <> struct Pack2<__nv_bfloat16> {
  using type = __nv_bfloat162;
};

template <typename T>
__global__ void __launch_bounds__(kArgmaxThreads) argmax16_kernel(const T* __restrict__ logits,
                                                                  int32_t* __restrict__ out, int vocab,
                                                                  long long row_stride) {
  TVK_PDL_ENTER();
  using T2 = typename Pack2<T>::type;
  __shared__ float sv[32];
  __shared__ int si[32];
  const T* row = logits + blockIdx.x * row_stride;
  float bv = -INFINITY;
  int bi = 0x7fffffff, nan_i = 0x7fffffff;
  const int nvec = vocab / 8;
  auto visit = [&](const uint4& u, int i0) {
    const T2* w = reinterpret_cast<const T2*>(&u);
    const T2 c = __hmax2_nan(__hmax2_nan(w[0], w[1]), __hmax2_nan(w[2], w[3]));
    const float fm = DT<T>::to_f(__hmax_nan(c.x, c.y));
    if (fm != fm) {  // a NaN in this vector: the thread's first NaN (vectors come in increasing order)
      if (nan_i == 0x7fffffff) {
        const T* h = reinterpret_cast<const T*>(&u);
        for (int e = 7; e >= 0; --e)
          if (DT<T>::to_f(h[e]) != DT<T>::to_f(h[e])) nan_i = i0 + e;
      }
    } else if (fm > bv || bi == 0x7fffffff) {  // new maximum (or the thread's first vector)
      const T* h = reinterpret_cast<const T*>(&u);
      int e0 = 7;
      for (int e = 7; e >= 0; --e)
        if (DT<T>::to_f(h[e]) == fm) e0 = e;
      bv = fm;
      bi = i0 + e0;
    }
  };
  constexpr int U = 8;
  int i = threadIdx.x;
  for (; i + (U - 1) * (int)blockDim.x < nvec; i += U * blockDim.x) {
    uint4 u[U];
#pragma unroll
    for (int k = 0; k < U; ++k) u[k] = __ldg(reinterpret_cast<const uint4*>(row + (size_t)(i + k * blockDim.x) * 8));
#pragma unroll
    for (int k = 0; k < U; ++k) visit(u[k], (i + k * blockDim.x) * 8);
  }
  for (; i < nvec; i += blockDim.x) visit(__ldg(reinterpret_cast<const uint4*>(row + (size_t)i * 8)), i * 8);
  for (int j = nvec * 8 + threadIdx.x; j < vocab; j += blockDim.x) {  // tail of a row not a multiple of 8
    const float f = DT<T>::to_f(row[j]);
    if (f != f) {
      nan_i = min(nan_i, j);
    } else if (better(f, j, bv, bi)) {
      bv = f;
      bi = j;
    }
  }
  // A NaN anywhere wins: carry it as the candidate value (better() ranks NaN first).
  if (nan_i != 0x7fffffff) {
    bv = __int_as_float(0x7fc00000);
    bi = nan_i;
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    const float ov = __shfl_xor_sync(0xffffffffu, bv, o);
    const int oi = __shfl_xor_sync(0xffffffffu, bi, o);
    if (better(ov, oi, bv, bi)) {
      bv = ov;
      bi = oi;
    }
  }
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  if (lane == 0) {
    sv[warp] = bv;
    si[warp] = bi;
  }
  __syncthreads();
  if (warp == 0) {
    const int nw = blockDim.x >> 5;
    bv = lane < nw ? sv[lane] : -INFINITY;
    bi = lane < nw ? si[lane] : 0x7fffffff;
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
      const float ov = __shfl_xor_sync(0xffffffffu, bv, o);
      const int oi = __shfl_xor_sync(0xffffffffu, bi, o);
      if (better(ov, oi, bv, bi)) {
        bv = ov;
        bi = oi;
      }
    }
    if (lane == 0) out[blockIdx.x] = bi == 0x7fffffff ? 0 : bi;
  }
}

int grid_for(long long work, int threads) {
  long long g = (work + threads - 1) / threads;
  const long long cap = 148LL * 16;
  return (int)(g < 1 ? 1 : (g > cap ? cap : g));
}

bool aligned16(const void* p) { return ((uintptr_t)p & 15) == 0; }

#define TVK_DISPATCH(dtype, ...)                                   \
  switch (dtype) {                                                 \
    case TVK_DTYPE_F16: { using T = __half; __VA_ARGS__; break; }  \
    case TVK_DTYPE_BF16: { using T = __nv_bfloat16; __VA_ARGS__; break; } \
    case TVK_DTYPE_F32: { using T = float; __VA_ARGS__; break; }   \
    default: ::tvk::set_error("unknown dtype %d", dtype); return TVK_ERR_INVALID; \
  }

int vec_elems(int dtype) { return dtype == TVK_DTYPE_F32 ? 4 : 8; }

template <typename T>
void launch_rms_norm(int rows, int dim, cudaStream_t s, const T* x, const T* residual, T* residual_out, const T* w,
                     T* out, float eps, const KvAppend<T>& kv) {
  const int vpt = (dim / Vec<T>::N + kNormThreads - 1) / kNormThreads;
  if (vpt <= 1) tvk::launch_pdl(rms_norm_kernel<T, 1>, rows, kNormThreads, 0, s, x, residual, residual_out, w, out, dim, eps, kv);
  else if (vpt <= 2) tvk::launch_pdl(rms_norm_kernel<T, 2>, rows, kNormThreads, 0, s, x, residual, residual_out, w, out, dim, eps, kv);
  else if (vpt <= 4) tvk::launch_pdl(rms_norm_kernel<T, 4>, rows, kNormThreads, 0, s, x, residual, residual_out, w, out, dim, eps, kv);
  else tvk::launch_pdl(rms_norm_kernel<T, kNormMaxVec>, rows, kNormThreads, 0, s, x, residual, residual_out, w, out, dim, eps, kv);
}

}  // namespace

extern "C" int tvk_rms_norm(const void* x, const void* residual, void* residual_out, const void* weight, void* out,
                            int rows, int dim, float eps, int dtype, void* stream) {
  TVK_CHECK_ARG(rows >= 0 && dim > 0, "bad shape rows=%d dim=%d", rows, dim);
  if (rows == 0) return TVK_OK;
  TVK_CHECK_ARG(x && weight && out, "null pointer argument");
  TVK_CHECK_ARG(!residual == !residual_out, "residual and residual_out go together");
  TVK_CHECK_ARG(rows <= 0x7fffffff, "too many rows");
  const int N = vec_elems(dtype);
  TVK_CHECK_ARG(dim % N == 0 && dim / N <= kNormThreads * kNormMaxVec,
                "dim %d must be a multiple of %d and at most %d", dim, N, N * kNormThreads * kNormMaxVec);
  TVK_CHECK_ARG(aligned16(x) && aligned16(weight) && aligned16(out) && (!residual || (aligned16(residual) &&
                aligned16(residual_out))), "pointers must be 16-byte aligned");
  cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
  TVK_DISPATCH(dtype, launch_rms_norm<T>(rows, dim, s, (const T*)x, (const T*)residual, (T*)residual_out,
                                         (const T*)weight, (T*)out, eps, KvAppend<T>{}));
  TVK_CHECK_LAUNCH("rms_norm");
  return TVK_OK;
}

extern "C" int tvk_rms_norm_write_kv(const void* x, const void* residual, void* residual_out, const void* weight,
                                     void* out, int rows, int dim, float eps, const void* k, const void* v,
                                     const int64_t* slots, void* k_cache, void* v_cache, int n_kv_heads,
                                     int head_dim, int num_blocks, int block_size, int dtype, void* stream) {
  TVK_CHECK_ARG(rows >= 0 && dim > 0, "bad shape rows=%d dim=%d", rows, dim);
  if (rows == 0) return TVK_OK;
  TVK_CHECK_ARG(x && weight && out && k && v && slots && k_cache && v_cache, "null pointer argument");
  TVK_CHECK_ARG(!residual == !residual_out, "residual and residual_out go together");
  const int N = vec_elems(dtype);
  TVK_CHECK_ARG(dim % N == 0 && dim / N <= kNormThreads * kNormMaxVec,
                "dim %d must be a multiple of %d and at most %d", dim, N, N * kNormThreads * kNormMaxVec);
  TVK_CHECK_ARG(n_kv_heads > 0 && head_dim > 0 && (n_kv_heads * head_dim) % N == 0,
                "n_kv_heads * head_dim must be a positive multiple of %d", N);
  TVK_CHECK_ARG(num_blocks > 0 && block_size > 0, "num_blocks and block_size must be positive");
  TVK_CHECK_ARG(aligned16(x) && aligned16(weight) && aligned16(out) && aligned16(k) && aligned16(v) &&
                    aligned16(k_cache) && aligned16(v_cache) &&
                    (!residual || (aligned16(residual) && aligned16(residual_out))),
                "pointers must be 16-byte aligned");
  cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
  TVK_DISPATCH(dtype, launch_rms_norm<T>(rows, dim, s, (const T*)x, (const T*)residual, (T*)residual_out,
                                         (const T*)weight, (T*)out, eps,
                                         KvAppend<T>{(const T*)k, (const T*)v, slots, (T*)k_cache, (T*)v_cache,
                                                     n_kv_heads * head_dim, (long long)num_blocks * block_size}));
  TVK_CHECK_LAUNCH("rms_norm_write_kv");
  return TVK_OK;
}

extern "C" int tvk_rope(void* q, void* k, const float* cos_table, const float* sin_table, const int32_t* positions,
                        int n_tokens, int n_heads, int n_kv_heads, int head_dim, int max_pos, int dtype,
                        void* stream) {
  TVK_CHECK_ARG(n_tokens >= 0, "negative n_tokens");
  if (n_tokens == 0) return TVK_OK;
  TVK_CHECK_ARG(q && k && cos_table && sin_table && positions, "null pointer argument");
  TVK_CHECK_ARG(head_dim % vec_elems(dtype) == 0 && max_pos > 0, "head_dim must be a multiple of %d",
                vec_elems(dtype));
  TVK_CHECK_ARG(aligned16(q) && aligned16(k), "q and k must be 16-byte aligned");
  cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
  const long long work = (long long)n_tokens * (n_heads + n_kv_heads) * (head_dim / vec_elems(dtype));
  TVK_DISPATCH(dtype, tvk::launch_pdl(rope_kernel<T>, grid_for(work, 256), 256, 0, s, 
      (T*)q, (T*)k, nullptr, cos_table, sin_table, positions, n_tokens, n_heads, n_kv_heads, head_dim, max_pos,
      nullptr, nullptr, nullptr, 0));
  TVK_CHECK_LAUNCH("rope");
  return TVK_OK;
}

extern "C" int tvk_rope_write_kv(void* q, void* k, const void* v, const float* cos_table, const float* sin_table,
                                 const int32_t* positions, const int64_t* slots, void* k_cache, void* v_cache,
                                 int n_tokens, int n_heads, int n_kv_heads, int head_dim, int max_pos,
                                 int num_blocks, int block_size, int dtype, void* stream) {
  TVK_CHECK_ARG(n_tokens >= 0, "negative n_tokens");
  if (n_tokens == 0) return TVK_OK;
  TVK_CHECK_ARG(q && k && v && cos_table && sin_table && positions && slots && k_cache && v_cache,
                "null pointer argument");
  TVK_CHECK_ARG(head_dim % vec_elems(dtype) == 0 && max_pos > 0 && num_blocks > 0 && block_size > 0,
                "bad shape");
  TVK_CHECK_ARG(aligned16(q) && aligned16(k) && aligned16(v) && aligned16(k_cache) && aligned16(v_cache),
                "pointers must be 16-byte aligned");
  cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
  const long long work = (long long)n_tokens * (n_heads + n_kv_heads) * (head_dim / vec_elems(dtype));
  TVK_DISPATCH(dtype, tvk::launch_pdl(rope_kernel<T>, grid_for(work, 256), 256, 0, s, 
      (T*)q, (T*)k, (const T*)v, cos_table, sin_table, positions, n_tokens, n_heads, n_kv_heads, head_dim, max_pos,
      slots, (T*)k_cache, (T*)v_cache, (long long)num_blocks * block_size));
  TVK_CHECK_LAUNCH("rope_write_kv");
  return TVK_OK;
}

extern "C" int tvk_qkv_rope(const void* qkv, long long row_stride, void* q, void* k, void* v, const float* cos_table,
                            const float* sin_table, const int32_t* positions, const int64_t* slots, void* k_cache,
                            void* v_cache, int n_tokens, int n_heads, int n_kv_heads, int head_dim, int max_pos,
                            int num_blocks, int block_size, int dtype, void* stream) {
  TVK_CHECK_ARG(n_tokens >= 0, "negative n_tokens");
  if (n_tokens == 0) return TVK_OK;
  TVK_CHECK_ARG(qkv && q && k && v && cos_table && sin_table && positions, "null pointer argument");
  const int N = vec_elems(dtype);
  TVK_CHECK_ARG(head_dim % N == 0 && max_pos > 0 && row_stride % N == 0 &&
                    row_stride >= (long long)(n_heads + 2 * n_kv_heads) * head_dim,
                "bad shape (head_dim and row_stride multiples of %d, row_stride >= (n_heads + 2 n_kv_heads) head_dim)",
                N);
  TVK_CHECK_ARG(aligned16(qkv) && aligned16(q) && aligned16(k) && aligned16(v), "pointers must be 16-byte aligned");
  if (slots) {
    TVK_CHECK_ARG(k_cache && v_cache && num_blocks > 0 && block_size > 0 && aligned16(k_cache) && aligned16(v_cache),
                  "slots need 16-byte aligned k_cache and v_cache, num_blocks and block_size");
  }
  cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
  const long long work = (long long)n_tokens * (n_heads + 2 * n_kv_heads) * (head_dim / N);
  TVK_DISPATCH(dtype, tvk::launch_pdl(qkv_rope_kernel<T>, grid_for(work, 256), 256, 0, s, 
      (const T*)qkv, row_stride, (T*)q, (T*)k, (T*)v, cos_table, sin_table, positions, n_tokens, n_heads, n_kv_heads,
      head_dim, max_pos, slots, (T*)k_cache, (T*)v_cache, slots ? (long long)num_blocks * block_size : 0));
  TVK_CHECK_LAUNCH("qkv_rope");
  return TVK_OK;
}

extern "C" int tvk_write_kv_slots(const void* k, const void* v, const int64_t* slots, void* k_cache, void* v_cache,
                                  int n_tokens, int n_kv_heads, int head_dim, int num_blocks, int block_size,
                                  int dtype, void* stream) {
  TVK_CHECK_ARG(n_tokens >= 0, "negative n_tokens");
  if (n_tokens == 0) return TVK_OK;
  TVK_CHECK_ARG(k && v && slots && k_cache && v_cache, "null pointer argument");
  const int row = n_kv_heads * head_dim;
  TVK_CHECK_ARG(row > 0 && row % vec_elems(dtype) == 0 && num_blocks > 0 && block_size > 0, "bad shape");
  TVK_CHECK_ARG(aligned16(k) && aligned16(v) && aligned16(k_cache) && aligned16(v_cache),
                "pointers must be 16-byte aligned");
  cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
  const long long work = (long long)n_tokens * (row / vec_elems(dtype));
  TVK_DISPATCH(dtype, tvk::launch_pdl(write_kv_kernel<T>, grid_for(work, 256), 256, 0, s, 
      (const T*)k, (const T*)v, slots, (T*)k_cache, (T*)v_cache, n_tokens, row, (long long)num_blocks * block_size));
  TVK_CHECK_LAUNCH("write_kv");
  return TVK_OK;
}

extern "C" int tvk_silu_mul(const void* a, const void* b, void* out, int rows, int cols, long long a_stride,
                            long long b_stride, long long out_stride, int dtype, void* stream) {
  TVK_CHECK_ARG(rows >= 0 && cols > 0, "bad shape");
  if (rows == 0) return TVK_OK;
  TVK_CHECK_ARG(a && b && out, "null pointer argument");
  const int N = vec_elems(dtype);
  TVK_CHECK_ARG(cols % N == 0 && a_stride % N == 0 && b_stride % N == 0 && out_stride % N == 0,
                "cols and strides must be multiples of %d", N);
  TVK_CHECK_ARG(aligned16(a) && aligned16(b) && aligned16(out), "pointers must be 16-byte aligned");
  cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
  const long long work = (long long)rows * (cols / N);
  TVK_DISPATCH(dtype, tvk::launch_pdl(silu_mul_kernel<T>, grid_for(work, 256), 256, 0, s, 
      (const T*)a, (const T*)b, (T*)out, rows, cols, a_stride, b_stride, out_stride));
  TVK_CHECK_LAUNCH("silu_mul");
  return TVK_OK;
}

extern "C" int tvk_embedding(const void* table, const int32_t* tokens, void* out, int n_tokens, int dim, int vocab,
                             int dtype, int* status, void* stream) {
  TVK_CHECK_ARG(n_tokens >= 0 && dim > 0 && vocab > 0, "bad shape");
  if (n_tokens == 0) return TVK_OK;
  TVK_CHECK_ARG(table && tokens && out, "null pointer argument");
  TVK_CHECK_ARG(dim % vec_elems(dtype) == 0, "dim must be a multiple of %d", vec_elems(dtype));
  TVK_CHECK_ARG(aligned16(table) && aligned16(out), "pointers must be 16-byte aligned");
  cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
  const long long work = (long long)n_tokens * (dim / vec_elems(dtype));
  TVK_DISPATCH(dtype, tvk::launch_pdl(embedding_kernel<T>, grid_for(work, 256), 256, 0, s, 
      (const T*)table, tokens, (T*)out, n_tokens, dim, vocab, status));
  TVK_CHECK_LAUNCH("embedding");
  return TVK_OK;
}

extern "C" int tvk_argmax(const void* logits, int32_t* out, int rows, int vocab, long long row_stride, int dtype,
                          void* stream) {
  TVK_CHECK_ARG(rows >= 0 && vocab > 0 && row_stride >= vocab, "bad shape");
  if (rows == 0) return TVK_OK;
  TVK_CHECK_ARG(logits && out, "null pointer argument");
  const int vec = aligned16(logits) && row_stride % vec_elems(dtype) == 0;
  cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
  if (vec && dtype == TVK_DTYPE_F16) {
    tvk::launch_pdl(argmax16_kernel<__half>, rows, kArgmaxThreads, 0, s, (const __half*)logits, out, vocab, row_stride);
  } else if (vec && dtype == TVK_DTYPE_BF16) {
    tvk::launch_pdl(argmax16_kernel<__nv_bfloat16>, rows, kArgmaxThreads, 0, s, (const __nv_bfloat16*)logits, out, vocab,
                                                                    row_stride);
  } else {
    TVK_DISPATCH(dtype,
                 tvk::launch_pdl(argmax_kernel<T>, rows, kArgmaxThreads, 0, s, (const T*)logits, out, vocab, row_stride, vec));
  }
  TVK_CHECK_LAUNCH("argmax");
  return TVK_OK;
}
