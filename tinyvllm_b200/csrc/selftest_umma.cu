// selftest_umma.cu -- a one-tile tcgen05 GEMM that exercises exactly the
// operand paths of the prefill kernel: an A operand written into shared
// memory by threads in the 128-byte swizzled K-major layout (as P is), and a B
// operand brought in by TMA either K-major (as K is) or MN-major (as V is),
// accumulated in TMEM and read back with tcgen05.ld.  Tests compare it with a
// torch matmul to validate descriptors and layouts in isolation.
#include <type_traits>

#include "tvk_common.cuh"
#include "sm100_umma.cuh"

namespace {

template <typename T>
__global__ void __launch_bounds__(128, 1)
    umma_selftest_kernel(const T* __restrict__ a, float* __restrict__ c, int n, int k, int b_mn_major,
                         int a_in_tmem, int* status, const __grid_constant__ CUtensorMap tm_b) {
  extern __shared__ uint8_t smem_raw[];
  const uint32_t raw = ptx::smem_u32(smem_raw);
  const uint32_t base_u32 = (raw + 1023u) & ~1023u;
  uint8_t* base = smem_raw + (base_u32 - raw);
  uint8_t* sa = base;                    // A: (k/64) blocks of [128 rows x 128 B]
  uint8_t* sb = base + 128 * k * 2;      // B: 128*... bytes
  uint64_t* bar_tma = reinterpret_cast<uint64_t*>(sb + n * k * 2);
  uint64_t* bar_mma = bar_tma + 1;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bar_mma + 1);

  const int tid = threadIdx.x, warp = tid >> 5;
  if (warp == 0) {
    umma::tmem_alloc(tmem_slot, 256);  // D in columns [0, n), A (when in TMEM) in [128, 128 + k/2)
    umma::tmem_relinquish();
  }
  if (tid == 0) {
    ptx::mbar_init(bar_tma, 1);
    ptx::mbar_init(bar_mma, 1);
    ptx::fence_mbar_init();
  }
  // A rows -> swizzled K-major tiles
  for (int i = tid; i < 128 * k / 8; i += 128) {
    const int r = i / (k / 8), c8 = (i % (k / 8)) * 8;
    const uint4 v = *reinterpret_cast<const uint4*>(a + (size_t)r * k + c8);
    *reinterpret_cast<uint4*>(sa + (c8 / 64) * (128 * 128) + umma::sw128_off(r, c8 % 64)) = v;
  }
  umma::fence_proxy_async_smem();
  umma::fence_before_sync();
  __syncthreads();
  umma::fence_after_sync();
  const uint32_t tmem = *tmem_slot;
  if (a_in_tmem) {
    // row r of A -> TMEM lane r, columns 128 + j hold elements (2j, 2j+1)
    const int row = warp * 32 + (tid & 31);
    for (int c0 = 0; c0 < k / 2; c0 += 32) {
      uint32_t u[32];
      const uint32_t* src = reinterpret_cast<const uint32_t*>(a + (size_t)row * k) + c0;
      for (int j = 0; j < 32; ++j) u[j] = src[j];
      umma::st_32x32b_x32_u(tmem + ((uint32_t)(warp * 32) << 16) + 128 + c0, u);
    }
    umma::st_wait();
  }
  umma::fence_before_sync();
  __syncthreads();
  umma::fence_after_sync();

  bool ok = true;
  if (tid == 0) {
    const uint32_t bytes = (uint32_t)(n * k * 2);
    ptx::mbar_arrive_expect_tx(bar_tma, bytes);
    if (!b_mn_major) {
      // B is [n, k] (k contiguous): k/64 boxes of [n rows x 64]
      for (int kb = 0; kb < k / 64; ++kb)
        asm volatile(
            "cp.async.bulk.tensor.2d.shared::cluster.global.tile.mbarrier::complete_tx::bytes"
            " [%0], [%1, {%2, %3}], [%4];" ::"r"(ptx::smem_u32(sb + kb * n * 128)),
            "l"(reinterpret_cast<uint64_t>(&tm_b)), "r"(kb * 64), "r"(0), "r"(ptx::smem_u32(bar_tma))
            : "memory");
    } else {
      // B is [k, n] (n contiguous): n/64 boxes of [k rows x 64]
      for (int nb = 0; nb < n / 64; ++nb)
        asm volatile(
            "cp.async.bulk.tensor.2d.shared::cluster.global.tile.mbarrier::complete_tx::bytes"
            " [%0], [%1, {%2, %3}], [%4];" ::"r"(ptx::smem_u32(sb + nb * k * 128)),
            "l"(reinterpret_cast<uint64_t>(&tm_b)), "r"(nb * 64), "r"(0), "r"(ptx::smem_u32(bar_tma))
            : "memory");
    }
    if (!ptx::mbar_wait(bar_tma, 0)) ok = false;
    if (ok) {
      umma::fence_after_sync();
      const uint32_t idesc = umma::idesc_f16(128, n, sizeof(T) == 2 && !std::is_same<T, __half>::value,
                                             b_mn_major != 0);
      for (int ks = 0; ks < k / 16; ++ks) {
        const uint64_t ad = umma::smem_desc_sw128(ptx::smem_u32(sa) + (ks / 4) * 128 * 128 + (ks % 4) * 32, 16, 1024);
        uint64_t bd;
        if (!b_mn_major)
          bd = umma::smem_desc_sw128(ptx::smem_u32(sb) + (ks / 4) * n * 128 + (ks % 4) * 32, 16, 1024);
        else
          bd = umma::smem_desc_sw128(ptx::smem_u32(sb) + ks * 16 * 128, k * 128, 1024);
        if (a_in_tmem)
          umma::mma_f16_ts(tmem, tmem + 128 + ks * 8, bd, idesc, ks > 0 ? 1u : 0u);
        else
          umma::mma_f16_ss(tmem, ad, bd, idesc, ks > 0 ? 1u : 0u);
      }
      umma::commit(bar_mma);
    }
  }
  __syncthreads();
  if (ok && !ptx::mbar_wait(bar_mma, 0)) ok = false;
  if (!ok) {
    if (status) atomicExch(status, tvk::kStatusWaitTimeout);
  } else {
    umma::fence_after_sync();
    const int row = warp * 32 + (tid & 31);
    for (int c0 = 0; c0 < n; c0 += 32) {
      float r[32];
      umma::ld_32x32b_x32(tmem + ((uint32_t)(warp * 32) << 16) + c0, r);
      umma::ld_wait();
      for (int j = 0; j < 32; ++j) c[(size_t)row * n + c0 + j] = r[j];
    }
  }
  umma::fence_before_sync();
  __syncthreads();
  if (warp == 0) {
    umma::fence_after_sync();
    umma::tmem_dealloc(tmem, 256);
  }
}

}  // namespace

// A comes from shared memory (written swizzled by threads) or, with a_in_tmem,
// from TMEM (written with tcgen05.st, two elements per column).
// C[128, n] (fp32) = A[128, k] . B^T  (B given [n, k]) when b_mn_major == 0,
//                  = A[128, k] . B    (B given [k, n]) when b_mn_major == 1.
// n, k in {64, 128}; dtype fp16 or bf16.  status (may be null) gets 1 on a wait time-out.
extern "C" int tvk_selftest_umma_gemm(const void* a, const void* b, float* c, int n, int k, int b_mn_major,
                                      int a_in_tmem, int dtype, int* status, void* stream) {
  TVK_CHECK_ARG(a && b && c, "null pointer argument");
  TVK_CHECK_ARG((n == 64 || n == 128) && (k == 64 || k == 128), "n and k must be 64 or 128");
  TVK_CHECK_ARG(dtype == TVK_DTYPE_F16 || dtype == TVK_DTYPE_BF16, "dtype must be fp16 or bf16");
  TVK_CHECK_ARG((uintptr_t)a % 16 == 0 && (uintptr_t)b % 16 == 0, "a and b must be 16-byte aligned");
  tvk::EncodeTiledFn encode = tvk::encode_tiled_fn();
  if (!encode) {
    tvk::set_error("cuTensorMapEncodeTiled unavailable");
    return TVK_ERR_CUDA;
  }
  CUtensorMap tm;
  const cuuint64_t inner = b_mn_major ? n : k, outer = b_mn_major ? k : n;
  cuuint64_t dims[2] = {inner, outer};
  cuuint64_t strides[1] = {inner * 2};
  cuuint32_t box[2] = {64u, (cuuint32_t)outer};
  cuuint32_t estr[2] = {1u, 1u};
  CUresult r = encode(&tm, dtype == TVK_DTYPE_F16 ? CU_TENSOR_MAP_DATA_TYPE_FLOAT16 : CU_TENSOR_MAP_DATA_TYPE_BFLOAT16,
                      2, const_cast<void*>(b), dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
                      CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_NONE, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) {
    tvk::set_error("cuTensorMapEncodeTiled failed (%d)", (int)r);
    return TVK_ERR_CUDA;
  }
  const int smem = 128 * k * 2 + n * k * 2 + 64 + 1024;
  cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
  if (dtype == TVK_DTYPE_F16) {
    TVK_CHECK_CUDA(cudaFuncSetAttribute(umma_selftest_kernel<__half>, cudaFuncAttributeMaxDynamicSharedMemorySize, smem));
    umma_selftest_kernel<__half><<<1, 128, smem, s>>>(static_cast<const __half*>(a), c, n, k, b_mn_major, a_in_tmem,
                                                     status, tm);
  } else {
    TVK_CHECK_CUDA(
        cudaFuncSetAttribute(umma_selftest_kernel<__nv_bfloat16>, cudaFuncAttributeMaxDynamicSharedMemorySize, smem));
    umma_selftest_kernel<__nv_bfloat16><<<1, 128, smem, s>>>(static_cast<const __nv_bfloat16*>(a), c, n, k,
                                                             b_mn_major, a_in_tmem, status, tm);
  }
  TVK_CHECK_LAUNCH("umma_selftest");
  return TVK_OK;
}
