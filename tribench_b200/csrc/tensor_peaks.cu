// tensor_peaks.cu — dense tcgen05 throughput microbenchmark (libsm100_peaks.so, C ABI in
// include/sm100_peaks.h). It measures the denominators of the attention kernel's roofline on the
// machine itself: kind::i8 (the QK^T of the sage path), kind::f16 (its 16-bit P.V and the flash
// pack) and kind::f8f6f4 with e4m3 operands (its FP8 P.V).
//
// One CTA per SM (the launch asks for more than half of the SM's shared memory, so no second CTA
// fits). Its 128 threads fill one A tile (128 rows x 128 bytes) and one B tile (N rows x 128
// bytes) in shared memory with pseudo-random operands (finite values for the float kinds, so the
// tensor pipe sees realistic switching and the power draw is realistic), allocate all 512 TMEM
// columns, and one elected thread then issues `mma_per_cta` tcgen05.mma of shape M128 x N x K32B
// (K = 32 bytes of each row: 32 int8 / e4m3 or 16 fp16 elements) back to back, four K-steps per
// 128-byte swizzle atom, alternating between two accumulators. No global memory is touched after
// the launch: the kernel is bound by the tensor pipe alone.
//
// The final wait for the MMAs is bounded (wall-clock limit); on expiry the kernel records the
// failure in *status, waits once more with the same limit, frees TMEM and returns, so a fault in
// this benchmark cannot leave a hung GPU behind.
#include <cuda_runtime.h>

#include <cstdint>
#include <cstdio>
#include <string>

#include "../../include/sm100_peaks.h"
#include "sm100_ptx.cuh"

namespace {

thread_local std::string g_err;

using namespace sage;

__device__ __forceinline__ void umma_f8_ss(uint32_t d_tmem, uint64_t a_desc, uint64_t b_desc, uint32_t idesc,
                                           uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f8f6f4 [%0], %1, %2, %3, p;\n\t}" ::"r"(d_tmem),
      "l"(a_desc), "l"(b_desc), "r"(idesc), "r"(accumulate)
      : "memory");
}

__device__ __forceinline__ uint32_t mix32(uint32_t x) {
  x ^= x >> 16;
  x *= 0x7feb352du;
  x ^= x >> 15;
  x *= 0x846ca68bu;
  x ^= x >> 16;
  return x;
}

// A random operand word: any bytes for int8; for fp16, two values with a random sign and
// mantissa and an exponent in [2^-2, 2^1]; for e4m3, four values with exponents below the
// NaN encoding (S.1111.111 never occurs).
template <int KIND>
__device__ __forceinline__ uint32_t operand_word(uint32_t h) {
  if constexpr (KIND == SM100_PEAK_I8) {
    return h;
  } else if constexpr (KIND == SM100_PEAK_F16) {
    // fp16: sign bit 15, exponent bits 10-14 (bias 15), mantissa 0-9; exponents 13..16
    const uint32_t lo = (h & 0x83FFu) | ((13u + ((h >> 10) & 3u)) << 10);
    const uint32_t hi = ((h >> 16) & 0x83FFu) | ((13u + ((h >> 26) & 3u)) << 10);
    return lo | (hi << 16);
  } else {
    return h & 0xF7F7F7F7u;  // e4m3 exponent field at most 0b1110: finite, never NaN
  }
}

template <int KIND>
__host__ __device__ constexpr uint32_t idesc_for(int n) {
  return KIND == SM100_PEAK_I8    ? make_idesc(kFmtD_S32, kFmtS8, kFmtS8, 0, 0, 128, static_cast<uint32_t>(n))
         : KIND == SM100_PEAK_F16 ? make_idesc(kFmtD_F32, kFmtF16, kFmtF16, 0, 0, 128, static_cast<uint32_t>(n))
                                  : make_idesc(kFmtD_F32, kFmtE4M3, kFmtE4M3, 0, 0, 128, static_cast<uint32_t>(n));
}

constexpr int kThreads = 128;
constexpr int kATile = 128 * 128;  // bytes
// more than half of the SM's 228 KB: one CTA per SM, so each CTA owns all 512 TMEM columns
constexpr int kSmemBytes = 120 * 1024;

template <int KIND, int N>
__global__ void __launch_bounds__(kThreads, 1)
    tensor_peak_kernel(long long mma_per_cta, uint32_t seed, unsigned long long limit_ns, int* status,
                       long long* timing) {
  static_assert(N % 16 == 0 && N >= 64 && N <= 256, "M = 128 takes N in [16, 256], multiple of 16");
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* a = smem;
  uint8_t* b = smem + kATile;
  uint64_t* bar = reinterpret_cast<uint64_t*>(b + N * 128);
  uint32_t* tslot = reinterpret_cast<uint32_t*>(bar + 1);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tslot + 1);

  uint32_t* words = reinterpret_cast<uint32_t*>(smem);
  const uint32_t base = mix32(seed ^ (blockIdx.x * 0x9E3779B9u));
  for (int i = threadIdx.x; i < (kATile + N * 128) / 4; i += kThreads) words[i] = operand_word<KIND>(mix32(base + i));
  fence_proxy_async_smem();  // operands written by threads, read by the tensor core
  if (threadIdx.x == 0) {
    mbar_init(bar, 1);
    *abort_flag = 0;
    fence_barrier_init();
  }
  if (warp_id() == 0) {
    tmem_alloc(tslot, 512);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tbase = *tslot;

  if (warp_id() == 0) {
    if (elect_one()) {
      constexpr uint32_t idesc = idesc_for<KIND>(N);
      const uint64_t ad = make_smem_desc(smem_u32(a), 16, 1024, kLayoutSW128);
      const uint64_t bd = make_smem_desc(smem_u32(b), 16, 1024, kLayoutSW128);
      const long long c0 = clock64();
      const uint64_t t0 = globaltimer_ns();
      for (long long it = 0; it < mma_per_cta; it += 4) {
        const uint32_t acc = tbase + static_cast<uint32_t>((it >> 2) & 1) * 256u;
#pragma unroll
        for (int kk = 0; kk < 4; ++kk) {
          const uint32_t accumulate = (it >= 8 || kk > 0) ? 1u : 0u;  // each accumulator starts at 0
          const uint64_t adk = desc_advance(ad, 32 * kk), bdk = desc_advance(bd, 32 * kk);
          if constexpr (KIND == SM100_PEAK_I8)
            umma_i8_ss(acc, adk, bdk, idesc, accumulate);
          else if constexpr (KIND == SM100_PEAK_F16)
            umma_f16_ss(acc, adk, bdk, idesc, accumulate);
          else
            umma_f8_ss(acc, adk, bdk, idesc, accumulate);
        }
      }
      umma_commit(bar);
      if (!mbar_wait(bar, 0, abort_flag, 1, limit_ns)) {
        atomicOr(status, 1);
        // once more, with the same limit, for the MMAs still in flight before TMEM is freed
        *abort_flag = 0;
        if (!mbar_wait(bar, 0, abort_flag, 1, limit_ns)) atomicOr(status, 2);
      }
      // SM cycles and wall time from the first MMA issued to the last one completed
      if (timing) {
        timing[2 * blockIdx.x] = clock64() - c0;
        timing[2 * blockIdx.x + 1] = static_cast<long long>(globaltimer_ns() - t0);
      }
    }
    __syncwarp();
  }
  tc_fence_before();
  __syncthreads();
  if (warp_id() == 0) {
    tc_fence_after();
    tmem_dealloc(tbase, 512);
  }
}

template <int KIND, int N>
int launch(int ctas, long long mma_per_cta, unsigned seed, unsigned long long limit_ns, int* status,
           long long* timing, cudaStream_t st) {
  auto kern = tensor_peak_kernel<KIND, N>;
  cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, kSmemBytes);
  if (e != cudaSuccess) {
    g_err = std::string("cudaFuncSetAttribute failed: ") + cudaGetErrorString(e);
    return SM100_PEAK_ERR_CUDA;
  }
  kern<<<ctas, kThreads, kSmemBytes, st>>>(mma_per_cta, seed, limit_ns, status, timing);
  e = cudaGetLastError();
  if (e != cudaSuccess) {
    g_err = std::string("launch failed: ") + cudaGetErrorString(e);
    return SM100_PEAK_ERR_CUDA;
  }
  return SM100_PEAK_OK;
}

template <int KIND>
int launch_n(int n, int ctas, long long mma_per_cta, unsigned seed, unsigned long long limit_ns, int* status,
             long long* timing, cudaStream_t st) {
  switch (n) {
    case 64: return launch<KIND, 64>(ctas, mma_per_cta, seed, limit_ns, status, timing, st);
    case 128: return launch<KIND, 128>(ctas, mma_per_cta, seed, limit_ns, status, timing, st);
    case 256: return launch<KIND, 256>(ctas, mma_per_cta, seed, limit_ns, status, timing, st);
    default: break;
  }
  g_err = "n must be 64, 128 or 256";
  return SM100_PEAK_ERR_INVALID_ARG;
}

}  // namespace

extern "C" {

const char* sm100_peak_last_error(void) { return g_err.c_str(); }

double sm100_peak_ops_per_mma(int kind, int n) {
  if (kind != SM100_PEAK_I8 && kind != SM100_PEAK_F16 && kind != SM100_PEAK_E4M3) return 0.0;
  if (n != 64 && n != 128 && n != 256) return 0.0;
  const double k = kind == SM100_PEAK_F16 ? 16.0 : 32.0;
  return 2.0 * 128.0 * n * k;
}

int sm100_tensor_peak_launch(int kind, int n, int ctas, long long mma_per_cta, unsigned seed,
                             unsigned limit_ms, int* status, long long* timing, void* stream) {
  g_err.clear();
  if (ctas <= 0 || ctas > 4096 || mma_per_cta <= 0 || (mma_per_cta % 4) != 0 || !status || limit_ms == 0) {
    g_err = "ctas in [1, 4096], mma_per_cta a positive multiple of 4, status non-NULL and limit_ms > 0 required";
    return SM100_PEAK_ERR_INVALID_ARG;
  }
  int dev = 0, major = 0, minor = 0;
  if (cudaGetDevice(&dev) != cudaSuccess ||
      cudaDeviceGetAttribute(&major, cudaDevAttrComputeCapabilityMajor, dev) != cudaSuccess ||
      cudaDeviceGetAttribute(&minor, cudaDevAttrComputeCapabilityMinor, dev) != cudaSuccess) {
    g_err = "no CUDA device";
    return SM100_PEAK_ERR_CUDA;
  }
  if (major != 10 || minor != 0) {
    g_err = "the tcgen05 microbenchmark needs sm_100";
    return SM100_PEAK_ERR_CUDA;
  }
  const unsigned long long limit_ns = static_cast<unsigned long long>(limit_ms) * 1000000ull;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  switch (kind) {
    case SM100_PEAK_I8: return launch_n<SM100_PEAK_I8>(n, ctas, mma_per_cta, seed, limit_ns, status, timing, st);
    case SM100_PEAK_F16: return launch_n<SM100_PEAK_F16>(n, ctas, mma_per_cta, seed, limit_ns, status, timing, st);
    case SM100_PEAK_E4M3: return launch_n<SM100_PEAK_E4M3>(n, ctas, mma_per_cta, seed, limit_ns, status, timing, st);
    default: break;
  }
  g_err = "kind must be SM100_PEAK_I8, SM100_PEAK_F16 or SM100_PEAK_E4M3";
  return SM100_PEAK_ERR_INVALID_ARG;
}

}  // extern "C"
