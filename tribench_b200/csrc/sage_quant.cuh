// sage_quant.cuh — the pre-pass of the sage path: K smoothing statistics, V absmax
// statistics, and the per-block INT8 quantisation of Q and K (plus FP8 e4m3 V).
//
// Quantisation scheme (restates quant_per_block_int8_kernel,
// kernels/sage_attn/triton_impl.py:7-33, bit for bit):
//   x     = fp32(in) * mult                 (mult = fp32(sm_scale*1.44269504) for Q, 1 for K)
//   scale = max_{block} |x| / 127.0f        (IEEE division, whole [BLK, D] block)
//   y     = x / scale                       (IEEE division, never reciprocal-multiply)
//   y    += (y >= 0 ? 0.5f : -0.5f)         (fp32 add)
//   q     = trunc(y) as int8                (NaN -> 0, so an all-zero block gives 0s and scale 0)
// Blocks are 128 rows for Q and 64 rows for K (triton_impl.py:166-173); rows past the
// sequence end read as zero and are not stored (triton_impl.py:25, 32).
//
// Smoothing (SageAttention's K mean subtraction; the reference accepts `km` at
// triton_impl.py:39-40 but never passes it): km[d] = fp32(sum_s fp64(k[s,d]) / S), with the
// fp64 sum taken in a fixed order (per chunk: row r + i*RPP accumulated per thread in
// increasing i, thread partials summed in increasing r, chunks summed in increasing
// order) so that a host restatement reproduces it bit for bit. K is then quantised from
// fp32(k) - km[d], matching per_block_int8(q, k, km=<fp32 km>) of the reference.
#pragma once

#include "sm100_ptx.cuh"

namespace sage {

constexpr int kQuantThreads = 256;
constexpr int kStatsChunk = 512;  // rows of K/V per statistics CTA

template <typename T> struct Vec8;
template <> struct Vec8<__half> {
  __device__ static __forceinline__ void to_float(const uint4& u, float (&f)[8]) {
    const __half2* h = reinterpret_cast<const __half2*>(&u);
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      float2 t = __half22float2(h[i]);
      f[2 * i] = t.x;
      f[2 * i + 1] = t.y;
    }
  }
};
template <> struct Vec8<__nv_bfloat16> {
  __device__ static __forceinline__ void to_float(const uint4& u, float (&f)[8]) {
    const __nv_bfloat162* h = reinterpret_cast<const __nv_bfloat162*>(&u);
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      float2 t = __bfloat1622float2(h[i]);
      f[2 * i] = t.x;
      f[2 * i + 1] = t.y;
    }
  }
};

__device__ __forceinline__ uint4 ldg_nc_v4(const void* p) {
  uint4 r;
  asm volatile("ld.global.nc.L1::no_allocate.v4.u32 {%0,%1,%2,%3}, [%4];"
               : "=r"(r.x), "=r"(r.y), "=r"(r.z), "=r"(r.w)
               : "l"(p));
  return r;
}

__device__ __forceinline__ float block_absmax(float v, float* red) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
  const int w = threadIdx.x >> 5;
  if ((threadIdx.x & 31) == 0) red[w] = v;
  __syncthreads();
  float m = red[0];
#pragma unroll
  for (int i = 1; i < kQuantThreads / 32; ++i) m = fmaxf(m, red[i]);
  return m;
}

__device__ __forceinline__ int8_t quant_one(float x, float scale) {
  float y = __fdiv_rn(x, scale);
  y = __fadd_rn(y, (y >= 0.0f) ? 0.5f : -0.5f);
  return static_cast<int8_t>(__float2int_rz(y));
}

struct StatsParams {
  const void* k;  // nullptr when not smoothing
  const void* v;  // nullptr when V is not quantised to FP8
  int64_t k_sb, k_sh, k_ss, v_sb, v_sh, v_ss;
  double* ksum_part;   // [B, Hkv, nchunk, D]
  float* vmax_part;    // [B, Hkv, nchunk, D]
  int Hkv, S, nchunk;
};

// Grid (nchunk, Hkv, B). Per chunk of kStatsChunk rows: fp64 column sums of K and fp32
// column absmax of V.
template <int D, typename T>
__global__ void __launch_bounds__(kQuantThreads) kv_stats_kernel(StatsParams p) {
  constexpr int TPR = D / 8;                 // threads per row (8 channels each)
  constexpr int RPP = kQuantThreads / TPR;   // rows per pass
  __shared__ double sum_red[RPP][D];
  __shared__ float max_red[RPP][D];
  const int c = blockIdx.x, h = blockIdx.y, b = blockIdx.z;
  const int g = threadIdx.x % TPR, r = threadIdx.x / TPR;
  const int row0 = c * kStatsChunk;
  const int row1 = min(p.S, row0 + kStatsChunk);
  double acc[8];
  float amax[8];
#pragma unroll
  for (int i = 0; i < 8; ++i) { acc[i] = 0.0; amax[i] = 0.0f; }
  const char* kb = p.k ? reinterpret_cast<const char*>(p.k) +
                             (b * p.k_sb + h * p.k_sh) * (int64_t)sizeof(T) + g * 16
                       : nullptr;
  const char* vb = p.v ? reinterpret_cast<const char*>(p.v) +
                             (b * p.v_sb + h * p.v_sh) * (int64_t)sizeof(T) + g * 16
                       : nullptr;
  for (int row = row0 + r; row < row1; row += RPP) {
    if (kb) {
      float f[8];
      Vec8<T>::to_float(ldg_nc_v4(kb + row * p.k_ss * (int64_t)sizeof(T)), f);
#pragma unroll
      for (int i = 0; i < 8; ++i) acc[i] = __dadd_rn(acc[i], static_cast<double>(f[i]));
    }
    if (vb) {
      float f[8];
      Vec8<T>::to_float(ldg_nc_v4(vb + row * p.v_ss * (int64_t)sizeof(T)), f);
#pragma unroll
      for (int i = 0; i < 8; ++i) amax[i] = fmaxf(amax[i], fabsf(f[i]));
    }
  }
#pragma unroll
  for (int i = 0; i < 8; ++i) {
    sum_red[r][g * 8 + i] = acc[i];
    max_red[r][g * 8 + i] = amax[i];
  }
  __syncthreads();
  if (threadIdx.x < D) {
    const int d = threadIdx.x;
    const size_t o = (((size_t)b * p.Hkv + h) * p.nchunk + c) * D + d;
    if (p.k) {
      double s = 0.0;
      for (int i = 0; i < RPP; ++i) s = __dadd_rn(s, sum_red[i][d]);
      p.ksum_part[o] = s;
    }
    if (p.v) {
      float m = 0.0f;
      for (int i = 0; i < RPP; ++i) m = fmaxf(m, max_red[i][d]);
      p.vmax_part[o] = m;
    }
  }
}

struct FinalizeParams {
  const double* ksum_part;  // nullable
  const float* vmax_part;   // nullable
  float* k_mean;            // [B, Hkv, D]
  float* v_scale;           // [B, Hkv, D]
  int Hkv, S, nchunk, D;
};

// Grid (Hkv, B), D threads: km = fp32(sum / S), v_scale = absmax / 448.
__global__ void kv_finalize_kernel(FinalizeParams p) {
  const int h = blockIdx.x, b = blockIdx.y, d = threadIdx.x;
  if (d >= p.D) return;
  const size_t head = (size_t)b * p.Hkv + h;
  if (p.ksum_part) {
    double s = 0.0;
    for (int c = 0; c < p.nchunk; ++c) s = __dadd_rn(s, p.ksum_part[(head * p.nchunk + c) * p.D + d]);
    p.k_mean[head * p.D + d] = __double2float_rn(__ddiv_rn(s, static_cast<double>(p.S)));
  }
  if (p.vmax_part) {
    float m = 0.0f;
    for (int c = 0; c < p.nchunk; ++c) m = fmaxf(m, p.vmax_part[(head * p.nchunk + c) * p.D + d]);
    p.v_scale[head * p.D + d] = __fdiv_rn(m, 448.0f);
  }
}

struct QuantParams {
  const void* q;
  const void* k;
  const void* v;  // FP8 V quantisation (nullable)
  int64_t q_sb, q_sh, q_ss, k_sb, k_sh, k_ss, v_sb, v_sh, v_ss;
  int8_t* q_i8;
  float* q_scale;
  int8_t* k_i8;
  float* k_scale;
  const float* k_mean;  // nullable: smoothing off
  uint8_t* v_fp8;
  const float* v_scale;
  float q_mult;
  int B, Hq, Hkv, Sq, Skv;
  int nqb, nkb, nvb;        // blocks per head
  int n_q_ctas, n_k_ctas;   // CTA ranges: [0,nq) Q, [nq,nq+nk) K, rest V
};

// One CTA per quantisation block. Blocks of Q come first in the grid, then K, then V.
template <int D, typename T>
__global__ void __launch_bounds__(kQuantThreads) quant_kernel(QuantParams p) {
  constexpr int TPR = D / 8;
  constexpr int RPP = kQuantThreads / TPR;
  __shared__ float red[kQuantThreads / 32];
  const int g = threadIdx.x % TPR, r = threadIdx.x / TPR;
  int cta = blockIdx.x;

  if (cta < p.n_q_ctas || cta < p.n_q_ctas + p.n_k_ctas) {
    const bool isq = cta < p.n_q_ctas;
    if (!isq) cta -= p.n_q_ctas;
    const int BLK = isq ? 128 : 64;
    const int nb = isq ? p.nqb : p.nkb;
    const int H = isq ? p.Hq : p.Hkv;
    const int S = isq ? p.Sq : p.Skv;
    const int blk = cta % nb;
    const int hh = (cta / nb) % H;
    const int bb = cta / (nb * H);
    const char* src = reinterpret_cast<const char*>(isq ? p.q : p.k) +
                      (bb * (isq ? p.q_sb : p.k_sb) + hh * (isq ? p.q_sh : p.k_sh)) *
                          (int64_t)sizeof(T) +
                      g * 16;
    const int64_t ss = (isq ? p.q_ss : p.k_ss) * (int64_t)sizeof(T);
    const float mult = isq ? p.q_mult : 1.0f;
    float km[8];
#pragma unroll
    for (int i = 0; i < 8; ++i) km[i] = 0.0f;
    const bool smooth = !isq && p.k_mean != nullptr;
    if (smooth) {
      const float* kmp = p.k_mean + ((size_t)bb * p.Hkv + hh) * D + g * 8;
#pragma unroll
      for (int i = 0; i < 8; ++i) km[i] = kmp[i];
    }
    constexpr int MAXP = 128 / RPP;  // passes for a 128-row block
    float x[MAXP][8];
    float amax = 0.0f;
    const int row0 = blk * BLK;
    const int npass = BLK / RPP;
#pragma unroll
    for (int i = 0; i < MAXP; ++i) {
      const int row = row0 + r + i * RPP;
      if (i < npass && row < S) {
        float f[8];
        Vec8<T>::to_float(ldg_nc_v4(src + row * ss), f);
#pragma unroll
        for (int e = 0; e < 8; ++e) {
          float t = smooth ? __fsub_rn(f[e], km[e]) : f[e];
          t = isq ? __fmul_rn(t, mult) : t;
          x[i][e] = t;
          amax = fmaxf(amax, fabsf(t));
        }
      } else {
#pragma unroll
        for (int e = 0; e < 8; ++e) x[i][e] = 0.0f;
      }
    }
    const float m = block_absmax(amax, red);
    const float scale = __fdiv_rn(m, 127.0f);
    const size_t head = (size_t)bb * H + hh;
    if (threadIdx.x == 0) (isq ? p.q_scale : p.k_scale)[head * nb + blk] = scale;
    int8_t* dst = (isq ? p.q_i8 : p.k_i8) + head * (size_t)S * D + g * 8;
#pragma unroll
    for (int i = 0; i < MAXP; ++i) {
      const int row = row0 + r + i * RPP;
      if (i < npass && row < S) {
        uint32_t w[2] = {0u, 0u};
#pragma unroll
        for (int e = 0; e < 8; ++e)
          w[e >> 2] |= (static_cast<uint32_t>(static_cast<uint8_t>(quant_one(x[i][e], scale))))
                       << (8 * (e & 3));
        *reinterpret_cast<uint2*>(dst + (size_t)row * D) = make_uint2(w[0], w[1]);
      }
    }
    return;
  }

  // ---- V -> FP8 e4m3 with per-channel scales (64-row blocks).
  cta -= p.n_q_ctas + p.n_k_ctas;
  const int blk = cta % p.nvb;
  const int hh = (cta / p.nvb) % p.Hkv;
  const int bb = cta / (p.nvb * p.Hkv);
  const size_t head = (size_t)bb * p.Hkv + hh;
  const char* src = reinterpret_cast<const char*>(p.v) +
                    (bb * p.v_sb + hh * p.v_sh) * (int64_t)sizeof(T) + g * 16;
  float vs[8];
#pragma unroll
  for (int e = 0; e < 8; ++e) vs[e] = p.v_scale[head * D + g * 8 + e];
  uint8_t* dst = p.v_fp8 + head * (size_t)p.Skv * D + g * 8;
  for (int row = blk * 64 + r; row < min(p.Skv, blk * 64 + 64); row += RPP) {
    float f[8];
    Vec8<T>::to_float(ldg_nc_v4(src + row * p.v_ss * (int64_t)sizeof(T)), f);
    uint32_t w[2] = {0u, 0u};
#pragma unroll
    for (int e = 0; e < 8; e += 2) {
      const float a = vs[e] > 0.0f ? __fdiv_rn(f[e], vs[e]) : 0.0f;
      const float c = vs[e + 1] > 0.0f ? __fdiv_rn(f[e + 1], vs[e + 1]) : 0.0f;
      const __nv_fp8x2_storage_t pr =
          __nv_cvt_float2_to_fp8x2(make_float2(a, c), __NV_SATFINITE, __NV_E4M3);
      w[e >> 2] |= static_cast<uint32_t>(pr) << (8 * (e & 3));
    }
    *reinterpret_cast<uint2*>(dst + (size_t)row * D) = make_uint2(w[0], w[1]);
  }
}

}  // namespace sage
