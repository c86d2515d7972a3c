// sage_quant.cuh — the pre-pass of the sage path: K smoothing statistics, V absmax
// statistics, and the per-block INT8 quantisation of Q and K (plus FP8 e4m3 V).
//
// Quantisation scheme (restates quant_per_block_int8_kernel,
// kernels/sage_attn/triton_impl.py:7-33, bit for bit):
//   x     = fp32(in) * mult                 (mult = fp32(sm_scale*1.44269504) for Q, 1 for K)
//   scale = max_{block} |x| / 127.0f        (IEEE division, whole [BLK, D] block)
//   y     = x / scale                       (correctly rounded quotient, see quotient_rn)
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
//
// Launches. Each launch runs a list of CTA roles (see PrepassParams):
//   A: Q quantisation + K/V statistics (+ K quantisation when K needs no statistics)
//   finalize: K mean / V scales from the statistics
//   B: K quantisation (smoothed) + V to e4m3
#pragma once

#include "sage_seq.cuh"
#include "sm100_ptx.cuh"

namespace sage {

constexpr int kQuantThreads = 256;
constexpr int kStatsChunk = 512;  // rows of K/V per statistics CTA
// Scale blocks per quantisation CTA: at D = 64 a block holds half the bytes, so a CTA takes
// several, keeping eight 16-byte loads per thread in flight as at D = 128.
template <int D> constexpr int kQBlocksPerCta = (D == 64) ? 2 : 1;
template <int D> constexpr int kKBlocksPerCta = (D == 64) ? 4 : 1;
// Rows of V per e4m3 CTA: eight passes of the CTA's threads (V needs no per-block reduction).
template <int D> constexpr int kVRowsPerCta = 8 * (kQuantThreads / (D / 8));

template <typename T> struct Half8;
template <> struct Half8<__half> {
  using H2 = __half2;
  __device__ static __forceinline__ void to_float(const uint4& u, float (&f)[8]) {
    const __half2* h = reinterpret_cast<const __half2*>(&u);
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      float2 t = __half22float2(h[i]);
      f[2 * i] = t.x;
      f[2 * i + 1] = t.y;
    }
  }
  // max |h| over the 8 halves, exact (comparisons of 16-bit values), as fp32
  __device__ static __forceinline__ float absmax(const uint4& u) {
    const __half2* h = reinterpret_cast<const __half2*>(&u);
    __half2 m = __hmax2(__hmax2(__habs2(h[0]), __habs2(h[1])), __hmax2(__habs2(h[2]), __habs2(h[3])));
    return fmaxf(__low2float(m), __high2float(m));
  }
};
template <> struct Half8<__nv_bfloat16> {
  using H2 = __nv_bfloat162;
  __device__ static __forceinline__ void to_float(const uint4& u, float (&f)[8]) {
    const __nv_bfloat162* h = reinterpret_cast<const __nv_bfloat162*>(&u);
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      float2 t = __bfloat1622float2(h[i]);
      f[2 * i] = t.x;
      f[2 * i + 1] = t.y;
    }
  }
  __device__ static __forceinline__ float absmax(const uint4& u) {
    const __nv_bfloat162* h = reinterpret_cast<const __nv_bfloat162*>(&u);
    __nv_bfloat162 m = __hmax2(__hmax2(__habs2(h[0]), __habs2(h[1])), __hmax2(__habs2(h[2]), __habs2(h[3])));
    return fmaxf(__low2float(m), __high2float(m));
  }
};

__device__ __forceinline__ uint4 ldg_nc_v4(const void* p) {
  uint4 r;
  asm volatile("ld.global.nc.L1::no_allocate.v4.u32 {%0,%1,%2,%3}, [%4];"
               : "=r"(r.x), "=r"(r.y), "=r"(r.z), "=r"(r.w)
               : "l"(p));
  return r;
}

// Block-wide maxima of N values per thread in one reduction round; red holds
// N * (kQuantThreads / 32) floats. Called once per CTA.
template <int N, int NT = kQuantThreads>
__device__ __forceinline__ void block_max_n(float (&v)[N], float* red) {
  constexpr int W = NT / 32;
#pragma unroll
  for (int n = 0; n < N; ++n)
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v[n] = fmaxf(v[n], __shfl_xor_sync(0xffffffffu, v[n], o));
  if ((threadIdx.x & 31) == 0)
#pragma unroll
    for (int n = 0; n < N; ++n) red[n * W + (threadIdx.x >> 5)] = v[n];
  __syncthreads();
#pragma unroll
  for (int n = 0; n < N; ++n) {
    float m = red[n * W];
#pragma unroll
    for (int i = 1; i < W; ++i) m = fmaxf(m, red[n * W + i]);
    v[n] = m;
  }
}

// Correctly rounded x / s from r = RN(1/s): q0 = RN(x*r) is within a couple of ulps, the
// residual x - s*q0 is exact in one FMA, and one more FMA q0 + residual*r rounds to the
// IEEE quotient (Markstein's final-correction step, IBM J. Res. Dev. 34(1), 1990). Used with
// |x| <= 127*s; s = 0 gives NaN like the IEEE division it replaces.
__device__ __forceinline__ float quotient_rn(float x, float s, float r) {
  const float q0 = __fmul_rn(x, r);
  const float e = __fmaf_rn(-s, q0, x);
  return __fmaf_rn(e, r, q0);
}

// Two INT8 codes as 32-bit integers (only their low bytes are used), with packed f32x2
// arithmetic (each lane an IEEE operation): y = x / s via Markstein's correction, then
// y + copysign(0.5, y) — the reference's y + (y >= 0 ? 0.5 : -0.5) for every y, -0.0 and NaN
// included (both truncate to 0) — then truncation.
__device__ __forceinline__ void quant_two(float2 x, float2 s, float2 ns, float2 r, int& a, int& b) {
  const float2 q0 = fmul2(x, r);
  const float2 e = ffma2(ns, q0, x);
  const float2 y = ffma2(e, r, q0);
  const float2 z = fadd2(y, make_float2(copysignf(0.5f, y.x), copysignf(0.5f, y.y)));
  a = __float2int_rz(z.x);
  b = __float2int_rz(z.y);
}

// Two INT8 codes (as integers in [-127, 127]) as an fp16 pair: c + 25728 is the bit pattern of
// the fp16 value c + 1152 (exponent 10: ulp 1 in [1024, 2048)), and subtracting 1152 is exact.
__device__ __forceinline__ uint32_t codes_to_half2(int a, int b) {
  const uint32_t bits = __byte_perm(static_cast<uint32_t>(a + 25728), static_cast<uint32_t>(b + 25728), 0x5410);
  const __half2 h = __hsub2(*reinterpret_cast<const __half2*>(&bits), __float2half2_rn(1152.0f));
  return *reinterpret_cast<const uint32_t*>(&h);
}

// Low bytes of four integers packed little-endian into one word (three byte permutes).
__device__ __forceinline__ uint32_t pack4_lo_bytes(int a, int b, int c, int d) {
  const uint32_t ab = __byte_perm(static_cast<uint32_t>(a), static_cast<uint32_t>(b), 0x0040);
  const uint32_t cd = __byte_perm(static_cast<uint32_t>(c), static_cast<uint32_t>(d), 0x0040);
  return __byte_perm(ab, cd, 0x5410);
}

struct PrepassParams {
  const void* q;
  const void* k;
  const void* v;
  int64_t q_sb, q_sh, q_ss, k_sb, k_sh, k_ss, v_sb, v_sh, v_ss;
  int8_t* q_i8;
  float* q_scale;
  int8_t* k_i8;
  float* k_scale;
  const float* k_mean;  // K quantisation: subtract this channel mean (nullable: no smoothing)
  uint8_t* v_fp8;
  const float* v_scale;
  double* ksum_part;    // statistics: [B, Hkv, nchunk, D]
  float* vmax_part;     // statistics: [B, Hkv, nchunk, D]
  float q_mult;
  int B, Hq, Hkv, Sq, Skv;  // variable-length batches: Sq / Skv = longest sequence
  int nqb, nkb, nvb, nchunk;
  int qblk;                 // rows per Q scale block: 128 (quant_block_role), or 1/16/32/64 (qquant_fine_kernel)
  // Variable-length batches (nullable): sequence b owns token rows [cu_q[b], cu_q[b+1]) of Q and
  // [cu_k[b], cu_k[b+1]) of K/V (batch extent 1, q_tokens / k_tokens rows); the int8 / e4m3
  // outputs are [H, tokens, D], the scales and statistics stay per sequence.
  const int* cu_q;
  const int* cu_k;
  int q_tokens, k_tokens;
  // fp16 codes (C16 instantiations): the same INT8 codes as fp16 values, for the attention
  // kernel's kind::f16 QK^T. Q's go to q_c16 with element strides qc_sb/qc_sh/qc_ss (batch,
  // head, token), K's to k_c16 in k_i8's layout.
  __half* q_c16;
  int64_t qc_sb, qc_sh, qc_ss;
  __half* k_c16;
  // CTA roles of this launch, in grid order: Q blocks, statistics chunks, K blocks, V blocks
  int n_q, n_stat, n_k, n_v;
  int stat_k, stat_v;   // which statistics the statistics CTAs gather
};

// ---------------------------------------------------------------- roles
// NSUB consecutive scale blocks of BLK rows, all rows loaded up front, by a CTA of NT threads.
template <int D, typename T, int BLK, int NSUB, bool PACKED, bool C16, int NT = kQuantThreads>
__device__ __forceinline__ void quant_block_role(const PrepassParams& p, int cta, bool isq, float* red) {
  constexpr int TPR = D / 8;                 // threads per row (8 channels each)
  constexpr int RPP = NT / TPR;              // rows per pass
  constexpr int PPB = BLK / RPP;             // passes per scale block
  constexpr int NP = NSUB * PPB;             // passes
  const int g = threadIdx.x % TPR, r = threadIdx.x / TPR;
  const int nb = isq ? p.nqb : p.nkb;
  const int ng = (nb + NSUB - 1) / NSUB;     // CTAs per head
  const int H = isq ? p.Hq : p.Hkv;
  const int grp = cta % ng;
  const int hh = (cta / ng) % H;
  const int bb = cta / (ng * H);
  const SeqSpan sp = isq ? seq_span(PACKED ? p.cu_q : nullptr, bb, p.Sq, p.q_tokens)
                          : seq_span(PACKED ? p.cu_k : nullptr, bb, p.Skv, p.k_tokens);
  const int S = sp.len;
  const int row0 = grp * NSUB * BLK;
  if (row0 >= S) return;  // a block past the end of a shorter sequence (uniform over the CTA)
  const int64_t ss_elts = isq ? p.q_ss : p.k_ss;
  const char* src = reinterpret_cast<const char*>(isq ? p.q : p.k) +
                    (sp.batch * (isq ? p.q_sb : p.k_sb) + hh * (isq ? p.q_sh : p.k_sh) + sp.base * ss_elts) *
                        (int64_t)sizeof(T) + g * 16;
  const int64_t ss = ss_elts * (int64_t)sizeof(T);
  const bool smooth = !isq && p.k_mean != nullptr;
  float km[8];
#pragma unroll
  for (int i = 0; i < 8; ++i) km[i] = 0.0f;
  if (smooth) {
    const float* kmp = p.k_mean + ((size_t)bb * p.Hkv + hh) * D + g * 8;
#pragma unroll
    for (int i = 0; i < 8; ++i) km[i] = kmp[i];
  }
  uint4 raw[NP];
#pragma unroll
  for (int i = 0; i < NP; ++i) {
    const int row = row0 + r + i * RPP;
    raw[i] = (row < S) ? ldg_nc_v4(src + row * ss) : make_uint4(0u, 0u, 0u, 0u);
  }
  float amax[NSUB];
#pragma unroll
  for (int b = 0; b < NSUB; ++b) amax[b] = 0.0f;
  if (smooth) {
#pragma unroll
    for (int i = 0; i < NP; ++i) {
      float f[8];
      Half8<T>::to_float(raw[i], f);
      const bool in = row0 + r + i * RPP < S;
      if (in) {
#pragma unroll
        for (int e = 0; e < 8; e += 2) {
          const float2 x = fsub2(make_float2(f[e], f[e + 1]), make_float2(km[e], km[e + 1]));
          amax[i / PPB] = fmax3(amax[i / PPB], fabsf(x.x), fabsf(x.y));
        }
      }
    }
  } else {
    // max |in| on the raw 16-bit values; RN(|in| * mult) is monotone in |in|, so this gives
    // max |x| exactly after one multiplication
#pragma unroll
    for (int i = 0; i < NP; ++i) amax[i / PPB] = fmaxf(amax[i / PPB], Half8<T>::absmax(raw[i]));
  }
  block_max_n<NSUB, NT>(amax, red);
  float scale[NSUB], rcp[NSUB];
#pragma unroll
  for (int b = 0; b < NSUB; ++b) {
    const float m = isq ? __fmul_rn(amax[b], p.q_mult) : amax[b];
    scale[b] = __fdiv_rn(m, 127.0f);
    rcp[b] = __frcp_rn(scale[b]);
  }
  const float2 mult2 = make_float2(p.q_mult, p.q_mult);
  const size_t head = (size_t)bb * H + hh;
#pragma unroll
  for (int b = 0; b < NSUB; ++b)
    if (threadIdx.x == b && grp * NSUB + b < nb) (isq ? p.q_scale : p.k_scale)[head * nb + grp * NSUB + b] = scale[b];
  const size_t first_row = PACKED ? (size_t)hh * (isq ? p.q_tokens : p.k_tokens) + sp.base : head * (size_t)S;
  int8_t* dst = (isq ? p.q_i8 : p.k_i8) + first_row * D + g * 8;
  // C16: Q codes at q_c16 (its own strides), K codes at k_c16 (k_i8's layout, 2 bytes each)
  __half* dst16 = nullptr;
  int64_t ss16 = D;
  if constexpr (C16) {
    if (isq) {
      dst16 = p.q_c16 + (int64_t)sp.batch * p.qc_sb + (int64_t)hh * p.qc_sh + (int64_t)sp.base * p.qc_ss + g * 8;
      ss16 = p.qc_ss;
    } else {
      dst16 = p.k_c16 + first_row * D + g * 8;
    }
  }
#pragma unroll
  for (int i = 0; i < NP; ++i) {
    const int row = row0 + r + i * RPP;
    const float sc = scale[i / PPB], rc = rcp[i / PPB];
    const float2 s2 = make_float2(sc, sc), ns2 = make_float2(-sc, -sc), r2 = make_float2(rc, rc);
    if (row < S) {
      float f[8];
      Half8<T>::to_float(raw[i], f);
      int qv[8];
#pragma unroll
      for (int e = 0; e < 8; e += 2) {
        float2 x = make_float2(f[e], f[e + 1]);
        if (smooth) x = fsub2(x, make_float2(km[e], km[e + 1]));
        if (isq) x = fmul2(x, mult2);
        quant_two(x, s2, ns2, r2, qv[e], qv[e + 1]);
      }
      if constexpr (C16) {
        *reinterpret_cast<uint4*>(dst16 + (int64_t)row * ss16) =
            make_uint4(codes_to_half2(qv[0], qv[1]), codes_to_half2(qv[2], qv[3]), codes_to_half2(qv[4], qv[5]),
                       codes_to_half2(qv[6], qv[7]));
      } else {
        *reinterpret_cast<uint2*>(dst + (size_t)row * D) =
            make_uint2(pack4_lo_bytes(qv[0], qv[1], qv[2], qv[3]), pack4_lo_bytes(qv[4], qv[5], qv[6], qv[7]));
      }
    }
  }
}

// Statistics over one chunk of kStatsChunk rows: fp64 column sums of K, fp32 column absmax of V.
// U: rows in flight per thread. KONLY: the K column sums only (no V statistics).
template <int D, typename T, bool PACKED, int U = 4, bool KONLY = false>
__device__ __forceinline__ void stats_role(const PrepassParams& p, int cta, double (*sum_red)[D], float (*max_red)[D]) {
  constexpr int TPR = D / 8;
  constexpr int RPP = kQuantThreads / TPR;
  const int c = cta % p.nchunk;
  const int h = (cta / p.nchunk) % p.Hkv;
  const int b = cta / (p.nchunk * p.Hkv);
  const int g = threadIdx.x % TPR, r = threadIdx.x / TPR;
  const SeqSpan sp = seq_span(PACKED ? p.cu_k : nullptr, b, p.Skv, p.k_tokens);
  const int row0 = c * kStatsChunk;
  const int row1 = min(sp.len, row0 + kStatsChunk);  // chunks past the end contribute zeros
  double acc[8];
  float amax[8];
#pragma unroll
  for (int i = 0; i < 8; ++i) { acc[i] = 0.0; amax[i] = 0.0f; }
  const char* kb = p.stat_k ? reinterpret_cast<const char*>(p.k) +
                                  (sp.batch * p.k_sb + h * p.k_sh + sp.base * p.k_ss) * (int64_t)sizeof(T) + g * 16
                            : nullptr;
  const char* vb = (!KONLY && p.stat_v) ? reinterpret_cast<const char*>(p.v) +
                                  (sp.batch * p.v_sb + h * p.v_sh + sp.base * p.v_ss) * (int64_t)sizeof(T) + g * 16
                            : nullptr;
  for (int base = row0 + r; base < row1; base += U * RPP) {
    uint4 kr[U], vr[U];
#pragma unroll
    for (int u = 0; u < U; ++u) {
      const int row = base + u * RPP;
      const bool in = row < row1;
      kr[u] = (kb && in) ? ldg_nc_v4(kb + row * p.k_ss * (int64_t)sizeof(T)) : make_uint4(0u, 0u, 0u, 0u);
      vr[u] = (vb && in) ? ldg_nc_v4(vb + row * p.v_ss * (int64_t)sizeof(T)) : make_uint4(0u, 0u, 0u, 0u);
    }
#pragma unroll
    for (int u = 0; u < U; ++u) {
      if (base + u * RPP < row1) {  // rows in increasing order: the fixed summation order
        if (kb) {
          float f[8];
          Half8<T>::to_float(kr[u], f);
#pragma unroll
          for (int e = 0; e < 8; ++e) acc[e] = __dadd_rn(acc[e], static_cast<double>(f[e]));
        }
        if (vb) {
          float f[8];
          Half8<T>::to_float(vr[u], f);
#pragma unroll
          for (int e = 0; e < 8; ++e) amax[e] = fmaxf(amax[e], fabsf(f[e]));
        }
      }
    }
  }
#pragma unroll
  for (int e = 0; e < 8; ++e) {
    sum_red[r][g * 8 + e] = acc[e];
    max_red[r][g * 8 + e] = amax[e];
  }
  __syncthreads();
  if (threadIdx.x < D) {
    const int d = threadIdx.x;
    const size_t o = (((size_t)b * p.Hkv + h) * p.nchunk + c) * D + d;
    if (kb) {
      double s = 0.0;
      for (int i = 0; i < RPP; ++i) s = __dadd_rn(s, sum_red[i][d]);
      p.ksum_part[o] = s;
    }
    if (vb) {
      float mx = 0.0f;
      for (int i = 0; i < RPP; ++i) mx = fmaxf(mx, max_red[i][d]);
      p.vmax_part[o] = mx;
    }
  }
}

// V -> e4m3 with per-channel scales, kVRowsPerCta rows per CTA: v / v_scale (correctly rounded quotient),
// then cvt.rn.satfinite; a channel whose scale is 0 gives 0.
template <int D, typename T, bool PACKED>
__device__ __forceinline__ void vquant_role(const PrepassParams& p, int cta) {
  constexpr int TPR = D / 8;
  constexpr int RPP = kQuantThreads / TPR;
  const int g = threadIdx.x % TPR, r = threadIdx.x / TPR;
  const int blk = cta % p.nvb;
  const int hh = (cta / p.nvb) % p.Hkv;
  const int bb = cta / (p.nvb * p.Hkv);
  const size_t head = (size_t)bb * p.Hkv + hh;
  const SeqSpan sp = seq_span(PACKED ? p.cu_k : nullptr, bb, p.Skv, p.k_tokens);
  const int S = sp.len;
  if (blk * kVRowsPerCta<D> >= S) return;  // past the end of a shorter sequence (uniform)
  const char* src = reinterpret_cast<const char*>(p.v) +
                    (sp.batch * p.v_sb + hh * p.v_sh + sp.base * p.v_ss) * (int64_t)sizeof(T) + g * 16;
  float vs[8], rv[8];
#pragma unroll
  for (int e = 0; e < 8; ++e) {
    vs[e] = p.v_scale[head * D + g * 8 + e];
    rv[e] = __frcp_rn(vs[e]);
  }
  const size_t first_row = PACKED ? (size_t)hh * p.k_tokens + sp.base : head * (size_t)S;
  uint8_t* dst = p.v_fp8 + first_row * D + g * 8;
  constexpr int NP = kVRowsPerCta<D> / RPP;
  uint4 raw[NP];
#pragma unroll
  for (int i = 0; i < NP; ++i) {
    const int row = blk * kVRowsPerCta<D> + r + i * RPP;
    raw[i] = (row < S) ? ldg_nc_v4(src + row * p.v_ss * (int64_t)sizeof(T)) : make_uint4(0u, 0u, 0u, 0u);
  }
#pragma unroll
  for (int i = 0; i < NP; ++i) {
    const int row = blk * kVRowsPerCta<D> + r + i * RPP;
    if (row >= S) continue;
    float f[8];
    Half8<T>::to_float(raw[i], f);
    uint32_t w[2] = {0u, 0u};
#pragma unroll
    for (int e = 0; e < 8; e += 2) {
      const float a = vs[e] > 0.0f ? quotient_rn(f[e], vs[e], rv[e]) : 0.0f;
      const float c = vs[e + 1] > 0.0f ? quotient_rn(f[e + 1], vs[e + 1], rv[e + 1]) : 0.0f;
      const __nv_fp8x2_storage_t pr = __nv_cvt_float2_to_fp8x2(make_float2(a, c), __NV_SATFINITE, __NV_E4M3);
      w[e >> 2] |= static_cast<uint32_t>(pr) << (8 * (e & 3));
    }
    *reinterpret_cast<uint2*>(dst + (size_t)row * D) = make_uint2(w[0], w[1]);
  }
}

// One launch of the pre-pass: CTA roles in grid order Q blocks | statistics chunks | K blocks | V blocks.
// PACKED: variable-length batches (p.cu_q / p.cu_k set); a separate instantiation keeps the
// dense path's code and registers as they are without the sequence offsets. C16: codes stored as
// fp16 values (q_c16 / k_c16) instead of INT8 bytes.
template <int D, typename T, bool PACKED, bool C16 = false>
__global__ void __launch_bounds__(kQuantThreads) prepass_kernel(PrepassParams p) {
  constexpr int RPP = kQuantThreads / (D / 8);
  __shared__ double sum_red[RPP][D];
  __shared__ float max_red[RPP][D];
  __shared__ float red[4 * (kQuantThreads / 32)];
  int cta = blockIdx.x;
  if (cta < p.n_q) { quant_block_role<D, T, 128, kQBlocksPerCta<D>, PACKED, C16>(p, cta, true, red); return; }
  cta -= p.n_q;
  if (cta < p.n_stat) { stats_role<D, T, PACKED>(p, cta, sum_red, max_red); return; }
  cta -= p.n_stat;
  // K and V blocks run in reverse head order: the statistics CTAs of the previous launch read
  // the last heads most recently, so their rows are the ones still in L2
  if (cta < p.n_k) { quant_block_role<D, T, 64, kKBlocksPerCta<D>, PACKED, C16>(p, p.n_k - 1 - cta, false, red); return; }
  cta -= p.n_k;
  vquant_role<D, T, PACKED>(p, p.n_v - 1 - cta);
}

// K statistics alone (the launch before the K quantisation when Q is quantised in the attention
// kernel): eight rows per thread in flight instead of four, and at 64 registers four CTAs per SM
// instead of the combined kernel's three, so the launch streams K closer to the HBM rate
// (H8K step 1.78-1.80 -> 1.76 ms).
template <int D, typename T, bool PACKED>
__global__ void __launch_bounds__(kQuantThreads, 4) kstats_kernel(PrepassParams p) {
  constexpr int RPP = kQuantThreads / (D / 8);
  __shared__ double sum_red[RPP][D];
  __shared__ float max_red[RPP][D];
  stats_role<D, T, PACKED, 8, true>(p, blockIdx.x, sum_red, max_red);
}

// K quantisation alone (launch B when no V block needs e4m3 codes): CTAs of 128 threads, each
// thread with eight 16-byte rows in flight (one 64-row block at head_dim 128, two at 64), and at
// most 64 registers so that eight CTAs share an SM. The combined kernel's CTAs carry the 24 KB
// statistics buffers and 80 registers (three per SM, four rows in flight per thread); on the
// H8K shape this launch streams K at ~5.7 TB/s against ~3.2 TB/s there (pre-pass 97 -> 80 us,
// C3 191 -> 148 us, bit-identical codes).
constexpr int kKQuantThreads = 128;
template <int D> constexpr int kKQuantBlocks = (D == 64) ? 2 : 1;  // 64-row blocks per CTA
template <int D, typename T, bool PACKED, bool C16>
__global__ void __launch_bounds__(kKQuantThreads, 8) kquant_kernel(PrepassParams p) {
  __shared__ float red[kKQuantBlocks<D> * (kKQuantThreads / 32)];
  // reverse head order, as in the combined kernel: the statistics launch read the last heads last
  quant_block_role<D, T, 64, kKQuantBlocks<D>, PACKED, C16, kKQuantThreads>(p, p.n_k - 1 - (int)blockIdx.x, false,
                                                                           red);
}

// Q quantisation alone at head_dim 64 (the launch before the statistics): the same 128-thread
// shape, one 128-row block per CTA (eight 16-byte rows in flight per thread).
template <typename T, bool PACKED, bool C16>
__global__ void __launch_bounds__(kKQuantThreads, 8) qquant_kernel(PrepassParams p) {
  __shared__ float red[kKQuantThreads / 32];
  quant_block_role<64, T, 128, 1, PACKED, C16, kKQuantThreads>(p, (int)blockIdx.x, true, red);
}

// Q quantisation with finer scale blocks than the default 128 rows: p.qblk rows per scale (1 =
// one scale per token, or 16, 32, 64), as per_block_int8's BLKQ argument allows
// (triton_impl.py:35, 57, 63). 128 threads per CTA and 128 rows per CTA: thread t loads the
// 16-byte piece g = t % (D/8) of rows r + i * RPP (r = t / (D/8), i < NP). Block maxima:
//   * qblk = 1: each row's (D/8) threads are consecutive lanes of one warp, so the row's absmax
//     is a shuffle reduction over those lanes;
//   * qblk >= RPP (16, 32, 64 >= 8 or 16 rows per pass): each pass's absmax over the CTA, then
//     the maximum over the qblk / RPP passes of a block.
// Scale, quotient and rounding arithmetic as quant_block_role, so the codes are bit-identical to
// the reference's at that BLKQ. The default 128-row blocks keep quant_block_role.
template <int D, typename T, bool PACKED, bool C16>
__global__ void __launch_bounds__(128, (D == 128) ? 3 : 4) qquant_fine_kernel(PrepassParams p) {
  constexpr int NT = 128, TPR = D / 8, RPP = NT / TPR, NP = 128 / RPP;
  __shared__ float red[NP][NT / 32];
  __shared__ float pmax[NP];
  const int g = threadIdx.x % TPR, r = threadIdx.x / TPR;
  const int blk = p.qblk;
  const int nb = p.nqb;                      // scale blocks per (batch, head) = ceil(Sq / qblk)
  const int ng = (p.Sq + 127) / 128;         // CTAs per head
  const int cta = blockIdx.x;
  const int grp = cta % ng;
  const int hh = (cta / ng) % p.Hq;
  const int bb = cta / (ng * p.Hq);
  const SeqSpan sp = seq_span(PACKED ? p.cu_q : nullptr, bb, p.Sq, p.q_tokens);
  const int S = sp.len;
  const int row0 = grp * 128;
  if (row0 >= S) return;  // uniform over the CTA
  const char* src = reinterpret_cast<const char*>(p.q) +
                    (sp.batch * p.q_sb + hh * p.q_sh + sp.base * p.q_ss) * (int64_t)sizeof(T) + g * 16;
  const int64_t ss = p.q_ss * (int64_t)sizeof(T);
  uint4 raw[NP];
#pragma unroll
  for (int i = 0; i < NP; ++i) {
    const int row = row0 + r + i * RPP;
    raw[i] = (row < S) ? ldg_nc_v4(src + row * ss) : make_uint4(0u, 0u, 0u, 0u);
  }
  float m[NP];
#pragma unroll
  for (int i = 0; i < NP; ++i) m[i] = Half8<T>::absmax(raw[i]);
  if (blk == 1) {
#pragma unroll
    for (int i = 0; i < NP; ++i)
#pragma unroll
      for (int o = TPR / 2; o > 0; o >>= 1) m[i] = fmaxf(m[i], __shfl_xor_sync(0xffffffffu, m[i], o));
  } else {
#pragma unroll
    for (int i = 0; i < NP; ++i) {
#pragma unroll
      for (int o = 16; o > 0; o >>= 1) m[i] = fmaxf(m[i], __shfl_xor_sync(0xffffffffu, m[i], o));
      if ((threadIdx.x & 31) == 0) red[i][threadIdx.x >> 5] = m[i];
    }
    __syncthreads();
    if (threadIdx.x < NP) {
      float x = red[threadIdx.x][0];
#pragma unroll
      for (int w = 1; w < NT / 32; ++w) x = fmaxf(x, red[threadIdx.x][w]);
      pmax[threadIdx.x] = x;
    }
    __syncthreads();
    const int ppb = blk / RPP;  // passes per scale block
#pragma unroll
    for (int i = 0; i < NP; ++i) {
      const int i0 = (i / ppb) * ppb;  // the block's first pass
      float x = 0.0f;
      for (int j = 0; j < ppb; ++j) x = fmaxf(x, pmax[i0 + j]);
      m[i] = x;
    }
  }
  float scale[NP];
#pragma unroll
  for (int i = 0; i < NP; ++i) scale[i] = __fdiv_rn(__fmul_rn(m[i], p.q_mult), 127.0f);
  const size_t head = (size_t)bb * p.Hq + hh;
  if (blk == 1) {
    if (g == 0) {
#pragma unroll
      for (int i = 0; i < NP; ++i) {
        const int row = row0 + r + i * RPP;
        if (row < S) p.q_scale[head * nb + row] = scale[i];
      }
    }
  } else if (r == 0 && g == 0) {
    // one thread per CTA stores the CTA's block scales: block b spans passes [b*ppb, (b+1)*ppb)
    const int ppb = blk / RPP;
#pragma unroll
    for (int i = 0; i < NP; ++i) {
      const int b = (row0 + i * RPP) / blk;
      if (i % ppb == 0 && b < nb) p.q_scale[head * nb + b] = scale[i];
    }
  }
  const size_t first_row = PACKED ? (size_t)hh * p.q_tokens + sp.base : head * (size_t)S;
  int8_t* dst = p.q_i8 + first_row * D + g * 8;
  __half* dst16 = nullptr;
  if constexpr (C16)
    dst16 = p.q_c16 + (int64_t)sp.batch * p.qc_sb + (int64_t)hh * p.qc_sh + (int64_t)sp.base * p.qc_ss + g * 8;
  const float2 mult2 = make_float2(p.q_mult, p.q_mult);
#pragma unroll
  for (int i = 0; i < NP; ++i) {
    const int row = row0 + r + i * RPP;
    if (row >= S) continue;
    const float rcp = __frcp_rn(scale[i]);
    const float2 s2 = make_float2(scale[i], scale[i]), ns2 = make_float2(-scale[i], -scale[i]);
    const float2 r2 = make_float2(rcp, rcp);
    float f[8];
    Half8<T>::to_float(raw[i], f);
    int qv[8];
#pragma unroll
    for (int e = 0; e < 8; e += 2) quant_two(fmul2(make_float2(f[e], f[e + 1]), mult2), s2, ns2, r2, qv[e], qv[e + 1]);
    if constexpr (C16) {
      *reinterpret_cast<uint4*>(dst16 + (int64_t)row * p.qc_ss) =
          make_uint4(codes_to_half2(qv[0], qv[1]), codes_to_half2(qv[2], qv[3]), codes_to_half2(qv[4], qv[5]),
                     codes_to_half2(qv[6], qv[7]));
    } else {
      *reinterpret_cast<uint2*>(dst + (size_t)row * D) =
          make_uint2(pack4_lo_bytes(qv[0], qv[1], qv[2], qv[3]), pack4_lo_bytes(qv[4], qv[5], qv[6], qv[7]));
    }
  }
}

struct FinalizeParams {
  const double* ksum_part;  // nullable
  const float* vmax_part;   // nullable
  float* k_mean;            // [B, Hkv, D]
  float* v_scale;           // [B, Hkv, D]
  int Hkv, S, nchunk, D;
  const int* cu;            // variable-length batches: K/V sequence b is rows [cu[b], cu[b+1])
  int tokens;
};

// Grid (Hkv, B), D threads: km = fp32(sum / S), v_scale = absmax / 448.
__global__ void kv_finalize_kernel(FinalizeParams p) {
  const int h = blockIdx.x, b = blockIdx.y, d = threadIdx.x;
  if (d >= p.D) return;
  const size_t head = (size_t)b * p.Hkv + h;
  if (p.ksum_part) {
    double s = 0.0;
    for (int c = 0; c < p.nchunk; ++c) s = __dadd_rn(s, p.ksum_part[(head * p.nchunk + c) * p.D + d]);
    const int len = seq_span(p.cu, b, p.S, p.tokens).len;
    // an empty sequence has no K rows to smooth: its mean is never used; 0 keeps it finite
    p.k_mean[head * p.D + d] = len > 0 ? __double2float_rn(__ddiv_rn(s, static_cast<double>(len))) : 0.0f;
  }
  if (p.vmax_part) {
    float m = 0.0f;
    for (int c = 0; c < p.nchunk; ++c) m = fmaxf(m, p.vmax_part[(head * p.nchunk + c) * p.D + d]);
    p.v_scale[head * p.D + d] = __fdiv_rn(m, 448.0f);
  }
}

}  // namespace sage
