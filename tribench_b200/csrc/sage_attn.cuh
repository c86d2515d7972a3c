// sage_attn.cuh — fused INT8-QK attention for sm_100a (tcgen05 + TMEM + TMA).
//
// Computes what _attn_fwd / _attn_fwd_inner compute (kernels/sage_attn/triton_impl.py:86-160):
// for each query row, over 128-key tiles,
//   s   = float(q_i8 . k_i8) * (q_scale * k_scale)         (:99; q_scale carries sm_scale*log2 e)
//   m'  = max(m, rowmax(s)); p = exp2(s - m'); alpha = exp2(m - m')   (:102-107)
//   l   = l * alpha + rowsum(p); acc = acc * alpha + p . V  (:108-113)
//   o   = acc / l, cast to the output dtype                  (:159-160)
// with masked keys (past seq_kv, :95,100; and, unlike the Triton kernel, key > query when
// causal) excluded. P.V accumulates in fp32 in TMEM (the reference accumulates each
// 64-key block in fp16, :113).
//
// CTA = QT query tiles of 128 rows that share every K/V tile (QT = 2: 256 query rows).
// Warp roles:
//   warps [0, 4*QT)   softmax: warpgroup t owns query tile t; thread i owns TMEM lane i
//   warp 4*QT         TMA producer: Q once, then K/V tiles through an NS-stage ring
//   warp 4*QT + 1     MMA issuer: QK^T (kind::i8 -> int32) and P.V (kind::f16/f8f6f4 -> fp32);
//                     also allocates / frees TMEM
// TMEM (columns): tile t has S_t at 256*t (128 int32 columns) and O_t at 256*t + 128 (D fp32
// columns). P_t (16-bit or e4m3) is written over the upper columns of S_t after the thread has
// read its whole S row, and feeds the P.V MMA straight from TMEM.
// MMA order per key tile j: PV_t(j) then QK_t(j+1) for each t; the tensor pipe executes
// tcgen05.mma in issue order, so QK_t(j+1) cannot overwrite P_t(j) before PV_t(j) read it.
#pragma once

#include "sm100_ptx.cuh"

namespace sage {

enum PvKind : int { kPvF16 = 0, kPvBF16 = 1, kPvE4M3 = 2 };

struct AttnParams {
  const float* q_scale;  // [B, Hq, nqb]
  const float* k_scale;  // [B, Hkv, nkb]
  const float* v_scale;  // [B, Hkv, D]  (e4m3 P.V only)
  void* o;
  int64_t o_sb, o_sh, o_ss;  // output strides, elements
  int B, Hq, Hkv, Sq, Skv, groups;
  int nqb, nkb;
  int causal;
  int n_m_ctas;              // CTAs along the query axis
  unsigned long long wait_limit_ns;
};

template <int D, int PV, int QT>
struct AttnCfg {
  static constexpr int BM = 128;               // query rows per tile
  static constexpr int BN = 128;               // keys per tile
  static constexpr int V_ELT = (PV == kPvE4M3) ? 1 : 2;
  static constexpr int NS = (D == 128) ? ((PV == kPvE4M3) ? 4 : 3) : 4;  // K/V ring stages
  static constexpr int Q_TILE = BM * D;        // bytes (int8)
  static constexpr int K_TILE = BN * D;        // bytes (int8)
  static constexpr int V_TILE = BN * D * V_ELT;
  static constexpr int OFF_Q = 0;
  static constexpr int OFF_K = OFF_Q + QT * Q_TILE;
  static constexpr int OFF_V = OFF_K + NS * K_TILE;
  static constexpr int OFF_BAR = OFF_V + NS * V_TILE;
  static constexpr int NUM_BARS = 1 + 3 * NS + 3 * QT;
  static constexpr int OFF_MISC = OFF_BAR + NUM_BARS * 8;
  static constexpr int SMEM_USED = OFF_MISC + 16;
  // Pad to > half of the SM's shared memory so that exactly one CTA is resident per SM:
  // each CTA allocates all 512 TMEM columns when QT == 2.
  static constexpr int SMEM_MIN = (QT == 2) ? 118 * 1024 : 0;
  static constexpr int SMEM_BYTES = 1024 + (SMEM_USED > SMEM_MIN ? SMEM_USED : SMEM_MIN);
  static constexpr int NUM_THREADS = 32 * (4 * QT + 2);
  static constexpr int TMEM_COLS = (QT == 2) ? 512 : 256;
  // K-major operands: SW128 for 128-byte rows, SW64 for 64-byte rows.
  static constexpr uint32_t QK_LAYOUT = (D == 128) ? kLayoutSW128 : kLayoutSW64;
  static constexpr uint32_t QK_SBO = (D == 128) ? 1024 : 512;
  // V (MN-major B of P.V): rows of D*V_ELT bytes split into 128-byte swizzle atoms.
  static constexpr int V_ROW_BYTES = D * V_ELT;
  static constexpr uint32_t V_LAYOUT = (V_ROW_BYTES >= 128) ? kLayoutSW128 : kLayoutSW64;
  static constexpr uint32_t V_SBO = (V_ROW_BYTES >= 128) ? 1024 : 512;
  static constexpr uint32_t V_LBO = BN * 128;  // distance between 128-byte column atoms
  static constexpr int V_ATOM_ROW = (V_ROW_BYTES >= 128) ? 128 : V_ROW_BYTES;  // bytes per key row in an atom
  static constexpr int V_BOXES = (V_ROW_BYTES > 128) ? V_ROW_BYTES / 128 : 1;
  static constexpr int PV_K = (PV == kPvE4M3) ? 32 : 16;  // keys per P.V MMA
  static constexpr uint32_t P_COL = (PV == kPvE4M3) ? 96 : 64;  // P offset inside S_t
  static constexpr uint32_t IDESC_QK =
      make_idesc(kFmtD_S32, kFmtS8, kFmtS8, 0, 0, BM, BN);
  static constexpr uint32_t PV_FMT = (PV == kPvBF16) ? kFmtBF16 : ((PV == kPvE4M3) ? kFmtE4M3 : kFmtF16);
  static constexpr uint32_t IDESC_PV = make_idesc(kFmtD_F32, PV_FMT, PV_FMT, 0, 1, BM, D);
};

// Bounded-wait limit sentinel codes (match SAGE_DEV_* in sage_sm100.h).
enum : int { kDevTimeoutProducer = 1, kDevTimeoutMma = 2, kDevTimeoutSoftmax = 4, kDevTimeoutEpilogue = 8 };

template <int D, int PV, int QT, bool OBF16>
__global__ void __launch_bounds__(AttnCfg<D, PV, QT>::NUM_THREADS, 1)
    sage_attn_kernel(const __grid_constant__ CUtensorMap tmQ, const __grid_constant__ CUtensorMap tmK,
                     const __grid_constant__ CUtensorMap tmV, const AttnParams p) {
  using C = AttnCfg<D, PV, QT>;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + C::OFF_BAR);
  uint64_t* bar_q = bars;
  uint64_t* bar_kfull = bars + 1;
  uint64_t* bar_vfull = bar_kfull + C::NS;
  uint64_t* bar_kvempty = bar_vfull + C::NS;
  uint64_t* bar_sfull = bar_kvempty + C::NS;
  uint64_t* bar_pfull = bar_sfull + QT;
  uint64_t* bar_odone = bar_pfull + QT;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(smem + C::OFF_MISC);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(smem + C::OFF_MISC + 4);

  const uint32_t warp = warp_id();
  const uint32_t lane = lane_id();
  const int m_cta = p.causal ? (p.n_m_ctas - 1 - static_cast<int>(blockIdx.x)) : static_cast<int>(blockIdx.x);
  const int h = blockIdx.y;
  const int b = blockIdx.z;
  const int hkv = h / p.groups;
  const int nkv_all = (p.Skv + C::BN - 1) / C::BN;

  // Key tiles each query tile needs (0 for a tile entirely past seq_q).
  int nkv[QT];
  int nkv_max = 0;
#pragma unroll
  for (int t = 0; t < QT; ++t) {
    const int r0 = (m_cta * QT + t) * C::BM;
    int n = nkv_all;
    if (p.causal) n = min(n, r0 / C::BN + 1);
    if (r0 >= p.Sq) n = 0;
    nkv[t] = n;
    nkv_max = max(nkv_max, n);
  }

  if (threadIdx.x == 0) {
    mbar_init(bar_q, 1);
    for (int s = 0; s < C::NS; ++s) {
      mbar_init(bar_kfull + s, 1);
      mbar_init(bar_vfull + s, 1);
      mbar_init(bar_kvempty + s, 1);
    }
    for (int t = 0; t < QT; ++t) {
      mbar_init(bar_sfull + t, 1);
      mbar_init(bar_pfull + t, 128);
      mbar_init(bar_odone + t, 1);
    }
    *abort_flag = 0;
    fence_barrier_init();
  }
  if (warp == 4 * QT + 1) {  // MMA warp owns TMEM
    tmem_alloc(tmem_slot, C::TMEM_COLS);
    tmem_relinquish();
  }
  if (warp == 4 * QT && lane == 0) {
    tma_prefetch_desc(&tmQ);
    tma_prefetch_desc(&tmK);
    tma_prefetch_desc(&tmV);
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;

  if (warp == 4 * QT) {
    // ------------------------------------------------------------ TMA producer
    if (elect_one() && nkv_max > 0) {
      mbar_arrive_expect_tx(bar_q, QT * C::Q_TILE);
#pragma unroll
      for (int t = 0; t < QT; ++t)
        tma_load_4d(smem + C::OFF_Q + t * C::Q_TILE, &tmQ, bar_q, 0, (m_cta * QT + t) * C::BM, h, b);
      for (int j = 0; j < nkv_max; ++j) {
        const int s = j % C::NS;
        if (j >= C::NS) {
          if (!mbar_wait(bar_kvempty + s, ((j / C::NS) - 1) & 1, abort_flag, kDevTimeoutProducer, p.wait_limit_ns)) break;
        }
        mbar_arrive_expect_tx(bar_kfull + s, C::K_TILE);
        tma_load_4d(smem + C::OFF_K + s * C::K_TILE, &tmK, bar_kfull + s, 0, j * C::BN, hkv, b);
        mbar_arrive_expect_tx(bar_vfull + s, C::V_TILE);
#pragma unroll
        for (int x = 0; x < C::V_BOXES; ++x)
          tma_load_4d(smem + C::OFF_V + s * C::V_TILE + x * (C::BN * 128), &tmV, bar_vfull + s,
                      x * (128 / C::V_ELT), j * C::BN, hkv, b);
      }
    }
  } else if (warp == 4 * QT + 1) {
    // ------------------------------------------------------------ MMA issuer
    if (elect_one() && nkv_max > 0) {
      const uint32_t q_addr = smem_u32(smem + C::OFF_Q);
      const uint32_t k_addr = smem_u32(smem + C::OFF_K);
      const uint32_t v_addr = smem_u32(smem + C::OFF_V);
      bool ok = mbar_wait(bar_q, 0, abort_flag, kDevTimeoutMma, p.wait_limit_ns);
      // QK of tile 0 for every query tile.
      if (ok) ok = mbar_wait(bar_kfull, 0, abort_flag, kDevTimeoutMma, p.wait_limit_ns);
      tc_fence_after();
      if (ok) {
#pragma unroll
        for (int t = 0; t < QT; ++t) {
          if (nkv[t] == 0) continue;
          const uint64_t qd = make_smem_desc(q_addr + t * C::Q_TILE, 16, C::QK_SBO, C::QK_LAYOUT);
          const uint64_t kd = make_smem_desc(k_addr, 16, C::QK_SBO, C::QK_LAYOUT);
#pragma unroll
          for (int kk = 0; kk < D / 32; ++kk)
            umma_i8_ss(tmem_base + 256 * t, desc_advance(qd, 32 * kk), desc_advance(kd, 32 * kk), C::IDESC_QK, kk > 0);
          umma_commit(bar_sfull + t);
        }
      }
      for (int j = 0; ok && j < nkv_max; ++j) {
        const int s = j % C::NS;
        bool v_ready = false, knext_ready = false;
#pragma unroll
        for (int t = 0; t < QT; ++t) {
          if (j >= nkv[t]) continue;
          if (!mbar_wait(bar_pfull + t, j & 1, abort_flag, kDevTimeoutMma, p.wait_limit_ns)) { ok = false; break; }
          if (!v_ready) {
            if (!mbar_wait(bar_vfull + s, (j / C::NS) & 1, abort_flag, kDevTimeoutMma, p.wait_limit_ns)) { ok = false; break; }
            v_ready = true;
          }
          tc_fence_after();
          const uint64_t vd = make_smem_desc(v_addr + s * C::V_TILE, C::V_LBO, C::V_SBO, C::V_LAYOUT);
          const uint32_t p_tmem = tmem_base + 256 * t + C::P_COL;
          const uint32_t o_tmem = tmem_base + 256 * t + 128;
#pragma unroll
          for (int kk = 0; kk < C::BN / C::PV_K; ++kk) {
            const uint64_t vdk = desc_advance(vd, kk * C::PV_K * C::V_ATOM_ROW);
            if constexpr (PV == kPvE4M3)
              umma_f8_ts(o_tmem, p_tmem + kk * 8, vdk, C::IDESC_PV, (j > 0 || kk > 0) ? 1u : 0u);
            else
              umma_f16_ts(o_tmem, p_tmem + kk * 8, vdk, C::IDESC_PV, (j > 0 || kk > 0) ? 1u : 0u);
          }
          umma_commit(bar_odone + t);
          if (j + 1 < nkv[t]) {
            const int s1 = (j + 1) % C::NS;
            if (!knext_ready) {
              if (!mbar_wait(bar_kfull + s1, ((j + 1) / C::NS) & 1, abort_flag, kDevTimeoutMma, p.wait_limit_ns)) { ok = false; break; }
              knext_ready = true;
              tc_fence_after();
            }
            const uint64_t qd = make_smem_desc(q_addr + t * C::Q_TILE, 16, C::QK_SBO, C::QK_LAYOUT);
            const uint64_t kd = make_smem_desc(k_addr + s1 * C::K_TILE, 16, C::QK_SBO, C::QK_LAYOUT);
#pragma unroll
            for (int kk = 0; kk < D / 32; ++kk)
              umma_i8_ss(tmem_base + 256 * t, desc_advance(qd, 32 * kk), desc_advance(kd, 32 * kk), C::IDESC_QK, kk > 0);
            umma_commit(bar_sfull + t);
          }
        }
        umma_commit(bar_kvempty + s);  // K_s / V_s reusable once every MMA issued so far is done
      }
    }
  } else {
    // ------------------------------------------------------------ softmax warpgroups
    const int t = warp / 4;
    const int row_in_tile = (warp % 4) * 32 + lane;
    const int r0 = (m_cta * QT + t) * C::BM;
    const int row = r0 + row_in_tile;
    const uint32_t lane_base = ((warp % 4) * 32u) << 16;
    const uint32_t s_tmem = tmem_base + lane_base + 256 * t;
    const uint32_t o_tmem = s_tmem + 128;
    const int n = nkv[t];
    const float qs = (n > 0) ? p.q_scale[((size_t)b * p.Hq + h) * p.nqb + r0 / C::BM] : 0.0f;
    const float* ksp = p.k_scale + ((size_t)b * p.Hkv + hkv) * p.nkb;
    float m_run = -INFINITY, l_run = 0.0f;
    bool ok = true;
    for (int j = 0; j < n; ++j) {
      if (!__all_sync(0xffffffffu, mbar_wait(bar_sfull + t, j & 1, abort_flag, kDevTimeoutSoftmax, p.wait_limit_ns))) { ok = false; break; }
      tc_fence_after();
      uint32_t sr[128];
      tmem_ld64_sync(s_tmem, *reinterpret_cast<uint32_t(*)[64]>(&sr[0]));
      tmem_ld64_sync(s_tmem + 64, *reinterpret_cast<uint32_t(*)[64]>(&sr[64]));
      const int kb0 = 2 * j;
      const float sc0 = qs * ksp[kb0];
      const float sc1 = (kb0 + 1 < p.nkb) ? qs * ksp[kb0 + 1] : 0.0f;
      float sf[128];
#pragma unroll
      for (int c = 0; c < 128; ++c) sf[c] = i2f_exact22(sr[c]) * (c < 64 ? sc0 : sc1);
      const int key0 = j * C::BN;
      const bool need_mask = (key0 + C::BN > p.Skv) || (p.causal && key0 + C::BN - 1 > r0);
      if (need_mask) {
        const int lim = p.causal ? min(p.Skv, row + 1) : p.Skv;  // keys [key0, lim) visible
#pragma unroll
        for (int c = 0; c < 128; ++c)
          if (key0 + c >= lim) sf[c] = -INFINITY;
      }
      float mx = m_run;
#pragma unroll
      for (int c = 0; c < 128; ++c) mx = fmaxf(mx, sf[c]);
      const float m_use = (mx == -INFINITY) ? 0.0f : mx;
      const float alpha = ex2_approx(m_run - m_use);
      float rs = 0.0f;
      uint32_t pk[C::BN * C::V_ELT / 4];
      if constexpr (PV == kPvE4M3) {
        // P scaled by 2^8 into e4m3 range (exact power-of-two shift; undone in the epilogue).
        const float m8 = m_use - 8.0f;
#pragma unroll
        for (int c = 0; c < 128; c += 4) {
          const float e0 = ex2_approx(sf[c] - m8), e1 = ex2_approx(sf[c + 1] - m8);
          const float e2 = ex2_approx(sf[c + 2] - m8), e3 = ex2_approx(sf[c + 3] - m8);
          rs += (e0 + e1) + (e2 + e3);
          const uint32_t lo = __nv_cvt_float2_to_fp8x2(make_float2(e0, e1), __NV_SATFINITE, __NV_E4M3);
          const uint32_t hi = __nv_cvt_float2_to_fp8x2(make_float2(e2, e3), __NV_SATFINITE, __NV_E4M3);
          pk[c / 4] = lo | (hi << 16);
        }
      } else {
#pragma unroll
        for (int c = 0; c < 128; c += 2) {
          const float e0 = ex2_approx(sf[c] - m_use), e1 = ex2_approx(sf[c + 1] - m_use);
          rs += e0 + e1;
          if constexpr (PV == kPvBF16) {
            __nv_bfloat162 v2 = __floats2bfloat162_rn(e0, e1);
            pk[c / 2] = *reinterpret_cast<uint32_t*>(&v2);
          } else {
            __half2 v2 = __floats2half2_rn(e0, e1);
            pk[c / 2] = *reinterpret_cast<uint32_t*>(&v2);
          }
        }
      }
      l_run = l_run * alpha + rs;
      m_run = mx;
      // P into TMEM over the upper columns of S_t.
      if constexpr (PV == kPvE4M3) {
        tmem_st32(s_tmem + C::P_COL, *reinterpret_cast<uint32_t(*)[32]>(&pk[0]));
      } else {
        tmem_st32(s_tmem + C::P_COL, *reinterpret_cast<uint32_t(*)[32]>(&pk[0]));
        tmem_st32(s_tmem + C::P_COL + 32, *reinterpret_cast<uint32_t(*)[32]>(&pk[32]));
      }
      if (j > 0) {
        // O_t *= alpha once PV_t(j-1) has landed.
        if (!__all_sync(0xffffffffu, mbar_wait(bar_odone + t, (j - 1) & 1, abort_flag, kDevTimeoutSoftmax, p.wait_limit_ns))) { ok = false; break; }
        tc_fence_after();
        if (__any_sync(0xffffffffu, alpha != 1.0f)) {
#pragma unroll
          for (int c0 = 0; c0 < D; c0 += 32) {
            uint32_t orow[32];
            tmem_ld32_sync(o_tmem + c0, orow);
#pragma unroll
            for (int c = 0; c < 32; ++c) orow[c] = __float_as_uint(__uint_as_float(orow[c]) * alpha);
            tmem_st32(o_tmem + c0, orow);
          }
        }
      }
      tmem_st_wait();
      tc_fence_before();
      mbar_arrive(bar_pfull + t);
    }
    // ---------------------------------------------------------- epilogue
    if (ok && n > 0 &&
        __all_sync(0xffffffffu, mbar_wait(bar_odone + t, (n - 1) & 1, abort_flag, kDevTimeoutEpilogue, p.wait_limit_ns))) {
      tc_fence_after();
      const float inv_l = 1.0f / l_run;
      const bool valid = row < p.Sq;
      char* orow_ptr = reinterpret_cast<char*>(p.o) +
                       ((int64_t)b * p.o_sb + (int64_t)h * p.o_sh + (int64_t)row * p.o_ss) * 2;
      const float* vsp = p.v_scale + ((size_t)b * p.Hkv + hkv) * D;
#pragma unroll
      for (int c0 = 0; c0 < D; c0 += 32) {
        uint32_t orow[32];
        tmem_ld32_sync(o_tmem + c0, orow);
        uint32_t packed[16];
#pragma unroll
        for (int c = 0; c < 32; c += 2) {
          float a = __uint_as_float(orow[c]) * inv_l;
          float z = __uint_as_float(orow[c + 1]) * inv_l;
          if constexpr (PV == kPvE4M3) {
            a *= vsp[c0 + c];
            z *= vsp[c0 + c + 1];
          }
          if constexpr (OBF16) {
            __nv_bfloat162 v2 = __floats2bfloat162_rn(a, z);
            packed[c / 2] = *reinterpret_cast<uint32_t*>(&v2);
          } else {
            __half2 v2 = __floats2half2_rn(a, z);
            packed[c / 2] = *reinterpret_cast<uint32_t*>(&v2);
          }
        }
        if (valid) {
          uint4* dst = reinterpret_cast<uint4*>(orow_ptr + c0 * 2);
#pragma unroll
          for (int v = 0; v < 4; ++v)
            dst[v] = make_uint4(packed[4 * v], packed[4 * v + 1], packed[4 * v + 2], packed[4 * v + 3]);
        }
      }
    }
  }

  // ------------------------------------------------------------ teardown
  tc_fence_before();
  __syncthreads();
  if (warp == 4 * QT + 1) {
    tc_fence_after();
    tmem_dealloc(tmem_base, C::TMEM_COLS);
  }
}

}  // namespace sage
