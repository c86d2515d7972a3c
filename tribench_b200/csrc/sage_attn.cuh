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
// FLASH = true instantiates the same pipeline without quantisation, for the flash_attn pack
// (kernels/flash_attn/triton_impl.py:13-108): Q and K stay fp16/bf16, QK^T is kind::f16 into fp32
// scores, and the scale is sm_scale * log2(e) for every key.
//
// CTA = QT query tiles of 128 rows that share every K/V tile (QT = 2: 256 query rows).
// Warp roles:
//   warps [0, 4*QT)   softmax: warpgroup t owns query tile t; thread i owns TMEM lane i
//   warp 4*QT         TMA producer: Q once, then K/V tiles through an NS-stage ring
//   warp 4*QT + 1     MMA issuer: QK^T (kind::i8 -> int32) and P.V (kind::f16/f8f6f4 -> fp32);
//                     also allocates / frees TMEM
// TMEM (columns): tile t has S_t at 256*t (128 int32 columns) and O_t at 256*t + 128 (D fp32
// columns); P_t (16-bit or e4m3) feeds the P.V MMA straight from TMEM.
//   D = 128: P_t is written over the upper columns of S_t after the thread has read its whole S
//     row. MMA order per key tile j: PV_t(j) then QK_t(j+1) for each t; the tensor pipe executes
//     tcgen05.mma in issue order, so QK_t(j+1) cannot overwrite P_t(j) before PV_t(j) read it.
//   D = 64: P_t has its own columns (256*t + 192), so QK_t(j+1) is issued as soon as softmax has
//     read S_t(j) (sload) and runs while softmax works on tile j; softmax in turn waits for
//     PV_t(j-1) to finish (pvdone) before it writes P_t(j) or rescales O_t.
#pragma once

#include <type_traits>

#include "sage_quant.cuh"
#include "sage_seq.cuh"
#include "sm100_ptx.cuh"

namespace sage {

enum PvKind : int { kPvF16 = 0, kPvBF16 = 1, kPvE4M3 = 2 };

struct AttnParams {
  const float* q_scale;  // [B, Hq, nqb]: one scale per 2^qblk_shift query rows
  const float* k_scale;  // [B, Hkv, nkb]
  const float* v_scale;  // [B, Hkv, D]  (e4m3 P.V only)
  void* o;
  int64_t o_sb, o_sh, o_ss;  // output strides, elements
  int B, Hq, Hkv, Sq, Skv, groups;  // variable-length batches: Sq / Skv = longest sequence
  int nqb, nkb;
  // Q scale blocks of 2^qblk_shift rows: 7 (128 rows, the reference's default BLKQ), 6, 5, 4, or
  // 0 (one scale per token). Every softmax thread owns one query row, so it simply reads its
  // own row's scale.
  int qblk_shift;
  // Variable-length batches (nullable): sequence b owns token rows [cu_q[b], cu_q[b+1]) of Q/O
  // and [cu_k[b], cu_k[b+1]) of K/V, whose tensors have batch extent 1 and q_tokens / k_tokens
  // rows; the scales stay [B, H, nqb / nkb] per sequence.
  const int* cu_q;
  const int* cu_k;
  int q_tokens, k_tokens;
  int causal;
  int o_stage;               // 1: o is not this GPU's own memory (e.g. a peer mapping): line-coalesced stores
  int n_m_ctas;              // CTAs along the query axis
  unsigned long long wait_limit_ns;
  float qk_scale;            // FLASH only: sm_scale * log2(e)
  // Q quantised inside the kernel (nullable): q_src is the caller's 16-bit Q with element strides
  // q_sb/q_sh/q_ss (batch, head, token), quantised per 128-row tile exactly as the pre-pass
  // does (multiplier q_mult). q_i8_out / q_scale_out (nullable) receive the codes and scales in
  // the pre-pass's layouts.
  const void* q_src;
  int64_t q_sb, q_sh, q_ss;
  float q_mult;
  int8_t* q_i8_out;
  float* q_scale_out;
};

// C16: the INT8 codes of Q and K arrive as fp16 values (exact: |code| <= 127) and QK^T runs as a
// kind::f16 MMA into fp32 scores. Each product is an integer below 2^14 and each row sum one
// below 2^21 (D <= 128), so every partial sum is exact in fp32 and the scores equal the INT8
// MMA's to the bit, as floats, with no int32 -> float step in the softmax.
template <int D, int PV, int QT, bool FLASH = false, bool C16 = false>
struct AttnCfg {
  static_assert(!FLASH || PV != kPvE4M3, "the flash variant keeps P in the input dtype");
  static_assert(!(FLASH && C16), "C16 is the INT8 path's operand form");
  static constexpr bool QK_F16 = FLASH || C16;  // Q/K tiles hold 16-bit values, QK^T is kind::f16
  static constexpr int BM = 128;               // query rows per tile
  static constexpr int BN = 128;               // keys per tile
  static constexpr int V_ELT = (PV == kPvE4M3) ? 1 : 2;
  static constexpr int QK_ELT = QK_F16 ? 2 : 1; // bytes per Q/K element (int8, or fp16/bf16)
  // K/V ring stages (shared memory: QT Q tiles + NS x (K + V) tiles within 227 KB)
  static constexpr int NS = FLASH ? ((D == 128) ? 2 : 4) : ((D == 128) ? ((PV == kPvE4M3) ? 4 : 3) : 4);
  static constexpr int Q_TILE = BM * D * QK_ELT;  // bytes
  static constexpr int K_TILE = BN * D * QK_ELT;  // bytes
  static constexpr int V_TILE = BN * D * V_ELT;
  static constexpr int OFF_Q = 0;
  static constexpr int OFF_K = OFF_Q + QT * Q_TILE;
  static constexpr int OFF_V = OFF_K + NS * K_TILE;
  // INT8 scores start from a bias block: S = 0x4B400000 + s directly (see issue_qk), so the
  // softmax needs no integer add per score. The copy shape follows the measurements: with 16-bit
  // P.V, whose MMAs keep the tensor pipe busier, the broadcasting 32x128b.warpx4 copy (s8k_d64
  // 1.618 -> 1.587 ms; 128x256b made it slower); with FP8 P.V the 128x256b copy (C4 1.807 ->
  // 1.772 ms). At D = 128 (same-call A/B against the integer add: H8K 1.817-1.821 -> 1.742-1.789
  // ms, C2 0.978 -> 0.966 ms, bit-identical output) the copy into S_t(j+1) is issued after
  // P.V_t(j), which reads P_t(j) from the upper columns of S_t: like the QK^T MMA that follows it,
  // the copy executes in issue order in the tensor pipe, after P.V_t(j).
  static constexpr bool PRE_BIAS = !QK_F16;
  static constexpr int OFF_BIAS = OFF_V + NS * V_TILE;          // 4 KB of 0x4B400000 words
  static constexpr int OFF_BAR = OFF_BIAS + (PRE_BIAS ? 4096 : 0);
  // q, kfull/vfull/kvempty per stage, sfull/phalf/pfull/odone/sload/pvdone per query tile
  static constexpr int NUM_BARS = 1 + 3 * NS + 6 * QT;
  static constexpr int OFF_MISC = OFF_BAR + NUM_BARS * 8;
  static constexpr int OFF_QRED = OFF_MISC + 16;  // fused Q quantisation: per-warp maxima
  // fused Q quantisation with finer Q blocks: per tile, per-warp maxima of each load pass
  // (16 passes x 4 warps) and the 128 row scales
  static constexpr int OFF_QFINE = OFF_QRED + 16 * QT;
  static constexpr int QFINE_BYTES = (16 * 4 + 128) * 4;
  // epilogue staging: per tile 64 output rows (half the tile) at a time, so that the copy-out
  // writes whole lines (consecutive threads, consecutive 16-byte pieces)
  static constexpr int OFF_OST = (OFF_QFINE + QFINE_BYTES * QT + 127) / 128 * 128;
  static constexpr int OST_BYTES = 64 * D * 2;
  static constexpr int SMEM_USED = OFF_OST + OST_BYTES * QT;
  // Pad to > half of the SM's shared memory so that exactly one CTA is resident per SM:
  // each CTA allocates all 512 TMEM columns when QT == 2.
  static constexpr int SMEM_MIN = (QT == 2) ? 118 * 1024 : 0;
  static constexpr int SMEM_BYTES = 1024 + (SMEM_USED > SMEM_MIN ? SMEM_USED : SMEM_MIN);
  static_assert(SMEM_BYTES <= 227 * 1024, "dynamic shared memory per CTA");
  // softmax warpgroups, then one warpgroup with the producer, the MMA issuer and two idle warps
  static constexpr int NUM_THREADS = 32 * (4 * QT + 4);
  // Launch allocation 168 registers/thread (3 warps per SM sub-partition); the softmax
  // warpgroups take 216, the producer/MMA warpgroup keeps 72:
  // 4*QT*32*216 + 128*72 <= NUM_THREADS*168 for QT = 2 (55296 + 9216 = 64512).
  static constexpr int REGS_SOFTMAX = 216;
  static constexpr int REGS_OTHER = 72;
  static constexpr int TMEM_COLS = (QT == 2) ? 512 : 256;
  // K-major Q/K: SW64 for 64-byte rows, SW128 for rows of 128 bytes or more, which TMA
  // splits into 128-byte column atoms of BM (or BN) rows each. Every MMA K-step covers 32 bytes
  // of a row (32 int8 or 16 fp16/bf16 elements).
  static constexpr int QK_ROW_BYTES = D * QK_ELT;
  static constexpr uint32_t QK_LAYOUT = (QK_ROW_BYTES >= 128) ? kLayoutSW128 : kLayoutSW64;
  static constexpr uint32_t QK_SBO = (QK_ROW_BYTES >= 128) ? 1024 : 512;
  static constexpr int QK_ATOMS = (QK_ROW_BYTES > 128) ? QK_ROW_BYTES / 128 : 1;
  static constexpr int QK_BOX = (QK_ROW_BYTES > 128) ? 128 / QK_ELT : D;  // TMA box width, elements
  static constexpr int QK_STEPS = QK_ROW_BYTES / 32;
  // byte offset of K-step kk inside a K-major tile of `rows` rows
  static __device__ __forceinline__ uint32_t qk_step_offset(int kk, int rows) {
    return (32 * kk / 128) * rows * 128 + (32 * kk) % 128;
  }
  // V (MN-major B of P.V): rows of D*V_ELT bytes split into 128-byte swizzle atoms.
  static constexpr int V_ROW_BYTES = D * V_ELT;
  static constexpr uint32_t V_LAYOUT = (V_ROW_BYTES >= 128) ? kLayoutSW128 : kLayoutSW64;
  static constexpr uint32_t V_SBO = (V_ROW_BYTES >= 128) ? 1024 : 512;
  static constexpr uint32_t V_LBO = BN * 128;  // distance between 128-byte column atoms
  static constexpr int V_ATOM_ROW = (V_ROW_BYTES >= 128) ? 128 : V_ROW_BYTES;  // bytes per key row in an atom
  static constexpr int V_BOXES = (V_ROW_BYTES > 128) ? V_ROW_BYTES / 128 : 1;
  static constexpr int PV_K = (PV == kPvE4M3) ? 32 : 16;  // keys per P.V MMA
  // P_t in its own TMEM columns when O leaves room (D = 64), else over the upper half of S_t
  static constexpr bool SEP_P = (D == 64);
  static constexpr uint32_t P_COL = SEP_P ? 128 + D : ((PV == kPvE4M3) ? 96 : 64);  // offset in the tile
  static constexpr bool PV_FP8 = (PV == kPvE4M3);
  static constexpr uint32_t PV_FMT = (PV == kPvBF16) ? kFmtBF16 : ((PV == kPvE4M3) ? kFmtE4M3 : kFmtF16);
  static constexpr uint32_t IDESC_QK = FLASH ? make_idesc(kFmtD_F32, PV_FMT, PV_FMT, 0, 0, BM, BN)
                                     : C16   ? make_idesc(kFmtD_F32, kFmtF16, kFmtF16, 0, 0, BM, BN)
                                             : make_idesc(kFmtD_S32, kFmtS8, kFmtS8, 0, 0, BM, BN);
  static constexpr uint32_t IDESC_PV = make_idesc(kFmtD_F32, PV_FMT, PV_FMT, 0, 1, BM, D);
  // Softmax: the running max is only raised when a tile's max exceeds it by more than LAZY
  // (log2 units), so P = 2^(s - m) <= 2^LAZY and O needs rescaling only on those rare tiles.
  // FP8 P is scaled by 2^P_SHIFT into the e4m3 range; its threshold keeps
  // P <= 2^(P_SHIFT + LAZY) = 2^8.8 ~ 445.7 below e4m3's largest finite value, 448.
  static constexpr float LAZY = (PV == kPvE4M3) ? 0.8f : 8.0f;
  static constexpr float P_SHIFT = (PV == kPvE4M3) ? 8.0f : 0.0f;
  // Exponentials per 32 columns computed by the FMA-pipe polynomial instead of MUFU.ex2, by
  // measurement: 12 at head_dim 128 and for the flash variant; 8 for the INT8 scheme at 64
  // (same-call A/B against 12: s4k_d64 step 842 -> 803 us, s8k_d64 1549 -> 1479 us, C4
  // 1851 -> 1799 us; 0, 4 and 6 were slower than 8; the flash variant is 3-4 % slower at 8).
#ifdef SAGE_EMU_PER_32
  static constexpr int EMU = SAGE_EMU_PER_32;
#else
  static constexpr int EMU = (D == 64 && !FLASH) ? 8 : 12;
#endif
};

// Bounded-wait limit sentinel codes (match SAGE_DEV_* in sage_sm100.h).
enum : int { kDevTimeoutProducer = 1, kDevTimeoutMma = 2, kDevTimeoutSoftmax = 4, kDevTimeoutEpilogue = 8 };

// QK^T of one query tile against one K tile: S (TMEM) = Q (smem) . K (smem)^T. With PRE_BIAS
// the S columns are first filled with the word 0x4B400000 (tcgen05.cp from a constant block) and
// the MMA accumulates onto it, so each int32 score s arrives as the bit pattern of the float
// 1.5 * 2^23 + s (|s| <= 127^2 * 128 < 2^22), which softmax uses without an integer add.
template <class C>
__device__ __forceinline__ void issue_qk(uint32_t s_tmem, uint32_t q_tile, uint32_t k_tile, uint32_t bias_addr) {
  if constexpr (C::PRE_BIAS) {
    const uint64_t bd = make_smem_desc(bias_addr, 128, 256, 0);  // any layout: every word is equal
    if constexpr (C::PV_FP8) {
#pragma unroll
      for (int c = 0; c < C::BN; c += 8) tmem_cp_128x256b(s_tmem + c, bd);
    } else {
#pragma unroll
      for (int c = 0; c < C::BN; c += 4) tmem_cp_32x128b_warpx4(s_tmem + c, bd);
    }
  }
#pragma unroll
  for (int kk = 0; kk < C::QK_STEPS; ++kk) {
    const uint64_t qd = make_smem_desc(q_tile + C::qk_step_offset(kk, C::BM), 16, C::QK_SBO, C::QK_LAYOUT);
    const uint64_t kd = make_smem_desc(k_tile + C::qk_step_offset(kk, C::BN), 16, C::QK_SBO, C::QK_LAYOUT);
    if constexpr (C::QK_F16)
      umma_f16_ss(s_tmem, qd, kd, C::IDESC_QK, kk > 0);
    else
      umma_i8_ss(s_tmem, qd, kd, C::IDESC_QK, (kk > 0 || C::PRE_BIAS) ? 1u : 0u);
  }
}

// Q quantisation inside the attention kernel. The 128 threads of warpgroup t quantise query
// tile t (one 128-row scale block): thread r loads the 16-byte pieces r, r + 128, r + 256, ...
// of the tile in row-major order (consecutive threads read consecutive bytes of the caller's
// rows), the warpgroup takes the tile's absmax, and each piece's eight INT8 codes go straight
// into the tile's shared-memory image in the layout the TMA load would have produced (K-major,
// 128-byte swizzle for 128-byte rows, 64-byte swizzle for 64-byte rows). The arithmetic is the
// pre-pass's (quant_block_role in sage_quant.cuh), so codes and scale are bit-identical to it.
// Every softmax thread arrives on bar_q after a proxy fence, so the MMA warp may read the tile.
// Returns the tile's scale.
// Named barrier of warpgroup t's 128 threads (ids 3 and 4; immediate ids keep the count known).
__device__ __forceinline__ void warpgroup_sync(int t) {
  if (t == 0) asm volatile("bar.sync 3, 128;" ::: "memory");
  else asm volatile("bar.sync 4, 128;" ::: "memory");
}
// The same barrier, returning whether v holds for all 128 threads (bar.red.and).
__device__ __forceinline__ bool warpgroup_and(int t, bool v) {
  uint32_t r;
  if (t == 0)
    asm volatile("{\n\t.reg .pred p, q;\n\tsetp.ne.u32 p, %1, 0;\n\tbar.red.and.pred q, 3, 128, p;\n\t"
                 "selp.u32 %0, 1, 0, q;\n\t}" : "=r"(r) : "r"(v ? 1u : 0u) : "memory");
  else
    asm volatile("{\n\t.reg .pred p, q;\n\tsetp.ne.u32 p, %1, 0;\n\tbar.red.and.pred q, 4, 128, p;\n\t"
                 "selp.u32 %0, 1, 0, q;\n\t}" : "=r"(r) : "r"(v ? 1u : 0u) : "memory");
  return r != 0;
}

// fused_q_tile with Q scale blocks of 2^qblk_shift < 128 rows (1 = per token, 16, 32, 64). Pass
// i of the loads covers rows [i * RPI, (i + 1) * RPI) of the tile (RPI = 128 / (D / 8)); a row's
// D / 8 pieces sit in consecutive lanes of one warp. Per token: the row's absmax is a shuffle
// reduction over those lanes. Blocks of 16-64 rows (>= RPI): each pass's absmax over the
// warpgroup, then the maximum over the passes of a block. The scales go through shared memory
// (qfine: 64 per-warp pass maxima, then 128 row scales) to the thread that owns each row in the
// softmax. Returns that row's scale.
template <class C, int D, bool OBF16>
__device__ __forceinline__ float fused_q_tile_fine(const AttnParams& p, uint8_t* qtile, float* qfine, int t, int r,
                                                const SeqSpan& sq, int b, int h, int tile, uint64_t* bar_q,
                                                int row_in_tile) {
  using T = typename std::conditional<OBF16, __nv_bfloat16, __half>::type;
  constexpr int PR = D / 8;
  constexpr int NP = C::BM * PR / 128;
  constexpr int RPI = 128 / PR;  // rows per load pass
  float* wmax = qfine;           // [NP][4]
  float* rsc = qfine + 16 * 4;   // [128]
  const int blk_shift = p.qblk_shift;
  const int row0 = tile * C::BM;
  const char* base = reinterpret_cast<const char*>(p.q_src) +
                     ((int64_t)sq.batch * p.q_sb + (int64_t)h * p.q_sh + (int64_t)(sq.base + row0) * p.q_ss) * 2;
  uint4 raw[NP];
#pragma unroll
  for (int i = 0; i < NP; ++i) {
    const int pc = i * 128 + r, row = pc / PR, c = pc % PR;
    raw[i] = (row0 + row < sq.len) ? ldg_nc_v4(base + (int64_t)row * p.q_ss * 2 + c * 16) : make_uint4(0u, 0u, 0u, 0u);
  }
  float m[NP];
#pragma unroll
  for (int i = 0; i < NP; ++i) m[i] = Half8<T>::absmax(raw[i]);
  if (blk_shift == 0) {
#pragma unroll
    for (int i = 0; i < NP; ++i)
#pragma unroll
      for (int o = PR / 2; o > 0; o >>= 1) m[i] = fmaxf(m[i], __shfl_xor_sync(0xffffffffu, m[i], o));
  } else {
#pragma unroll
    for (int i = 0; i < NP; ++i) {
#pragma unroll
      for (int o = 16; o > 0; o >>= 1) m[i] = fmaxf(m[i], __shfl_xor_sync(0xffffffffu, m[i], o));
      if ((r & 31) == 0) wmax[i * 4 + (r >> 5)] = m[i];
    }
    warpgroup_sync(t);
    const int ppb = (1 << blk_shift) / RPI;  // passes per scale block
#pragma unroll
    for (int i = 0; i < NP; ++i) {
      const int i0 = (i / ppb) * ppb;  // the block's first pass
      float x = 0.0f;
      for (int j = i0; j < i0 + ppb; ++j)
        x = fmaxf(x, fmaxf(fmaxf(wmax[j * 4], wmax[j * 4 + 1]), fmaxf(wmax[j * 4 + 2], wmax[j * 4 + 3])));
      m[i] = x;
    }
  }
  float scale[NP];
#pragma unroll
  for (int i = 0; i < NP; ++i) scale[i] = __fdiv_rn(__fmul_rn(m[i], p.q_mult), 127.0f);
  const float2 mult2 = make_float2(p.q_mult, p.q_mult);
  int8_t* dump = nullptr;
  if (p.q_i8_out != nullptr) {
    const size_t first = p.cu_q ? (size_t)h * p.q_tokens + sq.base : ((size_t)b * p.Hq + h) * (size_t)sq.len;
    dump = p.q_i8_out + (first + row0) * D;
  }
  const size_t scale_head = ((size_t)b * p.Hq + h) * p.nqb;
#pragma unroll
  for (int i = 0; i < NP; ++i) {
    const int pc = i * 128 + r, row = pc / PR, c = pc % PR;
    const float rcp = __frcp_rn(scale[i]);
    const float2 s2 = make_float2(scale[i], scale[i]), ns2 = make_float2(-scale[i], -scale[i]);
    const float2 r2 = make_float2(rcp, rcp);
    float f[8];
    Half8<T>::to_float(raw[i], f);
    int qv[8];
#pragma unroll
    for (int e = 0; e < 8; e += 2)
      quant_two(fmul2(make_float2(f[e], f[e + 1]), mult2), s2, ns2, r2, qv[e], qv[e + 1]);
    const uint2 codes = make_uint2(pack4_lo_bytes(qv[0], qv[1], qv[2], qv[3]), pack4_lo_bytes(qv[4], qv[5], qv[6], qv[7]));
    const int sw = (D == 128) ? ((c >> 1) ^ (row & 7)) : ((c >> 1) ^ ((row >> 1) & 3));
    *reinterpret_cast<uint2*>(qtile + row * D + sw * 16 + (c & 1) * 8) = codes;
    if (dump && row0 + row < sq.len) *reinterpret_cast<uint2*>(dump + row * D + c * 8) = codes;
    if (c == 0) {
      rsc[row] = scale[i];
      // the codes' scale, once per block: the block's first row
      if (p.q_scale_out != nullptr && row0 + row < sq.len && ((row0 + row) & ((1 << blk_shift) - 1)) == 0)
        p.q_scale_out[scale_head + ((row0 + row) >> blk_shift)] = scale[i];
    }
  }
  warpgroup_sync(t);
  const float own = rsc[row_in_tile];
  fence_proxy_async_smem();  // the codes are read by tcgen05.mma (async proxy)
  mbar_arrive(bar_q);
  return own;
}

template <class C, int D, bool OBF16>
__device__ __forceinline__ float fused_q_tile(const AttnParams& p, uint8_t* qtile, float* red, int t, int r,
                                              const SeqSpan& sq, int b, int h, int tile, uint64_t* bar_q) {
  using T = typename std::conditional<OBF16, __nv_bfloat16, __half>::type;
  constexpr int PR = D / 8;              // 16-byte pieces (8 elements) per row
  constexpr int NP = C::BM * PR / 128;   // pieces per thread
  const int row0 = tile * C::BM;
  const char* base = reinterpret_cast<const char*>(p.q_src) +
                     ((int64_t)sq.batch * p.q_sb + (int64_t)h * p.q_sh + (int64_t)(sq.base + row0) * p.q_ss) * 2;
  uint4 raw[NP];
#pragma unroll
  for (int i = 0; i < NP; ++i) {
    const int pc = i * 128 + r, row = pc / PR, c = pc % PR;
    raw[i] = (row0 + row < sq.len) ? ldg_nc_v4(base + (int64_t)row * p.q_ss * 2 + c * 16) : make_uint4(0u, 0u, 0u, 0u);
  }
  float amax = 0.0f;
#pragma unroll
  for (int i = 0; i < NP; ++i) amax = fmaxf(amax, Half8<T>::absmax(raw[i]));
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, o));
  if ((r & 31) == 0) red[r >> 5] = amax;
  warpgroup_sync(t);
  amax = fmaxf(fmaxf(red[0], red[1]), fmaxf(red[2], red[3]));
  const float scale = __fdiv_rn(__fmul_rn(amax, p.q_mult), 127.0f);
  const float rcp = __frcp_rn(scale);
  const float2 s2 = make_float2(scale, scale), ns2 = make_float2(-scale, -scale), r2 = make_float2(rcp, rcp);
  const float2 mult2 = make_float2(p.q_mult, p.q_mult);
  int8_t* dump = nullptr;
  if (p.q_i8_out != nullptr) {
    const size_t first = p.cu_q ? (size_t)h * p.q_tokens + sq.base : ((size_t)b * p.Hq + h) * (size_t)sq.len;
    dump = p.q_i8_out + (first + row0) * D;
  }
#pragma unroll
  for (int i = 0; i < NP; ++i) {
    const int pc = i * 128 + r, row = pc / PR, c = pc % PR;
    float f[8];
    Half8<T>::to_float(raw[i], f);
    int qv[8];
#pragma unroll
    for (int e = 0; e < 8; e += 2)
      quant_two(fmul2(make_float2(f[e], f[e + 1]), mult2), s2, ns2, r2, qv[e], qv[e + 1]);
    const uint2 codes = make_uint2(pack4_lo_bytes(qv[0], qv[1], qv[2], qv[3]), pack4_lo_bytes(qv[4], qv[5], qv[6], qv[7]));
    // 16-byte swizzle unit c/2 of the row, half c%2 of it
    const int sw = (D == 128) ? ((c >> 1) ^ (row & 7)) : ((c >> 1) ^ ((row >> 1) & 3));
    *reinterpret_cast<uint2*>(qtile + row * D + sw * 16 + (c & 1) * 8) = codes;
    if (dump && row0 + row < sq.len) *reinterpret_cast<uint2*>(dump + row * D + c * 8) = codes;
  }
  if (p.q_scale_out != nullptr && r == 0 && row0 < sq.len) p.q_scale_out[((size_t)b * p.Hq + h) * p.nqb + tile] = scale;
  fence_proxy_async_smem();  // the codes are read by tcgen05.mma (async proxy)
  mbar_arrive(bar_q);
  return scale;
}

// FQ: Q arrives as the caller's 16-bit tensor and is quantised by the softmax warps
// (fused_q_tile); a separate instantiation, so the default kernel carries none of that code.
template <int D, int PV, int QT, bool OBF16, bool FLASH, bool FQ = false, bool C16 = false>
__global__ void __launch_bounds__(AttnCfg<D, PV, QT, FLASH, C16>::NUM_THREADS, 1)
    sage_attn_kernel(const __grid_constant__ CUtensorMap tmQ, const __grid_constant__ CUtensorMap tmK,
                     const __grid_constant__ CUtensorMap tmV, const AttnParams p) {
  using C = AttnCfg<D, PV, QT, FLASH, C16>;
  static_assert(!(FQ && C16), "Q quantised in the kernel is stored as INT8 codes");
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + C::OFF_BAR);
  uint64_t* bar_q = bars;
  uint64_t* bar_kfull = bars + 1;
  uint64_t* bar_vfull = bar_kfull + C::NS;
  uint64_t* bar_kvempty = bar_vfull + C::NS;
  uint64_t* bar_sfull = bar_kvempty + C::NS;
  uint64_t* bar_phalf = bar_sfull + QT;
  uint64_t* bar_pfull = bar_phalf + QT;
  uint64_t* bar_odone = bar_pfull + QT;
  uint64_t* bar_sload = bar_odone + QT;  // [tile]: softmax holds S_t(j) in registers (SEP_P)
  uint64_t* bar_pvdone = bar_sload + QT; // [tile]: PV_t(j) has landed in O_t (SEP_P)
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(smem + C::OFF_MISC);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(smem + C::OFF_MISC + 4);

  const uint32_t warp = warp_id();
  const uint32_t lane = lane_id();
  const int m_cta = p.causal ? (p.n_m_ctas - 1 - static_cast<int>(blockIdx.x)) : static_cast<int>(blockIdx.x);
  const int h = blockIdx.y;
  const int b = blockIdx.z;
  const int hkv = h / p.groups;
  const SeqSpan sq = seq_span(p.cu_q, b, p.Sq, p.q_tokens);
  const SeqSpan sk = seq_span(p.cu_k, b, p.Skv, p.k_tokens);
  const int Sq = sq.len, Skv = sk.len;
  const int nkb_seq = (Skv + 63) / 64;  // 64-key scale blocks of this sequence
  const int nkv_all = (Skv + C::BN - 1) / C::BN;

  // Key tiles each query tile needs (0 for a tile entirely past seq_q).
  int nkv[QT];
  int nkv_max = 0;
#pragma unroll
  for (int t = 0; t < QT; ++t) {
    const int r0 = (m_cta * QT + t) * C::BM;
    int n = nkv_all;
    if (p.causal) n = min(n, r0 / C::BN + 1);
    if (r0 >= Sq) n = 0;
    nkv[t] = n;
    nkv_max = max(nkv_max, n);
  }

  if (threadIdx.x == 0) {
    mbar_init(bar_q, FQ ? 128 * QT : 1);  // fused Q: every softmax thread arrives
    for (int s = 0; s < C::NS; ++s) {
      mbar_init(bar_kfull + s, 1);
      mbar_init(bar_vfull + s, 1);
      mbar_init(bar_kvempty + s, 1);
    }
    for (int t = 0; t < QT; ++t) {
      mbar_init(bar_sfull + t, 1);
      mbar_init(bar_phalf + t, 128);
      mbar_init(bar_pfull + t, 128);
      mbar_init(bar_odone + t, 1);
      mbar_init(bar_sload + t, 128);
      mbar_init(bar_pvdone + t, 1);
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
  if constexpr (C::PRE_BIAS) {
    uint32_t* bias = reinterpret_cast<uint32_t*>(smem + C::OFF_BIAS);
    for (int i = threadIdx.x; i < 1024; i += C::NUM_THREADS) bias[i] = 0x4B400000u;
    fence_proxy_async_smem();  // visible to tcgen05.cp after the barrier below
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;

  if (warp >= 4 * QT) {
  // ---------------------------------------------------------------- producer / MMA warpgroup
#ifndef SAGE_NO_SETMAXNREG
  regs_dec<C::REGS_OTHER>();
#endif
  if (warp == 4 * QT) {
    // ------------------------------------------------------------ TMA producer
    SAGE_T_DECL
    if (elect_one() && nkv_max > 0) {
      if constexpr (!FQ) {
        mbar_arrive_expect_tx(bar_q, QT * C::Q_TILE);
#pragma unroll
        for (int t = 0; t < QT; ++t)
#pragma unroll
          for (int x = 0; x < C::QK_ATOMS; ++x)
            tma_load_4d(smem + C::OFF_Q + t * C::Q_TILE + x * (C::BM * 128), &tmQ, bar_q, x * C::QK_BOX,
                        sq.base + (m_cta * QT + t) * C::BM, h, sq.batch);
      }
      for (int j = 0; j < nkv_max; ++j) {
        const int s = j % C::NS;
        SAGE_T_MARK(1)
        if (j >= C::NS) {
          if (!mbar_wait(bar_kvempty + s, ((j / C::NS) - 1) & 1, abort_flag, kDevTimeoutProducer, p.wait_limit_ns)) break;
        }
        SAGE_T_MARK(0)
        mbar_arrive_expect_tx(bar_kfull + s, C::K_TILE);
#pragma unroll
        for (int x = 0; x < C::QK_ATOMS; ++x)
          tma_load_4d(smem + C::OFF_K + s * C::K_TILE + x * (C::BN * 128), &tmK, bar_kfull + s, x * C::QK_BOX,
                      sk.base + j * C::BN, hkv, sk.batch);
        mbar_arrive_expect_tx(bar_vfull + s, C::V_TILE);
#pragma unroll
        for (int x = 0; x < C::V_BOXES; ++x)
          tma_load_4d(smem + C::OFF_V + s * C::V_TILE + x * (C::BN * 128), &tmV, bar_vfull + s,
                      x * (128 / C::V_ELT), sk.base + j * C::BN, hkv, sk.batch);
      }
    }
    SAGE_T_FLUSH(blockIdx.x + gridDim.x * (blockIdx.y + gridDim.y * blockIdx.z), warp)
  } else if (warp == 4 * QT + 1) {
    // ------------------------------------------------------------ MMA issuer
    SAGE_T_DECL
    if (elect_one() && nkv_max > 0) {
      const uint32_t q_addr = smem_u32(smem + C::OFF_Q);
      const uint32_t k_addr = smem_u32(smem + C::OFF_K);
      const uint32_t v_addr = smem_u32(smem + C::OFF_V);
      const uint32_t bias_addr = smem_u32(smem + C::OFF_BIAS);
      bool ok = mbar_wait(bar_q, 0, abort_flag, kDevTimeoutMma, p.wait_limit_ns);
      // QK of tile 0 for every query tile.
      if (ok) ok = mbar_wait(bar_kfull, 0, abort_flag, kDevTimeoutMma, p.wait_limit_ns);
      tc_fence_after();
      if (ok) {
#pragma unroll
        for (int t = 0; t < QT; ++t) {
          if (nkv[t] == 0) continue;
          issue_qk<C>(tmem_base + 256 * t, q_addr + t * C::Q_TILE, k_addr, bias_addr);
          umma_commit(bar_sfull + t);
        }
      }
      for (int j = 0; ok && j < nkv_max; ++j) {
        const int s = j % C::NS;
        const int s1 = (j + 1) % C::NS;
        bool v_ready = false, knext_ready = false;
        if constexpr (C::SEP_P) {
          // the next scores first: S_t(j+1) only needs softmax to have read S_t(j)
#pragma unroll
          for (int t = 0; t < QT; ++t) {
            if (j + 1 >= nkv[t]) continue;
            SAGE_T_MARK(4)
            if (!mbar_wait(bar_sload + t, j & 1, abort_flag, kDevTimeoutMma, p.wait_limit_ns)) { ok = false; break; }
            if (!knext_ready) {
              if (!mbar_wait(bar_kfull + s1, ((j + 1) / C::NS) & 1, abort_flag, kDevTimeoutMma, p.wait_limit_ns)) { ok = false; break; }
              knext_ready = true;
            }
            SAGE_T_MARK(3)
            tc_fence_after();
            issue_qk<C>(tmem_base + 256 * t, q_addr + t * C::Q_TILE, k_addr + s1 * C::K_TILE, bias_addr);
            umma_commit(bar_sfull + t);
          }
          if (!ok) break;
        }
#pragma unroll
        for (int t = 0; t < QT; ++t) {
          if (j >= nkv[t]) continue;
          const uint64_t vd = make_smem_desc(v_addr + s * C::V_TILE, C::V_LBO, C::V_SBO, C::V_LAYOUT);
          const uint32_t p_tmem = tmem_base + 256 * t + C::P_COL;
          const uint32_t o_tmem = tmem_base + 256 * t + 128;
          // P.V over the first 64 keys as soon as their P is in TMEM, then the rest
#pragma unroll
          for (int half = 0; half < 2; ++half) {
            SAGE_T_MARK(4)
            if (!mbar_wait((half ? bar_pfull : bar_phalf) + t, j & 1, abort_flag, kDevTimeoutMma, p.wait_limit_ns)) { ok = false; break; }
            SAGE_T_MARK(half)
            if (!v_ready) {
              if (!mbar_wait(bar_vfull + s, (j / C::NS) & 1, abort_flag, kDevTimeoutMma, p.wait_limit_ns)) { ok = false; break; }
              v_ready = true;
              SAGE_T_MARK(2)
            }
            tc_fence_after();
            constexpr int NK = C::BN / C::PV_K;  // MMAs per key tile
#pragma unroll
            for (int kk = half * NK / 2; kk < (half + 1) * NK / 2; ++kk) {
              const uint64_t vdk = desc_advance(vd, kk * C::PV_K * C::V_ATOM_ROW);
              if constexpr (PV == kPvE4M3)
                umma_f8_ts(o_tmem, p_tmem + kk * 8, vdk, C::IDESC_PV, (j > 0 || kk > 0) ? 1u : 0u);
              else
                umma_f16_ts(o_tmem, p_tmem + kk * 8, vdk, C::IDESC_PV, (j > 0 || kk > 0) ? 1u : 0u);
            }
          }
          if (!ok) break;
          if (j + 1 == nkv[t]) umma_commit(bar_odone + t);  // O_t final once this lands
          if constexpr (C::SEP_P) {
            umma_commit(bar_pvdone + t);  // P_t may be rewritten, O_t rescaled, once this lands
          } else if (j + 1 < nkv[t]) {
            if (!knext_ready) {
              SAGE_T_MARK(4)
              if (!mbar_wait(bar_kfull + s1, ((j + 1) / C::NS) & 1, abort_flag, kDevTimeoutMma, p.wait_limit_ns)) { ok = false; break; }
              SAGE_T_MARK(3)
              knext_ready = true;
              tc_fence_after();
            }
            issue_qk<C>(tmem_base + 256 * t, q_addr + t * C::Q_TILE, k_addr + s1 * C::K_TILE, bias_addr);
            umma_commit(bar_sfull + t);
          }
        }
        umma_commit(bar_kvempty + s);  // K_s / V_s reusable once every MMA issued so far is done
      }
    }
    SAGE_T_FLUSH(blockIdx.x + gridDim.x * (blockIdx.y + gridDim.y * blockIdx.z), warp)
  }
  // Leave from this branch (warps of the two kinds run with different register budgets):
  // the MMA warp, which owns TMEM, frees it once every warp has arrived on named barrier 2.
  tc_fence_before();
  if (warp == 4 * QT + 1) {
    asm volatile("bar.sync 2, %0;" ::"n"(C::NUM_THREADS) : "memory");
    tc_fence_after();
    tmem_dealloc(tmem_base, C::TMEM_COLS);
  } else {
    asm volatile("bar.arrive 2, %0;" ::"n"(C::NUM_THREADS) : "memory");
  }
  } else {
    // ------------------------------------------------------------ softmax warpgroups
#ifndef SAGE_NO_SETMAXNREG
    regs_inc<C::REGS_SOFTMAX>();
#endif
    const int t = warp / 4;
    const int row_in_tile = (warp % 4) * 32 + lane;
    const int r0 = (m_cta * QT + t) * C::BM;
    const int row = r0 + row_in_tile;
    const uint32_t lane_base = ((warp % 4) * 32u) << 16;
    const uint32_t s_tmem = tmem_base + lane_base + 256 * t;
    const uint32_t o_tmem = s_tmem + 128;
    const int n = nkv[t];
    float qs;
    if constexpr (FQ) {
      static_assert(!FLASH && QT == 2, "fused Q quantisation: INT8 path, two query tiles");
      if (p.qblk_shift == 7)
        qs = fused_q_tile<C, D, OBF16>(p, smem + C::OFF_Q + t * C::Q_TILE,
                                       reinterpret_cast<float*>(smem + C::OFF_QRED) + 4 * t, t, row_in_tile, sq, b,
                                       h, r0 / C::BM, bar_q);
      else
        qs = fused_q_tile_fine<C, D, OBF16>(p, smem + C::OFF_Q + t * C::Q_TILE,
                                            reinterpret_cast<float*>(smem + C::OFF_QFINE + t * C::QFINE_BYTES), t,
                                            row_in_tile, sq, b, h, r0 / C::BM, bar_q, row_in_tile);
    } else {
      // this thread's query row's scale (rows past the sequence end use the last row's block)
      qs = (!FLASH && n > 0) ? p.q_scale[((size_t)b * p.Hq + h) * p.nqb + (min(row, Sq - 1) >> p.qblk_shift)]
                             : 0.0f;
    }
    const float* ksp = FLASH ? nullptr : p.k_scale + ((size_t)b * p.Hkv + hkv) * p.nkb;
    float m_run = -INFINITY, l_run = 0.0f;
    bool ok = true;
    SAGE_T_DECL
    // INT8 scores are biased: 1.5 * 2^23 has bit pattern 0x4B400000, and 0x4B400000 + s is the
    // float 1.5 * 2^23 + s for |s| < 2^22. fp32 scores (FLASH, C16) are used as they are.
    constexpr float kMagic = C::QK_F16 ? 0.0f : 12582912.0f;
    // D = 128: the two K block scales of tile j+1 are loaded during iteration j, so the loads
    // are in flight while tile j+1's scores are computed (H8K 1.681 -> 1.655 ms). At D = 64 the
    // same change made s8k_d64 4 % slower, so there they are loaded where they are used.
    constexpr bool KS_AHEAD = !FLASH && D == 128;
    float ks_next0 = 0.0f, ks_next1 = 0.0f;
    if constexpr (KS_AHEAD) {
      if (n > 0) {
        ks_next0 = ksp[0];
        ks_next1 = (1 < nkb_seq) ? ksp[1] : ks_next0;
      }
    }
    for (int j = 0; j < n; ++j) {
      const float ks0 = ks_next0, ks1 = ks_next1;
      if constexpr (KS_AHEAD) {
        if (j + 1 < n) {
          ks_next0 = ksp[2 * j + 2];
          ks_next1 = (2 * j + 3 < nkb_seq) ? ksp[2 * j + 3] : ks_next0;
        }
      }
      SAGE_T_MARK(5)
      if (!__all_sync(0xffffffffu, mbar_wait(bar_sfull + t, j & 1, abort_flag, kDevTimeoutSoftmax, p.wait_limit_ns))) { ok = false; break; }
      tc_fence_after();
      SAGE_T_MARK(0)
      float b[128];
      {
        uint32_t sr[128];
        tmem_ld128_sync(s_tmem, sr);
        if constexpr (C::SEP_P) {
          tc_fence_before();
          mbar_arrive(bar_sload + t);  // S_t(j) is in registers: QK_t(j+1) may overwrite it
        }
        // int32 score s -> float 12582912 + s exactly (an integer add instead of a conversion);
        // monotone in s, so maxima can be taken on these biased values.
#pragma unroll
        for (int c = 0; c < 128; ++c) b[c] = __uint_as_float((C::QK_F16 || C::PRE_BIAS) ? sr[c] : sr[c] + 0x4B400000u);
      }
      SAGE_T_MARK(1)
      const int key0 = j * C::BN;
      if ((key0 + C::BN > Skv) || (p.causal && key0 + C::BN - 1 > r0)) {
        const int lim = (p.causal ? min(Skv, row + 1) : Skv) - key0;  // visible keys: [0, lim)
#pragma unroll
        for (int c = 0; c < 128; ++c)
          if (c >= lim) b[c] = -INFINITY;
      }
      // maxima of the two 64-key halves (one k_scale each), short dependency chains
      float hm[2];
#pragma unroll
      for (int h2 = 0; h2 < 2; ++h2) {
        float a[8];
#pragma unroll
        for (int i = 0; i < 8; ++i) {
          const float* v = b + h2 * 64 + i;
          a[i] = fmaxf(fmax3(fmax3(v[0], v[8], v[16]), v[24], v[32]), fmax3(v[40], v[48], v[56]));
        }
        hm[h2] = fmax3(fmax3(a[0], a[1], a[2]), fmax3(a[3], a[4], a[5]), fmaxf(a[6], a[7]));
      }
      // a zero scale (all-zero block) is replaced by FLT_MIN: its scores are exactly 0 either
      // way, and masked -inf entries stay -inf instead of becoming NaN
      float sc0, sc1;
      if constexpr (FLASH) {
        sc0 = sc1 = p.qk_scale;
      } else if constexpr (KS_AHEAD) {
        sc0 = fmaxf(qs * ks0, 1.17549435e-38f);
        sc1 = fmaxf(qs * ks1, 1.17549435e-38f);
      } else {
        const int kb0 = 2 * j;
        sc0 = fmaxf(qs * ksp[kb0], 1.17549435e-38f);
        sc1 = (kb0 + 1 < nkb_seq) ? fmaxf(qs * ksp[kb0 + 1], 1.17549435e-38f) : sc0;
      }
      const float tmax = fmaxf((hm[0] - kMagic) * sc0, (hm[1] - kMagic) * sc1);
      const bool upd = tmax > m_run + C::LAZY;
      const float m_new = upd ? tmax : m_run;
      const float alpha = upd ? ex2_approx(m_run - m_new) : 1.0f;
      const bool rescale = j > 0 && __any_sync(0xffffffffu, upd);
      SAGE_T_MARK(2)
      const float m_use = (m_new == -INFINITY) ? 0.0f : m_new;
      // exponent argument = s*sc - m = b*sc - (12582912*sc + m): one packed FMA per two scores
      const float cc0 = -fmaf(kMagic, sc0, m_use - C::P_SHIFT);
      const float cc1 = -fmaf(kMagic, sc1, m_use - C::P_SHIFT);
      float2 acc[4] = {make_float2(0.f, 0.f), make_float2(0.f, 0.f), make_float2(0.f, 0.f), make_float2(0.f, 0.f)};
#pragma unroll
      for (int h2 = 0; h2 < 2; ++h2) {
        const float2 scv = h2 ? make_float2(sc1, sc1) : make_float2(sc0, sc0);
        const float2 ccv = h2 ? make_float2(cc1, cc1) : make_float2(cc0, cc0);
        constexpr int NW = (PV == kPvE4M3) ? 16 : 32;  // packed P words per 64 keys
        uint32_t pk[NW];
#pragma unroll
        for (int pr = 0; pr < 32; ++pr) {
          const int c = h2 * 64 + 2 * pr;
          const float2 a = ffma2(make_float2(b[c], b[c + 1]), scv, ccv);
          float2 e;
          if ((c % 32) >= 32 - C::EMU) {
            e = exp2_poly2(a);
          } else {
            e.x = ex2_approx(a.x);
            e.y = ex2_approx(a.y);
          }
          acc[pr & 3] = fadd2(acc[pr & 3], e);
          if constexpr (PV == kPvE4M3) {
            const uint32_t w = __nv_cvt_float2_to_fp8x2(e, __NV_SATFINITE, __NV_E4M3);
            if (pr & 1) pk[pr >> 1] |= w << 16; else pk[pr >> 1] = w;
          } else if constexpr (PV == kPvBF16) {
            __nv_bfloat162 v2 = __floats2bfloat162_rn(e.x, e.y);
            pk[pr] = *reinterpret_cast<uint32_t*>(&v2);
          } else {
            __half2 v2 = __floats2half2_rn(e.x, e.y);
            pk[pr] = *reinterpret_cast<uint32_t*>(&v2);
          }
        }
        if (h2 == 1) {
          // Release the first half of P (stored before these exponentials were computed, so
          // its TMEM store has completed in their shadow) and the rescaled O.
          tmem_st_wait();
          tc_fence_before();
          mbar_arrive(bar_phalf + t);
        } else if (C::SEP_P && j > 0) {
          // P_t(j-1) must have been read and O_t(j-1) accumulated before P_t(j) / the rescale
          if (!__all_sync(0xffffffffu, mbar_wait(bar_pvdone + t, (j - 1) & 1, abort_flag, kDevTimeoutSoftmax, p.wait_limit_ns))) { ok = false; break; }
          tc_fence_after();
        }
        // P over the upper columns of S_t (the whole S row is already in registers)
        if constexpr (PV == kPvE4M3)
          tmem_st16(s_tmem + C::P_COL + 16 * h2, pk);
        else
          tmem_st32(s_tmem + C::P_COL + 32 * h2, *reinterpret_cast<uint32_t(*)[32]>(&pk[0]));
        if (h2 == 0 && rescale) {
          // O_t *= alpha before any P.V of this tile is released. PV_t(j-1) has completed:
          // S_t(j) was issued after it and tcgen05 operations complete in order (D = 128), or
          // pvdone said so above (D = 64).
#pragma unroll
          for (int c0 = 0; c0 < D; c0 += 32) {
            uint32_t orow[32];
            tmem_ld32_sync(o_tmem + c0, orow);
#pragma unroll
            for (int c = 0; c < 32; ++c) orow[c] = __float_as_uint(__uint_as_float(orow[c]) * alpha);
            tmem_st32(o_tmem + c0, orow);
          }
        }
        SAGE_T_MARK(3 + h2)
      }
      if (!ok) break;  // a wait inside the loop above gave up
      tmem_st_wait();
      tc_fence_before();
      mbar_arrive(bar_pfull + t);
      const float2 s01 = fadd2(fadd2(acc[0], acc[1]), fadd2(acc[2], acc[3]));
      l_run = fmaf(l_run, alpha, s01.x + s01.y);
      m_run = m_new;
    }
    SAGE_T_MARK(5)
    // ---------------------------------------------------------- epilogue
    // O = acc / l in the output type. Into this GPU's own memory each thread stores its row
    // directly. Into other memory (p.o_stage: a peer-mapped output of a multi-GPU gather) each
    // half of the tile (64 rows, two warps' TMEM lanes) goes through shared memory and out with
    // whole-line stores: thread i writes 16-byte piece i of the half's rows, so a warp's store
    // covers 512 contiguous bytes of a head's rows instead of 32 rows' separate pieces, which
    // NVLink carries far more efficiently. Row r's 16-byte piece c sits in the stage at piece
    // c ^ (r mod PR) (PR pieces per row) against bank conflicts. On that path all four warps of
    // the warpgroup execute every barrier, and whether the tile stores anything is one
    // warpgroup-wide decision (bar.red.and), so a warp whose wait gave up cannot leave the
    // others waiting.
    const bool valid = row < Sq;
    const int64_t o_row0 = (int64_t)sq.batch * p.o_sb + (int64_t)h * p.o_sh + (int64_t)(sq.base + r0) * p.o_ss;
    char* orow_ptr = reinterpret_cast<char*>(p.o) + (o_row0 + (int64_t)row_in_tile * p.o_ss) * 2;
    const float inv_l = 1.0f / l_run;
    const float* vsp = p.v_scale + ((size_t)b * p.Hkv + hkv) * D;
    // output columns [c0, c0 + 32) of this thread's row, scaled and packed to 16-bit pairs
    auto out32 = [&](int c0, uint32_t (&packed)[16]) {
      uint32_t orow[32];
      tmem_ld32_sync(o_tmem + c0, orow);
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
    };
    if (n > 0 && p.o_stage) {  // uniform over the warpgroup
      const bool mine = ok && __all_sync(0xffffffffu, mbar_wait(bar_odone + t, 0, abort_flag, kDevTimeoutEpilogue,
                                                               p.wait_limit_ns));
      const bool store = warpgroup_and(t, mine);
      tc_fence_after();
      constexpr int PR = D / 8;  // 16-byte pieces per output row
      uint4* stage = reinterpret_cast<uint4*>(smem + C::OFF_OST + t * C::OST_BYTES);
#pragma unroll
      for (int half = 0; half < 2; ++half) {
        if (store && (warp % 4) / 2 == half) {
          const int lr = row_in_tile - 64 * half;
#pragma unroll
          for (int c0 = 0; c0 < D; c0 += 32) {
            uint32_t packed[16];
            out32(c0, packed);
#pragma unroll
            for (int v = 0; v < 4; ++v) {
              const int piece = c0 / 8 + v;
              stage[lr * PR + (piece ^ (lr % PR))] =
                  make_uint4(packed[4 * v], packed[4 * v + 1], packed[4 * v + 2], packed[4 * v + 3]);
            }
          }
        }
        warpgroup_sync(t);
        if (store) {
#pragma unroll
          for (int i = 0; i < 64 * PR / 128; ++i) {
            const int idx = i * 128 + row_in_tile;
            const int lr = idx / PR, piece = idx % PR, r = 64 * half + lr;
            if (r0 + r < Sq)
              *reinterpret_cast<uint4*>(reinterpret_cast<char*>(p.o) + (o_row0 + (int64_t)r * p.o_ss) * 2 + piece * 16) =
                  stage[lr * PR + (piece ^ (lr % PR))];
          }
        }
        warpgroup_sync(t);  // the stage is free for the next half
      }
    } else if (ok && n > 0 &&
               __all_sync(0xffffffffu, mbar_wait(bar_odone + t, 0, abort_flag, kDevTimeoutEpilogue, p.wait_limit_ns))) {
      tc_fence_after();
#pragma unroll
      for (int c0 = 0; c0 < D; c0 += 32) {
        uint32_t packed[16];
        out32(c0, packed);
        if (valid) {
          uint4* dst = reinterpret_cast<uint4*>(orow_ptr + c0 * 2);
#pragma unroll
          for (int v = 0; v < 4; ++v)
            dst[v] = make_uint4(packed[4 * v], packed[4 * v + 1], packed[4 * v + 2], packed[4 * v + 3]);
        }
      }
    } else if (Skv == 0 && valid) {
      // a sequence without keys (variable-length batches): the reference's matmuls over an
      // empty key axis give O = 0
      uint4* dst = reinterpret_cast<uint4*>(orow_ptr);
#pragma unroll
      for (int v = 0; v < D / 8; ++v) dst[v] = make_uint4(0u, 0u, 0u, 0u);
    }
    SAGE_T_MARK(6)
    SAGE_T_FLUSH(blockIdx.x + gridDim.x * (blockIdx.y + gridDim.y * blockIdx.z), warp)
    tc_fence_before();
    asm volatile("bar.arrive 2, %0;" ::"n"(C::NUM_THREADS) : "memory");
  }
}

}  // namespace sage
