// sage_abi.cu — the C ABI of libsage_sm100.so (declared in include/sage_sm100.h): argument
// validation, TMA descriptor encoding, kernel launches and error reporting. This is the
// single translation unit of the library; the kernels live in the included .cuh files.
#include <cuda.h>
#include <cuda_runtime.h>
#include <cudaTypedefs.h>

#include <algorithm>
#include <cstdarg>
#include <cstdio>
#include <cmath>
#include <cstdlib>
#include <cstring>
#include <map>
#include <mutex>
#include <string>

#include "../../include/sage_sm100.h"
#include "sage_attn.cuh"
#include "sage_quant.cuh"

namespace {

thread_local std::string g_last_error;

int fail(int code, const char* fmt, ...) {
  char buf[512];
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(buf, sizeof(buf), fmt, ap);
  va_end(ap);
  g_last_error = buf;
  return code;
}

#define SAGE_CUDA_TRY(expr)                                                               \
  do {                                                                                    \
    cudaError_t e_ = (expr);                                                              \
    if (e_ != cudaSuccess)                                                                \
      return fail(SAGE_ERR_CUDA, "%s failed: %s", #expr, cudaGetErrorString(e_));         \
  } while (0)

constexpr int kMaxDevices = 64;
std::mutex g_mutex;
int g_arch_ok[kMaxDevices];  // 0 unknown, 1 sm_100, -1 other
PFN_cuTensorMapEncodeTiled_v12000 g_encode = nullptr;

int current_device(int* dev) {
  SAGE_CUDA_TRY(cudaGetDevice(dev));
  if (*dev < 0 || *dev >= kMaxDevices) return fail(SAGE_ERR_CUDA, "device ordinal %d out of range", *dev);
  return SAGE_OK;
}

int check_arch() {
  int dev = 0;
  if (int rc = current_device(&dev)) return rc;
  std::lock_guard<std::mutex> lk(g_mutex);
  if (g_arch_ok[dev] == 0) {
    int major = 0, minor = 0;
    SAGE_CUDA_TRY(cudaDeviceGetAttribute(&major, cudaDevAttrComputeCapabilityMajor, dev));
    SAGE_CUDA_TRY(cudaDeviceGetAttribute(&minor, cudaDevAttrComputeCapabilityMinor, dev));
    g_arch_ok[dev] = (major == 10 && minor == 0) ? 1 : -1;
    if (g_arch_ok[dev] < 0)
      return fail(SAGE_ERR_UNSUPPORTED_ARCH, "device %d is sm_%d%d; libsage_sm100 needs sm_100", dev, major, minor);
  }
  if (g_arch_ok[dev] < 0) return fail(SAGE_ERR_UNSUPPORTED_ARCH, "device %d is not sm_100", dev);
  if (!g_encode) {
    void* fn = nullptr;
    cudaDriverEntryPointQueryResult q;
    SAGE_CUDA_TRY(cudaGetDriverEntryPointByVersion("cuTensorMapEncodeTiled", &fn, 12000, cudaEnableDefault, &q));
    if (q != cudaDriverEntryPointSuccess || !fn)
      return fail(SAGE_ERR_CUDA, "cuTensorMapEncodeTiled not available from the driver");
    g_encode = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(fn);
  }
  return SAGE_OK;
}

// Raise the dynamic shared-memory limit of `func` once per (device, kernel).
std::map<std::pair<const void*, int>, int> g_smem_set;

int ensure_smem(const void* func, int bytes) {
  int dev = 0;
  if (int rc = current_device(&dev)) return rc;
  std::lock_guard<std::mutex> lk(g_mutex);
  int& cur = g_smem_set[{func, dev}];
  if (cur != bytes) {
    SAGE_CUDA_TRY(cudaFuncSetAttribute(func, cudaFuncAttributeMaxDynamicSharedMemorySize, bytes));
    cur = bytes;
  }
  return SAGE_OK;
}

bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

int check_strides(const char* name, const int64_t s[3]) {
  if (!s) return fail(SAGE_ERR_INVALID_ARG, "%s strides are NULL", name);
  for (int i = 0; i < 3; ++i)
    if (s[i] <= 0 || (s[i] % 8) != 0)
      return fail(SAGE_ERR_INVALID_ARG, "%s stride[%d]=%lld must be a positive multiple of 8 elements", name, i,
                  (long long)s[i]);
  return SAGE_OK;
}

int check_shape(int dtype, int64_t B, int64_t Hq, int64_t Hkv, int64_t Sq, int64_t Skv, int64_t D) {
  if (dtype != SAGE_DTYPE_F16 && dtype != SAGE_DTYPE_BF16)
    return fail(SAGE_ERR_INVALID_ARG, "dtype %d is neither SAGE_DTYPE_F16 nor SAGE_DTYPE_BF16", dtype);
  if (D != 64 && D != 128) return fail(SAGE_ERR_INVALID_ARG, "head_dim %lld unsupported (64 or 128)", (long long)D);
  if (B <= 0 || Hq <= 0 || Hkv <= 0 || Sq <= 0 || Skv <= 0)
    return fail(SAGE_ERR_INVALID_ARG, "empty or negative shape B=%lld Hq=%lld Hkv=%lld Sq=%lld Skv=%lld",
                (long long)B, (long long)Hq, (long long)Hkv, (long long)Sq, (long long)Skv);
  if (Hq % Hkv != 0)
    return fail(SAGE_ERR_INVALID_ARG, "heads_q=%lld is not a multiple of heads_kv=%lld", (long long)Hq, (long long)Hkv);
  if (B > 65535 || Hq > 65535 || Sq > (1LL << 30) || Skv > (1LL << 30))
    return fail(SAGE_ERR_INVALID_ARG, "shape exceeds launch limits");
  return SAGE_OK;
}

int64_t cdiv(int64_t a, int64_t b) { return (a + b - 1) / b; }

// Rows per Q scale block from the SAGE_FLAG_QBLK_* field of `flags` (per_block_int8's BLKQ).
int qblk_from_flags(unsigned flags, int* rows) {
  static const int kRows[8] = {128, 64, 32, 16, 1, 0, 0, 0};
  *rows = kRows[(flags & SAGE_FLAG_QBLK_MASK) >> 8];
  if (!*rows) return fail(SAGE_ERR_INVALID_ARG, "Q block field 0x%x of flags is not a SAGE_FLAG_QBLK_* value",
                          flags & SAGE_FLAG_QBLK_MASK);
  return SAGE_OK;
}
int qblk_shift(int rows) { return rows == 1 ? 0 : rows == 16 ? 4 : rows == 32 ? 5 : rows == 64 ? 6 : 7; }
// Rows per Q block of flags that passed qblk_from_flags.
int qblk_of(unsigned flags) {
  int rows = 128;
  qblk_from_flags(flags, &rows);
  return rows;
}
// The attention-only entry points take the Q block field and nothing else.
int check_attn_flags(unsigned flags, int* rows) {
  if (flags & ~SAGE_FLAG_QBLK_MASK)
    return fail(SAGE_ERR_INVALID_ARG, "flags 0x%x: the attention entry points take only SAGE_FLAG_QBLK_*", flags);
  return qblk_from_flags(flags, rows);
}

// ---------------------------------------------------------------- output aliasing
// Byte range [lo, hi) a buffer covers. A strided [B, H, S, D] tensor (element strides {batch,
// head, seq}, D contiguous) covers everything between its first and its last element.
struct Span {
  uintptr_t lo = 0, hi = 0;
};
Span buffer_span(const void* p, size_t bytes) {
  const uintptr_t lo = reinterpret_cast<uintptr_t>(p);
  return p ? Span{lo, lo + bytes} : Span{};
}
Span tensor_span(const void* p, const int64_t* s, int64_t B, int64_t H, int64_t S, int64_t D, int elt) {
  if (!p || !s) return Span{};
  const int64_t last = (B - 1) * s[0] + (H - 1) * s[1] + (S - 1) * s[2] + D;  // elements
  return buffer_span(p, static_cast<size_t>(last) * static_cast<size_t>(elt));
}
bool spans_overlap(const Span& a, const Span& b) { return a.lo < a.hi && b.lo < b.hi && a.lo < b.hi && b.lo < a.hi; }
struct NamedSpan {
  const char* name;
  Span span;
};

// The output o is written while the call still reads its other operands (another CTA's K/V
// tiles, the intermediates, and on the head_dim-64 route of sage_run Q's codes parked in o
// itself), so o must not share a byte with any of them. The one permitted overlap is o = q as
// the identical view (same base and strides): every CTA reads its own query rows before it
// writes the same rows of o. The check compares byte ranges, so it is conservative: o
// interleaved with k or v inside one packed buffer is rejected too.
int check_out_alias(const void* o, const int64_t* os, const Span& o_span, const void* q, const int64_t* qs,
                    const Span& q_span, const NamedSpan* others, int n_others) {
  if (spans_overlap(o_span, q_span)) {
    const bool same_view = o == q && os && qs && os[0] == qs[0] && os[1] == qs[1] && os[2] == qs[2];
    if (!same_view)
      return fail(SAGE_ERR_INVALID_ARG,
                  "o overlaps q without being the same view (same base pointer and strides): the result "
                  "would be corrupted");
  }
  for (int i = 0; i < n_others; ++i)
    if (spans_overlap(o_span, others[i].span))
      return fail(SAGE_ERR_INVALID_ARG, "o overlaps %s: the result would be corrupted", others[i].name);
  return SAGE_OK;
}

// check_out_alias over everything an attention call reads: q (identical view allowed), k, v
// and the caller's intermediates (NULL ones are skipped). q_rows / k_rows = rows of the token
// axis summed over the batch (dense: B * S; packed sequences: the token counts); nqb / nkb =
// scale blocks per (batch, head).
int check_attn_alias(const void* o, const int64_t* os, const Span& o_span, const void* q, const int64_t* qs,
                     const Span& q_span, const Span& k_span, const Span& v_span, int64_t B, int64_t Hq, int64_t Hkv,
                     int64_t q_rows, int64_t k_rows, int64_t nqb, int64_t nkb, int64_t D, const void* q_i8,
                     const void* q_scale, const void* k_i8, const void* k_scale, const void* k_mean,
                     const void* v_fp8, const void* v_scale, const void* ws, size_t ws_bytes) {
  const size_t f4 = sizeof(float);
  const NamedSpan others[] = {
      {"k", k_span},
      {"v", v_span},
      {"q_i8", buffer_span(q_i8, static_cast<size_t>(Hq * q_rows * D))},
      {"q_scale", buffer_span(q_scale, static_cast<size_t>(B * Hq * nqb) * f4)},
      {"k_i8", buffer_span(k_i8, static_cast<size_t>(Hkv * k_rows * D))},
      {"k_scale", buffer_span(k_scale, static_cast<size_t>(B * Hkv * nkb) * f4)},
      {"k_mean", buffer_span(k_mean, static_cast<size_t>(B * Hkv * D) * f4)},
      {"v_fp8", buffer_span(v_fp8, static_cast<size_t>(Hkv * k_rows * D))},
      {"v_scale", buffer_span(v_scale, static_cast<size_t>(B * Hkv * D) * f4)},
      {"workspace", buffer_span(ws, ws_bytes)},
  };
  return check_out_alias(o, os, o_span, q, qs, q_span, others, static_cast<int>(sizeof(others) / sizeof(others[0])));
}

size_t ws_ksum_bytes(int64_t B, int64_t Hkv, int64_t Skv, int64_t D) {
  return static_cast<size_t>(B * Hkv * cdiv(Skv, sage::kStatsChunk) * D) * sizeof(double);
}
size_t ws_vmax_bytes(int64_t B, int64_t Hkv, int64_t Skv, int64_t D) {
  return static_cast<size_t>(B * Hkv * cdiv(Skv, sage::kStatsChunk) * D) * sizeof(float);
}
size_t align256(size_t x) { return (x + 255) & ~size_t(255); }

// Variable-length batches: the device prefix sums of sequence lengths and the token rows of the
// packed tensors. A null Varlen* means dense [B, H, S, D] tensors.
struct Varlen {
  const int* cu_q;
  const int* cu_k;
  int64_t q_tokens, k_tokens;
};

// INT8 codes held as fp16 values (the head_dim-64 route of sage_run): Q's in a tensor with
// {batch, head, seq} strides qs, K's in k_i8's layout (contiguous, or [Hkv, tokens, D] packed).
struct Codes16 {
  __half* q;
  const int64_t* qs;
  __half* k;
};

// Workspace of the statistics (K column sums, V absmax) and, for sage_run's fp16-code route,
// of K's fp16 codes after them.
size_t stats_ws_bytes(int64_t B, int64_t Hkv, int64_t Skv, int64_t D, int pv_mode, unsigned flags) {
  if (B <= 0 || Hkv <= 0 || Skv <= 0 || D <= 0) return 0;
  size_t n = 0;
  const bool smooth = (flags & SAGE_FLAG_SMOOTH_K) != 0;
  const bool fp8 = pv_mode == SAGE_PV_FP8;
  if (smooth || fp8) n += align256(ws_ksum_bytes(B, Hkv, Skv, D));
  if (fp8) n += align256(ws_vmax_bytes(B, Hkv, Skv, D));
  return n;
}
size_t codes_ws_bytes(int64_t B, int64_t Hkv, int64_t Skv, int64_t D) {
  return align256(static_cast<size_t>(B * Hkv * Skv * D) * sizeof(__half));
}
// sage_run's route at head_dim 64: INT8 codes as fp16 values and a kind::f16 QK^T, unless a
// flag asks for the INT8 operands (SAGE_FLAG_PREPASS_Q) or Q quantised in the kernel
// (SAGE_FLAG_FUSED_Q, whose codes are INT8).
bool c16_route(unsigned flags, int64_t head_dim) {
  return head_dim == 64 && !(flags & (SAGE_FLAG_PREPASS_Q | SAGE_FLAG_FUSED_Q));
}

int encode_4d(CUtensorMap* map, CUtensorMapDataType dt, int elt_bytes, const void* base, int64_t d0, int64_t d1,
              int64_t d2, int64_t d3, int64_t s1, int64_t s2, int64_t s3, uint32_t box0, uint32_t box1,
              CUtensorMapSwizzle sw) {
  cuuint64_t dims[4] = {(cuuint64_t)d0, (cuuint64_t)d1, (cuuint64_t)d2, (cuuint64_t)d3};
  cuuint64_t strides[3] = {(cuuint64_t)(s1 * elt_bytes), (cuuint64_t)(s2 * elt_bytes), (cuuint64_t)(s3 * elt_bytes)};
  cuuint32_t box[4] = {box0, box1, 1, 1};
  cuuint32_t estr[4] = {1, 1, 1, 1};
  CUresult r = g_encode(map, dt, 4, const_cast<void*>(base), dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
                        sw, CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) return fail(SAGE_ERR_CUDA, "cuTensorMapEncodeTiled failed (CUresult %d)", (int)r);
  return SAGE_OK;
}

// Wall-time limit of every device-side mbarrier wait: 2 s, or SAGE_WAIT_LIMIT_MS if set.
unsigned long long wait_limit_ns() {
  static const unsigned long long v = [] {
    const char* e = std::getenv("SAGE_WAIT_LIMIT_MS");
    const long long ms = e ? std::atoll(e) : 0;
    return ms > 0 ? static_cast<unsigned long long>(ms) * 1000000ull : 2000000000ull;
  }();
  return v;
}

// ---------------------------------------------------------------- pre-pass launches
// The four instantiations: dense or packed sequences, INT8 or (head_dim 64 only) fp16 codes.
template <int D, typename T>
void launch_prepass_kernel(const sage::PrepassParams& p, int64_t grid, bool packed, bool c16, cudaStream_t st) {
  const dim3 g((unsigned)grid);
  if constexpr (D == 64) {
    if (c16) {
      if (packed) sage::prepass_kernel<D, T, true, true><<<g, sage::kQuantThreads, 0, st>>>(p);
      else sage::prepass_kernel<D, T, false, true><<<g, sage::kQuantThreads, 0, st>>>(p);
      return;
    }
  }
  if (packed) sage::prepass_kernel<D, T, true><<<g, sage::kQuantThreads, 0, st>>>(p);
  else sage::prepass_kernel<D, T, false><<<g, sage::kQuantThreads, 0, st>>>(p);
}

// K quantisation alone (launch B without V blocks): the 128-thread kernel.
template <int D, typename T>
void launch_kquant_kernel(const sage::PrepassParams& p, bool packed, bool c16, cudaStream_t st) {
  const dim3 g((unsigned)p.n_k);
  if constexpr (D == 64) {
    if (c16) {
      if (packed) sage::kquant_kernel<D, T, true, true><<<g, sage::kKQuantThreads, 0, st>>>(p);
      else sage::kquant_kernel<D, T, false, true><<<g, sage::kKQuantThreads, 0, st>>>(p);
      return;
    }
  }
  if (packed) sage::kquant_kernel<D, T, true, false><<<g, sage::kKQuantThreads, 0, st>>>(p);
  else sage::kquant_kernel<D, T, false, false><<<g, sage::kKQuantThreads, 0, st>>>(p);
}

// Q quantisation alone at head_dim 64: the 128-thread kernel, one block per CTA.
template <typename T>
void launch_qquant_kernel(const sage::PrepassParams& p, bool packed, bool c16, cudaStream_t st) {
  const dim3 g((unsigned)p.n_q);
  if (c16) {
    if (packed) sage::qquant_kernel<T, true, true><<<g, sage::kKQuantThreads, 0, st>>>(p);
    else sage::qquant_kernel<T, false, true><<<g, sage::kKQuantThreads, 0, st>>>(p);
  } else {
    if (packed) sage::qquant_kernel<T, true, false><<<g, sage::kKQuantThreads, 0, st>>>(p);
    else sage::qquant_kernel<T, false, false><<<g, sage::kKQuantThreads, 0, st>>>(p);
  }
}

// Q quantisation with blocks finer than 128 rows (SAGE_FLAG_QBLK_*): one 128-row CTA each.
template <int D, typename T>
void launch_qquant_fine_kernel(const sage::PrepassParams& p, bool packed, bool c16, cudaStream_t st) {
  const dim3 g((unsigned)p.n_q);
  if constexpr (D == 64) {
    if (c16) {
      if (packed) sage::qquant_fine_kernel<D, T, true, true><<<g, sage::kKQuantThreads, 0, st>>>(p);
      else sage::qquant_fine_kernel<D, T, false, true><<<g, sage::kKQuantThreads, 0, st>>>(p);
      return;
    }
  }
  if (packed) sage::qquant_fine_kernel<D, T, true, false><<<g, sage::kKQuantThreads, 0, st>>>(p);
  else sage::qquant_fine_kernel<D, T, false, false><<<g, sage::kKQuantThreads, 0, st>>>(p);
}

template <int D, typename T>
int launch_prepass(const void* q, const void* k, const void* v, int64_t B, int64_t Hq, int64_t Hkv, int64_t Sq,
                   int64_t Skv, const int64_t* qs, const int64_t* ks, const int64_t* vs, float q_mult, bool smooth,
                   bool km_given, int8_t* q_i8, float* q_scale, int8_t* k_i8, float* k_scale, float* k_mean,
                   uint8_t* v_fp8, float* v_scale, void* ws, const Varlen* vl, const Codes16* c16,
                   cudaStream_t st, int qblk) {
  const int nchunk = static_cast<int>(cdiv(Skv, sage::kStatsChunk));
  const bool want_v = v_fp8 != nullptr;
  const bool want_km = smooth && !km_given && k != nullptr;
  sage::PrepassParams p{};
  p.q = q; p.k = k; p.v = want_v ? v : nullptr;
  if (q) { p.q_sb = qs[0]; p.q_sh = qs[1]; p.q_ss = qs[2]; }
  if (k) { p.k_sb = ks[0]; p.k_sh = ks[1]; p.k_ss = ks[2]; }
  if (want_v) { p.v_sb = vs[0]; p.v_sh = vs[1]; p.v_ss = vs[2]; }
  p.q_i8 = q_i8; p.q_scale = q_scale; p.k_i8 = k_i8; p.k_scale = k_scale;
  p.k_mean = smooth ? k_mean : nullptr;
  p.v_fp8 = v_fp8; p.v_scale = v_scale;
  p.q_mult = q_mult;
  p.B = (int)B; p.Hq = (int)Hq; p.Hkv = (int)Hkv; p.Sq = (int)Sq; p.Skv = (int)Skv;
  if (vl) { p.cu_q = vl->cu_q; p.cu_k = vl->cu_k; p.q_tokens = (int)vl->q_tokens; p.k_tokens = (int)vl->k_tokens; }
  if (c16) {
    if (D != 64) return fail(SAGE_ERR_INVALID_ARG, "fp16 codes are the head_dim-64 route");
    p.q_c16 = c16->q; p.k_c16 = c16->k;
    if (c16->qs) { p.qc_sb = vl ? 0 : c16->qs[0]; p.qc_sh = c16->qs[1]; p.qc_ss = c16->qs[2]; }
  }
  p.qblk = qblk;
  p.nqb = (int)cdiv(Sq, qblk); p.nkb = (int)cdiv(Skv, 64); p.nvb = (int)cdiv(Skv, sage::kVRowsPerCta<D>); p.nchunk = nchunk;
  const int64_t n_q = q ? B * Hq * cdiv(p.nqb, sage::kQBlocksPerCta<D>) : 0;
  const int64_t n_k = k ? B * Hkv * cdiv(p.nkb, sage::kKBlocksPerCta<D>) : 0;
  const int64_t n_v = want_v ? B * Hkv * p.nvb : 0;
  const bool need_stats = want_km || want_v;
  const int64_t n_stat = need_stats ? B * Hkv * nchunk : 0;
  if (n_q + n_k + n_v + n_stat > 0x7fffffffLL) return fail(SAGE_ERR_INVALID_ARG, "too many quantisation blocks");
  if (need_stats) {
    char* w = static_cast<char*>(ws);
    p.ksum_part = want_km ? reinterpret_cast<double*>(w) : nullptr;
    p.vmax_part = want_v ? reinterpret_cast<float*>(w + align256(ws_ksum_bytes(B, Hkv, Skv, D))) : nullptr;
    p.stat_k = want_km ? 1 : 0;
    p.stat_v = want_v ? 1 : 0;
  }
  // Q blocks finer than 128 rows: their own 128-thread launch (qquant_fine_kernel) at either
  // head_dim, before the statistics
  bool q_done = false;
  if (n_q > 0 && qblk != 128) {
    p.n_q = (int)(B * Hq * cdiv(Sq, 128));
    p.n_stat = p.n_k = p.n_v = 0;
    launch_qquant_fine_kernel<D, T>(p, vl != nullptr, c16 != nullptr, st);
    SAGE_CUDA_TRY(cudaGetLastError());
    q_done = true;
  }
  // Q blocks at head_dim 64 in their own 128-thread launch (every Q block the pre-pass sees at
  // 64: the fp16-code and INT8 routes)
  if constexpr (D == 64) {
    if (n_q > 0 && !q_done) {
      p.n_q = (int)(B * Hq * p.nqb);
      p.n_stat = p.n_k = p.n_v = 0;
      launch_qquant_kernel<T>(p, vl != nullptr, c16 != nullptr, st);
      SAGE_CUDA_TRY(cudaGetLastError());
      q_done = true;
    }
  }
  // launch A: Q blocks and statistics chunks (and K blocks when K needs no statistics)
  p.n_q = q_done ? 0 : (int)n_q;
  p.n_stat = (int)n_stat;
  p.n_k = want_km ? 0 : (int)n_k;
  p.n_v = 0;
  const int64_t grid_a = (int64_t)p.n_q + p.n_stat + p.n_k;
  if (grid_a > 0 && grid_a == p.n_stat && !want_v) {
    // K statistics alone (Q quantised in the attention kernel): the lighter statistics kernel
    if (vl) sage::kstats_kernel<D, T, true><<<(unsigned)grid_a, sage::kQuantThreads, 0, st>>>(p);
    else sage::kstats_kernel<D, T, false><<<(unsigned)grid_a, sage::kQuantThreads, 0, st>>>(p);
    SAGE_CUDA_TRY(cudaGetLastError());
  } else if (grid_a > 0) {
    launch_prepass_kernel<D, T>(p, grid_a, vl != nullptr, c16 != nullptr, st);
    SAGE_CUDA_TRY(cudaGetLastError());
  }
  if (need_stats) {
    sage::FinalizeParams fp{};
    fp.ksum_part = p.ksum_part; fp.vmax_part = p.vmax_part; fp.k_mean = k_mean; fp.v_scale = v_scale;
    fp.Hkv = (int)Hkv; fp.S = (int)Skv; fp.nchunk = nchunk; fp.D = D;
    if (vl) { fp.cu = vl->cu_k; fp.tokens = (int)vl->k_tokens; }
    sage::kv_finalize_kernel<<<dim3((unsigned)Hkv, (unsigned)B), 128, 0, st>>>(fp);
    SAGE_CUDA_TRY(cudaGetLastError());
    // launch B: K blocks that needed the mean, and V blocks
    p.n_q = 0;
    p.n_stat = 0;
    p.n_k = want_km ? (int)n_k : 0;
    p.n_v = (int)n_v;
    const int64_t grid_b = (int64_t)p.n_k + p.n_v;
    if (p.n_k > 0) {
      // K blocks in the 128-thread kernel, then V blocks (if any) in the combined one
      const int n_v_b = p.n_v;
      p.n_k = (int)(B * Hkv * cdiv(p.nkb, sage::kKQuantBlocks<D>));
      p.n_v = 0;
      launch_kquant_kernel<D, T>(p, vl != nullptr, c16 != nullptr, st);
      SAGE_CUDA_TRY(cudaGetLastError());
      if (n_v_b > 0) {
        p.n_k = 0;
        p.n_v = n_v_b;
        launch_prepass_kernel<D, T>(p, n_v_b, vl != nullptr, c16 != nullptr, st);
        SAGE_CUDA_TRY(cudaGetLastError());
      }
    } else if (grid_b > 0) {
      launch_prepass_kernel<D, T>(p, grid_b, vl != nullptr, c16 != nullptr, st);
      SAGE_CUDA_TRY(cudaGetLastError());
    }
  }
  return SAGE_OK;
}

int prepass_dispatch(int dtype, int64_t D, const void* q, const void* k, const void* v, int64_t B, int64_t Hq,
                     int64_t Hkv, int64_t Sq, int64_t Skv, const int64_t* qs, const int64_t* ks, const int64_t* vs,
                     float q_mult, bool smooth, bool km_given, int8_t* q_i8, float* q_scale, int8_t* k_i8, float* k_scale,
                     float* k_mean, uint8_t* v_fp8, float* v_scale, void* ws, cudaStream_t st,
                     const Varlen* vl = nullptr, const Codes16* c16 = nullptr, int qblk = 128) {
  if (dtype == SAGE_DTYPE_F16) {
    if (D == 128)
      return launch_prepass<128, __half>(q, k, v, B, Hq, Hkv, Sq, Skv, qs, ks, vs, q_mult, smooth, km_given, q_i8, q_scale, k_i8,
                                         k_scale, k_mean, v_fp8, v_scale, ws, vl, c16, st, qblk);
    return launch_prepass<64, __half>(q, k, v, B, Hq, Hkv, Sq, Skv, qs, ks, vs, q_mult, smooth, km_given, q_i8, q_scale, k_i8,
                                      k_scale, k_mean, v_fp8, v_scale, ws, vl, c16, st, qblk);
  }
  if (D == 128)
    return launch_prepass<128, __nv_bfloat16>(q, k, v, B, Hq, Hkv, Sq, Skv, qs, ks, vs, q_mult, smooth, km_given, q_i8, q_scale,
                                              k_i8, k_scale, k_mean, v_fp8, v_scale, ws, vl, c16, st, qblk);
  return launch_prepass<64, __nv_bfloat16>(q, k, v, B, Hq, Hkv, Sq, Skv, qs, ks, vs, q_mult, smooth, km_given, q_i8, q_scale,
                                           k_i8, k_scale, k_mean, v_fp8, v_scale, ws, vl, c16, st, qblk);
}

// ---------------------------------------------------------------- attention launch
template <int D, int PV, bool OBF16, bool FLASH = false, bool FQ = false, bool C16 = false>
int launch_attn(const CUtensorMap& tq, const CUtensorMap& tk, const CUtensorMap& tv, const sage::AttnParams& p,
                cudaStream_t st) {
  constexpr int QT = 2;
  using C = sage::AttnCfg<D, PV, QT, FLASH, C16>;
  auto kern = sage::sage_attn_kernel<D, PV, QT, OBF16, FLASH, FQ, C16>;
  if (int rc = ensure_smem(reinterpret_cast<const void*>(kern), C::SMEM_BYTES)) return rc;
  dim3 grid((unsigned)p.n_m_ctas, (unsigned)p.Hq, (unsigned)p.B);
  kern<<<grid, C::NUM_THREADS, C::SMEM_BYTES, st>>>(tq, tk, tv, p);
  SAGE_CUDA_TRY(cudaGetLastError());
  return SAGE_OK;
}

// Batch stride (elements) for a tensor map over packed sequences, whose batch extent is 1: any
// valid stride serves; this one covers the whole tensor.
int64_t packed_batch_stride(const int64_t* s, int64_t H, int64_t rows) { return std::max(s[1] * H, s[2] * rows); }

// Whether o is anything but memory of the current device (a peer GPU's memory mapped here for a
// multi-GPU gather, managed or host memory): the attention epilogue then stages its rows and
// stores whole lines. A failed query counts as remote (the staged path is correct for any o).
bool out_is_remote(const void* o) {
  cudaPointerAttributes a{};
  if (cudaPointerGetAttributes(&a, o) != cudaSuccess) {
    (void)cudaGetLastError();
    return true;
  }
  int dev = -1;
  if (cudaGetDevice(&dev) != cudaSuccess) return true;
  return a.type != cudaMemoryTypeDevice || a.device != dev;
}

// Sets the tensor-shape fields that dense and packed batches share; rows / batch extents of the
// tensor maps come from here too.
void set_seq_params(sage::AttnParams& p, const Varlen* vl, const int64_t* os, int64_t B, int64_t Hq, int64_t Hkv,
                    int64_t Sq, int64_t Skv, int causal) {
  p.o_sb = vl ? 0 : os[0]; p.o_sh = os[1]; p.o_ss = os[2];
  p.B = (int)B; p.Hq = (int)Hq; p.Hkv = (int)Hkv; p.Sq = (int)Sq; p.Skv = (int)Skv;
  p.groups = (int)(Hq / Hkv);
  p.nqb = (int)cdiv(Sq, 128); p.nkb = (int)cdiv(Skv, 64);
  p.qblk_shift = 7;
  p.causal = causal ? 1 : 0;
  p.o_stage = out_is_remote(p.o) ? 1 : 0;
  p.n_m_ctas = (int)cdiv(Sq, 256);
  p.wait_limit_ns = wait_limit_ns();
  if (vl) { p.cu_q = vl->cu_q; p.cu_k = vl->cu_k; p.q_tokens = (int)vl->q_tokens; p.k_tokens = (int)vl->k_tokens; }
}

// The INT8 attention instantiations: head_dim x P.V mode x output type, with Q quantised by the
// pre-pass (FQ = false) or inside the kernel (FQ = true).
template <bool FQ, bool C16 = false>
int attn_dispatch(int64_t D, bool fp8, bool obf, const CUtensorMap& tq, const CUtensorMap& tk, const CUtensorMap& tv,
                  const sage::AttnParams& p, cudaStream_t st) {
  if constexpr (C16) {  // head_dim 64 only
    if (D != 64) return fail(SAGE_ERR_INVALID_ARG, "fp16 codes are the head_dim-64 route");
    if (fp8) return obf ? launch_attn<64, sage::kPvE4M3, true, false, false, true>(tq, tk, tv, p, st)
                        : launch_attn<64, sage::kPvE4M3, false, false, false, true>(tq, tk, tv, p, st);
    return obf ? launch_attn<64, sage::kPvBF16, true, false, false, true>(tq, tk, tv, p, st)
               : launch_attn<64, sage::kPvF16, false, false, false, true>(tq, tk, tv, p, st);
  }
  if (D == 128) {
    if (fp8) return obf ? launch_attn<128, sage::kPvE4M3, true, false, FQ>(tq, tk, tv, p, st)
                        : launch_attn<128, sage::kPvE4M3, false, false, FQ>(tq, tk, tv, p, st);
    return obf ? launch_attn<128, sage::kPvBF16, true, false, FQ>(tq, tk, tv, p, st)
               : launch_attn<128, sage::kPvF16, false, false, FQ>(tq, tk, tv, p, st);
  }
  if (fp8) return obf ? launch_attn<64, sage::kPvE4M3, true, false, FQ>(tq, tk, tv, p, st)
                      : launch_attn<64, sage::kPvE4M3, false, false, FQ>(tq, tk, tv, p, st);
  return obf ? launch_attn<64, sage::kPvBF16, true, false, FQ>(tq, tk, tv, p, st)
             : launch_attn<64, sage::kPvF16, false, false, FQ>(tq, tk, tv, p, st);
}

// Q quantised inside the attention kernel instead of by the pre-pass: the caller's 16-bit Q,
// its {batch, head, seq} strides and multiplier; the codes / scales are also stored where
// q_i8_out / q_scale_out are not NULL.
struct FusedQ {
  const void* q;
  const int64_t* qs;
  float q_mult;
  int8_t* q_i8_out;
  float* q_scale_out;
};

int attn_impl(const int8_t* q_i8, const float* q_scale, const int8_t* k_i8, const float* k_scale, const void* v,
              const int64_t* vs, const float* v_scale, void* o, const int64_t* os, int dtype, int pv_mode, int causal,
              int64_t B, int64_t Hq, int64_t Hkv, int64_t Sq, int64_t Skv, int64_t D, cudaStream_t st,
              const Varlen* vl = nullptr, const FusedQ* fq = nullptr, const Codes16* c16 = nullptr,
              int qblk = 128) {
  const bool fp8 = pv_mode == SAGE_PV_FP8;
  // rows of the token axis and batch extent of every tensor map (packed sequences: one batch)
  const int64_t rq = vl ? vl->q_tokens : Sq, rk = vl ? vl->k_tokens : Skv, nb = vl ? 1 : B;
  CUtensorMap tq, tk, tv;
  const CUtensorMapSwizzle swqk = (D == 128) ? CU_TENSOR_MAP_SWIZZLE_128B : CU_TENSOR_MAP_SWIZZLE_64B;
  if (!c16) {
    if (int rc = encode_4d(&tk, CU_TENSOR_MAP_DATA_TYPE_UINT8, 1, k_i8, D, rk, Hkv, nb, D, rk * D, Hkv * rk * D,
                           (uint32_t)D, 128, swqk))
      return rc;
  }
  if (c16) {  // fp16 codes: 128-byte rows at head_dim 64
    const int64_t* cs = c16->qs;
    if (int rc = encode_4d(&tq, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 2, c16->q, D, rq, Hq, nb, cs[2], cs[1],
                           vl ? packed_batch_stride(cs, Hq, rq) : cs[0], (uint32_t)D, 128, CU_TENSOR_MAP_SWIZZLE_128B))
      return rc;
    if (int rc = encode_4d(&tk, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 2, c16->k, D, rk, Hkv, nb, D, rk * D, Hkv * rk * D,
                           (uint32_t)D, 128, CU_TENSOR_MAP_SWIZZLE_128B))
      return rc;
  } else if (fq) {
    tq = tk;  // not read: the kernel loads Q itself
  } else if (int rc = encode_4d(&tq, CU_TENSOR_MAP_DATA_TYPE_UINT8, 1, q_i8, D, rq, Hq, nb, D, rq * D, Hq * rq * D,
                                (uint32_t)D, 128, swqk)) {
    return rc;
  }
  if (fp8) {
    if (int rc = encode_4d(&tv, CU_TENSOR_MAP_DATA_TYPE_UINT8, 1, v, D, rk, Hkv, nb, D, rk * D, Hkv * rk * D,
                           (uint32_t)D, 128, swqk))
      return rc;
  } else {
    const CUtensorMapDataType dt =
        dtype == SAGE_DTYPE_BF16 ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16 : CU_TENSOR_MAP_DATA_TYPE_FLOAT16;
    if (int rc = encode_4d(&tv, dt, 2, v, D, rk, Hkv, nb, vs[2], vs[1], vl ? packed_batch_stride(vs, Hkv, rk) : vs[0],
                           64, 128, CU_TENSOR_MAP_SWIZZLE_128B))
      return rc;
  }
  sage::AttnParams p{};
  p.q_scale = q_scale; p.k_scale = k_scale; p.v_scale = v_scale; p.o = o;
  set_seq_params(p, vl, os, B, Hq, Hkv, Sq, Skv, causal);
  p.qblk_shift = qblk_shift(qblk);
  p.nqb = (int)cdiv(Sq, qblk);
  if (fq) {
    p.q_src = fq->q;
    p.q_sb = vl ? 0 : fq->qs[0]; p.q_sh = fq->qs[1]; p.q_ss = fq->qs[2];
    p.q_mult = fq->q_mult;
    p.q_i8_out = fq->q_i8_out; p.q_scale_out = fq->q_scale_out;
  }
  const bool obf = dtype == SAGE_DTYPE_BF16;
  if (c16) return attn_dispatch<false, true>(D, fp8, obf, tq, tk, tv, p, st);
  return fq ? attn_dispatch<true>(D, fp8, obf, tq, tk, tv, p, st) : attn_dispatch<false>(D, fp8, obf, tq, tk, tv, p, st);
}

// flash_attn pack: the same pipeline on fp16/bf16 Q and K (no pre-pass)
int flash_impl(const void* q, const int64_t* qs, const void* k, const int64_t* ks, const void* v, const int64_t* vs,
               void* o, const int64_t* os, int dtype, int causal, int64_t B, int64_t Hq, int64_t Hkv, int64_t Sq,
               int64_t Skv, int64_t D, float sm_scale, cudaStream_t st, const Varlen* vl = nullptr) {
  const CUtensorMapDataType dt =
      dtype == SAGE_DTYPE_BF16 ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16 : CU_TENSOR_MAP_DATA_TYPE_FLOAT16;
  const int64_t rq = vl ? vl->q_tokens : Sq, rk = vl ? vl->k_tokens : Skv, nb = vl ? 1 : B;
  CUtensorMap tq, tk, tv;
  if (int rc = encode_4d(&tq, dt, 2, q, D, rq, Hq, nb, qs[2], qs[1], vl ? packed_batch_stride(qs, Hq, rq) : qs[0], 64,
                         128, CU_TENSOR_MAP_SWIZZLE_128B))
    return rc;
  if (int rc = encode_4d(&tk, dt, 2, k, D, rk, Hkv, nb, ks[2], ks[1], vl ? packed_batch_stride(ks, Hkv, rk) : ks[0],
                         64, 128, CU_TENSOR_MAP_SWIZZLE_128B))
    return rc;
  if (int rc = encode_4d(&tv, dt, 2, v, D, rk, Hkv, nb, vs[2], vs[1], vl ? packed_batch_stride(vs, Hkv, rk) : vs[0],
                         64, 128, CU_TENSOR_MAP_SWIZZLE_128B))
    return rc;
  sage::AttnParams p{};
  p.o = o;
  set_seq_params(p, vl, os, B, Hq, Hkv, Sq, Skv, causal);
  const double s = sm_scale > 0.0f ? static_cast<double>(sm_scale) : 1.0 / std::sqrt(static_cast<double>(D));
  p.qk_scale = static_cast<float>(s * 1.4426950408889634);  // exp(x) = exp2(x * log2(e))
  if (dtype == SAGE_DTYPE_BF16)
    return D == 128 ? launch_attn<128, sage::kPvBF16, true, true>(tq, tk, tv, p, st)
                    : launch_attn<64, sage::kPvBF16, true, true>(tq, tk, tv, p, st);
  return D == 128 ? launch_attn<128, sage::kPvF16, false, true>(tq, tk, tv, p, st)
                  : launch_attn<64, sage::kPvF16, false, true>(tq, tk, tv, p, st);
}

float q_multiplier(float sm_scale, int64_t D) {
  const double s = sm_scale > 0.0f ? static_cast<double>(sm_scale) : 1.0 / std::sqrt(static_cast<double>(D));
  return static_cast<float>(s * 1.44269504);
}

__global__ void watchdog_selftest_kernel(unsigned long long limit_ns) {
  __shared__ __align__(8) uint64_t bar;
  __shared__ int abort_flag;
  if (threadIdx.x == 0) {
    sage::mbar_init(&bar, 1);
    abort_flag = 0;
    sage::fence_barrier_init();
  }
  __syncthreads();
  if (threadIdx.x == 0) {
    // Nothing ever arrives on `bar`: the bounded wait must give up and report.
    (void)sage::mbar_wait(&bar, 0, &abort_flag, sage::kDevTimeoutEpilogue, limit_ns);
  }
  __syncthreads();
}

// ---------------------------------------------------------------- allocation-free variant
// Scratch of sage_per_block_int8_noalloc: the fp64 K column partial sums of the smoothing
// statistics. It lives in the library image, so every GPU that loads the library holds it
// until the process exits, and no call allocates device memory.
constexpr size_t kNoAllocScratchBytes = size_t(4) << 20;  // 4 MiB = 524288 fp64 partial sums
static __device__ __align__(256) double g_noalloc_scratch[kNoAllocScratchBytes / sizeof(double)];

// Device address of g_noalloc_scratch on the current device. In host code the symbol is only a
// host-side stand-in, so the address is looked up once per device (with that device current)
// and cached; the first call on a device does this lookup.
int noalloc_scratch(void** out) {
  int dev = 0;
  if (int rc = current_device(&dev)) return rc;
  static void* addr[kMaxDevices];
  std::lock_guard<std::mutex> lk(g_mutex);
  if (!addr[dev]) {
    void* ptr = nullptr;
    const cudaError_t e = cudaGetSymbolAddress(&ptr, g_noalloc_scratch);
    if (e != cudaSuccess || !ptr)
      return fail(SAGE_ERR_CUDA, "cudaGetSymbolAddress(g_noalloc_scratch) failed: %s", cudaGetErrorString(e));
    addr[dev] = ptr;
  }
  *out = addr[dev];
  return SAGE_OK;
}

}  // namespace

extern "C" {

int sage_abi_version(void) { return SAGE_ABI_VERSION; }

const char* sage_last_error(void) { return g_last_error.c_str(); }

size_t sage_workspace_bytes(int64_t batch, int64_t heads_kv, int64_t seq_kv, int64_t head_dim, int pv_mode,
                            unsigned flags) {
  if (batch <= 0 || heads_kv <= 0 || seq_kv <= 0 || head_dim <= 0) return 0;
  return stats_ws_bytes(batch, heads_kv, seq_kv, head_dim, pv_mode, flags) +
         (c16_route(flags, head_dim) ? codes_ws_bytes(batch, heads_kv, seq_kv, head_dim) : 0);
}

int sage_per_block_int8(const void* q, const void* k, int dtype, int64_t batch, int64_t heads_q, int64_t heads_kv,
                        int64_t seq_q, int64_t seq_kv, int64_t head_dim, const int64_t q_strides[3],
                        const int64_t k_strides[3], float sm_scale, unsigned flags, int8_t* q_i8, float* q_scale,
                        int8_t* k_i8, float* k_scale, float* k_mean, void* workspace, size_t workspace_bytes,
                        void* stream) {
  g_last_error.clear();
  if (int rc = check_shape(dtype, batch, heads_q, heads_kv, seq_q, seq_kv, head_dim)) return rc;
  if (int rc = check_strides("q", q_strides)) return rc;
  if (int rc = check_strides("k", k_strides)) return rc;
  int qblk = 128;
  if (int rc = qblk_from_flags(flags, &qblk)) return rc;
  if (!q || !k || !q_i8 || !q_scale || !k_i8 || !k_scale) return fail(SAGE_ERR_INVALID_ARG, "NULL tensor pointer");
  if (!aligned16(q) || !aligned16(k) || !aligned16(q_i8) || !aligned16(k_i8))
    return fail(SAGE_ERR_INVALID_ARG, "q/k/q_i8/k_i8 must be 16-byte aligned");
  const bool smooth = (flags & SAGE_FLAG_SMOOTH_K) != 0;
  if (smooth && !k_mean) return fail(SAGE_ERR_INVALID_ARG, "SAGE_FLAG_SMOOTH_K needs k_mean");
  const bool km_given = smooth && (flags & SAGE_FLAG_KM_GIVEN) != 0;
  const size_t need = km_given ? 0 : stats_ws_bytes(batch, heads_kv, seq_kv, head_dim, SAGE_PV_16BIT, flags);
  if (need && (!workspace || workspace_bytes < need))
    return fail(SAGE_ERR_WORKSPACE, "workspace of %zu bytes needed, %zu given", need, workspace_bytes);
  if (int rc = check_arch()) return rc;
  return prepass_dispatch(dtype, head_dim, q, k, nullptr, batch, heads_q, heads_kv, seq_q, seq_kv, q_strides,
                          k_strides, nullptr, q_multiplier(sm_scale, head_dim), smooth, km_given, q_i8, q_scale, k_i8,
                          k_scale, k_mean, nullptr, nullptr, workspace, static_cast<cudaStream_t>(stream), nullptr,
                          nullptr, qblk);
}

int sage_per_block_int8_noalloc(const void* q, const void* k, int dtype, int64_t batch, int64_t heads_q,
                                int64_t heads_kv, int64_t seq_q, int64_t seq_kv, int64_t head_dim,
                                const int64_t q_strides[3], const int64_t k_strides[3], float sm_scale,
                                unsigned flags, int8_t* q_i8, float* q_scale, int8_t* k_i8, float* k_scale,
                                float* k_mean, void* stream) {
  g_last_error.clear();
  if (int rc = check_shape(dtype, batch, heads_q, heads_kv, seq_q, seq_kv, head_dim)) return rc;
  if (int rc = check_strides("q", q_strides)) return rc;
  if (int rc = check_strides("k", k_strides)) return rc;
  int qblk = 128;
  if (int rc = qblk_from_flags(flags, &qblk)) return rc;
  if (!q || !k || !q_i8 || !q_scale || !k_i8 || !k_scale) return fail(SAGE_ERR_INVALID_ARG, "NULL tensor pointer");
  if (!aligned16(q) || !aligned16(k) || !aligned16(q_i8) || !aligned16(k_i8))
    return fail(SAGE_ERR_INVALID_ARG, "q/k/q_i8/k_i8 must be 16-byte aligned");
  const bool smooth = (flags & SAGE_FLAG_SMOOTH_K) != 0;
  if (smooth && !k_mean) return fail(SAGE_ERR_INVALID_ARG, "SAGE_FLAG_SMOOTH_K needs k_mean");
  const bool km_given = smooth && (flags & SAGE_FLAG_KM_GIVEN) != 0;
  const size_t need = km_given ? 0 : stats_ws_bytes(batch, heads_kv, seq_kv, head_dim, SAGE_PV_16BIT, flags);
  if (need > kNoAllocScratchBytes)
    return fail(SAGE_ERR_INVALID_ARG,
                "sizes need %zu bytes of statistics scratch; the built-in scratch of "
                "sage_per_block_int8_noalloc holds %zu (batch*heads_kv*ceil(seq_kv/512)*head_dim <= %zu)",
                need, kNoAllocScratchBytes, kNoAllocScratchBytes / sizeof(double));
  if (int rc = check_arch()) return rc;
  void* scratch = nullptr;
  if (need) {
    if (int rc = noalloc_scratch(&scratch)) return rc;
  }
  return prepass_dispatch(dtype, head_dim, q, k, nullptr, batch, heads_q, heads_kv, seq_q, seq_kv, q_strides,
                          k_strides, nullptr, q_multiplier(sm_scale, head_dim), smooth, km_given, q_i8, q_scale, k_i8,
                          k_scale, k_mean, nullptr, nullptr, scratch, static_cast<cudaStream_t>(stream), nullptr,
                          nullptr, qblk);
}

int sage_quant_v_fp8(const void* v, int dtype, int64_t batch, int64_t heads_kv, int64_t seq_kv, int64_t head_dim,
                     const int64_t v_strides[3], uint8_t* v_fp8, float* v_scale, void* workspace,
                     size_t workspace_bytes, void* stream) {
  g_last_error.clear();
  if (int rc = check_shape(dtype, batch, heads_kv, heads_kv, seq_kv, seq_kv, head_dim)) return rc;
  if (int rc = check_strides("v", v_strides)) return rc;
  if (!v || !v_fp8 || !v_scale) return fail(SAGE_ERR_INVALID_ARG, "NULL tensor pointer");
  if (!aligned16(v) || !aligned16(v_fp8)) return fail(SAGE_ERR_INVALID_ARG, "v/v_fp8 must be 16-byte aligned");
  const size_t need = stats_ws_bytes(batch, heads_kv, seq_kv, head_dim, SAGE_PV_FP8, 0);
  if (!workspace || workspace_bytes < need)
    return fail(SAGE_ERR_WORKSPACE, "workspace of %zu bytes needed, %zu given", need, workspace_bytes);
  if (int rc = check_arch()) return rc;
  return prepass_dispatch(dtype, head_dim, nullptr, nullptr, v, batch, heads_kv, heads_kv, seq_kv, seq_kv, nullptr,
                          nullptr, v_strides, 1.0f, false, false, nullptr, nullptr, nullptr, nullptr, nullptr, v_fp8,
                          v_scale, workspace, static_cast<cudaStream_t>(stream));
}

int sage_attn_fwd(const int8_t* q_i8, const float* q_scale, const int8_t* k_i8, const float* k_scale, const void* v,
                  const int64_t v_strides[3], const float* v_scale, void* o, const int64_t o_strides[3], int dtype,
                  int pv_mode, int causal, unsigned flags, int64_t batch, int64_t heads_q, int64_t heads_kv,
                  int64_t seq_q, int64_t seq_kv, int64_t head_dim, void* stream) {
  g_last_error.clear();
  if (int rc = check_shape(dtype, batch, heads_q, heads_kv, seq_q, seq_kv, head_dim)) return rc;
  int qblk = 128;
  if (int rc = check_attn_flags(flags, &qblk)) return rc;
  if (pv_mode != SAGE_PV_16BIT && pv_mode != SAGE_PV_FP8)
    return fail(SAGE_ERR_INVALID_ARG, "pv_mode %d unknown", pv_mode);
  if (causal && seq_q != seq_kv)
    return fail(SAGE_ERR_INVALID_ARG, "causal attention needs seq_q == seq_kv (got %lld, %lld)", (long long)seq_q,
                (long long)seq_kv);
  if (int rc = check_strides("o", o_strides)) return rc;
  if (pv_mode == SAGE_PV_16BIT) {
    if (int rc = check_strides("v", v_strides)) return rc;
  } else if (!v_scale) {
    return fail(SAGE_ERR_INVALID_ARG, "SAGE_PV_FP8 needs v_scale");
  }
  if (!q_i8 || !q_scale || !k_i8 || !k_scale || !v || !o) return fail(SAGE_ERR_INVALID_ARG, "NULL tensor pointer");
  if (!aligned16(q_i8) || !aligned16(k_i8) || !aligned16(v) || !aligned16(o))
    return fail(SAGE_ERR_INVALID_ARG, "q_i8/k_i8/v/o must be 16-byte aligned");
  {
    const bool fp8 = pv_mode == SAGE_PV_FP8;
    const Span vsp = fp8 ? buffer_span(v, static_cast<size_t>(batch * heads_kv * seq_kv * head_dim))
                         : tensor_span(v, v_strides, batch, heads_kv, seq_kv, head_dim, 2);
    if (int rc = check_attn_alias(o, o_strides, tensor_span(o, o_strides, batch, heads_q, seq_q, head_dim, 2), nullptr,
                                  nullptr, Span{}, Span{}, vsp, batch, heads_q, heads_kv, batch * seq_q, batch * seq_kv,
                                  cdiv(seq_q, qblk), cdiv(seq_kv, 64), head_dim, q_i8, q_scale, k_i8, k_scale, nullptr,
                                  nullptr, fp8 ? v_scale : nullptr, nullptr, 0))
      return rc;
  }
  if (int rc = check_arch()) return rc;
  return attn_impl(q_i8, q_scale, k_i8, k_scale, v, v_strides, v_scale, o, o_strides, dtype, pv_mode, causal, batch,
                   heads_q, heads_kv, seq_q, seq_kv, head_dim, static_cast<cudaStream_t>(stream), nullptr, nullptr,
                   nullptr, qblk);
}

int sage_attn_fwd_fused_q(const void* q, const int64_t q_strides[3], float sm_scale, const int8_t* k_i8,
                          const float* k_scale, const void* v, const int64_t v_strides[3], const float* v_scale,
                          void* o, const int64_t o_strides[3], int dtype, int pv_mode, int causal,
                          unsigned flags, int64_t batch, int64_t heads_q, int64_t heads_kv, int64_t seq_q,
                          int64_t seq_kv, int64_t head_dim, int8_t* q_i8_out, float* q_scale_out, void* stream) {
  g_last_error.clear();
  if (int rc = check_shape(dtype, batch, heads_q, heads_kv, seq_q, seq_kv, head_dim)) return rc;
  int qblk = 128;
  if (int rc = check_attn_flags(flags, &qblk)) return rc;
  if (pv_mode != SAGE_PV_16BIT && pv_mode != SAGE_PV_FP8)
    return fail(SAGE_ERR_INVALID_ARG, "pv_mode %d unknown", pv_mode);
  if (causal && seq_q != seq_kv)
    return fail(SAGE_ERR_INVALID_ARG, "causal attention needs seq_q == seq_kv (got %lld, %lld)", (long long)seq_q,
                (long long)seq_kv);
  if (int rc = check_strides("q", q_strides)) return rc;
  if (int rc = check_strides("o", o_strides)) return rc;
  if (pv_mode == SAGE_PV_16BIT) {
    if (int rc = check_strides("v", v_strides)) return rc;
  } else if (!v_scale) {
    return fail(SAGE_ERR_INVALID_ARG, "SAGE_PV_FP8 needs v_scale");
  }
  if (!q || !k_i8 || !k_scale || !v || !o || (!q_i8_out != !q_scale_out))
    return fail(SAGE_ERR_INVALID_ARG, "NULL tensor pointer");
  if (!aligned16(q) || !aligned16(k_i8) || !aligned16(v) || !aligned16(o) || (q_i8_out && !aligned16(q_i8_out)))
    return fail(SAGE_ERR_INVALID_ARG, "q/k_i8/v/o/q_i8_out must be 16-byte aligned");
  {
    const bool fp8 = pv_mode == SAGE_PV_FP8;
    const Span vsp = fp8 ? buffer_span(v, static_cast<size_t>(batch * heads_kv * seq_kv * head_dim))
                         : tensor_span(v, v_strides, batch, heads_kv, seq_kv, head_dim, 2);
    if (int rc = check_attn_alias(o, o_strides, tensor_span(o, o_strides, batch, heads_q, seq_q, head_dim, 2), q,
                                  q_strides, tensor_span(q, q_strides, batch, heads_q, seq_q, head_dim, 2), Span{}, vsp,
                                  batch, heads_q, heads_kv, batch * seq_q, batch * seq_kv, cdiv(seq_q, qblk),
                                  cdiv(seq_kv, 64), head_dim, q_i8_out, q_scale_out, k_i8, k_scale, nullptr, nullptr,
                                  fp8 ? v_scale : nullptr, nullptr, 0))
      return rc;
  }
  if (int rc = check_arch()) return rc;
  const FusedQ fq{q, q_strides, q_multiplier(sm_scale, head_dim), q_i8_out, q_scale_out};
  return attn_impl(nullptr, nullptr, k_i8, k_scale, v, v_strides, v_scale, o, o_strides, dtype, pv_mode, causal,
                   batch, heads_q, heads_kv, seq_q, seq_kv, head_dim, static_cast<cudaStream_t>(stream), nullptr, &fq,
                   nullptr, qblk);
}

int sage_attn_fwd_codes16(const void* q_c16, const float* q_scale, const void* k_c16, const float* k_scale,
                          const void* v, const int64_t v_strides[3], const float* v_scale, void* o,
                          const int64_t o_strides[3], int dtype, int pv_mode, int causal, unsigned flags,
                          int64_t batch, int64_t heads_q, int64_t heads_kv, int64_t seq_q, int64_t seq_kv,
                          int64_t head_dim, void* stream) {
  g_last_error.clear();
  if (int rc = check_shape(dtype, batch, heads_q, heads_kv, seq_q, seq_kv, head_dim)) return rc;
  int qblk = 128;
  if (int rc = check_attn_flags(flags, &qblk)) return rc;
  if (head_dim != 64) return fail(SAGE_ERR_INVALID_ARG, "fp16 codes are the head_dim-64 route");
  if (pv_mode != SAGE_PV_16BIT && pv_mode != SAGE_PV_FP8)
    return fail(SAGE_ERR_INVALID_ARG, "pv_mode %d unknown", pv_mode);
  if (causal && seq_q != seq_kv)
    return fail(SAGE_ERR_INVALID_ARG, "causal attention needs seq_q == seq_kv (got %lld, %lld)", (long long)seq_q,
                (long long)seq_kv);
  if (int rc = check_strides("o", o_strides)) return rc;
  if (pv_mode == SAGE_PV_16BIT) {
    if (int rc = check_strides("v", v_strides)) return rc;
  } else if (!v_scale) {
    return fail(SAGE_ERR_INVALID_ARG, "SAGE_PV_FP8 needs v_scale");
  }
  if (!q_c16 || !q_scale || !k_c16 || !k_scale || !v || !o) return fail(SAGE_ERR_INVALID_ARG, "NULL tensor pointer");
  if (!aligned16(q_c16) || !aligned16(k_c16) || !aligned16(v) || !aligned16(o))
    return fail(SAGE_ERR_INVALID_ARG, "q_c16/k_c16/v/o must be 16-byte aligned");
  const int64_t qcs[3] = {heads_q * seq_q * head_dim, seq_q * head_dim, head_dim};
  {
    // q_c16 may be o itself (contiguous o, as sage_run arranges it); k_c16 holds 2-byte codes
    const bool fp8 = pv_mode == SAGE_PV_FP8;
    const Span vsp = fp8 ? buffer_span(v, static_cast<size_t>(batch * heads_kv * seq_kv * head_dim))
                         : tensor_span(v, v_strides, batch, heads_kv, seq_kv, head_dim, 2);
    const Span ksp = buffer_span(k_c16, static_cast<size_t>(batch * heads_kv * seq_kv * head_dim) * 2);
    if (int rc = check_attn_alias(o, o_strides, tensor_span(o, o_strides, batch, heads_q, seq_q, head_dim, 2), q_c16,
                                  qcs, tensor_span(q_c16, qcs, batch, heads_q, seq_q, head_dim, 2), ksp, vsp, batch,
                                  heads_q, heads_kv, batch * seq_q, batch * seq_kv, cdiv(seq_q, qblk), cdiv(seq_kv, 64),
                                  head_dim, nullptr, q_scale, nullptr, k_scale, nullptr, nullptr,
                                  fp8 ? v_scale : nullptr, nullptr, 0))
      return rc;
  }
  if (int rc = check_arch()) return rc;
  const Codes16 c16{static_cast<__half*>(const_cast<void*>(q_c16)), qcs,
                    static_cast<__half*>(const_cast<void*>(k_c16))};
  return attn_impl(nullptr, q_scale, nullptr, k_scale, v, v_strides, v_scale, o, o_strides, dtype, pv_mode, causal,
                   batch, heads_q, heads_kv, seq_q, seq_kv, head_dim, static_cast<cudaStream_t>(stream), nullptr,
                   nullptr, &c16, qblk);
}

namespace {
// Where sage_run / sage_run_varlen quantise Q: inside the attention kernel at head_dim 128
// (H8K 1.817 -> 1.774 ms per call: the pre-pass no longer reads Q and writes its INT8 copy) or
// with SAGE_FLAG_FUSED_Q, else in the pre-pass (at head_dim 64 the fused kernel was 3 % slower).
// SAGE_FLAG_PREPASS_Q keeps Q in the pre-pass at head_dim 128.
bool fused_q_for(unsigned flags, int64_t head_dim) {
  if (flags & SAGE_FLAG_PREPASS_Q) return false;
  return (flags & SAGE_FLAG_FUSED_Q) != 0 || head_dim == 128;
}

// The three ways sage_run can feed the attention kernel.
enum class Route { kInt8, kFusedQ, kCodes16 };
Route run_route(unsigned flags, int64_t head_dim) {
  if (fused_q_for(flags, head_dim)) return Route::kFusedQ;
  return c16_route(flags, head_dim) ? Route::kCodes16 : Route::kInt8;
}

// Shared validation of sage_prepass / sage_run; returns SAGE_OK or the failing status.
int check_run_args(const void* q, const void* k, const void* v, int dtype, int64_t batch, int64_t heads_q,
                   int64_t heads_kv, int64_t seq_q, int64_t seq_kv, int64_t head_dim, const int64_t* q_strides,
                   const int64_t* k_strides, const int64_t* v_strides, int pv_mode, unsigned flags,
                   const int8_t* q_i8, const float* q_scale, const int8_t* k_i8, const float* k_scale,
                   const float* k_mean, const uint8_t* v_fp8, const float* v_scale, const void* workspace,
                   size_t workspace_bytes, Route route, bool run) {
  if (int rc = check_shape(dtype, batch, heads_q, heads_kv, seq_q, seq_kv, head_dim)) return rc;
  if (pv_mode != SAGE_PV_16BIT && pv_mode != SAGE_PV_FP8)
    return fail(SAGE_ERR_INVALID_ARG, "pv_mode %d unknown", pv_mode);
  if ((flags & SAGE_FLAG_FUSED_Q) && (flags & SAGE_FLAG_PREPASS_Q))
    return fail(SAGE_ERR_INVALID_ARG, "SAGE_FLAG_FUSED_Q and SAGE_FLAG_PREPASS_Q exclude each other");
  int qblk = 128;
  if (int rc = qblk_from_flags(flags, &qblk)) return rc;
  if (int rc = check_strides("q", q_strides)) return rc;
  if (int rc = check_strides("k", k_strides)) return rc;
  if (int rc = check_strides("v", v_strides)) return rc;
  // Q quantised in the attention kernel: its codes / scales are optional outputs; sage_run's
  // fp16-code route keeps the codes in o and the workspace: q_i8 / k_i8 are not used
  if (!q || !k || !v || !k_scale || (route != Route::kCodes16 && !k_i8) || (route == Route::kCodes16 && !q_scale) ||
      (route == Route::kInt8 && (!q_i8 || !q_scale)) || (route == Route::kFusedQ && !q_i8 != !q_scale))
    return fail(SAGE_ERR_INVALID_ARG, "NULL tensor pointer");
  if (!aligned16(q) || !aligned16(k) || !aligned16(v) || (q_i8 && !aligned16(q_i8)) || (k_i8 && !aligned16(k_i8)))
    return fail(SAGE_ERR_INVALID_ARG, "q/k/v/q_i8/k_i8 must be 16-byte aligned");
  const bool smooth = (flags & SAGE_FLAG_SMOOTH_K) != 0;
  const bool fp8 = pv_mode == SAGE_PV_FP8;
  if (smooth && !k_mean) return fail(SAGE_ERR_INVALID_ARG, "SAGE_FLAG_SMOOTH_K needs k_mean");
  if (fp8 && (!v_fp8 || !v_scale || !aligned16(v_fp8)))
    return fail(SAGE_ERR_INVALID_ARG, "SAGE_PV_FP8 needs 16-byte aligned v_fp8 and v_scale");
  const bool km_given = smooth && (flags & SAGE_FLAG_KM_GIVEN) != 0;
  const size_t need = stats_ws_bytes(batch, heads_kv, seq_kv, head_dim, pv_mode, km_given ? 0u : flags) +
                      ((run && route == Route::kCodes16) ? codes_ws_bytes(batch, heads_kv, seq_kv, head_dim) : 0);
  if (need && (!workspace || workspace_bytes < need))
    return fail(SAGE_ERR_WORKSPACE, "workspace of %zu bytes needed, %zu given", need, workspace_bytes);
  return SAGE_OK;
}
}  // namespace

int sage_prepass(const void* q, const void* k, const void* v, int dtype, int64_t batch, int64_t heads_q,
                 int64_t heads_kv, int64_t seq_q, int64_t seq_kv, int64_t head_dim, const int64_t q_strides[3],
                 const int64_t k_strides[3], const int64_t v_strides[3], float sm_scale, int pv_mode,
                 unsigned flags, int8_t* q_i8, float* q_scale, int8_t* k_i8, float* k_scale, float* k_mean,
                 uint8_t* v_fp8, float* v_scale, void* workspace, size_t workspace_bytes, void* stream) {
  g_last_error.clear();
  const bool fused_q = (flags & SAGE_FLAG_FUSED_Q) != 0;  // Q is left to sage_attn_fwd_fused_q
  const bool codes16 = (flags & SAGE_FLAG_CODES16) != 0;  // codes as fp16 values, for sage_attn_fwd_codes16
  if (codes16 && (fused_q || head_dim != 64))
    return fail(SAGE_ERR_INVALID_ARG, "SAGE_FLAG_CODES16 is the head_dim-64 route and needs Q from the pre-pass");
  if (int rc = check_run_args(q, k, v, dtype, batch, heads_q, heads_kv, seq_q, seq_kv, head_dim, q_strides,
                              k_strides, v_strides, pv_mode, flags, q_i8, q_scale, k_i8, k_scale, k_mean, v_fp8,
                              v_scale, workspace, workspace_bytes, fused_q ? Route::kFusedQ : Route::kInt8, false))
    return rc;
  if (int rc = check_arch()) return rc;
  const bool fp8 = pv_mode == SAGE_PV_FP8;
  const bool smooth = (flags & SAGE_FLAG_SMOOTH_K) != 0;
  const int64_t qcs[3] = {heads_q * seq_q * head_dim, seq_q * head_dim, head_dim};  // contiguous Q codes
  const Codes16 c16{reinterpret_cast<__half*>(q_i8), qcs, reinterpret_cast<__half*>(k_i8)};
  return prepass_dispatch(dtype, head_dim, fused_q ? nullptr : q, k, fp8 ? v : nullptr, batch, heads_q, heads_kv,
                          seq_q, seq_kv, q_strides, k_strides, v_strides, q_multiplier(sm_scale, head_dim), smooth,
                          smooth && (flags & SAGE_FLAG_KM_GIVEN) != 0, fused_q ? nullptr : q_i8,
                          fused_q ? nullptr : q_scale, k_i8, k_scale, k_mean, fp8 ? v_fp8 : nullptr,
                          fp8 ? v_scale : nullptr, workspace, static_cast<cudaStream_t>(stream), nullptr,
                          codes16 ? &c16 : nullptr, qblk_of(flags));
}

int sage_run(const void* q, const void* k, const void* v, void* o, int dtype, int64_t batch, int64_t heads_q,
             int64_t heads_kv, int64_t seq_q, int64_t seq_kv, int64_t head_dim, const int64_t q_strides[3],
             const int64_t k_strides[3], const int64_t v_strides[3], const int64_t o_strides[3], int causal,
             float sm_scale, int pv_mode, unsigned flags, int8_t* q_i8, float* q_scale, int8_t* k_i8,
             float* k_scale, float* k_mean, uint8_t* v_fp8, float* v_scale, void* workspace,
             size_t workspace_bytes, void* stream) {
  g_last_error.clear();
  const Route route = run_route(flags, head_dim);
  if (int rc = check_run_args(q, k, v, dtype, batch, heads_q, heads_kv, seq_q, seq_kv, head_dim, q_strides,
                              k_strides, v_strides, pv_mode, flags, q_i8, q_scale, k_i8, k_scale, k_mean, v_fp8,
                              v_scale, workspace, workspace_bytes, route, true))
    return rc;
  if (causal && seq_q != seq_kv)
    return fail(SAGE_ERR_INVALID_ARG, "causal attention needs seq_q == seq_kv (got %lld, %lld)", (long long)seq_q,
                (long long)seq_kv);
  if (int rc = check_strides("o", o_strides)) return rc;
  if (!o || !aligned16(o)) return fail(SAGE_ERR_INVALID_ARG, "o must be a 16-byte aligned pointer");
  if (int rc = check_attn_alias(o, o_strides, tensor_span(o, o_strides, batch, heads_q, seq_q, head_dim, 2), q,
                                q_strides, tensor_span(q, q_strides, batch, heads_q, seq_q, head_dim, 2),
                                tensor_span(k, k_strides, batch, heads_kv, seq_kv, head_dim, 2),
                                tensor_span(v, v_strides, batch, heads_kv, seq_kv, head_dim, 2), batch, heads_q,
                                heads_kv, batch * seq_q, batch * seq_kv, cdiv(seq_q, qblk_of(flags)), cdiv(seq_kv, 64),
                                head_dim,
                                q_i8, q_scale, k_i8, k_scale, k_mean, pv_mode == SAGE_PV_FP8 ? v_fp8 : nullptr,
                                pv_mode == SAGE_PV_FP8 ? v_scale : nullptr, workspace, workspace_bytes))
    return rc;
  if (int rc = check_arch()) return rc;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  const bool fp8 = pv_mode == SAGE_PV_FP8;
  const bool smooth = (flags & SAGE_FLAG_SMOOTH_K) != 0;
  // head_dim 128 (or SAGE_FLAG_FUSED_Q): Q quantised by the attention kernel itself, the pre-pass
  // handles K (and V). head_dim 64: the pre-pass stores the codes as fp16 values, Q's in o (each
  // CTA reads its own query rows before it writes the same rows of o) and K's in the workspace
  // after the statistics, for the kernel's kind::f16 QK^T. SAGE_FLAG_PREPASS_Q: INT8 operands.
  const bool fused_q = route == Route::kFusedQ;
  const bool km_given = smooth && (flags & SAGE_FLAG_KM_GIVEN) != 0;
  const float q_mult = q_multiplier(sm_scale, head_dim);
  Codes16 c16{};
  if (route == Route::kCodes16) {
    const size_t off = stats_ws_bytes(batch, heads_kv, seq_kv, head_dim, pv_mode, km_given ? 0u : flags);
    c16 = Codes16{static_cast<__half*>(o), o_strides, reinterpret_cast<__half*>(static_cast<char*>(workspace) + off)};
  }
  const Codes16* cp = route == Route::kCodes16 ? &c16 : nullptr;
  if (int rc = prepass_dispatch(dtype, head_dim, fused_q ? nullptr : q, k, fp8 ? v : nullptr, batch, heads_q,
                                heads_kv, seq_q, seq_kv, q_strides, k_strides, v_strides, q_mult, smooth, km_given,
                                fused_q ? nullptr : q_i8, fused_q ? nullptr : q_scale, k_i8, k_scale, k_mean,
                                fp8 ? v_fp8 : nullptr, fp8 ? v_scale : nullptr, workspace, st, nullptr, cp,
                                qblk_of(flags)))
    return rc;
  const FusedQ fq{q, q_strides, q_mult, q_i8, q_scale};
  return attn_impl(q_i8, q_scale, k_i8, k_scale, fp8 ? static_cast<const void*>(v_fp8) : v, v_strides,
                   fp8 ? v_scale : nullptr, o, o_strides, dtype, pv_mode, causal, batch, heads_q, heads_kv, seq_q,
                   seq_kv, head_dim, st, nullptr, fused_q ? &fq : nullptr, cp, qblk_of(flags));
}

int sage_flash_attn_fwd(const void* q, const void* k, const void* v, void* o, int dtype, int64_t batch,
                        int64_t heads_q, int64_t heads_kv, int64_t seq_q, int64_t seq_kv, int64_t head_dim,
                        const int64_t q_strides[3], const int64_t k_strides[3], const int64_t v_strides[3],
                        const int64_t o_strides[3], int causal, float sm_scale, void* stream) {
  g_last_error.clear();
  if (int rc = check_shape(dtype, batch, heads_q, heads_kv, seq_q, seq_kv, head_dim)) return rc;
  if (causal && seq_q != seq_kv)
    return fail(SAGE_ERR_INVALID_ARG, "causal attention needs seq_q == seq_kv (got %lld, %lld)", (long long)seq_q,
                (long long)seq_kv);
  if (int rc = check_strides("q", q_strides)) return rc;
  if (int rc = check_strides("k", k_strides)) return rc;
  if (int rc = check_strides("v", v_strides)) return rc;
  if (int rc = check_strides("o", o_strides)) return rc;
  if (!q || !k || !v || !o) return fail(SAGE_ERR_INVALID_ARG, "NULL tensor pointer");
  if (!aligned16(q) || !aligned16(k) || !aligned16(v) || !aligned16(o))
    return fail(SAGE_ERR_INVALID_ARG, "q/k/v/o must be 16-byte aligned");
  if (int rc = check_attn_alias(o, o_strides, tensor_span(o, o_strides, batch, heads_q, seq_q, head_dim, 2), q,
                                q_strides, tensor_span(q, q_strides, batch, heads_q, seq_q, head_dim, 2),
                                tensor_span(k, k_strides, batch, heads_kv, seq_kv, head_dim, 2),
                                tensor_span(v, v_strides, batch, heads_kv, seq_kv, head_dim, 2), batch, heads_q,
                                heads_kv, batch * seq_q, batch * seq_kv, 0, 0, head_dim, nullptr, nullptr, nullptr,
                                nullptr, nullptr, nullptr, nullptr, nullptr, 0))
    return rc;
  if (int rc = check_arch()) return rc;
  return flash_impl(q, q_strides, k, k_strides, v, v_strides, o, o_strides, dtype, causal, batch, heads_q, heads_kv,
                    seq_q, seq_kv, head_dim, sm_scale, static_cast<cudaStream_t>(stream));
}

namespace {
// Shared validation of the variable-length entry points. The cu arrays live on the device and
// are not read here: the kernels clamp every sequence to [0, max_seq] rows inside the tokens.
int check_varlen(int dtype, int64_t batch, int64_t heads_q, int64_t heads_kv, int64_t total_q, int64_t total_kv,
                 int64_t max_seq_q, int64_t max_seq_kv, int64_t head_dim, const int32_t* cu_q, const int32_t* cu_kv) {
  if (int rc = check_shape(dtype, batch, heads_q, heads_kv, max_seq_q, max_seq_kv, head_dim)) return rc;
  if (total_q <= 0 || total_kv <= 0 || total_q > 0x7fffffffLL || total_kv > 0x7fffffffLL)
    return fail(SAGE_ERR_INVALID_ARG, "total_q=%lld / total_kv=%lld outside [1, 2^31)", (long long)total_q,
                (long long)total_kv);
  if (max_seq_q > total_q || max_seq_kv > total_kv)
    return fail(SAGE_ERR_INVALID_ARG, "max_seq_q=%lld / max_seq_kv=%lld exceed the token counts %lld / %lld",
                (long long)max_seq_q, (long long)max_seq_kv, (long long)total_q, (long long)total_kv);
  if (!cu_q || !cu_kv || (reinterpret_cast<uintptr_t>(cu_q) & 3u) || (reinterpret_cast<uintptr_t>(cu_kv) & 3u))
    return fail(SAGE_ERR_INVALID_ARG, "cu_seqlens_q / cu_seqlens_kv must be 4-byte aligned device pointers");
  return SAGE_OK;
}

// {head, token} strides of a packed tensor -> the {batch, head, seq} form used inside (batch 0).
int packed_strides(const char* name, const int64_t* s2, int64_t out[3]) {
  if (!s2) return fail(SAGE_ERR_INVALID_ARG, "%s strides are NULL", name);
  for (int i = 0; i < 2; ++i)
    if (s2[i] <= 0 || (s2[i] % 8) != 0)
      return fail(SAGE_ERR_INVALID_ARG, "%s stride[%d]=%lld must be a positive multiple of 8 elements", name, i,
                  (long long)s2[i]);
  out[0] = 0; out[1] = s2[0]; out[2] = s2[1];
  return SAGE_OK;
}
}  // namespace

int sage_per_block_int8_varlen(const void* q, const void* k, int dtype, int64_t batch, int64_t heads_q,
                               int64_t heads_kv, int64_t total_q, int64_t total_kv, int64_t max_seq_q,
                               int64_t max_seq_kv, int64_t head_dim, const int32_t* cu_seqlens_q,
                               const int32_t* cu_seqlens_kv, const int64_t q_strides[2], const int64_t k_strides[2],
                               float sm_scale, unsigned flags, int8_t* q_i8, float* q_scale, int8_t* k_i8,
                               float* k_scale, float* k_mean, void* workspace, size_t workspace_bytes, void* stream) {
  g_last_error.clear();
  if (int rc = check_varlen(dtype, batch, heads_q, heads_kv, total_q, total_kv, max_seq_q, max_seq_kv, head_dim,
                            cu_seqlens_q, cu_seqlens_kv))
    return rc;
  int64_t qs[3], ks[3];
  if (int rc = packed_strides("q", q_strides, qs)) return rc;
  if (int rc = packed_strides("k", k_strides, ks)) return rc;
  int qblk = 128;
  if (int rc = qblk_from_flags(flags, &qblk)) return rc;
  if (!q || !k || !q_i8 || !q_scale || !k_i8 || !k_scale) return fail(SAGE_ERR_INVALID_ARG, "NULL tensor pointer");
  if (!aligned16(q) || !aligned16(k) || !aligned16(q_i8) || !aligned16(k_i8))
    return fail(SAGE_ERR_INVALID_ARG, "q/k/q_i8/k_i8 must be 16-byte aligned");
  const bool smooth = (flags & SAGE_FLAG_SMOOTH_K) != 0;
  if (smooth && !k_mean) return fail(SAGE_ERR_INVALID_ARG, "SAGE_FLAG_SMOOTH_K needs k_mean");
  const bool km_given = smooth && (flags & SAGE_FLAG_KM_GIVEN) != 0;
  const size_t need = km_given ? 0 : stats_ws_bytes(batch, heads_kv, max_seq_kv, head_dim, SAGE_PV_16BIT, flags);
  if (need && (!workspace || workspace_bytes < need))
    return fail(SAGE_ERR_WORKSPACE, "workspace of %zu bytes needed, %zu given", need, workspace_bytes);
  if (int rc = check_arch()) return rc;
  const Varlen vl{cu_seqlens_q, cu_seqlens_kv, total_q, total_kv};
  return prepass_dispatch(dtype, head_dim, q, k, nullptr, batch, heads_q, heads_kv, max_seq_q, max_seq_kv, qs, ks,
                          nullptr, q_multiplier(sm_scale, head_dim), smooth, km_given, q_i8, q_scale, k_i8, k_scale,
                          k_mean, nullptr, nullptr, workspace, static_cast<cudaStream_t>(stream), &vl, nullptr, qblk);
}

int sage_run_varlen(const void* q, const void* k, const void* v, void* o, int dtype, int64_t batch, int64_t heads_q,
                    int64_t heads_kv, int64_t total_q, int64_t total_kv, int64_t max_seq_q, int64_t max_seq_kv,
                    int64_t head_dim, const int32_t* cu_seqlens_q, const int32_t* cu_seqlens_kv,
                    const int64_t q_strides[2], const int64_t k_strides[2], const int64_t v_strides[2],
                    const int64_t o_strides[2], int causal, float sm_scale, int pv_mode, unsigned flags,
                    int8_t* q_i8, float* q_scale, int8_t* k_i8, float* k_scale, float* k_mean, uint8_t* v_fp8,
                    float* v_scale, void* workspace, size_t workspace_bytes, void* stream) {
  g_last_error.clear();
  if (int rc = check_varlen(dtype, batch, heads_q, heads_kv, total_q, total_kv, max_seq_q, max_seq_kv, head_dim,
                            cu_seqlens_q, cu_seqlens_kv))
    return rc;
  int64_t qs[3], ks[3], vs[3], os[3];
  if (int rc = packed_strides("q", q_strides, qs)) return rc;
  if (int rc = packed_strides("k", k_strides, ks)) return rc;
  if (int rc = packed_strides("v", v_strides, vs)) return rc;
  if (int rc = packed_strides("o", o_strides, os)) return rc;
  if (pv_mode != SAGE_PV_16BIT && pv_mode != SAGE_PV_FP8)
    return fail(SAGE_ERR_INVALID_ARG, "pv_mode %d unknown", pv_mode);
  if ((flags & SAGE_FLAG_FUSED_Q) && (flags & SAGE_FLAG_PREPASS_Q))
    return fail(SAGE_ERR_INVALID_ARG, "SAGE_FLAG_FUSED_Q and SAGE_FLAG_PREPASS_Q exclude each other");
  int qblk = 128;
  if (int rc = qblk_from_flags(flags, &qblk)) return rc;
  const Route route = run_route(flags, head_dim);
  const bool fused_q = route == Route::kFusedQ;
  if (!q || !k || !v || !o || !k_scale || (route != Route::kCodes16 && !k_i8) ||
      (route == Route::kCodes16 && !q_scale) || (route == Route::kInt8 && (!q_i8 || !q_scale)) ||
      (fused_q && !q_i8 != !q_scale))
    return fail(SAGE_ERR_INVALID_ARG, "NULL tensor pointer");
  if (!aligned16(q) || !aligned16(k) || !aligned16(v) || !aligned16(o) || (q_i8 && !aligned16(q_i8)) ||
      (k_i8 && !aligned16(k_i8)))
    return fail(SAGE_ERR_INVALID_ARG, "q/k/v/o/q_i8/k_i8 must be 16-byte aligned");
  const bool smooth = (flags & SAGE_FLAG_SMOOTH_K) != 0;
  const bool fp8 = pv_mode == SAGE_PV_FP8;
  if (smooth && !k_mean) return fail(SAGE_ERR_INVALID_ARG, "SAGE_FLAG_SMOOTH_K needs k_mean");
  if (fp8 && (!v_fp8 || !v_scale || !aligned16(v_fp8)))
    return fail(SAGE_ERR_INVALID_ARG, "SAGE_PV_FP8 needs 16-byte aligned v_fp8 and v_scale");
  const bool km_given = smooth && (flags & SAGE_FLAG_KM_GIVEN) != 0;
  const size_t stats = stats_ws_bytes(batch, heads_kv, max_seq_kv, head_dim, pv_mode, km_given ? 0u : flags);
  // batch * max_seq_kv >= total_kv: the codes' region also holds the packed [Hkv, total_kv, D] codes
  const size_t need = stats + (route == Route::kCodes16 ? codes_ws_bytes(batch, heads_kv, max_seq_kv, head_dim) : 0);
  if (need && (!workspace || workspace_bytes < need))
    return fail(SAGE_ERR_WORKSPACE, "workspace of %zu bytes needed, %zu given", need, workspace_bytes);
  if (int rc = check_attn_alias(o, os, tensor_span(o, os, 1, heads_q, total_q, head_dim, 2), q, qs,
                                tensor_span(q, qs, 1, heads_q, total_q, head_dim, 2),
                                tensor_span(k, ks, 1, heads_kv, total_kv, head_dim, 2),
                                tensor_span(v, vs, 1, heads_kv, total_kv, head_dim, 2), batch, heads_q, heads_kv,
                                total_q, total_kv, cdiv(max_seq_q, qblk), cdiv(max_seq_kv, 64), head_dim, q_i8, q_scale,
                                k_i8, k_scale, k_mean, fp8 ? v_fp8 : nullptr, fp8 ? v_scale : nullptr, workspace,
                                workspace_bytes))
    return rc;
  if (int rc = check_arch()) return rc;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  const Varlen vl{cu_seqlens_q, cu_seqlens_kv, total_q, total_kv};
  const float q_mult = q_multiplier(sm_scale, head_dim);
  const Codes16 c16{static_cast<__half*>(o), os, reinterpret_cast<__half*>(static_cast<char*>(workspace) + stats)};
  const Codes16* cp = route == Route::kCodes16 ? &c16 : nullptr;
  if (int rc = prepass_dispatch(dtype, head_dim, fused_q ? nullptr : q, k, fp8 ? v : nullptr, batch, heads_q,
                                heads_kv, max_seq_q, max_seq_kv, qs, ks, vs, q_mult, smooth, km_given,
                                fused_q ? nullptr : q_i8, fused_q ? nullptr : q_scale, k_i8, k_scale, k_mean,
                                fp8 ? v_fp8 : nullptr, fp8 ? v_scale : nullptr, workspace, st, &vl, cp, qblk))
    return rc;
  const FusedQ fq{q, qs, q_mult, q_i8, q_scale};
  return attn_impl(q_i8, q_scale, k_i8, k_scale, fp8 ? static_cast<const void*>(v_fp8) : v, vs,
                   fp8 ? v_scale : nullptr, o, os, dtype, pv_mode, causal, batch, heads_q, heads_kv, max_seq_q,
                   max_seq_kv, head_dim, st, &vl, fused_q ? &fq : nullptr, cp, qblk);
}

int sage_flash_attn_varlen_fwd(const void* q, const void* k, const void* v, void* o, int dtype, int64_t batch,
                               int64_t heads_q, int64_t heads_kv, int64_t total_q, int64_t total_kv,
                               int64_t max_seq_q, int64_t max_seq_kv, int64_t head_dim, const int32_t* cu_seqlens_q,
                               const int32_t* cu_seqlens_kv, const int64_t q_strides[2], const int64_t k_strides[2],
                               const int64_t v_strides[2], const int64_t o_strides[2], int causal, float sm_scale,
                               void* stream) {
  g_last_error.clear();
  if (int rc = check_varlen(dtype, batch, heads_q, heads_kv, total_q, total_kv, max_seq_q, max_seq_kv, head_dim,
                            cu_seqlens_q, cu_seqlens_kv))
    return rc;
  int64_t qs[3], ks[3], vs[3], os[3];
  if (int rc = packed_strides("q", q_strides, qs)) return rc;
  if (int rc = packed_strides("k", k_strides, ks)) return rc;
  if (int rc = packed_strides("v", v_strides, vs)) return rc;
  if (int rc = packed_strides("o", o_strides, os)) return rc;
  if (!q || !k || !v || !o) return fail(SAGE_ERR_INVALID_ARG, "NULL tensor pointer");
  if (!aligned16(q) || !aligned16(k) || !aligned16(v) || !aligned16(o))
    return fail(SAGE_ERR_INVALID_ARG, "q/k/v/o must be 16-byte aligned");
  if (int rc = check_attn_alias(o, os, tensor_span(o, os, 1, heads_q, total_q, head_dim, 2), q, qs,
                                tensor_span(q, qs, 1, heads_q, total_q, head_dim, 2),
                                tensor_span(k, ks, 1, heads_kv, total_kv, head_dim, 2),
                                tensor_span(v, vs, 1, heads_kv, total_kv, head_dim, 2), batch, heads_q, heads_kv,
                                total_q, total_kv, 0, 0, head_dim, nullptr, nullptr, nullptr, nullptr, nullptr, nullptr,
                                nullptr, nullptr, 0))
    return rc;
  if (int rc = check_arch()) return rc;
  const Varlen vl{cu_seqlens_q, cu_seqlens_kv, total_q, total_kv};
  return flash_impl(q, qs, k, ks, v, vs, o, os, dtype, causal, batch, heads_q, heads_kv, max_seq_q, max_seq_kv,
                    head_dim, sm_scale, static_cast<cudaStream_t>(stream), &vl);
}

int sage_device_status(int* status_bits, void* stream) {
  g_last_error.clear();
  if (!status_bits) return fail(SAGE_ERR_INVALID_ARG, "status_bits is NULL");
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  SAGE_CUDA_TRY(cudaStreamSynchronize(st));
  int v = 0;
  SAGE_CUDA_TRY(cudaMemcpyFromSymbol(&v, sage::g_dev_status, sizeof(int)));
  const int zero = 0;
  SAGE_CUDA_TRY(cudaMemcpyToSymbol(sage::g_dev_status, &zero, sizeof(int)));
  *status_bits = v;
  if (v) return fail(SAGE_ERR_TIMEOUT, "device-side wait timed out (status bits 0x%x)", v);
  return SAGE_OK;
}

int sage_watchdog_selftest(unsigned limit_us, void* stream) {
  g_last_error.clear();
  if (int rc = check_arch()) return rc;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  watchdog_selftest_kernel<<<1, 32, 0, st>>>(static_cast<unsigned long long>(limit_us) * 1000ull);
  SAGE_CUDA_TRY(cudaGetLastError());
  return SAGE_OK;
}

#ifdef SAGE_TIMING
// Profiling build only: copy the per-warp phase timers of the last attention launches.
int sage_debug_phase_cycles(unsigned long long* host, size_t count) {
  const size_t n = count < sizeof(sage::g_phase_cycles) / 8 ? count : sizeof(sage::g_phase_cycles) / 8;
  SAGE_CUDA_TRY(cudaMemcpyFromSymbol(host, sage::g_phase_cycles, n * 8));
  return SAGE_OK;
}
#endif

}  // extern "C"
