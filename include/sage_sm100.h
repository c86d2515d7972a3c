/*
 * sage_sm100.h — C ABI of libsage_sm100.so, the B200 (sm_100a) implementation of
 * TriBench's sage_attn path (SageAttention-style INT8-QK attention).
 *
 * Everything here is plain C: pointers, sizes and status codes. No C++ exception and
 * no framework type crosses this boundary. The caller owns every buffer (inputs,
 * outputs, workspace); the hot path allocates nothing. Every call is asynchronous on the
 * CUDA stream passed as `stream` (a cudaStream_t, or NULL for the legacy default stream).
 *
 * Tensor convention (the reference's "HND" layout, kernels/sage_attn/triton_impl.py:42-48):
 *   a logical [B, H, S, D] tensor whose last dimension is contiguous, described by three
 *   element strides {batch, head, seq}. The reference's "NHD" layout ([B, S, H, D],
 *   triton_impl.py:49-55) is the same logical tensor with strides {S*H*D, D, H*D}.
 *   Base pointers must be 16-byte aligned and strides multiples of 8 elements (16 bytes);
 *   head_dim must be 64 or 128.
 *
 * Quantised intermediates, all owned by the caller and always contiguous:
 *   q_i8    int8  [B, Hq,  Sq,  D]      per-block INT8 Q (sm_scale*log2(e) folded in), blocks of
 *                                       BLKQ = 128 rows unless SAGE_FLAG_QBLK_* says otherwise
 *   q_scale fp32  [B, Hq,  ceil(Sq/BLKQ)]
 *   k_i8    int8  [B, Hkv, Skv, D]      per-64-row-block INT8 K (after optional smoothing)
 *   k_scale fp32  [B, Hkv, ceil(Skv/64)]
 *   k_mean  fp32  [B, Hkv, D]           per-channel token mean of K (smoothing only)
 *   v_fp8   e4m3  [B, Hkv, Skv, D]      per-channel scaled V (FP8 P.V mode only)
 *   v_scale fp32  [B, Hkv, D]
 *
 * Output aliasing: every entry point that writes an attention output o rejects, with
 * SAGE_ERR_INVALID_ARG and before any CUDA call, an o whose bytes overlap k, v, an
 * intermediate or the workspace, or overlap q other than as the identical view (same base
 * pointer and strides; in place, o = q, is allowed). The check compares the byte ranges the
 * tensors span, so an o interleaved with k or v inside one packed buffer is rejected too.
 *
 * Output placement: o may be memory of the calling GPU, another GPU's memory mapped into
 * this one (CUDA IPC or peer access over NVLink: each GPU of a multi-GPU job writes its rows
 * straight into one GPU's output buffer), or mapped pinned host memory. When o is not memory of
 * the current device (cudaPointerGetAttributes), the attention epilogue stages each half tile
 * in shared memory and writes whole 128-byte lines, which NVLink carries far better than one
 * row's 16-byte pieces; results are bit-identical either way.
 */
#ifndef SAGE_SM100_H_
#define SAGE_SM100_H_

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define SAGE_ABI_VERSION 2

/* Status codes. 0 is success; everything else is negative. */
#define SAGE_OK                    0
#define SAGE_ERR_INVALID_ARG      -1  /* shape, stride, dtype, alignment or size rejected  */
#define SAGE_ERR_UNSUPPORTED_ARCH -2  /* device is not sm_100 (B200/GB200)                  */
#define SAGE_ERR_CUDA             -3  /* a CUDA runtime/driver call failed                  */
#define SAGE_ERR_TIMEOUT          -4  /* a device-side wait hit its limit (see status API)  */
#define SAGE_ERR_WORKSPACE        -5  /* workspace pointer NULL or smaller than required    */

/* Element types of q/k/v/o. */
#define SAGE_DTYPE_F16  0
#define SAGE_DTYPE_BF16 1

/* P.V modes. */
#define SAGE_PV_16BIT 0   /* P and V in the input's 16-bit type, fp32 accumulation in TMEM */
#define SAGE_PV_FP8   1   /* P and V in FP8 e4m3, per-channel V scales, fp32 accumulation  */

/* Quantisation flags. */
#define SAGE_FLAG_SMOOTH_K 1u  /* subtract K's per-channel token mean before quantising */
#define SAGE_FLAG_KM_GIVEN 2u  /* with SMOOTH_K: k_mean is an input supplied by the caller
                                  (the reference's `km` argument) instead of being computed */
#define SAGE_FLAG_FUSED_Q  4u  /* Q is quantised by the attention kernel itself (bit-identical
                                  codes and output), not by the pre-pass: sage_run /
                                  sage_run_varlen do this at head_dim 128 anyway and with this
                                  flag at 64 too, q_i8 / q_scale then being optional outputs
                                  (both NULL: not stored); sage_prepass with it skips Q, for
                                  sage_attn_fwd_fused_q to follow */
#define SAGE_FLAG_PREPASS_Q 8u /* sage_run / sage_run_varlen: INT8 operands from the pre-pass
                                  (q_i8 / k_i8 required) at either head_dim: exactly
                                  sage_prepass + sage_attn_fwd */
#define SAGE_FLAG_CODES16  16u /* sage_prepass only, head_dim 64: q_i8 / k_i8 receive the codes
                                  as fp16 values (2 bytes each: buffers of twice the size, same
                                  layouts), for sage_attn_fwd_codes16 */

/* Q scale block size: per_block_int8's BLKQ argument (kernels/sage_attn/triton_impl.py:35, 57,
 * 63), a 3-bit field of `flags`. One fp32 scale per BLKQ query rows: q_scale is
 * [B, Hq, ceil(Sq / BLKQ)]. The default, 128 rows, is the reference's default and the one its
 * attention kernel assumes (run_sage_attn, triton_impl.py:166); the finer blocks trade nothing
 * in the attention kernel (each softmax thread owns one query row and reads that row's scale)
 * for smaller INT8 rounding errors on rows with outliers. The attention entry points take the
 * same field, so that they read the scales the pre-pass wrote. */
#define SAGE_FLAG_QBLK_MASK 0x700u
#define SAGE_FLAG_QBLK_128  0x000u  /* 128-row blocks (default) */
#define SAGE_FLAG_QBLK_64   0x100u
#define SAGE_FLAG_QBLK_32   0x200u
#define SAGE_FLAG_QBLK_16   0x300u
#define SAGE_FLAG_QBLK_1    0x400u  /* one scale per token */

/* Device-side status bits reported by sage_device_status(). */
#define SAGE_DEV_TIMEOUT_PRODUCER 0x1
#define SAGE_DEV_TIMEOUT_MMA      0x2
#define SAGE_DEV_TIMEOUT_SOFTMAX  0x4
#define SAGE_DEV_TIMEOUT_EPILOGUE 0x8

/* ABI version of the loaded library (SAGE_ABI_VERSION at build time). */
int sage_abi_version(void);

/* Message of the last failing call on this host thread ("" when none). */
const char* sage_last_error(void);

/*
 * Bytes of scratch that sage_run needs for these sizes: the K-mean and V-absmax partial sums
 * (0 when neither smoothing nor the FP8 P.V mode is requested) and, at head_dim 64 unless flags
 * hold SAGE_FLAG_PREPASS_Q or SAGE_FLAG_FUSED_Q, K's codes as fp16 values (2 bytes per K
 * element). sage_per_block_int8, sage_prepass and sage_quant_v_fp8 need the partial sums only;
 * this size serves them too.
 */
size_t sage_workspace_bytes(int64_t batch, int64_t heads_kv, int64_t seq_kv, int64_t head_dim,
                            int pv_mode, unsigned flags);

/*
 * Quantise Q and K (and, with SAGE_FLAG_SMOOTH_K, smooth K first).
 * Replaces per_block_int8(q, k, km, BLKQ=128, BLKK=64, sm_scale, tensor_layout)
 *   — kernels/sage_attn/triton_impl.py:35-82, kernel quant_per_block_int8_kernel :7-33.
 * Q is multiplied by fp32(sm_scale * 1.44269504) (triton_impl.py:69); sm_scale <= 0 means
 * head_dim**-0.5 (triton_impl.py:60-61). K uses multiplier 1.0 (triton_impl.py:79).
 * k_mean may be NULL unless SAGE_FLAG_SMOOTH_K is set; it is written (the per-channel mean
 * is computed here) unless SAGE_FLAG_KM_GIVEN is also set, in which case it is read.
 * The reference never passes km (triton_impl.py:171-173); given an fp32 km it evaluates
 * k - km in fp32 exactly as here.
 */
int sage_per_block_int8(const void* q, const void* k, int dtype,
                        int64_t batch, int64_t heads_q, int64_t heads_kv,
                        int64_t seq_q, int64_t seq_kv, int64_t head_dim,
                        const int64_t q_strides[3], const int64_t k_strides[3],
                        float sm_scale, unsigned flags,
                        int8_t* q_i8, float* q_scale, int8_t* k_i8, float* k_scale,
                        float* k_mean, void* workspace, size_t workspace_bytes, void* stream);

/*
 * sage_per_block_int8 without a workspace argument, for callers that cannot allocate device
 * memory themselves: code whose device memory is owned by someone else (a host framework or
 * inference server that hands out only its own buffers), or that must not call cudaMalloc /
 * cudaFree because those may synchronise the device. The smoothing statistics use a scratch
 * array compiled into the library (4 MiB, held on every GPU that loads the library until the
 * process exits); sizes needing more (batch * heads_kv * ceil(seq_kv / 512) * head_dim above
 * 524288) are rejected with SAGE_ERR_INVALID_ARG. The caller still passes every input and
 * output. The first call on a device looks up the scratch's device address (no allocation),
 * so make that first call before any stream capture. The address is cached per device ordinal
 * for the life of the process: after cudaDeviceReset (which destroys the context holding the
 * array) the cached address is stale, so do not call this entry point again in that process.
 * Every call on a device shares the one scratch array: calls that overlap on the GPU (other
 * streams, other threads) race and must be serialised by the caller. No counterpart in the
 * reference.
 */
int sage_per_block_int8_noalloc(const void* q, const void* k, int dtype,
                                int64_t batch, int64_t heads_q, int64_t heads_kv,
                                int64_t seq_q, int64_t seq_kv, int64_t head_dim,
                                const int64_t q_strides[3], const int64_t k_strides[3],
                                float sm_scale, unsigned flags,
                                int8_t* q_i8, float* q_scale, int8_t* k_i8, float* k_scale,
                                float* k_mean, void* stream);

/*
 * Quantise V to FP8 e4m3 with one scale per (batch, head, channel):
 * v_scale = max_s |v| / 448, v_fp8 = e4m3_rn_satfinite(v / v_scale).
 * No counterpart in the reference (its P.V runs in fp16, triton_impl.py:111-113); it is
 * the FP8 P.V extension of the same kernel pack.
 */
int sage_quant_v_fp8(const void* v, int dtype, int64_t batch, int64_t heads_kv, int64_t seq_kv,
                     int64_t head_dim, const int64_t v_strides[3],
                     uint8_t* v_fp8, float* v_scale, void* workspace, size_t workspace_bytes,
                     void* stream);

/*
 * Fused attention over the quantised operands.
 * Replaces the _attn_fwd launch (kernels/sage_attn/triton_impl.py:121-160, inner loop
 * :86-119, grid :186-199): S = dequant(q_i8 . k_i8^T), online softmax in base 2,
 * O = softmax . V, O stored in the input dtype. Unlike the reference Triton kernel,
 * `causal` is honoured (key j visible to query i iff j <= i; requires seq_q == seq_kv,
 * like reference.py:19-22). v is the 16-bit V ({batch, head, seq} strides v_strides)
 * for SAGE_PV_16BIT, or v_fp8 (contiguous) with v_scale for SAGE_PV_FP8.
 * GQA: heads_q % heads_kv == 0, query head h reads KV head h / (heads_q / heads_kv).
 * flags: only the SAGE_FLAG_QBLK_* field (the Q scale block size q_scale was written with);
 * any other bit is rejected. (ABI version 2 added this argument.)
 */
int sage_attn_fwd(const int8_t* q_i8, const float* q_scale, const int8_t* k_i8,
                  const float* k_scale, const void* v, const int64_t v_strides[3],
                  const float* v_scale, void* o, const int64_t o_strides[3],
                  int dtype, int pv_mode, int causal, unsigned flags,
                  int64_t batch, int64_t heads_q, int64_t heads_kv,
                  int64_t seq_q, int64_t seq_kv, int64_t head_dim, void* stream);

/*
 * sage_attn_fwd over INT8 codes held as fp16 values (head_dim 64 only; from sage_prepass with
 * SAGE_FLAG_CODES16): QK^T runs as a kind::f16 MMA, whose fp32 scores equal the INT8 MMA's
 * (every partial sum is an integer below 2^24), with no int32 -> float step in the softmax.
 * q_c16 [B, Hq, Sq, 64] and k_c16 [B, Hkv, Skv, 64] contiguous fp16. This is the second half of
 * sage_run at head_dim 64 (which keeps the Q codes in o and the K codes in its workspace).
 * flags: the SAGE_FLAG_QBLK_* field only, as for sage_attn_fwd.
 */
int sage_attn_fwd_codes16(const void* q_c16, const float* q_scale, const void* k_c16, const float* k_scale,
                          const void* v, const int64_t v_strides[3], const float* v_scale, void* o,
                          const int64_t o_strides[3], int dtype, int pv_mode, int causal, unsigned flags,
                          int64_t batch, int64_t heads_q, int64_t heads_kv, int64_t seq_q, int64_t seq_kv,
                          int64_t head_dim, void* stream);

/*
 * sage_attn_fwd with the Q quantisation inside the kernel: each CTA's softmax warps load their
 * 128-row tiles of the caller's 16-bit q ({batch, head, seq} strides q_strides), quantise them
 * exactly as sage_per_block_int8 does (multiplier sm_scale * log2 e, sm_scale <= 0 meaning
 * head_dim^-0.5) straight into shared memory, and attend. q_i8_out / q_scale_out, both NULL or
 * both set, receive the codes and scales in sage_per_block_int8's layouts. This is the second
 * half of sage_run at head_dim 128 (its first half: sage_prepass with SAGE_FLAG_FUSED_Q).
 * flags: the SAGE_FLAG_QBLK_* field only: the Q blocks quantised here (finer blocks are reduced
 * over the rows of each block inside the 128-row tile; codes and scales bit-identical to
 * sage_per_block_int8 with the same field).
 * Replaces per_block_int8's Q half + the _attn_fwd launch (triton_impl.py:62-72, 121-160).
 */
int sage_attn_fwd_fused_q(const void* q, const int64_t q_strides[3], float sm_scale, const int8_t* k_i8,
                          const float* k_scale, const void* v, const int64_t v_strides[3], const float* v_scale,
                          void* o, const int64_t o_strides[3], int dtype, int pv_mode, int causal,
                          unsigned flags, int64_t batch, int64_t heads_q, int64_t heads_kv, int64_t seq_q,
                          int64_t seq_kv, int64_t head_dim, int8_t* q_i8_out, float* q_scale_out, void* stream);

/*
 * The pre-pass half of sage_run on its own: K smoothing statistics, INT8 Q/K and (for
 * SAGE_PV_FP8) e4m3 V, in the same launches sage_run makes. Together with sage_attn_fwd it
 * is exactly sage_run at head_dim 64; with SAGE_FLAG_FUSED_Q it leaves Q out (q_i8 / q_scale
 * may be NULL) and together with sage_attn_fwd_fused_q is exactly sage_run at head_dim 128.
 * Callers use the split to time or overlap the two halves.
 * Replaces per_block_int8 + v.to(float16) of run_sage_attn (triton_impl.py:171-173, 189).
 */
int sage_prepass(const void* q, const void* k, const void* v, int dtype,
                 int64_t batch, int64_t heads_q, int64_t heads_kv,
                 int64_t seq_q, int64_t seq_kv, int64_t head_dim,
                 const int64_t q_strides[3], const int64_t k_strides[3], const int64_t v_strides[3],
                 float sm_scale, int pv_mode, unsigned flags,
                 int8_t* q_i8, float* q_scale, int8_t* k_i8, float* k_scale, float* k_mean,
                 uint8_t* v_fp8, float* v_scale, void* workspace, size_t workspace_bytes,
                 void* stream);

/*
 * Whole path in one call: quantise (+ smooth, + V to FP8) then attend.
 * Replaces run_sage_attn(q, k, v, causal, sm_scale) — kernels/sage_attn/triton_impl.py:162-200.
 * The caller provides every intermediate buffer listed at the top of this header
 * (v_fp8/v_scale only for SAGE_PV_FP8, k_mean only with SAGE_FLAG_SMOOTH_K) and a workspace
 * of at least sage_workspace_bytes(...) bytes. At head_dim 128 (or with SAGE_FLAG_FUSED_Q) Q
 * is quantised inside the attention kernel (sage_prepass with SAGE_FLAG_FUSED_Q, then
 * sage_attn_fwd_fused_q) and q_i8 / q_scale are optional outputs; the result is bit-identical
 * to the pre-pass route (sage_prepass + sage_attn_fwd). At head_dim 64 (unless a flag above
 * says otherwise) the pre-pass stores the codes as fp16 values, Q's in o itself (each CTA
 * reads its own query rows before it writes the same rows of o; o overlapping k or v is
 * rejected, see "Output aliasing" above) and K's in the workspace, and QK^T runs on them as a kind::f16 MMA (sage_prepass with
 * SAGE_FLAG_CODES16 + sage_attn_fwd_codes16): q_i8 / k_i8 are then not used (may be NULL), the
 * scores are the INT8 MMA's exactly, and the output matches the INT8 route to float rounding.
 */
int sage_run(const void* q, const void* k, const void* v, void* o, int dtype,
             int64_t batch, int64_t heads_q, int64_t heads_kv,
             int64_t seq_q, int64_t seq_kv, int64_t head_dim,
             const int64_t q_strides[3], const int64_t k_strides[3],
             const int64_t v_strides[3], const int64_t o_strides[3],
             int causal, float sm_scale, int pv_mode, unsigned flags,
             int8_t* q_i8, float* q_scale, int8_t* k_i8, float* k_scale, float* k_mean,
             uint8_t* v_fp8, float* v_scale, void* workspace, size_t workspace_bytes,
             void* stream);

/*
 * Unquantised attention with the same pipeline, for TriBench's flash_attn pack.
 * Replaces run_flash_attn(q, k, v, causal, sm_scale) — kernels/flash_attn/triton_impl.py:110-128
 * (its kernel: :13-108). q/k/v/o fp16 or bf16 (dtype), [batch, heads, seq, head_dim] with
 * element strides, last dimension contiguous; head_dim 64 or 128; heads_q a multiple of
 * heads_kv (GQA). O = softmax(Q K^T * sm_scale [causal: key <= query]) V, sm_scale <= 0 meaning
 * head_dim^-0.5; QK^T and P.V on the tensor cores with fp32 accumulation, P in the input dtype,
 * softmax in fp32. Allocates nothing; runs on `stream`.
 */
int sage_flash_attn_fwd(const void* q, const void* k, const void* v, void* o, int dtype,
                        int64_t batch, int64_t heads_q, int64_t heads_kv,
                        int64_t seq_q, int64_t seq_kv, int64_t head_dim,
                        const int64_t q_strides[3], const int64_t k_strides[3],
                        const int64_t v_strides[3], const int64_t o_strides[3],
                        int causal, float sm_scale, void* stream);

/*
 * Variable-length batches (packed sequences). `batch` sequences of different lengths are packed
 * along one token axis, flash-attention style: q is [total_q, heads_q, head_dim] (any head and
 * token strides, head_dim contiguous), k/v are [total_kv, heads_kv, head_dim], and sequence b
 * owns token rows [cu_seqlens_q[b], cu_seqlens_q[b+1]) of q / o and [cu_seqlens_kv[b],
 * cu_seqlens_kv[b+1]) of k / v. cu_seqlens_* are int32 DEVICE arrays of batch + 1 prefix sums
 * starting at 0; max_seq_q / max_seq_kv bound every sequence's length (the launches are sized
 * from them; the kernels clamp a longer or malformed sequence to these bounds and to the token
 * counts, so no access leaves the buffers). Strides are {head, token} element strides.
 * Every sequence is quantised and attended on its own, exactly as a dense batch of one:
 * Q blocks of 128 rows and K blocks of 64 rows start at each sequence's first token, and the
 * smoothing mean is per (sequence, head). Packed intermediates and per-sequence scales:
 *   q_i8    int8  [heads_q,  total_q,  head_dim]   q_scale fp32 [batch, heads_q,  ceil(max_seq_q/128)]
 *   k_i8    int8  [heads_kv, total_kv, head_dim]   k_scale fp32 [batch, heads_kv, ceil(max_seq_kv/64)]
 *   k_mean  fp32  [batch, heads_kv, head_dim]
 *   v_fp8   e4m3  [heads_kv, total_kv, head_dim]   v_scale fp32 [batch, heads_kv, head_dim]
 * Scale entries past a sequence's own block count are not written. A sequence with query rows
 * but no keys gets O = 0 (softmax over an empty key set in the reference's matmuls). causal
 * masks key j of a sequence for its query i iff j > i (lengths should match per sequence).
 * Workspace: sage_workspace_bytes(batch, heads_kv, max_seq_kv, head_dim, pv_mode, flags).
 * The reference has no packed-sequence entry point; these extend per_block_int8 and
 * run_sage_attn (kernels/sage_attn/triton_impl.py:35-82, :162-200) and run_flash_attn
 * (kernels/flash_attn/triton_impl.py:110-128) to packed batches, one sequence at a time.
 */
int sage_per_block_int8_varlen(const void* q, const void* k, int dtype, int64_t batch, int64_t heads_q,
                               int64_t heads_kv, int64_t total_q, int64_t total_kv, int64_t max_seq_q,
                               int64_t max_seq_kv, int64_t head_dim, const int32_t* cu_seqlens_q,
                               const int32_t* cu_seqlens_kv, const int64_t q_strides[2], const int64_t k_strides[2],
                               float sm_scale, unsigned flags, int8_t* q_i8, float* q_scale, int8_t* k_i8,
                               float* k_scale, float* k_mean, void* workspace, size_t workspace_bytes, void* stream);

int sage_run_varlen(const void* q, const void* k, const void* v, void* o, int dtype, int64_t batch, int64_t heads_q,
                    int64_t heads_kv, int64_t total_q, int64_t total_kv, int64_t max_seq_q, int64_t max_seq_kv,
                    int64_t head_dim, const int32_t* cu_seqlens_q, const int32_t* cu_seqlens_kv,
                    const int64_t q_strides[2], const int64_t k_strides[2], const int64_t v_strides[2],
                    const int64_t o_strides[2], int causal, float sm_scale, int pv_mode, unsigned flags,
                    int8_t* q_i8, float* q_scale, int8_t* k_i8, float* k_scale, float* k_mean, uint8_t* v_fp8,
                    float* v_scale, void* workspace, size_t workspace_bytes, void* stream);

int sage_flash_attn_varlen_fwd(const void* q, const void* k, const void* v, void* o, int dtype, int64_t batch,
                               int64_t heads_q, int64_t heads_kv, int64_t total_q, int64_t total_kv,
                               int64_t max_seq_q, int64_t max_seq_kv, int64_t head_dim, const int32_t* cu_seqlens_q,
                               const int32_t* cu_seqlens_kv, const int64_t q_strides[2], const int64_t k_strides[2],
                               const int64_t v_strides[2], const int64_t o_strides[2], int causal, float sm_scale,
                               void* stream);

/*
 * Synchronise `stream`, then read and clear the device-side status word of the current
 * device (SAGE_DEV_* bits; 0 = no wait ran out). Returns SAGE_OK, or SAGE_ERR_TIMEOUT
 * when any bit was set, or SAGE_ERR_CUDA.
 */
int sage_device_status(int* status_bits, void* stream);

/*
 * Test hook for the watchdog: launches the attention pipeline's bounded mbarrier wait
 * on a barrier that nothing completes, with the given limit in microseconds. The wait
 * gives up, sets SAGE_DEV_TIMEOUT_EPILOGUE and the kernel returns normally, leaving the
 * context usable. No counterpart in the reference.
 */
int sage_watchdog_selftest(unsigned limit_us, void* stream);

#ifdef __cplusplus
}
#endif

#endif /* SAGE_SM100_H_ */
