/*
 * sm100_peaks.h — C ABI of libsm100_peaks.so, a dense tcgen05 throughput microbenchmark for
 * B200 (sm_100a). It measures, on the machine the sage path runs on, the tensor-core rates that
 * the attention kernel's roofline divides by: kind::i8 (QK^T), kind::f16 (16-bit P.V and the
 * flash_attn pack) and kind::f8f6f4 with e4m3 operands (FP8 P.V).
 *
 * No counterpart in the reference: TriBench has no peak measurement for this path; its
 * BenchResult only reports TFLOP/s from `estimate` (tribench/bench.py:178-180).
 */
#ifndef SM100_PEAKS_H_
#define SM100_PEAKS_H_

#ifdef __cplusplus
extern "C" {
#endif

#define SM100_PEAK_OK               0
#define SM100_PEAK_ERR_INVALID_ARG -1
#define SM100_PEAK_ERR_CUDA        -3

/* Operand kinds. */
#define SM100_PEAK_I8   0  /* tcgen05.mma kind::i8, s8 x s8 -> s32, K = 32 per MMA        */
#define SM100_PEAK_F16  1  /* tcgen05.mma kind::f16, f16 x f16 -> f32, K = 16 per MMA      */
#define SM100_PEAK_E4M3 2  /* tcgen05.mma kind::f8f6f4, e4m3 x e4m3 -> f32, K = 32 per MMA */

/* Message of the last failing call on this host thread ("" when none). */
const char* sm100_peak_last_error(void);

/* Multiply-add operations (2 per MAC) of one M128 x n MMA of `kind`; 0 for an unknown kind or n. */
double sm100_peak_ops_per_mma(int kind, int n);

/*
 * Launch `ctas` CTAs (one per SM: pass the SM count) on `stream`; each issues `mma_per_cta`
 * (a multiple of 4) dense M128 x n MMAs (n = 64, 128 or 256) of `kind` from shared-memory
 * operands into TMEM, back to back. Total work = ctas * mma_per_cta * sm100_peak_ops_per_mma.
 * `status` is a device int the kernel ORs with 1 (and 2) if its bounded wait for the MMAs ran
 * past `limit_ms`; the kernel then still frees TMEM and returns. `timing` (device, nullable,
 * 2 * ctas values) receives per CTA the SM cycles (clock64) and the nanoseconds (globaltimer)
 * from its first MMA issue to the completion of its last MMA, from which the caller gets the
 * rate per SM clock and the clock itself. Asynchronous; the caller times it with CUDA events
 * on `stream`.
 */
int sm100_tensor_peak_launch(int kind, int n, int ctas, long long mma_per_cta, unsigned seed,
                             unsigned limit_ms, int* status, long long* timing, void* stream);

#ifdef __cplusplus
}
#endif

#endif /* SM100_PEAKS_H_ */
