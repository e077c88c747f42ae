/*
 * wbk.h — C ABI of libwbk.so, the B200 (sm_100a) kernels behind the
 * `whisper_blaze_kernels` op surface of whisper-blaze.
 *
 * Conventions
 *   - Every entry point is asynchronous on `stream` (a cudaStream_t / CUstream;
 *     NULL = legacy default stream) and runs on the CURRENT CUDA device. All
 *     pointers are device pointers unless a parameter says "host".
 *   - Return value: WBK_OK (0) or a WBK_ERR_* code; wbk_last_error() returns a
 *     thread-local human-readable message for the most recent failure.
 *   - Argument errors are detected on the host before anything is launched,
 *     so a failing call never leaves partial work on the stream.
 *   - fp16 = IEEE binary16, fp8 = OCP E4M3FN / E5M2 bytes (uint8 storage).
 *   - No entry point allocates memory or synchronises the device, except
 *     wbk_device_error() which reads a flag back (it synchronises).
 *
 * Citations are to the reference project techbysaurabh/whisper-blaze v0.1.17.
 */
#ifndef WBK_H_
#define WBK_H_

#include <stdint.h>
#include <stddef.h>

#ifdef __cplusplus
extern "C" {
#endif

typedef struct CUstream_st* wbk_stream_t;

/* status codes */
#define WBK_OK                   0
#define WBK_ERR_INVALID_ARG      1   /* bad pointer / size / alignment / enum */
#define WBK_ERR_UNSUPPORTED      2   /* shape or device outside what the kernel supports */
#define WBK_ERR_CUDA             3   /* a CUDA runtime/driver call failed */
#define WBK_ERR_DEVICE_TIMEOUT   4   /* a bounded device-side wait gave up (see wbk_device_error) */

/* fp8 formats */
#define WBK_FMT_E4M3 0
#define WBK_FMT_E5M2 1

/* GEMM epilogues */
#define WBK_EPI_NONE          0   /* out = fp16(acc*descale [+ bias]) */
#define WBK_EPI_GELU          1   /* out = fp16(gelu_erf(acc*descale + bias)) */
#define WBK_EPI_RESIDUAL      2   /* out = fp16(acc*descale + bias + residual) */
#define WBK_EPI_RESIDUAL_CLAMP 3  /* as RESIDUAL, then clamp to +-(65504-1000) (HF fp16 encoder clamp) */
#define WBK_EPI_BIAS_MAXKEY   4   /* as NONE; out_amax_bits (required) max-accumulates the order key of the
                                     largest fp16 output, for wbk_quantise_gelu_f16 */

/* ---------------------------------------------------------------- misc */

/* Library ABI version (major*10000 + minor*100 + patch). */
int wbk_version(void);

/* Thread-local message describing the last failing call on this thread. */
const char* wbk_last_error(void);

/* Read (and clear) the device-side error word of the current device that the
 * bounded waits inside the GEMM kernel set when they give up. Synchronises the
 * current device. *code_out = 0 when no device-side error happened. */
int wbk_device_error(uint32_t* code_out);

/* Sets the wall-clock limit of every bounded device-side wait (GEMM, skinny
 * GEMM, attention, in-kernel quantise arrivals) for launches made after this
 * call, on every device; 0 restores the default (WBK_WAIT_TIMEOUT_MS, else
 * 4 s). At most 60 s. A wait that runs out records WBK_ERR_DEVICE_TIMEOUT in
 * the device error word and the kernel returns early, so a very short limit
 * makes a launch give up: tests use it to run the kernels' abort paths.
 * No reference counterpart (the reference's kernels have no bounded waits). */
int wbk_set_wait_timeout_ns(uint64_t timeout_ns);

/* Self-test of the bounded-wait machinery: launches one CTA that waits on an
 * mbarrier nothing ever arrives on, for at most `timeout_ns`, and records
 * WBK_ERR_DEVICE_TIMEOUT in the device error word. Used by tests to prove that
 * a wait which runs out returns a status instead of hanging. */
int wbk_selftest_bounded_wait(uint64_t timeout_ns, wbk_stream_t stream);

/* ------------------------------------------------------------ quantiser */

/* Max-accumulate max(|x|) over n fp16 values into *amax_bits, which holds the
 * fp16 bit pattern of the running maximum in its low 16 bits (uint32 so it can
 * be updated with atomicMax). NaNs are ignored (as fmaxf does in the
 * reference). The caller zeroes *amax_bits before the first accumulation.
 * Replaces: compute_scale_kernel, csrc/kernels/fp8_quantize.cu:45-74, and the
 * host block-max loop of compute_fp8_scale, fp8_quantize.cu:194-219. */
int wbk_amax_f16(const void* x, int64_t n, uint32_t* amax_bits, wbk_stream_t stream);

/* Given an accumulated *amax_bits, compute the per-tensor scale exactly as the
 * reference does — scale = amax / max_fp8 (fast-math division, as compiled by
 * the reference), 1.0 when that is not > 0 — and inv_scale = 1/scale rounded
 * to nearest; write scale to scale_out[0] (device float, may be NULL) and
 * quantise: q = fp8_rn_satfinite(clamp(float(x)*inv_scale, -max_fp8, max_fp8)).
 * fmt = WBK_FMT_E4M3 (max 448) or WBK_FMT_E5M2 (max 57344). Any n >= 0.
 * Replaces: quantise_fp16_to_e4m3_kernel / _e5m2_kernel, fp8_quantize.cu:81-137,
 * and quantise_to_e4m3 / quantise_to_e5m2, fp8_quantize.cu:222-257. */
int wbk_quantise_from_amax_f16(const void* x, int64_t n, int fmt,
                               const uint32_t* amax_bits, void* q_out,
                               float* scale_out, wbk_stream_t stream);

/* Convenience: zero *amax_ws, accumulate amax, then quantise (three stream
 * operations, no host synchronisation). amax_ws is a caller-owned device
 * uint32 used as the accumulator; it ends holding the amax bits. Tensors of
 * up to 262144 elements take one single-CTA launch instead (same results).
 * Replaces: quantise_to_e4m3 / quantise_to_e5m2, fp8_quantize.cu:222-257
 * (without its device->host copy of per-block partials, fp8_quantize.cu:212). */
int wbk_quantise_f16(const void* x, int64_t n, int fmt, void* q_out,
                     float* scale_out, uint32_t* amax_ws, wbk_stream_t stream);

/* Same result as wbk_quantise_f16 (bit for bit), for callers that cannot
 * allocate device memory: code running where cudaMalloc is forbidden or must
 * not be called (a host callback or real-time audio thread with a
 * no-allocation rule, a plugin whose host owns every device allocation, a
 * driver path that must not fail on allocation). It takes no amax_ws; its
 * scratch is a file-scope static device array of 4096 words (16 KB, held on
 * every GPU that loads libwbk until the process exits): per-CTA partial
 * maxima, one CTA per 65536 elements, plus the final amax.
 * Limit: n <= 268369920 elements (4095 CTAs); larger n returns
 * WBK_ERR_UNSUPPORTED with a message, before anything is launched.
 * The first call on a device looks up the array's device address (with that
 * device current) and caches it; make that first call before any stream
 * capture. Every call shares the one array and rewrites every word it reads
 * (nothing needs to start at zero); calls that overlap on the GPU, e.g. on
 * two streams at once, race on it. Allocates nothing: no cudaMalloc, no
 * cudaFree, no allocating library routine.
 * No counterpart in the reference (its quantiser allocates a per-call
 * torch::zeros buffer, csrc/kernels/fp8_quantize.cu:201). */
int wbk_quantise_f16_noalloc(const void* x, int64_t n, int fmt, void* q_out,
                             float* scale_out, wbk_stream_t stream);

/* Same codes, scale and amax bits as wbk_quantise_f16 (bit for bit), with x
 * read from HBM about once instead of twice: ONE cooperative launch (one CTA
 * per SM) keeps the end of each CTA's slice on chip -- 224 KB in shared
 * memory and 256 KB in tensor memory (TMEM) per SM -- and reads the rest of
 * the slice with an L2 evict-last hint so that it is still in L2, agrees on the
 * amax through one bounded grid-wide arrival, then quantises the on-chip part
 * and re-reads the rest.
 * sync_ws: WBK_QUANT_SYNC_BYTES of device memory (16-byte aligned), zero-filled
 * before first use; every call that completes leaves it zeroed; not used by two
 * calls at once. After a WBK_ERR_DEVICE_TIMEOUT it must be zero-filled again.
 * amax_ws ends holding the amax bits, as in wbk_quantise_f16.
 * When n < 2^22 or n > 88 x 2^20, n % 8 != 0, x is not 16-byte aligned,
 * q_out not 8-byte aligned, sync_ws is NULL, or the device cannot hold one
 * CTA per SM at once (it is shared or partitioned), this is wbk_quantise_f16
 * (same results).
 * Replaces: quantise_to_e4m3 / quantise_to_e5m2, fp8_quantize.cu:222-257, for
 * the large activations (e.g. the 48000 x 1280 cross-attention input). */
#define WBK_QUANT_SYNC_BYTES 16
int wbk_quantise_f16_resident(const void* x, int64_t n, int fmt, void* q_out,
                              float* scale_out, uint32_t* amax_ws, uint32_t* sync_ws,
                              wbk_stream_t stream);

/* scale_inv[0] = scale, scale_inv[1] = 1/scale for an accumulated amax, by the
 * same rule (and the same compiled division) as wbk_quantise_from_amax_f16.
 * Used by fused producers that quantise their own output. */
int wbk_scale_from_amax(const uint32_t* amax_bits, int fmt, float* scale_inv,
                        wbk_stream_t stream);

/* FFN activation quantiser: g = fp16(gelu_erf(float(y))) for n fp16 values y
 * (the fc1 output), then the per-tensor quantise of g exactly as
 * wbk_quantise_f16 does it (scale from max|g|). g itself is not stored.
 * ymax_key (may be NULL): the key of the largest y written by a GEMM with the
 * WBK_EPI_BIAS_MAXKEY epilogue; when gelu(y_max) >= 0.171 the amax of g is
 * taken from it (exact: GELU is increasing above -0.7518 and |GELU| < 0.17
 * below), otherwise one pass computes it. amax_ws: caller-owned device uint32.
 * gelu_erf uses the erf of Abramowitz & Stegun 7.1.26 (|error| <= 1.5e-7).
 * Replaces: HF's GELU on the fp16 fc1 output followed by quantise_e4m3 of it
 * (whisper_blaze/model.py:93-96 applied to the fc2 input). */
int wbk_quantise_gelu_f16(const void* y, int64_t n, int fmt, const uint32_t* ymax_key,
                          void* q_out, float* scale_out, uint32_t* amax_ws,
                          wbk_stream_t stream);

/* out = fp16(float(q) * scale) for n fp8 values; scale is a host float.
 * Replaces: dequantise_e4m3_to_fp16_kernel / _e5m2, fp8_quantize.cu:143-187,
 * and dequantise_e4m3 / dequantise_e5m2, fp8_quantize.cu:260-291. */
int wbk_dequantise_f16(const void* q, int64_t n, int fmt, float scale,
                       void* out, wbk_stream_t stream);

/* ------------------------------------------------------------- norms */

/* Row-wise over [rows, D] fp16, D % 8 == 0:
 *   s = x (+ residual);  out = fp16((s - mean) * rsqrt(var + eps) * gamma + beta)
 *   sum_out (may be NULL) = fp16(s)
 *   out_amax_bits (may be NULL): max-accumulate max|out| (fp16 bits), for a
 *   following wbk_quantise_from_amax_f16 without another pass over `out`.
 * residual may be NULL (plain LayerNorm).
 * Replaces: layernorm_fused_kernel + layernorm_fused_impl,
 * csrc/kernels/layernorm_fused.cu:50-184, :266-300 (bound as layernorm_fused /
 * layernorm_fused_residual, csrc/ops/bindings.cpp:101-135). */
int wbk_layernorm_f16(const void* x, const void* residual, const void* gamma,
                      const void* beta, void* out, void* sum_out,
                      int64_t rows, int64_t D, float eps,
                      uint32_t* out_amax_bits, wbk_stream_t stream);

/* LayerNorm followed by the per-tensor FP8 quantise of its output, without
 * storing the fp16 output: pass 1 writes each row's mean and rstd to `ws` and
 * the amax of the fp16 LayerNorm outputs to *amax_ws; pass 2 recomputes the
 * same fp16 outputs from x and the stored statistics and writes only their
 * fp8 codes. Bit-identical to wbk_layernorm_f16 (residual NULL) followed by
 * wbk_quantise_f16, with 2 fewer bytes of HBM traffic per element.
 * D % 8 == 0 and D <= 4096. ws: caller-owned device buffer of
 * wbk_layernorm_quantise_ws_bytes(rows) bytes; amax_ws: a device uint32.
 * Replaces: layernorm_fused (csrc/kernels/layernorm_fused.cu:50-184) followed
 * by quantise_to_e4m3 (csrc/kernels/fp8_quantize.cu:222-238), as the FP8 linear
 * after a pre-LN (whisper_blaze/model.py:93-96) would run them. */
int wbk_layernorm_quantise_f16(const void* x, const void* gamma, const void* beta,
                               int64_t rows, int64_t D, float eps, int fmt,
                               void* q_out, float* scale_out, void* ws,
                               uint32_t* amax_ws, wbk_stream_t stream);
int64_t wbk_layernorm_quantise_ws_bytes(int64_t rows);

/* out = fp16((x + residual) * rsqrt(mean((x+residual)^2) + eps) * gamma),
 * residual required, D % 8 == 0.
 * Replaces: rmsnorm_fused_kernel + rmsnorm_fused,
 * csrc/kernels/layernorm_fused.cu:191-258, :312-335. */
int wbk_rmsnorm_f16(const void* x, const void* residual, const void* gamma,
                    void* out, int64_t rows, int64_t D, float eps,
                    wbk_stream_t stream);

/* --------------------------------------------------------------- GEMM */

/* FP8 x FP8 -> fp32 (TMEM) -> fp16 scaled GEMM on tcgen05 tensor cores:
 *   out[M,N] = epilogue( (sum_k A[m,k] * W[n,k]) * descale (+ bias[n]) ... )
 *   descale = alpha * (a_scale ? *a_scale : 1) * (w_scale ? *w_scale : 1)
 * A [M,K] and W [N,K] are row-major fp8 (K contiguous, the nn.Linear weight
 * layout), formats a_fmt / w_fmt (WBK_FMT_*); K % 16 == 0 and both base
 * pointers 16-byte aligned (TMA). bias fp16 [N] or NULL; residual fp16 [M,N]
 * (row stride N) required for the RESIDUAL epilogues; out fp16 [M,N].
 * out_amax_bits (may be NULL): max-accumulate max|out| as fp16 bits.
 * Replaces the intent of gemm_fp8_e4m3_kernel / gemm_fp8_e4m3,
 * csrc/kernels/gemm_hopper.cu:179-269, :298-322 (never bound in the
 * reference), and the dequantise + F.linear of BlazeLinear.forward,
 * whisper_blaze/model.py:80-109. */
int wbk_gemm_fp8(const void* A, const void* W, int64_t M, int64_t N, int64_t K,
                 int a_fmt, int w_fmt, float alpha,
                 const float* a_scale, const float* w_scale,
                 const void* bias, const void* residual, void* out,
                 int epilogue, uint32_t* out_amax_bits, wbk_stream_t stream);

/* ------------------------------------------------------------ attention */

/* Non-causal multi-head attention forward for head_dim 64:
 *   out[b,h,i,:] = sum_j softmax_j(scale * q[b,h,i,:] . k[b,h,j,:]) v[b,h,j,:]
 * fp16 q/k/v/out, fp32 scores, softmax and accumulation (tcgen05 kind::f16).
 * Each of q, k, v, out is a [batch, heads, seq, 64] view with the 64 dims
 * contiguous and element strides given in the HOST array
 *   strides[12] = {q_b, q_h, q_s, k_b, k_h, k_s, v_b, v_h, v_s, o_b, o_h, o_s},
 * each a positive multiple of 8; pointers 16-byte aligned. seq_q and seq_k may
 * differ (cross-attention). If out_amax_bits is non-NULL, max|out| (fp16 bits,
 * NaN ignored) is max-accumulated into it as wbk_amax_f16 does.
 * Replaces: encoder_self_attn and decoder_cross_attn, bound at
 * csrc/ops/bindings.cpp:152-167, 229-235 (flash_attn_forward,
 * csrc/kernels/flash_attn_hopper.cu:297-365, scale = 1/sqrt(D), whose kernel
 * is unfinished upstream); in the encoder stack it stands where
 * HF WhisperAttention calls torch SDPA. */
int wbk_attention_f16(const void* q, const void* k, const void* v, void* out,
                      int64_t batch, int64_t heads, int64_t seq_q, int64_t seq_k, int64_t head_dim,
                      const int64_t* strides, float scale, uint32_t* out_amax_bits, wbk_stream_t stream);

/* wbk_gemm_fp8 with a split-K workspace. For very short-M shapes (M <= 32 rows,
 * K >= 2048) whose 64-wide column tiles cannot cover the SMs, K is split into
 * slices computed by different CTAs; each writes an fp32 partial into
 * `workspace` and the last slice of each tile to finish sums the partials in
 * slice order (bit-deterministic) and applies the epilogue. `workspace` (device,
 * 256-byte aligned, at least wbk_gemm_fp8_ws_bytes(M, N, K) bytes) must be
 * zero-filled before its first use; calls leave it reusable, but two calls must
 * not use the same workspace concurrently. With workspace == NULL, or a shape
 * that needs none, this is wbk_gemm_fp8. No reference counterpart (the
 * reference binds no GEMM). */
int wbk_gemm_fp8_ws(const void* A, const void* W, int64_t M, int64_t N, int64_t K,
                    int a_fmt, int w_fmt, float alpha,
                    const float* a_scale, const float* w_scale,
                    const void* bias, const void* residual, void* out,
                    int epilogue, uint32_t* out_amax_bits,
                    void* workspace, int64_t workspace_bytes, wbk_stream_t stream);

/* Bytes of workspace wbk_gemm_fp8_ws (split-K) and wbk_linear_fp8_f16 (its
 * in-kernel quantise) use for this shape (0: none). */
int64_t wbk_gemm_fp8_ws_bytes(int64_t M, int64_t N, int64_t K);

/* FP8 linear on an fp16 activation: quantises A16 [M, K] per tensor exactly as
 * wbk_quantise_f16 (codes into a_q_out, scale into *a_scale_out, amax bits into
 * *a_amax_ws), then out = wbk_gemm_fp8_ws(codes, W, ...) with that scale.
 * Replaces the pair of calls BlazeLinear.forward makes per FP8 linear
 * (quantise_e4m3 then the scaled GEMM, whisper_blaze/model.py:80-109).
 * For 0 < M <= 128 with 16-byte aligned A16 / a_q_out and a workspace
 * (wbk_gemm_fp8_ws_bytes(M, N, K) bytes, zero-filled before first use, not used
 * by two calls at once) it is ONE cooperative kernel: the GEMM's CTAs quantise
 * A together (grid-wide amax, then codes) before their tiles, so the short-M
 * decoder-step linears launch one kernel instead of two. Otherwise it is the two
 * launches. Codes, scale, amax bits and output are identical either way. After
 * a WBK_ERR_DEVICE_TIMEOUT the workspace must be zero-filled again. */
int wbk_linear_fp8_f16(const void* A16, int64_t M, int64_t N, int64_t K, int a_fmt,
                       void* a_q_out, float* a_scale_out, uint32_t* a_amax_ws,
                       const void* W, int w_fmt, const float* w_scale, float alpha,
                       const void* bias, const void* residual, void* out,
                       int epilogue, uint32_t* out_amax_bits,
                       void* workspace, int64_t workspace_bytes, wbk_stream_t stream);

#ifdef __cplusplus
}  /* extern "C" */
#endif

#endif  /* WBK_H_ */
