/*
 * pcb200.h -- C ABI of the B200 (sm_100a) FP8 quantize / scaled-BMM library
 * (libpcb200.so).  Plain pointers, sizes and strides; no torch types.
 *
 * Conventions shared by every entry point
 *   - Strides are in ELEMENTS of the tensor they describe.
 *   - Every tensor pointer is a device pointer on the current CUDA device.
 *   - `stream` is a cudaStream_t (NULL = legacy default stream).  Nothing is
 *     synchronised; nothing is allocated: the caller owns every buffer.
 *   - The return value is a pcb_status.  PCB_ERR_LAYOUT means the strides or
 *     alignment do not fit the TMA-fed path; callers repack with
 *     pcb_pack_u8() and call again.  Kernel-side failures (a bounded wait that
 *     ran out) are recorded in a device error word read by
 *     pcb_get_device_error().
 *   - Entry points are stateless and re-entrant (safe from the autograd
 *     worker thread); the only global state is a per-process cache of
 *     device attributes and the device error word.
 *
 * The reference interfaces these replace are the Python impl functions that
 * its plugin registry binds (fp8_training/fp8_bench/registry.py:116-169);
 * each declaration names the reference function and file:line it stands in for.
 */
#ifndef PCB200_H
#define PCB200_H

#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define PCB200_ABI_VERSION 1

typedef enum pcb_status {
  PCB_OK = 0,
  PCB_ERR_INVALID = 1,     /* bad argument (null pointer, negative size, ...) */
  PCB_ERR_UNSUPPORTED = 2, /* valid request this build does not implement       */
  PCB_ERR_LAYOUT = 3,      /* strides / alignment unusable by TMA: repack       */
  PCB_ERR_LAUNCH = 4,      /* cudaLaunch* failed (cudaGetLastError text kept)   */
  PCB_ERR_DEVICE = 5,      /* no usable sm_100 device                          */
  PCB_ERR_TIMEOUT = 6      /* reported through pcb_get_device_error()           */
} pcb_status;

typedef enum pcb_dtype {
  PCB_DTYPE_F32 = 0,
  PCB_DTYPE_F16 = 1,
  PCB_DTYPE_BF16 = 2,
  PCB_DTYPE_E4M3 = 3, /* float8_e4m3fn */
  PCB_DTYPE_E5M2 = 4  /* float8_e5m2   */
} pcb_dtype;

typedef enum pcb_activation {
  PCB_ACT_NONE = 0,
  PCB_ACT_GELU = 1 /* exact erf GELU: fp8_bench/kernels/bmm/activation.py:12-19 */
} pcb_activation;

/* Library ABI version (PCB200_ABI_VERSION of the build). */
int pcb_version(void);

/* Static name of a pcb_status ("PCB_OK", ...). */
const char* pcb_status_name(int status);

/* Text of the last host-side CUDA error seen by this thread (or ""). */
const char* pcb_last_error_text(void);

/* Read and clear the device error word of the current device.  *code is 0
 * when no kernel reported a failure; otherwise a pcb_status (PCB_ERR_TIMEOUT
 * for a bounded wait that ran out), *site the kernel/wait site and *info the
 * block index.  Synchronises the device. */
int pcb_get_device_error(int* code, int* site, int* info);

/* Test hook: the next pcb_bmm_scaled launch makes its kernel report `code`
 * through the device error word (no real fault, no hang). 0 disarms. */
int pcb_debug_inject_error(int code);

/*
 * Per-block quantization.  Replaces triton_per_block_quant
 * (fp8_training/fp8_bench/impls/triton_per_block.py:60-150) and its kernel
 * fp8_per_block_quant_kernel (fp8_bench/kernels/quant/per_block.py:6-48).
 * For each block_m x block_n tile of x[b] (tails masked):
 *   amax = max|x|, q = fp8_max * (1/max(amax, eps)), scale = 1/q,
 *   y = sat_cast(x * q).
 * x dtype: F32/F16/BF16; y dtype: E4M3/E5M2; scale fp32 [batch, mb, nb].
 */
int pcb_quant_per_block(const void* x, int x_dtype, int64_t batch, int64_t m, int64_t n,
                        int64_t sxb, int64_t sxm, int64_t sxn,
                        void* y, int y_dtype, int64_t syb, int64_t sym, int64_t syn,
                        float* scale, int64_t ssb, int64_t ssm, int64_t ssn,
                        int64_t block_m, int64_t block_n, float eps, void* stream);

/*
 * pcb_quant_per_block with power-of-two scales (E8M0 recipe of the per-block
 * FP8 training linears; no counterpart in the reference, whose per-block
 * scales are 1 / (448 / amax)).  Per block: r = RN(max(amax, eps) / fp8_max),
 * e = smallest integer with 2^e >= r, y = fp8(x * 2^-e), scale = 2^e (fp32).
 * Supported where x and y are contiguous along n with 16-byte aligned rows
 * (PCB_ERR_UNSUPPORTED otherwise).  Same arguments as pcb_quant_per_block.
 */
int pcb_quant_per_block_pow2(const void* x, int x_dtype, int64_t batch, int64_t m, int64_t n, int64_t sxb,
                             int64_t sxm, int64_t sxn, void* y, int y_dtype, int64_t syb, int64_t sym, int64_t syn,
                             float* scale, int64_t ssb, int64_t ssm, int64_t ssn, int64_t block_m, int64_t block_n,
                             float eps, void* stream);

/*
 * Per-channel quantization.  Replaces triton_per_channel_quant
 * (fp8_training/fp8_bench/impls/triton_per_channel.py:90-219) and the torch
 * quantizer fp8_per_channel_quant_torch_compile
 * (fp8_bench/kernels/quant/per_channel.py:9-29).
 * channel_axis = -2: one scale per row (reduce over n);
 * channel_axis = -1: one scale per column (reduce over m).
 *   q = fp8_max * (1/max(amax, eps)), scale = amax_clamped / fp8_max.
 * scale fp32 [batch, channels] with strides (ssb, ssc).
 */
int pcb_quant_per_channel(const void* x, int x_dtype, int64_t batch, int64_t m, int64_t n,
                          int64_t sxb, int64_t sxm, int64_t sxn,
                          void* y, int y_dtype, int64_t syb, int64_t sym, int64_t syn,
                          float* scale, int64_t ssb, int64_t ssc,
                          int channel_axis, float eps, void* stream);

/* Floats of device workspace pcb_quant_per_tensor needs (per-CTA partials). */
int64_t pcb_quant_per_tensor_workspace_floats(void);

/*
 * Per-tensor quantization.  Replaces triton_per_tensor_quant
 * (fp8_training/fp8_bench/impls/triton_per_tensor.py:28-96) and the legacy
 * fp8_quant_triton (kernels/fp8_bmm/fp8_warper.py:9-77).
 * amax over the whole tensor; scale arithmetic rounded to `scale_dtype`
 * (F32 for fp8_bench; the input dtype for the legacy entry point, which does
 * it in x's dtype); writes quant_scale (q) and dequant_scale (1/q) as one
 * fp32 each (values exactly representable in scale_dtype).  `workspace` is
 * pcb_quant_per_tensor_workspace_floats() floats of device memory.
 */
int pcb_quant_per_tensor(const void* x, int x_dtype, int64_t batch, int64_t m, int64_t n,
                         int64_t sxb, int64_t sxm, int64_t sxn,
                         void* y, int y_dtype, int64_t syb, int64_t sym, int64_t syn,
                         float* quant_scale, float* dequant_scale, int scale_dtype,
                         float fp8_max, float eps, float* workspace, void* stream);

/*
 * Dynamic float8 cast of the FP8 training linear.  Replaces the casts of
 * hp_tensor_to_float8_dynamic (fp8_training/fp8_bench/modules/float8/
 * float8_scaling_utils.py:29-72; amax_to_scale float8_utils.py:31-53,
 * to_fp8_saturated :118-139) that Float8BMMLinear runs before every GEMM
 * (modules/bmm_linear.py:229-310):
 *   scale = fp8_max / max(amax, eps)  (fp32 IEEE divide: the reference's
 *                                      float64 divide rounded to fp32 is the
 *                                      same value), y = sat(fp8(x * scale)).
 * The stored scale is this QUANT scale (Float8TrainingTensor._scale), not a
 * dequant scale.  axiswise = 0: one scale for the whole tensor (tensorwise;
 * `workspace` = pcb_quant_per_tensor_workspace_floats() floats, scale[0]);
 * axiswise = 1: one scale per (batch, row), reduced over n (axiswise_dim=-1;
 * scale[b*ssb + row*ssm], workspace unused).
 */
int pcb_quant_float8_dynamic(const void* x, int x_dtype, int64_t batch, int64_t m, int64_t n,
                             int64_t sxb, int64_t sxm, int64_t sxn,
                             void* y, int y_dtype, int64_t syb, int64_t sym, int64_t syn,
                             float* scale, int64_t ssb, int64_t ssm, int axiswise, float eps,
                             float* workspace, void* stream);

/*
 * Per-tensor quantization that allocates nothing -- not even the small
 * workspace pcb_quant_per_tensor asks for.  No counterpart in the reference:
 * it exists for callers that cannot hand the library a scratch buffer, such
 * as a plugin slot whose host framework passes only the input and output
 * tensors, or a latency-critical loop that must not call cudaMalloc (which
 * can synchronise the whole device).  Same arguments, results and scale
 * semantics as pcb_quant_per_tensor, minus `workspace`.
 *
 * Scratch: the amax partials live in a 1024-slot fp32 array (4 KiB) compiled
 * into the library; every GPU that loads the library holds it until the
 * process exits.  The amax pass launches at most four CTAs per SM (592 on a
 * B200), one slot each, so on such a GPU every tensor size is accepted; a
 * launch that would need more than the 1024 slots is rejected with
 * PCB_ERR_INVALID and an explanatory pcb_last_error_text().
 * The first call on each device looks up that array's device address (with
 * the device current) and caches it, so make the first call on a device
 * before any stream capture.  All calls share the one array: two calls whose
 * kernels overlap on the GPU (e.g. on two streams at once) race and may
 * return wrong scales; serialise them.  Nothing in the array has to start at
 * zero: each call writes every slot it later reads.
 */
int pcb_quant_per_tensor_noalloc(const void* x, int x_dtype, int64_t batch, int64_t m, int64_t n,
                                 int64_t sxb, int64_t sxm, int64_t sxn,
                                 void* y, int y_dtype, int64_t syb, int64_t sym, int64_t syn,
                                 float* quant_scale, float* dequant_scale, int scale_dtype,
                                 float fp8_max, float eps, void* stream);

/*
 * Scaled FP8 batched GEMM on the tcgen05 tensor cores:
 *   C[b,m,n] = act( sum_g (sum_{k in g} A[b,m,k] B[b,k,n]) * sa(b,m,g) * sb(b,g,n)
 *                   + bias[b,m,n] )
 * with k-groups of qbk elements (qbk a multiple of 128, or >= k for a single
 * group), sa(b,m,g) = scale_a[b*ssab + (m/qbm)*ssam + g*ssak] and
 * sb(b,g,n) = scale_b[b*ssbb + g*ssbk + (n/qbn)*ssbn]; a NULL scale pointer
 * reads as 1.0.  This one entry point covers the three reference BMMs:
 *   per-block   batch_fp8_per_block_bmm_kernel   (fp8_bench/kernels/bmm/per_block.py:9-137,
 *               wrapper impls/triton_per_block.py:232-420),
 *   per-channel batch_fp8_per_channel_bmm_kernel (kernels/bmm/per_channel.py:9-123,
 *               wrapper impls/triton_per_channel.py:271-427): qbm=qbn=1, ssak=ssbk=0,
 *   per-tensor  batch_fp8_per_tensor_bmm_kernel  (kernels/bmm/per_tensor.py:9-100,
 *               wrapper impls/triton_per_tensor.py:140-305): ssam=ssbn=0,
 * and the legacy fp8_bmm_quant_triton (kernels/fp8_bmm/fp8_warper.py:79-129).
 * A: K-major (sak == 1) or M-major (sam == 1); B: K-major (sbk == 1) or
 * N-major (sbn == 1); non-unit strides must be multiples of 16 bytes, else
 * PCB_ERR_LAYOUT.  ab_dtype E4M3 or E5M2 (both operands).  C dtype
 * BF16/F16/F32/E4M3/E5M2 (fp8 outputs saturate), scn == 1.
 * bias (optional) dtype F32/F16/BF16 with arbitrary strides.
 */
int pcb_bmm_scaled(const void* a, int64_t sab, int64_t sam, int64_t sak,
                   const void* b, int64_t sbb, int64_t sbk, int64_t sbn, int ab_dtype,
                   int64_t batch, int64_t m, int64_t n, int64_t k,
                   const float* scale_a, int64_t ssab, int64_t ssam, int64_t ssak, int64_t qbm,
                   const float* scale_b, int64_t ssbb, int64_t ssbk, int64_t ssbn, int64_t qbn,
                   int64_t qbk,
                   const void* bias, int bias_dtype, int64_t sbib, int64_t sbim, int64_t sbin,
                   void* c, int c_dtype, int64_t scb, int64_t scm, int64_t scn,
                   int activation, void* stream);

/*
 * pcb_bmm_scaled with A and B in different fp8 formats (a_dtype, b_dtype each
 * E4M3 or E5M2), e.g. an E5M2 gradient times an E4M3 weight.  Replaces the
 * mixed-format launches of the FP8 training linear's op
 * fp8_bench::bmm_linear_tma (fp8_training/fp8_bench/modules/bmm_linear.py:121-227,
 * called for dX and dW at :390-440 with E5M2 grad_output).  Other arguments as
 * pcb_bmm_scaled.
 */
int pcb_bmm_scaled_mixed(const void* a, int64_t sab, int64_t sam, int64_t sak, int a_dtype,
                         const void* b, int64_t sbb, int64_t sbk, int64_t sbn, int b_dtype,
                         int64_t batch, int64_t m, int64_t n, int64_t k,
                         const float* scale_a, int64_t ssab, int64_t ssam, int64_t ssak, int64_t qbm,
                         const float* scale_b, int64_t ssbb, int64_t ssbk, int64_t ssbn, int64_t qbn,
                         int64_t qbk,
                         const void* bias, int bias_dtype, int64_t sbib, int64_t sbim, int64_t sbin,
                         void* c, int c_dtype, int64_t scb, int64_t scm, int64_t scn,
                         int activation, void* stream);

/*
 * pcb_bmm_scaled for power-of-two scales (the E8M0 recipe of the per-block
 * FP8 training linears, pcb_quant_per_block_pow2; no counterpart in the
 * reference).  Same arguments; requires qbk == 128 and both scale tensors,
 * and uses only the exponent bits of every scale (a scale that is not a
 * power of two is truncated to 2^floor(log2)).  The caller passes a device
 * workspace of pcb_bmm_block_scaled_workspace_bytes() bytes, into which a
 * pre-pass packs the scales in the layout the tensor core's scale copy reads.  The tensor core applies the
 * scales (tcgen05.mma.kind::mxf8f6f4.block_scale), so the fp32 accumulator
 * stays in TMEM for the whole K loop.
 */
int pcb_bmm_block_scaled(const void* a, int64_t sab, int64_t sam, int64_t sak, const void* b, int64_t sbb,
                         int64_t sbk, int64_t sbn, int ab_dtype, int64_t batch, int64_t m, int64_t n, int64_t k,
                         const float* scale_a, int64_t ssab, int64_t ssam, int64_t ssak, int64_t qbm,
                         const float* scale_b, int64_t ssbb, int64_t ssbk, int64_t ssbn, int64_t qbn, int64_t qbk,
                         const void* bias, int bias_dtype, int64_t sbib, int64_t sbim, int64_t sbin, void* c,
                         int c_dtype, int64_t scb, int64_t scm, int64_t scn, int activation, void* workspace,
                         int64_t workspace_bytes, void* stream);

/* Device workspace (bytes, 16-byte aligned) pcb_bmm_block_scaled needs for
 * the packed E8M0 scale factors of both operands. */
int64_t pcb_bmm_block_scaled_workspace_bytes(int64_t batch, int64_t m, int64_t n, int64_t k);

/*
 * Fused quantize -> scaled FP8 GEMM (BASELINE cfg4).  The reference's fused
 * kernel (kernels/fp8_bmm/kernel/fp8_quant_bmm_fused_kernel.py:39-146) does not
 * run (its produce_quant_scale is called with one argument and returns
 * nothing); this is the working equivalent of what it intended:
 *   A = per-block 1x128 quantization of x (bf16/fp16, K contiguous) with the
 *       arithmetic of pcb_quant_per_block, done inside the GEMM;
 *   C[b] = act(sum_g (A_g B_g) * a_scale(b,m,g) * sb(b,g,n) + bias)
 * with 128-deep K groups and sb as in pcb_bmm_scaled (B e4m3, K- or N-major).
 * Optional outputs: xq (fp8 [B,M,K], K contiguous, row stride sxqm) and xs
 * (fp32 [B,M,ceil(K/128)]) receive the quantized activation and its scales,
 * bit-identical to pcb_quant_per_block (NULL to skip).  K % 8 == 0.
 */
int pcb_quant_bmm_fused(const void* x, int x_dtype, int64_t sxb, int64_t sxm, int64_t sxk,
                        const void* b, int64_t sbb, int64_t sbk, int64_t sbn, int b_dtype,
                        int64_t batch, int64_t m, int64_t n, int64_t k,
                        const float* scale_b, int64_t ssbb, int64_t ssbk, int64_t ssbn, int64_t qbn,
                        const void* bias, int bias_dtype, int64_t sbib, int64_t sbim, int64_t sbin,
                        void* c, int c_dtype, int64_t scb, int64_t scm, int64_t scn,
                        void* xq, int64_t sxqb, int64_t sxqm,
                        float* xs, int64_t sxsb, int64_t sxsm, int64_t sxsk,
                        int activation, float eps, void* stream);

/*
 * Byte repack: dst[b, r, c] = src[b*ssb + r*ssr + c*ssc] for c < cols and 0
 * for cols <= c < cols_padded.  Used by the host shims to turn an fp8 operand
 * whose strides do not fit TMA into a K-major, 16-byte aligned copy -- the
 * in-call packing of the reference's do_transpose_a / do_transpose_b
 * (fp8_bench/impls/triton_per_block.py:254-275).
 */
int pcb_pack_u8(const void* src, int64_t batch, int64_t rows, int64_t cols,
                int64_t ssb, int64_t ssr, int64_t ssc,
                void* dst, int64_t dsb, int64_t dsr, int64_t cols_padded, void* stream);

#ifdef __cplusplus
}
#endif

#endif /* PCB200_H */
