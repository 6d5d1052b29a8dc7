/*
 * ddpm_b200.h — C ABI of the B200 (sm_100a) DDPM dynamic-convolution library.
 *
 * The library replaces the GPU half of lartpang/DynamicConvolutionOperator:
 * every Triton kernel in `_triton_kernels.py` and the launch logic of its two
 * autograd functions. All entry points are plain C: device pointers, sizes,
 * dtype codes and a CUDA stream handle. No entry point allocates, frees or
 * synchronises; callers own every buffer (outputs and workspaces included).
 * Work is enqueued on `stream` (a `cudaStream_t`, NULL = legacy default stream).
 *
 * Layout conventions (identical to the reference, which forces `.contiguous()`
 * at `_triton_kernels.py:817-818, 874-877`):
 *   x, y, grad_x, grad_y : [N, C, H, W]            contiguous NCHW
 *   kernels, grad_k      : [N, 3, C, K*K, H, W]    contiguous
 *   out, grad_out        : [N, 4*C, H, W]          = concat(x, d0, d1, d2)
 *   weight, grad_weight  : [3*C*K*K, C] (a Conv2d [3CK^2, C, 1, 1] weight)
 *   bias, grad_bias      : [3*C*K*K]
 * Weight row index = (branch*C + c)*K*K + tap (`_triton_kernels.py:322`).
 *
 * Return value: 0 on success, a negative DDPM_ERR_* code otherwise; the
 * message of the last error on the calling thread is `ddpm_last_error()`.
 */
#ifndef DDPM_B200_H
#define DDPM_B200_H

#include <stddef.h>
#include <stdint.h>

#if defined(__GNUC__)
#define DDPM_API __attribute__((visibility("default")))
#else
#define DDPM_API
#endif

#ifdef __cplusplus
extern "C" {
#endif

/* Element types (torch.float32 / torch.bfloat16 / torch.float16). */
#define DDPM_F32  0
#define DDPM_BF16 1
#define DDPM_F16  2

#define DDPM_OK                 0
#define DDPM_ERR_INVALID_ARG   -1  /* bad size, dtype, null pointer, misalignment */
#define DDPM_ERR_UNSUPPORTED   -2  /* valid request outside this build's limits   */
#define DDPM_ERR_CUDA          -3  /* a CUDA launch/runtime call failed           */
#define DDPM_ERR_WORKSPACE     -4  /* workspace pointer/size too small            */

/* Library ABI version (major*100 + minor). */
DDPM_API int ddpm_version(void);

/* Message of the last failed call on this thread ("" if none). */
DDPM_API const char* ddpm_last_error(void);

/* Number of kernels this library has launched in this process (all devices,
 * all threads). Benchmarks read it to count the library's launches. */
DDPM_API unsigned long long ddpm_launch_count(void);

/* Device-side failure code of the current device (no reference counterpart):
 * every wait inside the tensor-core kernels is bounded; one that gives up
 * records a nonzero code here and the kernel returns early (its outputs are
 * then invalid). Synchronises the device; `reset` != 0 clears the code. */
DDPM_API int ddpm_device_status(int reset, int* code);

/*
 * Materialised dynamic filter, forward.
 * Replaces `_DynamicCat.forward` + `_dynamic_cat_fwd`
 * (reference `_triton_kernels.py:814-842` and `:21-101`).
 *   out[n, 0:C]         = x
 *   out[n, (b+1)C + c]  = sum_tap x[c, p + off(tap)*d_b] * kernels[n, b, c, tap, p]
 * with zero padding, FP32 accumulation, and out stored in `k_dtype`
 * (the reference allocates `out` with `kernels.dtype`, `:820-822`).
 * `x_dtype` may differ from `k_dtype` (autocast: fp32 x, bf16 kernels).
 * ksize must be odd, 1 <= ksize <= 7; dilations >= 1.
 */
DDPM_API int ddpm_dyncat_fwd(const void* x, int x_dtype,
                    const void* kernels, int k_dtype,
                    void* out,
                    int n, int c, int h, int w,
                    int ksize, int d0, int d1, int d2,
                    void* stream);

/*
 * Materialised dynamic filter, backward.
 * Replaces `_DynamicCat.backward` + `_dynamic_cat_bwd_x` + `_dynamic_cat_bwd_k`
 * (reference `_triton_kernels.py:844-866`, `:104-190`, `:193-254`).
 *   grad_x[c,q] = grad_out[c,q]
 *               + sum_{b,tap} kernels[b,c,tap,q-off*d_b] * grad_out[(b+1)C+c, q-off*d_b]
 *   grad_k[b,c,tap,p] = x[c, p+off*d_b] * grad_out[(b+1)C+c, p]
 * grad_out has `k_dtype`; grad_x has `x_dtype`; grad_k has `k_dtype`.
 * Either output may be NULL to skip it (one fused launch computes both);
 * `kernels` may be NULL when grad_x is (grad_k does not read the taps).
 */
DDPM_API int ddpm_dyncat_bwd(const void* x, int x_dtype,
                    const void* kernels, const void* grad_out, int k_dtype,
                    void* grad_x, void* grad_k,
                    int n, int c, int h, int w,
                    int ksize, int d0, int d1, int d2,
                    void* stream);

/*
 * Fused generator + dynamic filter: weight packing.
 * The fused kernels read the generator weight W [3*C*K*K, C] (the Conv2d
 * weight of reference `triton_impl.py:293`, row (b*C + c)*K*K + tap) from a
 * packed copy in the exact shared-memory operand layout of the tensor-core
 * MMAs (fp32 weights are split into bf16 hi + lo parts). Callers pack once per
 * weight version into a buffer of ddpm_gencat_pack_bytes() bytes (16-byte
 * aligned) and pass it to every fused launch that uses that weight.
 * Limits of this build: C <= 64; K in {1, 3} with dilation halos
 * (K/2)*max(d) <= 8, or K = 5 with halos <= 16 (the dY + dW entry points
 * cover K = 5 for 16-bit data through the staged merged pass, rows of a
 * multiple of 8 pixels); other sizes return DDPM_ERR_UNSUPPORTED (callers
 * then take the materialised path).
 */
DDPM_API size_t ddpm_gencat_pack_bytes(int c, int ksize, int dtype);
DDPM_API int ddpm_gencat_pack(const void* weight, const void* bias, int c, int ksize,
                              int dtype, void* packed, size_t packed_bytes, void* stream);

/*
 * Fused generator + dynamic filter, forward (inference and training forward).
 * Replaces `_launch_generator_dynamic_cat` + `_generator_dynamic_cat_fwd`
 * (reference `_triton_kernels.py:873-908`, `:268-420`):
 *   gen = W * y + bias (tensor cores, FP32 accumulation), rounded to `dtype`
 *   for bf16/fp16 as the reference does (`:332-335`), then
 *   out = cat(x, sum_tap gen * shifted x for dilations d0, d1, d2).
 * x, y, bias, out share `dtype` (bias: the generator bias [3*C*K*K], also
 * packed; which copy a kernel reads is an implementation detail). The taps
 * never reach global memory.
 */
DDPM_API int ddpm_gencat_fwd(const void* x, const void* y, const void* packed,
                             const void* bias, void* out,
                             int n, int c, int h, int w,
                             int ksize, int d0, int d1, int d2, int dtype,
                             void* stream);

/*
 * ddpm_gencat_fwd reading x and y from the staged operands (ddpm_gencat_stage
 * with x and y, same sizes and dtype): tiles arrive by TMA copies. Same
 * result; replaces the same reference kernel (`_triton_kernels.py:268-420`).
 * The staged buffer can then be reused by the backward of the same x and y.
 */
DDPM_API int ddpm_gencat_fwd_staged(const void* staged, size_t staged_bytes,
                                    const void* packed, const void* bias, void* out,
                                    int n, int c, int h, int w,
                                    int ksize, int d0, int d1, int d2, int dtype,
                                    void* stream);

/*
 * ddpm_gencat_fwd_staged that also writes its output as the staged planes of
 * the fuse convolution that consumes it (no counterpart in the reference,
 * whose cuDNN conv reads the NCHW output): `planes` is laid out as
 * ddpm_fuseconv_stage would write it for src = out (C = 4c channels,
 * ddpm_fuseconv_stage_bytes(n, 4c, h, w, dtype) bytes, 256-byte aligned) and
 * holds the same bytes, so ddpm_fuseconv_fwd_staged can use it directly and
 * the separate staging pass over the output is saved. `out` is written as
 * well. Requires c % 8 == 0 (-2 otherwise).
 */
DDPM_API int ddpm_gencat_fwd_staged_planes(const void* staged, size_t staged_bytes,
                                           const void* packed, const void* bias, void* out,
                                           void* planes, size_t planes_bytes, int n, int c,
                                           int h, int w, int ksize, int d0, int d1, int d2,
                                           int dtype, void* stream);

/*
 * Fused generator backward: input gradient dX, recomputing the taps.
 * Replaces `_generator_dynamic_cat_bwd_x` (reference `_triton_kernels.py:430-531`):
 *   grad_x[c,q] = grad_out[c,q]
 *               + sum_{b,tap} gen[(b,c,tap), q-o] * grad_out[(b+1)C+c, q-o]
 * with gen = round_dtype(W*y + bias) exactly as in the forward. `packed` is
 * the buffer filled by ddpm_gencat_pack for the same weight and bias.
 */
DDPM_API int ddpm_gencat_bwd_x(const void* y, const void* packed, const void* bias,
                               const void* grad_out, void* grad_x,
                               int n, int c, int h, int w,
                               int ksize, int d0, int d1, int d2, int dtype,
                               void* stream);

/*
 * Staged operands for the fused backward, written once per backward:
 * y channel-last, zero padded by the dilation halo, in the tensor-core operand
 * type (fp32: bf16 hi and residual parts) with the constant-one bias channel,
 * and (when x is given) x as 16-byte cells (fp32: FP32, 4 channels per cell;
 * bf16 / fp16: the input type, 8 channels per cell). The backward kernels
 * then stage every tile with bulk / TMA copies. Same role as the per-tile x
 * and y loads inside `_generator_dynamic_cat_bwd_x` and
 * `_generator_dynamic_cat_bwd_y` / `_bwd_weight_partial` (reference
 * `_triton_kernels.py:430-751`), done once per backward instead.
 * ddpm_gencat_stage_bytes() gives the size with the x part (0 for unsupported
 * shapes); with x == NULL only the leading y part is written (enough for
 * ddpm_gencat_bwd_x_staged). `staged` must be 256-byte aligned. The contents
 * depend on x and y only.
 */
DDPM_API size_t ddpm_gencat_stage_bytes(int n, int c, int h, int w, int ksize,
                                        int d0, int d1, int d2, int dtype);
DDPM_API int ddpm_gencat_stage(const void* x, const void* y, void* staged, size_t staged_bytes,
                               int n, int c, int h, int w,
                               int ksize, int d0, int d1, int d2, int dtype,
                               void* stream);

/*
 * ddpm_gencat_bwd_x reading y from the staged operands (ddpm_gencat_stage with
 * the same sizes and dtype; x may have been NULL there). Same result as ddpm_gencat_bwd_x; replaces the
 * same reference kernel (`_triton_kernels.py:430-531`).
 */
DDPM_API int ddpm_gencat_bwd_x_staged(const void* staged_y, size_t staged_bytes,
                                      const void* packed, const void* bias,
                                      const void* grad_out, void* grad_x,
                                      int n, int c, int h, int w,
                                      int ksize, int d0, int d1, int d2, int dtype,
                                      void* stream);

/*
 * Fused generator backward: dY and dW/db with dK = shifted(x) * grad formed on
 * chip. Replaces `_generator_dynamic_cat_bwd_y` (`_triton_kernels.py:534-623`),
 * `_generator_dynamic_cat_bwd_weight_partial` (`:626-751`) and
 * `_generator_dynamic_cat_bwd_weight_reduce` (`:754-811`):
 *   grad_y[i,p]        = sum_{b,c,tap} W[(b,c,tap), i] * dK[(b,c,tap), p]
 *   grad_weight[m, i]  = sum_p dK[m, p] * y[i, p]       ([3*C*K*K, C], dtype)
 *   grad_bias[m]       = sum_p dK[m, p]                  ([3*C*K*K], dtype)
 * grad_y may be NULL (skipped); grad_weight and grad_bias are given together
 * or both NULL. The weight gradient is a split spatial reduction into FP32
 * partials in `workspace` (ddpm_gencat_bwd_workspace_bytes() bytes, 16-byte
 * aligned) followed by a short reduce kernel.
 */
DDPM_API size_t ddpm_gencat_bwd_workspace_bytes(int n, int c, int h, int w, int ksize);
DDPM_API int ddpm_gencat_bwd_yw(const void* x, const void* y, const void* packed,
                                const void* grad_out, void* grad_y,
                                void* grad_weight, void* grad_bias,
                                void* workspace, size_t workspace_bytes,
                                int n, int c, int h, int w,
                                int ksize, int d0, int d1, int d2, int dtype,
                                void* stream);

/*
 * ddpm_gencat_bwd_yw reading x and y from the staged operands
 * (ddpm_gencat_stage with x and y, same sizes and dtype). grad_y, grad_weight,
 * grad_bias and the workspace are all required. Same results; replaces the
 * same reference kernels (`_triton_kernels.py:534-811`).
 */
DDPM_API int ddpm_gencat_bwd_yw_staged(const void* staged, size_t staged_bytes,
                                       const void* packed, const void* grad_out,
                                       void* grad_y, void* grad_weight, void* grad_bias,
                                       void* workspace, size_t workspace_bytes,
                                       int n, int c, int h, int w,
                                       int ksize, int d0, int d1, int d2, int dtype,
                                       void* stream);

/*
 * Native 3x3 fuse convolution (stride 1, zero padding 1, Cin <= 256,
 * Cout <= 64), replacing the cuDNN call `self.fuse(cat_out)` of
 * `triton_impl.py:294, 392` and its backward. FP32 runs on the tensor cores as
 * bf16 hi + lo operands (3 MMAs per step, no TF32); the bias is added to the
 * FP32 accumulator before the one output rounding. Weights are packed once
 * per weight version (ddpm_fuseconv_pack_bytes() bytes, 16-byte aligned).
 *   weight [Cout, Cin, 3, 3], bias [Cout] (may be NULL), x/grad_x [N, Cin, H, W],
 *   out/grad_out [N, Cout, H, W], all of `dtype`.
 */
DDPM_API size_t ddpm_fuseconv_pack_bytes(int cin, int cout, int dtype);
DDPM_API int ddpm_fuseconv_pack(const void* weight, int cin, int cout, int dtype,
                                void* packed, size_t packed_bytes, void* stream);
DDPM_API int ddpm_fuseconv_fwd(const void* x, const void* packed, const void* bias, void* out,
                               int n, int cin, int cout, int h, int w, int dtype, void* stream);
/* grad_x[i, p] = sum_{o, t} W[o, i, t] * grad_out[o, p - off(t)] */
DDPM_API int ddpm_fuseconv_bwd_data(const void* grad_out, const void* packed, void* grad_x,
                                    int n, int cin, int cout, int h, int w, int dtype,
                                    void* stream);
/*
 * Staged source planes of the fuse convolution (no counterpart in the
 * reference, whose cuDNN call reads NCHW directly): ddpm_fuseconv_stage
 * writes src [N, C, H, W] once as zero-padded channel-group planes in the
 * tensor-core operand type (ddpm_fuseconv_stage_bytes() bytes, 256-byte
 * aligned), which the staged entry points then read with one TMA copy per
 * K slab instead of per-thread loads and register transposes. The forward
 * stages x (C = cin), the data gradient stages grad_out (C = cout); the
 * results equal ddpm_fuseconv_fwd / ddpm_fuseconv_bwd_data on the same
 * inputs bit for bit. The planes are valid while src is unchanged.
 */
DDPM_API size_t ddpm_fuseconv_stage_bytes(int n, int c, int h, int w, int dtype);
DDPM_API int ddpm_fuseconv_stage(const void* src, void* planes, size_t planes_bytes, int n, int c,
                                 int h, int w, int dtype, void* stream);
DDPM_API int ddpm_fuseconv_fwd_staged(const void* planes, size_t planes_bytes, const void* packed,
                                      const void* bias, void* out, int n, int cin, int cout, int h,
                                      int w, int dtype, void* stream);
DDPM_API int ddpm_fuseconv_bwd_data_staged(const void* planes, size_t planes_bytes,
                                           const void* packed, void* grad_x, int n, int cin,
                                           int cout, int h, int w, int dtype, void* stream);
/* grad_weight[o, i, ky, kx] = sum_p grad_out[o, p] * x[i, p + (ky-1, kx-1)] and
 * grad_bias[o] = sum_p grad_out[o, p] (grad_bias may be NULL): the cuDNN weight
 * gradient of the same convolution. FP32 split partials in `workspace`
 * (ddpm_fuseconv_bwd_weight_workspace_bytes() bytes, 16-byte aligned), then a
 * reduce kernel; weight layout [Cout, Cin, 3, 3]. */
DDPM_API size_t ddpm_fuseconv_bwd_weight_workspace_bytes(int n, int cin, int cout, int h, int w);
DDPM_API int ddpm_fuseconv_bwd_weight(const void* x, const void* grad_out, void* grad_weight,
                                      void* grad_bias, void* workspace, size_t workspace_bytes,
                                      int n, int cin, int cout, int h, int w, int dtype,
                                      void* stream);

/*
 * Data gradient and weight / bias gradient of the fuse convolution in one call
 * (no counterpart in the reference, whose cuDNN backward runs them separately):
 * the results of ddpm_fuseconv_bwd_data and ddpm_fuseconv_bwd_weight with the
 * same arguments (bit for bit for grad_x). For widths that are a multiple of 8
 * the data gradient reads grad_out from the channel-last copy the weight
 * gradient writes into `workspace` anyway, instead of staging it a second
 * time. Workspace as ddpm_fuseconv_bwd_weight.
 */
DDPM_API int ddpm_fuseconv_bwd(const void* x, const void* grad_out, const void* packed,
                               void* grad_x, void* grad_weight, void* grad_bias, void* workspace,
                               size_t workspace_bytes, int n, int cin, int cout, int h, int w,
                               int dtype, void* stream);

/*
 * ddpm_fuseconv_bwd with grad_x written channel-last ([N][H][W][Cin],
 * Cin % 16 == 0, 16-byte aligned) instead of NCHW (no reference
 * counterpart). Same values bit for bit. In the DDPM module grad_x is the
 * gradient of the generator forward's output, and the fused generator's
 * backward (the *_nhwc entry points below) reads it channel-last: a pixel's
 * channels are one contiguous run, loaded with 16-byte vectors.
 */
DDPM_API int ddpm_fuseconv_bwd_nhwc(const void* x, const void* grad_out, const void* packed,
                                    void* grad_x, void* grad_weight, void* grad_bias,
                                    void* workspace, size_t workspace_bytes, int n, int cin,
                                    int cout, int h, int w, int dtype, void* stream);

/*
 * ddpm_gencat_bwd_x_staged / ddpm_gencat_bwd_yw_staged reading grad_out
 * channel-last ([N][H][W][4C], as ddpm_fuseconv_bwd_nhwc writes it; no
 * reference counterpart). C == 64 (DDPM_ERR_UNSUPPORTED otherwise); same
 * results as the NCHW entry points (dX bit for bit, dY and dW/db to the FP32
 * summation order of dY's reductions). The kernels load a pixel's 16 channels
 * as 16-byte vectors instead of 16 strided elements.
 */
DDPM_API int ddpm_gencat_bwd_x_staged_nhwc(const void* staged_y, size_t staged_bytes,
                                           const void* packed, const void* bias,
                                           const void* grad_out, void* grad_x, int n, int c,
                                           int h, int w, int ksize, int d0, int d1, int d2,
                                           int dtype, void* stream);
DDPM_API int ddpm_gencat_bwd_yw_staged_nhwc(const void* staged, size_t staged_bytes,
                                            const void* packed, const void* grad_out,
                                            void* grad_y, void* grad_weight, void* grad_bias,
                                            void* workspace, size_t workspace_bytes, int n,
                                            int c, int h, int w, int ksize, int d0, int d1,
                                            int d2, int dtype, void* stream);

/*
 * No-allocation variant of ddpm_gencat_bwd_yw (no counterpart in the
 * reference, whose Triton backward allocates its partials with torch).
 * Same arguments and results minus the workspace: the FP32 dW/db partials
 * live in an 8 MiB static device array inside the library, so the call
 * allocates nothing. For hosts that own no allocator, or that must not call
 * cudaMalloc mid-step because it can synchronise the device.
 *  - The split count of the dW reduction is capped to fit the 8 MiB; shapes
 *    whose single split does not fit return DDPM_ERR_WORKSPACE. dW/db match
 *    ddpm_gencat_bwd_yw to FP32 rounding (different summation order).
 *  - Nothing needs to start at zero: every partial read is written earlier
 *    in the same call.
 *  - The scratch is shared per device: overlapping calls (unordered streams,
 *    several host threads) race and corrupt dW/db; order them.
 *  - The first call on a device (with that device current) looks up the
 *    scratch's device address; make it before any stream capture begins.
 */
DDPM_API int ddpm_gencat_bwd_yw_static(const void* x, const void* y, const void* packed,
                                       const void* grad_out, void* grad_y,
                                       void* grad_weight, void* grad_bias,
                                       int n, int c, int h, int w,
                                       int ksize, int d0, int d1, int d2, int dtype,
                                       void* stream);

/* ---------------------------------------------------------------------------
 * Test-only exports (no reference counterpart). They exist for this
 * library's own tests; production callers never need them.
 * ------------------------------------------------------------------------- */

/*
 * Test hook of the bounded waits: with `enable` != 0, the next fused generator
 * forwards (ddpm_gencat_fwd*) on the current device have one producer thread
 * of CTA 0 withhold an mbarrier arrival, so a wait in that CTA runs out after
 * its limit (2 s): the kernel records a nonzero code (ddpm_device_status),
 * unwinds, frees its tensor memory and returns; its outputs are invalid.
 * No fault and no hang: the context stays usable. Call again with 0 to
 * restore normal operation.
 */
DDPM_API int ddpm_test_skip_arrive(int enable);

/*
 * Test hook of the materialised filter: with `disabled` != 0 (this process,
 * all devices) ddpm_dyncat_fwd / ddpm_dyncat_bwd skip their TMA-fed kernels
 * and run the register-fed ones, so tests can compare the two bit for bit.
 */
DDPM_API int ddpm_test_disable_tma(int disabled);

/*
 * Diagnostic (test-only; no reference counterpart): one 128 x n x k bf16 tcgen05 UMMA
 * on a single CTA with the operand layouts the fused kernels use.
 * a: [128 + shift, k] row-major bf16, b: [n, k] row-major bf16,
 * d: [128, n] row-major fp32, d[m, j] = sum_i a[shift + m, i] * b[j, i].
 * variant 0: K-major A; 1: MN-major A; 2: K-major A read from row `shift`;
 * 3: MN-major B (given as [n, k + shift]) read from K row `shift`,
 *    d[m, n] = sum_i a[m, i] * b[n, shift + i].
 */
DDPM_API int ddpm_umma_selftest(int variant, const void* a, const void* b, float* d,
                                int n, int k, int shift, void* stream);

#ifdef __cplusplus
}  /* extern "C" */
#endif

#endif  /* DDPM_B200_H */
