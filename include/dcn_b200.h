/*
 * dcn_b200.h -- C ABI of libdcn_b200, the B200 (sm_100a) deformable
 * convolution library (DCNv1 / DCNv2, fp32 NCHW).
 *
 * This is the drop-in boundary for the hot path of
 * ilirium/pytorch_mps_deform_conv2d.  The reference exports its path as
 * PyTorch operator schemas registered from ObjC++
 * (src/deform_conv2d_mps/_C/deform_conv2d_mps.mm:892-925); each entry point
 * below replaces one of those schemas and keeps its argument meaning:
 *
 *   dcn_forward       <- deform_conv2d_forward   (.mm:905-909, impl :192-374)
 *   dcn_backward      <- deform_conv2d_backward  (.mm:910-915, impl :682-890)
 *   dcn_col2im        <- deformable_col2im       (.mm:895-898, impl :388-504)
 *   dcn_col2im_coord  <- deformable_col2im_coord (.mm:900-904, impl :516-651)
 *
 * Conventions (same as the reference op):
 *   - all tensors are dense, contiguous fp32 in device memory of the current
 *     CUDA device: input (N, C, H, W); weight (outC, C/groups, kh, kw);
 *     offset (N, 2*dg*kh*kw, Ho, Wo) with (dy, dx) interleaved per tap;
 *     mask (N, dg*kh*kw, Ho, Wo); bias (outC); output (N, outC, Ho, Wo);
 *   - mask == NULL means DCNv1 (the reference passes an empty mask tensor,
 *     .mm:247); bias == NULL means no bias (Tensor? bias);
 *   - Ho = (H + 2*pad_h - dilation_h*(kh-1) - 1) / stride_h + 1, likewise Wo
 *     (.mm:231-234);
 *   - inputs are never written; outputs are fully overwritten;
 *   - work is enqueued on `stream` (a cudaStream_t, NULL = legacy default
 *     stream) and nothing synchronises the host, like the reference's lazy
 *     MPS encoding (.mm:372);
 *   - invalid arguments return DCN_ERR_INVALID_ARGUMENT and leave a message
 *     with the reference's wording in dcn_last_error() (the reference raises
 *     RuntimeError from TORCH_CHECK, .mm:202-267 and :693-760);
 *   - scratch memory is caller-provided (`workspace`, at least the size the
 *     matching *_workspace_size query returns); the library itself never
 *     allocates device memory.
 */
#ifndef DCN_B200_H_
#define DCN_B200_H_

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#if defined(__GNUC__)
#define DCN_API __attribute__((visibility("default")))
#else
#define DCN_API
#endif

#define DCN_ABI_VERSION 1

/* status codes */
#define DCN_OK 0
#define DCN_ERR_INVALID_ARGUMENT 1
#define DCN_ERR_WORKSPACE 2
#define DCN_ERR_CUDA 3
#define DCN_ERR_UNSUPPORTED 4

/* `flags` of dcn_forward / dcn_backward.  The low byte selects the math:
 *   DCN_MATH_FP32  fp32 FFMA on the CUDA cores (strict parity mode);
 *   DCN_MATH_TF32  tcgen05 tensor cores with TF32 operands and fp32
 *                  accumulation where a tensor-core kernel covers the shape,
 *                  fp32 FFMA elsewhere;
 *   DCN_MATH_3XTF32  the same tensor-core kernels with every operand split
 *                  into high and low TF32 parts (hi*hi + hi*lo + lo*hi):
 *                  close to fp32 accuracy at tensor-core speed.
 * The second byte can pin a kernel family (0 = automatic):
 *   DCN_ALGO_SIMT_GEMM / DCN_ALGO_SIMT_DIRECT  fp32 CUDA-core kernels (tests);
 *   DCN_ALGO_TC_GATHER_WEIGHT  tensor-core backward without the column buffer
 *                  where the fused kernel does not run (3xTF32, more than 256
 *                  out channels a group): the weight gradient re-gathers its
 *                  columns, so the backward workspace drops
 *                  kernel_h*kernel_w*N*Ho*Wo*C floats (x2 in 3xTF32) at some
 *                  speed. */
#define DCN_MATH_FP32 0x0
#define DCN_MATH_TF32 0x1
#define DCN_MATH_3XTF32 0x2
#define DCN_ALGO_SIMT_GEMM 0x100
#define DCN_ALGO_SIMT_DIRECT 0x200
#define DCN_ALGO_TC_GATHER_WEIGHT 0x400
/*   DCN_ALGO_TC_COLUMN_BUFFER  TF32 backward through the column buffer (the
 *                  grad-column kernel writes the sampled columns, a dense GEMM
 *                  reads them for the weight gradient) instead of the fused
 *                  kernel that keeps them on chip; for comparisons.  (3xTF32,
 *                  and groups with more than 256 out channels, always take
 *                  the column buffer.) */
#define DCN_ALGO_TC_COLUMN_BUFFER 0x800
/* Third byte: operand conventions.
 *   DCN_MASK_LOGITS  `mask` holds logits: the kernels use sigmoid(mask) and
 *                    dcn_backward's grad_mask is the gradient with respect to
 *                    the logits -- the DCNv2 block's mask sigmoid fused into
 *                    the op (no reference counterpart: the reference takes
 *                    the mask after the sigmoid). */
#define DCN_MASK_LOGITS 0x10000
/*   DCN_INPUT_NHWC   `input` and `grad_input` are channels-last buffers
 *                    (N, H, W, C) instead of (N, C, H, W); every other
 *                    operand keeps its layout.  The kernels gather from an
 *                    NHWC copy of the input in any case, so this replaces the
 *                    two transposes (input in, grad_input out) with a plain
 *                    copy and none: the layout of torch's channels_last
 *                    tensors (no reference counterpart: the reference makes
 *                    every operand contiguous NCHW). */
#define DCN_INPUT_NHWC 0x20000
/*   DCN_INPUT_STAGED `input` of dcn_forward / dcn_backward is not the input
 *                    tensor but its staging copy as dcn_stage_input wrote it
 *                    (NHWC plus one zero pixel row, dcn_staged_input_size
 *                    bytes): the call skips its own staging, and the
 *                    workspace queries drop the copy.  A training step stages
 *                    once and passes the copy to both passes instead of
 *                    transposing the input twice (no reference counterpart;
 *                    with DCN_INPUT_NHWC, grad_input is still channels-last). */
#define DCN_INPUT_STAGED 0x40000
/*   DCN_KEEP_STAGED  dcn_forward stages the input as usual and leaves the
 *                    staging copy (the layout dcn_stage_input writes) in the
 *                    first dcn_staged_input_size bytes of the workspace,
 *                    counted from the workspace pointer rounded up to 256
 *                    bytes, for a later call with DCN_INPUT_STAGED: a
 *                    training step stages inside its forward, where the
 *                    weight pack runs beside the staging, instead of in a
 *                    call of its own.  Not with DCN_INPUT_STAGED; dcn_forward
 *                    only (no reference counterpart). */
#define DCN_KEEP_STAGED 0x80000
/* Fourth byte: test switches (no reference counterpart).
 *   DCN_TEST_WAIT_TIMEOUT  the tensor-core kernels' TMA producers issue no
 *                    copies and every mbarrier wait gives up after about a
 *                    millisecond, so the waits run out: the kernels raise
 *                    their error word and return without results.  For
 *                    testing dcn_device_status only; never in production. */
#define DCN_TEST_WAIT_TIMEOUT 0x1000000

/* Bits of the error word dcn_device_status reports: a bounded wait of that
 * tensor-core kernel family ran out (no reference counterpart: the reference
 * has no device-side waits).  The kernel then stops where it is -- its
 * results are incomplete -- drains the copies and tensor-core operations it
 * issued, frees its tensor memory and returns; it never traps or hangs. */
#define DCN_STATUS_FWD_WAIT_TIMEOUT 0x1 /* forward (fwd_tc)                */
#define DCN_STATUS_BWD_DATA_TIMEOUT 0x2 /* grad-column kernel (bwd_data_tc) */
#define DCN_STATUS_BWD_WEIGHT_TIMEOUT 0x4 /* weight-gradient kernels        */

/* Geometry of one deformable convolution: the shapes of the reference op's
 * tensors plus its integer arguments. */
typedef struct dcn_shape {
  int64_t batch, in_channels, height, width;  /* input (N, C, H, W)          */
  int64_t out_channels, kernel_h, kernel_w;   /* weight (outC, C/g, kh, kw)  */
  int64_t stride_h, stride_w;
  int64_t pad_h, pad_w;
  int64_t dilation_h, dilation_w;
  int64_t groups, deformable_groups;
} dcn_shape;

/* ABI version of the loaded library (DCN_ABI_VERSION). */
DCN_API int dcn_abi_version(void);

/* Message of the last failed call on this host thread ("" if none). */
DCN_API const char* dcn_last_error(void);

/* Output spatial size of `shape` (.mm:231-234).  Returns DCN_OK, or
 * DCN_ERR_INVALID_ARGUMENT when it is non-positive. */
DCN_API int dcn_output_size(const dcn_shape* shape, int64_t* out_h, int64_t* out_w);

/* Bytes of workspace dcn_forward needs for `shape` and `flags`.  On the
 * tensor-core path this includes a scratch (sized for the current device's SM
 * count) with which the forward splits a short last round of tiles over all
 * SMs; given a workspace without that scratch, dcn_forward runs whole tiles
 * only -- the results differ only in the order of fp32 additions. */
DCN_API size_t dcn_forward_workspace_size(const dcn_shape* shape, uint32_t flags);

/* Row windows (no reference counterpart): output rows [row_begin,
 * row_begin + rows) of every image, for splitting one image's output rows
 * across devices.  `shape` describes the whole problem; offset, mask,
 * output (forward) and grad_output, grad_offset, grad_mask (backward) hold
 * only the window's rows, laid out as (N, channels, rows, out_w); input and
 * grad_input stay whole.  grad_input, grad_weight and grad_bias then hold
 * this window's contributions: summing them over a partition of the rows
 * gives the full gradients.  Otherwise as dcn_forward / dcn_backward. */
DCN_API size_t dcn_forward_rows_workspace_size(const dcn_shape* shape, int64_t rows,
                                               uint32_t flags);
DCN_API int dcn_forward_rows(const dcn_shape* shape, int64_t row_begin, int64_t rows,
                             const float* input, const float* weight, const float* offset,
                             const float* mask, const float* bias, float* output,
                             uint32_t flags, void* workspace, size_t workspace_bytes,
                             void* stream);
DCN_API size_t dcn_backward_rows_workspace_size(const dcn_shape* shape, int64_t rows,
                                                uint32_t flags);
DCN_API int dcn_backward_rows(const dcn_shape* shape, int64_t row_begin, int64_t rows,
                              const float* grad_output, const float* input, const float* weight,
                              const float* offset, const float* mask, float* grad_input,
                              float* grad_offset, float* grad_mask, float* grad_weight,
                              float* grad_bias, uint32_t flags, void* workspace,
                              size_t workspace_bytes, void* stream);

/* bf16 forward (no reference counterpart: the reference is fp32 only,
 * .mm:206-209).  Every tensor argument is bf16 (16-bit words, the layouts of
 * dcn_forward) and so is the output.  When channels per group and per
 * deformable group are multiples of 64, tcgen05 tensor cores run with bf16
 * operands and fp32 accumulation (bf16 gathers: half the bytes of fp32);
 * other shapes are upcast to fp32 inside the workspace and run on
 * dcn_forward's kernels under `flags`, the result rounded back to bf16. */
DCN_API size_t dcn_forward_bf16_workspace_size(const dcn_shape* shape, uint32_t flags);
DCN_API int dcn_forward_bf16(const dcn_shape* shape, const void* input, const void* weight,
                             const void* offset, const void* mask, const void* bias,
                             void* output, uint32_t flags, void* workspace,
                             size_t workspace_bytes, void* stream);

/* bf16 backward (no reference counterpart): every tensor argument and
 * gradient bf16; the gradients are computed by dcn_backward's kernels under
 * `flags` from fp32 copies made inside the workspace and rounded to bf16. */
DCN_API size_t dcn_backward_bf16_workspace_size(const dcn_shape* shape, uint32_t flags);
DCN_API int dcn_backward_bf16(const dcn_shape* shape, const void* grad_output, const void* input,
                              const void* weight, const void* offset, const void* mask,
                              void* grad_input, void* grad_offset, void* grad_mask,
                              void* grad_weight, void* grad_bias, uint32_t flags,
                              void* workspace, size_t workspace_bytes, void* stream);

/* fp16 forward and backward (no reference counterpart): as the bf16 entry
 * points with every tensor argument and gradient fp16; the tensor-core
 * forward runs kind::f16 UMMAs with fp16 operands. */
DCN_API size_t dcn_forward_f16_workspace_size(const dcn_shape* shape, uint32_t flags);
DCN_API int dcn_forward_f16(const dcn_shape* shape, const void* input, const void* weight,
                            const void* offset, const void* mask, const void* bias, void* output,
                            uint32_t flags, void* workspace, size_t workspace_bytes,
                            void* stream);
DCN_API size_t dcn_backward_f16_workspace_size(const dcn_shape* shape, uint32_t flags);
DCN_API int dcn_backward_f16(const dcn_shape* shape, const void* grad_output, const void* input,
                             const void* weight, const void* offset, const void* mask,
                             void* grad_input, void* grad_offset, void* grad_mask,
                             void* grad_weight, void* grad_bias, uint32_t flags, void* workspace,
                             size_t workspace_bytes, void* stream);

/* Forward pass; replaces deform_conv2d_forward (.mm:192-374).
 * output = bias + sum_{c,k} weight * mask * bilinear(input, sample(offset)). */
DCN_API int dcn_forward(const dcn_shape* shape, const float* input, const float* weight,
                        const float* offset, const float* mask, const float* bias,
                        float* output, uint32_t flags, void* workspace,
                        size_t workspace_bytes, void* stream);

/* Bytes of workspace dcn_backward needs for `shape` and `flags`. */
DCN_API size_t dcn_backward_workspace_size(const dcn_shape* shape, uint32_t flags);

/* Backward pass; replaces deform_conv2d_backward (.mm:682-890).  Writes all
 * five gradients.  grad_mask must be NULL when mask is NULL (the reference
 * returns an empty tensor there, .mm:766-767); grad_bias may be NULL when no
 * bias gradient is wanted (the reference returns an empty tensor when the
 * op had no bias, .mm:885-886). */
DCN_API int dcn_backward(const dcn_shape* shape, const float* grad_output,
                         const float* input, const float* weight, const float* offset,
                         const float* mask, float* grad_input, float* grad_offset,
                         float* grad_mask, float* grad_weight, float* grad_bias,
                         uint32_t flags, void* workspace, size_t workspace_bytes,
                         void* stream);

/* Single-image scatter of a column gradient into the input gradient;
 * replaces deformable_col2im (.mm:388-504).  columns (C*kh*kw, Ho*Wo) with
 * row c*kh*kw + k; offset (2*dg*kh*kw, Ho, Wo); mask (dg*kh*kw, Ho, Wo) or
 * NULL; grad_im (C, H, W) is overwritten. */
DCN_API int dcn_col2im(const float* columns, const float* offset, const float* mask,
                       float* grad_im, int64_t channels, int64_t height, int64_t width,
                       int64_t kernel_h, int64_t kernel_w, int64_t stride_h,
                       int64_t stride_w, int64_t pad_h, int64_t pad_w,
                       int64_t dilation_h, int64_t dilation_w,
                       int64_t deformable_groups, void* stream);

/* Single-image offset / mask gradients from a column gradient; replaces
 * deformable_col2im_coord (.mm:516-651).  input (C, H, W); grad_offset
 * (2*dg*kh*kw, Ho, Wo) and grad_mask (dg*kh*kw, Ho, Wo, NULL when mask is
 * NULL) are overwritten. */
DCN_API int dcn_col2im_coord(const float* columns, const float* input,
                             const float* offset, const float* mask, float* grad_offset,
                             float* grad_mask, int64_t channels, int64_t height,
                             int64_t width, int64_t kernel_h, int64_t kernel_w,
                             int64_t stride_h, int64_t stride_w, int64_t pad_h,
                             int64_t pad_w, int64_t dilation_h, int64_t dilation_w,
                             int64_t deformable_groups, void* stream);

/* Forward for callers that cannot allocate device memory.  No counterpart in
 * the reference: it exists for code that may not call cudaMalloc (inside an
 * allocator's or memory pool's own hooks, host-framework plugins that only
 * receive input and output buffers, deployments that fix device memory at
 * start-up).  Same arguments and results as dcn_forward without the workspace:
 * the scratch comes from a 16 MiB array compiled into the library, which every
 * GPU that loads the library holds until the process exits.  Shapes whose
 * least workspace (dcn_forward_workspace_size without the optional
 * split-round scratch) exceeds 16 MiB are rejected with DCN_ERR_WORKSPACE
 * before anything is launched.  The first call on a device (and in each
 * further CUDA context on it: a context of the caller's own, or the primary
 * context created again after cudaDeviceReset) looks up the array's device
 * address there (cudaGetSymbolAddress); make that first call before any
 * stream capture.  All calls share the one array:
 * calls that can overlap on the GPU (different streams, or different host
 * threads on the same device) race on it and must be serialised by the
 * caller.  Nothing in the array needs to start at zero: each call overwrites
 * the part it uses before reading it. */
DCN_API int dcn_forward_noalloc(const dcn_shape* shape, const float* input,
                                const float* weight, const float* offset, const float* mask,
                                const float* bias, float* output, uint32_t flags, void* stream);

/* Staging copy of an input for DCN_INPUT_STAGED (no reference counterpart):
 * `staged` (dcn_staged_input_size bytes of device memory) receives the input
 * in NHWC followed by one zero pixel row, the layout the kernels gather
 * from.  `input` is NCHW, or channels-last with DCN_INPUT_NHWC in `flags`.
 * Enqueued on `stream`; the copy stays valid while `input` is unchanged. */
DCN_API size_t dcn_staged_input_size(const dcn_shape* shape);
DCN_API int dcn_stage_input(const dcn_shape* shape, const float* input, float* staged,
                            uint32_t flags, void* stream);
/* The same for bf16 or fp16 tensors (16-bit values moved as they are):
 * dcn_staged_input_size_h16 bytes, for the 16-bit entry points with
 * DCN_INPUT_STAGED.  Those take a staging copy (DCN_INPUT_STAGED) or keep
 * theirs (dcn_forward_bf16 / _f16 with DCN_KEEP_STAGED, at the workspace
 * start as dcn_forward) only on their tensor-core routes:
 * dcn_h16_staging(shape, flags) is 1 when both the 16-bit forward and
 * backward take them for this shape and flags, 0 otherwise (then the calls
 * refuse both flags).  No reference counterpart. */
DCN_API size_t dcn_staged_input_size_h16(const dcn_shape* shape);
DCN_API int dcn_stage_input_h16(const dcn_shape* shape, const void* input, void* staged,
                                uint32_t flags, void* stream);
DCN_API int dcn_h16_staging(const dcn_shape* shape, uint32_t flags);

/* Device error word of the current device (DCN_STATUS_* bits; 0 when every
 * wait of the tensor-core kernels completed in time).  No reference
 * counterpart.  The word is sticky: a bit stays raised, across calls, until a
 * call with `clear` non-zero reads it, so a check after a batch of calls sees
 * a failure of any of them.  The read is ordered after the work already
 * enqueued on `stream` and the host waits for it (call it outside stream
 * capture). */
DCN_API int dcn_device_status(void* stream, int clear, int* status);

/* L2 <-> SM bandwidth probe (a diagnostic; no reference counterpart).
 * Enqueues on `stream` one kernel over all SMs that sweeps `passes` times over
 * `bytes` (rounded down to 16) of the device buffer `buf` (16-byte aligned):
 * kind 0 reads 16-byte vectors cached in L2 only, as the corner gathers do;
 * kind 1 adds 1.0f to every fp32 with 16-byte reductions, as the col2im
 * scatter does (kind 1 modifies the buffer); kind 2 does both in one loop,
 * five 16-byte loads to two 16-byte reductions: of the bytes swept (rounded
 * down to a multiple of 3584) the first 5/7 are read, 1.0f is added to every
 * fp32 of the last 2/7; kind 3 reads 16-byte vectors (L2 only) from random
 * 128-byte lines of the buffer, 8 lanes to a line, as the corner gathers do;
 * kind 4 adds 1.0f with 16-byte reductions in the same random pattern, as the
 * col2im scatter does (kinds 3 and 4 need bytes / 512 >= 4 x the probe's 2048
 * threads an SM x SMs / 32).  With
 * `bytes` well under the L2 size, bytes x passes over the kernel's device
 * time is the L2 -> SM (kind 0), SM -> L2 reduction (kind 1), mixed (kind 2),
 * gather (kind 3) or scatter (kind 4) bandwidth the hot kernels are set
 * against (kinds 3 and 4 move 512 x floor(bytes / 512 / W / 4) x 4 x W bytes
 * a pass, W = 64 warps a SM x SMs).
 * The caller times it (CUDA events on `stream`). */
DCN_API int dcn_l2_probe(int kind, void* buf, size_t bytes, int passes, void* stream);

/* Kernel profiler (no reference counterpart: the reference times its ops
 * with wall clocks around torch.mps.synchronize(), benchmarks/bench.py:39-49).
 * When enabled, every kernel launch and scratch memset of the entry points
 * above is bracketed by a CUDA event pair on its stream.  dcn_profiler_read
 * waits for the recorded events, reports per-name launch counts and summed
 * device milliseconds (at most max_stats entries; *count gets the number of
 * names) and clears the records.  Events are created on first use. */
typedef struct dcn_kernel_stat {
  char name[48];
  int64_t launches;
  double total_ms;
} dcn_kernel_stat;

DCN_API int dcn_profiler_enable(int enable);
DCN_API int dcn_profiler_read(dcn_kernel_stat* stats, int max_stats, int* count);

#ifdef __cplusplus
}
#endif

#endif /* DCN_B200_H_ */
