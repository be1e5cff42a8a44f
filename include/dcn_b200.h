/*
 * dcn_b200.h -- C ABI of the B200 (sm_100a) deformable-convolution library
 * (libdcn_b200.so).
 *
 * Plain pointers and sizes only: every tensor argument is a device pointer to
 * a dense, row-major (NCHW) array of the element type named by desc->dtype,
 * and every call is enqueued asynchronously on the CUDA stream passed as
 * `stream` (a cudaStream_t; NULL = legacy default stream).  No call
 * synchronises the host, and no call allocates device memory: scratch space
 * is the caller's `workspace` (size from the *_workspace_size query, 256-byte
 * aligned).  Inputs are never written.
 *
 * Each entry point replaces one function of the reference's native FFI (the
 * pybind11 module `_C` of mps-deform-conv, mps_deform_conv/csrc/
 * deform_conv2d_mps.mm:1221-1249), with the same argument meaning; the tensor
 * arguments there become pointers plus the shape fields of dcn_conv_desc here.
 *
 * Layouts (B = batch, C = in_channels, G = n_weight_grps, OG = n_offset_grps,
 * T = kernel_h * kernel_w, Ho/Wo = output size):
 *   input       [B][C][H][W]
 *   weight      [Co][C/G][kernel_h][kernel_w]
 *   offset      [B][OG*T*2][Ho][Wo]   channel o*2T + 2t is dy, + 1 is dx
 *   mask        [B][OG*T][Ho][Wo]     (ignored unless use_mask)
 *   bias        [Co]                  (NULL = no bias)
 *   output      [B][Co][Ho][Wo]
 *   columns     [C*T][B*Ho*Wo]        row c*T + t
 *
 * Return value: DCN_OK or an error code; dcn_last_error() gives the message
 * (thread-local).  Arithmetic: fp32 accumulation for every dtype.
 */
#ifndef DCN_B200_H
#define DCN_B200_H

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

/* element types (desc.dtype) */
#define DCN_FLOAT32 0
#define DCN_FLOAT16 1
#define DCN_BFLOAT16 2

/* status codes */
#define DCN_OK 0
#define DCN_ERR_INVALID_ARGUMENT 1 /* shape / parameter check failed          */
#define DCN_ERR_UNSUPPORTED 2      /* dtype or size outside what is built     */
#define DCN_ERR_CUDA 3             /* a CUDA runtime call or launch failed    */
#define DCN_ERR_WORKSPACE 4        /* workspace pointer NULL or too small     */
#define DCN_ERR_DEVICE_TIMEOUT 5   /* a kernel's bounded wait expired         */

/* Problem descriptor: the integer arguments of the reference FFI
 * (stride_h ... use_mask, deform_conv2d_mps.mm:603-615) plus the tensor
 * shapes that the reference reads from its at::Tensor arguments. */
typedef struct dcn_conv_desc {
  int32_t dtype;          /* DCN_FLOAT32 / DCN_FLOAT16 / DCN_BFLOAT16 */
  int32_t use_mask;       /* 0: DCNv1 (mask ignored), 1: DCNv2 */
  int64_t batch, in_channels, in_h, in_w;
  int64_t out_channels, kernel_h, kernel_w;
  int64_t stride_h, stride_w, pad_h, pad_w, dilation_h, dilation_w;
  int64_t n_weight_grps, n_offset_grps;
} dcn_conv_desc;

/* Version of this ABI (major*10000 + minor*100 + patch). */
DCN_API int dcn_abi_version(void);

/* Number of CUDA kernels this library has launched in this process (all
 * devices, all threads).  For launch accounting in benchmarks and tests. */
DCN_API uint64_t dcn_launch_count(void);

/* Per-kernel device timing.  While enabled, every launch this library makes
 * is bracketed by a CUDA event pair recorded on its stream (launches inside a
 * stream capture are not timed).  dcn_profile_enable(1) clears old records
 * and starts; dcn_profile_enable(0) stops.  dcn_profile_summary waits for
 * the recorded events and writes, per kernel name in order of first launch,
 * the name (into names + i*name_stride), the launch count and the summed
 * device time in ms; it returns the number of distinct names (-1 on a CUDA
 * error) and writes at most max_entries entries. */
DCN_API void dcn_profile_enable(int enable);
DCN_API int dcn_profile_summary(int max_entries, char *names, size_t name_stride,
                                uint64_t *launches, double *total_ms);

/* Message of the last failed call on this host thread ("" if none). */
DCN_API const char *dcn_last_error(void);

/* Output spatial size for a descriptor; DCN_ERR_INVALID_ARGUMENT when it is
 * not positive ("Invalid output dimensions", mps_deform_conv/__init__.py:208-216). */
DCN_API int dcn_output_size(const dcn_conv_desc *desc, int64_t *out_h, int64_t *out_w);

/* Checks a descriptor the way the reference's host code does
 * (deform_conv2d_mps.mm:617-657: positive stride/dilation/groups,
 * non-negative padding, int32 dispatch sizes) plus divisibility of the
 * channel counts by the groups. */
DCN_API int dcn_validate(const dcn_conv_desc *desc);

/* ---------------------------------------------------------------------
 * Forward.  Replaces `_C.deform_conv2d_forward` (deform_conv2d_mps.mm:603-800;
 * argument-for-argument the torchvision::deform_conv2d schema):
 * output = deformable conv of input with weight, offset, optional mask and
 * bias.  Writes `output` completely.
 */
DCN_API size_t dcn_forward_workspace_size(const dcn_conv_desc *desc);
DCN_API int dcn_deform_conv2d_forward(const dcn_conv_desc *desc, const void *input, const void *weight,
                              const void *offset, const void *mask, const void *bias,
                              void *output, void *workspace, size_t workspace_bytes,
                              void *stream);

/* ---------------------------------------------------------------------
 * Column buffer.  Replaces `_C.deformable_im2col` (deform_conv2d_mps.mm:806-936):
 * columns[c*T + t][b*Ho*Wo + p] = mask * bilinear(input[b, c], tap t at p).
 * desc->out_channels, n_weight_grps are ignored.
 */
DCN_API int dcn_deformable_im2col(const dcn_conv_desc *desc, const void *input, const void *offset,
                          const void *mask, void *columns, void *stream);

/* ---------------------------------------------------------------------
 * Input gradient from a column gradient.  Replaces
 * `_C.deform_conv2d_backward_input` (deform_conv2d_mps.mm:942-1069):
 * grad_input = col2im(grad_col) (transpose of the bilinear gather, fp32
 * accumulation).  grad_col has the columns layout.  Overwrites grad_input.
 */
DCN_API size_t dcn_backward_input_workspace_size(const dcn_conv_desc *desc);
DCN_API int dcn_deform_conv2d_backward_input(const dcn_conv_desc *desc, const void *grad_col,
                                     const void *offset, const void *mask, void *grad_input,
                                     void *workspace, size_t workspace_bytes, void *stream);

/* ---------------------------------------------------------------------
 * Input gradient from a column gradient, allocating nothing.  No counterpart
 * in the reference: it exists for callers that hold only their input and
 * output buffers and cannot allocate device memory (plugin interfaces that
 * hand a kernel library pointers but no allocator; real-time loops that
 * forbid allocation after start-up).  Same arguments and result as
 * dcn_deform_conv2d_backward_input, without the workspace: the fp32
 * accumulator for fp16/bf16 data is a fixed 8 MiB array in device memory
 * that every GPU which loads the library holds until the process exits.
 *   - Limit: for fp16/bf16, grad_input (B*C*H*W) may have at most 2,097,152
 *     elements; larger problems return DCN_ERR_UNSUPPORTED.  fp32 data
 *     accumulates in grad_input itself, never uses the array and has no
 *     such limit.
 *   - The first fp16/bf16 call on a device looks up the array's device
 *     address (cudaGetSymbolAddress) with that device current, and looks it
 *     up again after the device's context was reset (cudaDeviceReset); make
 *     that first call before any stream capture.
 *   - All calls share the one array and each call clears the part it uses.
 *     Calls that overlap on the GPU (other streams, other host threads, same
 *     device) race on it: issue them on one stream.
 */
DCN_API int dcn_deform_conv2d_backward_input_noalloc(const dcn_conv_desc *desc, const void *grad_col,
                                                     const void *offset, const void *mask,
                                                     void *grad_input, void *stream);

/* ---------------------------------------------------------------------
 * Offset and mask gradients from a column gradient.  Replaces
 * `_C.deform_conv2d_backward_offset_mask` (deform_conv2d_mps.mm:1075-1215).
 * Overwrites grad_offset, and grad_mask when use_mask (grad_mask may be
 * NULL otherwise).
 */
DCN_API int dcn_deform_conv2d_backward_offset_mask(const dcn_conv_desc *desc, const void *grad_col,
                                           const void *input, const void *offset,
                                           const void *mask, void *grad_offset,
                                           void *grad_mask, void *stream);

/* ---------------------------------------------------------------------
 * Fused backward: all five gradients from grad_output in one call, with the
 * grouped products done per group.  Replaces the reference's Python-side
 * backward composition (mps_deform_conv/__init__.py:245-322: im2col
 * recompute, two torch.mm GEMMs, backward_input, backward_offset_mask) --
 * the schema of torchvision::_deform_conv2d_backward.  Any gradient pointer
 * may be NULL to skip that gradient (grad_mask is only written when
 * use_mask, grad_bias only when non-NULL).  Overwrites what it writes.
 */
DCN_API size_t dcn_backward_workspace_size(const dcn_conv_desc *desc);
DCN_API int dcn_deform_conv2d_backward(const dcn_conv_desc *desc, const void *grad_output,
                               const void *input, const void *weight, const void *offset,
                               const void *mask, void *grad_input, void *grad_weight,
                               void *grad_offset, void *grad_mask, void *grad_bias,
                               void *workspace, size_t workspace_bytes, void *stream);

/* ---------------------------------------------------------------------
 * Training pair.  The forward can leave state resident on the device for
 * the backward of the same call: a channels-last copy of the input and the
 * gathered column tiles of the forward's GEMM (the reference builds the
 * column buffer in its forward and rebuilds it in its backward,
 * deform_conv2d_mps.mm:679-758 and mps_deform_conv/__init__.py:266-273).
 * With it the backward skips the input re-layout and the column re-gather:
 * the weight-gradient GEMM streams the saved tiles.  The state costs
 * dcn_saved_state_bytes() of device memory (about B*Ho*Wo*C*kh*kw*2 bytes)
 * between the two calls.  Problems outside the fused fp16/bf16 kernels (fp32,
 * and shapes those kernels do not take) keep the forward's fp32 column buffer
 * [C*kh*kw][B*Ho*Wo] instead (4 bytes per element), when it fits in 1 GiB;
 * 0 means this problem keeps nothing, and the _train calls then behave like
 * the plain ones.  `saved` must not be modified between the forward and the
 * backward.
 */
DCN_API size_t dcn_saved_state_bytes(const dcn_conv_desc *desc);
DCN_API int dcn_deform_conv2d_forward_train(const dcn_conv_desc *desc, const void *input,
                                            const void *weight, const void *offset,
                                            const void *mask, const void *bias, void *output,
                                            void *saved, size_t saved_bytes, void *workspace,
                                            size_t workspace_bytes, void *stream);
DCN_API int dcn_deform_conv2d_backward_train(const dcn_conv_desc *desc, const void *grad_output,
                                             const void *input, const void *weight,
                                             const void *offset, const void *mask,
                                             const void *saved, size_t saved_bytes,
                                             void *grad_input, void *grad_weight,
                                             void *grad_offset, void *grad_mask, void *grad_bias,
                                             void *workspace, size_t workspace_bytes,
                                             void *stream);

/* ---------------------------------------------------------------------
 * DCNv2 offset/mask head, fused.  No reference counterpart: the reference's
 * ModulatedDeformConv2d (mps_deform_conv/__init__.py:500-511) slices the
 * output of its offset convolution into offsets and mask logits, applies a
 * sigmoid to the logits, and makes both contiguous before the operator runs.
 * Here the operator reads that output in place:
 *   offset_mask [B][OG*T*3][Ho][Wo]: channels [0, 2*OG*T) are the offsets
 *   (layout as `offset` above), channels [2*OG*T, 3*OG*T) are mask logits;
 *   the mask is sigmoid(logit), computed in fp32 inside the kernels.
 * desc->use_mask must be 1.  dcn_head_supported() says whether a problem can
 * take this layout (fp16/bf16 on the tensor-core kernels, offset groups of a
 * multiple of 32 channels, input below 2^31 elements); other problems return
 * DCN_ERR_UNSUPPORTED and use the plain entry points.  Workspace: the
 * dcn_forward_workspace_size / dcn_backward_workspace_size of the same
 * descriptor.  `saved` (dcn_saved_state_bytes, or NULL) works as in the
 * training pair.  The backward writes grad_offset_mask [B][OG*T*3][Ho][Wo]:
 * the offset gradients and the gradients of the mask logits
 * (m * (1 - m) * dL/dm); NULL gradient pointers are skipped.
 */
DCN_API int dcn_head_supported(const dcn_conv_desc *desc);  /* dcn_ex_supported, head = 1, backward */
DCN_API int dcn_deform_conv2d_forward_head(const dcn_conv_desc *desc, const void *input,
                                           const void *weight, const void *offset_mask,
                                           const void *bias, void *output, void *saved,
                                           size_t saved_bytes, void *workspace,
                                           size_t workspace_bytes, void *stream);
DCN_API int dcn_deform_conv2d_backward_head(const dcn_conv_desc *desc, const void *grad_output,
                                            const void *input, const void *weight,
                                            const void *offset_mask, const void *saved,
                                            size_t saved_bytes, void *grad_input,
                                            void *grad_weight, void *grad_offset_mask,
                                            void *grad_bias, void *workspace,
                                            size_t workspace_bytes, void *stream);

/* ---------------------------------------------------------------------
 * Memory formats and the DCNv2 head layout, in one pair of entry points.
 * No reference counterpart (the reference makes every tensor NCHW-contiguous
 * first, deform_conv2d_mps.mm:684-686).
 *   input_layout  applies to input and grad_input,
 *   output_layout applies to output and grad_output:
 *     DCN_LAYOUT_NCHW   [B][C][H][W] as above;
 *     DCN_LAYOUT_NHWC   channels-last [B][H][W][C] (PyTorch's channels_last
 *                       memory format), 16-byte aligned: the gather reads a
 *                       channels-last input in place, and a channels-last
 *                       grad_output is already the pixel-major operand of the
 *                       gradient GEMMs, so the NCHW <-> channels-last passes
 *                       are skipped.
 *   head = 1: `offset` is the DCNv2 head output described above and `mask`
 *             is ignored (grad_offset then receives the head gradient and
 *             grad_mask is ignored).
 * offset, mask and their gradients stay NCHW.  With plain options (both NCHW,
 * no head; or opt == NULL) these calls are the _train pair and every problem
 * is accepted; otherwise dcn_ex_supported(desc, opt, backward) says whether
 * the forward (backward = 0) or the backward (1) takes the problem, and the
 * calls return DCN_ERR_UNSUPPORTED when it does not.  Workspace and `saved`
 * as in the training pair (with a channels-last input the saved state's input
 * copy is not used).
 */
#define DCN_LAYOUT_NCHW 0
#define DCN_LAYOUT_NHWC 1
typedef struct dcn_ex_options {
  int32_t input_layout;   /* input and grad_input */
  int32_t output_layout;  /* output and grad_output */
  int32_t head;           /* 1: offset is a DCNv2 head output [B][OG*T*3][Ho][Wo] */
  int32_t flags;          /* 0, or DCN_EX_WEIGHT_IMAGE (forward only) */
} dcn_ex_options;
/* flags: `weight` is the forward weight image that dcn_weight_image built
 * (forward calls without saved state, tensor-core problems only). */
#define DCN_EX_WEIGHT_IMAGE 1
DCN_API int dcn_ex_supported(const dcn_conv_desc *desc, const dcn_ex_options *opt, int backward);
/* Forward weight image (no reference counterpart).  The tensor-core forward
 * reads its weights as a pre-swizzled tile image [G][K chunks][Cog][64] that
 * every call otherwise rebuilds from `weight`.  A caller whose weights do not
 * change between forward-only calls (inference) builds it once:
 * dcn_weight_image_bytes gives its size (as many elements as the weight; 0
 * when the problem does not take the tensor-core forward), dcn_weight_image
 * writes it (16-byte aligned) on `stream`, and dcn_deform_conv2d_forward_ex
 * with flags = DCN_EX_WEIGHT_IMAGE and `weight` = the image skips the
 * rebuild.  The image depends on the weight values, their dtype and the
 * group split only; rebuild it after the weights change. */
DCN_API size_t dcn_weight_image_bytes(const dcn_conv_desc *desc);
DCN_API int dcn_weight_image(const dcn_conv_desc *desc, const void *weight, void *image, size_t image_bytes,
                             void *stream);
DCN_API int dcn_deform_conv2d_forward_ex(const dcn_conv_desc *desc, const dcn_ex_options *opt,
                                         const void *input, const void *weight, const void *offset,
                                         const void *mask, const void *bias, void *output, void *saved,
                                         size_t saved_bytes, void *workspace, size_t workspace_bytes,
                                         void *stream);
DCN_API int dcn_deform_conv2d_backward_ex(const dcn_conv_desc *desc, const dcn_ex_options *opt,
                                          const void *grad_output, const void *input,
                                          const void *weight, const void *offset, const void *mask,
                                          const void *saved, size_t saved_bytes, void *grad_input,
                                          void *grad_weight, void *grad_offset, void *grad_mask,
                                          void *grad_bias, void *workspace, size_t workspace_bytes,
                                          void *stream);

/* ---------------------------------------------------------------------
 * Backward with a parameter-gradient callback, for overlapping the
 * data-parallel all-reduce of grad_weight / grad_bias with the rest of the
 * backward.  No reference counterpart: the reference's backward
 * (mps_deform_conv/__init__.py:245-322) returns all gradients at once and
 * its caller reduces them afterwards.
 *
 * Same arguments and results as dcn_deform_conv2d_backward_train (`saved`
 * may be NULL).  `params_ready(user_data)` is called exactly once, on the
 * calling thread, after every kernel that writes grad_weight and grad_bias
 * has been enqueued on `stream`: work that the callback enqueues on another
 * stream after waiting on an event it records on `stream` sees the final
 * parameter gradients.  On the tensor-core path the callback comes before
 * the final layout passes of the input / offset / mask gradients are
 * enqueued, so that work runs alongside them; on the other paths it comes
 * after all gradient kernels.  It is not called
 * when the function returns an error before enqueuing anything.  The callback
 * must not call back into this library on the same stream.
 */
typedef void (*dcn_params_ready_fn)(void *user_data);
DCN_API int dcn_deform_conv2d_backward_overlap(const dcn_conv_desc *desc, const void *grad_output,
                                               const void *input, const void *weight,
                                               const void *offset, const void *mask,
                                               const void *saved, size_t saved_bytes,
                                               void *grad_input, void *grad_weight,
                                               void *grad_offset, void *grad_mask,
                                               void *grad_bias, void *workspace,
                                               size_t workspace_bytes, void *stream,
                                               dcn_params_ready_fn params_ready, void *user_data);

/* ---------------------------------------------------------------------
 * Device status.  Kernels with bounded waits record an expired wait in a
 * device-side status word instead of hanging.  This call copies and clears
 * it (it synchronises `stream`): DCN_OK, or DCN_ERR_DEVICE_TIMEOUT.
 */
DCN_API int dcn_device_status(void *stream);

/* ---------------------------------------------------------------------
 * Bounds-checked build (no reference counterpart).  libdcn_b200_bounds.so,
 * built from the same sources with -DDCN_DEBUG_BOUNDS, checks the gather and
 * scatter index math of every kernel (corner, offset, mask, corner-quad
 * record, grad_input and offset/mask-gradient element indices) against the
 * extent of the tensor it addresses.  An index outside it is counted, the
 * first one kept (site, index, element width of the access, extent), and
 * the access redirected to element 0: the kernel neither traps nor stops.
 * dcn_debug_bounds_enabled() is 1 in that build, 0 in the release library.
 * dcn_debug_bounds_read synchronises the device, returns the record summed
 * over the kernel files (all zero in the release library) and clears it when
 * `reset` is non-zero.  Site codes: 1 bilinear corner, 2 coordinate-gradient
 * corner, 3 tensor-core gather input vector, 4 offset element, 5 mask
 * element, 6 corner-quad record, 7 dgrad corner vector, 8 dgrad grad_input
 * reduction, 9 corner-quad reduction, 10 offset/mask gradient element,
 * 11 general-path col2im, 12 general-path channels-last col2im, 13
 * general-path im2col column.
 */
typedef struct dcn_bounds_record {
  uint64_t count;         /* indices found outside their tensor */
  int64_t index, extent;  /* the first one, and its tensor's element count */
  int32_t site, width;    /* where it was computed; elements of the access */
} dcn_bounds_record;
DCN_API int dcn_debug_bounds_enabled(void);
DCN_API int dcn_debug_bounds_read(dcn_bounds_record *out, int reset);

/* Which implementation a descriptor runs on: 1 = the fused fp16/bf16
 * tensor-core (tcgen05) kernels, 0 = the general path (any shape, the fp32
 * path: materialized columns, GEMMs on tcgen05 tf32 MMAs, CUDA-core gather
 * and scatter). */
DCN_API int dcn_uses_tensor_cores(const dcn_conv_desc *desc);

#ifdef __cplusplus
}
#endif

#endif /* DCN_B200_H */
