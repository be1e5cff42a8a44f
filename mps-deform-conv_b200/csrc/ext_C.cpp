// ext_C.cpp -- the Python module `mps_deform_conv._C`: a thin PyTorch layer
// over the C ABI of libdcn_b200.so (include/dcn_b200.h).
//
// It mirrors the reference's pybind11 module of the same name
// (mps_deform_conv/csrc/deform_conv2d_mps.mm:1221-1249): the same four
// functions with the same arguments, plus the fused backward.  This layer
// only turns tensors into pointers and shapes, allocates outputs and
// workspace through the PyTorch caching allocator, and enqueues on the
// current CUDA stream.  All arithmetic is in the library.
#include <torch/extension.h>
#include <ATen/cuda/CUDAContext.h>
#include <c10/cuda/CUDAGuard.h>

#include <exception>
#include <optional>
#include <tuple>
#include <vector>

#include "dcn_b200.h"

namespace {

int32_t dtype_code(const at::Tensor& t) {
  switch (t.scalar_type()) {
    case at::kFloat: return DCN_FLOAT32;
    case at::kHalf: return DCN_FLOAT16;
    case at::kBFloat16: return DCN_BFLOAT16;
    default:
      TORCH_CHECK(false, "deform_conv2d: unsupported dtype ", t.scalar_type(),
                  " (expected float32, float16 or bfloat16)");
  }
  return 0;
}

void check_cuda(const at::Tensor& t, const char* name, const at::Tensor& ref) {
  TORCH_CHECK(t.is_cuda(), name, " must be a CUDA tensor");
  TORCH_CHECK(t.device() == ref.device(), name, " must be on the same device as input (",
              ref.device(), "), got ", t.device());
  TORCH_CHECK(t.scalar_type() == ref.scalar_type(), name, " must have the same dtype as input (",
              ref.scalar_type(), "), got ", t.scalar_type());
}

void check_status(int rc) {
  TORCH_CHECK(rc == DCN_OK, dcn_last_error());
}

dcn_conv_desc make_desc(const at::Tensor& input, int64_t out_channels, int64_t kh, int64_t kw,
                        int64_t sh, int64_t sw, int64_t ph, int64_t pw, int64_t dh, int64_t dw,
                        int64_t groups, int64_t offset_groups, bool use_mask) {
  TORCH_CHECK(input.dim() == 4, "input must be 4-D (N, C, H, W), got ", input.dim(), "-D");
  dcn_conv_desc d;
  d.dtype = dtype_code(input);
  d.use_mask = use_mask ? 1 : 0;
  d.batch = input.size(0);
  d.in_channels = input.size(1);
  d.in_h = input.size(2);
  d.in_w = input.size(3);
  d.out_channels = out_channels;
  d.kernel_h = kh;
  d.kernel_w = kw;
  d.stride_h = sh; d.stride_w = sw;
  d.pad_h = ph; d.pad_w = pw;
  d.dilation_h = dh; d.dilation_w = dw;
  d.n_weight_grps = groups;
  d.n_offset_grps = offset_groups;
  return d;
}

void check_offset_mask(const dcn_conv_desc& d, const at::Tensor& offset, const at::Tensor& mask,
                       int64_t out_h, int64_t out_w) {
  const int64_t T = d.kernel_h * d.kernel_w;
  TORCH_CHECK(offset.dim() == 4 && offset.size(0) == d.batch &&
                  offset.size(1) == 2 * T * d.n_offset_grps && offset.size(2) == out_h &&
                  offset.size(3) == out_w,
              "offset must have shape (", d.batch, ", ", 2 * T * d.n_offset_grps, ", ", out_h, ", ",
              out_w, "), got ", offset.sizes());
  if (d.use_mask) {
    TORCH_CHECK(mask.numel() == d.batch * T * d.n_offset_grps * out_h * out_w,
                "mask must have shape (", d.batch, ", ", T * d.n_offset_grps, ", ", out_h, ", ",
                out_w, "), got ", mask.sizes());
  }
}

at::Tensor workspace(size_t bytes, const at::Tensor& like) {
  return at::empty({(int64_t)std::max<size_t>(bytes, 1)}, like.options().dtype(at::kByte));
}

void* stream_of(const at::Tensor& t) {
  return (void*)at::cuda::getCurrentCUDAStream(t.device().index()).stream();
}

std::pair<int64_t, int64_t> out_size(const dcn_conv_desc& d) {
  int64_t oh = 0, ow = 0;
  check_status(dcn_validate(&d));
  check_status(dcn_output_size(&d, &oh, &ow));
  return {oh, ow};
}

// PyTorch's channels_last memory format (and not also plain contiguous, as
// when C == 1 or H*W == 1).
bool channels_last(const at::Tensor& t) {
  return t.dim() == 4 && !t.is_contiguous() && t.is_contiguous(at::MemoryFormat::ChannelsLast);
}

// Dense tensor in the requested format, 16-byte aligned when channels-last.
at::Tensor in_layout(const at::Tensor& t, bool nhwc) {
  if (!nhwc) return t.contiguous();
  at::Tensor r = t.contiguous(at::MemoryFormat::ChannelsLast);
  if ((reinterpret_cast<uintptr_t>(r.data_ptr()) & 15) != 0) r = r.clone(at::MemoryFormat::ChannelsLast);
  return r;
}

dcn_ex_options ex_options(bool in_nhwc, bool out_nhwc, bool head) {
  dcn_ex_options o;
  o.input_layout = in_nhwc ? DCN_LAYOUT_NHWC : DCN_LAYOUT_NCHW;
  o.output_layout = out_nhwc ? DCN_LAYOUT_NHWC : DCN_LAYOUT_NCHW;
  o.head = head ? 1 : 0;
  o.flags = 0;
  return o;
}

}  // namespace

// Reference: deform_conv2d_forward_mps, deform_conv2d_mps.mm:603-800.
at::Tensor deform_conv2d_forward(const at::Tensor& input, const at::Tensor& weight,
                                 const at::Tensor& offset, const at::Tensor& mask,
                                 const at::Tensor& bias, int64_t stride_h, int64_t stride_w,
                                 int64_t pad_h, int64_t pad_w, int64_t dilation_h,
                                 int64_t dilation_w, int64_t n_weight_grps, int64_t n_offset_grps,
                                 bool use_mask) {
  TORCH_CHECK(input.is_cuda(), "input must be a CUDA tensor");
  check_cuda(weight, "weight", input);
  check_cuda(offset, "offset", input);
  const bool has_mask = use_mask && mask.numel() > 0;
  if (has_mask) check_cuda(mask, "mask", input);
  const bool has_bias = bias.defined() && bias.numel() > 0;
  if (has_bias) check_cuda(bias, "bias", input);
  TORCH_CHECK(weight.dim() == 4, "weight must be 4-D");
  c10::cuda::CUDAGuard guard(input.device());
  dcn_conv_desc d = make_desc(input, weight.size(0), weight.size(2), weight.size(3), stride_h,
                              stride_w, pad_h, pad_w, dilation_h, dilation_w, n_weight_grps,
                              n_offset_grps, has_mask);
  TORCH_CHECK(weight.size(1) * n_weight_grps == input.size(1), "weight in_channels (",
              weight.size(1), ") x n_weight_grps (", n_weight_grps, ") must equal in_channels (",
              input.size(1), ")");
  auto [oh, ow] = out_size(d);
  check_offset_mask(d, offset, mask, oh, ow);
  if (has_bias) TORCH_CHECK(bias.numel() == weight.size(0), "bias must have out_channels elements");
  auto x = input.contiguous(), w = weight.contiguous(), off = offset.contiguous();
  auto m = has_mask ? mask.contiguous() : at::Tensor();
  auto b = has_bias ? bias.contiguous() : at::Tensor();
  auto out = at::empty({d.batch, d.out_channels, oh, ow}, input.options());
  auto ws = workspace(dcn_forward_workspace_size(&d), input);
  check_status(dcn_deform_conv2d_forward(&d, x.data_ptr(), w.data_ptr(), off.data_ptr(),
                                         has_mask ? m.data_ptr() : nullptr,
                                         has_bias ? b.data_ptr() : nullptr, out.data_ptr(),
                                         ws.data_ptr(), (size_t)ws.numel(), stream_of(input)));
  return out;
}

// Training forward: like deform_conv2d_forward, and also returns the device
// state the backward can reuse (a uint8 tensor; empty when this problem keeps
// nothing).
std::tuple<at::Tensor, at::Tensor> deform_conv2d_forward_train(
    const at::Tensor& input, const at::Tensor& weight, const at::Tensor& offset, const at::Tensor& mask,
    const at::Tensor& bias, int64_t stride_h, int64_t stride_w, int64_t pad_h, int64_t pad_w,
    int64_t dilation_h, int64_t dilation_w, int64_t n_weight_grps, int64_t n_offset_grps, bool use_mask) {
  TORCH_CHECK(input.is_cuda(), "input must be a CUDA tensor");
  check_cuda(weight, "weight", input);
  check_cuda(offset, "offset", input);
  const bool has_mask = use_mask && mask.numel() > 0;
  if (has_mask) check_cuda(mask, "mask", input);
  const bool has_bias = bias.defined() && bias.numel() > 0;
  if (has_bias) check_cuda(bias, "bias", input);
  TORCH_CHECK(weight.dim() == 4, "weight must be 4-D");
  c10::cuda::CUDAGuard guard(input.device());
  dcn_conv_desc d = make_desc(input, weight.size(0), weight.size(2), weight.size(3), stride_h,
                              stride_w, pad_h, pad_w, dilation_h, dilation_w, n_weight_grps,
                              n_offset_grps, has_mask);
  TORCH_CHECK(weight.size(1) * n_weight_grps == input.size(1), "weight in_channels (",
              weight.size(1), ") x n_weight_grps (", n_weight_grps, ") must equal in_channels (",
              input.size(1), ")");
  auto [oh, ow] = out_size(d);
  check_offset_mask(d, offset, mask, oh, ow);
  if (has_bias) TORCH_CHECK(bias.numel() == weight.size(0), "bias must have out_channels elements");
  auto x = input.contiguous(), w = weight.contiguous(), off = offset.contiguous();
  auto m = has_mask ? mask.contiguous() : at::Tensor();
  auto b = has_bias ? bias.contiguous() : at::Tensor();
  auto out = at::empty({d.batch, d.out_channels, oh, ow}, input.options());
  const size_t sbytes = dcn_saved_state_bytes(&d);
  auto saved = at::empty({(int64_t)sbytes}, input.options().dtype(at::kByte));
  auto ws = workspace(dcn_forward_workspace_size(&d), input);
  check_status(dcn_deform_conv2d_forward_train(&d, x.data_ptr(), w.data_ptr(), off.data_ptr(),
                                               has_mask ? m.data_ptr() : nullptr,
                                               has_bias ? b.data_ptr() : nullptr, out.data_ptr(),
                                               sbytes ? saved.data_ptr() : nullptr, sbytes,
                                               ws.data_ptr(), (size_t)ws.numel(), stream_of(input)));
  return {out, saved};
}

// Forward weight image of `weight` for this problem (dcn_weight_image), or an
// empty tensor when the problem does not take the tensor-core forward.
at::Tensor weight_image(const at::Tensor& input, const at::Tensor& weight, int64_t stride_h, int64_t stride_w,
                        int64_t pad_h, int64_t pad_w, int64_t dilation_h, int64_t dilation_w,
                        int64_t n_weight_grps, int64_t n_offset_grps, bool use_mask) {
  TORCH_CHECK(input.is_cuda(), "input must be a CUDA tensor");
  check_cuda(weight, "weight", input);
  TORCH_CHECK(weight.dim() == 4, "weight must be 4-D");
  c10::cuda::CUDAGuard guard(input.device());
  dcn_conv_desc d = make_desc(input, weight.size(0), weight.size(2), weight.size(3), stride_h, stride_w, pad_h,
                              pad_w, dilation_h, dilation_w, n_weight_grps, n_offset_grps, use_mask);
  const size_t n = dcn_weight_image_bytes(&d);
  auto image = at::empty({(int64_t)n}, input.options().dtype(at::kByte));
  if (n) {
    auto w = weight.contiguous();
    check_status(dcn_weight_image(&d, w.data_ptr(), image.data_ptr(), n, stream_of(input)));
  }
  return image;
}

// Forward of the autograd path: like forward_train, and a channels_last input
// gives a channels_last output (read and written in place by the tensor-core
// kernels; other problems run on NCHW copies and convert the output back).
// keep_saved: also return the state the backward reuses (else an empty tensor).
// image: the forward weight image of `weight` (weight_image), used instead of
// rebuilding it when non-empty and nothing is kept.
std::tuple<at::Tensor, at::Tensor> deform_conv2d_forward_ex(
    const at::Tensor& input, const at::Tensor& weight, const at::Tensor& offset, const at::Tensor& mask,
    const at::Tensor& bias, int64_t stride_h, int64_t stride_w, int64_t pad_h, int64_t pad_w,
    int64_t dilation_h, int64_t dilation_w, int64_t n_weight_grps, int64_t n_offset_grps, bool use_mask,
    bool keep_saved, const at::Tensor& image) {
  TORCH_CHECK(input.is_cuda(), "input must be a CUDA tensor");
  check_cuda(weight, "weight", input);
  check_cuda(offset, "offset", input);
  const bool has_mask = use_mask && mask.numel() > 0;
  if (has_mask) check_cuda(mask, "mask", input);
  const bool has_bias = bias.defined() && bias.numel() > 0;
  if (has_bias) check_cuda(bias, "bias", input);
  TORCH_CHECK(weight.dim() == 4, "weight must be 4-D");
  c10::cuda::CUDAGuard guard(input.device());
  dcn_conv_desc d = make_desc(input, weight.size(0), weight.size(2), weight.size(3), stride_h,
                              stride_w, pad_h, pad_w, dilation_h, dilation_w, n_weight_grps,
                              n_offset_grps, has_mask);
  TORCH_CHECK(weight.size(1) * n_weight_grps == input.size(1), "weight in_channels (",
              weight.size(1), ") x n_weight_grps (", n_weight_grps, ") must equal in_channels (",
              input.size(1), ")");
  auto [oh, ow] = out_size(d);
  check_offset_mask(d, offset, mask, oh, ow);
  if (has_bias) TORCH_CHECK(bias.numel() == weight.size(0), "bias must have out_channels elements");
  const bool want_nhwc = channels_last(input);
  dcn_ex_options o = ex_options(want_nhwc, want_nhwc, false);
  const bool nhwc = want_nhwc && dcn_ex_supported(&d, &o, 0);
  if (!nhwc) o = ex_options(false, false, false);
  // an image serves every problem of this weight that takes the tensor-core
  // forward (its size is then the weight's); others rebuild nothing and ignore it
  const bool use_image = !keep_saved && image.defined() && image.numel() > 0 &&
                         (size_t)image.numel() == dcn_weight_image_bytes(&d);
  if (use_image) {
    TORCH_CHECK(image.is_cuda() && image.device() == input.device() && image.is_contiguous(),
                "weight image must be a contiguous tensor on the input's device");
    o.flags = DCN_EX_WEIGHT_IMAGE;
  }
  auto x = in_layout(input, nhwc), w = use_image ? image : weight.contiguous(), off = offset.contiguous();
  auto m = has_mask ? mask.contiguous() : at::Tensor();
  auto b = has_bias ? bias.contiguous() : at::Tensor();
  auto out = at::empty({d.batch, d.out_channels, oh, ow},
                       input.options().memory_format(nhwc ? at::MemoryFormat::ChannelsLast : at::MemoryFormat::Contiguous));
  const size_t sbytes = keep_saved ? dcn_saved_state_bytes(&d) : 0;
  auto saved = at::empty({(int64_t)sbytes}, input.options().dtype(at::kByte));
  auto ws = workspace(dcn_forward_workspace_size(&d), input);
  check_status(dcn_deform_conv2d_forward_ex(&d, &o, x.data_ptr(), w.data_ptr(), off.data_ptr(),
                                            has_mask ? m.data_ptr() : nullptr, has_bias ? b.data_ptr() : nullptr,
                                            out.data_ptr(), sbytes ? saved.data_ptr() : nullptr, sbytes,
                                            ws.data_ptr(), (size_t)ws.numel(), stream_of(input)));
  if (want_nhwc && !nhwc) out = out.contiguous(at::MemoryFormat::ChannelsLast);
  return {out, saved};
}

// Reference: deformable_im2col_mps, deform_conv2d_mps.mm:806-936.
at::Tensor deformable_im2col(const at::Tensor& input, const at::Tensor& offset,
                             const at::Tensor& mask, int64_t kernel_h, int64_t kernel_w,
                             int64_t stride_h, int64_t stride_w, int64_t pad_h, int64_t pad_w,
                             int64_t dilation_h, int64_t dilation_w, int64_t n_offset_grps,
                             bool use_mask) {
  TORCH_CHECK(input.is_cuda(), "input must be a CUDA tensor");
  check_cuda(offset, "offset", input);
  const bool has_mask = use_mask && mask.numel() > 0;
  if (has_mask) check_cuda(mask, "mask", input);
  c10::cuda::CUDAGuard guard(input.device());
  dcn_conv_desc d = make_desc(input, 1, kernel_h, kernel_w, stride_h, stride_w, pad_h, pad_w,
                              dilation_h, dilation_w, 1, n_offset_grps, has_mask);
  auto [oh, ow] = out_size(d);
  check_offset_mask(d, offset, mask, oh, ow);
  auto x = input.contiguous(), off = offset.contiguous();
  auto m = has_mask ? mask.contiguous() : at::Tensor();
  auto cols = at::empty({d.in_channels * kernel_h * kernel_w, d.batch * oh * ow}, input.options());
  check_status(dcn_deformable_im2col(&d, x.data_ptr(), off.data_ptr(),
                                     has_mask ? m.data_ptr() : nullptr, cols.data_ptr(),
                                     stream_of(input)));
  return cols;
}

// Reference: deform_conv2d_backward_input_mps, deform_conv2d_mps.mm:942-1069.
at::Tensor deform_conv2d_backward_input(const at::Tensor& grad_col, const at::Tensor& input,
                                        const at::Tensor& offset, const at::Tensor& mask,
                                        int64_t in_h, int64_t in_w, int64_t stride_h,
                                        int64_t stride_w, int64_t pad_h, int64_t pad_w,
                                        int64_t dilation_h, int64_t dilation_w, int64_t kernel_h,
                                        int64_t kernel_w, int64_t n_offset_grps, bool use_mask) {
  TORCH_CHECK(input.is_cuda(), "input must be a CUDA tensor");
  check_cuda(grad_col, "grad_col", input);
  check_cuda(offset, "offset", input);
  const bool has_mask = use_mask && mask.numel() > 0;
  if (has_mask) check_cuda(mask, "mask", input);
  TORCH_CHECK(input.size(2) == in_h && input.size(3) == in_w, "in_h/in_w must match input");
  c10::cuda::CUDAGuard guard(input.device());
  dcn_conv_desc d = make_desc(input, 1, kernel_h, kernel_w, stride_h, stride_w, pad_h, pad_w,
                              dilation_h, dilation_w, 1, n_offset_grps, has_mask);
  auto [oh, ow] = out_size(d);
  check_offset_mask(d, offset, mask, oh, ow);
  TORCH_CHECK(grad_col.numel() == d.in_channels * kernel_h * kernel_w * d.batch * oh * ow,
              "grad_col must have shape (", d.in_channels * kernel_h * kernel_w, ", ",
              d.batch * oh * ow, ")");
  auto gc = grad_col.contiguous(), off = offset.contiguous();
  auto m = has_mask ? mask.contiguous() : at::Tensor();
  auto gin = at::empty_like(input, at::MemoryFormat::Contiguous);
  auto ws = workspace(dcn_backward_input_workspace_size(&d), input);
  check_status(dcn_deform_conv2d_backward_input(&d, gc.data_ptr(), off.data_ptr(),
                                                has_mask ? m.data_ptr() : nullptr, gin.data_ptr(),
                                                ws.data_ptr(), (size_t)ws.numel(),
                                                stream_of(input)));
  return gin;
}

// Reference: deform_conv2d_backward_offset_mask_mps, deform_conv2d_mps.mm:1075-1215.
std::tuple<at::Tensor, at::Tensor> deform_conv2d_backward_offset_mask(
    const at::Tensor& grad_col, const at::Tensor& input, const at::Tensor& offset,
    const at::Tensor& mask, int64_t kernel_h, int64_t kernel_w, int64_t stride_h, int64_t stride_w,
    int64_t pad_h, int64_t pad_w, int64_t dilation_h, int64_t dilation_w, int64_t n_offset_grps,
    bool use_mask) {
  TORCH_CHECK(input.is_cuda(), "input must be a CUDA tensor");
  check_cuda(grad_col, "grad_col", input);
  check_cuda(offset, "offset", input);
  const bool has_mask = use_mask && mask.numel() > 0;
  if (has_mask) check_cuda(mask, "mask", input);
  c10::cuda::CUDAGuard guard(input.device());
  dcn_conv_desc d = make_desc(input, 1, kernel_h, kernel_w, stride_h, stride_w, pad_h, pad_w,
                              dilation_h, dilation_w, 1, n_offset_grps, has_mask);
  auto [oh, ow] = out_size(d);
  check_offset_mask(d, offset, mask, oh, ow);
  TORCH_CHECK(grad_col.numel() == d.in_channels * kernel_h * kernel_w * d.batch * oh * ow,
              "grad_col has the wrong number of elements");
  auto gc = grad_col.contiguous(), x = input.contiguous(), off = offset.contiguous();
  auto m = has_mask ? mask.contiguous() : at::Tensor();
  auto goff = at::empty_like(off);
  auto gmask = has_mask ? at::empty_like(m) : at::empty({0}, input.options());
  check_status(dcn_deform_conv2d_backward_offset_mask(
      &d, gc.data_ptr(), x.data_ptr(), off.data_ptr(), has_mask ? m.data_ptr() : nullptr,
      goff.data_ptr(), has_mask ? gmask.data_ptr() : nullptr, stream_of(input)));
  return {goff, gmask};
}

// Fused backward (schema of torchvision::_deform_conv2d_backward, plus an
// output mask that skips gradients nobody asked for).  Replaces the
// reference's Python composition at mps_deform_conv/__init__.py:245-322.
// Returns (grad_input, grad_weight, grad_offset, grad_mask, grad_bias);
// skipped or absent gradients are undefined tensors.
std::tuple<at::Tensor, at::Tensor, at::Tensor, at::Tensor, at::Tensor> deform_conv2d_backward(
    const at::Tensor& grad_output, const at::Tensor& input, const at::Tensor& weight,
    const at::Tensor& offset, const at::Tensor& mask, const at::Tensor& bias, int64_t stride_h,
    int64_t stride_w, int64_t pad_h, int64_t pad_w, int64_t dilation_h, int64_t dilation_w,
    int64_t n_weight_grps, int64_t n_offset_grps, bool use_mask, std::vector<bool> output_mask,
    const std::optional<at::Tensor>& saved_opt, const std::optional<py::function>& params_ready) {
  TORCH_CHECK(input.is_cuda(), "input must be a CUDA tensor");
  check_cuda(grad_output, "grad_output", input);
  check_cuda(weight, "weight", input);
  check_cuda(offset, "offset", input);
  const bool has_mask = use_mask && mask.numel() > 0;
  if (has_mask) check_cuda(mask, "mask", input);
  const bool has_bias = bias.defined() && bias.numel() > 0;
  if (output_mask.size() < 5) output_mask.resize(5, true);
  c10::cuda::CUDAGuard guard(input.device());
  dcn_conv_desc d = make_desc(input, weight.size(0), weight.size(2), weight.size(3), stride_h,
                              stride_w, pad_h, pad_w, dilation_h, dilation_w, n_weight_grps,
                              n_offset_grps, has_mask);
  auto [oh, ow] = out_size(d);
  check_offset_mask(d, offset, mask, oh, ow);
  TORCH_CHECK(grad_output.dim() == 4 && grad_output.size(0) == d.batch &&
                  grad_output.size(1) == d.out_channels && grad_output.size(2) == oh &&
                  grad_output.size(3) == ow,
              "grad_output has shape ", grad_output.sizes(), ", expected (", d.batch, ", ",
              d.out_channels, ", ", oh, ", ", ow, ")");
  // channels_last input / grad_output are used in place when the tensor-core
  // kernels take the problem (grad_input then comes back channels_last too)
  bool in_nhwc = channels_last(input), out_nhwc = channels_last(grad_output);
  dcn_ex_options o = ex_options(in_nhwc, out_nhwc, false);
  if ((in_nhwc || out_nhwc) && !dcn_ex_supported(&d, &o, 1)) {
    in_nhwc = out_nhwc = false;
    o = ex_options(false, false, false);
  }
  auto go = in_layout(grad_output, out_nhwc), x = in_layout(input, in_nhwc), w = weight.contiguous(),
       off = offset.contiguous();
  auto m = has_mask ? mask.contiguous() : at::Tensor();
  at::Tensor gin, gw, goff, gm, gb;
  if (output_mask[0]) gin = at::empty_like(x);
  if (output_mask[1]) gw = at::empty_like(w);
  if (output_mask[2]) goff = at::empty_like(off);
  if (output_mask[3] && has_mask) gm = at::empty_like(m);
  if (output_mask[4] && has_bias) gb = at::empty({d.out_channels}, input.options());
  auto ws = workspace(dcn_backward_workspace_size(&d), input);
  auto ptr = [](const at::Tensor& t) -> void* { return t.defined() ? t.data_ptr() : nullptr; };
  const at::Tensor saved = saved_opt.has_value() ? *saved_opt : at::Tensor();
  const bool has_saved = saved.defined() && saved.numel() > 0;
  if (has_saved) {
    TORCH_CHECK(saved.is_cuda() && saved.device() == input.device() && saved.scalar_type() == at::kByte &&
                    saved.is_contiguous(),
                "saved state must be a contiguous uint8 tensor on the input's device");
  }
  const bool hook = params_ready.has_value() && !params_ready->is_none();
  if (!hook || in_nhwc || out_nhwc) {
    check_status(dcn_deform_conv2d_backward_ex(
        &d, &o, go.data_ptr(), x.data_ptr(), w.data_ptr(), off.data_ptr(), has_mask ? m.data_ptr() : nullptr,
        has_saved ? saved.data_ptr() : nullptr, has_saved ? (size_t)saved.numel() : 0, ptr(gin), ptr(gw),
        ptr(goff), ptr(gm), ptr(gb), ws.data_ptr(), (size_t)ws.numel(), stream_of(input)));
    if (hook)  // channels-last layouts have no callback entry point: the hook runs after the whole backward
      (*params_ready)(gw.defined() ? py::cast(gw) : py::none(), gb.defined() ? py::cast(gb) : py::none());
    return {gin, gw, goff, gm, gb};
  }
  // params_ready(grad_weight, grad_bias) runs inside the library call once
  // both are enqueued; a Python exception is held and re-raised after the
  // call returns, never thrown through the C ABI
  struct Ready {
    const py::function* fn;
    const at::Tensor* gw;
    const at::Tensor* gb;
    std::exception_ptr err;
  } ready{&*params_ready, &gw, &gb, nullptr};
  auto tramp = [](void* u) {
    auto* r = static_cast<Ready*>(u);
    try {
      (*r->fn)(r->gw->defined() ? py::cast(*r->gw) : py::none(), r->gb->defined() ? py::cast(*r->gb) : py::none());
    } catch (...) {
      r->err = std::current_exception();
    }
  };
  const int rc = dcn_deform_conv2d_backward_overlap(
      &d, go.data_ptr(), x.data_ptr(), w.data_ptr(), off.data_ptr(), has_mask ? m.data_ptr() : nullptr,
      has_saved ? saved.data_ptr() : nullptr, has_saved ? (size_t)saved.numel() : 0, ptr(gin), ptr(gw),
      ptr(goff), ptr(gm), ptr(gb), ws.data_ptr(), (size_t)ws.numel(), stream_of(input), tramp, &ready);
  if (ready.err) std::rethrow_exception(ready.err);
  check_status(rc);
  return {gin, gw, goff, gm, gb};
}

// ---------------------------------------------------------------- DCNv2 head layout
// offset_mask [B][3*OG*T][Ho][Wo] as ModulatedDeformConv2d's offset convolution
// produces it (offsets, then mask logits); no reference counterpart (the
// reference slices it and applies the sigmoid in Python, __init__.py:500-511).
dcn_conv_desc head_desc(const at::Tensor& input, const at::Tensor& weight, const at::Tensor& offset_mask,
                        int64_t stride_h, int64_t stride_w, int64_t pad_h, int64_t pad_w, int64_t dilation_h,
                        int64_t dilation_w, int64_t n_weight_grps, int64_t n_offset_grps) {
  TORCH_CHECK(weight.dim() == 4, "weight must be 4-D");
  dcn_conv_desc d = make_desc(input, weight.size(0), weight.size(2), weight.size(3), stride_h, stride_w, pad_h,
                              pad_w, dilation_h, dilation_w, n_weight_grps, n_offset_grps, true);
  TORCH_CHECK(weight.size(1) * n_weight_grps == input.size(1), "weight in_channels (", weight.size(1),
              ") x n_weight_grps (", n_weight_grps, ") must equal in_channels (", input.size(1), ")");
  auto [oh, ow] = out_size(d);
  const int64_t ch = 3 * n_offset_grps * weight.size(2) * weight.size(3);
  TORCH_CHECK(offset_mask.dim() == 4 && offset_mask.size(0) == d.batch && offset_mask.size(1) == ch &&
                  offset_mask.size(2) == oh && offset_mask.size(3) == ow,
              "offset_mask has shape ", offset_mask.sizes(), ", expected (", d.batch, ", ", ch, ", ", oh, ", ", ow,
              ")");
  return d;
}

bool head_supported(const at::Tensor& input, const at::Tensor& weight, int64_t stride_h, int64_t stride_w,
                    int64_t pad_h, int64_t pad_w, int64_t dilation_h, int64_t dilation_w, int64_t n_weight_grps,
                    int64_t n_offset_grps) {
  if (weight.dim() != 4) return false;
  dcn_conv_desc d = make_desc(input, weight.size(0), weight.size(2), weight.size(3), stride_h, stride_w, pad_h,
                              pad_w, dilation_h, dilation_w, n_weight_grps, n_offset_grps, true);
  return dcn_head_supported(&d) != 0;
}

std::tuple<at::Tensor, at::Tensor> deform_conv2d_forward_head(
    const at::Tensor& input, const at::Tensor& weight, const at::Tensor& offset_mask, const at::Tensor& bias,
    int64_t stride_h, int64_t stride_w, int64_t pad_h, int64_t pad_w, int64_t dilation_h, int64_t dilation_w,
    int64_t n_weight_grps, int64_t n_offset_grps, bool keep_saved) {
  TORCH_CHECK(input.is_cuda(), "input must be a CUDA tensor");
  check_cuda(weight, "weight", input);
  check_cuda(offset_mask, "offset_mask", input);
  const bool has_bias = bias.defined() && bias.numel() > 0;
  if (has_bias) check_cuda(bias, "bias", input);
  c10::cuda::CUDAGuard guard(input.device());
  dcn_conv_desc d = head_desc(input, weight, offset_mask, stride_h, stride_w, pad_h, pad_w, dilation_h, dilation_w,
                              n_weight_grps, n_offset_grps);
  if (has_bias) TORCH_CHECK(bias.numel() == weight.size(0), "bias must have out_channels elements");
  auto [oh, ow] = out_size(d);
  const bool want_nhwc = channels_last(input);
  dcn_ex_options o = ex_options(want_nhwc, want_nhwc, true);
  const bool nhwc = want_nhwc && dcn_ex_supported(&d, &o, 0);
  if (!nhwc) o = ex_options(false, false, true);
  auto x = in_layout(input, nhwc), w = weight.contiguous(), om = offset_mask.contiguous();
  auto b = has_bias ? bias.contiguous() : at::Tensor();
  auto out = at::empty({d.batch, d.out_channels, oh, ow},
                       input.options().memory_format(nhwc ? at::MemoryFormat::ChannelsLast : at::MemoryFormat::Contiguous));
  const size_t sbytes = keep_saved ? dcn_saved_state_bytes(&d) : 0;
  auto saved = at::empty({(int64_t)sbytes}, input.options().dtype(at::kByte));
  auto ws = workspace(dcn_forward_workspace_size(&d), input);
  check_status(dcn_deform_conv2d_forward_ex(&d, &o, x.data_ptr(), w.data_ptr(), om.data_ptr(), nullptr,
                                            has_bias ? b.data_ptr() : nullptr, out.data_ptr(),
                                            sbytes ? saved.data_ptr() : nullptr, sbytes, ws.data_ptr(),
                                            (size_t)ws.numel(), stream_of(input)));
  if (want_nhwc && !nhwc) out = out.contiguous(at::MemoryFormat::ChannelsLast);
  return {out, saved};
}

// output_mask: (input, weight, offset_mask, bias)
std::tuple<at::Tensor, at::Tensor, at::Tensor, at::Tensor> deform_conv2d_backward_head(
    const at::Tensor& grad_output, const at::Tensor& input, const at::Tensor& weight, const at::Tensor& offset_mask,
    const at::Tensor& bias, int64_t stride_h, int64_t stride_w, int64_t pad_h, int64_t pad_w, int64_t dilation_h,
    int64_t dilation_w, int64_t n_weight_grps, int64_t n_offset_grps, std::vector<bool> output_mask,
    const std::optional<at::Tensor>& saved_opt) {
  TORCH_CHECK(input.is_cuda(), "input must be a CUDA tensor");
  check_cuda(grad_output, "grad_output", input);
  check_cuda(weight, "weight", input);
  check_cuda(offset_mask, "offset_mask", input);
  const bool has_bias = bias.defined() && bias.numel() > 0;
  if (output_mask.size() < 4) output_mask.resize(4, true);
  c10::cuda::CUDAGuard guard(input.device());
  dcn_conv_desc d = head_desc(input, weight, offset_mask, stride_h, stride_w, pad_h, pad_w, dilation_h, dilation_w,
                              n_weight_grps, n_offset_grps);
  auto [oh, ow] = out_size(d);
  TORCH_CHECK(grad_output.dim() == 4 && grad_output.size(0) == d.batch && grad_output.size(1) == d.out_channels &&
                  grad_output.size(2) == oh && grad_output.size(3) == ow,
              "grad_output has shape ", grad_output.sizes(), ", expected (", d.batch, ", ", d.out_channels, ", ", oh,
              ", ", ow, ")");
  bool in_nhwc = channels_last(input), out_nhwc = channels_last(grad_output);
  dcn_ex_options o = ex_options(in_nhwc, out_nhwc, true);
  if ((in_nhwc || out_nhwc) && !dcn_ex_supported(&d, &o, 1)) {
    in_nhwc = out_nhwc = false;
    o = ex_options(false, false, true);
  }
  auto go = in_layout(grad_output, out_nhwc), x = in_layout(input, in_nhwc), w = weight.contiguous(),
       om = offset_mask.contiguous();
  at::Tensor gin, gw, gom, gb;
  if (output_mask[0]) gin = at::empty_like(x);
  if (output_mask[1]) gw = at::empty_like(w);
  if (output_mask[2]) gom = at::empty_like(om);
  if (output_mask[3] && has_bias) gb = at::empty({d.out_channels}, input.options());
  auto ws = workspace(dcn_backward_workspace_size(&d), input);
  auto ptr = [](const at::Tensor& t) -> void* { return t.defined() ? t.data_ptr() : nullptr; };
  const at::Tensor saved = saved_opt.has_value() ? *saved_opt : at::Tensor();
  const bool has_saved = saved.defined() && saved.numel() > 0;
  if (has_saved)
    TORCH_CHECK(saved.is_cuda() && saved.device() == input.device() && saved.scalar_type() == at::kByte &&
                    saved.is_contiguous(),
                "saved state must be a contiguous uint8 tensor on the input's device");
  check_status(dcn_deform_conv2d_backward_ex(
      &d, &o, go.data_ptr(), x.data_ptr(), w.data_ptr(), om.data_ptr(), nullptr,
      has_saved ? saved.data_ptr() : nullptr, has_saved ? (size_t)saved.numel() : 0, ptr(gin), ptr(gw), ptr(gom),
      nullptr, ptr(gb), ws.data_ptr(), (size_t)ws.numel(), stream_of(input)));
  return {gin, gw, gom, gb};
}

bool uses_tensor_cores(const at::Tensor& input, const at::Tensor& weight, int64_t stride_h,
                       int64_t stride_w, int64_t pad_h, int64_t pad_w, int64_t dilation_h,
                       int64_t dilation_w, int64_t n_weight_grps, int64_t n_offset_grps,
                       bool use_mask) {
  dcn_conv_desc d = make_desc(input, weight.size(0), weight.size(2), weight.size(3), stride_h,
                              stride_w, pad_h, pad_w, dilation_h, dilation_w, n_weight_grps,
                              n_offset_grps, use_mask);
  return dcn_uses_tensor_cores(&d) != 0;
}

void device_status() {
  check_status(dcn_device_status((void*)at::cuda::getCurrentCUDAStream().stream()));
}

PYBIND11_MODULE(TORCH_EXTENSION_NAME, m) {
  m.doc() = "B200 deformable convolution: PyTorch bindings over the dcn_b200 C ABI";
  m.def("deform_conv2d_forward", &deform_conv2d_forward, "Deformable Convolution 2D forward pass",
        py::arg("input"), py::arg("weight"), py::arg("offset"), py::arg("mask"), py::arg("bias"),
        py::arg("stride_h"), py::arg("stride_w"), py::arg("pad_h"), py::arg("pad_w"),
        py::arg("dilation_h"), py::arg("dilation_w"), py::arg("n_weight_grps"),
        py::arg("n_offset_grps"), py::arg("use_mask"));
  m.def("deformable_im2col", &deformable_im2col, "Deformable im2col (column buffer)");
  m.def("deform_conv2d_backward_input", &deform_conv2d_backward_input,
        "Deformable Convolution 2D backward pass for input gradient");
  m.def("deform_conv2d_backward_offset_mask", &deform_conv2d_backward_offset_mask,
        "Deformable Convolution 2D backward pass for offset and mask gradients");
  m.def("deform_conv2d_backward", &deform_conv2d_backward,
        "Fused backward: (grad_input, grad_weight, grad_offset, grad_mask, grad_bias)",
        py::arg("grad_output"), py::arg("input"), py::arg("weight"), py::arg("offset"),
        py::arg("mask"), py::arg("bias"), py::arg("stride_h"), py::arg("stride_w"),
        py::arg("pad_h"), py::arg("pad_w"), py::arg("dilation_h"), py::arg("dilation_w"),
        py::arg("n_weight_grps"), py::arg("n_offset_grps"), py::arg("use_mask"),
        py::arg("output_mask") = std::vector<bool>{true, true, true, true, true},
        py::arg("saved") = py::none(), py::arg("params_ready") = py::none());
  m.def("deform_conv2d_forward_ex", &deform_conv2d_forward_ex,
        "Forward of the autograd path (channels_last in, channels_last out): (output, saved)");
  m.def("weight_image", &weight_image,
        "Forward weight image for forward-only calls (empty when the problem is not on the tensor cores)");
  m.def("deform_conv2d_forward_train", &deform_conv2d_forward_train,
        "Forward that also returns the device state its backward reuses: (output, saved)");
  m.def("uses_tensor_cores", &uses_tensor_cores, "True when the tcgen05 kernels run this problem");
  m.def("head_supported", &head_supported, "True when the fused DCNv2 offset/mask head layout runs this problem");
  m.def("deform_conv2d_forward_head", &deform_conv2d_forward_head,
        "Forward reading offsets and mask logits in place from the DCNv2 head output: (output, saved)");
  m.def("deform_conv2d_backward_head", &deform_conv2d_backward_head,
        "Backward of forward_head: (grad_input, grad_weight, grad_offset_mask, grad_bias)",
        py::arg("grad_output"), py::arg("input"), py::arg("weight"), py::arg("offset_mask"), py::arg("bias"),
        py::arg("stride_h"), py::arg("stride_w"), py::arg("pad_h"), py::arg("pad_w"), py::arg("dilation_h"),
        py::arg("dilation_w"), py::arg("n_weight_grps"), py::arg("n_offset_grps"),
        py::arg("output_mask") = std::vector<bool>{true, true, true, true}, py::arg("saved") = py::none());
  m.def("device_status", &device_status, "Raise if a kernel's bounded wait expired");
  m.def("abi_version", &dcn_abi_version);
}
