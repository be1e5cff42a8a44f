// dcn_tc.h -- tensor-core (tcgen05 / TMEM) kernel family: which problems it
// takes, how much workspace it needs, and its launchers.
#pragma once

#include "dcn_internal.h"

namespace dcn {

// True when the tensor-core kernels handle this problem's forward / backward
// (fp16/bf16 and the channel constraints listed in dcn_tc.cu).
bool tc_forward_supported(const dcn_conv_desc& d, const Geom& g);
bool tc_backward_supported(const dcn_conv_desc& d, const Geom& g);
size_t tc_forward_workspace(const dcn_conv_desc& d, const Geom& g);
size_t tc_backward_workspace(const dcn_conv_desc& d, const Geom& g);

// Training state the forward can leave resident for the backward:
//   xh    channels-last copy of the input [B][H][W][C]
//   cols  the forward's gathered A-operand tiles [G][n_tiles][NKC][16 KB],
//         each tile [128 pixels][64 channels] in the 128-byte-swizzled
//         shared-memory image, so the weight-gradient GEMM streams them back
//         with bulk copies instead of gathering again.
//   xq    corner-quad records of the input (offset groups of 8 channels)
//   wdt   dgrad's W^T tile image of the weight (the backward does not
//         rebuild it: the weight must not change between the two calls)
struct SavedLayout {
  size_t xh, cols, xq, wdt, total;
};

// Host: dgrad's W^T tile image of the weight into wdt (dcn_tc_bwd.cu).
template <typename T>
void weight_t_images(const T* w, T* wdt, const Geom& g, cudaStream_t st);
SavedLayout saved_layout(const Geom& g);

// `saved` may be null (nothing kept / nothing available).  weight_is_image:
// `weight` is the forward weight image from tc_weight_image (saved null).
cudaError_t tc_forward(const dcn_conv_desc& d, const Geom& g, const void* input, const void* weight,
                       bool weight_is_image, const void* offset, const void* mask, const void* bias,
                       void* output, void* workspace, void* saved, cudaStream_t st);
// The forward weight image [G][NKC][Cog][64] (pre-swizzled rows) of `weight`,
// as many elements as the weight.
cudaError_t tc_weight_image(const dcn_conv_desc& d, const Geom& g, const void* weight, void* image,
                            cudaStream_t st);
cudaError_t tc_backward(const dcn_conv_desc& d, const Geom& g, const void* grad_output,
                        const void* input, const void* weight, const void* offset, const void* mask,
                        const void* saved, void* grad_input, void* grad_weight, void* grad_offset,
                        void* grad_mask, void* grad_bias, void* workspace, cudaStream_t st,
                        dcn_params_ready_fn ready, void* user);
// Copies the device status word (non-zero after an expired bounded wait)
// into *out and clears it; synchronises the stream.
cudaError_t tc_read_and_clear_status(int* out, cudaStream_t st);

}  // namespace dcn
