// dcn_common.cuh -- shared device helpers for the deformable-convolution
// kernels: element conversion, problem geometry, the bilinear sample and its
// coordinate derivative.
//
// Sampling semantics follow the reference kernels in
// mps_deform_conv/csrc/deform_conv2d_mps.mm: bilinear_interpolate (:41-68) and
// get_coordinate_weight (:72-102).  Sampling points are split into an exact
// integer floor and an fp32 fraction (sample_pos); the reference's fp16 kernel
// computes them in half (:238-239), which torchvision does not.
#pragma once

#include <cuda_runtime.h>
#include <cuda_fp16.h>
#include <cuda_bf16.h>
#include <stdint.h>

#include "dcn_b200.h"
#include "dcn_debug.cuh"

namespace dcn {

// ---------------------------------------------------------------- elements
template <typename T> __device__ __forceinline__ float to_f(T v);
template <> __device__ __forceinline__ float to_f<float>(float v) { return v; }
template <> __device__ __forceinline__ float to_f<__half>(__half v) { return __half2float(v); }
template <> __device__ __forceinline__ float to_f<__nv_bfloat16>(__nv_bfloat16 v) { return __bfloat162float(v); }

template <typename T> __device__ __forceinline__ T from_f(float v);
template <> __device__ __forceinline__ float from_f<float>(float v) { return v; }
template <> __device__ __forceinline__ __half from_f<__half>(float v) { return __float2half_rn(v); }
template <> __device__ __forceinline__ __nv_bfloat16 from_f<__nv_bfloat16>(float v) { return __float2bfloat16_rn(v); }

// ---------------------------------------------------------------- geometry
// One deformable convolution problem.  All tensors are NCHW row-major:
//   input  [B][C][H][W]        weight [Co][C/G][kh][kw]
//   offset [B][OG][kh*kw][2][Ho][Wo] (dy, dx)   mask [B][OG][kh*kw][Ho][Wo]
//   output [B][Co][Ho][Wo]     columns [C*kh*kw][B*Ho*Wo]
struct Geom {
  int B, C, H, W;
  int Co, kh, kw;
  int sh, sw, ph, pw, dh, dw;
  int G, OG, use_mask;
  int Ho, Wo;
  int T;      // kh*kw
  int HWo;    // Ho*Wo
  int Cig;    // C / G   (input channels per weight group)
  int Cog;    // Co / G  (output channels per weight group)
  int cpo;    // C / OG  (input channels per offset group)
  long long P;  // B*Ho*Wo
  // Per-sample strides (elements) of the offset and mask tensors, and whether
  // the mask holds logits: OG*2*T*Ho*Wo, OG*T*Ho*Wo and 0 for the tensors
  // above; 3*OG*T*Ho*Wo, 3*OG*T*Ho*Wo and 1 when both are views of one DCNv2
  // head output [B][OG*T*3][Ho][Wo] (offsets first, then mask logits).
  long long off_bs, msk_bs;
  int msk_logit;
  // Memory formats: input / grad_input and output / grad_output are
  // channels-last ([B][H][W][C]) instead of NCHW (tensor-core path only).
  int in_nhwc, out_nhwc;
};

inline Geom make_geom(const dcn_conv_desc& d) {
  Geom g;
  g.B = (int)d.batch; g.C = (int)d.in_channels; g.H = (int)d.in_h; g.W = (int)d.in_w;
  g.Co = (int)d.out_channels; g.kh = (int)d.kernel_h; g.kw = (int)d.kernel_w;
  g.sh = (int)d.stride_h; g.sw = (int)d.stride_w; g.ph = (int)d.pad_h; g.pw = (int)d.pad_w;
  g.dh = (int)d.dilation_h; g.dw = (int)d.dilation_w;
  g.G = (int)d.n_weight_grps; g.OG = (int)d.n_offset_grps; g.use_mask = d.use_mask ? 1 : 0;
  g.Ho = (int)((d.in_h + 2 * d.pad_h - (d.dilation_h * (d.kernel_h - 1) + 1)) / d.stride_h + 1);
  g.Wo = (int)((d.in_w + 2 * d.pad_w - (d.dilation_w * (d.kernel_w - 1) + 1)) / d.stride_w + 1);
  g.T = g.kh * g.kw;
  g.HWo = g.Ho * g.Wo;
  g.Cig = g.C / g.G;
  g.Cog = g.Co / g.G;
  g.cpo = g.C / g.OG;
  g.P = (long long)g.B * g.HWo;
  g.off_bs = (long long)g.OG * 2 * g.T * g.HWo;
  g.msk_bs = (long long)g.OG * g.T * g.HWo;
  g.msk_logit = 0;
  g.in_nhwc = 0;
  g.out_nhwc = 0;
  return g;
}

// Mask value of a sample from its stored value: the value itself, or the
// sigmoid of a stored logit (DCNv2 head layout).
__device__ __forceinline__ float mask_of(const Geom& g, float v) {
  return g.msk_logit ? 1.f / (1.f + __expf(-v)) : v;
}

// Sampling point of a tap: the integer base position (oy*stride - pad +
// i*dilation) plus an offset.  The floor and the fraction are taken from the
// offset alone -- y0 = base + floor(dy), fy = dy - floor(dy) -- so the choice
// of corners is exact (it equals the float64 decision) even when base + dy
// lies within an fp32 rounding step of an integer, where the bilinear
// derivative jumps.
struct SamplePos {
  int y0, x0;     // floor of the sampling point
  float fy, fx;   // fractional parts, in [0, 1]
};

__device__ __forceinline__ SamplePos sample_pos(int base_y, int base_x, float dy, float dx) {
  const float ffy = floorf(dy), ffx = floorf(dx);
  SamplePos s;
  s.y0 = base_y + (int)ffy;
  s.x0 = base_x + (int)ffx;
  s.fy = dy - ffy;
  s.fx = dx - ffx;
  return s;
}

// Sampling point of tap t at output pixel p = oy*Wo+ox of image b, offset
// group o (reference :154-168).  Returns the mask value through *m.
template <typename T>
__device__ __forceinline__ SamplePos sample_point(const Geom& g, const T* __restrict__ offset,
                                                  const T* __restrict__ mask, int b, int o, int t,
                                                  int p, float* m) {
  const int oy = p / g.Wo, ox = p - oy * g.Wo;
  const int i = t / g.kw, j = t - i * g.kw;
  const long long obase = (long long)b * g.off_bs + (long long)(o * 2 * g.T + 2 * t) * g.HWo + p;
  const float dy = to_f(offset[obase]);
  const float dx = to_f(offset[obase + g.HWo]);
  *m = g.use_mask ? mask_of(g, to_f(mask[(long long)b * g.msk_bs + (long long)(o * g.T + t) * g.HWo + p])) : 1.0f;
  return sample_pos(oy * g.sh - g.ph + i * g.dh, ox * g.sw - g.pw + j * g.dw, dy, dx);
}

// Corner set of one bilinear sample.  w[k] is the weight of corner k
// (00, 01, 10, 11) and is zero for an invalid corner or when the whole sample
// lies outside (-1, H) x (-1, W) -- so the same weights serve the forward
// gather and the col2im scatter.  idx[k] is a safe in-plane index (0 when
// invalid).
struct Corners {
  float w[4];
  int idx[4];
};

__device__ __forceinline__ Corners corners_of(const SamplePos& s, int H, int W) {
  Corners c;
  // y > -1 and y < H with y = y0 + fy, fy in [0, 1]
  const bool in_y = (s.y0 > -1 || (s.y0 == -1 && s.fy > 0.0f)) && s.y0 < H;
  const bool in_x = (s.x0 > -1 || (s.x0 == -1 && s.fx > 0.0f)) && s.x0 < W;
  const bool inside = in_y && in_x;
  const int y0 = s.y0, x0 = s.x0, y1 = y0 + 1, x1 = x0 + 1;
  const float ly = s.fy, lx = s.fx, hy = 1.0f - ly, hx = 1.0f - lx;
  const bool vy0 = inside && y0 >= 0, vy1 = inside && y1 <= H - 1;
  const bool vx0 = x0 >= 0, vx1 = x1 <= W - 1;
  c.w[0] = (vy0 && vx0) ? hy * hx : 0.0f;
  c.w[1] = (vy0 && vx1) ? hy * lx : 0.0f;
  c.w[2] = (vy1 && vx0) ? ly * hx : 0.0f;
  c.w[3] = (vy1 && vx1) ? ly * lx : 0.0f;
  c.idx[0] = (vy0 && vx0) ? DCN_BOUND(y0 * W + x0, 1, (long long)H * W, DBG_CORNER) : 0;
  c.idx[1] = (vy0 && vx1) ? DCN_BOUND(y0 * W + x1, 1, (long long)H * W, DBG_CORNER) : 0;
  c.idx[2] = (vy1 && vx0) ? DCN_BOUND(y1 * W + x0, 1, (long long)H * W, DBG_CORNER) : 0;
  c.idx[3] = (vy1 && vx1) ? DCN_BOUND(y1 * W + x1, 1, (long long)H * W, DBG_CORNER) : 0;
  return c;
}

// Bilinear value of one plane (reference :41-68).
template <typename T>
__device__ __forceinline__ float bilinear(const T* __restrict__ plane, const Corners& c) {
  return c.w[0] * to_f(plane[c.idx[0]]) + c.w[1] * to_f(plane[c.idx[1]]) +
         c.w[2] * to_f(plane[c.idx[2]]) + c.w[3] * to_f(plane[c.idx[3]]);
}

// Coordinate-derivative corner set (reference :72-102): per-corner validity
// only, no whole-sample exit.  v = plane values at (y0,x0),(y0,x1),(y1,x0),(y1,x1).
struct CoordCorners {
  float fy, fx;     // fractional parts y - y0, x - x0
  bool v[4];
  int idx[4];
};

__device__ __forceinline__ CoordCorners coord_corners_of(const SamplePos& s, int H, int W) {
  CoordCorners c;
  const int y0 = s.y0, x0 = s.x0, y1 = y0 + 1, x1 = x0 + 1;
  c.fy = s.fy;
  c.fx = s.fx;
  const bool vy0 = 0 <= y0 && y0 < H, vy1 = 0 <= y1 && y1 < H;
  const bool vx0 = 0 <= x0 && x0 < W, vx1 = 0 <= x1 && x1 < W;
  c.v[0] = vy0 && vx0; c.v[1] = vy0 && vx1; c.v[2] = vy1 && vx0; c.v[3] = vy1 && vx1;
  c.idx[0] = c.v[0] ? DCN_BOUND(y0 * W + x0, 1, (long long)H * W, DBG_COORD_CORNER) : 0;
  c.idx[1] = c.v[1] ? DCN_BOUND(y0 * W + x1, 1, (long long)H * W, DBG_COORD_CORNER) : 0;
  c.idx[2] = c.v[2] ? DCN_BOUND(y1 * W + x0, 1, (long long)H * W, DBG_COORD_CORNER) : 0;
  c.idx[3] = c.v[3] ? DCN_BOUND(y1 * W + x1, 1, (long long)H * W, DBG_COORD_CORNER) : 0;
  return c;
}

// d/dy and d/dx of the bilinear sample from the four corner values.
__device__ __forceinline__ void coord_grads(const CoordCorners& c, float v00, float v01, float v10,
                                            float v11, float* dy, float* dx) {
  *dy = c.fx * (v11 - v01) + (1.0f - c.fx) * (v10 - v00);
  *dx = c.fy * (v11 - v10) + (1.0f - c.fy) * (v01 - v00);
}

}  // namespace dcn
