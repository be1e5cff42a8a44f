// dcn_simt.cu -- general-purpose CUDA-core kernels for deformable convolution.
//
// These handle every dtype and every shape (any channel count, kernel size,
// group split) with fp32 accumulation, and they implement the reference's
// column-buffer interface (im2col / col2im / col2im_coord).  The tensor-core
// kernels in dcn_tc.cu take over the shapes they support for fp16/bf16.
//
//   im2col        reference deformable_im2col_*      deform_conv2d_mps.mm:105-340
//   col2im        reference deformable_col2im_fp32   deform_conv2d_mps.mm:344-417
//   col2im_coord  reference deformable_col2im_coord  deform_conv2d_mps.mm:423-519
//   GEMMs         reference at::mm / at::bmm / torch.mm (mm:765-782,
//                 __init__.py:281, :289-290): tcgen05 tf32 MMAs with the
//                 three-term split that keeps fp32 accuracy
//                 (dcn_tf32_gemm.cuh), operands read through loader functors
//                 (materialised columns, or the gather itself when the
//                 columns are not kept).
#include "dcn_internal.h"
#include "dcn_tf32_gemm.cuh"

namespace dcn {

// ---------------------------------------------------------------- gather
// Column value col[c*T + t][b*HWo + p] computed on the fly.
template <typename T>
__device__ __forceinline__ float column_value(const Geom& g, const T* __restrict__ input,
                                              const T* __restrict__ offset,
                                              const T* __restrict__ mask, int b, int c, int t,
                                              int p) {
  float m;
  const SamplePos sp = sample_point(g, offset, mask, b, c / g.cpo, t, p, &m);
  const Corners cs = corners_of(sp, g.H, g.W);
  const T* plane = input + ((long long)b * g.C + c) * g.H * g.W;
  return m * bilinear(plane, cs);
}

// ---------------------------------------------------------------- GEMM
// C[M][N] = sum_k A(k, m) * B(k, n) per group, A and B read by loader
// functors float operator()(g, k, mn); A_KFAST / B_KFAST: the loader's source
// is contiguous along k (else along m / n).  ep(g, m, n, value) receives every
// element once (split: its partial over a K range, to be accumulated).
template <bool A_KFAST, bool B_KFAST, class LA, class LB, class EP>
static cudaError_t launch_gemm(const char* name, const LA& la, const LB& lb, const EP& ep, int M, int N,
                               int K, int groups, bool split, cudaStream_t st) {
  if (M <= 0 || N <= 0 || groups <= 0) return cudaSuccess;
  KernelScope ks(name, st);
  return tf32g::launch_tf32x3<A_KFAST, B_KFAST>(la, lb, ep, M, N, K, groups, split, st);
}

// ---------------------------------------------------------------- functors
// Operand loaders: float operator()(g, k, mn) reads one element.  kContig
// says which 4 consecutive elements are contiguous in memory (1: k..k+3 at
// one mn, 2: mn..mn+3 at one k, 0: neither); when `vec` is set (fp32 data,
// 16-byte aligned rows, set by the host) ld4(g, k, mn) reads them as one
// float4 at a k (kContig 1) or mn (kContig 2) that is a multiple of 4.
__host__ __device__ inline bool aligned16(const void* p) { return ((uintptr_t)p & 15) == 0; }

template <typename T>
struct WeightRowLoader {  // A(k, m) = W[g*Cog + m][k]   (forward)
  static constexpr int kContig = 1;
  const T* w; int Cog, Kg; bool vec;
  WeightRowLoader(const T* w_, int cog, int kg)
      : w(w_), Cog(cog), Kg(kg), vec(sizeof(T) == 4 && kg % 4 == 0 && aligned16(w_)) {}
  __device__ float operator()(int g, int k, int m) const {
    return to_f(w[(long long)(g * Cog + m) * Kg + k]);
  }
  __device__ float4 ld4(int g, int k, int m) const {
    return *reinterpret_cast<const float4*>(w + (long long)(g * Cog + m) * Kg + k);
  }
};
template <typename T>
struct WeightColLoader {  // A(co, m=k) = W[g*Cog + co][k]   (dgrad)
  static constexpr int kContig = 2;
  const T* w; int Cog, Kg; bool vec;
  WeightColLoader(const T* w_, int cog, int kg)
      : w(w_), Cog(cog), Kg(kg), vec(sizeof(T) == 4 && kg % 4 == 0 && aligned16(w_)) {}
  __device__ float operator()(int g, int co, int k) const {
    return to_f(w[(long long)(g * Cog + co) * Kg + k]);
  }
  __device__ float4 ld4(int g, int co, int k) const {
    return *reinterpret_cast<const float4*>(w + (long long)(g * Cog + co) * Kg + k);
  }
};
template <typename T>
struct ColumnLoader {  // B(k, n) = col[(g*Cig + k/T)*T + k%T][n]   (forward)
  static constexpr int kContig = 0;
  Geom geo; const T* x; const T* off; const T* msk; bool vec = false;
  ColumnLoader(const Geom& g_, const T* x_, const T* off_, const T* msk_) : geo(g_), x(x_), off(off_), msk(msk_) {}
  __device__ float operator()(int g, int k, int n) const {
    const int b = n / geo.HWo, p = n - b * geo.HWo;
    const int cl = k / geo.T, t = k - cl * geo.T;
    return column_value(geo, x, off, msk, b, g * geo.Cig + cl, t, p);
  }
  __device__ float4 ld4(int, int, int) const { return make_float4(0.f, 0.f, 0.f, 0.f); }
};
// n / d for 0 <= n: a float-reciprocal quotient corrected to the exact one
// (n < 2^24), else the integer division.
__device__ __forceinline__ int div_rcp(int n, int d, float rcp) {
  if (n >= (1 << 24)) return n / d;
  int q = __float2int_rz((float)n * rcp);
  const int r = n - q * d;
  if (r < 0) --q;
  else if (r >= d) ++q;
  return q;
}
// grad_output rows: 4 consecutive pixels px..px+3 (px a multiple of 4) are one
// image's when HWo is a multiple of 4.
template <typename T>
struct GradOutLoaderCN {  // B(co, n=px) = gO[b][g*Cog + co][p]   (dgrad)
  static constexpr int kContig = 2;
  Geom geo; const T* go; float rcp_hwo; bool vec;
  GradOutLoaderCN(const Geom& g_, const T* go_)
      : geo(g_), go(go_), rcp_hwo(1.f / (float)g_.HWo), vec(sizeof(T) == 4 && g_.HWo % 4 == 0 && aligned16(go_)) {}
  __device__ float operator()(int g, int co, int n) const {
    const int b = div_rcp(n, geo.HWo, rcp_hwo), p = n - b * geo.HWo;
    return to_f(go[((long long)b * geo.Co + g * geo.Cog + co) * geo.HWo + p]);
  }
  __device__ float4 ld4(int g, int co, int n) const {
    const int b = div_rcp(n, geo.HWo, rcp_hwo), p = n - b * geo.HWo;
    return *reinterpret_cast<const float4*>(go + ((long long)b * geo.Co + g * geo.Cog + co) * geo.HWo + p);
  }
};
template <typename T>
struct GradOutLoaderPM {  // A(px, m=co) = gO[b][g*Cog + co][p]   (wgrad)
  static constexpr int kContig = 1;
  Geom geo; const T* go; float rcp_hwo; bool vec;
  GradOutLoaderPM(const Geom& g_, const T* go_)
      : geo(g_), go(go_), rcp_hwo(1.f / (float)g_.HWo), vec(sizeof(T) == 4 && g_.HWo % 4 == 0 && aligned16(go_)) {}
  __device__ float operator()(int g, int px, int co) const {
    const int b = div_rcp(px, geo.HWo, rcp_hwo), p = px - b * geo.HWo;
    return to_f(go[((long long)b * geo.Co + g * geo.Cog + co) * geo.HWo + p]);
  }
  __device__ float4 ld4(int g, int px, int co) const {
    const int b = div_rcp(px, geo.HWo, rcp_hwo), p = px - b * geo.HWo;
    return *reinterpret_cast<const float4*>(go + ((long long)b * geo.Co + g * geo.Cog + co) * geo.HWo + p);
  }
};
struct ColumnBufferLoader {  // B(k, n) = cols[(g*Kg + k)][n]   (forward, materialized columns)
  static constexpr int kContig = 2;
  const float* cols; int Kg; long long P; bool vec;
  ColumnBufferLoader(const float* c, int kg, long long p) : cols(c), Kg(kg), P(p), vec(p % 4 == 0 && aligned16(c)) {}
  __device__ float operator()(int g, int k, int n) const { return cols[((long long)g * Kg + k) * P + n]; }
  __device__ float4 ld4(int g, int k, int n) const {
    return *reinterpret_cast<const float4*>(cols + ((long long)g * Kg + k) * P + n);
  }
};
struct ColumnBufferLoaderPK {  // B(px, n=k) = cols[(g*Kg + k)][px]   (wgrad, materialized columns)
  static constexpr int kContig = 1;
  const float* cols; int Kg; long long P; bool vec;
  ColumnBufferLoaderPK(const float* c, int kg, long long p) : cols(c), Kg(kg), P(p), vec(p % 4 == 0 && aligned16(c)) {}
  __device__ float operator()(int g, int px, int k) const { return cols[((long long)g * Kg + k) * P + px]; }
  __device__ float4 ld4(int g, int px, int k) const {
    return *reinterpret_cast<const float4*>(cols + ((long long)g * Kg + k) * P + px);
  }
};
template <typename T>
struct ForwardEpilogue {  // out[b][g*Cog + m][p] = acc + bias
  Geom geo; const T* bias; T* out;
  __device__ void operator()(int g, int m, int n, float acc) const {
    const int b = n / geo.HWo, p = n - b * geo.HWo;
    const int oc = g * geo.Cog + m;
    if (bias) acc += to_f(bias[oc]);
    out[((long long)b * geo.Co + oc) * geo.HWo + p] = from_f<T>(acc);
  }
};
struct ColumnStoreEpilogue {  // gcol[(g*Kg + m)][n] = acc
  float* gcol; int Kg; long long P;
  __device__ void operator()(int g, int m, int n, float acc) const {
    gcol[(long long)(g * Kg + m) * P + n] = acc;
  }
};
struct AtomicWeightEpilogue {  // gW32[(g*Cog + m)*Kg + n] += acc
  float* gw; int Cog, Kg;
  __device__ void operator()(int g, int m, int n, float acc) const {
    atomicAdd(&gw[(long long)(g * Cog + m) * Kg + n], acc);
  }
};

// ---------------------------------------------------------------- kernels
// Column buffer: thread e = (channel block q of IM2COL_CH channels, offset
// group o, tap t, pixel n), n fastest, computes the sampling point of (n, t, o)
// and writes rows (o*cpo + c)*T + t of its channels (coalesced over pixels
// n); its 4 * IM2COL_CH corner loads are independent.
constexpr int IM2COL_CH = 8;
__host__ __device__ inline long long im2col_threads(const Geom& g) {
  return (long long)((g.cpo + IM2COL_CH - 1) / IM2COL_CH) * g.OG * g.T * g.P;
}
template <typename T, typename TC>
__global__ void im2col_og_kernel(Geom g, const T* __restrict__ x, const T* __restrict__ off,
                                 const T* __restrict__ msk, TC* __restrict__ cols) {
  const long long total = im2col_threads(g);
  const long long row_stride = (long long)g.T * g.P;  // channel c -> c + 1
  const long long plane = (long long)g.H * g.W;
  for (long long e = blockIdx.x * (long long)blockDim.x + threadIdx.x; e < total;
       e += (long long)gridDim.x * blockDim.x) {
    const long long r = e / g.P, n = e - r * g.P;  // r = (q * OG + o) * T + t
    const long long r2 = r / g.T;
    const int t = (int)(r - r2 * g.T);
    const int q = (int)(r2 / g.OG), o = (int)(r2 - (long long)q * g.OG);
    const int b = (int)(n / g.HWo), p = (int)(n - (long long)b * g.HWo);
    float m;
    const SamplePos sp = sample_point(g, off, msk, b, o, t, p, &m);
    const Corners cs = corners_of(sp, g.H, g.W);
    const int c0 = o * g.cpo + q * IM2COL_CH;
    const int nc = min(IM2COL_CH, g.cpo - q * IM2COL_CH);
    const T* src = x + ((long long)b * g.C + c0) * plane;
    TC* dst = cols + ((long long)c0 * g.T + t) * g.P + n;
#pragma unroll
    for (int c = 0; c < IM2COL_CH; ++c)
      if (c < nc)
        dst[DCN_BOUND((long long)c * row_stride, 1, (long long)g.C * g.T * g.P - (dst - cols), DBG_SIMT_IM2COL)] =
            from_f<TC>(m * bilinear(src + (long long)c * plane, cs));
  }
}

// grad_input (fp32, zeroed) += col2im(gcol); gcol in the column layout.
template <typename TC, typename T>
__global__ void col2im_kernel(Geom g, const TC* __restrict__ gcol, const T* __restrict__ off,
                              const T* __restrict__ msk, float* __restrict__ gin) {
  const long long total = (long long)g.C * g.T * g.P;
  for (long long e = blockIdx.x * (long long)blockDim.x + threadIdx.x; e < total;
       e += (long long)gridDim.x * blockDim.x) {
    const long long row = e / g.P, n = e - row * g.P;
    const int c = (int)(row / g.T), t = (int)(row - (long long)c * g.T);
    const int b = (int)(n / g.HWo), p = (int)(n - (long long)b * g.HWo);
    float m;
    const SamplePos sp = sample_point(g, off, msk, b, c / g.cpo, t, p, &m);
    const Corners cs = corners_of(sp, g.H, g.W);
    const float v = m * to_f(gcol[e]);
#pragma unroll
    for (int k = 0; k < 4; ++k)
      if (cs.w[k] != 0.0f)
        atomicAdd(gin + DCN_BOUND(((long long)b * g.C + c) * g.H * g.W + cs.idx[k], 1, (long long)g.B * g.C * g.H * g.W,
                                  DBG_SIMT_COL2IM),
                  cs.w[k] * v);
  }
}

__device__ __forceinline__ void red_add_v4(float* p, float a, float b, float c, float d) {
  asm volatile("red.global.add.v4.f32 [%0], {%1, %2, %3, %4};" ::"l"(p), "f"(a), "f"(b), "f"(c), "f"(d)
               : "memory");
}

// grad_input (channels-last fp32 [B][H][W][C], zeroed) += col2im(gcol), four
// channels of one sample per thread: the sampling point once for the four,
// and one 16-byte red.global.add.v4.f32 per corner (a quarter of
// col2im_kernel's reduction requests).  C and the channels per offset group
// are multiples of 4; acc is 16-byte aligned.
template <typename TC, typename T>
__global__ void col2im_nhwc4_kernel(Geom g, const TC* __restrict__ gcol, const T* __restrict__ off,
                                    const T* __restrict__ msk, float* __restrict__ acc) {
  const long long total = (long long)(g.C / 4) * g.T * g.P;
  for (long long e = blockIdx.x * (long long)blockDim.x + threadIdx.x; e < total;
       e += (long long)gridDim.x * blockDim.x) {
    const long long row = e / g.P, n = e - row * g.P;  // row = (c/4)*T + t
    const int c4 = (int)(row / g.T), t = (int)(row - (long long)c4 * g.T);
    const int c = 4 * c4;
    const int b = (int)(n / g.HWo), p = (int)(n - (long long)b * g.HWo);
    float m;
    const SamplePos sp = sample_point(g, off, msk, b, c / g.cpo, t, p, &m);
    const Corners cs = corners_of(sp, g.H, g.W);
    const long long rs = (long long)g.T * g.P;  // channel c -> c + 1 in the column layout
    const TC* src = gcol + ((long long)c * g.T + t) * g.P + n;
    const float v0 = m * to_f(src[0]), v1 = m * to_f(src[rs]), v2 = m * to_f(src[2 * rs]), v3 = m * to_f(src[3 * rs]);
#pragma unroll
    for (int k = 0; k < 4; ++k) {
      const float w = cs.w[k];
      if (w != 0.0f)
        red_add_v4(acc + DCN_BOUND(((long long)b * g.H * g.W + cs.idx[k]) * g.C + c, 4, (long long)g.B * g.H * g.W * g.C,
                                   DBG_SIMT_COL2IM_NHWC),
                   w * v0, w * v1, w * v2, w * v3);
    }
  }
}

// channels-last fp32 [B][HW][C] -> NCHW T [B][C][HW], 32 x 32 tiles through
// shared memory (33-word rows).  grid (HW/32, C/32, B), 256 threads.
template <typename T>
__global__ void nhwc_f32_to_nchw_kernel(const float* __restrict__ src, T* __restrict__ dst, int C, int HW) {
  __shared__ float tile[32][33];
  const int b = blockIdx.z, c0 = blockIdx.y * 32, hw0 = blockIdx.x * 32;
  const float* s = src + (long long)b * HW * C;
  T* d = dst + (long long)b * C * HW;
  for (int e = threadIdx.x; e < 32 * 32; e += blockDim.x) {
    const int hh = e >> 5, cc = e & 31;
    if (hw0 + hh < HW && c0 + cc < C) tile[cc][hh] = s[(long long)(hw0 + hh) * C + c0 + cc];
  }
  __syncthreads();
  for (int e = threadIdx.x; e < 32 * 32; e += blockDim.x) {
    const int cc = e >> 5, hh = e & 31;
    if (hw0 + hh < HW && c0 + cc < C) d[(long long)(c0 + cc) * HW + hw0 + hh] = from_f<T>(tile[cc][hh]);
  }
}

// grad_offset / grad_mask.  A block of 256 threads takes 256 / nq
// consecutive samples (b, offset group, tap, pixel; pixel fastest) and nq
// channel slices: thread (q, s) sums channels q, q + nq, ... of sample s's
// group, consecutive threads on consecutive samples (coalesced reads of each
// channel plane and of the column gradient).  The nq partial sums of a sample
// are added in slice order through shared memory (deterministic).  The mask
// term reuses the corner values of the coordinate derivative (the same plane
// reads bilinear() makes: the sample weights are zero wherever a corner is
// invalid).
constexpr int COORD_THREADS = 256;
template <typename TC, typename T>
__global__ void __launch_bounds__(COORD_THREADS)
col2im_coord_kernel(Geom g, const TC* __restrict__ gcol, const T* __restrict__ x, const T* __restrict__ off,
                    const T* __restrict__ msk, T* __restrict__ goff, T* __restrict__ gmsk, int nq) {
  __shared__ float part[3][COORD_THREADS];
  const long long samples = (long long)g.B * g.OG * g.T * g.HWo;
  const int ns = COORD_THREADS / nq;
  const int q = threadIdx.x / ns, si = threadIdx.x - q * ns;
  const long long nblk = (samples + ns - 1) / ns;
  for (long long blk = blockIdx.x; blk < nblk; blk += gridDim.x) {
    const long long sidx = blk * ns + si;
    const bool active = sidx < samples;
    const int p = (int)(sidx % g.HWo);
    long long r = sidx / g.HWo;
    const int t = (int)(r % g.T); r /= g.T;
    const int o = (int)(r % g.OG);
    const int b = (int)(r / g.OG);
    float gy = 0.f, gx = 0.f, gm = 0.f, m = 1.f;
    if (active) {
      const SamplePos sp = sample_point(g, off, msk, b, o, t, p, &m);
      const CoordCorners cc = coord_corners_of(sp, g.H, g.W);
      const Corners cs = corners_of(sp, g.H, g.W);
      const TC* gsrc = gcol + (long long)t * g.P + (long long)b * g.HWo + p;
#pragma unroll 4
      for (int cl = q; cl < g.cpo; cl += nq) {
        const int c = o * g.cpo + cl;
        const T* plane = x + ((long long)b * g.C + c) * g.H * g.W;
        const float v = to_f(gsrc[(long long)c * g.T * g.P]);
        const float v00 = cc.v[0] ? to_f(plane[cc.idx[0]]) : 0.f;
        const float v01 = cc.v[1] ? to_f(plane[cc.idx[1]]) : 0.f;
        const float v10 = cc.v[2] ? to_f(plane[cc.idx[2]]) : 0.f;
        const float v11 = cc.v[3] ? to_f(plane[cc.idx[3]]) : 0.f;
        float dy, dx;
        coord_grads(cc, v00, v01, v10, v11, &dy, &dx);
        gy += dy * v;
        gx += dx * v;
        gm += v * (cs.w[0] * v00 + cs.w[1] * v01 + cs.w[2] * v10 + cs.w[3] * v11);
      }
    }
    if (nq > 1) {
      part[0][threadIdx.x] = gy;
      part[1][threadIdx.x] = gx;
      part[2][threadIdx.x] = gm;
      __syncthreads();
      if (q == 0) {
        for (int k = 1; k < nq; ++k) {
          gy += part[0][k * ns + si];
          gx += part[1][k * ns + si];
          gm += part[2][k * ns + si];
        }
      }
      __syncthreads();  // the next round rewrites the partial sums
    }
    if (active && q == 0) {
      const long long ob = ((long long)(b * g.OG + o) * 2 * g.T + 2 * t) * g.HWo + p;
      goff[ob] = from_f<T>(m * gy);
      goff[ob + g.HWo] = from_f<T>(m * gx);
      if (g.use_mask && gmsk) gmsk[((long long)(b * g.OG + o) * g.T + t) * g.HWo + p] = from_f<T>(gm);
    }
  }
}

// Channel slices of col2im_coord_kernel: doubled (up to 8, and not beyond the
// group's channels) while the launch has fewer than 148 x 2048 threads.
inline int coord_slices(const Geom& g) {
  const long long samples = (long long)g.B * g.OG * g.T * g.HWo;
  int nq = 1;
  while (nq < 8 && nq < g.cpo && samples * nq < 148LL * 2048) nq *= 2;
  return nq;
}

// grad_bias[co] = sum over (b, p) of grad_out[b][co][p]; one block per co,
// four independent partial sums per thread.
template <typename T, typename TO>
__global__ void bias_grad_kernel(Geom g, const T* __restrict__ go, TO* __restrict__ gb) {
  const int co = blockIdx.x;
  float s0 = 0.f, s1 = 0.f, s2 = 0.f, s3 = 0.f;
  const int bd = blockDim.x;
  for (int b = 0; b < g.B; ++b) {
    const T* row = go + ((long long)b * g.Co + co) * g.HWo;
    int p = threadIdx.x;
    for (; p + 3 * bd < g.HWo; p += 4 * bd) {
      s0 += to_f(row[p]);
      s1 += to_f(row[p + bd]);
      s2 += to_f(row[p + 2 * bd]);
      s3 += to_f(row[p + 3 * bd]);
    }
    for (; p < g.HWo; p += bd) s0 += to_f(row[p]);
  }
  float s = (s0 + s1) + (s2 + s3);
  __shared__ float red[32];
  for (int o = 16; o > 0; o >>= 1) s += __shfl_xor_sync(0xffffffffu, s, o);
  if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = s;
  __syncthreads();
  if (threadIdx.x < 32) {
    s = (threadIdx.x < (blockDim.x >> 5)) ? red[threadIdx.x] : 0.f;
    for (int o = 16; o > 0; o >>= 1) s += __shfl_xor_sync(0xffffffffu, s, o);
    if (threadIdx.x == 0) gb[co] = from_f<TO>(s);
  }
}

template <typename T>
__global__ void f32_to_kernel(const float* __restrict__ src, T* __restrict__ dst, long long n) {
  for (long long e = blockIdx.x * (long long)blockDim.x + threadIdx.x; e < n;
       e += (long long)gridDim.x * blockDim.x)
    dst[e] = from_f<T>(src[e]);
}

static inline int grid_for(long long n, int threads = 256) {
  long long b = (n + threads - 1) / threads;
  const long long cap = 148LL * 32;  // 148 SMs x 32 resident blocks of 256 max
  return (int)(b < 1 ? 1 : (b > cap ? cap : b));
}

// The forward materializes fp32 columns [C*T][slice pixels] (im2col_og_kernel)
// for slices of whole images whose columns take at most 1 GiB (at least one
// image per slice), then runs the GEMM on each slice; the workspace holds one
// slice's columns.
static int simt_fwd_slice_images(const Geom& g) {
  const long long per_image = (long long)sizeof(float) * g.C * g.T * g.HWo;
  long long n = per_image > 0 ? (1LL << 30) / per_image : g.B;
  if (n < 1) n = 1;
  return (int)(n < g.B ? n : g.B);
}
static size_t simt_fwd_cols_bytes(const Geom& g) {
  return sizeof(float) * (size_t)g.C * g.T * (size_t)g.HWo * (size_t)simt_fwd_slice_images(g);
}

size_t simt_forward_workspace(const Geom& g) { return ws_align(simt_fwd_cols_bytes(g)); }

size_t simt_saved_columns_bytes(const Geom& g) {
  return g.B > 0 && simt_fwd_slice_images(g) == g.B ? ws_align(simt_fwd_cols_bytes(g)) : 0;
}

// ---------------------------------------------------------------- host side
template <typename T>
cudaError_t simt_forward(const Geom& g, const T* x, const T* w, const T* off, const T* msk,
                         const T* bias, T* out, void* workspace, cudaStream_t st) {
  const int Kg = g.Cig * g.T;
  WeightRowLoader<T> la(w, g.Cog, Kg);
  if (!workspace || simt_fwd_cols_bytes(g) == 0) {  // no column buffer: the loader gathers
    ColumnLoader<T> lb(g, x, off, msk);
    return launch_gemm<true, false>("tf32_fwd_gemm", la, lb, ForwardEpilogue<T>{g, bias, out}, g.Cog, (int)g.P,
                                    Kg, g.G, false, st);
  }
  float* cols = static_cast<float*>(workspace);
  const int slice = simt_fwd_slice_images(g);
  for (int b0 = 0; b0 < g.B; b0 += slice) {
    // the images [b0, b0 + gs.B) as a problem of their own
    Geom gs = g;
    gs.B = g.B - b0 < slice ? g.B - b0 : slice;
    gs.P = (long long)gs.B * g.HWo;
    const T* xs = x + (long long)b0 * g.C * g.H * g.W;
    const T* offs = off + (long long)b0 * g.off_bs;
    const T* msks = msk ? msk + (long long)b0 * g.msk_bs : nullptr;
    T* outs = out + (long long)b0 * g.Co * g.HWo;
    cudaError_t e;
    {
      KernelScope ks("im2col_og", st);
      im2col_og_kernel<T, float><<<grid_for(im2col_threads(gs)), 256, 0, st>>>(gs, xs, offs, msks, cols);
    }
    if ((e = cudaGetLastError()) != cudaSuccess) return e;
    ColumnBufferLoader lb(cols, Kg, gs.P);
    if ((e = launch_gemm<true, false>("tf32_fwd_gemm", la, lb, ForwardEpilogue<T>{gs, bias, outs}, gs.Cog,
                                      (int)gs.P, Kg, gs.G, false, st)) != cudaSuccess)
      return e;
  }
  return cudaSuccess;
}

template <typename T>
cudaError_t simt_im2col(const Geom& g, const T* x, const T* off, const T* msk, T* cols,
                        cudaStream_t st) {
  const long long total = (long long)g.C * g.T * g.P;
  if (total == 0) return cudaSuccess;
  KernelScope ks("im2col", st);
  im2col_og_kernel<T, T><<<grid_for(im2col_threads(g)), 256, 0, st>>>(g, x, off, msk, cols);
  return cudaGetLastError();
}

template <typename TC, typename T>
cudaError_t simt_col2im(const Geom& g, const TC* gcol, const T* off, const T* msk, float* gin32,
                        cudaStream_t st) {
  const long long total = (long long)g.C * g.T * g.P;
  if (total == 0) return cudaSuccess;
  KernelScope ks("col2im", st);
  col2im_kernel<TC, T><<<grid_for(total), 256, 0, st>>>(g, gcol, off, msk, gin32);
  return cudaGetLastError();
}

template <typename TC, typename T>
cudaError_t simt_col2im_coord(const Geom& g, const TC* gcol, const T* x, const T* off,
                              const T* msk, T* goff, T* gmsk, cudaStream_t st) {
  const long long samples = (long long)g.B * g.OG * g.T * g.HWo;
  if (samples == 0) return cudaSuccess;
  const int nq = coord_slices(g);
  KernelScope ks("col2im_coord", st);
  col2im_coord_kernel<TC, T><<<grid_for(samples * nq, COORD_THREADS), COORD_THREADS, 0, st>>>(g, gcol, x, off, msk,
                                                                                               goff, gmsk, nq);
  return cudaGetLastError();
}

template <typename T>
cudaError_t convert_f32(const float* src, T* dst, long long n, cudaStream_t st) {
  if (n == 0) return cudaSuccess;
  KernelScope ks("f32_convert", st);
  f32_to_kernel<T><<<grid_for(n), 256, 0, st>>>(src, dst, n);
  return cudaGetLastError();
}

// Full backward on the SIMT kernels.  Workspace: gcol (fp32 columns), plus
// fp32 accumulators for grad_input / grad_weight when T is not float.
template <typename T>
cudaError_t simt_backward(const Geom& g, const T* go, const T* x, const T* w, const T* off,
                          const T* msk, T* gin, T* gw, T* goff, T* gmsk, T* gb,
                          const SimtBackwardWs& ws, cudaStream_t st) {
  cudaError_t e = cudaSuccess;
  const int Kg = g.Cig * g.T;
  if (gb) {
    {
      KernelScope ks("bias_grad", st);
      bias_grad_kernel<T, T><<<g.Co, 512, 0, st>>>(g, go, gb);
    }
    if ((e = cudaGetLastError()) != cudaSuccess) return e;
  }
  if (gw) {
    float* gw32 = ws.gw32 ? ws.gw32 : reinterpret_cast<float*>(gw);
    if ((e = cudaMemsetAsync(gw32, 0, sizeof(float) * (size_t)g.Co * Kg, st)) != cudaSuccess) return e;
    GradOutLoaderPM<T> la(g, go);
    AtomicWeightEpilogue ep{gw32, g.Cog, Kg};
    // the forward's columns when it kept them, else gathered again into the
    // column gradient's buffer (free until the dgrad GEMM below writes it)
    const float* cols = ws.cols;
    if (!cols) {
      KernelScope ks("im2col_og", st);
      im2col_og_kernel<T, float><<<grid_for(im2col_threads(g)), 256, 0, st>>>(g, x, off, msk, ws.gcol);
      if ((e = cudaGetLastError()) != cudaSuccess) return e;
      cols = ws.gcol;
    }
    ColumnBufferLoaderPK lb(cols, Kg, g.P);
    if ((e = launch_gemm<true, true>("tf32_wgrad_gemm", la, lb, ep, g.Cog, Kg, (int)g.P, g.G, true, st)) !=
        cudaSuccess)
      return e;
    if (ws.gw32 && (e = convert_f32<T>(ws.gw32, gw, (long long)g.Co * Kg, st)) != cudaSuccess) return e;
  }
  if (gin || goff || gmsk) {
    WeightColLoader<T> la(w, g.Cog, Kg);
    GradOutLoaderCN<T> lb(g, go);
    ColumnStoreEpilogue ep{ws.gcol, Kg, g.P};
    if ((e = launch_gemm<false, false>("tf32_dgrad_gemm", la, lb, ep, Kg, (int)g.P, g.Cog, g.G, false, st)) !=
        cudaSuccess)
      return e;
    if (gin) {
      const long long n = (long long)g.B * g.C * g.H * g.W;
      if (ws.gacc && g.C % 4 == 0 && g.cpo % 4 == 0 && n > 0) {
        // four channels per thread into a channels-last accumulator, then NCHW
        if ((e = cudaMemsetAsync(ws.gacc, 0, sizeof(float) * (size_t)n, st)) != cudaSuccess) return e;
        {
          KernelScope ks("col2im_nhwc4", st);
          col2im_nhwc4_kernel<float, T><<<grid_for((long long)(g.C / 4) * g.T * g.P), 256, 0, st>>>(
              g, ws.gcol, off, msk, ws.gacc);
        }
        if ((e = cudaGetLastError()) != cudaSuccess) return e;
        KernelScope ks("nhwc_f32_to_nchw", st);
        const dim3 grid((unsigned)((g.H * g.W + 31) / 32), (unsigned)((g.C + 31) / 32), (unsigned)g.B);
        nhwc_f32_to_nchw_kernel<T><<<grid, 256, 0, st>>>(ws.gacc, gin, g.C, g.H * g.W);
        if ((e = cudaGetLastError()) != cudaSuccess) return e;
      } else {
        float* gin32 = ws.gin32 ? ws.gin32 : reinterpret_cast<float*>(gin);
        if ((e = cudaMemsetAsync(gin32, 0, sizeof(float) * (size_t)n, st)) != cudaSuccess) return e;
        if ((e = simt_col2im<float, T>(g, ws.gcol, off, msk, gin32, st)) != cudaSuccess) return e;
        if (ws.gin32 && (e = convert_f32<T>(ws.gin32, gin, n, st)) != cudaSuccess) return e;
      }
    }
    if (goff || gmsk) {
      T* goff_t = goff ? goff : reinterpret_cast<T*>(ws.goff_scratch);
      if ((e = simt_col2im_coord<float, T>(g, ws.gcol, x, off, msk, goff_t, gmsk, st)) != cudaSuccess)
        return e;
    }
  }
  return cudaSuccess;
}

// ---------------------------------------------------------------- instances
#define DCN_SIMT_INSTANCES(T)                                                                    \
  template cudaError_t simt_forward<T>(const Geom&, const T*, const T*, const T*, const T*,      \
                                       const T*, T*, void*, cudaStream_t);                       \
  template cudaError_t simt_im2col<T>(const Geom&, const T*, const T*, const T*, T*,            \
                                      cudaStream_t);                                             \
  template cudaError_t simt_col2im<T, T>(const Geom&, const T*, const T*, const T*, float*,     \
                                         cudaStream_t);                                          \
  template cudaError_t simt_col2im_coord<T, T>(const Geom&, const T*, const T*, const T*,       \
                                               const T*, T*, T*, cudaStream_t);                  \
  template cudaError_t convert_f32<T>(const float*, T*, long long, cudaStream_t);               \
  template cudaError_t simt_backward<T>(const Geom&, const T*, const T*, const T*, const T*,    \
                                        const T*, T*, T*, T*, T*, T*, const SimtBackwardWs&,     \
                                        cudaStream_t);

DCN_SIMT_INSTANCES(float)
DCN_SIMT_INSTANCES(__half)
DCN_SIMT_INSTANCES(__nv_bfloat16)

DCN_DEBUG_BOUNDS_TU(simt)

}  // namespace dcn
